"""moe-stream B200: sm_100a CUDA backend for moe-stream's quantized MoE decode path.

The compute lives in libmoestream_cuda.so (C ABI: include/moestream_cuda.h); this package
is the Python host side (ctypes) plus GGUF I/O and seeded synthetic models.
"""
from . import gguf, synth  # noqa: F401

__version__ = "0.1.0"


def __getattr__(name):
    # the CUDA binding is imported lazily so GGUF tooling works without the built library
    if name in ("Context", "Engine", "config_from_model"):
        from . import engine
        return getattr(engine, name)
    raise AttributeError(name)
