"""CPU-side checks of the C ABI boundary: the library loads, exports every symbol the
public header declares, and refuses bad calls without touching a GPU."""
import ctypes as C
import os
import subprocess

import pytest

from moe_stream_b200 import _lib


@pytest.fixture(scope="module")
def L():
    from moe_stream_b200 import build
    build.build()
    return _lib.lib()


def test_exports_every_header_symbol(L):
    syms = _lib.header_symbols()
    assert len(syms) >= 30
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    missing = [s for s in syms if s not in exported]
    assert not missing, missing
    for s in syms:
        assert getattr(L, s) is not None
    assert set(syms) == set(_lib._SIGS), "ctypes signatures out of sync with the header"


def test_static_library_built():
    from moe_stream_b200 import build
    assert os.path.exists(build.A)


def test_abi_version_and_status_strings(L):
    assert L.ms_abi_version() == 4
    assert L.ms_status_string(0) == b"ok"
    assert L.ms_status_string(5) == b"device wait timed out"
    assert L.ms_status_string(99) == b"unknown status"


def test_null_arguments_rejected_without_gpu(L):
    assert L.ms_ctx_create(0, None) == 1
    assert L.ms_sync(None) == 1
    assert L.ms_model_destroy(None) == 1
    assert L.ms_model_forward(None, None, 0, None) == 1
    assert L.ms_last_error(None) == b"null context"


def test_no_device_ctx_create_fails_cleanly(L):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = C.c_void_p()
    assert L.ms_ctx_create(0, C.byref(h)) == 1 and not h.value


def test_header_compiles_as_c(tmp_path):
    src = tmp_path / "t.c"
    src.write_text('#include "moestream_cuda.h"\nint main(void){ return ms_abi_version() == MS_ABI_VERSION ? 0 : 1; }\n')
    inc = os.path.join(os.path.dirname(_lib.HERE), "include")
    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-c", str(src), "-I", inc, "-o", str(tmp_path / "t.o")],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
