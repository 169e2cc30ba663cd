"""Build libmoestream_cuda (shared, for ctypes / FFI callers, and static, for a Rust build.rs)
in-tree under moe_stream_b200/_build/ with nvcc for sm_100a.  Run: python -m moe_stream_b200.build"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "_build")
SOURCES = ["kernels_dense.cu", "kernels_moe.cu", "kernels_moe_tc.cu", "kernels_prefill.cu", "kernels_prefill_attn.cu", "kernels_exact.cu", "kernels_sample.cu", "kernels_ssm.cu", "kernels_batch.cu", "runtime.cu"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
         "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr"]
SO = os.path.join(OUT, "libmoestream_cuda.so")
A = os.path.join(OUT, "libmoestream_cuda.a")


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False) -> str:
    os.makedirs(OUT, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    headers.append(os.path.join(os.path.dirname(HERE), "include", "moestream_cuda.h"))
    objs, cmds = [], []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(OUT, src.replace(".cu", ".o"))
        if _stale(o, [s] + headers):
            cmds.append([NVCC, *FLAGS, "-c", s, "-o", o])
        objs.append(o)
    # translation units compile in parallel (one nvcc process each)
    procs = []
    for cmd in cmds:
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        procs.append((cmd, subprocess.Popen(cmd)))
    failed = [cmd for cmd, p in procs if p.wait() != 0]
    if failed:
        raise subprocess.CalledProcessError(1, failed[0])
    if _stale(SO, objs):
        subprocess.run([NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", SO, *objs,
                        "-Xcompiler", "-fPIC", "-lcuda"], check=True)
    if _stale(A, objs):
        if os.path.exists(A):
            os.remove(A)
        subprocess.run([NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-lib", "-o", A, *objs], check=True)
    return SO


if __name__ == "__main__":
    print(build(verbose=True))
