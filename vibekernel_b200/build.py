"""Build libvkgemm.so in-tree for sm_100a (nvcc cross-compiles; no GPU needed).

    python vibekernel_b200/build.py [--verbose]

(run it as a script: importing the package first would load a stale library).

The library is one shared object with a plain C ABI (include/vkgemm.h).  It links the CUDA
runtime statically; NCCL is opened lazily (dlopen) by the sharded layer only.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
# Kernel and C-ABI sources live under task-1/src/vkgemm so that the playground's own anti-library
# scan (it walks task-1/src and task-1/include) covers every kernel.
CSRC = os.path.join(ROOT, "task-1", "src", "vkgemm")
LIB = os.path.join(HERE, "libvkgemm.so")
SOURCES = ["vkgemm.cu", "sharded.cu", "host_gemm.cu", "peer_ipc.cu", "nvls.cu"]
DEPS = SOURCES + ["ptx.cuh", "tc_gemm.cuh", "simt_gemm.cuh", "vk_internal.h"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, d) for d in DEPS] + [os.path.join(ROOT, "include", "vkgemm.h"),
                                                    os.path.abspath(__file__)]
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> str:
    if not force and not _stale():
        return LIB
    cmd = [NVCC, "-std=c++17", "-O3", "-lineinfo", *ARCH, "-Xcompiler", "-fPIC,-O3", "-shared",
           "-I" + os.path.join(ROOT, "include"), "-o", LIB + ".tmp",
           *[os.path.join(CSRC, s) for s in SOURCES], "-ldl"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    if extra:
        cmd[1:1] = extra
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed building libvkgemm.so")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force=True, verbose="--verbose" in sys.argv)
    print(LIB)
