"""Builds libqsamp.so in-tree for sm_100a (nvcc cross-compiles without a GPU)."""
from __future__ import annotations

import os
import shutil
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libqsamp.so")
SOURCES = [os.path.join(CSRC, f) for f in ("qsamp_kernels.cu", "qsamp_api.cu", "qsamp_static.cu",
                                            "qsamp_trie_api.cpp")] + [os.path.join(HERE, "trie", "compact_trie.cpp")]
HEADERS = [os.path.join(CSRC, f) for f in ("qs_math.h", "qsamp_device.h", "qsamp_hist.cuh")] + [
    os.path.join(ROOT, "include", "qsamp.h"), os.path.join(HERE, "trie", "compact_trie.h")]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# IEEE float semantics are part of the contract: no --use_fast_math.
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-extended-lambda", "-Xcompiler", "-fPIC", "-cudart", "shared"]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(p) > t for p in SOURCES + HEADERS)


COMM_LIB = os.path.join(HERE, "libqsamp_comm.so")
COMM_SOURCES = [os.path.join(CSRC, "qsamp_comm.cpp")]
COMM_HEADERS = [os.path.join(ROOT, "include", "qsamp_comm.h"), os.path.join(ROOT, "include", "qsamp.h")]


def nccl_flags() -> list:
    """Compile and link against the NCCL that torch loads (the nvidia-nccl
    wheel), so that a process holding both libraries holds one NCCL; the
    system NCCL otherwise."""
    try:
        import nvidia.nccl as nn

        base = os.path.dirname(nn.__file__) if nn.__file__ else list(nn.__path__)[0]
        inc, lib = os.path.join(base, "include"), os.path.join(base, "lib")
        if os.path.exists(os.path.join(inc, "nccl.h")) and os.path.exists(os.path.join(lib, "libnccl.so.2")):
            return ["-I" + inc, "-L" + lib, "-Xlinker", "-rpath," + lib, "-l:libnccl.so.2"]
    except ImportError:
        pass
    return ["-lnccl"]


def build_comm(force: bool = False) -> str:
    """libqsamp_comm.so: the NCCL candidate exchange with deadlines (host
    code; links the system NCCL)."""
    if not force and os.path.exists(COMM_LIB) and all(
            os.path.getmtime(p) <= os.path.getmtime(COMM_LIB) for p in COMM_SOURCES + COMM_HEADERS):
        return COMM_LIB
    cmd = [nvcc(), "-shared", "-O2", "-std=c++17", "-Xcompiler", "-fPIC", "-Wno-deprecated-gpu-targets", "-o",
           COMM_LIB, *COMM_SOURCES, *nccl_flags()]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + res.stdout + res.stderr)
    return COMM_LIB


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not stale():
        return LIB
    cmd = [nvcc(), "-shared", *ARCH, *FLAGS, "-o", LIB, *SOURCES]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + res.stdout + res.stderr)
    if verbose:
        print(res.stdout + res.stderr)
    return LIB


if __name__ == "__main__":
    print(build(force=True, verbose=True))
    print(build_comm(force=True))
