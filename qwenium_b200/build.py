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
