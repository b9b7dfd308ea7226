"""Build the sm_100a CUDA library ``libmi_b200.so`` in-tree.

The library is one nvcc translation unit (csrc/mi_b200_unity.cu) exposing the
C ABI declared in include/mi_b200.h.  It links the CUDA runtime statically, so
loading it needs no GPU; the driver is reached at the first CUDA call.

    python -m mamba_integer_b200.build
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
ROOT = os.path.dirname(HERE)
SO = os.path.join(HERE, "libmi_b200.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    # IEEE-exact float arithmetic: no contraction, IEEE div/sqrt, no flush-to-zero
    "-fmad=false", "-prec-div=true", "-prec-sqrt=true", "-ftz=false",
    "-Xcompiler", "-fPIC", "-shared",
]


def _sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh")))


def needs_build() -> bool:
    if not os.path.exists(SO):
        return True
    t = os.path.getmtime(SO)
    deps = _sources() + [os.path.join(ROOT, "include", "mi_b200.h")]
    return any(os.path.getmtime(s) > t for s in deps)


BPE_SO = os.path.join(HERE, "libmi_bpe.so")
BPE_SRC = os.path.join(HERE, "tokenizer", "bpe.cpp")


def build_bpe(force: bool = False) -> str:
    """The host-side tokenizer library libmi_bpe.so (g++, C++17)."""
    deps = [BPE_SRC, os.path.join(HERE, "tokenizer", "unicode_classes.h"), os.path.join(ROOT, "include", "mi_bpe.h")]
    if not force and os.path.exists(BPE_SO) and all(os.path.getmtime(d) <= os.path.getmtime(BPE_SO) for d in deps):
        return BPE_SO
    cxx = shutil.which("g++") or "g++"
    subprocess.run([cxx, "-O2", "-std=c++17", "-fPIC", "-shared", "-Wall", "-o", BPE_SO + ".tmp", BPE_SRC], check=True)
    os.replace(BPE_SO + ".tmp", BPE_SO)
    return BPE_SO


def build(verbose: bool = False, force: bool = False) -> str:
    build_bpe(force=force)
    if not force and not needs_build():
        return SO
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    cmd = [nvcc, *NVCC_FLAGS, "-o", SO + ".tmp", os.path.join(CSRC, "mi_b200_unity.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True, cwd=CSRC)
    os.replace(SO + ".tmp", SO)
    return SO


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force=True))
