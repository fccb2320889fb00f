"""Build the sm_100a shared library in-tree: ``pagedbatch_b200/_pb_sample.so``.

``python -m pagedbatch_b200.build`` compiles every ``.cu`` file under ``csrc/`` with nvcc for
``sm_100a`` (``-gencode arch=compute_100a,code=sm_100a``) into one C-ABI shared library that
exports the functions declared in ``include/pagedbatch_b200.h``. nvcc cross-compiles without a
GPU, so the library is built on the CPU machine and travels with the source tree.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(REPO, "include")
LIB = os.path.join(PKG, "_pb_sample.so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "-diag-suppress",
    "177",
]


def sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _inputs() -> list[str]:
    files = sources() + [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    return files + [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)]


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(f) <= t for f in _inputs())


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library if any source is newer than it; returns its path."""
    if not force and up_to_date():
        return LIB
    tmp = LIB + ".tmp"
    # -cudart shared: the library binds to the CUDA runtime already loaded in the process (torch's),
    # so both see the same current device; the rpath is the fallback for plain C callers.
    cmd = [nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, "-I", INCLUDE, "-shared", "-cudart", "shared",
           "-Xlinker", "-rpath,/usr/local/cuda/lib64", "-o", tmp, *sources()]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
