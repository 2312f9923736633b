"""Builds libunpopped_sm100.so in-tree with nvcc for sm_100a (B200 only).

    python -m unpopped_b200.build          # or: python unpopped_b200/build.py

Sources: unpopped_b200/csrc/*.cu. Output: unpopped_b200/libunpopped_sm100.so, which the snapshot carries to
the GPU box. Objects are compiled in parallel and relinked only when a source or header changed.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libunpopped_sm100.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include"),
]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the sm_100a library cannot be built")


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + [os.path.join(ROOT, "include", "up_sm100.h")]


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def revision_hash(path: str) -> int:
    """FNV-1a 64 over a source file's bytes: the reference's revision hash (crates/unpopped/src/revision.rs)."""
    h = 0xCBF29CE484222325
    with open(path, "rb") as f:
        for b in f.read():
            h = ((h ^ b) * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


def _compile(src: str, extra) -> str:
    obj = os.path.join(OBJ, os.path.basename(src) + ".o")
    if _stale(obj, [src] + _headers()):
        rev = f"-DUP_SOURCE_REVISION=0x{revision_hash(src):016x}ull"
        cmd = [nvcc()] + NVCC_FLAGS + [rev] + list(extra) + ["-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(verbose: bool = False, extra=()) -> str:
    """Compile every csrc/*.cu for sm_100a and link the shared library; returns its path."""
    os.makedirs(OBJ, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra), srcs))
    if _stale(LIB, objs):
        tmp = LIB + ".tmp"
        cmd = [nvcc()] + ARCH + ["-shared", "-o", tmp] + objs + ["-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    if verbose:
        print(LIB)
    return LIB


def ptxas_report(src_name: str) -> str:
    """Register / spill / shared-memory report of one source (nvcc -Xptxas -v)."""
    src = os.path.join(CSRC, src_name)
    cmd = [nvcc()] + NVCC_FLAGS + ["-Xptxas", "-v", "-c", src, "-o", os.devnull]
    r = subprocess.run(cmd, capture_output=True, text=True)
    return r.stdout + r.stderr


if __name__ == "__main__":
    if len(sys.argv) > 1 and sys.argv[1] == "--ptxas":
        for name in sys.argv[2:]:
            print(ptxas_report(name))
    else:
        build(verbose=True)
