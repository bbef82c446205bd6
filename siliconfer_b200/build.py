"""Build the sm_100a kernel library in-tree: siliconfer_b200/libsf_q4.so.

    python -m siliconfer_b200.build

nvcc cross-compiles for sm_100a without a GPU.  The library is a plain C ABI
(include/sf_q4.h) loaded with ctypes, so no torch headers are involved.
"""
from __future__ import annotations

import os
import pathlib
import shutil
import subprocess
import sys

PKG = pathlib.Path(__file__).resolve().parent
ROOT = PKG.parent
LIB = PKG / "libsf_q4.so"
SOURCES = [PKG / "csrc" / "sf_q4.cu", PKG / "csrc" / "sf_q4_gemm_tc.cu", PKG / "csrc" / "sf_q4_tile.cu",
           PKG / "csrc" / "sf_q4_tp.cu", PKG / "csrc" / "sf_kv_attention.cu"]
HEADERS = [ROOT / "include" / "sf_q4.h", PKG / "csrc" / "sf_q4_internal.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and pathlib.Path(c).exists():
            return c
    raise RuntimeError("nvcc not found")


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.exists() and p.stat().st_mtime > t for p in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False) -> pathlib.Path:
    """Compiles every source to an object in parallel (nvcc is single-threaded
    per file), then links the shared library."""
    from concurrent.futures import ThreadPoolExecutor
    if not force and not needs_build():
        return LIB
    srcs = [p for p in SOURCES if p.exists()]
    objdir = PKG / "_build"
    objdir.mkdir(exist_ok=True)
    flags = [*ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
             f"-I{ROOT / 'include'}", f"-I{PKG / 'csrc'}"]
    if verbose:
        flags.insert(0, "-Xptxas=-v")

    def compile_one(src):
        obj = objdir / (src.stem + ".o")
        cmd = [nvcc(), *flags, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
        return str(obj)

    with ThreadPoolExecutor(max_workers=max(1, min(len(srcs), os.cpu_count() or 1))) as ex:
        objs = list(ex.map(compile_one, srcs))
    subprocess.run([nvcc(), *ARCH, "-shared", "-o", str(LIB) + ".tmp", *objs], check=True)
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
