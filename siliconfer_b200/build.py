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
        if ext_stale():
            build_ext(verbose)
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
        futs = list(ex.map(compile_one, srcs))
    subprocess.run([nvcc(), *ARCH, "-shared", "-o", str(LIB) + ".tmp", *futs], check=True)
    os.replace(str(LIB) + ".tmp", LIB)
    build_ext(verbose)
    return LIB


def ext_stale() -> bool:
    out, src = ext_path(), PKG / "csrc" / "sf_torch_ext.cpp"
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(p.stat().st_mtime > t for p in (src, LIB, ROOT / "include" / "sf_q4.h") if p.exists())


def ext_path() -> pathlib.Path:
    import sysconfig
    return PKG / ("_sf_ext" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_ext(verbose: bool = False) -> pathlib.Path:
    """The thin torch binding (csrc/sf_torch_ext.cpp), compiled in-tree with
    torch's headers and linked against libsf_q4.so (found next to it)."""
    import sysconfig
    import torch
    from torch.utils import cpp_extension as ce
    src = PKG / "csrc" / "sf_torch_ext.cpp"
    out = ext_path()
    incs = ce.include_paths(device_type="cuda")
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-DTORCH_EXTENSION_NAME=_sf_ext",
           f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
           *[f"-I{p}" for p in incs], f"-I{sysconfig.get_paths()['include']}", f"-I{ROOT / 'include'}",
           str(src), "-o", str(out) + ".tmp",
           *[f"-L{p}" for p in ce.library_paths()], "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
           "-ltorch_cuda", "-ltorch_python", f"-L{PKG}", "-l:libsf_q4.so", "-Wl,-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(str(out) + ".tmp", out)
    return out


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
