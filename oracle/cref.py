"""ctypes access to the compiled CPU checkers -- TEST/BASELINE INFRASTRUCTURE ONLY.

* ``oracle_gemm``: our C restatement (``oracle/q4_oracle.c``), threaded over rows.
* ``ref_gemm``: the reference's own ``q4_gemv_sym_neon`` / ``q4_gemv_asym_neon``
  (siliconfer/kernels/neon/q4_gemv.cpp) compiled from the reference tree into
  ``oracle/_ref/libsf_ref.so`` by ``oracle/Makefile``; rows are split over host
  threads and each slice runs the reference kernel per token as
  siliconfer/kernels/neon/q4_gemm.cpp:19-24 does.
"""
from __future__ import annotations

import ctypes
import os
import pathlib
import subprocess

import numpy as np

_HERE = pathlib.Path(__file__).resolve().parent
_P = ctypes.c_void_p
_I = ctypes.c_int


def reference_root() -> str | None:
    """Root of the siliconfer reference tree: $SILICONFER_REF, else the
    ``reference_path`` that BASELINE.json records; None when neither exists."""
    ref = os.environ.get("SILICONFER_REF")
    if not ref:
        meta = _HERE.parent / "BASELINE.json"
        if meta.exists():
            import json
            ref = json.loads(meta.read_text()).get("reference_path")
    return ref if ref and pathlib.Path(ref).is_dir() else None


def build() -> None:
    """Compile the checkers (make -C oracle); the reference's own kernels only
    when its source tree is present (see reference_root)."""
    ref = reference_root()
    subprocess.run(["make", "-s", "-C", str(_HERE)] + ([f"REF={ref}"] if ref else []), check=True)


def _load(path: pathlib.Path):
    if not path.exists():
        build()
    return ctypes.CDLL(str(path))


_lib_oracle = None
_lib_ref = None


def oracle_lib():
    global _lib_oracle
    if _lib_oracle is None:
        _lib_oracle = _load(_HERE / "liboracle_q4.so")
        _lib_oracle.oracle_q4_gemm.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I]
        _lib_oracle.oracle_q4_gemm.restype = _I
        _lib_oracle.oracle_q4_dequant.argtypes = [_P, _P, _P, _P, _I, _I, _I]
    return _lib_oracle


def ref_lib():
    """The reference's compiled kernels, or None when they were never built."""
    global _lib_ref
    if _lib_ref is None:
        p = _HERE / "_ref" / "libsf_ref.so"
        if not p.exists():
            return None
        _lib_ref = ctypes.CDLL(str(p))
        _lib_ref.ref_q4_gemm.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I]
        _lib_ref.ref_q4_gemm.restype = _I
        _lib_ref.ref_asym_is_correct.restype = _I
    return _lib_ref


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _prep(packed, scales, zeros, X):
    packed = np.ascontiguousarray(packed, np.uint8)
    scales = np.ascontiguousarray(scales, np.float32)
    zeros = None if zeros is None else np.ascontiguousarray(zeros, np.float32)
    X = np.ascontiguousarray(np.atleast_2d(X), np.float32)
    return packed, scales, zeros, X


def oracle_gemm(packed, scales, zeros, X, group_size=128, threads=None):
    packed, scales, zeros, X = _prep(packed, scales, zeros, X)
    n, k = packed.shape[0], packed.shape[1] * 2
    Y = np.empty((X.shape[0], n), np.float32)
    rc = oracle_lib().oracle_q4_gemm(_ptr(packed), _ptr(scales), _ptr(zeros), _ptr(X),
                                     _ptr(Y), n, k, X.shape[0], group_size,
                                     threads or os.cpu_count() or 1)
    if rc:
        raise ValueError("oracle_q4_gemm rejected the shapes")
    return Y


def oracle_dequant(packed, scales, zeros, group_size=128):
    packed = np.ascontiguousarray(packed, np.uint8)
    scales = np.ascontiguousarray(scales, np.float32)
    zeros = None if zeros is None else np.ascontiguousarray(zeros, np.float32)
    n, k = packed.shape[0], packed.shape[1] * 2
    out = np.empty((n, k), np.float32)
    oracle_lib().oracle_q4_dequant(_ptr(packed), _ptr(scales), _ptr(zeros), _ptr(out),
                                   n, k, group_size)
    return out


def ref_available(asym: bool = False) -> bool:
    lib = ref_lib()
    if lib is None:
        return False
    return bool(lib.ref_asym_is_correct()) if asym else True


def ref_gemm(packed, scales, zeros, X, group_size=128, threads=None):
    lib = ref_lib()
    if lib is None:
        raise RuntimeError("oracle/_ref/libsf_ref.so was not built")
    if zeros is not None and not lib.ref_asym_is_correct():
        raise RuntimeError("the reference's asym kernel is wrong on this host "
                           "(q4_gemv.cpp:249-255); use the oracle port")
    packed, scales, zeros, X = _prep(packed, scales, zeros, X)
    n, k = packed.shape[0], packed.shape[1] * 2
    Y = np.empty((X.shape[0], n), np.float32)
    rc = lib.ref_q4_gemm(_ptr(packed), _ptr(scales), _ptr(zeros), _ptr(X), _ptr(Y),
                         n, k, X.shape[0], group_size, threads or os.cpu_count() or 1)
    if rc:
        raise ValueError("ref_q4_gemm rejected the shapes")
    return Y
