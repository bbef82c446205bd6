"""ctypes binding of the C ABI in include/sf_q4.h (libsf_q4.so).

There is no CPU fallback: if the library is missing or no CUDA device is
present, every compute call raises.  Status codes map to RuntimeError with the
library's message, as the reference's pybind layer raises std::runtime_error
(siliconfer/kernels/neon/bindings.cpp:24-40).
"""
from __future__ import annotations

import ctypes
import pathlib

_PKG = pathlib.Path(__file__).resolve().parent
LIB_PATH = _PKG / "libsf_q4.so"

SF_F32, SF_F16, SF_BF16 = 0, 1, 2
SF_FLAG_PDL = 1
SF_EPI_SWIGLU = 1
SF_OK = 0

_P, _I, _LL = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong
_SZ = ctypes.c_size_t


class Q4Task(ctypes.Structure):
    """Mirror of sf_q4_task (include/sf_q4.h)."""
    _fields_ = [("W", _P), ("scales", _P), ("zeros", _P), ("bias", _P), ("X", _P), ("Y", _P),
                ("N", _I), ("K", _I), ("T", _I), ("group_size", _I), ("x_dtype", _I),
                ("y_dtype", _I), ("wait_before", _I), ("epilogue", _I), ("bits", _I)]

# name -> argtypes (restype is int unless listed in _RESTYPES)
SIGNATURES = {
    "sf_status_string": [_I],
    "sf_last_error": [],
    "sf_version": [],
    "sf_q4_gemv_sym": [_P, _P, _P, _P, _I, _I, _I, _P],
    "sf_q4_gemv_scalar": [_P, _P, _P, _P, _I, _I, _I, _P],
    "sf_q4_gemv_asym": [_P, _P, _P, _P, _P, _I, _I, _I, _P],
    "sf_q4_gemm_sym": [_P, _P, _P, _P, _I, _I, _I, _I, _P],
    "sf_q4_gemm_asym": [_P, _P, _P, _P, _P, _I, _I, _I, _I, _P],
    "sf_q4_linear": [_P, _P, _P, _P, _P, _I, _P, _I, _I, _I, _I, _I, _I, _P],
    "sf_q4_linear_static_scratch": [_P, _P, _P, _P, _P, _I, _P, _I, _I, _I, _I, _I, _P],
    "sf_q4_linear_swiglu": [_P, _P, _P, _P, _P, _I, _P, _I, _I, _I, _I, _I, _P],
    "sf_q2_linear": [_P, _P, _P, _P, _P, _I, _P, _I, _I, _I, _I, _I, _P],
    "sf_swiglu_interleaved": [_P, _P, _I, _I, _I, _P, _P],
    "sf_q4_dequant": [_P, _P, _P, _P, _I, _I, _I, _I, _P],
    "sf_q4_quantize_pack": [_P, _P, _P, _P, _I, _I, _I, _P],
    "sf_q4_check_device_error": [],
    "sf_q4_launch_count": [],
    "sf_q4_step_workspace_bytes": [ctypes.POINTER(Q4Task), _I],
    "sf_q4_step_create": [ctypes.POINTER(Q4Task), _I, _P, _SZ, ctypes.POINTER(_P)],
    "sf_q4_step_run": [_P, _P],
    "sf_q4_step_destroy": [_P],
    "sf_tp_handle_bytes": [],
    "sf_tp_comm_init": [_I, _I, _SZ, _SZ, ctypes.POINTER(_P), _P],
    "sf_q4_step_create_tp": [ctypes.POINTER(Q4Task), ctypes.POINTER(_I), _I, _P, _P, _SZ, ctypes.POINTER(_P)],
    "sf_tp_comm_connect": [_P, _P],
    "sf_tp_allreduce": [_P, _P, _P, _I, _P, _LL, _I, _P],
    "sf_q4_linear_allreduce": [_P, _P, _P, _P, _P, _P, _I, _P, _I, _I, _I, _I, _I, _P],
    "sf_tp_comm_destroy": [_P],
    "sf_kv_attention_workspace_bytes": [_I, _I, _I, _I],
    "sf_kv_attention_splits": [_I, _I, _I],
    "sf_kv_attention_decode": [_P, _I, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P, _SZ, _P],
}
_RESTYPES = {"sf_status_string": ctypes.c_char_p, "sf_last_error": ctypes.c_char_p,
             "sf_q4_launch_count": _LL, "sf_q4_step_workspace_bytes": _SZ,
             "sf_q4_step_destroy": None, "sf_tp_handle_bytes": _SZ, "sf_tp_comm_destroy": None,
             "sf_kv_attention_workspace_bytes": _SZ}

_lib = None


def load():
    """Load libsf_q4.so (building it first if nvcc is available here)."""
    global _lib
    if _lib is not None:
        return _lib
    from . import build as _build
    if _build.needs_build():
        try:
            _build.build()
        except Exception as exc:  # no nvcc on this host and no prebuilt library
            if not LIB_PATH.exists():
                raise RuntimeError(f"{LIB_PATH} is missing and could not be built: {exc}") from exc
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = _RESTYPES.get(name, _I)
    _lib = lib
    return lib


_ext = None


def ext():
    """The torch binding (_sf_ext, built from csrc/sf_torch_ext.cpp next to
    libsf_q4.so).  It calls the same C entry points as the ctypes handle
    above, on torch's current stream; RuntimeError if it is missing."""
    global _ext
    if _ext is None:
        load()
        from . import build as _build
        if _build.ext_stale():
            try:
                _build.build_ext()
            except Exception as exc:
                if not _build.ext_path().exists():
                    raise RuntimeError(f"{_build.ext_path()} is missing and could not be built: {exc}") from exc
        from . import _sf_ext
        _ext = _sf_ext
    return _ext


def check(rc: int) -> None:
    if rc != SF_OK:
        lib = load()
        msg = lib.sf_last_error().decode() or lib.sf_status_string(rc).decode()
        raise RuntimeError(msg)


def launch_count() -> int:
    return int(load().sf_q4_launch_count())
