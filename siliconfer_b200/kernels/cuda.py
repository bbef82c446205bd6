"""B200 replacement of ``siliconfer.kernels.neon`` (same names, same semantics).

Mirrors siliconfer/kernels/neon/__init__.py:230-239:
``pack_weights_sym``, ``pack_weights_asym``, ``gemv_sym``, ``gemv_scalar``,
``gemv_asym``, ``gemm_sym``, ``gemm_asym``, plus ``CUDA_AVAILABLE`` (the
counterpart of ``NEON_AVAILABLE``) and ``dequant``.

* numpy inputs -> numpy float32 outputs, exactly like the reference.  The
  arrays are copied to the current CUDA device, the kernel runs there, and the
  result is copied back (synchronous, like the reference's GIL-holding call).
* torch CUDA tensors -> torch tensors on the same device, asynchronous on the
  current stream (no host round trip).

There is no numpy or CPU fallback: without a CUDA device every compute call
raises RuntimeError.  Shape checks raise RuntimeError with the reference
binding's messages (siliconfer/kernels/neon/bindings.cpp:24-40, 98-140).
"""
from __future__ import annotations

import numpy as np

from .. import _lib
from ..quant import pack_weights_asym, pack_weights_sym  # noqa: F401  (re-exported API)

try:
    import torch
except ImportError:  # pragma: no cover - torch is part of the image
    torch = None


def _cuda_available() -> bool:
    if torch is None or not torch.cuda.is_available():
        return False
    try:
        _lib.load()
        return True
    except Exception:
        return False


CUDA_AVAILABLE = _cuda_available()
_BACKEND = "cuda-sm100a" if CUDA_AVAILABLE else "unavailable"

def _dtype_code(t) -> int:
    if t.dtype == torch.float32:
        return _lib.SF_F32
    if t.dtype == torch.float16:
        return _lib.SF_F16
    if t.dtype == torch.bfloat16:
        return _lib.SF_BF16
    raise RuntimeError(f"unsupported activation dtype {t.dtype}")


def _require_cuda():
    if not CUDA_AVAILABLE:
        raise RuntimeError("siliconfer_b200 needs a CUDA device and libsf_q4.so; "
                           "there is no CPU fallback")


def _as_device(a, dtype, device):
    """numpy / torch -> contiguous torch tensor of `dtype` on `device`."""
    if isinstance(a, torch.Tensor):
        return a.to(device=device, dtype=dtype).contiguous()
    return torch.from_numpy(np.ascontiguousarray(a)).to(device=device, dtype=dtype)


def _shape(a):
    return tuple(a.shape)


def _check_weights(W, scales, group_size, zeros=None, bits: int = 4):
    if len(_shape(W)) != 2:
        raise RuntimeError("W must be 2-D [out, in/2]" if bits == 4 else "W must be 2-D [out, in/4]")
    if len(_shape(scales)) != 2:
        raise RuntimeError("scales must be 2-D [out, n_groups]")
    out_f, in_f = _shape(W)[0], _shape(W)[1] * (8 // bits)
    if group_size <= 0:
        raise RuntimeError("group_size must be positive")
    n_groups = in_f // group_size
    if _shape(scales) != (out_f, n_groups):
        raise RuntimeError("scales shape mismatch")
    if zeros is not None and _shape(zeros) != (out_f, n_groups):
        raise RuntimeError("zeros shape mismatch")
    return out_f, in_f


def linear(packed, scales, zeros, X, group_size: int = 128, bias=None,
           out_dtype=None, pdl: bool = False, bits: int = 4):
    """Y[T, N] = X[T, K] @ dequant(W)^T (+ bias) on the GPU.

    All tensor arguments must already be CUDA tensors on one device; X may be
    fp32, fp16 or bf16; Y is fp32 unless ``out_dtype`` says otherwise.  The
    call goes through the torch binding (_sf_ext), which allocates Y and runs
    sf_q4_linear / sf_q2_linear on torch's current stream.
    ``bits=2``: ``packed`` holds four 2-bit weights per byte (sf_q2_linear).
    """
    _require_cuda()
    return _lib.ext().linear(packed, scales, zeros, bias, X, group_size,
                             out_dtype or torch.float32, bits, pdl)


def _run(packed, scales, zeros, X, group_size, scalar=False):
    """Shared body of gemv_* / gemm_*: X is [T, K] (numpy or torch)."""
    _require_cuda()
    host = not isinstance(X, torch.Tensor)
    dev = X.device if not host and X.is_cuda else torch.device("cuda", torch.cuda.current_device())
    Wd = _as_device(packed, torch.uint8, dev)
    Sd = _as_device(scales, torch.float32, dev)
    Zd = None if zeros is None else _as_device(zeros, torch.float32, dev)
    if host:
        Xd = _as_device(np.asarray(X, np.float32), torch.float32, dev)
    else:
        Xd = X.to(dev).contiguous()
        if Xd.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            Xd = Xd.float()
    T, K = Xd.shape
    N = Wd.shape[0]
    with torch.cuda.device(dev):
        if scalar:
            Y = torch.empty((T, N), dtype=torch.float32, device=dev)
            lib = _lib.load()
            stream = torch.cuda.current_stream(dev).cuda_stream
            if Xd.dtype != torch.float32:
                Xd = Xd.float()
            for t in range(T):
                _lib.check(lib.sf_q4_gemv_scalar(Wd.data_ptr(), Sd.data_ptr(),
                                                 Xd[t].data_ptr(), Y[t].data_ptr(),
                                                 N, K, group_size, stream))
        else:
            Y = _lib.ext().linear(Wd, Sd, Zd, None, Xd, group_size, torch.float32)
    if host:
        return Y.cpu().numpy()
    return Y


def _vec(x):
    if len(_shape(x)) != 1:
        raise RuntimeError("x must be 1-D [in_f]")
    return x[None, :]


def _mat(X, in_f):
    if len(_shape(X)) != 2:
        raise RuntimeError("X must be 2-D [T, in_f]")
    if _shape(X)[1] != in_f:
        raise RuntimeError("X/W in_features mismatch")
    return X


def _gemv(packed, scales, zeros, x, group_size, scalar=False):
    _, in_f = _check_weights(packed, scales, group_size, zeros)
    X = _vec(x)
    if _shape(X)[1] != in_f:
        raise RuntimeError("x length mismatch")
    if in_f % group_size != 0:
        raise RuntimeError("in_features must be divisible by group_size")
    return _run(packed, scales, zeros, X, group_size, scalar)[0]


def gemv_sym(packed, scales, x, group_size: int = 128):
    """Symmetric int4 GEMV y = dequant(W) @ x (reference __init__.py:127-141)."""
    return _gemv(packed, scales, None, x, group_size)


def gemv_scalar(packed, scales, x, group_size: int = 128):
    """The simple one-warp-per-row kernel (the reference's scalar-C role,
    __init__.py:144-158)."""
    return _gemv(packed, scales, None, x, group_size, scalar=True)


def gemv_asym(packed, scales, zeros, x, group_size: int = 128):
    """Asymmetric int4 GEMV (reference __init__.py:161-176)."""
    return _gemv(packed, scales, zeros, x, group_size)


def gemm_sym(packed, scales, X, group_size: int = 128):
    """Y[T, out] = X[T, in] @ W_q4.T (reference __init__.py:179-197)."""
    _, in_f = _check_weights(packed, scales, group_size)
    X = _mat(X, in_f)
    if in_f % group_size != 0:
        raise RuntimeError("in_features must be divisible by group_size")
    return _run(packed, scales, None, X, group_size)


def gemm_asym(packed, scales, zeros, X, group_size: int = 128):
    """Y = X @ ((W_q4 - zero) * scale).T (reference __init__.py:200-227)."""
    _, in_f = _check_weights(packed, scales, group_size, zeros)
    X = _mat(X, in_f)
    if in_f % group_size != 0:
        raise RuntimeError("in_features must be divisible by group_size")
    return _run(packed, scales, zeros, X, group_size)


def dequant(packed, scales, zeros=None, group_size: int = 128, out_dtype=None):
    """Device dequant -> torch [N, K]; fp32 is bit-exact with the reference's
    dequantize_sym / dequantize_asym."""
    _require_cuda()
    out_f, in_f = _check_weights(packed, scales, group_size, zeros)
    dev = packed.device if isinstance(packed, torch.Tensor) and packed.is_cuda else \
        torch.device("cuda", torch.cuda.current_device())
    Wd = _as_device(packed, torch.uint8, dev)
    Sd = _as_device(scales, torch.float32, dev)
    Zd = None if zeros is None else _as_device(zeros, torch.float32, dev)
    out_dtype = out_dtype or torch.float32
    out = torch.empty((out_f, in_f), dtype=out_dtype, device=dev)
    lib = _lib.load()
    with torch.cuda.device(dev):
        _lib.check(lib.sf_q4_dequant(Wd.data_ptr(), Sd.data_ptr(),
                                     None if Zd is None else Zd.data_ptr(), out.data_ptr(),
                                     _dtype_code(out), out_f, in_f, group_size,
                                     torch.cuda.current_stream(dev).cuda_stream))
    return out


__all__ = ["CUDA_AVAILABLE", "pack_weights_sym", "pack_weights_asym", "gemv_sym",
           "gemv_scalar", "gemv_asym", "gemm_sym", "gemm_asym", "dequant", "linear"]
