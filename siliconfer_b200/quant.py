"""Format producers for the Q4Linear storage (host numpy + device CUDA).

The packed triple (packed uint8 [N, K/2], fp32 scales [N, G], fp32 zeros
[N, G] or None) is siliconfer's storage format, so the outputs of its
RTN/GPTQ/AWQ/HQQ/SINQ pipelines load unchanged.  The host functions restate
the reference's packers bit for bit:

* ``quantize_sym``  -- siliconfer/quant/primitives.py:24-51
* ``quantize_asym`` -- siliconfer/quant/primitives.py:82-114
* ``pack_weights_sym`` / ``pack_weights_asym`` --
  siliconfer/kernels/neon/__init__.py:42-81 (low nibble = even column)

``pack_weights_*_device`` run the same RTN arithmetic on the GPU
(``sf_q4_quantize_pack``), for weights too large to quantize on the host.
"""
from __future__ import annotations

import numpy as np

from . import _lib


def _grouped(w: np.ndarray, group_size: int) -> np.ndarray:
    rows, cols = w.shape
    if cols % group_size != 0:
        raise ValueError(f"cols={cols} not divisible by group_size={group_size}")
    return w.reshape(rows, cols // group_size, group_size)


def quantize_sym(w: np.ndarray, group_size: int = 128):
    """int4 in [-8, 7] and fp32 scale = absmax / 7 per group."""
    g = _grouped(np.asarray(w, np.float32), group_size)
    scale = (np.abs(g).max(axis=-1, keepdims=True) / np.float32(7)).astype(np.float32)
    div = np.where(scale == 0.0, np.float32(1.0), scale)
    q = np.round(g / div).clip(-8, 7).astype(np.int8)
    return q.reshape(w.shape), scale[..., 0]


def quantize_asym(w: np.ndarray, group_size: int = 128):
    """uint4 in [0, 15], fp32 scale = (max - min) / 15, integer-valued fp32 zero."""
    g = _grouped(np.asarray(w, np.float32), group_size)
    lo, hi = g.min(axis=-1, keepdims=True), g.max(axis=-1, keepdims=True)
    scale = ((hi - lo) / np.float32(15)).astype(np.float32)
    div = np.where(scale == 0.0, np.float32(1.0), scale)
    zero = np.round(-lo / div).clip(0, 15).astype(np.float32)
    q = (np.round(g / div) + zero).clip(0, 15).astype(np.uint8)
    return q.reshape(w.shape), scale[..., 0], zero[..., 0]


def _pack(q: np.ndarray) -> np.ndarray:
    nib = q.astype(np.uint8) & np.uint8(0x0F)
    return (nib[:, 0::2] | (nib[:, 1::2] << 4)).astype(np.uint8)


def pack_weights_sym(W: np.ndarray, group_size: int = 128):
    """-> (packed uint8 [out, in/2], scales fp32 [out, in/group_size])."""
    q, s = quantize_sym(np.asarray(W, np.float32), group_size)
    return _pack(q), s


def pack_weights_asym(W: np.ndarray, group_size: int = 128):
    """-> (packed uint8 [out, in/2], scales fp32, zeros fp32 [out, in/group_size])."""
    q, s, z = quantize_asym(np.asarray(W, np.float32), group_size)
    return _pack(q), s, z


# ---------------------------------------------------------------------------
# 2-bit weights (siliconfer/quant/primitives.py:154-245, 383-404)
# ---------------------------------------------------------------------------
def quantize_sym_int2(w: np.ndarray, group_size: int = 128):
    """int2 in [-2, 1] and fp32 scale = absmax / 1 per group (primitives.py:154-181)."""
    g = _grouped(np.asarray(w, np.float32), group_size)
    scale = (np.abs(g).max(axis=-1, keepdims=True) / np.float32(1)).astype(np.float32)
    div = np.where(scale == 0.0, np.float32(1.0), scale)
    q = np.round(g / div).clip(-2, 1).astype(np.int8)
    return q.reshape(w.shape), scale[..., 0]


def quantize_asym_int2(w: np.ndarray, group_size: int = 128):
    """uint2 in [0, 3], fp32 scale = (max - min) / 3, integer-valued fp32 zero
    (primitives.py:203-231)."""
    g = _grouped(np.asarray(w, np.float32), group_size)
    lo, hi = g.min(axis=-1, keepdims=True), g.max(axis=-1, keepdims=True)
    scale = ((hi - lo) / np.float32(3)).astype(np.float32)
    div = np.where(scale == 0.0, np.float32(1.0), scale)
    zero = np.round(-lo / div).clip(0, 3).astype(np.float32)
    q = (np.round(g / div) + zero).clip(0, 3).astype(np.uint8)
    return q.reshape(w.shape), scale[..., 0], zero[..., 0]


def pack_int2(q: np.ndarray) -> np.ndarray:
    """Four 2-bit values per byte, element i in bits 2i..2i+1 (primitives.py:383-404);
    rows are packed independently ([N, K] -> [N, K/4])."""
    v = (np.asarray(q).astype(np.int32) & 3).astype(np.uint8)
    return (v[:, 0::4] | (v[:, 1::4] << 2) | (v[:, 2::4] << 4) | (v[:, 3::4] << 6)).astype(np.uint8)


def pack_weights_int2_sym(W: np.ndarray, group_size: int = 128):
    """-> (packed uint8 [out, in/4], scales fp32 [out, in/group_size])."""
    q, s = quantize_sym_int2(np.asarray(W, np.float32), group_size)
    return pack_int2(q), s


def pack_weights_int2_asym(W: np.ndarray, group_size: int = 128):
    """-> (packed uint8 [out, in/4], scales fp32, zeros fp32 [out, in/group_size])."""
    q, s, z = quantize_asym_int2(np.asarray(W, np.float32), group_size)
    return pack_int2(q), s, z


def pack_weights_device(W, group_size: int = 128, sym: bool = True):
    """RTN quantize + pack an fp32 CUDA tensor [N, K] on its device.

    Bit-exact with ``pack_weights_sym`` / ``pack_weights_asym``; returns torch
    tensors (packed, scales[, zeros]) on the same device."""
    import torch
    if not (isinstance(W, torch.Tensor) and W.is_cuda):
        raise TypeError("pack_weights_device needs a CUDA tensor")
    W = W.contiguous().float()
    n, k = W.shape
    if k % group_size or group_size % 2:
        raise ValueError(f"cols={k} not divisible by group_size={group_size}")
    packed = torch.empty((n, k // 2), dtype=torch.uint8, device=W.device)
    scales = torch.empty((n, k // group_size), dtype=torch.float32, device=W.device)
    zeros = None if sym else torch.empty_like(scales)
    lib = _lib.load()
    with torch.cuda.device(W.device):
        _lib.check(lib.sf_q4_quantize_pack(
            W.data_ptr(), packed.data_ptr(), scales.data_ptr(),
            None if zeros is None else zeros.data_ptr(), n, k, group_size,
            torch.cuda.current_stream(W.device).cuda_stream))
    return (packed, scales) if sym else (packed, scales, zeros)
