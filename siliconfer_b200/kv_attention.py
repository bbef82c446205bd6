"""Decode-phase attention over an int8-quantized KV cache on the GPU.

Mirrors siliconfer's ``fused_quantized_attention_decode``
(siliconfer/kernels/metal/q4_attention.py:200-260) and its cache format
(``quantize_kv``, siliconfer/model/kv_cache.py:49-69): int8 codes with one
fp32 scale per (batch, kv head, token) vector, dequantized inline, online
softmax split over the cache length, merged with the flash-attention rule.
The kernels are in libsf_q4.so (``sf_kv_attention_decode``); there is no
CPU fallback.
"""
from __future__ import annotations

import torch

from . import _lib


def quantize_kv(x: torch.Tensor):
    """Symmetric int8 per-vector quantization (kv_cache.py:49-62) on the device:
    returns (codes int8 [..., D], scales fp32 [...])."""
    x32 = x.float()
    amax = x32.abs().amax(dim=-1, keepdim=True)
    scale = torch.where(amax == 0, torch.ones_like(amax), amax / 127.0)
    q = torch.clamp(torch.round(x32 / scale), -128, 127).to(torch.int8)
    return q, scale.squeeze(-1)


def fused_quantized_attention_decode(q, k_codes, k_scales, v_codes, v_scales, n_tiles=None,
                                     out_dtype=torch.float32):
    """q [B, H, D]; k/v codes [B, Hkv, T, D] int8; k/v scales [B, Hkv, T] (or
    [B, Hkv, T, 1]) fp32 -> [B, H, D]."""
    from .kernels.cuda import _dtype_code, _require_cuda
    _require_cuda()
    B, H, D = q.shape
    Hkv, T = k_codes.shape[1], k_codes.shape[2]
    if k_codes.shape != (B, Hkv, T, D) or v_codes.shape != (B, Hkv, T, D):
        raise RuntimeError("k/v codes must be [B, n_kv_heads, T, head_dim]")
    ks = k_scales.reshape(B, Hkv, T).float().contiguous()
    vs = v_scales.reshape(B, Hkv, T).float().contiguous()
    kc, vc, qc = k_codes.contiguous(), v_codes.contiguous(), q.contiguous()
    lib = _lib.load()
    ns = int(n_tiles) if n_tiles else int(lib.sf_kv_attention_splits(B, Hkv, T))
    ns = max(1, min(ns, T))
    nbytes = int(lib.sf_kv_attention_workspace_bytes(B, H, D, ns))
    ws = torch.empty(nbytes // 4 + 1, dtype=torch.float32, device=q.device)
    out = torch.empty((B, H, D), dtype=out_dtype, device=q.device)
    _lib.check(lib.sf_kv_attention_decode(
        qc.data_ptr(), _dtype_code(qc), kc.data_ptr(), ks.data_ptr(), vc.data_ptr(), vs.data_ptr(),
        out.data_ptr(), _dtype_code(out), B, H, Hkv, T, D, ns, ws.data_ptr(), nbytes,
        torch.cuda.current_stream(q.device).cuda_stream))
    return out


__all__ = ["quantize_kv", "fused_quantized_attention_decode"]
