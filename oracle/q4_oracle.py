"""CPU oracle for siliconfer's Q4Linear int4 path -- TEST INFRASTRUCTURE ONLY.

This module is a plain numpy restatement of the reference's algorithm for the
hot path.  It exists to *check* the CUDA implementation; nothing in the product
(``siliconfer_b200``) imports it.  Only ``tests/``, ``__graft_entry__.smoke()``
and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may use it.

Parity pin: every function here is checked against golden vectors produced by
the reference's own Python code (``tests/golden/make_golden.py`` imports
``siliconfer.kernels.neon`` and ``siliconfer.quant`` from the reference tree
and stores their outputs in ``tests/golden/*.npz``), see
``tests/test_oracle_golden.py``.

Reference citations are ``path:line`` inside the siliconfer project.
"""

from __future__ import annotations

import numpy as np

INT4_SYM_MIN, INT4_SYM_MAX, INT4_UINT_MAX = -8, 7, 15


# ---------------------------------------------------------------------------
# Format producers (siliconfer/quant/primitives.py, kernels/neon/__init__.py)
# ---------------------------------------------------------------------------

def quantize_sym(w: np.ndarray, group_size: int = 128):
    """Group-wise symmetric RTN int4 (siliconfer/quant/primitives.py:24-51).

    scale = absmax / 7 in fp32; a zero scale divides by 1; q = round-half-even
    (w / scale) clipped to [-8, 7].
    """
    rows, cols = w.shape
    if cols % group_size:
        raise ValueError(f"cols={cols} not divisible by group_size={group_size}")
    g = w.reshape(rows, cols // group_size, group_size)
    absmax = np.max(np.abs(g), axis=-1, keepdims=True)
    scale = (absmax / np.float32(7)).astype(np.float32)
    safe = np.where(scale == 0, np.float32(1), scale)
    q = np.clip(np.round(g / safe), -8, 7).astype(np.int8)
    return q.reshape(rows, cols), scale[..., 0]


def quantize_asym(w: np.ndarray, group_size: int = 128):
    """Group-wise asymmetric RTN int4 (siliconfer/quant/primitives.py:82-114).

    scale = (max - min) / 15; zero = clip(round(-min / scale), 0, 15) kept as an
    integer-valued float32; q = clip(round(w / scale) + zero, 0, 15).
    """
    rows, cols = w.shape
    if cols % group_size:
        raise ValueError(f"cols={cols} not divisible by group_size={group_size}")
    g = w.reshape(rows, cols // group_size, group_size)
    lo = g.min(axis=-1, keepdims=True)
    hi = g.max(axis=-1, keepdims=True)
    scale = ((hi - lo) / np.float32(15)).astype(np.float32)
    safe = np.where(scale == 0, np.float32(1), scale)
    zero = np.clip(np.round(-lo / safe), 0, 15).astype(np.float32)
    q = np.clip(np.round(g / safe) + zero, 0, 15).astype(np.uint8)
    return q.reshape(rows, cols), scale[..., 0], zero[..., 0]


def pack_nibbles(q: np.ndarray) -> np.ndarray:
    """Even column -> low nibble, odd column -> high nibble
    (siliconfer/kernels/neon/__init__.py:57-62, 76-80)."""
    lo = q[:, 0::2].astype(np.uint8) & 0x0F
    hi = q[:, 1::2].astype(np.uint8) & 0x0F
    return (lo | (hi << 4)).astype(np.uint8)


def pack_weights_sym(w: np.ndarray, group_size: int = 128):
    """siliconfer/kernels/neon/__init__.py:42-63."""
    q, s = quantize_sym(np.asarray(w, np.float32), group_size)
    return pack_nibbles(q), s


def pack_weights_asym(w: np.ndarray, group_size: int = 128):
    """siliconfer/kernels/neon/__init__.py:66-81."""
    q, s, z = quantize_asym(np.asarray(w, np.float32), group_size)
    return pack_nibbles(q), s, z


def unpack_nibbles(packed: np.ndarray, signed: bool) -> np.ndarray:
    """Inverse of pack_nibbles; signed nibbles are two's complement
    (siliconfer/quant/primitives.py:353-376, kernels/neon/q4_gemv.h:5-12)."""
    n, kh = packed.shape
    lo = (packed & 0x0F).astype(np.int16)
    hi = (packed >> 4).astype(np.int16)
    out = np.empty((n, 2 * kh), np.int16)
    out[:, 0::2] = lo
    out[:, 1::2] = hi
    if signed:
        out = np.where(out > 7, out - 16, out)
    return out


def dequantize(packed, scales, zeros=None, group_size: int = 128) -> np.ndarray:
    """fp32 dequant: q*s (sym) or (q - z)*s (asym), one rounding each
    (siliconfer/quant/primitives.py:54-75, 117-140).  This is the bit-exact
    target for the device dequant."""
    q = unpack_nibbles(packed, signed=zeros is None).astype(np.float32)
    n, k = q.shape
    qg = q.reshape(n, k // group_size, group_size)
    if zeros is None:
        w = qg * scales[..., None].astype(np.float32)
    else:
        w = (qg - zeros[..., None].astype(np.float32)) * scales[..., None].astype(np.float32)
    return w.reshape(n, k).astype(np.float32)


# ---------------------------------------------------------------------------
# GEMV / GEMM (siliconfer/kernels/neon/__init__.py:88-124, 179-227)
# ---------------------------------------------------------------------------

def gemv_sym(packed, scales, x, group_size: int = 128) -> np.ndarray:
    """Per group: y += (W_g @ x_g) * s[:, g] with sign-extended nibbles
    (siliconfer/kernels/neon/__init__.py:88-106)."""
    q = unpack_nibbles(packed, signed=True).astype(np.float32)
    x = np.asarray(x, np.float32)
    n, k = q.shape
    y = np.zeros(n, np.float32)
    for g in range(k // group_size):
        sl = slice(g * group_size, (g + 1) * group_size)
        y += (q[:, sl] @ x[sl]) * scales[:, g]
    return y


def gemv_asym(packed, scales, zeros, x, group_size: int = 128) -> np.ndarray:
    """Per group: y += (W_g @ x_g - z[:, g] * sum(x_g)) * s[:, g] with unsigned
    nibbles (siliconfer/kernels/neon/__init__.py:109-124)."""
    q = unpack_nibbles(packed, signed=False).astype(np.float32)
    x = np.asarray(x, np.float32)
    n, k = q.shape
    y = np.zeros(n, np.float32)
    for g in range(k // group_size):
        sl = slice(g * group_size, (g + 1) * group_size)
        y += (q[:, sl] @ x[sl] - zeros[:, g] * x[sl].sum()) * scales[:, g]
    return y


def gemm(packed, scales, zeros, X, group_size: int = 128) -> np.ndarray:
    """Y[T, N] for T tokens.  The reference loops the GEMV per token
    (siliconfer/kernels/neon/__init__.py:191-197, 221-227); this restatement
    evaluates all tokens per group at once with the same per-group algebra."""
    X = np.atleast_2d(np.asarray(X, np.float32))
    signed = zeros is None
    q = unpack_nibbles(packed, signed=signed).astype(np.float32)
    n, k = q.shape
    Y = np.zeros((X.shape[0], n), np.float32)
    for g in range(k // group_size):
        sl = slice(g * group_size, (g + 1) * group_size)
        part = X[:, sl] @ q[:, sl].T
        if not signed:
            part -= X[:, sl].sum(axis=1, keepdims=True) * zeros[:, g][None, :]
        Y += part * scales[:, g][None, :]
    return Y


def q4linear_forward(packed, scales, zeros, bias, x, group_size: int = 128):
    """Q4Linear.__call__ restated (siliconfer/model/q4_linear.py:49-68):
    reshape [..., K] -> [T, K] fp32, gemm_{sym,asym}, reshape, + bias."""
    x = np.asarray(x, np.float32)
    k = packed.shape[1] * 2
    y = gemm(packed, scales, zeros, x.reshape(-1, k), group_size)
    y = y.reshape(*x.shape[:-1], packed.shape[0])
    if bias is not None:
        y = y + np.asarray(bias, np.float32)
    return y


def normwise_rel_err(y, y_ref) -> float:
    """max|y - y_ref| / max|y_ref| -- the tolerance measure the parity tests use."""
    y = np.asarray(y, np.float64)
    y_ref = np.asarray(y_ref, np.float64)
    den = np.max(np.abs(y_ref))
    if den == 0:
        return float(np.max(np.abs(y)))
    return float(np.max(np.abs(y - y_ref)) / den)


def algorithmic_bytes(n: int, k: int, t: int, group_size: int, asym: bool,
                      x_bytes: int = 4, y_bytes: int = 4, zero_bytes: int = 4) -> int:
    """Bytes one GEMV/GEMM must move (scripts/benchmark.py:97-102, extended with
    zeros and the output)."""
    g = k // group_size
    return (n * k // 2 + n * g * 4 + (n * g * zero_bytes if asym else 0)
            + t * k * x_bytes + t * n * y_bytes)


# ---------------------------------------------------------------------------
# Decode attention over the int8 KV cache (siliconfer/model/kv_cache.py:49-69,
# siliconfer/kernels/metal/q4_attention.py:80-175, 200-260).  Parity for this
# part is UNPINNED against reference outputs: the reference runs it through
# MLX/Metal, absent here; these functions restate its arithmetic and are
# checked in tests against an independent fp64 dequant + softmax.
# ---------------------------------------------------------------------------

def quantize_kv(x: np.ndarray):
    """kv_cache.py:49-62: scale = absmax/127 (1 where absmax == 0),
    q = clip(round(x / scale), -128, 127); returns (int8 codes, fp32 scales [..., ])."""
    x32 = x.astype(np.float32)
    amax = np.max(np.abs(x32), axis=-1, keepdims=True)
    scale = np.where(amax == 0, np.float32(1.0), amax / np.float32(127.0)).astype(np.float32)
    q = np.clip(np.round(x32 / scale), -128, 127).astype(np.int8)
    return q, scale[..., 0]


def kv_attention_decode(q, k_codes, k_scales, v_codes, v_scales, n_tiles: int = 1):
    """q4_attention.py:80-175 + 248-256 in fp32: per tile an online softmax
    over its timesteps (score = q.(k*s)/sqrt(D)), then the flash-attention
    merge of the tiles' (m, l, acc)."""
    B, H, D = q.shape
    Hkv, T = k_codes.shape[1], k_codes.shape[2]
    G = H // Hkv
    ts = -(-T // n_tiles)
    out = np.zeros((B, H, D), np.float32)
    sf = np.float32(1.0 / np.sqrt(D))
    for b in range(B):
        for h in range(H):
            kvh = h // G
            k = k_codes[b, kvh].astype(np.float32) * k_scales[b, kvh][:, None].astype(np.float32)
            v = v_codes[b, kvh].astype(np.float32) * v_scales[b, kvh][:, None].astype(np.float32)
            ms, ls, accs = [], [], []
            for t0 in range(0, T, ts):
                sc = (k[t0:t0 + ts] @ q[b, h].astype(np.float32)) * sf
                m = sc.max()
                p = np.exp(sc - m)
                ms.append(m); ls.append(p.sum()); accs.append(p @ v[t0:t0 + ts])
            M = max(ms)
            c = np.exp(np.array(ms, np.float32) - M)
            L = float(np.sum(np.array(ls) * c))
            out[b, h] = np.sum(np.stack(accs) * c[:, None], axis=0) / max(L, 1e-20)
    return out


def kv_attention_fp64(q, k_codes, k_scales, v_codes, v_scales):
    """Independent check: full fp64 dequant, softmax, weighted sum."""
    B, H, D = q.shape
    Hkv = k_codes.shape[1]
    G = H // Hkv
    k = k_codes.astype(np.float64) * k_scales[..., None]
    v = v_codes.astype(np.float64) * v_scales[..., None]
    out = np.zeros((B, H, D))
    for h in range(H):
        s = np.einsum("bd,btd->bt", q[:, h].astype(np.float64), k[:, h // G]) / np.sqrt(D)
        s = np.exp(s - s.max(axis=1, keepdims=True))
        s /= s.sum(axis=1, keepdims=True)
        out[:, h] = np.einsum("bt,btd->bd", s, v[:, h // G])
    return out


# ---------------------------------------------------------------------------
# HQQ grid search (asymmetric, calibration-free): test-data producer for the
# config-2 weights (the quantizer itself is outside the Q4Linear path).
# ---------------------------------------------------------------------------
_EPS = 1e-8
DEFAULT_K_GRID = (150.0, 100.0, 80.0, None)


def hqq_quantize_weight(W: np.ndarray, group_size: int = 128, p: float = 0.7,
                        k_grid=DEFAULT_K_GRID, bits: int = 4) -> np.ndarray:
    """Fake-quantized fp32 weights on the HQQ-chosen asymmetric grid.

    For each group, candidate clip ranges [median - k*1.4826*MAD,
    median + k*1.4826*MAD] (k = None: the full min-max range) are quantized in
    float64 and the one with the lowest mean (|w - recon| + 1e-8)^p wins
    (first best kept on ties).  Restates siliconfer/quant/hqq.py:84-164.
    """
    qmax = float(2 ** bits - 1)
    n, k = W.shape
    if k < group_size:
        q, s, z = quantize_asym(np.asarray(W, np.float32), k)   # one group per row
        return ((q.astype(np.float32) - z) * s).astype(np.float32)
    g = W.reshape(n, k // group_size, group_size).astype(np.float64)
    lo_full = g.min(axis=-1, keepdims=True)
    hi_full = g.max(axis=-1, keepdims=True)
    med = np.median(g, axis=-1, keepdims=True)
    mad = np.median(np.abs(g - med), axis=-1, keepdims=True)
    rstd = np.where(mad == 0.0, _EPS, mad) * 1.4826
    best = None
    for kk in k_grid:
        if kk is None:
            lo, hi = lo_full, hi_full
        else:
            lo = np.maximum(lo_full, med - kk * rstd)
            hi = np.minimum(hi_full, med + kk * rstd)
        scale = (hi - lo) / qmax
        scale = np.where(scale <= 0, 1.0, scale)
        zero = np.clip(np.round(-lo / scale), 0, qmax)
        q = np.clip(np.round(g / scale + zero), 0, qmax)
        loss = ((np.abs(g - scale * (q - zero)) + _EPS) ** p).mean(axis=-1, keepdims=True)
        if best is None:
            best = [loss, scale, zero]
        else:
            better = loss < best[0]
            best = [np.where(better, loss, best[0]), np.where(better, scale, best[1]),
                    np.where(better, zero, best[2])]
    _, scale, zero = best
    q = np.clip(np.round(g / scale + zero), 0, qmax)
    return (scale * (q - zero)).reshape(n, k).astype(np.float32)


# ---------------------------------------------------------------------------
# 2-bit weights: the reference quantizes and packs them (primitives.py:154-245,
# 383-425) but has no kernel for them, so the oracle is its dequant followed
# by the product, the same arithmetic Q4Linear's gemm paths use for 4 bits.
# ---------------------------------------------------------------------------
def unpack_int2(packed: np.ndarray, signed: bool) -> np.ndarray:
    """[N, K/4] uint8 -> [N, K] (unpack_int2, primitives.py:407-425, row by row)."""
    p = np.asarray(packed, np.uint8)
    out = np.empty((p.shape[0], p.shape[1] * 4), np.int32)
    for i in range(4):
        out[:, i::4] = (p >> (2 * i)) & 3
    if signed:
        out = np.where(out > 1, out - 4, out)
    return out


def dequantize_int2(packed, scales, zeros=None, group_size: int = 128) -> np.ndarray:
    """(q - z) * s in fp32 (dequantize_sym_int2 / dequantize_asym_int2,
    primitives.py:184-198, 234-245)."""
    q = unpack_int2(packed, signed=zeros is None).astype(np.float32)
    n, k = q.shape
    g = q.reshape(n, k // group_size, group_size)
    if zeros is not None:
        g = g - np.asarray(zeros, np.float32)[..., None]
    return (g * np.asarray(scales, np.float32)[..., None]).reshape(n, k).astype(np.float32)


def gemm_int2(packed, scales, zeros, X, group_size: int = 128) -> np.ndarray:
    """Y [T, N] = X [T, K] @ dequant(W)^T, fp64 accumulation of the fp32 products."""
    W = dequantize_int2(packed, scales, zeros, group_size).astype(np.float64)
    return (np.asarray(X, np.float64) @ W.T).astype(np.float32)
