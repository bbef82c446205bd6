"""Decode attention over the int8 KV cache.

CPU: the oracle's restatement of the reference's tiled online softmax
(q4_attention.py:80-175, merge 248-256) agrees with an independent fp64
dequant + softmax, for any tiling.  GPU: sf_kv_attention_decode against that
oracle at normwise 1e-4 (fp32 math; only summation order differs), at
Qwen2.5-0.5B (14 heads, 2 kv heads, head_dim 64), 7B (32/32/128) and 70B
(64/8/128) head shapes, T from 1 to 8192, with empty tiles and all-zero
vectors.
"""
import numpy as np
import pytest
import torch

from oracle import q4_oracle as O


def _case(seed, B, H, Hkv, T, D):
    rng = np.random.default_rng(seed)
    q = rng.normal(0, 1, (B, H, D)).astype(np.float32)
    k = rng.normal(0, 1, (B, Hkv, T, D)).astype(np.float32)
    v = rng.normal(0, 1, (B, Hkv, T, D)).astype(np.float32)
    if T > 3:
        k[0, 0, 2] = 0.0          # an all-zero vector: scale 1, codes 0
    kc, ks = O.quantize_kv(k)
    vc, vs = O.quantize_kv(v)
    return q, kc, ks, vc, vs


@pytest.mark.parametrize("n_tiles", [1, 3, 16])
def test_oracle_tiling_matches_fp64(n_tiles):
    q, kc, ks, vc, vs = _case(0, 2, 4, 2, 100, 64)
    ref = O.kv_attention_fp64(q, kc, ks, vc, vs)
    got = O.kv_attention_decode(q, kc, ks, vc, vs, n_tiles=n_tiles)
    assert np.max(np.abs(got - ref)) / np.max(np.abs(ref)) < 1e-5


def test_quantize_kv_zero_vector_and_range():
    x = np.zeros((1, 1, 2, 8), np.float32)
    x[0, 0, 1] = np.linspace(-3, 3, 8)
    c, s = O.quantize_kv(x)
    assert s[0, 0, 0] == 1.0 and np.all(c[0, 0, 0] == 0)
    assert c[0, 0, 1].min() == -127 and c[0, 0, 1].max() == 127


SHAPES = [(1, 14, 2, 1, 64), (1, 14, 2, 37, 64), (2, 14, 2, 1000, 64), (1, 32, 32, 513, 128),
          (4, 64, 8, 2048, 128), (1, 16, 2, 8192, 256), (3, 8, 4, 77, 128), (1, 7, 1, 300, 64)]


@pytest.mark.gpu
@pytest.mark.parametrize("B,H,Hkv,T,D", SHAPES)
def test_gpu_matches_oracle(cuda, B, H, Hkv, T, D):
    from siliconfer_b200 import _lib
    from siliconfer_b200.kv_attention import fused_quantized_attention_decode
    q, kc, ks, vc, vs = _case(B * H + T, B, H, Hkv, T, D)
    dev = lambda a: torch.from_numpy(a).cuda()
    n0 = _lib.launch_count()
    out = fused_quantized_attention_decode(dev(q), dev(kc), dev(ks), dev(vc), dev(vs)).cpu().numpy()
    assert _lib.launch_count() >= n0 + 2
    ref = O.kv_attention_decode(q, kc, ks, vc, vs, n_tiles=1)
    assert np.max(np.abs(out - ref)) / np.max(np.abs(ref)) < 1e-4


@pytest.mark.gpu
@pytest.mark.parametrize("n_tiles", [1, 5, 64])
def test_gpu_tilings_and_dtypes(cuda, n_tiles):
    from siliconfer_b200.kv_attention import fused_quantized_attention_decode, quantize_kv
    torch.manual_seed(0)
    B, H, Hkv, T, D = 2, 32, 8, 300, 128
    q = torch.randn(B, H, D, device="cuda")
    kc, ks = quantize_kv(torch.randn(B, Hkv, T, D, device="cuda"))
    vc, vs = quantize_kv(torch.randn(B, Hkv, T, D, device="cuda"))
    ref = O.kv_attention_fp64(q.cpu().numpy(), kc.cpu().numpy(), ks.cpu().numpy(), vc.cpu().numpy(),
                              vs.cpu().numpy())
    for qdt, odt, tol in ((torch.float32, torch.float32, 1e-4), (torch.bfloat16, torch.bfloat16, 2e-2),
                          (torch.float16, torch.float32, 5e-3)):
        qq = q.to(qdt)
        out = fused_quantized_attention_decode(qq, kc, ks, vc, vs, n_tiles=n_tiles, out_dtype=odt)
        r = O.kv_attention_fp64(qq.float().cpu().numpy(), kc.cpu().numpy(), ks.cpu().numpy(),
                                vc.cpu().numpy(), vs.cpu().numpy()) if qdt != torch.float32 else ref
        assert np.max(np.abs(out.float().cpu().numpy() - r)) / np.max(np.abs(r)) < tol


# ---- pinned to the reference: its own quantize_kv on its own test inputs -----
import cases as C   # noqa: E402


def _kv_golden(g, name):
    return tuple(g[f"{name}/{f}"] for f in ("q", "k_codes", "k_scales", "v_codes", "v_scales"))


@pytest.mark.parametrize("name", list(C.KV_CASES))
def test_quantize_kv_matches_reference(golden, name):
    """The int8 codes and scales the reference's quantize_kv (kv_cache.py:49-63)
    computed on the inputs of its attention tests: bit-exact."""
    g, _ = golden
    seed, B, H, Hkv, D, T = C.KV_CASES[name]
    rng = np.random.default_rng(seed)
    rng.normal(0, 1, (B, H, D))
    k = rng.normal(0, 1, (B, Hkv, T, D)).astype(np.float32)
    v = rng.normal(0, 1, (B, Hkv, T, D)).astype(np.float32)
    _, kc, ks, vc, vs = _kv_golden(g, name)
    for x, c_ref, s_ref in ((k, kc, ks), (v, vc, vs)):
        c, s = O.quantize_kv(x)
        assert np.array_equal(c, c_ref) and np.array_equal(s.view(np.uint32), s_ref.view(np.uint32))


@pytest.mark.parametrize("name", list(C.KV_CASES))
def test_oracle_attention_on_reference_cases(golden, name):
    """The reference test's criterion (tests/test_metal_attention.py: max
    |out - ref| < 1e-4 against dequant + softmax attention), with the tile
    count its heuristic picks (q4_attention.py:183-197)."""
    g, _ = golden
    q, kc, ks, vc, vs = _kv_golden(g, name)
    T = kc.shape[2]
    n_tiles = 1 if T <= 16 else min(256, -(-T // 16))
    got = O.kv_attention_decode(q, kc, ks, vc, vs, n_tiles=n_tiles)
    assert np.max(np.abs(got - O.kv_attention_fp64(q, kc, ks, vc, vs))) < 1e-4


@pytest.mark.gpu
@pytest.mark.parametrize("name", [n for n, c in C.KV_CASES.items() if c[4] in (64, 128, 256)])
def test_gpu_on_reference_cases(cuda, golden, name):
    """The CUDA kernel on the reference-quantized caches, at the reference
    test's own tolerance (max abs difference < 1e-4)."""
    from siliconfer_b200.kv_attention import fused_quantized_attention_decode
    g, _ = golden
    q, kc, ks, vc, vs = _kv_golden(g, name)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    out = fused_quantized_attention_decode(dev(q), dev(kc), dev(ks), dev(vc), dev(vs)).cpu().numpy()
    assert np.max(np.abs(out - O.kv_attention_fp64(q, kc, ks, vc, vs))) < 1e-4
