"""Seeded input cases shared by the golden generator and the parity tests.

Each case regenerates its fp32 weights and activations from a seed, so the
golden file only has to hold the reference's OUTPUTS (or their SHA-256 for the
large packed tensors).  Shapes follow the reference's tests
(siliconfer tests/test_kernel.py, tests/test_integration.py) and the
BASELINE configs (Qwen2.5-0.5B layer, 7B layer, prefill, 70B shards).
"""
from __future__ import annotations

import hashlib

import numpy as np

# Qwen2.5-0.5B projections as (N=out, K=in)  -- config 1/2
QWEN05B = {"q": (896, 896), "k": (128, 896), "v": (128, 896), "o": (896, 896),
           "gate": (4864, 896), "up": (4864, 896), "down": (896, 4864)}
# 7B projections -- config 3/4
LLAMA7B = {"q": (4096, 4096), "k": (4096, 4096), "v": (4096, 4096), "o": (4096, 4096),
           "gate": (11008, 4096), "up": (11008, 4096), "down": (4096, 11008)}
# 70B projections -- config 5
LLAMA70B = {"q": (8192, 8192), "k": (1024, 8192), "v": (1024, 8192), "o": (8192, 8192),
            "gate": (28672, 8192), "up": (28672, 8192), "down": (8192, 28672)}
PROJ_ORDER = ("q", "k", "v", "o", "gate", "up", "down")


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def weights(seed: int, n: int, k: int, std: float = 0.02) -> np.ndarray:
    return np.random.default_rng(seed).normal(0, std, (n, k)).astype(np.float32)


def acts(seed: int, t: int, k: int) -> np.ndarray:
    return np.random.default_rng(seed).normal(0, 1, (t, k)).astype(np.float32)


def layer_seed(config: int, layer: int, proj: str) -> int:
    return config * 100_000 + layer * 100 + PROJ_ORDER.index(proj)


QWEN_LAYERS = 24   # config 2: the full Qwen2.5-0.5B decode step

# int8 KV attention cases of the reference's own tests
# (tests/test_metal_attention.py): name -> (seed, B, H, Hkv, D, T)
KV_CASES = {"kv_mha_T128": (0, 1, 4, 4, 8, 128), "kv_gqa_T512": (3, 1, 14, 2, 64, 512),
            "kv_batch": (9, 3, 4, 2, 16, 32), "kv_tiles_T100": (11, 1, 14, 2, 64, 100),
            "kv_gqa_T2048": (17, 1, 14, 2, 64, 2048)}

# 2-bit cases: name -> (seed, out_f, in_f, group_size, std)
INT2_CASES = {"int2_sym": (71, 96, 512, 128, 0.02), "int2_asym": (72, 96, 512, 128, 0.02),
              "int2_sym_unit": (73, 64, 256, 128, 1.0), "int2_asym_g256": (74, 40, 1024, 256, 0.02)}


def bf16_round(a: np.ndarray) -> np.ndarray:
    """fp32 values rounded to the nearest bfloat16 (ties to even), as fp32."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    return r.view(np.float32)


# One injected outlier of 60 sigma in a down_proj group (config 2).
OUTLIER = {"row": 17, "col": 1234, "sigma": 60.0}


def qwen_asym_weights(layer: int, proj: str) -> np.ndarray:
    n, k = QWEN05B[proj]
    w = weights(layer_seed(2, layer, proj), n, k)
    if proj == "down" and layer == 0:
        w[OUTLIER["row"], OUTLIER["col"]] = np.float32(OUTLIER["sigma"] * 0.02)
    return w


# ---- small cases restating the reference's unit tests ----------------------
# name -> (seed, out_f, in_f, group_size, T, std, shift)
UNIT_CASES = {
    "pack_round_trip": (0, 32, 128, 128, 1, 1.0, 0.0),      # test_kernel.py:38-61
    "gemv_sym_g64": (42, 128, 256, 64, 1, 1.0, 0.0),       # test_kernel.py:68-80
    "gemv_sym_g128": (42, 128, 256, 128, 1, 1.0, 0.0),
    "gemv_large": (1, 4096, 4096, 128, 1, 1.0, 0.0),       # test_kernel.py:97-109
    "single_row": (5, 1, 128, 128, 1, 1.0, 0.0),           # test_kernel.py:121-129
    "gemm_T1": (99, 64, 128, 128, 1, 1.0, 0.0),            # test_kernel.py:136-151
    "gemm_T4": (99, 64, 128, 128, 4, 1.0, 0.0),
    "gemm_T32": (99, 64, 128, 128, 32, 1.0, 0.0),
    "gemv_asym_g64": (42, 128, 256, 64, 1, 1.0, 0.0),      # test_kernel.py:167-178
    "gemv_asym_g128": (42, 128, 256, 128, 1, 1.0, 0.0),
    "gemm_asym_matmul": (3, 32, 128, 128, 8, 1.0, 0.0),    # test_kernel.py:198-210
    "q4linear_sym": (1, 32, 64, 64, 1, 1.0, 0.0),          # test_integration.py:81-97
    "q4linear_asym_skewed": (4, 32, 64, 64, 1, 1.0, 1.0),  # test_integration.py:132-149
}


def unit_case(name: str):
    """Weights and activations in the draw order of the reference test."""
    seed, n, k, gs, t, std, shift = UNIT_CASES[name]
    rng = np.random.default_rng(seed)
    w = (rng.normal(0, std, (n, k)) + shift).astype(np.float32)
    if t == 1 and not name.startswith("gemm"):
        x = rng.normal(0, 1, k).astype(np.float32)[None, :]
    else:
        x = rng.normal(0, 1, (t, k)).astype(np.float32)
    return w, x, gs


def is_asym(name: str) -> bool:
    return "asym" in name
