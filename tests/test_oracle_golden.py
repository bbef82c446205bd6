"""Pin the CPU oracle to the reference's own outputs (golden vectors)."""
import numpy as np
import pytest

import cases as C
from oracle import cref
from oracle import q4_oracle as O


@pytest.mark.parametrize("name", list(C.UNIT_CASES))
def test_oracle_packers_match_reference(name, golden):
    g, meta = golden
    w, x, gs = C.unit_case(name)
    if C.is_asym(name):
        p, s, z = O.pack_weights_asym(w, gs)
        assert np.array_equal(z, g[f"{name}/zeros"])
    else:
        p, s = O.pack_weights_sym(w, gs)
        z = None
    assert C.sha(p) == meta["hashes"][f"{name}/packed"]
    assert C.sha(s) == meta["hashes"][f"{name}/scales"]
    if f"{name}/dequant" in g:
        # bit-exact dequant target
        assert np.array_equal(O.dequantize(p, s, z, gs), g[f"{name}/dequant"])
        assert np.array_equal(cref.oracle_dequant(p, s, z, gs), g[f"{name}/dequant"])
    y = O.gemm(p, s, z, x, gs)
    np.testing.assert_allclose(y, g[f"{name}/y"], rtol=1e-5, atol=1e-5)
    yc = cref.oracle_gemm(p, s, z, x, gs)
    assert O.normwise_rel_err(yc, g[f"{name}/y"]) < 1e-6


def test_oracle_zero_input_and_boundaries(golden):
    g, _ = golden
    w = np.random.default_rng(0).normal(0, 1, (32, 128)).astype(np.float32)
    p, s = O.pack_weights_sym(w)
    assert np.all(O.gemv_sym(p, s, np.zeros(128, np.float32)) == g["zero_input/y"])
    qs = np.arange(-8, 8, dtype=np.int8)[None, :]
    assert np.array_equal(O.pack_nibbles(qs)[0], g["boundary/packed_sym"])
    assert np.array_equal(O.unpack_nibbles(O.pack_nibbles(qs), True)[0], g["boundary/unpacked_sym"])
    qa = np.arange(16, dtype=np.uint8)[None, :]
    assert np.array_equal(O.pack_nibbles(qa)[0], g["boundary/packed_asym"])


@pytest.mark.parametrize("proj", list(C.QWEN05B))
def test_oracle_config1_layer(proj, golden):
    g, meta = golden
    n, k = C.QWEN05B[proj]
    w = C.weights(C.layer_seed(1, 0, proj), n, k)
    x = C.acts(C.layer_seed(1, 0, proj) + 7, 1, k)
    p, s = O.pack_weights_sym(w, 128)
    assert C.sha(p) == meta["hashes"][f"c1/{proj}/packed"]
    assert C.sha(s) == meta["hashes"][f"c1/{proj}/scales"]
    assert O.normwise_rel_err(O.gemm(p, s, None, x), g[f"c1/{proj}/y"]) < 1e-6


def test_oracle_matches_compiled_reference_sym():
    """The reference's own scalar/NEON sym kernel, compiled from its sources."""
    if not cref.ref_available():
        pytest.skip("oracle/_ref not built (reference sources absent)")
    rng = np.random.default_rng(11)
    w = rng.normal(0, 0.02, (257, 1024)).astype(np.float32)
    x = rng.normal(0, 1, (3, 1024)).astype(np.float32)
    for gs in (64, 128):
        p, s = O.pack_weights_sym(w, gs)
        assert O.normwise_rel_err(cref.ref_gemm(p, s, None, x, gs), O.gemm(p, s, None, x, gs)) < 1e-5


def test_compiled_reference_asym_is_flagged():
    """On x86 the reference's asym C entry runs the sym kernel
    (q4_gemv.cpp:249-255); the wrapper must refuse to use it."""
    if not cref.ref_available() or cref.ref_available(asym=True):
        pytest.skip("not applicable on this host")
    with pytest.raises(RuntimeError):
        cref.ref_gemm(np.zeros((1, 64), np.uint8), np.ones((1, 1), np.float32),
                      np.zeros((1, 1), np.float32), np.zeros((1, 128), np.float32))


@pytest.mark.parametrize("proj", ["gate", "down"])
def test_oracle_config3_batch16(proj, golden):
    g, meta = golden
    n, k = C.LLAMA7B[proj]
    p, s = O.pack_weights_sym(C.weights(C.layer_seed(3, 0, proj), n, k), 128)
    assert C.sha(p) == meta["hashes"][f"c3/{proj}/packed"]
    x = C.acts(C.layer_seed(3, 0, proj) + 7, 16, k)
    assert O.normwise_rel_err(O.gemm(p, s, None, x), g[f"c3b16/{proj}/y"]) < 1e-6


@pytest.mark.parametrize("tag,proj,t,keep", [("c4t64", "q", 64, 1), ("c4t512", "down", 512, 16)])
def test_oracle_config4_tensor_core_sizes(tag, proj, t, keep, golden):
    g, meta = golden
    n, k = C.LLAMA7B[proj]
    p, s, z = O.pack_weights_asym(C.weights(C.layer_seed(4, 0, proj), n, k), 128)
    assert C.sha(p) == meta["hashes"][f"{tag}/packed"]
    x = C.bf16_round(C.acts(C.layer_seed(4, 0, proj) + 11, t, k))[::keep]
    assert O.normwise_rel_err(O.gemm(p, s, z, x), g[f"{tag}/y"]) < 1e-6


def test_oracle_config2_step_layers(golden):
    """Config 2's 24-layer step (layers 1-23: the reference's asymmetric RTN)."""
    g, meta = golden
    for layer in (1, C.QWEN_LAYERS - 1):
        for proj, (n, k) in C.QWEN05B.items():
            p, s, z = O.pack_weights_asym(C.qwen_asym_weights(layer, proj), 128)
            assert C.sha(p) == meta["hashes"][f"c2L/{layer}/{proj}/packed"]
            x = C.acts(C.layer_seed(2, layer, proj) + 7, 1, k)
            assert O.normwise_rel_err(O.gemm(p, s, z, x), g[f"c2L/{layer}/{proj}/y"]) < 1e-6


@pytest.mark.parametrize("name", list(C.INT2_CASES))
def test_int2_packers_and_oracle_match_reference(name, golden):
    """2-bit quantize/pack (siliconfer/quant/primitives.py:154-245, 383-425):
    the product packers and the oracle's unpack/dequant are bit-exact with the
    reference; the oracle product equals the reference dequant times x."""
    from siliconfer_b200 import quant as Q
    g, _ = golden
    seed, n, k, gs, std = C.INT2_CASES[name]
    w = C.weights(seed, n, k, std)
    x = C.acts(seed + 7, 3, k)
    asym = name.startswith("int2_asym")
    if asym:
        p, s, z = Q.pack_weights_int2_asym(w, gs)
        assert np.array_equal(z, g[f"{name}/zeros"])
    else:
        (p, s), z = Q.pack_weights_int2_sym(w, gs), None
    assert np.array_equal(p, g[f"{name}/packed"])
    assert np.array_equal(s, g[f"{name}/scales"])
    assert np.array_equal(O.dequantize_int2(p, s, z, gs), g[f"{name}/dequant"])
    assert O.normwise_rel_err(O.gemm_int2(p, s, z, x, gs), g[f"{name}/y"]) < 1e-6
