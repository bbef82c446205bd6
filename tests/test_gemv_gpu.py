"""GPU parity of the decode GEMV / dequant / device packer against the oracle
and the reference's golden vectors.

Tolerances: fp32-accumulate kernels must reach normwise relative error
max|y - y_ref| / max|y_ref| <= 1e-3 and also the
reference's own elementwise tolerances (tests/test_kernel.py:80, 109, 178).
Dequant (fp32) and packing are bit-exact.
"""
import ctypes

import numpy as np
import pytest
import torch

import cases as C
from oracle import q4_oracle as O
from siliconfer_b200 import _lib, quant as Q
from siliconfer_b200.kernels import cuda as K

pytestmark = pytest.mark.gpu
TOL = 1e-3


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t if dtype is None else t.to(dtype)


def run_linear(p, s, z, X, gs, bias=None, xdtype=torch.float32, ydtype=torch.float32):
    Xd = dev(X).to(xdtype)
    return K.linear(dev(p), dev(s), None if z is None else dev(z), Xd, gs,
                    bias=None if bias is None else dev(bias), out_dtype=ydtype)


def rand_case(seed, n, k, gs, asym, t=1, std=0.02, shift=0.0):
    rng = np.random.default_rng(seed)
    w = (rng.normal(0, std, (n, k)) + shift).astype(np.float32)
    x = rng.normal(0, 1, (t, k)).astype(np.float32)
    if asym:
        p, s, z = Q.pack_weights_asym(w, gs)
    else:
        (p, s), z = Q.pack_weights_sym(w, gs), None
    return p, s, z, x


# ---- reference unit cases -------------------------------------------------
@pytest.mark.parametrize("name", list(C.UNIT_CASES))
def test_unit_cases_match_reference(cuda, golden, name):
    g, _ = golden
    w, x, gs = C.unit_case(name)
    if C.is_asym(name):
        p, s, z = Q.pack_weights_asym(w, gs)
    else:
        (p, s), z = Q.pack_weights_sym(w, gs), None
    n0 = _lib.launch_count()
    y = run_linear(p, s, z, x, gs).cpu().numpy()
    assert _lib.launch_count() > n0          # the CUDA kernel really ran
    yr = g[f"{name}/y"]
    assert O.normwise_rel_err(y, yr) <= TOL
    atol, rtol = (5e-3, 1e-3) if w.shape == (4096, 4096) else ((1e-3, 1e-3) if z is not None else (1e-4, 1e-4))
    np.testing.assert_allclose(y, yr, atol=atol, rtol=rtol)
    # the reference's own check: against the fake-quant matmul
    np.testing.assert_allclose(y, g[f"{name}/y_fakequant"], atol=max(atol, 1e-3), rtol=rtol)


def test_numpy_api_round_trip(cuda, golden):
    g, _ = golden
    w, x, gs = C.unit_case("gemv_sym_g128")
    p, s = K.pack_weights_sym(w, gs)
    y = K.gemv_sym(p, s, x[0], gs)
    assert isinstance(y, np.ndarray) and y.dtype == np.float32 and y.shape == (128,)
    np.testing.assert_allclose(y, g["gemv_sym_g128/y"][0], atol=1e-4, rtol=1e-4)
    ys = K.gemv_scalar(p, s, x[0], gs)
    np.testing.assert_allclose(ys, y, atol=1e-4, rtol=1e-4)
    w, x, gs = C.unit_case("gemv_asym_g64")
    p, s, z = K.pack_weights_asym(w, gs)
    np.testing.assert_allclose(K.gemv_asym(p, s, z, x[0], gs), g["gemv_asym_g64/y"][0],
                               atol=1e-3, rtol=1e-3)
    w, X, gs = C.unit_case("gemm_T32")
    p, s = K.pack_weights_sym(w, gs)
    Y = K.gemm_sym(p, s, X, gs)
    assert Y.shape == (32, 64)
    np.testing.assert_allclose(Y, g["gemm_T32/y"], atol=1e-4, rtol=1e-4)
    # GEMM equals a loop of GEMVs (test_kernel.py:136-151)
    loop = np.stack([K.gemv_sym(p, s, X[t], gs) for t in range(32)])
    np.testing.assert_allclose(Y, loop, atol=1e-5, rtol=1e-5)


def test_zero_input_gives_zero(cuda):
    w = np.random.default_rng(0).normal(0, 1, (32, 128)).astype(np.float32)
    p, s = K.pack_weights_sym(w)
    assert np.all(K.gemv_sym(p, s, np.zeros(128, np.float32)) == 0.0)


# ---- BASELINE configs at full size ----------------------------------------
@pytest.mark.parametrize("proj", list(C.QWEN05B))
def test_config1_qwen_layer_sym(cuda, golden, proj):
    g, _ = golden
    n, k = C.QWEN05B[proj]
    p, s = Q.pack_weights_sym(C.weights(C.layer_seed(1, 0, proj), n, k), 128)
    x = C.acts(C.layer_seed(1, 0, proj) + 7, 1, k)
    y = run_linear(p, s, None, x, 128).cpu().numpy()
    assert O.normwise_rel_err(y, g[f"c1/{proj}/y"]) <= TOL


@pytest.mark.parametrize("proj", list(C.QWEN05B))
def test_config2_qwen_layer_hqq_asym(cuda, golden, proj):
    g, _ = golden
    p, s, z = Q.pack_weights_asym(O.hqq_quantize_weight(C.qwen_asym_weights(0, proj), 128), 128)
    x = C.acts(C.layer_seed(2, 0, proj) + 7, 1, p.shape[1] * 2)
    y = run_linear(p, s, z, x, 128).cpu().numpy()
    assert O.normwise_rel_err(y, g[f"c2/{proj}/y"]) <= TOL


@pytest.mark.parametrize("proj", list(C.LLAMA7B))
@pytest.mark.parametrize("t", [1, 4])
def test_config3_7b_layer(cuda, golden, proj, t):
    g, _ = golden
    n, k = C.LLAMA7B[proj]
    Wd = dev(C.weights(C.layer_seed(3, 0, proj), n, k))
    p, s = Q.pack_weights_device(Wd, 128)
    X = C.acts(C.layer_seed(3, 0, proj) + 7, 4, k)[:t]
    y = K.linear(p, s, None, dev(X), 128).cpu().numpy()
    assert O.normwise_rel_err(y, g[f"c3/{proj}/y"][:t]) <= TOL
    # fp16 activations (config 3 states fp16 inputs): exact upcast on the oracle side
    Xh = X.astype(np.float16)
    yh = K.linear(p, s, None, dev(Xh), 128).cpu().numpy()
    yr = O.gemm(p.cpu().numpy(), s.cpu().numpy(), None, Xh.astype(np.float32))
    assert O.normwise_rel_err(yh, yr) <= TOL


# ---- device packer ---------------------------------------------------------
@pytest.mark.parametrize("sym", [True, False])
@pytest.mark.parametrize("n,k,gs", [(37, 256, 64), (896, 4864, 128), (128, 96, 32), (5, 30, 10)])
def test_device_pack_bit_exact(cuda, sym, n, k, gs):
    rng = np.random.default_rng(n * k + gs)
    w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
    w[0, :gs] = 0.0                       # all-zero group -> scale 0 path
    w[-1, 1] = 0.5                        # outlier
    out_d = Q.pack_weights_device(dev(w), gs, sym=sym)
    out_h = Q.pack_weights_sym(w, gs) if sym else Q.pack_weights_asym(w, gs)
    for a, b in zip(out_d, out_h):
        assert np.array_equal(a.cpu().numpy(), b)


# ---- dequant ----------------------------------------------------------------
@pytest.mark.parametrize("asym", [False, True])
@pytest.mark.parametrize("gs", [32, 64, 128])
def test_dequant_bit_exact(cuda, golden, asym, gs):
    p, s, z, _ = rand_case(gs + asym, 67, 512, gs, asym, shift=0.01 if asym else 0.0)
    ref = O.dequantize(p, s, z, gs)
    out = K.dequant(p, s, z, gs).cpu().numpy()
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))
    for dt in (torch.bfloat16, torch.float16):
        outh = K.dequant(p, s, z, gs, out_dtype=dt)
        assert torch.equal(outh, torch.from_numpy(ref).cuda().to(dt))


@pytest.mark.parametrize("name", [n for n in C.UNIT_CASES if n + "/dequant" in np.load(
    __import__("pathlib").Path(__file__).parent / "golden" / "golden.npz").files])
def test_dequant_matches_reference_golden(cuda, golden, name):
    g, _ = golden
    out = K.dequant(g[f"{name}/packed"], g[f"{name}/scales"],
                    g[f"{name}/zeros"] if C.is_asym(name) else None,
                    C.UNIT_CASES[name][3]).cpu().numpy()
    assert np.array_equal(out, g[f"{name}/dequant"])


# ---- shape / dtype coverage ---------------------------------------------------
SHAPES = [
    (1, 128, 128), (7, 256, 64), (33, 896, 128), (128, 896, 128), (300, 1024, 32),
    (4864, 896, 128), (896, 4864, 128), (1000, 3584, 128), (513, 11008, 128),
    (64, 8192, 128), (40, 28672, 128), (3, 32, 32), (96, 1056, 32),
]


@pytest.mark.parametrize("asym", [False, True])
@pytest.mark.parametrize("n,k,gs", SHAPES)
@pytest.mark.parametrize("t", [1, 2, 3, 4, 8, 9, 16])
def test_gemv_shapes(cuda, asym, n, k, gs, t):
    p, s, z, x = rand_case(n + k + t, n, k, gs, asym, t=t, shift=0.005 if asym else 0.0)
    y = run_linear(p, s, z, x, gs).cpu().numpy()
    assert O.normwise_rel_err(y, O.gemm(p, s, z, x, gs)) <= TOL


@pytest.mark.parametrize("n,k,gs", [(9, 30, 10), (17, 64, 16), (5, 12, 2), (40, 200, 40)])
@pytest.mark.parametrize("asym", [False, True])
def test_generic_group_sizes(cuda, n, k, gs, asym):
    """Group sizes the fast kernel does not take (not a multiple of 32)."""
    p, s, z, x = rand_case(n * gs, n, k, gs, asym, t=3)
    y = run_linear(p, s, z, x, gs).cpu().numpy()
    assert O.normwise_rel_err(y, O.gemm(p, s, z, x, gs)) <= TOL


@pytest.mark.parametrize("xdt", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("ydt", [torch.float32, torch.float16, torch.bfloat16])
def test_dtypes_and_bias(cuda, xdt, ydt):
    p, s, z, x = rand_case(5, 257, 2048, 128, False, t=2)
    b = np.random.default_rng(1).normal(0, 0.1, 257).astype(np.float32)
    xq = torch.from_numpy(x).to(xdt).float().numpy()
    y = run_linear(p, s, z, x, 128, bias=b, xdtype=xdt, ydtype=ydt).float().cpu().numpy()
    yr = O.gemm(p, s, z, xq, 128) + b
    tol = TOL if ydt == torch.float32 else (4e-3 if ydt == torch.float16 else 8e-3)
    assert O.normwise_rel_err(y, yr) <= tol


@pytest.mark.parametrize("t", [9, 16, 33])
@pytest.mark.parametrize("asym", [False, True])
def test_many_tokens(cuda, t, asym):
    p, s, z, x = rand_case(t, 384, 1024, 128, asym, t=t)
    y = run_linear(p, s, z, x, 128).cpu().numpy()
    assert O.normwise_rel_err(y, O.gemm(p, s, z, x, 128)) <= 5e-3


# ---- full-size properties -------------------------------------------------------
def test_linearity_at_7b_down_shape(cuda):
    """y(a*x1 + x2) == a*y(x1) + y(x2) for the 11008-wide down projection."""
    torch.manual_seed(0)
    W = torch.randn(4096, 11008, device="cuda") * 0.02
    p, s = Q.pack_weights_device(W, 128)
    x1, x2 = torch.randn(1, 11008, device="cuda"), torch.randn(1, 11008, device="cuda")
    y = lambda x: K.linear(p, s, None, x, 128).double()
    lhs = y(0.5 * x1 + x2)
    rhs = 0.5 * y(x1) + y(x2)
    assert ((lhs - rhs).abs().max() / rhs.abs().max()).item() < 1e-5
    # against the dequantized fp64 product
    Wd = K.dequant(p, s, None, 128).double()
    ref = x1.double() @ Wd.T
    assert ((y(x1) - ref).abs().max() / ref.abs().max()).item() < TOL


def test_device_error_word_clear(cuda):
    K.linear(*[dev(a) for a in rand_case(1, 64, 256, 128, False)[:2]], None,
             dev(np.ones((1, 256), np.float32)), 128)
    torch.cuda.synchronize()
    assert _lib.load().sf_q4_check_device_error() == 0


def test_c_abi_reference_named_entries(cuda):
    """sf_q4_gemv_sym / sf_q4_gemm_asym called directly through ctypes."""
    lib = _lib.load()
    p, s, z, x = rand_case(3, 96, 512, 64, True, t=5)
    P, S, Z, X = dev(p), dev(s), dev(z), dev(x)
    Y = torch.empty((5, 96), device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.sf_q4_gemm_asym(P.data_ptr(), S.data_ptr(), Z.data_ptr(), X.data_ptr(),
                                   Y.data_ptr(), 96, 512, 5, 64, st))
    assert O.normwise_rel_err(Y.cpu().numpy(), O.gemm(p, s, z, x, 64)) <= TOL
    p, s, _, x = rand_case(4, 96, 512, 64, False, t=1)
    P, S, X = dev(p), dev(s), dev(x[0])
    y = torch.empty(96, device="cuda")
    _lib.check(lib.sf_q4_gemv_sym(P.data_ptr(), S.data_ptr(), X.data_ptr(), y.data_ptr(),
                                  96, 512, 64, st))
    assert O.normwise_rel_err(y.cpu().numpy(), O.gemv_sym(p, s, x[0], 64)) <= TOL


def test_capture_without_warmup_fails_loudly(cuda):
    """A shape whose scratch would have to grow inside a stream capture is
    refused with SF_ERR_CAPTURE (never silently run on another kernel)."""
    p, s, _, x = rand_case(77, 4352, 12288, 128, False, t=3)
    P, S, X = dev(p), dev(s), dev(x)
    st = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with pytest.raises(RuntimeError, match="capture"):
        with torch.cuda.graph(g, stream=st):
            K.linear(P, S, None, X, 128)
    # after a warm-up on the capturing stream the same capture succeeds
    with torch.cuda.stream(st):
        ref = K.linear(P, S, None, X, 128)
    st.synchronize()
    g2 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g2, stream=st):
        out = K.linear(P, S, None, X, 128)
    g2.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


@pytest.mark.parametrize("proj", ["gate", "down"])
def test_config3_7b_batch16_one_pass(cuda, golden, proj):
    """Config 3's largest batch: 16 tokens in ONE launch of the decode kernel
    (each weight read once), against the reference's gemm_sym output."""
    g, _ = golden
    n, k = C.LLAMA7B[proj]
    p, s = Q.pack_weights_device(dev(C.weights(C.layer_seed(3, 0, proj), n, k)), 128)
    X = C.acts(C.layer_seed(3, 0, proj) + 7, 16, k)
    n0 = _lib.launch_count()
    y = K.linear(p, s, None, dev(X), 128).cpu().numpy()
    assert _lib.launch_count() - n0 == 2          # activation pre-pass + one GEMV launch
    assert O.normwise_rel_err(y, g[f"c3b16/{proj}/y"]) <= TOL
