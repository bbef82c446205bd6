"""GPU parity of the tcgen05 prefill GEMM (T >= 48 tokens).

The prefill path computes with bf16 operands and fp32 accumulation:
  * every weight is RNE-bf16 of the reference's fp32 dequant (q - z) * s
    (siliconfer/quant/primitives.py:54-75, 117-140);
  * X is bf16 (fp32/fp16 inputs are rounded to bf16 first).
Two checks per case:
  1. against the reference semantics (the fp32 oracle, O.gemm, which follows
     siliconfer/kernels/neon/__init__.py:88-124 and q4_gemm.cpp:12-51):
     normwise relative error <= 5e-3 (the bf16 tensor-core tolerance);
  2. against the same product formed in fp64 from the bf16-rounded operands
     (X_bf16 @ RNE_bf16(dequant_fp32(W))^T): normwise <= 2e-5.  Only fp32
     accumulation order separates the two, so this pins the in-kernel
     dequant to the bit-exact bf16 weights and shows that the tensor-core
     path (not the fp32 GEMV) produced the result.
"""
import numpy as np
import pytest
import torch

from oracle import q4_oracle as O
from siliconfer_b200 import _lib, quant as Q
from siliconfer_b200.kernels import cuda as K

pytestmark = pytest.mark.gpu
TOL_BF16 = 5e-3
TOL_EXACT_OPERANDS = 2e-5


def _rel(a, b):
    a, b = a.double(), b.double()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()


def _bf16_ref(p, s, z, X, gs, bias=None):
    """fp64 product of the bf16 operands the kernel multiplies."""
    Wd = K.dequant(p, s, z, gs, out_dtype=torch.bfloat16).double()
    Y = X.to(torch.bfloat16).double() @ Wd.T
    return Y if bias is None else Y + bias.double()


def _case(seed, n, k, gs, asym, t, xdtype=torch.float32, shift=0.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    W = torch.randn(n, k, device="cuda", generator=g) * 0.02 + shift
    p, s, *z = Q.pack_weights_device(W, gs, sym=not asym)
    X = torch.randn(t, k, device="cuda", generator=g).to(xdtype)
    return p, s, (z[0] if z else None), X


SMALL = [  # (T, N, K, gs, asym)
    (48, 64, 128, 128, False), (64, 96, 512, 64, True), (130, 200, 1024, 128, False),
    (129, 256, 256, 32, True), (300, 384, 2048, 256, False), (256, 4864, 896, 128, True),
    (513, 896, 4864, 128, False), (200, 128, 896, 128, True), (1000, 1000, 640, 64, False),
]


@pytest.mark.parametrize("t,n,k,gs,asym", SMALL)
def test_prefill_matches_oracle(cuda, t, n, k, gs, asym):
    p, s, z, X = _case(t * n + k, n, k, gs, asym, t, shift=0.004 if asym else 0.0)
    n0 = _lib.launch_count()
    Y = K.linear(p, s, z, X, gs)
    assert _lib.launch_count() > n0
    yo = O.gemm(p.cpu().numpy(), s.cpu().numpy(), None if z is None else z.cpu().numpy(),
                X.cpu().numpy(), gs)
    assert O.normwise_rel_err(Y.cpu().numpy(), yo) <= TOL_BF16
    assert _rel(Y, _bf16_ref(p, s, z, X, gs)) <= TOL_EXACT_OPERANDS


@pytest.mark.parametrize("xdt", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("ydt", [torch.float32, torch.float16, torch.bfloat16])
def test_prefill_dtypes_and_bias(cuda, xdt, ydt):
    p, s, z, X = _case(11, 333, 1024, 128, True, 177, xdtype=xdt, shift=0.003)
    b = torch.randn(333, device="cuda") * 0.1
    Y = K.linear(p, s, z, X, 128, bias=b, out_dtype=ydt)
    assert Y.dtype == ydt and Y.shape == (177, 333)
    ref = _bf16_ref(p, s, z, X, 128, bias=b)
    tol = TOL_EXACT_OPERANDS if ydt == torch.float32 else (2e-3 if ydt == torch.float16 else 8e-3)
    assert _rel(Y, ref) <= tol


def test_prefill_reference_named_entry_fp32(cuda):
    """sf_q4_gemm_asym (the q4_gemm_asym_neon replacement) with T = 64 fp32 tokens."""
    lib = _lib.load()
    p, s, z, X = _case(5, 256, 1024, 64, True, 64, shift=0.002)
    Y = torch.empty((64, 256), device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.sf_q4_gemm_asym(p.data_ptr(), s.data_ptr(), z.data_ptr(), X.data_ptr(), Y.data_ptr(),
                                   256, 1024, 64, 64, st))
    yo = O.gemm(p.cpu().numpy(), s.cpu().numpy(), z.cpu().numpy(), X.cpu().numpy(), 64)
    assert O.normwise_rel_err(Y.cpu().numpy(), yo) <= TOL_BF16


def test_prefill_zero_input_and_fractional_zero(cuda):
    p, s, z, X = _case(3, 128, 512, 128, True, 64)
    assert torch.count_nonzero(K.linear(p, s, z, torch.zeros_like(X), 128)).item() == 0
    # non-integer zero points (quantizers that store float zeros): two-step (q - z)
    zf = z + 0.25
    Y = K.linear(p, s, zf, X, 128)
    assert _rel(Y, _bf16_ref(p, s, zf, X, 128)) <= TOL_EXACT_OPERANDS


# ---- BASELINE config 4 at full size: gemm_asym prefill at 7B shapes ----------
@pytest.mark.parametrize("m", [512, 2048])
@pytest.mark.parametrize("k,n", [(4096, 4096), (4096, 11008), (11008, 4096)])
def test_config4_prefill_7b(cuda, m, k, n):
    p, s, z, X = _case(m + n + k, n, k, 128, True, m, xdtype=torch.bfloat16)
    Y = K.linear(p, s, z, X, 128)
    ref = _bf16_ref(p, s, z, X, 128)
    assert _rel(Y, ref) <= TOL_EXACT_OPERANDS
    # against the fp32-weight product (the reference's arithmetic), bf16 tolerance
    Wd = K.dequant(p, s, z, 128).double()
    assert _rel(Y, X.double() @ Wd.T) <= TOL_BF16
    torch.cuda.synchronize()
    assert _lib.load().sf_q4_check_device_error() == 0


def test_prefill_repeatable_and_stream_ordered(cuda):
    """Same inputs twice on a side stream give identical bits."""
    p, s, z, X = _case(9, 1024, 2048, 128, False, 384, xdtype=torch.bfloat16)
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        a = K.linear(p, s, z, X, 128)
        b = K.linear(p, s, z, X, 128)
    st.synchronize()
    assert torch.equal(a, b)


@pytest.mark.parametrize("tag,proj,t,keep", [("c4t64", "q", 64, 1), ("c4t512", "down", 512, 16)])
def test_prefill_matches_reference_gemm_asym_golden(cuda, golden, tag, proj, t, keep):
    """Config 4 on the tcgen05 path against the reference's own gemm_asym output
    (siliconfer/kernels/neon/__init__.py:200-227), bf16 activations."""
    import cases as C
    g, _ = golden
    n, k = C.LLAMA7B[proj]
    W = torch.from_numpy(C.weights(C.layer_seed(4, 0, proj), n, k)).cuda()
    p, s, z = Q.pack_weights_device(W, 128, sym=False)
    X = torch.from_numpy(C.bf16_round(C.acts(C.layer_seed(4, 0, proj) + 11, t, k))).cuda().to(torch.bfloat16)
    y = K.linear(p, s, z, X, 128).float().cpu().numpy()[::keep]
    assert O.normwise_rel_err(y, g[f"{tag}/y"]) <= TOL_BF16
