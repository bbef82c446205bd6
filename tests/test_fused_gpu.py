"""Fused same-input projections give the separate layers' outputs (the
k-split of the decode kernel depends on N, so fp32 summation order may differ:
normwise 1e-6), and every part matches the CPU oracle's Q4Linear forward
(normwise 1e-3; 5e-3 at 64 tokens, the bf16 tensor-core prefill)."""
import numpy as np
import pytest
import torch

from oracle import q4_oracle as O
from siliconfer_b200 import quant as Q
from siliconfer_b200.fused import FusedQ4Linear
from siliconfer_b200.q4_linear import Q4Linear

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("asym", [False, True])
@pytest.mark.parametrize("t", [1, 4, 64])
def test_qkv_and_gate_up_fused_equal_separate(cuda, asym, t):
    rng = np.random.default_rng(11)
    def lin(n, k, bias):
        w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
        trip = Q.pack_weights_asym(w, 128) if asym else (*Q.pack_weights_sym(w, 128), None)
        b = rng.normal(0, 0.1, n).astype(np.float32) if bias else None
        m = Q4Linear(trip[0], trip[1], zeros=trip[2], bias=b, group_size=128)
        m.host_triple = (trip[0], trip[1], trip[2], b)
        return m
    qkv = [lin(896, 896, True), lin(128, 896, True), lin(128, 896, False)]
    gu = [lin(4864, 896, False), lin(4864, 896, False)]
    x = torch.randn(t, 896, device="cuda")
    for group in (qkv, gu):
        fused = FusedQ4Linear(group)
        ys = fused(x)
        xo = x.cpu().numpy()
        for m, y in zip(group, ys):
            r = m(x).double()
            assert ((y.double() - r).abs().max() / r.abs().max()).item() <= 1e-6
            p, s_, z, b = m.host_triple
            ref = O.q4linear_forward(p, s_, z, b, xo, 128)
            assert O.normwise_rel_err(y.float().cpu().numpy(), ref) <= (5e-3 if t >= 48 else 1e-3)
