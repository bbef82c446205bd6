"""Fused same-input projections give the separate layers' outputs (the
k-split of the decode kernel depends on N, so fp32 summation order may differ:
normwise 1e-6)."""
import numpy as np
import pytest
import torch

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
        return Q4Linear(trip[0], trip[1], zeros=trip[2], bias=b, group_size=128)
    qkv = [lin(896, 896, True), lin(128, 896, True), lin(128, 896, False)]
    gu = [lin(4864, 896, False), lin(4864, 896, False)]
    x = torch.randn(t, 896, device="cuda")
    for group in (qkv, gu):
        fused = FusedQ4Linear(group)
        ys = fused(x)
        for m, y in zip(group, ys):
            r = m(x).double()
            assert ((y.double() - r).abs().max() / r.abs().max()).item() <= 1e-6
