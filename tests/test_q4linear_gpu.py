"""Q4Linear drop-in behaviour (restating siliconfer tests/test_integration.py:81-193)."""
import numpy as np
import pytest
import torch

import cases as C
from oracle import q4_oracle as O
from siliconfer_b200.q4_linear import Q4Linear
from siliconfer_b200.q4_loader import _pack_and_replace_linears, pack_sym_for_method
from siliconfer_b200.quant import pack_weights_asym, pack_weights_sym

pytestmark = pytest.mark.gpu


def test_q4linear_matches_fake_quant(cuda, golden):
    g, _ = golden
    w, x, gs = C.unit_case("q4linear_sym")
    layer = Q4Linear(*pack_weights_sym(w, gs), group_size=gs)
    y = layer(torch.from_numpy(x).cuda()).cpu().numpy()
    np.testing.assert_allclose(y, g["q4linear_sym/y_fakequant"], atol=1e-4, rtol=1e-4)


def test_q4linear_bias(cuda):
    rng = np.random.default_rng(2)
    w = rng.normal(0, 1, (16, 64)).astype(np.float32)
    b = rng.normal(0, 0.1, 16).astype(np.float32)
    x = torch.from_numpy(rng.normal(0, 1, (1, 64)).astype(np.float32)).cuda()
    p, s = pack_weights_sym(w, 64)
    y0 = Q4Linear(p, s, group_size=64)(x)
    y1 = Q4Linear(p, s, bias=b, group_size=64)(x)
    np.testing.assert_allclose(y1.cpu().numpy(), y0.cpu().numpy() + b, atol=1e-5)


def test_q4linear_batch_and_seq(cuda):
    rng = np.random.default_rng(3)
    p, s = pack_weights_sym(rng.normal(0, 1, (32, 64)).astype(np.float32), 64)
    layer = Q4Linear(p, s, group_size=64)
    x = rng.normal(0, 1, (2, 5, 64)).astype(np.float32)
    y = layer(torch.from_numpy(x).cuda())
    assert y.shape == (2, 5, 32)
    ref = O.q4linear_forward(p, s, None, None, x, 64)
    assert O.normwise_rel_err(y.cpu().numpy(), ref) <= 1e-3
    # numpy in -> numpy out
    yn = layer(x)
    assert isinstance(yn, np.ndarray) and yn.shape == (2, 5, 32)


def test_q4linear_asym_matches_fake_quant(cuda, golden):
    g, _ = golden
    w, x, gs = C.unit_case("q4linear_asym_skewed")
    layer = Q4Linear(*pack_weights_asym(w, gs), group_size=gs)
    assert layer.is_asym
    y = layer(torch.from_numpy(x).cuda()).cpu().numpy()
    np.testing.assert_allclose(y, g["q4linear_asym_skewed/y_fakequant"], atol=1e-3, rtol=1e-3)


def test_q4linear_asym_differs_from_sym(cuda):
    rng = np.random.default_rng(5)
    w = (rng.normal(0, 1, (16, 64)) + 2.0).astype(np.float32)
    x = torch.from_numpy(rng.normal(0, 1, (1, 64)).astype(np.float32)).cuda()
    ya = Q4Linear(*pack_weights_asym(w, 64), group_size=64)(x)
    ys = Q4Linear(*pack_weights_sym(w, 64), group_size=64)(x)
    assert not torch.allclose(ya, ys, atol=1e-3)


class _Attn(torch.nn.Module):
    def __init__(self, h):
        super().__init__()
        for n in ("q_proj", "k_proj", "v_proj", "o_proj"):
            setattr(self, n, torch.nn.Linear(h, h, bias=n != "o_proj"))


class _MLP(torch.nn.Module):
    def __init__(self, h, f):
        super().__init__()
        self.gate_proj = torch.nn.Linear(h, f, bias=False)
        self.up_proj = torch.nn.Linear(h, f, bias=False)
        self.down_proj = torch.nn.Linear(f, h, bias=False)


class _Layer(torch.nn.Module):
    def __init__(self, h, f):
        super().__init__()
        self.self_attn, self.mlp = _Attn(h), _MLP(h, f)


class _Tiny(torch.nn.Module):
    def __init__(self, h=64, f=128, n=2):
        super().__init__()
        self.layers = torch.nn.ModuleList([_Layer(h, f) for _ in range(n)])


@pytest.mark.parametrize("method", ["rtn", "hqq"])
def test_pack_and_replace(cuda, method):
    torch.manual_seed(0)
    m = _Tiny().cuda()
    for p in m.parameters():
        torch.nn.init.normal_(p, 0, 0.02)
    x = torch.randn(3, 64, device="cuda")
    ref_in = m.layers[0].self_attn.q_proj
    W = ref_in.weight.detach().cpu().numpy()
    b = ref_in.bias.detach().cpu().numpy()
    sym = pack_sym_for_method(method)
    n = _pack_and_replace_linears(m, group_size=64, pack_sym=sym)
    assert n == 14
    q = m.layers[0].self_attn.q_proj
    assert isinstance(q, Q4Linear) and (q._zeros is None) == sym
    trip = pack_weights_sym(W, 64) if sym else pack_weights_asym(W, 64)
    ref = O.q4linear_forward(trip[0], trip[1], None if sym else trip[2], b, x.cpu().numpy(), 64)
    assert O.normwise_rel_err(q(x).cpu().numpy(), ref) <= 1e-3
