"""Persistent packed-weight format: bit-exact round trips on the host."""
import numpy as np
import pytest
import torch

from siliconfer_b200 import quant as Q
from siliconfer_b200.packed_io import load_packed, load_q4_model, save_packed, save_q4_model
from siliconfer_b200.q4_loader import PROJECTIONS, _pack_and_replace_linears


def _triples():
    rng = np.random.default_rng(3)
    a = rng.normal(0, 0.02, (96, 512)).astype(np.float32)
    b = rng.normal(0, 0.02, (64, 256)).astype(np.float32)
    b[5, 7] = 1.2                                  # an outlier group
    ps, ss = Q.pack_weights_sym(a, 128)
    pa, sa, za = Q.pack_weights_asym(b, 128)
    return {"l0.q_proj": (ps, ss, None, rng.normal(0, 0.1, 96).astype(np.float32)),
            "l0.down_proj": (pa, sa, za)}


def test_round_trip_is_bit_exact(tmp_path):
    t = _triples()
    f = tmp_path / "m.safetensors"
    save_packed(f, t, group_size=128, method="hqq")
    got, meta = load_packed(f)
    assert meta["group_size"] == 128 and meta["method"] == "hqq"
    assert meta["layouts"] == {"l0.q_proj": "sym", "l0.down_proj": "asym"}
    for name, want in t.items():
        g = got[name]
        assert np.array_equal(g[0], want[0]) and g[0].dtype == np.uint8
        assert np.array_equal(g[1].view(np.uint32), want[1].view(np.uint32))
        if want[2] is None:
            assert g[2] is None
        else:
            assert np.array_equal(g[2].view(np.uint32), want[2].view(np.uint32))
        if len(want) > 3:
            assert np.array_equal(g[3], want[3])
        else:
            assert g[3] is None


def test_rejects_bad_shapes_and_foreign_files(tmp_path):
    p, s = Q.pack_weights_sym(np.zeros((8, 256), np.float32), 128)
    with pytest.raises(ValueError, match="group_size"):
        save_packed(tmp_path / "x.safetensors", {"a": (p, s, None)}, group_size=64)
    from safetensors.numpy import save_file
    save_file({"w": np.zeros(4, np.float32)}, str(tmp_path / "foreign.safetensors"))
    with pytest.raises(ValueError, match="not a"):
        load_packed(tmp_path / "foreign.safetensors")


class _Attn(torch.nn.Module):
    def __init__(self, h, kv):
        super().__init__()
        self.q_proj = torch.nn.Linear(h, h, bias=True)
        self.k_proj = torch.nn.Linear(h, kv, bias=True)
        self.v_proj = torch.nn.Linear(h, kv, bias=True)
        self.o_proj = torch.nn.Linear(h, h, bias=False)


class _MLP(torch.nn.Module):
    def __init__(self, h, f):
        super().__init__()
        self.gate_proj = torch.nn.Linear(h, f, bias=False)
        self.up_proj = torch.nn.Linear(h, f, bias=False)
        self.down_proj = torch.nn.Linear(f, h, bias=False)


class _Layer(torch.nn.Module):
    def __init__(self, h, kv, f):
        super().__init__()
        self.self_attn = _Attn(h, kv)
        self.mlp = _MLP(h, f)


class _Model(torch.nn.Module):
    def __init__(self, n=2, h=256, kv=128, f=512):
        super().__init__()
        self.layers = torch.nn.ModuleList([_Layer(h, kv, f) for _ in range(n)])


@pytest.mark.parametrize("sym", [True, False])
def test_model_save_and_load_skip_requantization(tmp_path, sym):
    torch.manual_seed(0)
    m = _Model()
    assert _pack_and_replace_linears(m, group_size=128, pack_sym=sym, device="cpu") == 14
    f = tmp_path / "model.safetensors"
    assert save_q4_model(m, f, method="rtn" if sym else "hqq") == 14
    fresh = _Model()
    assert load_q4_model(fresh, f, device="cpu") == 14
    for li in range(2):
        for parent, name in PROJECTIONS:
            a = getattr(getattr(m.layers[li], parent), name)
            b = getattr(getattr(fresh.layers[li], parent), name)
            assert np.array_equal(np.asarray(a._packed), np.asarray(b._packed))
            assert np.array_equal(np.asarray(a._scales), np.asarray(b._scales))
            assert (a._zeros is None) == (b._zeros is None) == sym
            assert b.in_features == a.in_features and b.out_features == a.out_features


@pytest.mark.gpu
def test_loaded_layers_compute_the_same_on_gpu(tmp_path, cuda):
    from siliconfer_b200.packed_io import load_packed
    from siliconfer_b200.q4_linear import Q4Linear
    t = _triples()
    f = tmp_path / "m.safetensors"
    save_packed(f, t, group_size=128)
    got, meta = load_packed(f)
    for name, (p, s, z, *b) in t.items():
        x = torch.randn(3, p.shape[1] * 2, device="cuda")
        a = Q4Linear(p, s, zeros=z, bias=b[0] if b else None, group_size=128)(x)
        g = got[name]
        c = Q4Linear(g[0], g[1], zeros=g[2], bias=g[3], group_size=meta["group_size"])(x)
        assert torch.equal(a, c)
