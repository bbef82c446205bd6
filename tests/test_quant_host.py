"""Product packers (siliconfer_b200.quant) are bit-exact with the reference."""
import numpy as np
import pytest

import cases as C
from oracle import q4_oracle as O
from siliconfer_b200 import quant as Q


@pytest.mark.parametrize("name", list(C.UNIT_CASES))
def test_pack_unit_cases(name, golden):
    _, meta = golden
    w, _, gs = C.unit_case(name)
    out = Q.pack_weights_asym(w, gs) if C.is_asym(name) else Q.pack_weights_sym(w, gs)
    assert C.sha(out[0]) == meta["hashes"][f"{name}/packed"]
    assert C.sha(out[1]) == meta["hashes"][f"{name}/scales"]


@pytest.mark.parametrize("proj", list(C.QWEN05B))
def test_pack_config1(proj, golden):
    _, meta = golden
    n, k = C.QWEN05B[proj]
    p, s = Q.pack_weights_sym(C.weights(C.layer_seed(1, 0, proj), n, k), 128)
    assert C.sha(p) == meta["hashes"][f"c1/{proj}/packed"]
    assert C.sha(s) == meta["hashes"][f"c1/{proj}/scales"]


@pytest.mark.parametrize("proj", list(C.QWEN05B))
def test_hqq_config2(proj, golden):
    """HQQ restatement + asym packing reproduce the reference's triple,
    including the 60-sigma outlier group of down_proj."""
    g, meta = golden
    wh = O.hqq_quantize_weight(C.qwen_asym_weights(0, proj), 128)
    assert C.sha(wh) == meta["hashes"][f"c2/{proj}/hqq"]
    p, s, z = Q.pack_weights_asym(wh, 128)
    assert C.sha(p) == meta["hashes"][f"c2/{proj}/packed"]
    assert C.sha(s) == meta["hashes"][f"c2/{proj}/scales"]
    assert C.sha(z) == meta["hashes"][f"c2/{proj}/zeros"]
    if proj == "down":
        gi = C.OUTLIER["col"] // 128
        assert s[C.OUTLIER["row"], gi] == g["c2/down/outlier_group_scale"][0]


def test_pack_validation():
    with pytest.raises(ValueError):
        Q.pack_weights_sym(np.zeros((4, 100), np.float32), 64)
    q, s = Q.quantize_sym(np.zeros((2, 64), np.float32), 64)
    assert np.all(q == 0) and np.all(s == 0)
    q, s, z = Q.quantize_asym(np.full((2, 64), 3.0, np.float32), 64)
    assert np.all(s == 0)


def test_pack_boundary_values():
    w = np.arange(-8, 8, dtype=np.float32)[None, :].repeat(2, 0) * np.float32(7 / 8)
    p, s = Q.pack_weights_sym(np.concatenate([w, w], 1), 32)
    lo, hi = p & 15, p >> 4
    assert lo.max() <= 15 and hi.max() <= 15
