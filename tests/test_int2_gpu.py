"""2-bit weights on the decode kernel (sf_q2_linear, Q4Linear(bits=2)).

The reference quantizes and packs 2-bit weights (siliconfer/quant/
primitives.py:154-245, 383-425) but refuses to serve them
(siliconfer/engine/q4_loader.py:142-154).  Checked here: the reference's own
golden packings through the GPU kernel against the reference's dequant times
x, and seeded shapes against the CPU oracle; normwise relative error <= 1e-3
(fp32 accumulation)."""
import numpy as np
import pytest
import torch

import cases as C
from oracle import q4_oracle as O
from siliconfer_b200 import _lib, quant as Q
from siliconfer_b200.q4_linear import Q4Linear

pytestmark = pytest.mark.gpu
TOL = 1e-3


@pytest.mark.parametrize("name", list(C.INT2_CASES))
def test_int2_golden(cuda, golden, name):
    g, _ = golden
    seed, n, k, gs, std = C.INT2_CASES[name]
    x = C.acts(seed + 7, 3, k)
    z = g[f"{name}/zeros"] if name.startswith("int2_asym") else None
    m = Q4Linear(g[f"{name}/packed"], g[f"{name}/scales"], zeros=z, group_size=gs, bits=2)
    n0 = _lib.launch_count()
    y = m(torch.from_numpy(x).cuda()).cpu().numpy()
    assert _lib.launch_count() > n0
    assert O.normwise_rel_err(y, g[f"{name}/y"]) <= TOL


@pytest.mark.parametrize("asym", [False, True])
@pytest.mark.parametrize("n,k,gs", [(4096, 4096, 128), (11008, 4096, 128), (4096, 11008, 128),
                                    (1000, 2048, 256), (33, 896, 128), (896, 4864, 128)])
@pytest.mark.parametrize("t", [1, 2, 4, 9, 16, 40])
def test_int2_matches_oracle(cuda, asym, n, k, gs, t):
    rng = np.random.default_rng(n + k + t)
    w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
    if asym:
        p, s, z = Q.pack_weights_int2_asym(w, gs)
    else:
        (p, s), z = Q.pack_weights_int2_sym(w, gs), None
    b = rng.normal(0, 0.1, n).astype(np.float32)
    x = rng.normal(0, 1, (t, k)).astype(np.float32)
    y = Q4Linear(p, s, zeros=z, bias=b, group_size=gs, bits=2)(torch.from_numpy(x).cuda()).cpu().numpy()
    ref = O.gemm_int2(p, s, z, x, gs) + b
    assert O.normwise_rel_err(y, ref) <= TOL
    assert _lib.load().sf_q4_check_device_error() == 0


def test_int2_step_task(cuda):
    """2-bit tasks in the persistent step (sf_q4_task.bits = 2)."""
    rng = np.random.default_rng(9)
    shapes = [(896, 896), (4864, 896), (896, 4864)]
    trips, xs, ys, tasks = [], [], [], []
    for n, k in shapes:
        p, s = Q.pack_weights_int2_sym(rng.normal(0, 0.02, (n, k)).astype(np.float32), 128)
        trips.append((torch.from_numpy(p).cuda(), torch.from_numpy(s).cuda(), p, s))
        xs.append(torch.from_numpy(rng.normal(0, 1, (1, k)).astype(np.float32)).cuda())
        ys.append(torch.zeros((1, n), device="cuda"))
    for (pd, sd, _, _), x, y, (n, k) in zip(trips, xs, ys, shapes):
        tasks.append(_lib.Q4Task(pd.data_ptr(), sd.data_ptr(), None, None, x.data_ptr(), y.data_ptr(), n, k, 1,
                                 128, _lib.SF_F32, _lib.SF_F32, 0, 0, 2))
    lib = _lib.load()
    arr = (_lib.Q4Task * len(tasks))(*tasks)
    nb = int(lib.sf_q4_step_workspace_bytes(arr, len(tasks)))
    assert nb > 0
    ws = torch.zeros(nb + 256, dtype=torch.uint8, device="cuda")
    h = _lib.ctypes.c_void_p()
    _lib.check(lib.sf_q4_step_create(arr, len(tasks), (ws.data_ptr() + 255) & ~255, nb, _lib.ctypes.byref(h)))
    try:
        for _ in range(2):
            _lib.check(lib.sf_q4_step_run(h, torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
    finally:
        lib.sf_q4_step_destroy(h)
    for (_, _, p, s), x, y in zip(trips, xs, ys):
        ref = O.gemm_int2(p, s, None, x.cpu().numpy(), 128)
        assert O.normwise_rel_err(y.cpu().numpy(), ref) <= TOL


def test_mixed_precision_blocks_are_served(cuda):
    """The reference's mixed 4/2-bit blocks (siliconfer/quant/mixed_precision.py:
    251-319), which its loader refuses (q4_loader.py:142-154), load here: a
    2-bit block's projections become Q4Linear(bits=2) on the asymmetric 2-bit
    grid, the 4-bit block stays 4-bit."""
    from test_q4linear_gpu import _Tiny
    from siliconfer_b200.q4_loader import _pack_and_replace_linears
    torch.manual_seed(1)
    m = _Tiny(h=256, f=512, n=2).cuda()
    for prm in m.parameters():
        torch.nn.init.normal_(prm, 0, 0.02)
    W = m.layers[1].mlp.down_proj.weight.detach().cpu().numpy()
    b = m.layers[1].mlp.down_proj.bias
    b = None if b is None else b.detach().cpu().numpy()
    assert _pack_and_replace_linears(m, group_size=128, bits_per_block=[4, 2]) == 14
    assert m.layers[0].mlp.down_proj.bits == 4 and m.layers[1].mlp.down_proj.bits == 2
    x = torch.randn(2, 512, device="cuda")
    p, s, z = Q.pack_weights_int2_asym(W, 128)
    ref = O.gemm_int2(p, s, z, x.cpu().numpy(), 128) + (0 if b is None else b)
    y = m.layers[1].mlp.down_proj(x).cpu().numpy()
    assert O.normwise_rel_err(y, ref) <= TOL
    with pytest.raises(ValueError):
        _pack_and_replace_linears(_Tiny(h=256, f=512, n=2), group_size=128, bits_per_block=[4, 3])
