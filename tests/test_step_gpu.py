"""The persistent multi-GEMV launch (sf_q4_step_*) against one launch per GEMV
and against the CPU oracle, including a chain where each task consumes the
previous task's output (the grid barrier must order them)."""
import ctypes

import numpy as np
import pytest
import torch

import cases as C
from oracle import q4_oracle as O
from siliconfer_b200 import _lib
from siliconfer_b200.kernels import cuda as K
from siliconfer_b200.q4_linear import Q4Linear
from siliconfer_b200.quant import pack_weights_device
from siliconfer_b200.runner import Q4StepRunner

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _layers(shapes, asym, seed=0):
    torch.manual_seed(seed)
    out = []
    for n, k in shapes:
        trip = pack_weights_device(torch.randn(n, k, device="cuda") * 0.02 + (0.003 if asym else 0),
                                   128, sym=not asym)
        out.append(Q4Linear(trip[0], trip[1], zeros=None if not asym else trip[2],
                            group_size=128, device="cuda"))
    return out


@pytest.mark.parametrize("asym", [False, True])
@pytest.mark.parametrize("t", [1, 4])
def test_step_matches_single_launches(cuda, asym, t):
    shapes = [(n, k) for n, k in C.QWEN05B.values()] * 2
    layers = _layers(shapes, asym)
    r = Q4StepRunner(layers, tokens=t, device="cuda")
    assert r.persistent or t > 1   # large T*K may not fit one persistent launch
    g = torch.Generator(device="cuda").manual_seed(3)
    r.x.copy_(torch.randn(r.x.shape, generator=g, device="cuda").half())
    n0 = _lib.launch_count()
    r.capture()
    for _ in range(2):
        r.run()
    r.stream.synchronize()
    assert _lib.launch_count() > n0
    for i, m in enumerate(layers):
        ref = K.linear(m.packed_d, m.scales_d, m.zeros_d, r.x_slot(i).contiguous(), 128)
        got = r.y_slot(i)
        assert (got - ref).abs().max().item() <= 1e-6 * ref.abs().max().item() + 1e-30, i
        if i < 7:
            yo = O.gemm(m.packed_d.cpu().numpy(), m.scales_d.cpu().numpy(),
                        None if m.zeros_d is None else m.zeros_d.cpu().numpy(),
                        r.x_slot(i).float().cpu().numpy(), 128)
            assert O.normwise_rel_err(got.cpu().numpy(), yo) <= TOL
    assert _lib.load().sf_q4_check_device_error() == 0


def test_step_chain_dependency(cuda):
    """y_{i+1} = W_{i+1} y_i: every task waits for the previous one."""
    n = 2048
    layers = _layers([(n, n)] * 6, False, seed=5)
    lib = _lib.load()
    x0 = torch.randn(1, n, device="cuda")
    bufs = [x0] + [torch.empty(1, n, device="cuda") for _ in layers]
    arr = (_lib.Q4Task * len(layers))()
    for i, m in enumerate(layers):
        arr[i] = _lib.Q4Task(m.packed_d.data_ptr(), m.scales_d.data_ptr(), None, None,
                             bufs[i].data_ptr(), bufs[i + 1].data_ptr(), n, n, 1, 128,
                             _lib.SF_F32, _lib.SF_F32, 1)
    nb = int(lib.sf_q4_step_workspace_bytes(arr, len(layers)))
    ws = torch.zeros(nb, dtype=torch.uint8, device="cuda")
    h = ctypes.c_void_p()
    _lib.check(lib.sf_q4_step_create(arr, len(layers), ws.data_ptr(), nb, ctypes.byref(h)))
    try:
        for rep in range(3):
            for b in bufs[1:]:
                b.fill_(float("nan"))
            _lib.check(lib.sf_q4_step_run(h, torch.cuda.current_stream().cuda_stream))
            torch.cuda.synchronize()
            ref = x0
            for i, m in enumerate(layers):
                ref = K.linear(m.packed_d, m.scales_d, None, ref, 128)
                assert torch.isfinite(bufs[i + 1]).all(), (rep, i)
                err = ((bufs[i + 1] - ref).abs().max() / ref.abs().max()).item()
                assert err <= 1e-5, (rep, i, err)
    finally:
        lib.sf_q4_step_destroy(h)
    assert lib.sf_q4_check_device_error() == 0


def test_step_rejects_mixed_tasks(cuda):
    lib = _lib.load()
    a = _layers([(256, 512)], False)[0]
    b = _layers([(256, 512)], True)[0]
    x = torch.zeros(1, 512, device="cuda")
    y = torch.zeros(2, 256, device="cuda")
    arr = (_lib.Q4Task * 2)()
    arr[0] = _lib.Q4Task(a.packed_d.data_ptr(), a.scales_d.data_ptr(), None, None, x.data_ptr(),
                         y.data_ptr(), 256, 512, 1, 128, 0, 0, 0)
    arr[1] = _lib.Q4Task(b.packed_d.data_ptr(), b.scales_d.data_ptr(), b.zeros_d.data_ptr(), None,
                         x.data_ptr(), y[1:].data_ptr(), 256, 512, 1, 128, 0, 0, 0)
    nb = int(lib.sf_q4_step_workspace_bytes(arr, 2))
    ws = torch.zeros(nb, dtype=torch.uint8, device="cuda")
    h = ctypes.c_void_p()
    assert lib.sf_q4_step_create(arr, 2, ws.data_ptr(), nb, ctypes.byref(h)) == 6
    assert b"same T" in lib.sf_last_error()
    assert lib.sf_q4_step_create(arr, 1, ws.data_ptr(), 8, ctypes.byref(h)) == 2


def test_config2_24_layer_asym_step_matches_reference(cuda, golden):
    """BASELINE config 2 as one persistent launch: 24 layers x 7 asymmetric
    projections (layer 0 HQQ with the 60 sigma outlier, layers 1-23 the
    reference's asymmetric RTN), batch 1, each projection on its own input,
    against the reference's gemm_asym outputs."""
    g, _ = golden
    layers, keys, xs = [], [], []
    for layer in range(C.QWEN_LAYERS):
        for proj, (n, k) in C.QWEN05B.items():
            w = C.qwen_asym_weights(layer, proj)
            if layer == 0:
                w = O.hqq_quantize_weight(w, 128)
                key = f"c2/{proj}/y"
            else:
                key = f"c2L/{layer}/{proj}/y"
            p, s, z = pack_weights_device(torch.from_numpy(w).cuda(), 128, sym=False)
            layers.append(Q4Linear(p, s, zeros=z, group_size=128, device="cuda"))
            keys.append(key)
            xs.append(C.acts(C.layer_seed(2, layer, proj) + 7, 1, k))
    r = Q4StepRunner(layers, tokens=1, x_dtype=torch.float32, device="cuda", waits=[False] * len(layers))
    assert r.persistent
    for i, x in enumerate(xs):
        r.x_slot(i).copy_(torch.from_numpy(x))
    r.capture()
    r.run()
    r.stream.synchronize()
    worst = max(O.normwise_rel_err(r.y_slot(i).cpu().numpy(), g[key]) for i, key in enumerate(keys))
    assert worst <= TOL, worst
    assert _lib.load().sf_q4_check_device_error() == 0


def _pack_np(w, gs, bits, asym):
    from siliconfer_b200 import quant as Q
    if bits == 2:
        return Q.pack_weights_int2_asym(w, gs) if asym else Q.pack_weights_int2_sym(w, gs)
    return Q.pack_weights_asym(w, gs) if asym else Q.pack_weights_sym(w, gs)


@pytest.mark.parametrize("t", [1, 2])
@pytest.mark.parametrize("bits,gs", [(4, 32), (4, 64), (4, 128), (4, 256), (2, 128), (2, 256)])
@pytest.mark.parametrize("asym", [False, True])
def test_step_chain_every_format(cuda, t, bits, gs, asym):
    """A dependent chain y_{i+1} = W_{i+1} y_i in every weight format, with K
    not a multiple of a weight stage (256 k at 4 bits, 512 at 2): each task's
    units read the previous task's output, written inside the same launch.
    Checked against the oracle run on the kernel's own intermediate inputs."""
    rng = np.random.default_rng(11 + gs + bits + t)
    dims = [gs * 9, gs * 5, gs * 14, gs * 3]
    trips = [_pack_np(rng.normal(0, 0.02, (dims[i + 1], dims[i])).astype(np.float32), gs, bits, asym)
             for i in range(len(dims) - 1)]
    dev = [[torch.from_numpy(a).cuda() for a in tr] for tr in trips]
    x0 = torch.from_numpy(rng.normal(0, 1, (t, dims[0])).astype(np.float32)).cuda()
    bufs = [x0] + [torch.full((t, d), float("nan"), device="cuda") for d in dims[1:]]
    arr = (_lib.Q4Task * len(trips))()
    for i, tr in enumerate(dev):
        arr[i] = _lib.Q4Task(tr[0].data_ptr(), tr[1].data_ptr(), tr[2].data_ptr() if asym else None, None,
                             bufs[i].data_ptr(), bufs[i + 1].data_ptr(), dims[i + 1], dims[i], t, gs,
                             _lib.SF_F32, _lib.SF_F32, 1 if i else 0, 0, bits)
    lib = _lib.load()
    nb = int(lib.sf_q4_step_workspace_bytes(arr, len(trips)))
    assert nb > 0
    ws = torch.zeros(nb + 256, dtype=torch.uint8, device="cuda")
    h = ctypes.c_void_p()
    _lib.check(lib.sf_q4_step_create(arr, len(trips), (ws.data_ptr() + 255) & ~255, nb, ctypes.byref(h)))
    try:
        for _ in range(3):
            for b in bufs[1:]:
                b.fill_(float("nan"))
            _lib.check(lib.sf_q4_step_run(h, torch.cuda.current_stream().cuda_stream))
            torch.cuda.synchronize()
            for i, tr in enumerate(trips):
                xin = bufs[i].cpu().numpy()
                f = O.gemm_int2 if bits == 2 else O.gemm
                ref = f(tr[0], tr[1], tr[2] if asym else None, xin, gs)
                got = bufs[i + 1].cpu().numpy()
                assert np.isfinite(got).all(), i
                assert O.normwise_rel_err(got, ref) <= TOL, i
    finally:
        lib.sf_q4_step_destroy(h)
    assert lib.sf_q4_check_device_error() == 0
