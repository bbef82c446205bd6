"""Gate/up with the SwiGLU activation fused (siliconfer/model/layers.py:144:
down_proj(silu(gate_proj(x)) * up_proj(x))).

Host: the interleaved row layout.  GPU: the fused decode GEMV (and, above 16
tokens, the stacked GEMM + activation kernel) against the CPU oracle:
silu(gate) * up from the oracle's Q4Linear forward of each projection,
normwise relative error <= 1e-3 (5e-3 when the stacked product runs on the
bf16 tensor-core prefill)."""
import numpy as np
import pytest
import torch

from oracle import q4_oracle as O
from siliconfer_b200 import _lib, quant as Q
from siliconfer_b200.fused import SwiGLUQ4Linear, interleave_gate_up
from siliconfer_b200.q4_linear import Q4Linear


def test_interleave_layout():
    g = np.arange(32 * 3).reshape(32, 3)
    u = -np.arange(32 * 3).reshape(32, 3)
    w = interleave_gate_up(g, u)
    assert w.shape == (64, 3)
    assert np.array_equal(w[0:16], g[0:16]) and np.array_equal(w[16:32], u[0:16])
    assert np.array_equal(w[32:48], g[16:32]) and np.array_equal(w[48:64], u[16:32])
    with pytest.raises(ValueError):
        interleave_gate_up(g[:24], u[:24])


def _silu(v):
    v = v.astype(np.float64)
    return v / (1.0 + np.exp(-v))


@pytest.mark.gpu
@pytest.mark.parametrize("n,k,gs", [(4864, 896, 128), (11008, 4096, 128), (256, 512, 64), (96, 256, 32)])
@pytest.mark.parametrize("asym", [False, True])
@pytest.mark.parametrize("t", [1, 2, 5, 16, 64])
def test_swiglu_matches_oracle(cuda, n, k, gs, asym, t):
    if gs == 32 and 8 < t <= 16:
        t = 8
    rng = np.random.default_rng(n + k + t + asym)
    lay, host = [], []
    for i in range(2):
        w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
        p, s, z = Q.pack_weights_asym(w, gs) if asym else (*Q.pack_weights_sym(w, gs), None)
        b = rng.normal(0, 0.05, n).astype(np.float32) if i == 1 or asym else None
        lay.append(Q4Linear(p, s, zeros=z, bias=b, group_size=gs))
        host.append((p, s, z, b))
    x = rng.normal(0, 1, (t, k)).astype(np.float32)
    n0 = _lib.launch_count()
    y = SwiGLUQ4Linear(*lay)(torch.from_numpy(x).cuda()).cpu().numpy()
    launched = _lib.launch_count() - n0
    gate = O.q4linear_forward(*host[0], x, gs)
    up = O.q4linear_forward(*host[1], x, gs)
    ref = (_silu(gate) * up).astype(np.float32)
    tol = 5e-3 if t >= 48 else 1e-3
    assert O.normwise_rel_err(y, ref) <= tol
    if t <= 16:
        assert launched == 2          # activation pre-pass + one GEMV launch with the fused epilogue
    assert _lib.load().sf_q4_check_device_error() == 0


@pytest.mark.gpu
def test_swiglu_task_in_a_step(cuda):
    """The same epilogue as a task of the persistent step (sf_q4_task.epilogue)."""
    rng = np.random.default_rng(3)
    n, k, gs, t = 2048, 1024, 128, 2
    trip = [Q.pack_weights_sym(rng.normal(0, 0.02, (n, k)).astype(np.float32), gs) for _ in range(2)]
    P = torch.from_numpy(interleave_gate_up(trip[0][0], trip[1][0])).cuda()
    S = torch.from_numpy(interleave_gate_up(trip[0][1], trip[1][1])).cuda()
    x = rng.normal(0, 1, (t, k)).astype(np.float32)
    X = torch.from_numpy(x).cuda()
    Y = torch.zeros((t, n), device="cuda")
    lib = _lib.load()
    arr = (_lib.Q4Task * 1)(_lib.Q4Task(P.data_ptr(), S.data_ptr(), None, None, X.data_ptr(), Y.data_ptr(),
                                        2 * n, k, t, gs, _lib.SF_F32, _lib.SF_F32, 0, _lib.SF_EPI_SWIGLU))
    nb = int(lib.sf_q4_step_workspace_bytes(arr, 1))
    ws = torch.zeros(nb + 256, dtype=torch.uint8, device="cuda")
    h = _lib.ctypes.c_void_p()
    _lib.check(lib.sf_q4_step_create(arr, 1, (ws.data_ptr() + 255) & ~255, nb, _lib.ctypes.byref(h)))
    try:
        for _ in range(2):
            _lib.check(lib.sf_q4_step_run(h, torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
    finally:
        lib.sf_q4_step_destroy(h)
    ref = (_silu(O.gemm(*trip[0], None, x, gs)) * O.gemm(*trip[1], None, x, gs)).astype(np.float32)
    assert O.normwise_rel_err(Y.cpu().numpy(), ref) <= 1e-3
