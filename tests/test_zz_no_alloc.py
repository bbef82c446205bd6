"""sf_q4_linear_static_scratch: the decode GEMV on the library's fixed device
buffer (no allocation) must give what sf_q4_linear gives, call after call.

Named to be collected last; it also passes when run on its own.
"""
import numpy as np
import pytest
import torch

from oracle import q4_oracle as O
from siliconfer_b200 import _lib, quant as Q

pytestmark = pytest.mark.gpu
TOL = 1e-3   # normwise relative error, as for every fp32-accumulate GEMV test


def _case(seed, n, k, gs, asym, t):
    rng = np.random.default_rng(seed)
    w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
    x = rng.normal(0, 1, (t, k)).astype(np.float32)
    if asym:
        p, s, z = Q.pack_weights_asym(w, gs)
    else:
        (p, s), z = Q.pack_weights_sym(w, gs), None
    d = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return d(p), d(s), d(z), torch.from_numpy(x).cuda().half(), x


def _call(fn, p, s, z, x, n, gs, static):
    lib = _lib.load()
    t, k = x.shape
    y = torch.full((t, n), float("nan"), dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    zp = None if z is None else z.data_ptr()
    if static:
        rc = lib.sf_q4_linear_static_scratch(p.data_ptr(), s.data_ptr(), zp, None, x.data_ptr(),
                                             _lib.SF_F16, y.data_ptr(), _lib.SF_F32, n, k, t, gs, st)
    else:
        rc = lib.sf_q4_linear(p.data_ptr(), s.data_ptr(), zp, None, x.data_ptr(), _lib.SF_F16,
                              y.data_ptr(), _lib.SF_F32, n, k, t, gs, 0, st)
    _lib.check(rc)
    return y


@pytest.mark.parametrize("n,k,gs,asym,t", [
    (4096, 4096, 128, False, 1),     # k-split with partial sums
    (11008, 4096, 128, False, 4),
    (4096, 11008, 128, True, 3),     # G = 86: per-lane scale copies
    (1000, 2048, 64, True, 8),       # ragged N, group 64
    # activation blocks of 3.2 MB: the k-split the allocating entry would pick
    # (64 ranges of partial sums, 1 MB) no longer fits beside them in the
    # buffer, so the entry lowers the k-split until it does
    (512, 131072, 128, False, 8),
])
def test_static_scratch_matches_linear_twice(cuda, n, k, gs, asym, t):
    p, s, z, x, xh = _case(n + k + t, n, k, gs, asym, t)
    ref = _call(None, p, s, z, x, n, gs, static=False)
    y1 = _call(None, p, s, z, x, n, gs, static=True)
    y2 = _call(None, p, s, z, x, n, gs, static=True)
    torch.cuda.synchronize()
    for y in (y1, y2):
        assert torch.isfinite(y).all()
        assert O.normwise_rel_err(y.cpu().numpy(), ref.cpu().numpy()) <= TOL
    # and against the oracle on the fp16-rounded activations
    xo = x.float().cpu().numpy()
    yo = O.gemm(p.cpu().numpy(), s.cpu().numpy(), None if z is None else z.cpu().numpy(), xo, gs)
    assert O.normwise_rel_err(y2.cpu().numpy(), yo) <= TOL
    assert _lib.load().sf_q4_check_device_error() == 0


def test_static_scratch_rejects_oversize(cuda):
    lib = _lib.load()
    n, k, t, gs = 32, 262144, 8, 128            # activation blocks ~6.3 MB > the 4 MiB buffer
    p = torch.zeros((n, k // 2), dtype=torch.uint8, device="cuda")
    s = torch.ones((n, k // gs), dtype=torch.float32, device="cuda")
    x = torch.zeros((t, k), dtype=torch.float16, device="cuda")
    y = torch.zeros((t, n), dtype=torch.float32, device="cuda")
    rc = lib.sf_q4_linear_static_scratch(p.data_ptr(), s.data_ptr(), None, None, x.data_ptr(),
                                         _lib.SF_F16, y.data_ptr(), _lib.SF_F32, n, k, t, gs,
                                         torch.cuda.current_stream().cuda_stream)
    assert rc == 2                              # SF_ERR_SHAPE
    assert b"static GEMV scratch" in lib.sf_last_error()
