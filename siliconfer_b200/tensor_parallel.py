"""Tensor-parallel Q4Linear across the GPUs of one node (one process per GPU).

siliconfer runs a model on one device (siliconfer/model/q4_linear.py:32-68,
siliconfer/model/layers.py:93-95, 133, 144).  For models that are larger than
one GPU's share of a decode step, the seven projections of a decoder layer are
sharded the usual way:

* column-parallel (q, k, v, gate, up): rank r owns a contiguous block of
  output rows -- rows of ``packed`` and ``scales``/``zeros`` together.  Each
  rank's output is its block of Y; attention heads and SwiGLU stay local, so
  there is no exchange.
* row-parallel (o, down): rank r owns a contiguous block of whole groups
  along K -- ``packed`` columns ``[g0*gs/2, g1*gs/2)`` and scale/zero columns
  ``[g0, g1)`` -- and reads the matching slice of X.  The partial products are
  summed over ranks: ``mode="peer"`` uses this library's one-shot all-reduce
  over NVLink peer memory (sf_q4_linear_allreduce), ``mode="nccl"`` runs the
  local GEMV and ``torch.distributed.all_reduce`` (the baseline).

Group-boundary sharding keeps the arithmetic of every group unchanged, so the
sum of the shards' partials equals the unsharded product up to fp32
summation order.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib


def shard_bounds(n: int, world: int, rank: int, unit: int = 1):
    """[lo, hi) of rank's share of n items split in whole units (as even as possible)."""
    units = n // unit
    if units * unit != n:
        raise ValueError(f"{n} is not a multiple of the shard unit {unit}")
    if units < world:
        raise ValueError(f"cannot split {units} units over {world} ranks")
    base, extra = divmod(units, world)
    lo = rank * base + min(rank, extra)
    hi = lo + base + (1 if rank < extra else 0)
    return lo * unit, hi * unit


def _slice(a, rows=None, cols=None):
    if a is None:
        return None
    if rows is not None:
        a = a[rows[0]:rows[1]]
    if cols is not None:
        a = a[:, cols[0]:cols[1]]
    if hasattr(a, "contiguous"):
        return a.contiguous()
    return np.ascontiguousarray(a)


def shard_column(packed, scales, zeros, rank: int, world: int, bias=None):
    """Rank's block of output rows (column-parallel): (packed, scales, zeros, bias)."""
    lo, hi = shard_bounds(packed.shape[0], world, rank)
    b = None if bias is None else bias[lo:hi]
    return _slice(packed, rows=(lo, hi)), _slice(scales, rows=(lo, hi)), _slice(zeros, rows=(lo, hi)), b


def shard_row(packed, scales, zeros, group_size: int, rank: int, world: int):
    """Rank's block of whole groups along K (row-parallel): (packed, scales, zeros, (k0, k1))."""
    K = packed.shape[1] * 2
    k0, k1 = shard_bounds(K, world, rank, unit=group_size)
    g0, g1 = k0 // group_size, k1 // group_size
    return (_slice(packed, cols=(k0 // 2, k1 // 2)), _slice(scales, cols=(g0, g1)),
            _slice(zeros, cols=(g0, g1)), (k0, k1))


class PeerComm:
    """This library's NVLink exchange buffers, connected over a process group.

    Collective: every rank constructs it with the same ``slot_bytes``."""

    def __init__(self, group=None, slot_bytes: int = 64 << 20):
        import torch
        import torch.distributed as dist
        self.lib = _lib.load()
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        hb = int(self.lib.sf_tp_handle_bytes())
        handle = (ctypes.c_ubyte * hb)()
        comm = ctypes.c_void_p()
        _lib.check(self.lib.sf_tp_comm_init(self.rank, self.world, slot_bytes, ctypes.byref(comm),
                                            ctypes.cast(handle, ctypes.c_void_p)))
        self.comm = comm
        mine = torch.tensor(bytearray(handle), dtype=torch.uint8)
        dev = torch.device("cuda", torch.cuda.current_device())
        backend = dist.get_backend(group)
        t = mine.to(dev) if backend == "nccl" else mine
        allh = [torch.empty_like(t) for _ in range(self.world)]
        dist.all_gather(allh, t, group=group)
        blob = b"".join(bytes(h.cpu().numpy().tobytes()) for h in allh)
        buf = (ctypes.c_ubyte * len(blob)).from_buffer_copy(blob)
        _lib.check(self.lib.sf_tp_comm_connect(self.comm, ctypes.cast(buf, ctypes.c_void_p)))
        dist.barrier(group=group)

    def close(self):
        if getattr(self, "comm", None):
            self.lib.sf_tp_comm_destroy(self.comm)
            self.comm = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class ColumnParallelQ4Linear:
    """Rank's block of output rows of a Q4Linear; forward gives that block of Y."""

    def __init__(self, packed, scales, zeros=None, bias=None, group_size: int = 128, *,
                 rank: int, world: int, device=None, out_dtype=None):
        from .q4_linear import Q4Linear
        p, s, z, b = shard_column(packed, scales, zeros, rank, world, bias)
        self.rows = shard_bounds(packed.shape[0], world, rank)
        self.local = Q4Linear(p, s, zeros=z, bias=b, group_size=group_size, device=device,
                              out_dtype=out_dtype)

    def __call__(self, x):
        return self.local(x)


class RowParallelQ4Linear:
    """Rank's block of K groups of a Q4Linear; forward(x_shard) gives the full Y.

    ``x_shard`` is X[..., k0:k1] (``self.k_range``).  ``mode="peer"`` sums the
    partials with the library's NVLink all-reduce (needs a PeerComm);
    ``mode="nccl"`` runs the local GEMV then torch.distributed.all_reduce."""

    def __init__(self, packed, scales, zeros=None, bias=None, group_size: int = 128, *,
                 rank: int, world: int, device=None, out_dtype=None, mode: str = "peer",
                 comm: PeerComm | None = None, group=None):
        import torch
        from .q4_linear import Q4Linear
        if mode not in ("peer", "nccl"):
            raise ValueError("mode must be 'peer' or 'nccl'")
        if mode == "peer" and comm is None:
            raise ValueError("mode='peer' needs a PeerComm")
        p, s, z, self.k_range = shard_row(packed, scales, zeros, group_size, rank, world)
        self.local = Q4Linear(p, s, zeros=z, group_size=group_size, device=device)
        dev = self.local.packed_d.device
        self.bias_d = None if bias is None else torch.as_tensor(np.asarray(bias, np.float32)).to(dev)
        self.mode, self.comm, self.group = mode, comm, group
        self.out_dtype = out_dtype or torch.float32
        self.out_features = self.local.out_features

    def __call__(self, x):
        import torch
        import torch.distributed as dist
        from .kernels.cuda import _dtype_code
        orig = x.shape
        xt = x.reshape(-1, orig[-1]).contiguous()
        T = xt.shape[0]
        N = self.out_features
        if self.mode == "nccl":
            y = self.local(xt)                       # fp32 partial
            dist.all_reduce(y, group=self.group)
            if self.bias_d is not None:
                y = y + self.bias_d
            y = y.to(self.out_dtype)
        else:
            y = torch.empty((T, N), dtype=self.out_dtype, device=xt.device)
            L = self.local
            _lib.check(self.comm.lib.sf_q4_linear_allreduce(
                self.comm.comm, L.packed_d.data_ptr(), L.scales_d.data_ptr(),
                None if L.zeros_d is None else L.zeros_d.data_ptr(),
                None if self.bias_d is None else self.bias_d.data_ptr(),
                xt.data_ptr(), _dtype_code(xt), y.data_ptr(), _dtype_code(y), N, L.in_features, T,
                L.group_size, torch.cuda.current_stream(xt.device).cuda_stream))
        return y.reshape(*orig[:-1], N)


__all__ = ["shard_bounds", "shard_column", "shard_row", "PeerComm", "ColumnParallelQ4Linear",
           "RowParallelQ4Linear"]
