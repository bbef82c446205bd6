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


def shard_column(packed, scales, zeros, rank: int, world: int, bias=None, unit: int = 1):
    """Rank's block of output rows (column-parallel): (packed, scales, zeros, bias).

    ``unit`` > 1 keeps blocks of ``unit`` rows together -- ``head_dim`` for
    q/k/v, so that attention heads stay whole on one rank -- and then the
    blocks must divide evenly over the ranks (every rank the same head count);
    a ValueError says so otherwise."""
    n = packed.shape[0]
    if unit > 1 and (n % unit or (n // unit) % world):
        raise ValueError(f"{n} rows = {n / unit:g} heads of {unit} rows do not divide evenly over {world} ranks")
    lo, hi = shard_bounds(n, world, rank, unit)
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

    def __init__(self, group=None, slot_bytes: int = 64 << 20, arena_bytes: int = 0):
        import torch
        import torch.distributed as dist
        self.lib = _lib.load()
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        hb = int(self.lib.sf_tp_handle_bytes())
        handle = (ctypes.c_ubyte * hb)()
        comm = ctypes.c_void_p()
        _lib.check(self.lib.sf_tp_comm_init(self.rank, self.world, slot_bytes, arena_bytes, ctypes.byref(comm),
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
    """Rank's block of output rows of a Q4Linear; forward gives that block of Y.

    Pass ``unit=head_dim`` for q/k/v so that heads are never split."""

    def __init__(self, packed, scales, zeros=None, bias=None, group_size: int = 128, *,
                 rank: int, world: int, device=None, out_dtype=None, unit: int = 1):
        from .q4_linear import Q4Linear
        p, s, z, b = shard_column(packed, scales, zeros, rank, world, bias, unit)
        self.rows = shard_bounds(packed.shape[0], world, rank, unit)
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


class TPStepRunner:
    """A tensor-parallel decode step as one CUDA graph per rank.

    ``layers``: per decoder layer, the rank's seven Q4Linear shards in the
    order q, k, v, o, gate, up, down (q/k/v/gate/up column-parallel, o/down
    row-parallel).  Each half layer is one persistent multi-GEMV launch
    (sf_q4_step_run: q/k/v/o-partial, then gate/up/down-partial), followed by
    the all-reduce of the row-parallel partial -- the library's NVLink
    all-reduce (``mode="peer"``) or NCCL (``mode="nccl"``).  ``mode="fused"``
    runs the whole step as ONE persistent launch: row-parallel tiles are pushed
    to every rank over NVLink as they finish and summed by reduce tasks inside
    the same kernel (sf_q4_step_create_tp; the communicator needs
    ``arena_bytes(...)`` of arena).  With one rank the all-reduces are skipped.  As in the single-GPU step, every projection
    reads its own input slot (attention, norms and SwiGLU are outside this
    path); only the exchange points of the decoder are kept.
    """

    ROW_PARALLEL = (False, False, False, True, False, False, True)
    # with ordered=True (fused mode): which projections wait for everything
    # before them -- q (the previous layer's down all-reduce), o (q/k/v), gate
    # (the o all-reduce), down (gate/up); the decoder's order
    # (siliconfer/model/layers.py:93-95, 133, 144)
    LAYER_WAITS = (True, False, False, True, True, False, True)

    def __init__(self, layers, tokens: int = 1, x_dtype=None, mode: str = "peer",
                 comm: PeerComm | None = None, group=None, device=None, ordered: bool = False,
                 exchange: bool = True):
        import torch
        import torch.distributed as dist
        self.torch = torch
        self.layers = [list(l) for l in layers]
        self.tokens = int(tokens)
        self.x_dtype = x_dtype or torch.float16
        self.mode, self.comm, self.group = mode, comm, group
        if ordered and mode != "fused":
            raise ValueError("ordered=True needs mode='fused' (the unfused modes run in order already)")
        self.ordered = bool(ordered)
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        # exchange=False (fused mode, measurement only): the row-parallel shards'
        # partial products are written locally and not summed across ranks
        self.exchange = bool(exchange) and self.world > 1
        if not exchange and mode != "fused":
            raise ValueError("exchange=False needs mode='fused'")
        if self.world > 1 and (mode == "peer" or (mode == "fused" and self.exchange)) and comm is None:
            raise ValueError(f"mode={mode!r} needs a PeerComm")
        self.device = torch.device(device) if device is not None else self.layers[0][0].packed_d.device
        self.lib = _lib.load()
        align = 64
        xo = yo = 0
        self.slots = []           # per layer: list of (x_off, y_off)
        for lay in self.layers:
            s = []
            for m in lay:
                s.append((xo, yo))
                xo += -(-self.tokens * m.in_features // align) * align
                yo += -(-self.tokens * m.out_features // align) * align
            self.slots.append(s)
        self.x = torch.zeros(xo, dtype=self.x_dtype, device=self.device)
        self.y = torch.zeros(yo, dtype=torch.float32, device=self.device)   # GEMV outputs / partials
        hidden = self.layers[0][3].out_features
        # all-reduced outputs of o and down, per layer
        self.red = torch.zeros((len(self.layers), 2, self.tokens, hidden), dtype=torch.float32, device=self.device)
        self.x_host = torch.zeros(xo, dtype=self.x_dtype, pin_memory=True)
        self.red_host = torch.zeros(self.red.shape, dtype=torch.float32, pin_memory=True)
        self.stream = torch.cuda.Stream(self.device)
        self._handles, self._ws = [], []
        if mode == "fused":
            self._handles.append(self._make_fused())
        else:
            for li, lay in enumerate(self.layers):
                for half in ((0, 1, 2, 3), (4, 5, 6)):
                    self._handles.append(self._make_step(li, half))
        self.graph = None

    @staticmethod
    def arena_bytes(n_layers: int, tokens: int, hidden: int, world: int) -> int:
        """Communicator arena a fused step needs (two exchange regions per layer)."""
        par = -(-(world * tokens * hidden * 4) // 256) * 256
        flags = -(-((hidden + 31) // 32 * world * 8) // 256) * 256
        return 2 * n_layers * (2 * par + flags)

    def _make_fused(self):
        """Every layer's seven projections and two all-reduces as one step.

        Independent (default): every task reads its pre-supplied input at once.
        Ordered: the projections named in LAYER_WAITS open a new phase and read
        their input only after every earlier task (all-reduces included) has
        written its output, as a decoder would."""
        from .kernels.cuda import _dtype_code
        torch = self.torch
        tasks, roles, pending = [], [], []
        xs = self.x.element_size()
        for li, lay in enumerate(self.layers):
            for i, m in enumerate(lay):
                xo, yo = self.slots[li][i]
                row = self.ROW_PARALLEL[i]
                wait = 1 if (self.ordered and self.LAYER_WAITS[i] and (li, i) != (0, 0)) else 0
                base = (m.packed_d.data_ptr(), m.scales_d.data_ptr(),
                        None if m.zeros_d is None else m.zeros_d.data_ptr())
                xp = self.x.data_ptr() + xo * xs
                if not row:
                    tasks.append(_lib.Q4Task(*base, None if m.bias_d is None else m.bias_d.data_ptr(), xp,
                                             self.y.data_ptr() + yo * 4, m.out_features, m.in_features,
                                             self.tokens, m.group_size, _dtype_code(self.x), _lib.SF_F32, wait))
                    roles.append(0)
                    continue
                out = self.red[li, 0 if i == 3 else 1]
                if not self.exchange:
                    tasks.append(_lib.Q4Task(*base, None, xp, out.data_ptr(), m.out_features, m.in_features,
                                             self.tokens, m.group_size, _dtype_code(self.x), _lib.SF_F32, wait))
                    roles.append(0)
                    continue
                src = len(tasks)
                tasks.append(_lib.Q4Task(*base, None, xp, None, m.out_features, m.in_features, self.tokens,
                                         m.group_size, _dtype_code(self.x), _lib.SF_F32, wait))
                roles.append(1)
                red = (_lib.Q4Task(*base, None, xp, out.data_ptr(), m.out_features, m.in_features,
                                   self.tokens, m.group_size, _dtype_code(self.x), _lib.SF_F32, 0), 2 + src)
                if self.ordered:
                    # the next phase reads this output: reduce right away
                    tasks.append(red[0])
                    roles.append(red[1])
                else:
                    # nothing waits for it: reduce after the next row-parallel shard, so that
                    # the warps reaching its units find every rank's tiles long pushed
                    for t_, r_ in pending:
                        tasks.append(t_)
                        roles.append(r_)
                    pending = [red]
        for t_, r_ in pending:
            tasks.append(t_)
            roles.append(r_)
        n = len(tasks)
        arr = (_lib.Q4Task * n)(*tasks)
        rl = (_lib.ctypes.c_int * n)(*roles)
        nbytes = int(self.lib.sf_q4_step_workspace_bytes(arr, n))
        ws = torch.zeros(nbytes + 256, dtype=torch.uint8, device=self.device)
        self._ws.append(ws)
        h = _lib.ctypes.c_void_p()
        comm = self.comm.comm if (self.comm is not None and self.exchange) else None
        with torch.cuda.device(self.device):
            if self.exchange:
                _lib.check(self.lib.sf_q4_step_create_tp(arr, rl, n, comm, (ws.data_ptr() + 255) & ~255, nbytes,
                                                         _lib.ctypes.byref(h)))
            else:
                _lib.check(self.lib.sf_q4_step_create(arr, n, (ws.data_ptr() + 255) & ~255, nbytes,
                                                      _lib.ctypes.byref(h)))
        return h

    def _make_step(self, li, idx):
        from .kernels.cuda import _dtype_code
        torch = self.torch
        n = len(idx)
        arr = (_lib.Q4Task * n)()
        xs = self.x.element_size()
        for j, i in enumerate(idx):
            m = self.layers[li][i]
            xo, yo = self.slots[li][i]
            arr[j] = _lib.Q4Task(
                m.packed_d.data_ptr(), m.scales_d.data_ptr(),
                None if m.zeros_d is None else m.zeros_d.data_ptr(),
                None if m.bias_d is None else m.bias_d.data_ptr(),
                self.x.data_ptr() + xo * xs, self.y.data_ptr() + yo * 4,
                m.out_features, m.in_features, self.tokens, m.group_size,
                _dtype_code(self.x), _lib.SF_F32, 0)
        nbytes = int(self.lib.sf_q4_step_workspace_bytes(arr, n))
        ws = torch.zeros(nbytes + 256, dtype=torch.uint8, device=self.device)
        self._ws.append(ws)
        h = _lib.ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check(self.lib.sf_q4_step_create(arr, n, (ws.data_ptr() + 255) & ~255, nbytes,
                                                  _lib.ctypes.byref(h)))
        return h

    def y_slot(self, li, i):
        m = self.layers[li][i]
        yo = self.slots[li][i][1]
        return self.y[yo:yo + self.tokens * m.out_features].view(self.tokens, m.out_features)

    def _reduce(self, li, which, st):
        torch = self.torch
        i = 3 if which == 0 else 6
        part = self.y_slot(li, i)
        out = self.red[li, which]
        if self.world == 1:
            out.copy_(part)
        elif self.mode == "nccl":
            import torch.distributed as dist
            dist.all_reduce(part, group=self.group)
            out.copy_(part)
        else:
            _lib.check(self.lib.sf_tp_allreduce(self.comm.comm, part.data_ptr(), out.data_ptr(), _lib.SF_F32,
                                                None, part.numel(), part.shape[1], st.cuda_stream))

    def launches_per_step(self) -> int:
        """Kernels of this library per step: one per step handle (the
        persistent GEMV launch), plus one peer all-reduce per row-parallel
        projection when mode is 'peer' and world > 1."""
        red = 2 * len(self.layers) if (self.world > 1 and self.mode == "peer") else 0
        return len(self._handles) + red

    def _launch_all(self, st):
        if self.mode == "fused":
            _lib.check(self.lib.sf_q4_step_run(self._handles[0], st.cuda_stream))
            return
        for li in range(len(self.layers)):
            for half in range(2):
                _lib.check(self.lib.sf_q4_step_run(self._handles[2 * li + half], st.cuda_stream))
                self._reduce(li, half, st)

    def _sync_ranks(self):
        """Line the ranks up before a run whose kernels wait on peers: the
        exchange waits are bounded (about 2 s), so a rank that is still
        building its shards would otherwise make the others' waits expire."""
        if self.world > 1 and (self.mode == "peer" or (self.mode == "fused" and self.exchange)):
            import torch.distributed as dist
            self.torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
            self.torch.cuda.synchronize(self.device)

    def capture(self):
        torch = self.torch
        self._sync_ranks()
        with torch.cuda.device(self.device):
            self.stream.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self.stream):
                self._launch_all(self.stream)
            self.stream.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=self.stream):
                self._launch_all(self.stream)
            self.graph = g

    def run(self):
        if self.graph is None:
            self.capture()
        with self.torch.cuda.stream(self.stream):
            self.graph.replay()

    def run_host(self):
        """One step from pinned host activations to the pinned host copy of the
        all-reduced o/down outputs."""
        if self.graph is None:
            self.capture()
        with self.torch.cuda.stream(self.stream):
            self.x.copy_(self.x_host, non_blocking=True)
            self.graph.replay()
            self.red_host.copy_(self.red, non_blocking=True)

    def algorithmic_bytes(self) -> int:
        """This rank's bytes per step: packed weights, fp32 scales, activations
        in, GEMV outputs out (the all-reduce traffic is not counted)."""
        tot = 0
        xe = self.x.element_size()
        for lay in self.layers:
            for m in lay:
                g = m.in_features // m.group_size
                tot += m.out_features * m.in_features // 2 + m.out_features * g * 4
                if m.is_asym:
                    tot += m.out_features * g * 4
                tot += self.tokens * (m.in_features * xe + m.out_features * 4)
        return tot

    def __del__(self):
        for h in getattr(self, "_handles", []):
            try:
                self.lib.sf_q4_step_destroy(h)
            except Exception:
                pass
        self._handles = []


__all__.append("TPStepRunner")
