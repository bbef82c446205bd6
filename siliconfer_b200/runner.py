"""Q4StepRunner: a decode step's Q4Linear calls as one persistent launch.

A decode step calls every projection of every layer once (7 per layer,
siliconfer/model/layers.py:93-95, 133, 144).  The reference pays a device
sync and two host copies per call (siliconfer/model/q4_linear.py:51-63).
Here the whole sequence is ONE cooperative kernel launch (sf_q4_step_run,
captured in a CUDA graph): it streams every projection's weights back to back
and waits at a grid barrier only where the decoder has a data dependency --
before o_proj (it consumes attention over q/k/v), before gate/up (they
consume the residual stream after o_proj), before down_proj (SwiGLU of
gate/up) and before the next layer's q/k/v.  q/k/v share their input, as do
gate/up, so they run without a barrier between them.

Inputs and outputs live in two device arenas; ``run_host`` moves a whole
step's activations in with one host->device copy from pinned memory and the
results out with one device->host copy.  Every call still reads its own input
slot: the ops between projections (attention, norms, SwiGLU) are outside
this path, only their ordering is kept.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib
from .kernels import cuda as K
from .q4_linear import Q4Linear

_ESIZE = {torch.float32: 4, torch.float16: 2, torch.bfloat16: 2}


@dataclass
class _Call:
    layer: Q4Linear
    x_off: int   # element offset into the input arena
    y_off: int   # element offset into the output arena


class Q4StepRunner:
    # projection order inside a layer and whether each waits for the previous ones
    LAYER_WAITS = (True, False, False, True, True, False, True)   # q k v o gate up down

    def __init__(self, layers, tokens: int = 1, x_dtype=torch.float16,
                 y_dtype=torch.float32, pdl: bool = True, device=None, waits=None,
                 persistent: bool = True):
        self.layers = list(layers)
        if not self.layers:
            raise ValueError("no layers")
        self.tokens = int(tokens)
        self.x_dtype, self.y_dtype = x_dtype, y_dtype
        self.pdl = pdl
        self.device = torch.device(device) if device is not None else self.layers[0].packed_d.device
        self.calls = []
        xo = yo = 0
        align = 64  # elements: keeps every slot 128-byte aligned
        for m in self.layers:
            self.calls.append(_Call(m, xo, yo))
            xo += -(-self.tokens * m.in_features // align) * align
            yo += -(-self.tokens * m.out_features // align) * align
        self.x = torch.zeros(xo, dtype=x_dtype, device=self.device)
        self.y = torch.zeros(yo, dtype=y_dtype, device=self.device)
        self.x_host = torch.zeros(xo, dtype=x_dtype, pin_memory=True)
        self.y_host = torch.zeros(yo, dtype=y_dtype, pin_memory=True)
        self.graph = None
        self.stream = torch.cuda.Stream(self.device)
        if waits is None:
            waits = [self.LAYER_WAITS[i % 7] if len(self.layers) % 7 == 0 else True
                     for i in range(len(self.layers))]
        self.waits = list(waits)
        self.persistent = persistent
        self._handle = None
        self._workspace = None
        if persistent:
            self._create_step()

    def _create_step(self):
        lib = _lib.load()
        n = len(self.calls)
        arr = (_lib.Q4Task * n)()
        xs, ys = _ESIZE[self.x_dtype], _ESIZE[self.y_dtype]
        xc, yc = K._dtype_code(self.x), K._dtype_code(self.y)
        for i, c in enumerate(self.calls):
            m = c.layer
            arr[i] = _lib.Q4Task(
                m.packed_d.data_ptr(), m.scales_d.data_ptr(),
                None if m.zeros_d is None else m.zeros_d.data_ptr(),
                None if m.bias_d is None else m.bias_d.data_ptr(),
                self.x.data_ptr() + c.x_off * xs, self.y.data_ptr() + c.y_off * ys,
                m.out_features, m.in_features, self.tokens, m.group_size, xc, yc,
                1 if self.waits[i] else 0, 0, getattr(m, "bits", 4))
        nbytes = int(lib.sf_q4_step_workspace_bytes(arr, n))
        self._workspace = torch.zeros(nbytes + 256, dtype=torch.uint8, device=self.device)
        base = self._workspace.data_ptr()
        aligned = (base + 255) & ~255
        h = _lib.ctypes.c_void_p()
        with torch.cuda.device(self.device):
            rc = lib.sf_q4_step_create(arr, n, aligned, nbytes, _lib.ctypes.byref(h))
        if rc != 0:
            # shapes the persistent kernel does not take fall back to one launch per call
            self.persistent = False
            self._workspace = None
            return
        self._handle = h

    def __del__(self):
        if getattr(self, "_handle", None) is not None:
            try:
                _lib.load().sf_q4_step_destroy(self._handle)
            except Exception:
                pass
            self._handle = None

    # -- views -------------------------------------------------------------
    def x_slot(self, i: int, host: bool = False):
        c = self.calls[i]
        buf = self.x_host if host else self.x
        return buf[c.x_off:c.x_off + self.tokens * c.layer.in_features].view(
            self.tokens, c.layer.in_features)

    def y_slot(self, i: int, host: bool = False):
        c = self.calls[i]
        buf = self.y_host if host else self.y
        return buf[c.y_off:c.y_off + self.tokens * c.layer.out_features].view(
            self.tokens, c.layer.out_features)

    @property
    def kernels_per_step(self) -> int:
        """Kernels of this library one step launches: one persistent launch,
        or one GEMV launch per call (pre-pass + GEMV below the prefill size)."""
        return 1 if self.persistent else 2 * len(self.calls)

    def algorithmic_bytes(self) -> int:
        """Bytes one step must move: packed weights, fp32 scales (and zeros),
        activations in and outputs out."""
        tot = 0
        xe, ye = _ESIZE[self.x_dtype], _ESIZE[self.y_dtype]
        for c in self.calls:
            m = c.layer
            g = m.in_features // m.group_size
            tot += m.out_features * m.in_features * getattr(m, "bits", 4) // 8 + m.out_features * g * 4
            if m.is_asym:
                tot += m.out_features * g * 4
            if m.bias_d is not None:
                tot += m.out_features * 4
            tot += self.tokens * (m.in_features * xe + m.out_features * ye)
        return tot

    # -- launches ------------------------------------------------------------
    def _launch_all(self, stream) -> None:
        lib = _lib.load()
        if self.persistent:
            _lib.check(lib.sf_q4_step_run(self._handle, stream.cuda_stream))
            return
        xs = _ESIZE[self.x_dtype]
        ys = _ESIZE[self.y_dtype]
        xc, yc = K._dtype_code(self.x), K._dtype_code(self.y)
        flags = _lib.SF_FLAG_PDL if self.pdl else 0
        xb, yb = self.x.data_ptr(), self.y.data_ptr()
        st = stream.cuda_stream
        for c in self.calls:
            m = c.layer
            fn = lib.sf_q2_linear if getattr(m, "bits", 4) == 2 else None
            if fn is not None:
                _lib.check(fn(m.packed_d.data_ptr(), m.scales_d.data_ptr(),
                              None if m.zeros_d is None else m.zeros_d.data_ptr(),
                              None if m.bias_d is None else m.bias_d.data_ptr(),
                              xb + c.x_off * xs, xc, yb + c.y_off * ys, yc,
                              m.out_features, m.in_features, self.tokens, m.group_size, st))
                continue
            rc = lib.sf_q4_linear(
                m.packed_d.data_ptr(), m.scales_d.data_ptr(),
                None if m.zeros_d is None else m.zeros_d.data_ptr(),
                None if m.bias_d is None else m.bias_d.data_ptr(),
                xb + c.x_off * xs, xc, yb + c.y_off * ys, yc,
                m.out_features, m.in_features, self.tokens, m.group_size, flags, st)
            _lib.check(rc)

    def capture(self) -> None:
        """Warm up once eagerly, then capture the step as a CUDA graph."""
        with torch.cuda.device(self.device):
            self.stream.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self.stream):
                self._launch_all(self.stream)
            self.stream.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=self.stream):
                self._launch_all(self.stream)
            self.graph = g

    def run(self) -> None:
        """One step on the device arenas (asynchronous, on self.stream)."""
        if self.graph is None:
            self.capture()
        with torch.cuda.stream(self.stream):
            self.graph.replay()

    def run_host(self) -> None:
        """One step from pinned host inputs to pinned host outputs."""
        if self.graph is None:
            self.capture()
        with torch.cuda.stream(self.stream):
            self.x.copy_(self.x_host, non_blocking=True)
            self.graph.replay()
            self.y_host.copy_(self.y, non_blocking=True)
