"""Q4StepRunner: a decode step's Q4Linear calls captured once as a CUDA graph.

A decode step calls every projection of every layer once (7 per layer,
siliconfer/model/layers.py:93-95, 133, 144).  The reference pays a device
sync and two host copies per call (siliconfer/model/q4_linear.py:51-63); here
the whole sequence is one graph replay whose launches are chained with
programmatic dependent launch, so each GEMV starts streaming its weights while
the previous one finishes.  Inputs and outputs live in two device arenas;
``run_host`` moves a whole step's activations in with one host->device copy
from pinned memory and the results out with one device->host copy.

The runner treats every call as reading its own input slot: the data flow
between projections (attention, SwiGLU) is outside this path.
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
    def __init__(self, layers, tokens: int = 1, x_dtype=torch.float16,
                 y_dtype=torch.float32, pdl: bool = True, device=None):
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
        return len(self.calls)

    def algorithmic_bytes(self) -> int:
        """Bytes one step must move: packed weights, fp32 scales (and zeros),
        activations in and outputs out."""
        tot = 0
        xe, ye = _ESIZE[self.x_dtype], _ESIZE[self.y_dtype]
        for c in self.calls:
            m = c.layer
            g = m.in_features // m.group_size
            tot += m.out_features * m.in_features // 2 + m.out_features * g * 4
            if m.is_asym:
                tot += m.out_features * g * 4
            if m.bias_d is not None:
                tot += m.out_features * 4
            tot += self.tokens * (m.in_features * xe + m.out_features * ye)
        return tot

    # -- launches ------------------------------------------------------------
    def _launch_all(self, stream) -> None:
        lib = _lib.load()
        xs = _ESIZE[self.x_dtype]
        ys = _ESIZE[self.y_dtype]
        xc, yc = K._dtype_code(self.x), K._dtype_code(self.y)
        flags = _lib.SF_FLAG_PDL if self.pdl else 0
        xb, yb = self.x.data_ptr(), self.y.data_ptr()
        st = stream.cuda_stream
        for c in self.calls:
            m = c.layer
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
