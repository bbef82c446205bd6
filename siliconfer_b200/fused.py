"""Same-input projections as one Q4Linear.

q/k/v read the same normed hidden state (siliconfer/model/layers.py:93-95) and
so do gate/up (layers.py:144).  Stacking their packed rows, scales, zeros and
biases gives one GEMV over N = sum of the parts: the input is read and
converted once, one kernel task replaces two or three, and every output row
is computed with the same per-group arithmetic as before (a row does not
depend on the other rows); only the decode kernel's k-split, which is chosen
from N, may change the fp32 summation order.

``SwiGLUQ4Linear`` goes one step further for gate/up: the rows are
interleaved so that each 32-row tile of the decode kernel holds 16 gate rows
and the matching 16 up rows, and the kernel's epilogue writes
silu(gate) * up -- down_proj's input -- instead of the two projections.
"""
from __future__ import annotations

import numpy as np

from .q4_linear import Q4Linear


def _np(a, dt):
    if a is None:
        return None
    if hasattr(a, "detach"):
        a = a.detach().cpu().numpy()
    return np.asarray(a, dtype=dt)


class FusedQ4Linear:
    """``FusedQ4Linear([q, k, v])(x) -> (y_q, y_k, y_v)`` with one GEMV."""

    def __init__(self, layers, device=None):
        layers = list(layers)
        if len(layers) < 2:
            raise ValueError("need at least two projections")
        gs = {m.group_size for m in layers}
        kin = {m.in_features for m in layers}
        asym = {m.is_asym for m in layers}
        if len(gs) != 1 or len(kin) != 1 or len(asym) != 1:
            raise ValueError("fused projections need the same in_features, group_size and layout")
        self.splits = [m.out_features for m in layers]
        packed = np.concatenate([_np(m._packed, np.uint8) for m in layers])
        scales = np.concatenate([_np(m._scales, np.float32) for m in layers])
        zeros = np.concatenate([_np(m._zeros, np.float32) for m in layers]) if asym.pop() else None
        if any(m.bias is not None for m in layers):
            bias = np.concatenate([_np(m.bias, np.float32) if m.bias is not None
                                   else np.zeros(m.out_features, np.float32) for m in layers])
        else:
            bias = None
        if device is None:
            device = layers[0].packed_d.device
        self.layer = Q4Linear(packed, scales, zeros=zeros, bias=bias, group_size=gs.pop(), device=device,
                              out_dtype=layers[0].out_dtype)

    def __call__(self, x):
        y = self.layer(x)
        out, o = [], 0
        for n in self.splits:
            out.append(y[..., o:o + n])
            o += n
        return tuple(out)


def interleave_gate_up(gate, up, block: int = 16):
    """Rows of two [N, ...] arrays interleaved in blocks of `block`: rows
    2*block*i .. +block-1 are gate rows block*i .., the next `block` the same
    up rows (the layout sf_q4_linear_swiglu reads).  None stays None."""
    if gate is None and up is None:
        return None
    gate, up = np.asarray(gate), np.asarray(up)
    if gate.shape != up.shape or gate.shape[0] % block:
        raise ValueError(f"gate/up need the same shape with rows a multiple of {block}")
    n = gate.shape[0]
    rest = gate.shape[1:]
    return np.ascontiguousarray(np.stack([gate.reshape(n // block, block, *rest),
                                          up.reshape(n // block, block, *rest)], axis=1).reshape(2 * n, *rest))


class SwiGLUQ4Linear:
    """``SwiGLUQ4Linear(gate, up)(x) -> silu(gate(x)) * up(x)``: the MLP input
    of down_proj (siliconfer/model/layers.py:144) from ONE GEMV over the
    interleaved gate/up rows, the activation fused into its epilogue.

    Decode sizes (up to 16 tokens) run sf_q4_linear_swiglu; larger batches run
    the stacked GEMM (sf_q4_linear) and then sf_swiglu_interleaved, both on
    the GPU.  ``out_dtype`` defaults to fp32."""

    def __init__(self, gate, up, device=None, out_dtype=None):
        import torch
        if gate.group_size != up.group_size or gate.in_features != up.in_features \
                or gate.out_features != up.out_features or gate.is_asym != up.is_asym:
            raise ValueError("gate and up need the same shape, group_size and layout")
        if gate.out_features % 16:
            raise ValueError("gate/up out_features must be a multiple of 16")
        self.out_features = gate.out_features
        self.in_features = gate.in_features
        self.group_size = gate.group_size
        bias = None
        if gate.bias is not None or up.bias is not None:
            z = np.zeros(self.out_features, np.float32)
            bias = interleave_gate_up(_np(gate.bias, np.float32) if gate.bias is not None else z,
                                      _np(up.bias, np.float32) if up.bias is not None else z)
        zeros = interleave_gate_up(_np(gate._zeros, np.float32), _np(up._zeros, np.float32)) \
            if gate.is_asym else None
        if device is None:
            device = gate.packed_d.device
        self.layer = Q4Linear(interleave_gate_up(_np(gate._packed, np.uint8), _np(up._packed, np.uint8)),
                              interleave_gate_up(_np(gate._scales, np.float32), _np(up._scales, np.float32)),
                              zeros=zeros, bias=None, group_size=self.group_size, device=device)
        self.bias_d = None if bias is None else torch.from_numpy(bias).to(device)
        self.out_dtype = out_dtype or torch.float32

    def __call__(self, x):
        import torch
        from . import _lib
        from .kernels.cuda import _dtype_code, _require_cuda
        _require_cuda()
        L = self.layer
        orig = x.shape
        xt = x.reshape(-1, self.in_features).to(L.packed_d.device)
        if xt.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            xt = xt.float()
        xt = xt.contiguous()
        T, N = xt.shape[0], self.out_features
        y = torch.empty((T, N), dtype=self.out_dtype, device=xt.device)
        st = torch.cuda.current_stream(xt.device).cuda_stream
        lib = _lib.load()
        zp = None if L.zeros_d is None else L.zeros_d.data_ptr()
        bp = None if self.bias_d is None else self.bias_d.data_ptr()
        rc = lib.sf_q4_linear_swiglu(L.packed_d.data_ptr(), L.scales_d.data_ptr(), zp, bp, xt.data_ptr(),
                                     _dtype_code(xt), y.data_ptr(), _dtype_code(y), N, self.in_features, T,
                                     self.group_size, st)
        if rc == 6:   # SF_ERR_UNSUPPORTED: not a decode size -- stacked GEMM, then the activation
            tmp = torch.empty((T, 2 * N), dtype=torch.float32, device=xt.device)
            _lib.check(lib.sf_q4_linear(L.packed_d.data_ptr(), L.scales_d.data_ptr(), zp, None, xt.data_ptr(),
                                        _dtype_code(xt), tmp.data_ptr(), _lib.SF_F32, 2 * N, self.in_features,
                                        T, self.group_size, 0, st))
            _lib.check(lib.sf_swiglu_interleaved(tmp.data_ptr(), y.data_ptr(), _dtype_code(y), T, N, bp, st))
        else:
            _lib.check(rc)
        return y.reshape(*orig[:-1], N)


__all__ = ["FusedQ4Linear", "SwiGLUQ4Linear", "interleave_gate_up"]
