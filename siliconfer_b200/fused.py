"""Same-input projections as one Q4Linear.

q/k/v read the same normed hidden state (siliconfer/model/layers.py:93-95) and
so do gate/up (layers.py:144).  Stacking their packed rows, scales, zeros and
biases gives one GEMV over N = sum of the parts: the input is read and
converted once, one kernel task replaces two or three, and every output row
is computed with the same per-group arithmetic as before (a row does not
depend on the other rows); only the decode kernel's k-split, which is chosen
from N, may change the fp32 summation order.
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


__all__ = ["FusedQ4Linear"]
