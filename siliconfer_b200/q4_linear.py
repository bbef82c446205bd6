"""Q4Linear: drop-in int4 weight-only linear layer backed by the sm_100a kernels.

Restates siliconfer/model/q4_linear.py:12-68 as a ``torch.nn.Module``:

* same constructor ``Q4Linear(packed, scales, zeros=None, bias=None,
  group_size=128)`` and the same host attributes ``_packed``, ``_scales``,
  ``_zeros``, ``bias``, ``group_size``, ``out_features``, ``in_features``, so the
  packed triples produced by RTN/GPTQ/AWQ/HQQ/SINQ load unchanged;
* ``zeros is None`` selects the symmetric kernel, otherwise the asymmetric one
  (q4_linear.py:58-61);
* ``forward(x[..., K]) -> y[..., N]``, bias added after the product
  (q4_linear.py:63-66).

``bits=2`` serves the reference's 2-bit packing (pack_int2,
siliconfer/quant/primitives.py:383-404: ``packed`` is [N, K/4]), which the
reference quantizes but cannot serve (siliconfer/engine/q4_loader.py:142-154).

Differences that follow from the hardware: the triple is uploaded to the GPU
once at construction (device buffers ``packed_d``, ``scales_d``, ``zeros_d``);
activations stay on the GPU (no per-call host sync or copy, unlike
q4_linear.py:51-55); fp16/bf16 activations are read directly and accumulated
in fp32.  The output is fp32 like the reference unless ``out_dtype`` is set.
"""
from __future__ import annotations

import numpy as np
import torch

from .kernels import cuda as K


def _host_array(a, dtype):
    if a is None:
        return None
    if isinstance(a, torch.Tensor):
        return a.detach().cpu().numpy().astype(dtype, copy=False)
    return np.asarray(a, dtype=dtype)


class Q4Linear(torch.nn.Module):
    def __init__(self, packed, scales, zeros=None, bias=None, group_size: int = 128,
                 device=None, out_dtype=None, bits: int = 4):
        super().__init__()
        if bits not in (2, 4):
            raise RuntimeError("bits must be 4 or 2")
        self._packed = packed
        self._scales = scales
        self._zeros = zeros
        self.bits = int(bits)
        self.group_size = int(group_size)
        self.out_features = int(packed.shape[0])
        self.in_features = int(packed.shape[1]) * (8 // self.bits)
        self.out_dtype = out_dtype
        K._check_weights(packed, scales, self.group_size, zeros, bits=self.bits)
        if self.in_features % self.group_size:
            raise RuntimeError("in_features must be divisible by group_size")
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() \
                else torch.device("cpu")
        dev = torch.device(device)

        def up(a, dt):
            if a is None:
                return None
            if isinstance(a, torch.Tensor):
                return a.detach().to(device=dev, dtype=dt).contiguous()
            return torch.from_numpy(np.ascontiguousarray(a)).to(device=dev, dtype=dt)

        self.register_buffer("packed_d", up(packed, torch.uint8), persistent=False)
        self.register_buffer("scales_d", up(scales, torch.float32), persistent=False)
        self.register_buffer("zeros_d", up(zeros, torch.float32), persistent=False)
        self.register_buffer("bias_d", up(bias, torch.float32), persistent=False)
        self.bias = bias
        self.pdl = False   # set by callers that chain many projections in one stream

    @property
    def is_asym(self) -> bool:
        return self._zeros is not None

    def forward(self, x):
        host = not isinstance(x, torch.Tensor)
        xt = torch.from_numpy(np.asarray(x, np.float32)) if host else x
        orig = xt.shape
        if orig[-1] != self.in_features:
            raise RuntimeError("X/W in_features mismatch")
        xt = xt.reshape(-1, self.in_features).to(self.packed_d.device)
        if xt.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            xt = xt.float()
        xt = xt.contiguous()
        y = K.linear(self.packed_d, self.scales_d, self.zeros_d, xt, self.group_size,
                     bias=self.bias_d, out_dtype=self.out_dtype, pdl=self.pdl, bits=self.bits)
        y = y.reshape(*orig[:-1], self.out_features)
        return y.cpu().numpy() if host else y

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"group_size={self.group_size}, bits={self.bits}, {'asym' if self.is_asym else 'sym'}, "
                f"bias={self.bias is not None}")
