"""Pack a torch decoder's projections into Q4Linear, in place.

Restates siliconfer/engine/q4_loader.py:26-82 for ``torch.nn.Module`` models
that follow the Llama/Qwen naming (``layers[i].self_attn.{q,k,v,o}_proj`` and
``layers[i].mlp.{gate,up,down}_proj``): each projection's weight is re-packed
(``pack_weights_sym`` or ``pack_weights_asym``, chosen by ``pack_sym``) and
replaced by a Q4Linear with its bias.  Projections with
``in_features < group_size`` and layers in ``skip_layers`` are left alone
(q4_loader.py:51-52, 70-72).  ``pack_sym_for_method`` restates the loader's
rule that HQQ always packs asymmetrically (q4_loader.py:183).

``bits_per_block`` serves the reference's mixed precision
(siliconfer/quant/mixed_precision.py:251-319: each decoder block 4 or 2 bits),
which its loader refuses for lack of an int2 kernel (q4_loader.py:142-154):
a 2-bit block's projections are re-fitted on the 2-bit asymmetric grid
(quantize_asym_int2, the grid that method's HQQ output lies on) and served by
Q4Linear(bits=2).
"""
from __future__ import annotations

import numpy as np
import torch

from .q4_linear import Q4Linear
from .quant import pack_weights_asym, pack_weights_int2_asym, pack_weights_sym

PROJECTIONS = (("self_attn", "q_proj"), ("self_attn", "k_proj"), ("self_attn", "v_proj"),
               ("self_attn", "o_proj"), ("mlp", "gate_proj"), ("mlp", "up_proj"),
               ("mlp", "down_proj"))


def pack_sym_for_method(method: str, sym: bool = True) -> bool:
    return False if method == "hqq" else sym


def _pack_and_replace_linears(model, group_size: int = 128, skip_layers=None,
                              pack_sym: bool = True, device=None, bits_per_block=None) -> int:
    """Returns the number of projections replaced."""
    if bits_per_block is not None and len(bits_per_block) != len(model.layers):
        raise ValueError(f"bits_per_block has {len(bits_per_block)} entries, model has {len(model.layers)} layers")
    replaced = 0
    for i, layer in enumerate(model.layers):
        if skip_layers and i in skip_layers:
            continue
        bits = 4 if bits_per_block is None else int(bits_per_block[i])
        if bits not in (2, 4):
            raise ValueError(f"bits_per_block[{i}]={bits} must be 4 or 2")
        for parent_name, name in PROJECTIONS:
            parent = getattr(layer, parent_name)
            lin = getattr(parent, name)
            if isinstance(lin, Q4Linear):
                continue
            in_f = lin.weight.shape[1]
            if in_f < group_size:
                continue
            W = lin.weight.detach().float().cpu().numpy()
            bias = getattr(lin, "bias", None)
            bias = None if bias is None else bias.detach().float()
            dev = device if device is not None else lin.weight.device
            if bits == 2:
                packed, scales, zeros = pack_weights_int2_asym(W, group_size=group_size)
                q = Q4Linear(packed, scales, zeros=zeros, bias=bias, group_size=group_size, device=dev, bits=2)
            elif pack_sym:
                packed, scales = pack_weights_sym(W, group_size=group_size)
                q = Q4Linear(packed, scales, bias=bias, group_size=group_size, device=dev)
            else:
                packed, scales, zeros = pack_weights_asym(W, group_size=group_size)
                q = Q4Linear(packed, scales, zeros=zeros, bias=bias, group_size=group_size,
                             device=dev)
            setattr(parent, name, q)
            replaced += 1
    return replaced


def packed_bytes(model) -> int:
    """Packed weight footprint (restates q4_loader.py:196-212's count)."""
    total = 0
    for m in model.modules():
        if isinstance(m, Q4Linear):
            total += np.asarray(m._packed).nbytes + np.asarray(m._scales).nbytes
            if m._zeros is not None:
                total += np.asarray(m._zeros).nbytes
    return total
