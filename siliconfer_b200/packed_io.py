"""Persistent packed-weight format: save once, load without re-quantizing.

The reference re-quantizes and re-packs every projection on every load
(siliconfer/engine/q4_loader.py:85-193: fake-quantize with RTN/GPTQ/AWQ/HQQ/SINQ,
then ``_pack_and_replace_linears``).  Here the packed triple of every
projection -- ``packed`` uint8 [N, K/2], ``scales`` fp32 [N, G], ``zeros``
fp32 [N, G] (asymmetric layout only) and the optional fp32 ``bias`` -- is
written to one safetensors file, with the group size, layout and producing
method in the file's metadata, so a later load is a file read plus one upload
per projection.  The tensors are stored exactly as the packers produce them
(siliconfer/kernels/neon/__init__.py:42-81), so the round trip is bit-exact.

Tensor names: ``<module name>.packed``, ``.scales``, ``.zeros``, ``.bias``.
"""
from __future__ import annotations

import json

import numpy as np

FORMAT = "siliconfer-q4"
VERSION = "1"


def _host(a, dtype):
    if a is None:
        return None
    if hasattr(a, "detach"):
        a = a.detach().cpu().numpy()
    return np.ascontiguousarray(np.asarray(a, dtype=dtype))


def save_packed(path, layers: dict, group_size: int = 128, method: str = "rtn") -> None:
    """Write ``{name: Q4Linear | (packed, scales, zeros[, bias])}`` to ``path``."""
    from safetensors.numpy import save_file
    tensors, layouts = {}, {}
    for name, m in layers.items():
        if isinstance(m, tuple):
            packed, scales, zeros = m[0], m[1], m[2]
            bias = m[3] if len(m) > 3 else None
            gs = group_size
        else:
            packed, scales, zeros, bias, gs = m._packed, m._scales, m._zeros, m.bias, m.group_size
        if gs != group_size:
            raise ValueError(f"{name}: group_size {gs} differs from the file's {group_size}")
        p = _host(packed, np.uint8)
        s = _host(scales, np.float32)
        if p.ndim != 2 or s.ndim != 2 or s.shape[0] != p.shape[0] or s.shape[1] * group_size != 2 * p.shape[1]:
            raise ValueError(f"{name}: packed {p.shape} and scales {s.shape} do not match group_size {group_size}")
        tensors[f"{name}.packed"] = p
        tensors[f"{name}.scales"] = s
        if zeros is not None:
            z = _host(zeros, np.float32)
            if z.shape != s.shape:
                raise ValueError(f"{name}: zeros {z.shape} must match scales {s.shape}")
            tensors[f"{name}.zeros"] = z
        if bias is not None:
            tensors[f"{name}.bias"] = _host(bias, np.float32)
        layouts[name] = "asym" if zeros is not None else "sym"
    meta = {"format": FORMAT, "version": VERSION, "group_size": str(group_size), "method": method,
            "layouts": json.dumps(layouts, sort_keys=True)}
    save_file(tensors, str(path), metadata=meta)


def load_packed(path):
    """Read a file written by ``save_packed``: (triples, meta).

    ``triples[name] = (packed, scales, zeros or None, bias or None)`` as numpy
    arrays; ``meta`` has ``group_size`` (int), ``method`` and ``layouts``."""
    from safetensors import safe_open
    with safe_open(str(path), framework="numpy") as f:
        meta = f.metadata() or {}
        if meta.get("format") != FORMAT:
            raise ValueError(f"{path}: not a {FORMAT} file")
        if meta.get("version") != VERSION:
            raise ValueError(f"{path}: format version {meta.get('version')} is not {VERSION}")
        layouts = json.loads(meta["layouts"])
        keys = set(f.keys())
        out = {}
        for name, layout in layouts.items():
            p = f.get_tensor(f"{name}.packed")
            s = f.get_tensor(f"{name}.scales")
            z = f.get_tensor(f"{name}.zeros") if f"{name}.zeros" in keys else None
            b = f.get_tensor(f"{name}.bias") if f"{name}.bias" in keys else None
            if (z is None) != (layout == "sym"):
                raise ValueError(f"{path}: {name} is marked {layout} but zeros are "
                                 f"{'absent' if z is None else 'present'}")
            out[name] = (p, s, z, b)
    return out, {"group_size": int(meta["group_size"]), "method": meta.get("method"), "layouts": layouts}


def save_q4_model(model, path, method: str = "rtn") -> int:
    """Save every Q4Linear of ``model`` (by module name); returns how many."""
    from .q4_linear import Q4Linear
    layers = {n: m for n, m in model.named_modules() if isinstance(m, Q4Linear)}
    if not layers:
        raise ValueError("model has no Q4Linear modules")
    gs = {m.group_size for m in layers.values()}
    if len(gs) != 1:
        raise ValueError(f"mixed group sizes {sorted(gs)}")
    save_packed(path, layers, group_size=gs.pop(), method=method)
    return len(layers)


def load_q4_model(model, path, device=None) -> int:
    """Replace the projections named in ``path`` by Q4Linear modules built from
    the stored triples (no quantization); returns how many were replaced."""
    from .q4_linear import Q4Linear
    triples, meta = load_packed(path)
    n = 0
    for name, (p, s, z, b) in triples.items():
        parent_name, _, attr = name.rpartition(".")
        parent = model.get_submodule(parent_name) if parent_name else model
        setattr(parent, attr, Q4Linear(p, s, zeros=z, bias=b, group_size=meta["group_size"], device=device))
        n += 1
    return n


__all__ = ["save_packed", "load_packed", "save_q4_model", "load_q4_model"]
