"""Generate tests/golden/golden.npz from the REFERENCE implementation.

Run in a container where the siliconfer reference tree is available:

    SILICONFER_REF=/path/to/siliconfer python tests/golden/make_golden.py

MLX is not needed: a minimal stand-in module is installed in ``sys.modules``
so that the reference's numpy functions import (they only reference MLX at
module level).  Every output below comes from the reference's own functions:
``siliconfer.kernels.neon.{pack_weights_sym, pack_weights_asym, gemv_sym,
gemm_sym, gemm_asym, _numpy_gemv_asym}``, ``siliconfer.quant.primitives.
{quantize_sym, quantize_asym, dequantize_sym, dequantize_asym, unpack_int4,
fake_quantize, quantize_sym_int2, quantize_asym_int2, pack_int2, unpack_int2,
dequantize_sym_int2, dequantize_asym_int2}`` and
``siliconfer.quant.hqq.hqq_quantize_weight``.
"""
from __future__ import annotations

import json
import os
import pathlib
import sys
import types

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import cases as C  # noqa: E402


def _install_mlx_standin() -> None:
    class _Any:
        def __init__(self, *a, **k): pass
        def __call__(self, *a, **k): return _Any()
        def __getattr__(self, n): return _Any()
        def __mro_entries__(self, bases): return (object,)

    for name in ("mlx", "mlx.core", "mlx.nn", "mlx.utils", "mlx.optimizers"):
        m = types.ModuleType(name)
        m.__getattr__ = lambda n: _Any()
        sys.modules[name] = m


def _load_with_numpy_mx(path: pathlib.Path, name: str):
    """Loads one reference module whose mlx.core calls are plain array
    functions (max/abs/where/ones_like/round/clip/astype) with numpy standing
    in for mlx.core, so that the reference's own code computes the vectors."""
    import importlib.util
    shim = types.ModuleType("mlx.core")
    for fn in ("max", "abs", "where", "ones_like", "round", "clip", "float32", "float16", "int8"):
        setattr(shim, fn, getattr(np, fn))
    shim.array = np.ndarray
    shim.Dtype = type(np.float32)
    saved = {k: sys.modules.get(k) for k in ("mlx", "mlx.core")}
    sys.modules["mlx.core"] = shim
    pkg = types.ModuleType("mlx")
    pkg.core = shim
    sys.modules["mlx"] = pkg
    try:
        spec = importlib.util.spec_from_file_location(name, path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
    finally:
        for k, v in saved.items():
            if v is None:
                sys.modules.pop(k, None)
            else:
                sys.modules[k] = v
    return mod


def main() -> None:
    ref = os.environ.get("SILICONFER_REF")
    if not ref:
        sys.exit("set SILICONFER_REF to the root of the siliconfer reference tree")
    _install_mlx_standin()
    sys.path.insert(0, ref)
    from siliconfer.kernels import neon as K
    from siliconfer.quant import primitives as P
    from siliconfer.quant.hqq import hqq_quantize_weight
    assert K._BACKEND == "numpy", "golden vectors come from the reference numpy path"

    out: dict[str, np.ndarray] = {}
    meta: dict[str, object] = {"backend": K._BACKEND, "hashes": {}}

    # --- reference unit-test cases --------------------------------------
    for name in C.UNIT_CASES:
        w, x, gs = C.unit_case(name)
        if C.is_asym(name):
            p, s, z = K.pack_weights_asym(w, gs)
            out[f"{name}/zeros"] = z
            y = np.stack([K._numpy_gemv_asym(p, s, z, xt, gs) for xt in x])
            y2 = K.gemm_asym(p, s, z, x, gs)
            assert np.array_equal(y, y2)
            wq = P.fake_quantize(w, group_size=gs, sym=False)
            out[f"{name}/dequant"] = P.dequantize_asym(
                P.unpack_int4(p.reshape(-1), w.size, signed=False).reshape(w.shape), s, z, gs)
        else:
            p, s = K.pack_weights_sym(w, gs)
            y = K.gemm_sym(p, s, x, gs)
            wq = P.fake_quantize(w, group_size=gs, sym=True)
            out[f"{name}/dequant"] = P.dequantize_sym(
                P.unpack_int4(p.reshape(-1), w.size, signed=True).reshape(w.shape), s, gs)
        if w.size <= 64 * 1024:
            out[f"{name}/packed"] = p
            out[f"{name}/scales"] = s
        else:
            out.pop(f"{name}/dequant")
        meta["hashes"][f"{name}/packed"] = C.sha(p)
        meta["hashes"][f"{name}/scales"] = C.sha(s)
        out[f"{name}/y"] = y.astype(np.float32)
        out[f"{name}/y_fakequant"] = (x @ wq.T).astype(np.float32)

    # --- zero input (test_kernel.py:112-118) --------------------------------
    w = np.random.default_rng(0).normal(0, 1, (32, 128)).astype(np.float32)
    p, s = K.pack_weights_sym(w)
    out["zero_input/y"] = K.gemv_sym(p, s, np.zeros(128, np.float32))

    # --- boundary nibbles -8..7 / 0..15 (test_primitives.py:146-151) --------
    qs = np.arange(-8, 8, dtype=np.int8)
    out["boundary/packed_sym"] = P.pack_int4(qs)
    out["boundary/unpacked_sym"] = P.unpack_int4(out["boundary/packed_sym"], 16, signed=True)
    qa = np.arange(0, 16, dtype=np.uint8)
    out["boundary/packed_asym"] = P.pack_int4(qa)

    # --- config 1: Qwen2.5-0.5B layer, sym RTN, batch 1 ----------------------
    for proj, (n, k) in C.QWEN05B.items():
        w = C.weights(C.layer_seed(1, 0, proj), n, k)
        x = C.acts(C.layer_seed(1, 0, proj) + 7, 1, k)
        p, s = K.pack_weights_sym(w, 128)
        meta["hashes"][f"c1/{proj}/packed"] = C.sha(p)
        meta["hashes"][f"c1/{proj}/scales"] = C.sha(s)
        out[f"c1/{proj}/y"] = K.gemm_sym(p, s, x, 128)

    # --- config 2: Qwen2.5-0.5B layer 0, HQQ asym with a 60 sigma outlier ------
    for proj, (n, k) in C.QWEN05B.items():
        w = C.qwen_asym_weights(0, proj)
        wh = hqq_quantize_weight(w, group_size=128)
        p, s, z = K.pack_weights_asym(wh, 128)
        x = C.acts(C.layer_seed(2, 0, proj) + 7, 1, k)
        meta["hashes"][f"c2/{proj}/hqq"] = C.sha(wh)
        meta["hashes"][f"c2/{proj}/packed"] = C.sha(p)
        meta["hashes"][f"c2/{proj}/scales"] = C.sha(s)
        meta["hashes"][f"c2/{proj}/zeros"] = C.sha(z)
        out[f"c2/{proj}/y"] = K.gemm_asym(p, s, z, x, 128)
        if proj == "down":
            g = C.OUTLIER["col"] // 128
            out["c2/down/outlier_group_scale"] = s[C.OUTLIER["row"], g:g + 1]

    # --- config 3: 7B layer 0 (sym), batch 1 and 4 ----------------------------
    for proj, (n, k) in C.LLAMA7B.items():
        w = C.weights(C.layer_seed(3, 0, proj), n, k)
        p, s = K.pack_weights_sym(w, 128)
        meta["hashes"][f"c3/{proj}/packed"] = C.sha(p)
        meta["hashes"][f"c3/{proj}/scales"] = C.sha(s)
        x = C.acts(C.layer_seed(3, 0, proj) + 7, 4, k)
        out[f"c3/{proj}/y"] = K.gemm_sym(p, s, x, 128)

    # --- config 4: prefill gemm_asym, (K, N) = (4096, 4096), first 4 tokens ----
    w = C.weights(C.layer_seed(4, 0, "q"), 4096, 4096)
    p, s, z = K.pack_weights_asym(w, 128)
    meta["hashes"]["c4/q/packed"] = C.sha(p)
    meta["hashes"]["c4/q/scales"] = C.sha(s)
    meta["hashes"]["c4/q/zeros"] = C.sha(z)
    x = C.acts(C.layer_seed(4, 0, "q") + 7, 4, 4096)
    out["c4/q/y"] = K.gemm_asym(p, s, z, x, 128)

    # --- config 3 at batch 16 (the sweep's largest batch): gate and down ------
    for proj in ("gate", "down"):
        n, k = C.LLAMA7B[proj]
        w = C.weights(C.layer_seed(3, 0, proj), n, k)
        p, s = K.pack_weights_sym(w, 128)
        x = C.acts(C.layer_seed(3, 0, proj) + 7, 16, k)
        out[f"c3b16/{proj}/y"] = K.gemm_sym(p, s, x, 128)

    # --- config 4 on the tensor-core sizes: bf16 activations ----------------------
    # T = 64 on (K, N) = (4096, 4096): every output;  T = 512 on (11008, 4096):
    # every 16th token (the kernel computes all 512)
    for tag, proj, t, keep in (("c4t64", "q", 64, 1), ("c4t512", "down", 512, 16)):
        n, k = C.LLAMA7B[proj]
        w = C.weights(C.layer_seed(4, 0, proj), n, k)
        p, s, z = K.pack_weights_asym(w, 128)
        meta["hashes"][f"{tag}/packed"] = C.sha(p)
        x = C.bf16_round(C.acts(C.layer_seed(4, 0, proj) + 11, t, k))
        out[f"{tag}/y"] = K.gemm_asym(p, s, z, x, 128)[::keep].astype(np.float32)

    # --- config 2 as a 24-layer step (one input per projection, batch 1) ---------
    # layer 0 is the HQQ layer above (60 sigma outlier); layers 1-23 are quantized
    # with the reference's asymmetric RTN packer (the same triple format)
    for layer in range(1, C.QWEN_LAYERS):
        for proj, (n, k) in C.QWEN05B.items():
            w = C.qwen_asym_weights(layer, proj)
            p, s, z = K.pack_weights_asym(w, 128)
            meta["hashes"][f"c2L/{layer}/{proj}/packed"] = C.sha(p)
            x = C.acts(C.layer_seed(2, layer, proj) + 7, 1, k)
            out[f"c2L/{layer}/{proj}/y"] = K.gemm_asym(p, s, z, x, 128)

    # --- 2-bit packing (quantized and packed by the reference, served here) ----
    # The reference has no int2 product; "y" is its own dequant times x.
    for name, (seed, n, k, gs, std) in C.INT2_CASES.items():
        w = C.weights(seed, n, k, std)
        x = C.acts(seed + 7, 3, k)
        if name.startswith("int2_asym"):
            q, s, z = P.quantize_asym_int2(w, gs)
            dq = P.dequantize_asym_int2(P.unpack_int2(P.pack_int2(q), w.size, signed=False).reshape(w.shape), s, z, gs)
            out[f"{name}/zeros"] = z
        else:
            q, s = P.quantize_sym_int2(w, gs)
            dq = P.dequantize_sym_int2(P.unpack_int2(P.pack_int2(q), w.size, signed=True).reshape(w.shape), s, gs)
        out[f"{name}/packed"] = P.pack_int2(q).reshape(n, k // 4)
        out[f"{name}/scales"] = s
        out[f"{name}/dequant"] = dq.astype(np.float32)
        out[f"{name}/y"] = (x.astype(np.float64) @ dq.astype(np.float64).T).astype(np.float32)

    # --- int8 KV cache: the reference's quantize_kv (model/kv_cache.py:49-63)
    # on the inputs of its own attention tests (tests/test_metal_attention.py:
    # _random_inputs with their seeds and shapes)
    kvmod = _load_with_numpy_mx(pathlib.Path(ref) / "siliconfer" / "model" / "kv_cache.py", "ref_kv_cache")
    for name, (seed, B, H, Hkv, D, T) in C.KV_CASES.items():
        rng = np.random.default_rng(seed)
        q = rng.normal(0, 1, (B, H, D)).astype(np.float32)
        k = rng.normal(0, 1, (B, Hkv, T, D)).astype(np.float32)
        v = rng.normal(0, 1, (B, Hkv, T, D)).astype(np.float32)
        kc, ks = kvmod.quantize_kv(k)
        vc, vs = kvmod.quantize_kv(v)
        out[f"{name}/q"] = q
        out[f"{name}/k_codes"] = np.asarray(kc, np.int8)
        out[f"{name}/k_scales"] = np.asarray(ks, np.float32)[..., 0]
        out[f"{name}/v_codes"] = np.asarray(vc, np.int8)
        out[f"{name}/v_scales"] = np.asarray(vs, np.float32)[..., 0]

    np.savez_compressed(HERE / "golden.npz", **out)
    (HERE / "golden_meta.json").write_text(json.dumps(meta, indent=1, sort_keys=True))
    print(f"wrote {len(out)} arrays, {len(meta['hashes'])} hashes")


if __name__ == "__main__":
    main()
