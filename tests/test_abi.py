"""The C-ABI library loads and exports every symbol include/sf_q4.h declares;
host-side validation runs without a GPU (no kernel is launched)."""
import ctypes
import pathlib
import re

import pytest

from siliconfer_b200 import _lib

HEADER = pathlib.Path(__file__).resolve().parent.parent / "include"


def declared_symbols():
    names = set()
    for h in HEADER.glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(sf_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    syms = declared_symbols()
    assert "sf_q4_gemv_sym" in syms and "sf_q4_linear" in syms
    for s in syms:
        assert hasattr(lib, s), s


def test_every_declared_symbol_has_a_ctypes_signature():
    missing = [s for s in declared_symbols() if s not in _lib.SIGNATURES]
    assert not missing, missing


def test_status_strings():
    lib = _lib.load()
    assert lib.sf_status_string(0) == b"ok"
    assert lib.sf_status_string(2) == b"shape mismatch"
    assert lib.sf_version() >= 10000


FAKE = ctypes.c_void_p(0x1000)  # never dereferenced: validation fails first


@pytest.mark.parametrize("args,msg", [
    ((FAKE, FAKE, None, None, FAKE, 0, FAKE, 0, 8, 96, 1, 64, 0, None), "divisible"),
    ((FAKE, FAKE, None, None, FAKE, 0, FAKE, 0, 8, 128, 1, 3, 0, None), "even"),
    ((None, FAKE, None, None, FAKE, 0, FAKE, 0, 8, 128, 1, 64, 0, None), "null"),
    ((FAKE, FAKE, None, None, FAKE, 7, FAKE, 0, 8, 128, 1, 64, 0, None), "dtype"),
])
def test_linear_validation_without_gpu(args, msg):
    lib = _lib.load()
    rc = lib.sf_q4_linear(*args)
    assert rc != 0
    assert msg in lib.sf_last_error().decode()


def test_asym_entry_requires_zeros():
    lib = _lib.load()
    rc = lib.sf_q4_gemv_asym(FAKE, FAKE, None, FAKE, FAKE, 8, 128, 64, None)
    assert rc == 1
    with pytest.raises(RuntimeError, match="zeros"):
        _lib.check(rc)


def test_empty_problem_is_a_noop():
    lib = _lib.load()
    assert lib.sf_q4_linear(FAKE, FAKE, None, None, FAKE, 0, FAKE, 0, 0, 128, 1, 64, 0, None) == 0
    assert lib.sf_q4_linear(FAKE, FAKE, None, None, FAKE, 0, FAKE, 0, 8, 128, 0, 64, 0, None) == 0


@pytest.mark.parametrize("args,code,msg", [
    # q, qdt, kc, ks, vc, vs, out, odt, B, H, Hkv, T, D, nsplit, ws, wsbytes, stream
    ((None, 0, FAKE, FAKE, FAKE, FAKE, FAKE, 0, 1, 8, 2, 16, 64, 1, FAKE, 1 << 20, None), 1, "null"),
    ((FAKE, 5, FAKE, FAKE, FAKE, FAKE, FAKE, 0, 1, 8, 2, 16, 64, 1, FAKE, 1 << 20, None), 3, "dtype"),
    ((FAKE, 0, FAKE, FAKE, FAKE, FAKE, FAKE, 0, 1, 8, 3, 16, 64, 1, FAKE, 1 << 20, None), 2, "divisible"),
    ((FAKE, 0, FAKE, FAKE, FAKE, FAKE, FAKE, 0, 1, 12, 4, 16, 64, 1, FAKE, 1 << 20, None), 6, "group size"),
    ((FAKE, 0, FAKE, FAKE, FAKE, FAKE, FAKE, 0, 1, 8, 2, 16, 96, 1, FAKE, 1 << 20, None), 6, "head_dim"),
    ((FAKE, 0, FAKE, FAKE, FAKE, FAKE, FAKE, 0, 1, 8, 2, 16, 64, 4, FAKE, 16, None), 2, "workspace"),
])
def test_kv_attention_validation_without_gpu(args, code, msg):
    lib = _lib.load()
    assert lib.sf_kv_attention_decode(*args) == code
    assert msg in lib.sf_last_error().decode()
    assert lib.sf_kv_attention_workspace_bytes(2, 8, 64, 4) == 2 * 8 * 4 * 66 * 4


def test_swiglu_validation_without_gpu():
    lib = _lib.load()
    # N not a multiple of 16
    assert lib.sf_q4_linear_swiglu(FAKE, FAKE, None, None, FAKE, 0, FAKE, 0, 24, 128, 1, 64, None) == 2
    assert "multiple of 16" in lib.sf_last_error().decode()
    assert lib.sf_q4_linear_swiglu(None, FAKE, None, None, FAKE, 0, FAKE, 0, 32, 128, 1, 64, None) == 1
    assert lib.sf_swiglu_interleaved(FAKE, FAKE, 0, 2, 24, None, None) == 2
    assert lib.sf_swiglu_interleaved(FAKE, FAKE, 0, 0, 32, None, None) == 0     # empty: nothing launched


def test_torch_binding_loads_and_checks_devices():
    """The torch binding imports next to libsf_q4.so, exposes both entry
    points, and rejects host tensors before any launch."""
    torch = pytest.importorskip("torch")
    ext = _lib.ext()
    assert callable(ext.linear) and callable(ext.linear_swiglu)
    W = torch.zeros((32, 64), dtype=torch.uint8)
    S = torch.ones((32, 1), dtype=torch.float32)
    X = torch.zeros((1, 128), dtype=torch.float32)
    with pytest.raises(RuntimeError, match="CUDA tensors"):
        ext.linear(W, S, None, None, X, 128, torch.float32)
    with pytest.raises(RuntimeError, match="CUDA tensors"):
        ext.linear_swiglu(W, S, None, None, X, 128, torch.float32)
