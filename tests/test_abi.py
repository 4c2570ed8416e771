"""CPU checks of the C ABI boundary: the library loads, exports every symbol the
public headers declare, keeps the reference's View layout, and validates
arguments before touching the GPU."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_c_functions():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        txt = h.read_text()
        names |= set(re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*(af_[a-z0-9_]+)\s*\(", txt, re.M))
        names |= set(re.findall(r'extern "C" int (af_[a-z0-9_]+)\(', txt))
    return names


def test_library_loads_and_exports_every_declared_symbol():
    from atomflow_b200._lib import C_SYMBOLS, CXX_SYMBOLS, lib
    L = lib()
    declared = declared_c_functions()
    assert {"af_w8a16_gemv", "af_lm_head_gemv", "af_argmax_f32"} <= declared
    for name in declared:
        assert hasattr(L, name), name
    assert declared == set(C_SYMBOLS), declared ^ set(C_SYMBOLS)
    for _, (mangled, _, _) in CXX_SYMBOLS.items():
        assert hasattr(L, mangled)
    hdr = (ROOT / "include" / "atomflow_view_ops.h").read_text()
    for name in CXX_SYMBOLS:
        assert f"void {name}(" in hdr


def test_view_layout_is_the_reference_layout():
    from atomflow_b200._lib import View
    assert ctypes.sizeof(View) == 56
    assert View.data_ptr.offset == 8 and View.dims.offset == 16
    assert View.strides.offset == 32 and View.num_dims.offset == 48


def test_status_strings_and_version():
    from atomflow_b200._lib import lib
    L = lib()
    assert L.af_version() >= 100
    assert L.af_status_string(0) == b"ok"
    assert L.af_status_string(5).startswith(b"workspace")


def test_argument_validation_needs_no_gpu():
    """These return before any CUDA call, so they run on a CPU-only machine."""
    from atomflow_b200._lib import lib
    L = lib()
    # group scales with group_size != 128, or K not a multiple of 128
    assert L.af_w8a16_gemv(1, 1, 1, 1, 1, 16, 256, 64, 0, None, 0, None) == 1
    assert L.af_w8a16_gemv(1, 1, 1, 1, 1, 16, 200, 128, 0, None, 0, None) == 1
    # unscaled kind with a scale pointer; unknown kind; negative sizes
    assert L.af_w8a16_gemv(1, 1, 1, 1, 1, 16, 256, 128, 2, None, 0, None) == 1
    assert L.af_w8a16_gemv(1, 1, 1, 1, 1, 16, 256, 128, 9, None, 0, None) == 1
    assert L.af_w8a16_gemv(1, 1, 1, 1, -1, 16, 256, 128, 0, None, 0, None) == 1
    # empty problems are a no-op
    assert L.af_w8a16_gemv(None, None, None, None, 0, 16, 256, 128, 0, None, 0, None) == 0
    assert L.af_w8a16_gemv(None, None, None, None, 1, 0, 256, 128, 0, None, 0, None) == 0
    # lm_head: fp16 weights take no row scale, fp8 weights need one, bad mode
    assert L.af_lm_head_gemv(1, 1, 0, 1, 1, 8, 64, None, 0, None, 0, None) == 1
    assert L.af_lm_head_gemv(1, 1, 1, None, 1, 8, 64, None, 0, None, 0, None) == 1
    assert L.af_lm_head_gemv(1, 1, 0, None, 1, 8, 64, None, 7, None, 0, None) == 1
    assert L.af_argmax_f32(None, 10, None, 0, None, 0, None) == 1


def test_python_ops_fail_loudly_without_library(monkeypatch, tmp_path):
    from atomflow_b200 import _lib
    monkeypatch.setattr(_lib, "_LIB_PATH", tmp_path / "missing.so")
    monkeypatch.setattr(_lib, "_lib", None)
    with pytest.raises(ImportError):
        _lib.lib()


def test_tp_buffer_holds_partials_and_row_epochs():
    """The exchange buffer of the fused all-reduce: a 1280-byte header (status,
    lm_head argmax pairs), partials [2 parity halves][8 source ranks][max_n] as
    64-bit words, then one 32-bit epoch per row (rounded to 16 bytes) -- the
    per-row epochs keep every row's tag alternating whatever grid a launch uses."""
    from atomflow_b200._lib import lib
    L = lib()
    for n in (1, 64, 3072, 4097):
        assert L.af_tp_buffer_bytes(n) == 1280 + 256 + 2 * 8 * n * 8 + ((n * 4 + 15) // 16) * 16
    assert L.af_tp_buffer_bytes(0) == 0
