"""C-ABI library: it loads, exports every declared symbol, and rejects bad
arguments before touching a GPU (no compute calls here)."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from sm90_fp8_wgrad import _lib

ROOT = Path(__file__).resolve().parents[1]


def _declared_symbols() -> list[str]:
    names = []
    for header in sorted((ROOT / "include").glob("*.h")):
        text = header.read_text()
        names += re.findall(r"SM100_WGRAD_API\s+[\w\s\*]+?\b(\w+)\s*\(", text)
    return sorted(set(names))


def test_header_declares_expected_symbols():
    assert set(_declared_symbols()) >= set(_lib.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in _declared_symbols():
        assert hasattr(lib, name), f"{name} declared in include/ but not exported by {_lib.library_path()}"


def test_version_and_status_strings():
    assert re.fullmatch(r"\d+\.\d+\.\d+", _lib.version())
    assert _lib.status_string(_lib.OK) == "ok"
    for code in range(1, 7):
        assert _lib.status_string(code) != "unknown status"
    assert _lib.status_string(99) == "unknown status"


def test_struct_layout_matches_header():
    # 21 fields: 9 pointers, 8 int64, 4 int32 (+ padding): offsets fixed by the C ABI
    assert ctypes.sizeof(_lib.Sm100WgradArgs) == 9 * 8 + 8 * 8 + 4 * 4
    assert _lib.Sm100WgradArgs.max_ctas.offset == ctypes.sizeof(_lib.Sm100WgradArgs) - 20
    assert _lib.Sm100WgradArgs.workspace.offset == ctypes.sizeof(_lib.Sm100WgradArgs) - 16
    assert _lib.Sm100WgradArgs.workspace_bytes.offset == ctypes.sizeof(_lib.Sm100WgradArgs) - 8
    assert ctypes.sizeof(_lib.Sm100WgradMetaOut) == 14 * 8
    # Sm100WgradQuantArgs: 18 eight-byte slots (int32 fields padded to 8)
    assert ctypes.sizeof(_lib.Sm100WgradQuantArgs) == 18 * 8
    assert _lib.Sm100WgradQuantArgs.block_rows.offset == 15 * 8
    assert _lib.Sm100WgradQuantArgs.x_rows.offset == 16 * 8
    assert _lib.Sm100WgradQuantArgs.scale_format.offset == 17 * 8


def test_invalid_arguments_rejected_without_gpu():
    lib = _lib.load()
    assert lib.sm100_fp8_grouped_wgrad(None, None) == _lib.ERR_INVALID_ARG
    a = _lib.Sm100WgradArgs()
    assert lib.sm100_fp8_grouped_wgrad(ctypes.byref(a), None) == _lib.ERR_INVALID_ARG  # null out / metadata
    a.out = 256
    a.block_offsets = 256
    a.k_row_offsets = 256
    a.m, a.n, a.num_experts = 64, 24, 1                                                  # N % 16 != 0
    assert lib.sm100_fp8_grouped_wgrad(ctypes.byref(a), None) == _lib.ERR_UNSUPPORTED
    a.n = 32
    a.out_dtype = 7
    assert lib.sm100_fp8_grouped_wgrad(ctypes.byref(a), None) == _lib.ERR_INVALID_ARG
    a.out_dtype = 0
    a.k_rows, a.total_blocks = 128, 1                                                   # operands missing
    assert lib.sm100_fp8_grouped_wgrad(ctypes.byref(a), None) == _lib.ERR_INVALID_ARG
    a.lhs_data = a.rhs_data = a.lhs_scales = a.rhs_scales = 256
    a.lhs_pitch = a.rhs_pitch = 120                                                     # pitch % 16
    assert lib.sm100_fp8_grouped_wgrad(ctypes.byref(a), None) == _lib.ERR_INVALID_ARG
    assert lib.sm100_wgrad_quantize_1x128(None, 5, 1, 1, None, None, 1, None, 128, None, None) == _lib.ERR_INVALID_ARG
    assert lib.sm100_wgrad_build_meta(None, 1, None, None) == _lib.ERR_INVALID_ARG


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setenv("SM100_WGRAD_LIB", str(tmp_path / "absent.so"))
    monkeypatch.setattr(_lib, "_lib", None)
    with pytest.raises(RuntimeError, match="not found"):
        _lib.load()


def test_profile_counters_unsupported_in_product_build():
    """The product library has no timing code: the counter read reports
    SM100_WGRAD_ERR_UNSUPPORTED (no CUDA call is made)."""
    assert _lib.profile_counters() is None


def test_sm90_only_kernel_modes_rejected(monkeypatch):
    """KERNEL_LAB_WGRAD_KERNEL_MODE values that select SM90 kernel variants are
    refused before anything touches the GPU."""
    from sm90_fp8_wgrad import fp8_grouped_wgrad_sm90

    monkeypatch.setenv("KERNEL_LAB_WGRAD_KERNEL_MODE", "tma_only")
    with pytest.raises(RuntimeError, match="no B200 counterpart"):
        fp8_grouped_wgrad_sm90(None, None, None, None)
