"""The C-ABI library loads on a CPU-only machine and exports every symbol its headers declare."""
from __future__ import annotations

import ctypes
import re

import pytest

from conftest import ROOT


def declared_symbols() -> list[str]:
    names = []
    for header in sorted((ROOT / "include").glob("*.h")):
        text = header.read_text()
        names += re.findall(r"NGP_API\s+[\w\s\*]+?\b(ngp_\w+)\s*\(", text)
    return sorted(set(names))


def test_headers_declare_entry_points():
    names = declared_symbols()
    assert "ngp_encode_grid_forward" in names and "ngp_last_error" in names
    assert len(names) >= 5


def test_library_exports_every_declared_symbol(ngp):
    lib = ngp.lib()
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert missing == []


def test_version_and_error_state(ngp):
    assert "sm_100a" in ngp.version()
    with pytest.raises(RuntimeError, match="n_levels"):
        ngp.grid_layout(0, 2, 19, 16, 1.0)
    # the message is per call: a later good call clears it
    ngp.grid_layout(8, 4, 19, 16, 1.0)
    assert ngp.lib().ngp_last_error() == b""


def test_struct_size_matches_header(ngp):
    # 4 u32 + double + 33 u32 + 32 u32 + 32 f32 + 2 u32 (+ alignment padding)
    assert ctypes.sizeof(ngp.GridLayout) == 4 * 4 + 8 + 33 * 4 + 32 * 4 + 32 * 4 + 2 * 4 + 4


def test_loss_scratch_size_refuses_sizes_beyond_32_bits(ngp):
    """The exported scratch size is a uint32: sizes that do not fit are refused (0, error set)
    instead of wrapping to a buffer that is too small."""
    lib = ngp.lib()
    lib.ngp_loss_scratch_bytes.restype = ctypes.c_uint32
    assert lib.ngp_loss_scratch_bytes(ctypes.c_uint32(1 << 18)) > 20 * (1 << 18)
    assert lib.ngp_last_error() == b""
    assert lib.ngp_loss_scratch_bytes(ctypes.c_uint32(0xFFFFFFFF)) == 0
    assert b"uint32" in lib.ngp_last_error()


def test_fault_injection_arguments(ngp):
    """Arming and disarming needs no GPU; bad sites are refused."""
    lib = ngp.lib()
    assert lib.ngp_fault_inject(ctypes.c_int(9), ctypes.c_int64(1)) == 1
    assert b"fault inject" in lib.ngp_last_error()
    ngp.fault_inject("launch", 0)
    ngp.fault_inject("alloc", 0)
