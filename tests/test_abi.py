"""CPU checks of the C ABI: libsemx.so loads, exports every symbol include/semx.h
declares, and its argument structs match the ctypes mirrors (no GPU calls)."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

from semambaxlinoss_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "semx.h"


def _declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(semx_[a-z0-9_]+)\s*\(", text)))


def test_header_and_binding_agree():
    assert _declared_functions() == _lib.declared_symbols()


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in _declared_functions():
        assert hasattr(lib, name), name
    assert lib.semx_abi_version() == _lib.ABI_VERSION


def test_struct_sizes_match():
    lib = _lib.load()
    for name, (cls, query) in _lib.STRUCTS.items():
        assert getattr(lib, query)() == ctypes.sizeof(cls), name


def test_status_strings_and_validation_without_gpu():
    lib = _lib.load()
    assert lib.semx_status_string(0) == b"ok"
    # A struct-size mismatch is rejected before anything touches the device.
    a = _lib.SemxLinossArgs()
    a.struct_size = 3
    assert lib.semx_linoss_fwd(ctypes.byref(a), None) == _lib.SEMX_ERR_ABI
    assert b"struct_size" in lib.semx_last_error()
    # Invalid chunk and missing pointers are rejected on the host.
    a = _lib.new_args(_lib.SemxLinossArgs)
    a.S, a.L, a.P, a.chunk, a.variant = 2, 5, 4, 12, _lib.LINOSS_IMEX
    assert lib.semx_linoss_fwd(ctypes.byref(a), None) == _lib.SEMX_ERR_UNSUPPORTED
    a.chunk = 16
    assert lib.semx_linoss_fwd(ctypes.byref(a), None) == _lib.SEMX_ERR_NULL
    a.variant = 9
    assert lib.semx_linoss_fwd(ctypes.byref(a), None) == _lib.SEMX_ERR_UNSUPPORTED
    b = _lib.new_args(_lib.SemxSelectiveLruArgs)
    b.S, b.L, b.C, b.N, b.chunk = 2, 5, 4, 40, 16
    assert lib.semx_selective_lru_fwd(ctypes.byref(b), None) == _lib.SEMX_ERR_UNSUPPORTED  # N > 32
    b.N, b.chunk = 4, 6
    assert lib.semx_selective_lru_fwd(ctypes.byref(b), None) == _lib.SEMX_ERR_UNSUPPORTED  # chunk
    b.chunk = 8
    assert lib.semx_selective_lru_fwd(ctypes.byref(b), None) == _lib.SEMX_ERR_NULL


def test_size_queries():
    lib = _lib.load()
    assert lib.semx_linoss_ckpt_bytes(404, 321, 256, 64) == 404 * (6 + 1) * 256 * 16
    a = _lib.new_args(_lib.SemxLinossArgs)
    a.S, a.P = 3, 10
    # per-sequence partial rows + one row per group of 32 sequences, 6 sums per oscillator
    assert lib.semx_linoss_workspace_bytes(ctypes.byref(a)) == (3 + 1) * 6 * 10 * 4
    b = _lib.new_args(_lib.SemxSelectiveLruArgs)
    b.S, b.L, b.C, b.N, b.chunk, b.real = 4, 10, 8, 4, 4, 0
    assert lib.semx_selective_lru_ckpt_bytes(ctypes.byref(b)) == 4 * 3 * 8 * 4 * 2 * 4
    b.real = 1
    assert lib.semx_selective_lru_ckpt_bytes(ctypes.byref(b)) == 4 * 3 * 8 * 4 * 4
    # partials (S rows of 4*C*N + C) + group sums (1 row per 32 sequences)
    assert lib.semx_selective_lru_workspace_bytes(ctypes.byref(b)) == (4 + 1) * (4 * 8 * 4 + 8) * 4
