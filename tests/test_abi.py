"""CPU checks of the drop-in boundary: libhs_ext.so builds for sm_100a, loads
without a GPU, and exports every entry point include/hs_ext.h declares with
the ctypes signatures the Python host layer binds."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent


def header_functions() -> list[str]:
    text = (REPO / "include" / "hs_ext.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(hs_[a-z0-9_]+)\s*\(", text)))


def test_library_builds_and_loads():
    from home_seek_b200 import _lib, build
    build.build()
    lib = _lib.load()
    assert lib.hs_abi_version() == 2
    assert lib.hs_status_string(3) == b"workspace too small"
    assert lib.hs_trace_buffer(0) is None  # the normal build carries no phase stamps


def test_every_declared_symbol_is_exported_and_bound():
    from home_seek_b200 import _lib
    lib = _lib.load()
    declared = header_functions()
    assert len(declared) >= 14
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in hs_ext.h but not exported"
        assert name in _lib.SIGNATURES, f"{name} not bound in _lib.SIGNATURES"
    assert set(_lib.SIGNATURES) == set(declared)


def test_host_side_argument_checks_without_gpu():
    """Shape / argument validation happens before any CUDA call."""
    from home_seek_b200 import _lib
    lib = _lib.load()
    # T = 0 is a no-op, bad shapes are rejected, sizes are reported
    assert lib.hs_router_topk(None, None, None, 0, 4096, 256, 6, 1.5, None, None, None, None, 0, None) == 0
    assert lib.hs_router_topk(None, None, None, 3, 4000, 256, 6, 1.5, None, None, None, None, 0, None) == 1
    assert lib.hs_router_workspace_size(3, 4096, 256) >= 8 * 3 * 256 * 4
    assert lib.hs_moe_workspace_size(3, 6, 4096, 2048, 2048) > 21 * 4096 * 4
    assert lib.hs_accept_greedy(None, 1, 3, 100, None, None, None, None, None, None) == 1  # V*2 % 16 != 0
    assert lib.hs_hash_route(None, 0, None, 10, 6, None, None, None, None) == 0
    w = _lib.hs_moe_weights()
    w.E, w.D, w.I, w.I_sh = 256, 4000, 2048, 2048
    buf = (ctypes.c_uint8 * 1024)()
    assert lib.hs_moe_make_desc(ctypes.byref(w), buf, 1024) == 1
    assert lib.hs_fill_bytes(None, 16, 0, 5, 2, None) == 2


def test_no_cpu_fallback():
    import torch
    from home_seek_b200 import ops
    with pytest.raises(ValueError, match="CUDA"):
        ops.router_topk(torch.zeros(3, 512, dtype=torch.bfloat16), torch.zeros(16, 512, dtype=torch.bfloat16), None)
