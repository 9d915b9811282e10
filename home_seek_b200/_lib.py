"""ctypes binding of libhs_ext.so (the C ABI declared in include/hs_ext.h).

This is exactly the stub a maintainer of the reference would add to call the
kernels from Python: plain pointers, int64 shapes, a cudaStream_t as void*, and
an int status turned into a Python exception (HsError), so the reference
engine's try/except fallback semantics are kept.

There is no CPU fallback: if the library cannot be loaded, every entry point
raises.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_float, c_int, c_int32, c_int64, c_size_t, c_uint64, c_void_p
from pathlib import Path

# HS_LIB_PATH: another build of the library (a tracing or a modified build);
# HS_TRACE=1: the tracing build next to this file
_LIB_PATH = Path(os.environ["HS_LIB_PATH"]).resolve() if os.environ.get("HS_LIB_PATH") else \
    Path(__file__).resolve().parent / ("libhs_ext_trace.so" if os.environ.get("HS_TRACE") == "1" else "libhs_ext.so")

HS_OK = 0
STATUS_NAMES = {0: "HS_OK", 1: "HS_ERR_BAD_SHAPE", 2: "HS_ERR_BAD_ARGUMENT", 3: "HS_ERR_WORKSPACE",
                4: "HS_ERR_ALIGN", 5: "HS_ERR_CUDA", 6: "HS_ERR_UNSUPPORTED", 7: "HS_ERR_NCCL"}
HS_DEV_BAD_EXPERT = 0x1
HS_DEV_BAD_TOKEN = 0x2
HS_DEV_TIMEOUT = 0x4
HS_DEV_BAD_DRAFT = 0x8
HS_DEV_SMEM_ALIGN = 0x10
HS_MOE_DESC_BYTES = 1024
HS_MOE_NOALLOC_BYTES = 16 << 20
HS_DUP_LAST = 0
HS_DUP_SUM = 1
HS_EP_MAX_RANKS = 8
HS_IPC_HANDLE_BYTES = 64
HS_NCCL_UNIQUE_ID_BYTES = 128


class HsEpPeers(ctypes.Structure):
    """hs_ep_peers: this rank, the group size, and every rank's receive buffer
    as mapped in this process (recv[rank] is the local buffer)."""
    _fields_ = [("rank", c_int32), ("world", c_int32), ("recv", c_void_p * HS_EP_MAX_RANKS),
                ("wait_limit_ns", c_int64)]


class HsError(RuntimeError):
    """A non-zero hs_status returned by the CUDA library."""

    def __init__(self, fn: str, status: int, cuda_error: int = 0):
        self.status = status
        self.cuda_error = cuda_error
        msg = f"{fn} failed: {STATUS_NAMES.get(status, status)}"
        if cuda_error:
            msg += f" (cuda error {cuda_error})"
        super().__init__(msg)


class hs_moe_weights(ctypes.Structure):
    _fields_ = [("w13", c_void_p), ("s13", c_void_p), ("w2", c_void_p), ("s2", c_void_p),
                ("sh_w13", c_void_p), ("sh_s13", c_void_p), ("sh_w2", c_void_p), ("sh_s2", c_void_p),
                ("E", c_int64), ("D", c_int64), ("I", c_int64), ("I_sh", c_int64)]


# name -> (restype, argtypes); kept in the order of include/hs_ext.h
SIGNATURES = {
    "hs_abi_version": (c_int, []),
    "hs_status_string": (ctypes.c_char_p, [c_int]),
    "hs_last_cuda_error": (c_int, []),
    "hs_router_workspace_size": (c_size_t, [c_int64, c_int64, c_int64]),
    "hs_router_topk": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_float,
                               c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "hs_hash_route": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p,
                              c_void_p]),
    "hs_moe_make_desc": (c_int, [POINTER(hs_moe_weights), c_void_p, c_size_t]),
    "hs_moe_workspace_size": (c_size_t, [c_int64, c_int64, c_int64, c_int64, c_int64]),
    "hs_moe_ffn_fp4": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int, c_int, c_void_p,
                               c_void_p, c_void_p, c_size_t, c_void_p, c_void_p]),
    "hs_moe_ffn_fp4_noalloc": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int, c_int,
                                       c_void_p, c_void_p, c_void_p, c_void_p]),
    "hs_moe_permute_workspace_size": (c_size_t, [c_int64, c_int64, c_int64]),
    "hs_moe_permute": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_void_p,
                               c_void_p, c_void_p, c_void_p, c_size_t, c_void_p, c_void_p]),
    "hs_moe_unpermute": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_int64, c_void_p,
                                 c_void_p]),
    "hs_accept_greedy": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p,
                                 c_void_p, c_void_p]),
    "hs_accept_rejection": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p, c_void_p,
                                    c_float, c_void_p, c_void_p, c_void_p, c_void_p]),
    "hs_lm_head_workspace_size": (c_size_t, [c_int64]),
    "hs_lm_head_argmax": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p,
                                  c_void_p, c_void_p, c_void_p, c_size_t, c_void_p, c_void_p]),
    "hs_rms_norm": (c_int, [c_void_p, c_void_p, c_float, c_int64, c_int64, c_void_p, c_void_p]),
    "hs_add_rms_norm": (c_int, [c_void_p, c_void_p, c_void_p, c_float, c_int64, c_int64, c_void_p, c_void_p,
                                c_void_p]),
    "hs_moe_ffn_fp4_partials": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int, c_int,
                                        c_void_p, c_void_p, c_void_p, c_size_t, c_void_p, c_void_p]),
    "hs_moe_route_ffn_fp4": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64,
                                     c_float, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                     c_size_t, c_void_p, c_void_p]),
    "hs_moe_route_ffn_fp4_partials": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                              c_int64, c_float, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                              c_void_p, c_void_p, c_size_t, c_void_p, c_void_p]),
    "hs_moe_layer_fp4": (c_int, [c_void_p, c_void_p, c_void_p, c_float, c_void_p, c_void_p, c_void_p, c_void_p,
                                 c_int64, c_int64, c_int64, c_int64, c_int64, c_float, c_int, c_int, c_void_p,
                                 c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p, c_void_p]),
    "hs_moe_layer_fp4_partials": (c_int, [c_void_p, c_void_p, c_void_p, c_float, c_void_p, c_void_p, c_void_p,
                                          c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64, c_float, c_int,
                                          c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                          c_size_t, c_void_p, c_void_p]),
    "hs_ep_buffer_bytes": (c_size_t, [c_int64, c_int64]),
    "hs_ep_buffer_alloc": (c_int, [c_size_t, POINTER(c_void_p)]),
    "hs_ep_buffer_free": (c_int, [c_void_p]),
    "hs_ipc_get_handle": (c_int, [c_void_p, c_void_p, c_size_t]),
    "hs_ipc_open_handle": (c_int, [c_void_p, POINTER(c_void_p)]),
    "hs_ipc_close_handle": (c_int, [c_void_p]),
    "hs_moe_layer_fp4_ep": (c_int, [c_void_p, c_void_p, c_void_p, c_float, c_void_p, c_void_p, c_void_p, c_void_p,
                                    c_int64, c_int64, c_int64, c_int64, c_int64, c_float, c_int, c_int, c_void_p,
                                    c_void_p, c_void_p, POINTER(HsEpPeers), c_void_p, c_void_p, c_size_t, c_void_p,
                                    c_void_p]),
    "hs_moe_layer_fp4_ep_chained": (c_int, [c_void_p, c_void_p, c_void_p, c_float, c_void_p, c_void_p, c_void_p,
                                            c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64, c_float, c_int,
                                            c_int, c_void_p, c_void_p, c_void_p, POINTER(HsEpPeers), c_int, c_int,
                                            c_void_p, c_size_t, c_void_p, c_void_p]),
    "hs_ep_combine_pending": (c_int, [POINTER(HsEpPeers), c_void_p, c_int64, c_int64, c_int, c_void_p, c_void_p]),
    "hs_lm_head_argmax_ep": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64, c_void_p,
                                     c_void_p, c_void_p, c_void_p, POINTER(HsEpPeers), c_void_p, c_size_t, c_void_p,
                                     c_void_p]),
    "hs_moe_combine": (c_int, [c_void_p, c_void_p, c_int, c_int64, c_int64, c_void_p, c_void_p]),
    "hs_moe_combine_add_rms_norm": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_float, c_int64, c_int64,
                                            c_void_p, c_void_p, c_void_p]),
    "hs_ep_nccl_unique_id": (c_int, [c_void_p]),
    "hs_ep_nccl_comm_init": (c_int, [c_void_p, c_int32, c_int32, POINTER(c_void_p)]),
    "hs_ep_nccl_comm_destroy": (c_int, [c_void_p]),
    "hs_ep_dispatch_plan": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_int32, c_int32, c_void_p, c_void_p,
                                    c_void_p, c_void_p]),
    "hs_ep_dispatch_combine_workspace_size": (c_size_t, [c_int64, c_int64, c_int64, c_int64, c_int64, c_int32]),
    "hs_ep_dispatch_combine": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                       c_int, c_int, c_void_p, c_void_p, c_size_t, c_void_p, c_void_p]),
    "hs_verify_state_snapshot": (c_int, [c_void_p, c_int64, c_int64, c_void_p]),
    "hs_verify_state_commit": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_int32, c_void_p]),
    "hs_fill_bytes": (c_int, [c_void_p, c_int64, c_uint64, c_int32, c_int32, c_void_p]),
    "hs_trace_buffer": (c_void_p, [c_int]),
}

_lib = None


def lib_path() -> Path:
    return _LIB_PATH


def load() -> ctypes.CDLL:
    """Load libhs_ext.so (building it first if the sources are newer)."""
    global _lib
    if _lib is not None:
        return _lib
    if os.environ.get("HS_NO_AUTOBUILD") != "1":
        from . import build as _build
        if _build.is_stale():
            _build.build()
    if not _LIB_PATH.exists():
        raise ImportError(f"{_LIB_PATH} is missing; run python -m home_seek_b200.build")
    lib = ctypes.CDLL(str(_LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def call(name: str, *args) -> None:
    """Call an hs_* entry point that returns a status; raise HsError if non-zero."""
    lib = load()
    st = getattr(lib, name)(*args)
    if st != HS_OK:
        raise HsError(name, st, lib.hs_last_cuda_error() if st == 5 else 0)


def exported_symbols() -> list[str]:
    return list(SIGNATURES)
