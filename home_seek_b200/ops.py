"""Tensor-level wrappers over the C ABI: validate, fetch a workspace, launch on
the current stream. Every op runs on the GPU through libhs_ext.so; there is
no CPU fallback (a CPU tensor raises).
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib
from ._lib import HsError, call

_workspaces: dict = {}
_status: dict = {}

# Number of this library's kernels each op launches; summed into `launches`
# so a caller can count the kernels of one decode iteration.
launches = 0
_KERNELS = {"hs_router_topk": 1, "hs_hash_route": 1, "hs_moe_ffn_fp4": 3, "hs_moe_permute": 2,
            "hs_moe_unpermute": 1, "hs_accept_greedy": 1, "hs_accept_rejection": 1, "hs_fill_bytes": 1,
            "hs_rms_norm": 1, "hs_add_rms_norm": 1, "hs_moe_ffn_fp4_partials": 3, "hs_moe_combine": 1,
            "hs_moe_route_ffn_fp4": 3, "hs_moe_route_ffn_fp4_partials": 3,
            "hs_moe_combine_add_rms_norm": 1, "hs_moe_layer_fp4": 3, "hs_moe_layer_fp4_partials": 3,
            "hs_moe_layer_fp4_ep": 4, "hs_moe_layer_fp4_ep_chained": 3, "hs_ep_combine_pending": 1,
            "hs_lm_head_argmax": 1,
            "hs_lm_head_argmax_ep": 1}


def _launch(name: str, *args, extra: int = 0) -> None:
    global launches
    call(name, *args)
    launches += _KERNELS.get(name, 0) + extra


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _check_cuda(*ts: Optional[torch.Tensor]) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("home_seek_b200 ops need CUDA tensors (there is no CPU path)")
        if not t.is_contiguous():
            raise ValueError("home_seek_b200 ops need contiguous tensors")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError("all tensors must be on the same device")
    return dev


def workspace(device: torch.device, nbytes: int, tag: str) -> torch.Tensor:
    """Grow-only scratch per (device, stream, tag), zero-filled when allocated
    (the kernels keep their counters at zero between calls). Calls on one
    stream are ordered, so reusing the buffer across calls is race-free."""
    key = (device.index, _stream(device), tag)
    buf = _workspaces.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(int(nbytes), 256), dtype=torch.uint8, device=device)
        _workspaces[key] = buf
    return buf


def status_word(device: torch.device) -> torch.Tensor:
    """Device int32 that kernels OR HS_DEV_* bits into; read with check_status().
    One word per GPU: torch.device("cuda") means the current device."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    s = _status.get(idx)
    if s is None:
        s = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _status[idx] = s
    return s


def check_status(device: torch.device, reset: bool = True) -> int:
    s = status_word(device)
    v = int(s.item())
    if reset and v:
        s.zero_()
    return v


# --- router / hash -------------------------------------------------------------

def router_topk(hidden: torch.Tensor, gate: torch.Tensor, bias: Optional[torch.Tensor], top_k: int = 6,
                routed_scaling: float = 1.5, return_logits: bool = False):
    """compute_expert_affinity_with_bias (router.py:22-36) on the GPU."""
    dev = _check_cuda(hidden, gate, bias)
    if hidden.dtype != torch.bfloat16 or gate.dtype != torch.bfloat16:
        hidden = hidden.to(torch.bfloat16).contiguous()
        gate = gate.to(torch.bfloat16).contiguous()
    if bias is not None and bias.dtype != torch.bfloat16:
        bias = bias.to(torch.bfloat16).contiguous()
    T, D = hidden.shape
    E = gate.shape[0]
    idx = torch.empty(T, top_k, dtype=torch.int64, device=dev)
    w = torch.empty(T, top_k, dtype=torch.float32, device=dev)
    lg = torch.empty(T, E, dtype=torch.bfloat16, device=dev) if return_logits else None
    lib = _lib.load()
    nb = lib.hs_router_workspace_size(T, D, E)
    ws = workspace(dev, nb, "router")
    _launch("hs_router_topk", hidden.data_ptr(), gate.data_ptr(), _ptr(bias), T, D, E, top_k, float(routed_scaling),
            idx.data_ptr(), w.data_ptr(), _ptr(lg), ws.data_ptr(), ws.numel(), _stream(dev),
            extra=0 if T <= 64 else 1)
    if return_logits:
        return idx, w, lg
    return idx, w


def hash_route(input_ids: torch.Tensor, tid2eid: torch.Tensor, top_k: int = 6):
    """_compute_hash_experts (engine.py:1018-1023) on the GPU; keeps input_ids' shape."""
    dev = _check_cuda(input_ids, tid2eid)
    ids = input_ids.to(torch.int64).contiguous()
    tid = tid2eid.to(torch.int64).contiguous()
    T = ids.numel()
    idx = torch.empty(*ids.shape, top_k, dtype=torch.int64, device=dev)
    w = torch.empty(*ids.shape, top_k, dtype=torch.float32, device=dev)
    _launch("hs_hash_route", ids.data_ptr(), T, tid.data_ptr(), tid.shape[0], top_k, idx.data_ptr(), w.data_ptr(),
         status_word(dev).data_ptr(), _stream(dev))
    return idx, w


# --- MoE FFN -------------------------------------------------------------------

def make_moe_desc(w13, s13, w2, s2, sh_w13=None, sh_s13=None, sh_w2=None, sh_s2=None) -> ctypes.Array:
    """Encode the per-layer TMA descriptor blob (host memory) for hs_moe_ffn_fp4.
    Tensors in the expert store's tiled layout (layout.py):
    w13 [E][I/128][D/128][2][128][64], sh_w13 [I_sh/128][D/128][2][128][128]."""
    E, it, kt, two, r, rb = w13.shape
    if two != 2 or r != 128 or rb != 64:
        raise ValueError(f"w13 {tuple(w13.shape)} is not in the tiled layout")
    I, D = it * 128, kt * 128
    I_sh = sh_w13.shape[0] * 128 if sh_w13 is not None else 0
    wts = _lib.hs_moe_weights(w13.data_ptr(), s13.data_ptr(), w2.data_ptr(), s2.data_ptr(),
                              _ptr(sh_w13), _ptr(sh_s13), _ptr(sh_w2), _ptr(sh_s2), E, D, I, I_sh)
    buf = (ctypes.c_uint8 * _lib.HS_MOE_DESC_BYTES)()
    with torch.cuda.device(w13.device):
        call("hs_moe_make_desc", ctypes.byref(wts), buf, ctypes.sizeof(buf))
    return buf


def moe_ffn(desc: ctypes.Array, dims: tuple, hidden: torch.Tensor, topk_idx: torch.Tensor, topk_w: torch.Tensor,
            use_shared: bool = True, dup_mode: int = _lib.HS_DUP_LAST, out: Optional[torch.Tensor] = None,
            out_f32: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Routed FP4 FFN (+ FP8 shared expert) for hidden [T, D] bf16. dims = (E, D, I, I_sh)."""
    dev = _check_cuda(hidden, topk_idx, topk_w, out, out_f32)
    if hidden.dtype != torch.bfloat16:
        raise TypeError("hidden must be bf16")
    topk_idx = topk_idx.to(torch.int64).contiguous()
    topk_w = topk_w.to(torch.float32).contiguous()
    T, D = hidden.shape
    K = topk_idx.shape[-1]
    E, Dd, I, I_sh = dims
    if D != Dd:
        raise ValueError(f"hidden dim {D} != store dim {Dd}")
    if out is None:
        out = torch.empty(T, D, dtype=torch.bfloat16, device=dev)
    lib = _lib.load()
    nb = lib.hs_moe_workspace_size(T, K, D, I, I_sh)
    ws = workspace(dev, nb, "moe")
    _launch("hs_moe_ffn_fp4", ctypes.addressof(desc), hidden.data_ptr(), topk_idx.data_ptr(), topk_w.data_ptr(), T, K,
         int(bool(use_shared)), int(dup_mode), out.data_ptr(), _ptr(out_f32), ws.data_ptr(), ws.numel(),
         status_word(dev).data_ptr(), _stream(dev), extra=0 if T * K <= 4096 else 1)
    return out


def moe_ffn_partials(desc: ctypes.Array, dims: tuple, hidden: torch.Tensor, topk_idx: torch.Tensor,
                     topk_w: torch.Tensor, use_shared: bool = True, dup_mode: int = _lib.HS_DUP_LAST,
                     out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The un-rounded f32 sums of one expert-parallel rank: returns [2, T, D] f32
    (routed over this store's experts, shared over its slice of the shared
    expert; ids outside the store must already be -1). Sum over ranks, then
    moe_combine / moe_combine_add_rms_norm."""
    dev = _check_cuda(hidden, topk_idx, topk_w, out)
    if hidden.dtype != torch.bfloat16:
        raise TypeError("hidden must be bf16")
    topk_idx = topk_idx.to(torch.int64).contiguous()
    topk_w = topk_w.to(torch.float32).contiguous()
    T, D = hidden.shape
    K = topk_idx.shape[-1]
    E, Dd, I, I_sh = dims
    if D != Dd:
        raise ValueError(f"hidden dim {D} != store dim {Dd}")
    if out is None:
        out = torch.empty(2, T, D, dtype=torch.float32, device=dev)
    if tuple(out.shape) != (2, T, D) or out.dtype != torch.float32:
        raise ValueError("out must be [2, T, D] float32")
    use_shared = bool(use_shared) and bool(I_sh)
    if not use_shared:
        out[1].zero_()
    lib = _lib.load()
    nb = lib.hs_moe_workspace_size(T, K, D, I, I_sh)
    ws = workspace(dev, nb, "moe")
    _launch("hs_moe_ffn_fp4_partials", ctypes.addressof(desc), hidden.data_ptr(), topk_idx.data_ptr(),
            topk_w.data_ptr(), T, K, int(use_shared), int(dup_mode), out[0].data_ptr(),
            out[1].data_ptr() if use_shared else None, ws.data_ptr(), ws.numel(), status_word(dev).data_ptr(),
            _stream(dev), extra=0 if T * K <= 4096 else 1)
    return out


def moe_route_ffn(desc: ctypes.Array, dims: tuple, hidden: torch.Tensor, gate: torch.Tensor,
                  bias: Optional[torch.Tensor], top_k: int, routed_scaling: float, use_shared: bool = True,
                  dup_mode: int = _lib.HS_DUP_LAST, expert_offset: int = 0, partials: bool = False,
                  out: Optional[torch.Tensor] = None):
    """Router + MoE FFN in one call for T <= 8 (hs_moe_route_ffn_fp4): returns
    (out, topk_idx, topk_w) with out [T, D] bf16, or [2, T, D] f32 partial sums
    when partials (expert parallelism: sum over ranks, then moe_combine)."""
    dev = _check_cuda(hidden, gate, bias, out)
    if hidden.dtype != torch.bfloat16 or gate.dtype != torch.bfloat16:
        raise TypeError("hidden and gate must be bf16")
    T, D = hidden.shape
    E, Dd, I, I_sh = dims
    if D != Dd:
        raise ValueError(f"hidden dim {D} != store dim {Dd}")
    n_exp = gate.shape[0]
    idx = torch.empty(T, top_k, dtype=torch.int64, device=dev)
    w = torch.empty(T, top_k, dtype=torch.float32, device=dev)
    lib = _lib.load()
    ws = workspace(dev, lib.hs_moe_workspace_size(T, top_k, D, I, I_sh), "moe")
    use_shared = bool(use_shared) and bool(I_sh)
    if partials:
        if out is None:
            out = torch.empty(2, T, D, dtype=torch.float32, device=dev)
        if not use_shared:
            out[1].zero_()
        _launch("hs_moe_route_ffn_fp4_partials", ctypes.addressof(desc), hidden.data_ptr(), gate.data_ptr(),
                _ptr(bias), n_exp, int(expert_offset), T, top_k, float(routed_scaling), int(use_shared),
                int(dup_mode), idx.data_ptr(), w.data_ptr(), out[0].data_ptr(),
                out[1].data_ptr() if use_shared else None, ws.data_ptr(), ws.numel(), status_word(dev).data_ptr(),
                _stream(dev))
    else:
        if out is None:
            out = torch.empty(T, D, dtype=torch.bfloat16, device=dev)
        _launch("hs_moe_route_ffn_fp4", ctypes.addressof(desc), hidden.data_ptr(), gate.data_ptr(), _ptr(bias),
                n_exp, int(expert_offset), T, top_k, float(routed_scaling), int(use_shared), int(dup_mode),
                idx.data_ptr(), w.data_ptr(), out.data_ptr(), None, ws.data_ptr(), ws.numel(),
                status_word(dev).data_ptr(), _stream(dev))
    return out, idx, w


def moe_layer(desc: ctypes.Array, dims: tuple, h: torch.Tensor, norm_w: torch.Tensor,
              gate: Optional[torch.Tensor], bias: Optional[torch.Tensor], top_k: int, routed_scaling: float,
              eps: float = 1e-6, use_shared: bool = True, dup_mode: int = _lib.HS_DUP_LAST,
              num_experts: Optional[int] = None, expert_offset: int = 0, ids: Optional[torch.Tensor] = None,
              tid2eid: Optional[torch.Tensor] = None, h_out: Optional[torch.Tensor] = None,
              x_out: Optional[torch.Tensor] = None, partials: bool = False, out: Optional[torch.Tensor] = None):
    """The MoE half of a decode layer for T <= 8 (hs_moe_layer_fp4):
    h_out = h + MoE(rms_norm(h, norm_w)), routed by the router (gate, bias) or,
    with tid2eid, by hash of ids. Returns (h_out, topk_idx, topk_w); h_out may
    be h. With partials the first value is the [2, T, D] f32 partial sums of
    this store's experts (expert parallelism) and h is left untouched."""
    dev = _check_cuda(h, norm_w, gate, bias, ids, tid2eid, h_out, x_out, out)
    h = _rows(h, "h")
    norm_w = _rows(norm_w, "norm_w")
    T, D = h.shape
    E, Dd, I, I_sh = dims
    if D != Dd:
        raise ValueError(f"hidden dim {D} != store dim {Dd}")
    if tid2eid is None and (gate is None or gate.dtype != torch.bfloat16):
        raise TypeError("router mode needs a bf16 gate")
    if tid2eid is not None and (ids is None or ids.dtype != torch.int64 or tid2eid.dtype != torch.int64):
        raise TypeError("hash mode needs int64 ids and tid2eid")
    n_exp = int(num_experts if num_experts is not None else (gate.shape[0] if gate is not None else E))
    idx = torch.empty(T, top_k, dtype=torch.int64, device=dev)
    w = torch.empty(T, top_k, dtype=torch.float32, device=dev)
    lib = _lib.load()
    ws = workspace(dev, lib.hs_moe_workspace_size(T, top_k, D, I, I_sh), "moe")
    use_shared = bool(use_shared) and bool(I_sh)
    ids_c = ids.reshape(-1).contiguous() if ids is not None else None
    vocab = int(tid2eid.shape[0]) if tid2eid is not None else 0
    route = (ctypes.addressof(desc), h.data_ptr(), norm_w.data_ptr(), float(eps),
             None if tid2eid is not None else gate.data_ptr(), None if tid2eid is not None else _ptr(bias),
             _ptr(ids_c), _ptr(tid2eid), vocab, n_exp, int(expert_offset), T, top_k, float(routed_scaling),
             int(use_shared), int(dup_mode), idx.data_ptr(), w.data_ptr(), _ptr(x_out))
    if partials:
        if out is None:
            out = torch.empty(2, T, D, dtype=torch.float32, device=dev)
        if not use_shared:
            out[1].zero_()
        _launch("hs_moe_layer_fp4_partials", *route, out[0].data_ptr(), out[1].data_ptr() if use_shared else None,
                ws.data_ptr(), ws.numel(), status_word(dev).data_ptr(), _stream(dev))
        return out, idx, w
    if h_out is None:
        h_out = torch.empty_like(h)
    _launch("hs_moe_layer_fp4", *route, h_out.data_ptr(), ws.data_ptr(), ws.numel(), status_word(dev).data_ptr(),
            _stream(dev))
    return h_out, idx, w


def moe_layer_ep(desc: ctypes.Array, dims: tuple, h: torch.Tensor, norm_w: torch.Tensor,
                 gate: Optional[torch.Tensor], bias: Optional[torch.Tensor], top_k: int, routed_scaling: float,
                 peers: "_lib.HsEpPeers", eps: float = 1e-6, use_shared: bool = True,
                 dup_mode: int = _lib.HS_DUP_LAST, num_experts: Optional[int] = None, expert_offset: int = 0,
                 ids: Optional[torch.Tensor] = None, tid2eid: Optional[torch.Tensor] = None,
                 h_out: Optional[torch.Tensor] = None, x_out: Optional[torch.Tensor] = None):
    """moe_layer for one rank of an expert-parallel group over NVLink peer
    memory (hs_moe_layer_fp4_ep): this rank's experts, their rows stored into
    every rank's receive buffer by the down phase, summed in rank order into
    h_out (identical on every rank). Every rank must make the same calls."""
    dev = _check_cuda(h, norm_w, gate, bias, ids, tid2eid, h_out, x_out)
    h = _rows(h, "h")
    norm_w = _rows(norm_w, "norm_w")
    T, D = h.shape
    E, Dd, I, I_sh = dims
    if D != Dd:
        raise ValueError(f"hidden dim {D} != store dim {Dd}")
    if tid2eid is None and (gate is None or gate.dtype != torch.bfloat16):
        raise TypeError("router mode needs a bf16 gate")
    n_exp = int(num_experts if num_experts is not None else (gate.shape[0] if gate is not None else E))
    idx = torch.empty(T, top_k, dtype=torch.int64, device=dev)
    w = torch.empty(T, top_k, dtype=torch.float32, device=dev)
    lib = _lib.load()
    ws = workspace(dev, lib.hs_moe_workspace_size(T, top_k, D, I, I_sh), "moe")
    ids_c = ids.reshape(-1).contiguous() if ids is not None else None
    vocab = int(tid2eid.shape[0]) if tid2eid is not None else 0
    if h_out is None:
        h_out = torch.empty_like(h)
    _launch("hs_moe_layer_fp4_ep", ctypes.addressof(desc), h.data_ptr(), norm_w.data_ptr(), float(eps),
            None if tid2eid is not None else gate.data_ptr(), None if tid2eid is not None else _ptr(bias),
            _ptr(ids_c), _ptr(tid2eid), vocab, n_exp, int(expert_offset), T, top_k, float(routed_scaling),
            int(bool(use_shared) and bool(I_sh)), int(dup_mode), idx.data_ptr(), w.data_ptr(), _ptr(x_out),
            ctypes.byref(peers), h_out.data_ptr(), ws.data_ptr(), ws.numel(), status_word(dev).data_ptr(),
            _stream(dev))
    return h_out, idx, w


def moe_layer_ep_chained(desc: ctypes.Array, dims: tuple, h: torch.Tensor, norm_w: torch.Tensor,
                         gate: Optional[torch.Tensor], bias: Optional[torch.Tensor], top_k: int,
                         routed_scaling: float, peers: "_lib.HsEpPeers", prev_pending: bool,
                         prev_use_shared: bool = True, eps: float = 1e-6, use_shared: bool = True,
                         dup_mode: int = _lib.HS_DUP_LAST, num_experts: Optional[int] = None,
                         expert_offset: int = 0, ids: Optional[torch.Tensor] = None,
                         tid2eid: Optional[torch.Tensor] = None, x_out: Optional[torch.Tensor] = None):
    """moe_layer_ep for a stack of layers, each call's exchange completed at
    the start of the next (hs_moe_layer_fp4_ep_chained): with prev_pending the
    previous chained call's output is first added to h in place, then this
    layer runs on it and leaves its own output pending. ep_combine_pending
    completes the last one. Consecutive calls take the same h. Returns
    (idx, w)."""
    dev = _check_cuda(h, norm_w, gate, bias, ids, tid2eid, x_out)
    if not h.is_contiguous() or h.dtype != torch.bfloat16 or h.dim() != 2:
        raise ValueError("h must be contiguous bf16 [T, D] (it is updated in place)")
    norm_w = _rows(norm_w, "norm_w")
    T, D = h.shape
    E, Dd, I, I_sh = dims
    if D != Dd:
        raise ValueError(f"hidden dim {D} != store dim {Dd}")
    if tid2eid is None and (gate is None or gate.dtype != torch.bfloat16):
        raise TypeError("router mode needs a bf16 gate")
    n_exp = int(num_experts if num_experts is not None else (gate.shape[0] if gate is not None else E))
    idx = torch.empty(T, top_k, dtype=torch.int64, device=dev)
    w = torch.empty(T, top_k, dtype=torch.float32, device=dev)
    lib = _lib.load()
    ws = workspace(dev, lib.hs_moe_workspace_size(T, top_k, D, I, I_sh), "moe")
    ids_c = ids.reshape(-1).contiguous() if ids is not None else None
    vocab = int(tid2eid.shape[0]) if tid2eid is not None else 0
    _launch("hs_moe_layer_fp4_ep_chained", ctypes.addressof(desc), h.data_ptr(), norm_w.data_ptr(), float(eps),
            None if tid2eid is not None else gate.data_ptr(), None if tid2eid is not None else _ptr(bias),
            _ptr(ids_c), _ptr(tid2eid), vocab, n_exp, int(expert_offset), T, top_k, float(routed_scaling),
            int(bool(use_shared) and bool(I_sh)), int(dup_mode), idx.data_ptr(), w.data_ptr(), _ptr(x_out),
            ctypes.byref(peers), int(bool(prev_pending)), int(bool(prev_use_shared)), ws.data_ptr(), ws.numel(),
            status_word(dev).data_ptr(), _stream(dev))
    return idx, w


def ep_combine_pending(peers: "_lib.HsEpPeers", h: torch.Tensor, use_shared: bool = True) -> torch.Tensor:
    """Completes the last moe_layer_ep_chained call: h += its MoE output, in
    place (hs_ep_combine_pending)."""
    dev = _check_cuda(h)
    if not h.is_contiguous() or h.dtype != torch.bfloat16 or h.dim() != 2:
        raise ValueError("h must be contiguous bf16 [T, D] (it is updated in place)")
    T, D = h.shape
    _launch("hs_ep_combine_pending", ctypes.byref(peers), h.data_ptr(), T, D, int(bool(use_shared)),
            status_word(dev).data_ptr(), _stream(dev))
    return h


def moe_combine(partials: torch.Tensor, use_shared: bool = True, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """bf16(bf16(routed) + bf16(shared)) from summed f32 partials [2, T, D]."""
    dev = _check_cuda(partials, out)
    _, T, D = partials.shape
    if out is None:
        out = torch.empty(T, D, dtype=torch.bfloat16, device=dev)
    _launch("hs_moe_combine", partials[0].data_ptr(), partials[1].data_ptr(), int(bool(use_shared)), T, D,
            out.data_ptr(), _stream(dev))
    return out


def moe_combine_add_rms_norm(partials: torch.Tensor, h: torch.Tensor, w: torch.Tensor, eps: float = 1e-6,
                             use_shared: bool = True, h_out: Optional[torch.Tensor] = None,
                             x_out: Optional[torch.Tensor] = None):
    """Combine f32 partials [2, T, D], add to the residual stream h and normalise:
    returns (h + combine, rms_norm(h + combine, w)). h_out may be h. With w
    None the norm is left out: returns (h + combine, None)."""
    dev = _check_cuda(partials, h, w, h_out, x_out)
    h = _rows(h, "h")
    if w is not None:
        w = _rows(w, "w")
    _, T, D = partials.shape
    if h_out is None:
        h_out = torch.empty_like(h)
    if x_out is None and w is not None:
        x_out = torch.empty_like(h)
    _launch("hs_moe_combine_add_rms_norm", partials[0].data_ptr(), partials[1].data_ptr(), int(bool(use_shared)),
            h.data_ptr(), _ptr(w), float(eps), T, D, h_out.data_ptr(), _ptr(x_out), _stream(dev))
    return h_out, x_out


def moe_permute(topk_idx: torch.Tensor, num_experts: int, x: Optional[torch.Tensor] = None):
    """Expert-major permutation (expand_to_fused, tests/_reference.py:108-121).

    Returns (token_topk_to_pos int32 [T, k], pos_to_expert int32 [T*k],
    expert_count int32 [E], num_pos int32 [1], x_expanded [T*k, D] or None).
    """
    dev = _check_cuda(topk_idx, x)
    idx = topk_idx.to(torch.int64).contiguous()
    T, K = idx.shape
    pos = torch.empty(T, K, dtype=torch.int32, device=dev)
    p2e = torch.empty(T * K, dtype=torch.int32, device=dev)
    cnt = torch.empty(num_experts, dtype=torch.int32, device=dev)
    npos = torch.empty(1, dtype=torch.int32, device=dev)
    xe = None
    if x is not None:
        xe = torch.empty(T * K, x.shape[1], dtype=x.dtype, device=dev)
    lib = _lib.load()
    ws = workspace(dev, lib.hs_moe_permute_workspace_size(T, K, num_experts), "permute")
    _launch("hs_moe_permute", idx.data_ptr(), T, K, num_experts, _ptr(x), x.shape[1] if x is not None else 0,
         pos.data_ptr(), p2e.data_ptr(), cnt.data_ptr(), npos.data_ptr(), _ptr(xe), ws.data_ptr(), ws.numel(),
         status_word(dev).data_ptr(), _stream(dev))
    return pos, p2e, cnt, npos, xe


def moe_unpermute(x_expanded: torch.Tensor, token_topk_to_pos: torch.Tensor,
                  topk_w: Optional[torch.Tensor] = None) -> torch.Tensor:
    """reduce_fused (tests/_reference.py:52-90): out[t] = sum_k w[t,k] * x[pos[t,k]] in f32, k order."""
    dev = _check_cuda(x_expanded, token_topk_to_pos, topk_w)
    pos = token_topk_to_pos.to(torch.int32).contiguous()
    w = topk_w.to(torch.float32).contiguous() if topk_w is not None else None
    T, K = pos.shape
    out = torch.empty(T, x_expanded.shape[1], dtype=torch.bfloat16, device=dev)
    _launch("hs_moe_unpermute", x_expanded.data_ptr(), x_expanded.shape[0], x_expanded.shape[1], pos.data_ptr(),
         _ptr(w), T, K, out.data_ptr(), _stream(dev))
    return out


# --- acceptance ----------------------------------------------------------------

def accept_greedy(logits: torch.Tensor, draft_ids: torch.Tensor, want_argmax: bool = False):
    """logits [B, T, V] bf16, draft_ids [B, T-1] -> (n_accept int32 [B], next_token int64 [B][, argmax [B, T]])."""
    dev = _check_cuda(logits, draft_ids)
    if logits.dtype != torch.bfloat16:
        raise TypeError("logits must be bf16")
    B, T, V = logits.shape
    ids = draft_ids.to(torch.int64).contiguous()
    n = torch.empty(B, dtype=torch.int32, device=dev)
    nxt = torch.empty(B, dtype=torch.int64, device=dev)
    am = torch.empty(B, T, dtype=torch.int64, device=dev) if want_argmax else None
    _launch("hs_accept_greedy", logits.data_ptr(), B, T, V, ids.data_ptr(), n.data_ptr(), nxt.data_ptr(), _ptr(am),
         status_word(dev).data_ptr(), _stream(dev))
    return (n, nxt, am) if want_argmax else (n, nxt)


def accept_rejection(target: torch.Tensor, draft: torch.Tensor, draft_ids: torch.Tensor, uniform: torch.Tensor,
                     temperature: float):
    """Speculative sampling: target [B, M+1, V], draft [B, R>=M, V] bf16, draft_ids [B, M], uniform [B, M+1]."""
    dev = _check_cuda(target, draft, draft_ids, uniform)
    B, M1, V = target.shape
    M = M1 - 1
    ids = draft_ids.to(torch.int64).contiguous()
    u = uniform.to(torch.float32).contiguous()
    n = torch.empty(B, dtype=torch.int32, device=dev)
    nxt = torch.empty(B, dtype=torch.int64, device=dev)
    _launch("hs_accept_rejection", target.data_ptr(), draft.data_ptr(), B, M, draft.shape[1], V, ids.data_ptr(),
         u.data_ptr(), float(temperature), n.data_ptr(), nxt.data_ptr(), status_word(dev).data_ptr(), _stream(dev))
    return n, nxt


def sample(logits: torch.Tensor, temperature: float, uniform: torch.Tensor) -> torch.Tensor:
    """One token per row from softmax(logits / temperature) by inverse CDF in
    ascending token order with a supplied uniform: the sampling of the draft
    (engine.py:2327-2331) and of the bonus token (engine.py:2908-2911) with
    torch.multinomial replaced by a given u in [0, 1). logits [B, V] bf16,
    uniform [B] f32 -> int64 [B]. (hs_accept_rejection with no drafts.)"""
    dev = _check_cuda(logits, uniform)
    if logits.dtype != torch.bfloat16:
        raise TypeError("logits must be bf16")
    if not temperature > 0:
        raise ValueError("sampling needs a temperature > 0 (use lm_head_argmax for t = 0)")
    B, V = logits.shape
    u = uniform.reshape(-1).to(torch.float32).contiguous()
    if u.numel() != B:
        raise ValueError(f"{u.numel()} uniforms for {B} rows")
    n = torch.empty(B, dtype=torch.int32, device=dev)
    nxt = torch.empty(B, dtype=torch.int64, device=dev)
    _launch("hs_accept_rejection", logits.contiguous().data_ptr(), None, B, 0, 0, V, None, u.data_ptr(),
            float(temperature), n.data_ptr(), nxt.data_ptr(), status_word(dev).data_ptr(), _stream(dev))
    return nxt


# --- lm_head + greedy decision ---------------------------------------------------

def lm_head_argmax(x: torch.Tensor, head: torch.Tensor, draft_ids: Optional[torch.Tensor] = None,
                   want_logits: bool = False, out: Optional[tuple] = None):
    """logits = x @ head.t() (bf16, f32 accumulate) with the argmax fused in
    (hs_lm_head_argmax): x [T, D] bf16 rows after the final norm (T <= 16),
    head [V, D] bf16. Returns (argmax int64 [T], n_accept int32 [1],
    next_token int64 [1]) and, with want_logits, the bf16 logits [T, V].
    With draft_ids [T-1] the greedy acceptance of the verify pass is applied
    (engine.py:2485-2497): n_accept leading matches, next_token =
    argmax[n_accept]; without them next_token = argmax[0]. `out` may supply
    the three result tensors (e.g. buffers that a CUDA graph reuses)."""
    dev = _check_cuda(x, head, draft_ids)
    x = _rows(x, "x")
    head = _rows(head, "head")
    T, D = x.shape
    V = head.shape[0]
    if head.shape[1] != D:
        raise ValueError(f"head has {head.shape[1]} columns, rows have {D}")
    ids = None
    if draft_ids is not None:
        ids = draft_ids.reshape(-1).to(torch.int64).contiguous()
        if ids.numel() != T - 1:
            raise ValueError(f"{ids.numel()} draft ids for {T} rows")
    if out is None:
        am = torch.empty(T, dtype=torch.int64, device=dev)
        n = torch.empty(1, dtype=torch.int32, device=dev)
        nxt = torch.empty(1, dtype=torch.int64, device=dev)
    else:
        am, n, nxt = out
    lg = torch.empty(T, V, dtype=torch.bfloat16, device=dev) if want_logits else None
    lib = _lib.load()
    ws = workspace(dev, lib.hs_lm_head_workspace_size(T), "head")
    _launch("hs_lm_head_argmax", x.data_ptr(), head.data_ptr(), T, D, V, _ptr(ids), am.data_ptr(), n.data_ptr(),
            nxt.data_ptr(), _ptr(lg), ws.data_ptr(), ws.numel(), status_word(dev).data_ptr(), _stream(dev))
    return (am, n, nxt, lg) if want_logits else (am, n, nxt)


def vocab_rows(V: int, rank: int, world: int) -> tuple[int, int]:
    """(row0, rows) of the head that rank `rank` of `world` streams in
    lm_head_argmax_ep: whole 128-row tiles, split as evenly as they go."""
    tiles = (V + 127) // 128
    lo, hi = tiles * rank // world * 128, tiles * (rank + 1) // world * 128
    return lo, min(hi, V) - lo


def lm_head_argmax_ep(x: torch.Tensor, head: torch.Tensor, peers: "_lib.HsEpPeers",
                      draft_ids: Optional[torch.Tensor] = None, out: Optional[tuple] = None):
    """lm_head_argmax with the vocabulary split over an expert-parallel group
    (hs_lm_head_argmax_ep): head is the whole [V, D] head (every rank holds
    it); this rank streams its rows (vocab_rows) and the ranks exchange their
    best keys through the peer buffers, so every rank returns the results of
    lm_head_argmax on the whole head. Every rank must make the same calls."""
    dev = _check_cuda(x, head, draft_ids)
    x = _rows(x, "x")
    head = _rows(head, "head")
    T, D = x.shape
    V = head.shape[0]
    if head.shape[1] != D:
        raise ValueError(f"head has {head.shape[1]} columns, rows have {D}")
    row0, rows = vocab_rows(V, peers.rank, peers.world)
    ids = None
    if draft_ids is not None:
        ids = draft_ids.reshape(-1).to(torch.int64).contiguous()
        if ids.numel() != T - 1:
            raise ValueError(f"{ids.numel()} draft ids for {T} rows")
    if out is None:
        am = torch.empty(T, dtype=torch.int64, device=dev)
        n = torch.empty(1, dtype=torch.int32, device=dev)
        nxt = torch.empty(1, dtype=torch.int64, device=dev)
    else:
        am, n, nxt = out
    lib = _lib.load()
    ws = workspace(dev, lib.hs_lm_head_workspace_size(T), "head")
    _launch("hs_lm_head_argmax_ep", x.data_ptr(), head[row0:].data_ptr(), T, D, V, row0, rows, _ptr(ids),
            am.data_ptr(), n.data_ptr(), nxt.data_ptr(), ctypes.byref(peers), ws.data_ptr(), ws.numel(),
            status_word(dev).data_ptr(), _stream(dev))
    return am, n, nxt


# --- RMSNorm / residual add + RMSNorm ---------------------------------------------

def _rows(x: torch.Tensor, name: str) -> torch.Tensor:
    if x.dtype != torch.bfloat16:
        raise TypeError(f"{name} must be bf16")
    return x.contiguous()


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """utils.py:6-9 in one launch: bf16(f32(w) * (f32(x) * rsqrt(mean(f32(x)^2) + eps))) over the last dim."""
    dev = _check_cuda(x, w, out)
    x = _rows(x, "x")
    w = _rows(w, "w")
    D = x.shape[-1]
    if w.numel() != D:
        raise ValueError(f"weight has {w.numel()} elements, rows have {D}")
    if out is None:
        out = torch.empty_like(x)
    _launch("hs_rms_norm", x.data_ptr(), w.data_ptr(), float(eps), x.numel() // D, D, out.data_ptr(), _stream(dev))
    return out


def add_rms_norm(h: torch.Tensor, y: torch.Tensor, w: torch.Tensor, eps: float = 1e-6,
                 h_out: Optional[torch.Tensor] = None, x_out: Optional[torch.Tensor] = None):
    """Residual add then RMSNorm in one launch: returns (bf16(h + y), rms_norm(bf16(h + y), w)).
    h_out may be h itself (in-place residual stream)."""
    dev = _check_cuda(h, y, w, h_out, x_out)
    h = _rows(h, "h")
    y = _rows(y, "y")
    w = _rows(w, "w")
    D = h.shape[-1]
    if y.shape != h.shape or w.numel() != D:
        raise ValueError(f"shapes h {tuple(h.shape)}, y {tuple(y.shape)}, w {tuple(w.shape)} do not match")
    if h_out is None:
        h_out = torch.empty_like(h)
    if x_out is None:
        x_out = torch.empty_like(h)
    _launch("hs_add_rms_norm", h.data_ptr(), y.data_ptr(), w.data_ptr(), float(eps), h.numel() // D, D,
            h_out.data_ptr(), x_out.data_ptr(), _stream(dev))
    return h_out, x_out


def fill_bytes(t: torch.Tensor, seed: int, lo: int = 0, hi: int = 255) -> torch.Tensor:
    """Counter-hash fill of a uint8 tensor with values in [lo, hi] (device side)."""
    dev = _check_cuda(t)
    _launch("hs_fill_bytes", t.data_ptr(), t.numel() * t.element_size(), int(seed) & 0xFFFFFFFFFFFFFFFF, lo, hi,
         _stream(dev))
    return t


__all__ = ["HsError", "router_topk", "hash_route", "make_moe_desc", "moe_ffn", "moe_permute", "moe_unpermute",
           "accept_greedy", "accept_rejection", "lm_head_argmax", "sample", "fill_bytes", "rms_norm", "add_rms_norm", "moe_ffn_partials",
           "moe_route_ffn",
           "moe_combine", "moe_combine_add_rms_norm", "check_status",
           "status_word", "workspace"]
