"""CPU restatement of the routed + shared MoE FFN, the router and hash routing.

Operation order and every rounding follow the reference exactly (torch CPU
ops on bf16 tensors), so for the same inputs this oracle reproduces the
reference's own CPU outputs bit for bit (checked against golden vectors).
"""
from __future__ import annotations

from typing import Callable, Optional

import numpy as np
import torch
import torch.nn.functional as F

from .fp4 import dequant_fp4, dequant_fp8_block

SWIGLU_LIMIT = 10.0


def stable_topk(scores: torch.Tensor, k: int) -> torch.Tensor:
    """router.py:5-7: stable descending sort, first k indices."""
    _, order = torch.sort(scores, dim=1, descending=True, stable=True)
    return order[:, :k].contiguous()


def router(hidden: torch.Tensor, gate: torch.Tensor, bias: Optional[torch.Tensor], top_k: int = 6,
           routed_scaling: float = 1.5, return_logits: bool = False):
    """router.py:22-36 (compute_expert_affinity_with_bias); bias=None gives router.py:10-19."""
    logits = torch.matmul(hidden.to(gate.dtype), gate.t())
    if bias is not None:
        logits = logits + bias.to(logits.dtype)
    lb = logits
    logits = logits.float()
    scores = F.softplus(logits).sqrt()
    idx = stable_topk(scores, top_k)
    raw = scores.gather(1, idx)
    s = raw.sum(dim=-1, keepdim=True).clamp(min=1e-20)
    w = raw / s * routed_scaling
    if return_logits:
        return idx, w, lb
    return idx, w


def router_from_logits(logits_bf16: torch.Tensor, top_k: int = 6, routed_scaling: float = 1.5):
    """router.py:30-36 applied to already-rounded (post-bias) bf16 logits."""
    scores = F.softplus(logits_bf16.float()).sqrt()
    idx = stable_topk(scores, top_k)
    raw = scores.gather(1, idx)
    s = raw.sum(dim=-1, keepdim=True).clamp(min=1e-20)
    return idx, raw / s * routed_scaling


def hash_route(input_ids: torch.Tensor, tid2eid: torch.Tensor, top_k: int = 6):
    """engine.py:1018-1023 (_compute_hash_experts): eids = tid2eid[ids], w = 1/k."""
    eids = tid2eid[input_ids]
    w = torch.full(tuple(input_ids.shape) + (top_k,), 1.0 / top_k)
    return eids, w


def _ffn_cat(h, w1, w3, w2, ew=None):
    """The GEMM/SwiGLU sequence of fused_moe.py:519-551 (cuBLAS branch)."""
    gate = h @ w1.T
    up = h @ w3.T
    g = gate.float().clamp(max=SWIGLU_LIMIT)
    u = up.float().clamp(min=-SWIGLU_LIMIT, max=SWIGLU_LIMIT)
    act = (g * g.sigmoid() * u).to(torch.bfloat16)
    if ew is not None:
        B = h.shape[0]
        n = ew.shape[1]
        act = (act.view(B, n, -1) * ew.unsqueeze(-1)).reshape(B, -1)
    return act @ w2.T


def moe_routed(hidden: torch.Tensor, topk_idx: torch.Tensor, topk_w: torch.Tensor,
               load_fp4: Callable[[int], tuple], dup_mode: str = "last") -> torch.Tensor:
    """fused_moe.py:458-551 (FusedMoEFFN._forward_legacy), 6-tuple FP4 loader.

    load_fp4(eid) -> (w1 u8 [I, D/2], s1 u8 [I, D/32], w3, s3, w2 u8 [D, I/2], s2 u8 [D, I/32]).
    dup_mode "last": duplicate experts in a row keep the last weight (index_put);
    "sum": weights of duplicates are summed (engine.py:1388-1393, the T=1 path).
    """
    B, D = hidden.shape
    K = topk_idx.shape[1]
    eids = sorted({int(e) for e in topk_idx.flatten().tolist() if e >= 0})
    if not eids:
        return torch.zeros_like(hidden)
    loaded = {}
    for e in eids:
        w1, s1, w3, s3, w2, s2 = load_fp4(e)
        loaded[e] = (dequant_fp4(w1, s1), dequant_fp4(w3, s3), dequant_fp4(w2, s2))
    W1 = torch.cat([loaded[e][0] for e in eids], dim=0)
    W3 = torch.cat([loaded[e][1] for e in eids], dim=0)
    W2 = torch.cat([loaded[e][2] for e in eids], dim=1)
    pos = {e: i for i, e in enumerate(eids)}
    ew = torch.zeros(B, len(eids), dtype=torch.bfloat16)
    if dup_mode == "sum":
        acc = {}
        for b in range(B):
            for k in range(K):
                e = int(topk_idx[b, k])
                if e >= 0:
                    acc[(b, e)] = acc.get((b, e), 0.0) + float(topk_w[b, k])
        for (b, e), v in acc.items():
            ew[b, pos[e]] = torch.tensor(v, dtype=torch.float32).to(torch.bfloat16)
    else:
        for b in range(B):
            for k in range(K):
                e = int(topk_idx[b, k])
                if e >= 0:
                    ew[b, pos[e]] = topk_w[b, k].to(torch.bfloat16)
    return _ffn_cat(hidden, W1, W3, W2, ew)


def shared_expert(hidden: torch.Tensor, sh: tuple) -> torch.Tensor:
    """weight_loader.py:22-32 + fused_moe.py:383-392 (fused_expert_ffn_pt) for M <= 8.

    sh = (w13 e4m3 u8 [2, I_sh, D], s13 u8 [2, I_sh/128, D/128], w2 u8 [D, I_sh], s2 u8 [D/128, I_sh/128]).
    """
    w13, s13, w2, s2 = sh
    w1 = dequant_fp8_block(w13[0], s13[0])
    w3 = dequant_fp8_block(w13[1], s13[1])
    w2b = dequant_fp8_block(w2, s2)
    return _ffn_cat(hidden, w1, w3, w2b)


def shared_expert_f32(hidden: torch.Tensor, sh: tuple) -> torch.Tensor:
    """The shared expert's output before its bf16 rounding (f32), for the
    expert-parallel combine: a slice of its intermediate rows gives a partial
    sum, and the slices' sum is the full output."""
    w13, s13, w2, s2 = sh
    w1 = dequant_fp8_block(w13[0], s13[0])
    w3 = dequant_fp8_block(w13[1], s13[1])
    w2b = dequant_fp8_block(w2, s2)
    gate = hidden @ w1.T
    up = hidden @ w3.T
    g = gate.float().clamp(max=SWIGLU_LIMIT)
    u = up.float().clamp(min=-SWIGLU_LIMIT, max=SWIGLU_LIMIT)
    act = (g * g.sigmoid() * u).to(torch.bfloat16)
    return act.float() @ w2b.float().T


def ep_combine(routed_f32: torch.Tensor, shared_f32: Optional[torch.Tensor]) -> torch.Tensor:
    """engine.py:1530-1536 applied to f32 sums: bf16(bf16(routed) + bf16(shared))."""
    out = routed_f32.to(torch.bfloat16)
    if shared_f32 is not None:
        out = out + shared_f32.to(torch.bfloat16)
    return out


def moe_layer(hidden, topk_idx, topk_w, load_fp4, sh=None, dup_mode="last"):
    """engine.py:1480-1536: routed output (bf16) + shared output (bf16), bf16 add."""
    out = moe_routed(hidden, topk_idx, topk_w, load_fp4, dup_mode)
    if sh is not None:
        out = out + shared_expert(hidden, sh)
    return out


def moe_routed_f32(hidden, topk_idx, topk_w, load_fp4):
    """The routed sum before its final bf16 rounding (f32), for the EP combine checks."""
    B, D = hidden.shape
    out = torch.zeros(B, D, dtype=torch.float32)
    eids = sorted({int(e) for e in topk_idx.flatten().tolist() if e >= 0})
    for e in eids:
        w1, s1, w3, s3, w2, s2 = load_fp4(e)
        W1, W3, W2 = dequant_fp4(w1, s1), dequant_fp4(w3, s3), dequant_fp4(w2, s2)
        for b in range(B):
            ks = [k for k in range(topk_idx.shape[1]) if int(topk_idx[b, k]) == e]
            if not ks:
                continue
            wb = topk_w[b, ks[-1]].to(torch.bfloat16)
            h = hidden[b:b + 1]
            g = (h @ W1.T).float().clamp(max=SWIGLU_LIMIT)
            u = (h @ W3.T).float().clamp(min=-SWIGLU_LIMIT, max=SWIGLU_LIMIT)
            a = (g * g.sigmoid() * u).to(torch.bfloat16) * wb
            out[b] += (a.float() @ W2.float().T)[0]
    return out


def permute_plan(topk_idx: np.ndarray, E: int):
    """Expert-major positions: ascending expert id, then ascending (token, k).

    Returns token_topk_to_pos [T, K] int32 (-1 invalid), pos_to_expert [T*K]
    (-1 past the end), expert_count [E], num_pos. This is the mapping the
    kernels use; its expand/reduce semantics are those of
    tests/_reference.py:52-121.
    """
    idx = np.asarray(topk_idx)
    T, K = idx.shape
    counts = np.zeros(E, dtype=np.int64)
    for e in idx.flatten():
        if 0 <= e < E:
            counts[e] += 1
    base = np.concatenate([[0], np.cumsum(counts)[:-1]])
    cursor = base.copy()
    pos = np.full((T, K), -1, dtype=np.int32)
    p2e = np.full(T * K, -1, dtype=np.int32)
    for e in range(E):
        for t in range(T):
            for k in range(K):
                if idx[t, k] == e:
                    pos[t, k] = cursor[e]
                    p2e[cursor[e]] = e
                    cursor[e] += 1
    return pos, p2e, counts.astype(np.int32), int(counts.sum())


def expand(x: torch.Tensor, token_topk_to_pos: np.ndarray, n_rows: int) -> torch.Tensor:
    """tests/_reference.py:108-121 (expand_to_fused)."""
    T, D = x.shape
    out = torch.zeros(n_rows, D, dtype=x.dtype)
    for t in range(T):
        for k in range(token_topk_to_pos.shape[1]):
            p = int(token_topk_to_pos[t, k])
            if p >= 0:
                out[p] = x[t]
    return out


def reduce(xe: torch.Tensor, topk_w: Optional[torch.Tensor], token_topk_to_pos: np.ndarray) -> torch.Tensor:
    """tests/_reference.py:52-90 (reduce_fused) without FP8: sum_k w*x[pos] in f32, k order."""
    T, K = token_topk_to_pos.shape
    out = torch.zeros(T, xe.shape[1], dtype=torch.float32)
    for k in range(K):
        for t in range(T):
            p = int(token_topk_to_pos[t, k])
            if p >= 0:
                s = float(topk_w[t, k]) if topk_w is not None else 1.0
                out[t] = xe[p].float() * torch.tensor(s, dtype=torch.float32) + out[t]
    return out.to(xe.dtype)
