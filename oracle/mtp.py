"""CPU restatement of the MTP decode step over the MoE path (test infrastructure:
only tests/, smoke() and bench.py's CPU baseline use it).

The layer body is the part of the reference's `_forward_layer` that the CUDA
path owns: ffn_norm (inference_engine/engine.py:2679, utils.py:6-9) -> router
or hash routing (engine.py:1018-1031) -> routed FP4 experts + FP8 shared
expert (engine.py:1480-1536) -> residual add (engine.py:2685). The final norm
and lm_head follow engine.py:2482; the draft step follows `_mtp_generate_draft`
at t = 0 (engine.py:2289-2336: enorm(embed(tok)) @ e_proj + hnorm(h) @ h_proj,
the MTP layer's MoE, its own norm, lm_head, argmax); acceptance is
oracle.accept.greedy.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Optional

import numpy as np
import torch

from . import accept as A
from . import moe as O


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """utils.py:6-9."""
    variance = x.to(torch.float32).pow(2).mean(-1, keepdim=True)
    x_normed = x.to(torch.float32) * torch.rsqrt(variance + eps)
    return (weight.to(torch.float32) * x_normed).to(x.dtype)


@dataclass
class LayerWeights:
    load_fp4: Callable[[int], tuple]      # eid -> (w1, s1, w3, s3, w2, s2) u8, reference layout
    shared: Optional[tuple] = None         # (w13, s13, w2, s2) e4m3 + block scales
    gate: Optional[torch.Tensor] = None    # [E, D] bf16
    bias: Optional[torch.Tensor] = None    # [E] bf16
    tid2eid: Optional[torch.Tensor] = None  # [V, K] int64 (hash layers)


@dataclass
class ModelWeights:
    layers: list                            # num_layers + 1 LayerWeights (the last is the MTP layer)
    embed: torch.Tensor
    lm_head: torch.Tensor
    norm_w: torch.Tensor
    ln_w: torch.Tensor                      # [num_layers + 1, D]
    e_proj: torch.Tensor
    h_proj: torch.Tensor
    enorm_w: torch.Tensor
    hnorm_w: torch.Tensor
    mtp_norm_w: torch.Tensor
    top_k: int = 6
    hash_layers: int = 3
    routed_scaling: float = 1.5
    num_draft: int = 2
    route_log: list = field(default_factory=list)


def moe(W: ModelWeights, x: torch.Tensor, layer: int, ids: torch.Tensor) -> torch.Tensor:
    """One MoE layer on normed rows x [T, D]; T = 1 sums duplicate weights
    (engine.py:1388-1393), T > 1 keeps the last (index_put)."""
    lw = W.layers[layer]
    if layer < W.hash_layers and lw.tid2eid is not None:
        idx, w = O.hash_route(ids, lw.tid2eid, W.top_k)
    else:
        idx, w = O.router(x, lw.gate, lw.bias, W.top_k, W.routed_scaling)
    W.route_log.append((layer, idx.clone()))
    return O.moe_layer(x, idx, w, lw.load_fp4, lw.shared, "sum" if x.shape[0] == 1 else "last")


def forward(W: ModelWeights, ids: torch.Tensor, num_layers: int):
    """-> (h, x): residual stream after the last layer and its final norm."""
    h = W.embed[ids]
    for layer in range(num_layers):
        h = h + moe(W, rms_norm(h, W.ln_w[layer]), layer, ids)
    return h, rms_norm(h, W.norm_w)


def logits(W: ModelWeights, x_normed: torch.Tensor) -> torch.Tensor:
    return x_normed @ W.lm_head.t()


def draft_step(W: ModelWeights, prev: torch.Tensor, tok: torch.Tensor, num_layers: int):
    """One MTP draft step: -> (hm, logits [1, V])."""
    L = num_layers
    e = rms_norm(W.embed[tok], W.enorm_w) @ W.e_proj.t()
    hc = rms_norm(prev, W.hnorm_w) @ W.h_proj.t() + e
    hm = hc + moe(W, rms_norm(hc, W.ln_w[L]), L, tok)
    return hm, rms_norm(hm, W.mtp_norm_w) @ W.lm_head.t()


def greedy_tokens(lg: torch.Tensor) -> np.ndarray:
    """argmax per row with torch.argmax's tie rule."""
    a = lg.float().numpy()
    return np.array([A._argmax_first(r) for r in a], dtype=np.int64)
