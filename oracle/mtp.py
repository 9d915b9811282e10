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


def weights_from_inputs(model: dict, num_layers: int, hash_layers: int, top_k: int = 6,
                        num_draft: int = 2) -> ModelWeights:
    """ModelWeights over the tensors of oracle.inputs.mtp_model (layers 0..L-1,
    then the MTP layer, which has no shared expert)."""
    layers = []
    for l in range(num_layers + 1):
        layers.append(LayerWeights(model["experts"][l], model["shared"][l] if l < num_layers else None,
                                   model["gate"][l], model["bias"][l], model["tid2eid"].get(l)))
    return ModelWeights(layers, model["embed"], model["lm_head"], model["norm_w"], model["ln_w"], model["e_proj"],
                        model["h_proj"], model["enorm_w"], model["hnorm_w"], model["mtp_norm_w"], top_k,
                        hash_layers, 1.5, num_draft)


def decode_loop(W: ModelWeights, first_token: int, iterations: int, num_layers: int):
    """generate()'s MTP loop at temperature 0 (engine.py:2809-2922, no stop
    token, no token budget reached): per iteration the main T = 1 step
    (engine.py:2811-2853), the M-step draft (_mtp_generate_draft,
    engine.py:2251-2336), the fused T = 1 + M verify with its greedy loop
    (_mtp_verify_batched, engine.py:2431-2497) and the bookkeeping
    (engine.py:2885-2916): append main_pred; if n_acc > 0 append the n_acc
    accepted drafts and the bonus token argmax(logits[n_acc]), which becomes
    the next input; else the next input is main_pred.

    Returns (tokens, records, logits) with records rows (main input, main_pred,
    drafts..., n_acc, next input) and logits {"main": [N, V], "draft": [N, M,
    V], "verify": [N, M + 1, V]}, the rows every argmax was taken of.
    """
    M = W.num_draft
    next_id = int(first_token)
    tokens, recs = [], []
    lg_main, lg_draft, lg_verify = [], [], []
    for _ in range(iterations):
        h, x = forward(W, torch.tensor([next_id]), num_layers)
        lg = logits(W, x)
        main_in, main_pred = next_id, int(greedy_tokens(lg)[0])
        tokens.append(main_pred)
        prev, tok = h, torch.tensor([main_pred])
        d, rows = [], []
        for _i in range(M):
            prev, lgd = draft_step(W, prev, tok, num_layers)
            t = int(greedy_tokens(lgd)[0])
            d.append(t)
            rows.append(lgd[0])
            tok = torch.tensor([t])
        _, xv = forward(W, torch.tensor([main_pred] + d), num_layers)
        lv = logits(W, xv)
        n_a, nxt, _ = A.greedy(lv.float().numpy()[None], np.array([d], dtype=np.int64))
        n = int(n_a[0])
        if n > 0:
            tokens.extend(d[:n])
            next_id = int(nxt[0])
            tokens.append(next_id)
        else:
            next_id = main_pred
        recs.append([main_in, main_pred] + d + [n, next_id])
        lg_main.append(lg[0])
        lg_draft.append(torch.stack(rows))
        lg_verify.append(lv)
    return (np.array(tokens, dtype=np.int64), np.array(recs, dtype=np.int64),
            {"main": torch.stack(lg_main), "draft": torch.stack(lg_draft), "verify": torch.stack(lg_verify)})
