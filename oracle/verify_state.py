"""CPU restatement of the verify-state handling of `_mtp_verify_batched`
(inference_engine/engine.py:2443-2459 snapshot, 2500-2538 trim / restore).
Test infrastructure: only tests/ use it.

States per layer: the KV latent cache [1, L, d] (appended along dim 1 by the
forward), the compressed KV data / index, and the compressor's
(accumulated, kv_state, score_state). Given the states before the verify
forward and after it, and n_accept of T positions:
  * n_accept < T: KV caches keep their first old_len + n_accept entries
    (engine.py:2500-2508); compressed data / index and compressor states go
    back to their snapshots (engine.py:2509-2518);
  * n_accept == 0: KV caches go back to their snapshots (engine.py:2523-2527),
    which the trim already gave;
  * n_accept == T (never produced by the verify loop, which stops at T - 1):
    everything stays as the forward left it;
  * the position becomes old + n_accept in every case (engine.py:2521).
"""
from __future__ import annotations

import copy


def commit(before: dict, after: dict, n_accept: int, t_total: int, pos_before: int):
    """before / after: {layer: {"kv": tensor [1, L, d], "cdata": tensor or None,
    "cidx": tensor or None, "comp": (accumulated, kv_state, score_state)}}.
    Returns (states, position) after the reference's trim / restore."""
    out = copy.deepcopy(after)
    if n_accept < t_total:
        for l, st in out.items():
            keep = before[l]["kv"].shape[1] + n_accept
            st["kv"] = st["kv"][:, :keep].contiguous()
            st["cdata"] = before[l]["cdata"]
            st["cidx"] = before[l]["cidx"]
            st["comp"] = before[l]["comp"]
    if n_accept == 0:
        for l, st in out.items():
            st["kv"] = before[l]["kv"]
    return out, pos_before + n_accept


# --- the test scenario: states and the mutations the mocked verify forward applies ---

def scenario_states(layers: int = 2, kv_len: int = 5, d: int = 16, seed: int = 7) -> dict:
    """Seeded per-layer states before a verify pass (the layout of
    LayerState / Compressor: kv [1, L, d] bf16, compressed data [1, C, d] bf16
    and index [C] int64, compressor (accumulated, kv_state [4, d] f32,
    score_state [4, d] f32))."""
    import torch
    g = torch.Generator().manual_seed(seed)
    out = {}
    for l in range(layers):
        out[l] = {"kv": torch.randn(1, kv_len + l, d, generator=g).to(torch.bfloat16),
                  "cdata": torch.randn(1, 3, d, generator=g).to(torch.bfloat16),
                  "cidx": torch.arange(3, dtype=torch.int64) * 4 + l,
                  "comp": (3 + l, torch.randn(4, d, generator=g), torch.randn(4, d, generator=g))}
    return out


def forward_rows(ids, layer: int, d: int):
    """The KV rows the mocked forward appends for token ids at a layer."""
    import torch
    ids = torch.as_tensor(ids).reshape(-1).to(torch.float32)
    return (ids.view(-1, 1) * 0.01 + layer + torch.arange(d, dtype=torch.float32) * 0.001).to(torch.bfloat16)


def forward_mutation(st: dict, ids, layer: int) -> None:
    """What the mocked verify forward does to one layer's state (in place):
    appends one KV row per token, appends one compressed row and index, and
    rewrites the compressor (accumulated += T, kv_state += 1 + layer,
    score_state *= 0.5)."""
    import torch
    d = st["kv"].shape[-1]
    T = len(ids)
    st["kv"] = torch.cat([st["kv"], forward_rows(ids, layer, d).unsqueeze(0)], dim=1)
    st["cdata"] = torch.cat([st["cdata"], forward_rows(ids[:1], layer + 100, d).unsqueeze(0)], dim=1)
    st["cidx"] = torch.cat([st["cidx"], torch.tensor([int(st["cidx"][-1]) + 4])])
    acc, kvs, scs = st["comp"]
    st["comp"] = (acc + T, kvs + (1 + layer), scs * 0.5)
