"""Router entry points with the reference's names and signatures
(home_seek/router.py:5-36, inference_engine/engine.py:1018-1031), running on
the sm_100a kernels."""
from __future__ import annotations

from typing import Optional

import torch

from . import ops


def compute_expert_affinity_with_bias(hidden_states: torch.Tensor, gate_weight: torch.Tensor,
                                      gate_bias: Optional[torch.Tensor], top_k: int = 6,
                                      routed_scaling_factor: float = 1.5):
    """router.py:22-36 -> (topk_indices int64 [T, k], topk_weights f32 [T, k])."""
    shape = hidden_states.shape
    h = hidden_states.reshape(-1, shape[-1]).contiguous()
    idx, w = ops.router_topk(h, gate_weight.contiguous(), None if gate_bias is None else gate_bias.contiguous(),
                             top_k, routed_scaling_factor)
    return idx, w


def compute_expert_affinity(hidden_states: torch.Tensor, gate_weight: torch.Tensor, top_k: int = 6,
                            routed_scaling_factor: float = 1.5):
    """router.py:10-19 (no bias)."""
    return compute_expert_affinity_with_bias(hidden_states, gate_weight, None, top_k, routed_scaling_factor)


def compute_hash_experts(input_ids: torch.Tensor, tid2eid: torch.Tensor, top_k: int = 6):
    """engine.py:1018-1023 (_compute_hash_experts) -> (eids [B, T, k], weights [B, T, k] = 1/k)."""
    return ops.hash_route(input_ids, tid2eid, top_k)
