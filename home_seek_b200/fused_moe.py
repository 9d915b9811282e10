"""FusedMoEFFN / SharedExpertFFN with the reference's operator surface, running
on the sm_100a kernels.

Reference: home_seek/fused_moe.py:402-598. `FusedMoEFFN.forward(hidden_states
[T, D] bf16, topk_idx [T, k] int64, topk_weights [T, k] f32, load_expert_fn,
layer_idx) -> [T, D] bf16` keeps its signature and its numerics
(fused_moe.py:458-551: bf16 gate/up, SwiGLU clamp 10 in f32, bf16 activation,
bf16 routing-weight multiply, one f32 accumulation over all experts, bf16
output). Two loader kinds are accepted:
  * HBMExpertStore.loader(): the kernel reads the store directly; no host
    synchronisation and no per-expert Python work;
  * any reference loader returning FP4 6-tuples (w1, s1, w3, s3, w2, s2): the
    touched experts are gathered once into a compact device store (like the
    reference's torch.cat at fused_moe.py:515-517) and the same kernel runs;
  * a loader returning the BF16 3-tuples the reference's T >= 2 path passes
    (`_bf16_load`, engine.py:1480-1486: FP4 experts dequantised to bf16): each
    weight is turned back into packed e2m1 + UE8M0 losslessly
    (layout.fp4_block_from_bf16) and gathered the same way; a bf16 weight that
    is not an FP4 block-scaled value raises TypeError.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch

from . import ops
from ._lib import HS_DUP_LAST, HS_DUP_SUM


def _e8m0_bytes(scale: torch.Tensor) -> torch.Tensor:
    """Scale tensor (float8_e8m0fnu, uint8, or float32 powers of two) -> UE8M0 bytes."""
    if scale.dtype == torch.float8_e8m0fnu or scale.dtype == torch.uint8:
        return scale.contiguous().view(torch.uint8)
    if scale.dtype == torch.float32:
        bits = scale.contiguous().view(torch.int32)
        e = (bits >> 23) & 0xFF
        return torch.where(bits == 0x00400000, torch.zeros_like(e), e).to(torch.uint8)
    raise TypeError(f"unsupported scale dtype {scale.dtype}")


class _PackedLayer:
    """A compact per-call store built from a reference loader's 6-tuples."""

    def __init__(self, tuples: list, device):
        from .expert_store import HBMExpertStore
        w1 = tuples[0][0]
        I, Dh = w1.shape
        D = Dh * 2
        self.store = HBMExpertStore(1, num_experts=len(tuples), hidden_size=D, intermediate_size=I,
                                    shared_intermediate_size=None, device=device, with_router=False)
        for i, (a, sa, b, sb, c, sc) in enumerate(tuples):
            self.store.set_expert(0, i, a.to(device), _e8m0_bytes(sa).to(device), b.to(device),
                                  _e8m0_bytes(sb).to(device), c.to(device), _e8m0_bytes(sc).to(device))


class FusedMoEFFN:
    def __init__(self, num_experts: int = 256, intermediate_size: int = 2048, hidden_size: int = 4096,
                 swiglu_limit: float = 10.0, use_triton: bool = True, triton_blocks=(16, 32, 64),
                 cublas_max_tokens: int = 8):
        if swiglu_limit != 10.0:
            raise ValueError("the kernels implement swiglu_limit = 10 (model_config.py:25)")
        self.num_experts = num_experts
        self.intermediate_size = intermediate_size
        self.hidden_size = hidden_size
        self.swiglu_limit = swiglu_limit
        self.use_triton = False  # no Triton anywhere on this path

    def forward(self, hidden_states: torch.Tensor, topk_idx: torch.Tensor, topk_weights: torch.Tensor,
                load_expert_fn: Callable, layer_idx: int, use_shared: bool = False,
                dup_mode: int = HS_DUP_LAST, out_f32: Optional[torch.Tensor] = None) -> torch.Tensor:
        store = getattr(load_expert_fn, "__hs_store__", None)
        if store is not None:
            idx = topk_idx
            if store.expert_offset or store.E_local != store.E:
                idx = _localise(topk_idx, store.expert_offset, store.E_local)
            return ops.moe_ffn(store.desc(layer_idx), store.dims, hidden_states, idx, topk_weights,
                               use_shared=use_shared, dup_mode=dup_mode, out_f32=out_f32)
        return self._forward_loader(hidden_states, topk_idx, topk_weights, load_expert_fn, layer_idx, dup_mode)

    def _forward_loader(self, hidden_states, topk_idx, topk_weights, load_expert_fn, layer_idx, dup_mode):
        # one host sync, as the reference's own .item() loop (fused_moe.py:466-471)
        eids = sorted({int(e) for e in topk_idx.flatten().tolist() if e >= 0})
        if not eids:
            return torch.zeros_like(hidden_states)
        tuples, kept = [], []
        for e in eids:
            v = load_expert_fn(layer_idx, e)
            if v is None:
                continue
            if len(v) == 3:  # bf16 (w1, w3, w2) of FP4 weights: back to the packed form
                from .layout import fp4_block_from_bf16
                (a, sa), (b, sb), (c, sc) = (fp4_block_from_bf16(x.to(torch.bfloat16)) for x in v)
                v = (a, sa, b, sb, c, sc)
            elif len(v) != 6:
                raise TypeError("load_expert_fn must return FP4 6-tuples or their BF16 3-tuples")
            tuples.append(v)
            kept.append(e)
        if not tuples:
            return torch.zeros_like(hidden_states)
        packed = _PackedLayer(tuples, hidden_states.device)
        remap = torch.full((max(kept) + 1,), -1, dtype=torch.int64, device=hidden_states.device)
        remap[torch.tensor(kept, device=hidden_states.device)] = torch.arange(len(kept), device=hidden_states.device)
        idx = topk_idx.to(hidden_states.device)
        ok = (idx >= 0) & (idx <= max(kept))
        local = torch.where(ok, remap[idx.clamp(min=0, max=max(kept))], torch.full_like(idx, -1))
        return ops.moe_ffn(packed.store.desc(0), packed.store.dims, hidden_states, local, topk_weights,
                           use_shared=False, dup_mode=dup_mode)

    def forward_m1_fp4(self, hidden_states: torch.Tensor, fp4_data: dict, routing_w: dict) -> torch.Tensor:
        """fused_moe.py:553-563: T=1, dict eid -> 6-tuple and eid -> summed weight."""
        eids = list(fp4_data)
        idx = torch.tensor([eids], dtype=torch.int64, device=hidden_states.device)
        w = torch.tensor([[float(routing_w.get(e, 0.0)) for e in eids]], dtype=torch.float32,
                         device=hidden_states.device)
        return self._forward_loader(hidden_states, idx, w, lambda l, e: fp4_data[e], 0, HS_DUP_SUM)


def _localise(topk_idx: torch.Tensor, offset: int, n_local: int) -> torch.Tensor:
    """Global expert ids -> ids local to a store holding [offset, offset + n_local); others -1."""
    local = topk_idx - offset
    return torch.where((topk_idx >= offset) & (local < n_local), local, torch.full_like(local, -1))


class SharedExpertFFN:
    """fused_moe.py:573-598: the FP8 shared expert, alone (the fused MoE call
    normally runs it in the same launches as the routed experts).

    forward(hidden_states [B, T, D], w1, w3, w2, dtype) takes the reference's
    arguments (fused_moe.py:585). Each weight is either the FP8 form the
    reference keeps before load_fp8_weight, a (e4m3 [R, C], UE8M0 128x128 block
    scales [R/128, C/128]) pair, or the bf16 tensor load_fp8_weight returned
    (engine.py:1451, 1469, 1534 pass those), which is turned back into the
    FP8 form losslessly (layout.fp8_block_from_bf16; a bf16 weight that is not
    an FP8 block-scaled value raises TypeError). The packed weights are built
    once per weight set and kept. forward(hidden_states, store, layer_idx,
    dtype) runs the shared expert held by an HBMExpertStore layer."""

    def __init__(self, hidden_size: int = 4096, intermediate_size: int = 2048, swiglu_limit: float = 10.0,
                 use_triton: bool = True, triton_blocks=(16, 32, 64), cublas_max_tokens: int = 8):
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.swiglu_limit = swiglu_limit
        self.use_triton = False
        self._packed: dict = {}

    @staticmethod
    def _fp8(w) -> tuple:
        from .layout import fp8_block_from_bf16
        if isinstance(w, (tuple, list)):
            data, scale = w
            return data.contiguous().view(torch.uint8), _e8m0_bytes(scale)
        if isinstance(w, torch.Tensor) and w.dtype == torch.bfloat16:
            return fp8_block_from_bf16(w)
        raise TypeError("shared-expert weights must be (e4m3, block scale) pairs or bf16 FP8 values")

    def _store_for(self, w1, w3, w2, device):
        """A one-layer store holding this shared expert (no routed expert is used),
        built once per weight set."""
        from .expert_store import HBMExpertStore
        key = tuple((w[0] if isinstance(w, (tuple, list)) else w).data_ptr() for w in (w1, w3, w2))
        st = self._packed.get(key)
        if st is not None:
            return st
        (a, sa), (b, sb), (c, sc) = (self._fp8(w) for w in (w1, w3, w2))
        I_sh, D = a.shape
        st = HBMExpertStore(1, num_experts=1, hidden_size=D, intermediate_size=512, shared_intermediate_size=I_sh,
                            device=device, with_router=False)
        st.set_shared(0, torch.stack([a, b]).to(device), torch.stack([sa, sb]).to(device), c.to(device),
                      sc.to(device))
        self._packed[key] = st
        return st

    def forward(self, hidden_states: torch.Tensor, w1, w3=None, w2=None, dtype: torch.dtype = torch.bfloat16):
        if hasattr(w1, "desc") and hasattr(w1, "layers"):  # (store, layer_idx[, dtype])
            store, layer_idx = w1, int(w3)
            if isinstance(w2, torch.dtype):
                dtype = w2
        else:
            store, layer_idx = self._store_for(w1, w3, w2, hidden_states.device), 0
        B, T, D = hidden_states.shape
        h = hidden_states.reshape(-1, D).contiguous()
        none = torch.full((h.shape[0], 1), -1, dtype=torch.int64, device=h.device)
        zero = torch.zeros((h.shape[0], 1), dtype=torch.float32, device=h.device)
        out = ops.moe_ffn(store.desc(layer_idx), store.dims, h, none, zero, use_shared=True)
        return out.reshape(B, T, D).to(dtype)
