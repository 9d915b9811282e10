"""HBM-resident expert store behind the reference's `_load_expert_weights` API.

Reference being replaced: the four-level expert cache of
inference_engine/engine.py:1033-1335 (GPU hot / GPU bf16 FIFO / pinned CPU FP4
LRU / safetensors mmap; `_load_expert_weights` engine.py:1084-1129,
`_load_expert_fp4_raw` engine.py:1173-1285, `ExpertWeightCache`
expert_cache.py:7-121) and the GPU-resident FP8 shared experts
(`_load_shared_experts_gpu` engine.py:1743-1777). On a B200 every expert of
every layer fits in HBM (43 x 256 x 13,369,344 B = 147.2 GB), so the cache
collapses into one allocation per layer, in the layout the kernels stream.

Layout per layer (what the kernels stream with TMA; see layout.py):
  w13 [E][I/128][D/128][2][128][64] u8 packed e2m1 tiles (w1 tile, w3 tile)
  s13 [E][I/128][D/128][2][512] u8 UE8M0 scale-factor atoms
  w2  [E][D/128][I/128][128][64] u8 packed e2m1 tiles
  s2  [E][D/128][I/128][512] u8 UE8M0 atoms
  sh_w13 [I_sh/128][D/128][2][128][128] e4m3 tiles, sh_s13 [I_sh/128][D/128][2][512]
  atoms of the 128x128 block scales, sh_w2 [D/128][I_sh/128][128][128],
  sh_s2 [D/128][I_sh/128][512]
  gate [E][D] bf16, bias [E] bf16, tid2eid [V][K] int64 (hash layers only)
Every stage of the kernels reads one contiguous 16 KB block of packed weights
(32 KB for the FP8 shared expert) and one contiguous 1 KB pair of scale atoms.
Reference callers get the reference's row-major tensors back as copies
(`_load_expert_fp4_raw`).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Optional

import numpy as np
import torch

from . import ops
from .layout import atoms_to_scales, block_scales_to_atoms, scales_to_atoms, tile_rows, untile_rows


@dataclass
class LayerWeights:
    w13: torch.Tensor
    s13: torch.Tensor
    w2: torch.Tensor
    s2: torch.Tensor
    sh_w13: Optional[torch.Tensor] = None
    sh_s13: Optional[torch.Tensor] = None
    sh_w2: Optional[torch.Tensor] = None
    sh_s2: Optional[torch.Tensor] = None
    gate: Optional[torch.Tensor] = None
    bias: Optional[torch.Tensor] = None
    tid2eid: Optional[torch.Tensor] = None
    desc: Optional[ctypes.Array] = field(default=None, repr=False)


class HBMExpertStore:
    """All routed + shared experts of `num_layers` MoE layers, resident in HBM.

    `expert_ids` restricts the routed experts held (expert parallelism: rank r
    holds a contiguous block); ids outside the block are remapped to -1 by the
    caller before the kernel runs.
    """

    def __init__(self, num_layers: int, num_experts: int = 256, hidden_size: int = 4096,
                 intermediate_size: int = 2048, shared_intermediate_size: Optional[int] = 2048,
                 device: str | torch.device = "cuda", with_router: bool = True, hash_layers: int = 0,
                 vocab_size: int = 129280, top_k: int = 6, expert_offset: int = 0,
                 experts_held: Optional[int] = None):
        self.num_layers = num_layers
        self.E = num_experts
        self.D = hidden_size
        self.I = intermediate_size
        self.I_sh = shared_intermediate_size or 0
        self.device = torch.device(device)
        self.K = top_k
        self.expert_offset = expert_offset
        self.E_local = experts_held if experts_held is not None else num_experts
        E, D, I, Ish = self.E_local, self.D, self.I, self.I_sh
        dev = self.device
        self.layers: list[LayerWeights] = []
        for layer in range(num_layers):
            lw = LayerWeights(
                w13=torch.zeros(E, I // 128, D // 128, 2, 128, 64, dtype=torch.uint8, device=dev),
                s13=torch.zeros(E, I // 128, D // 128, 2, 512, dtype=torch.uint8, device=dev),
                w2=torch.zeros(E, D // 128, I // 128, 128, 64, dtype=torch.uint8, device=dev),
                s2=torch.zeros(E, D // 128, I // 128, 512, dtype=torch.uint8, device=dev),
            )
            if Ish:
                lw.sh_w13 = torch.zeros(Ish // 128, D // 128, 2, 128, 128, dtype=torch.uint8, device=dev)
                lw.sh_s13 = torch.zeros(Ish // 128, D // 128, 2, 512, dtype=torch.uint8, device=dev)
                lw.sh_w2 = torch.zeros(D // 128, Ish // 128, 128, 128, dtype=torch.uint8, device=dev)
                lw.sh_s2 = torch.zeros(D // 128, Ish // 128, 512, dtype=torch.uint8, device=dev)
            if with_router:
                lw.gate = torch.zeros(num_experts, D, dtype=torch.bfloat16, device=dev)
                lw.bias = torch.zeros(num_experts, dtype=torch.bfloat16, device=dev)
            if layer < hash_layers:
                lw.tid2eid = torch.zeros(vocab_size, top_k, dtype=torch.int64, device=dev)
            self.layers.append(lw)

    # --- filling ---------------------------------------------------------------
    def _local(self, eid: int) -> int:
        le = int(eid) - self.expert_offset
        if not 0 <= le < self.E_local:
            raise KeyError(f"expert {eid} is not held by this store")
        return le

    def set_expert(self, layer: int, eid: int, w1, s1, w3, s3, w2, s2) -> None:
        """Copy one routed expert (reference 6-tuple layout, any byte dtype) into place."""
        lw = self.layers[layer]
        le = self._local(eid)

        def dev_u8(a):
            t = torch.from_numpy(np.ascontiguousarray(a)) if isinstance(a, np.ndarray) else a
            return t.contiguous().view(torch.uint8).to(self.device, non_blocking=True)

        lw.w13[le, :, :, 0].copy_(tile_rows(dev_u8(w1), 64))
        lw.w13[le, :, :, 1].copy_(tile_rows(dev_u8(w3), 64))
        lw.s13[le, :, :, 0].copy_(scales_to_atoms(dev_u8(s1)))
        lw.s13[le, :, :, 1].copy_(scales_to_atoms(dev_u8(s3)))
        lw.w2[le].copy_(tile_rows(dev_u8(w2), 64))
        lw.s2[le].copy_(scales_to_atoms(dev_u8(s2)))
        lw.desc = None

    def set_shared(self, layer: int, w13, s13, w2, s2) -> None:
        """Shared expert: e4m3 weights, 128x128 block scales [2][I_sh/128][D/128] and [D/128][I_sh/128]."""
        lw = self.layers[layer]

        def dev_u8(a):
            t = torch.from_numpy(np.ascontiguousarray(a)) if isinstance(a, np.ndarray) else a
            return t.contiguous().view(torch.uint8).to(self.device)

        w13 = dev_u8(w13).reshape(2, self.I_sh, self.D)
        lw.sh_w13[:, :, 0].copy_(tile_rows(w13[0], 128))
        lw.sh_w13[:, :, 1].copy_(tile_rows(w13[1], 128))
        lw.sh_w2.copy_(tile_rows(dev_u8(w2).reshape(self.D, self.I_sh), 128))
        s13 = dev_u8(s13).reshape(2, self.I_sh // 128, self.D // 128)
        lw.sh_s13.copy_(block_scales_to_atoms(s13.permute(1, 2, 0)))
        lw.sh_s2.copy_(block_scales_to_atoms(dev_u8(s2).reshape(self.D // 128, self.I_sh // 128)))
        lw.desc = None

    def set_router(self, layer: int, gate: torch.Tensor, bias: Optional[torch.Tensor]) -> None:
        lw = self.layers[layer]
        lw.gate.copy_(gate.to(torch.bfloat16))
        if bias is not None:
            lw.bias.copy_(bias.to(torch.bfloat16))
        else:
            lw.bias = None

    def fill_random(self, seed: int = 0) -> None:
        """Random-init every weight on the device (bench: full model shape in seconds).

        Packed e2m1 bytes uniform over 0..255, UE8M0 scale bytes over 118..122
        (2^-9..2^-5), e4m3 shared weights over finite codes, shared scales 2^-6,
        gate ~ N(0, 0.02^2), bias ~ N(0, 0.01^2), tid2eid uniform.
        """
        g = torch.Generator(device=self.device)
        for layer, lw in enumerate(self.layers):
            s = seed * 1000003 + layer * 7919
            ops.fill_bytes(lw.w13, s + 1)
            ops.fill_bytes(lw.s13, s + 2, 118, 122)
            ops.fill_bytes(lw.w2, s + 3)
            ops.fill_bytes(lw.s2, s + 4, 118, 122)
            if lw.sh_w13 is not None:
                # e4m3 bytes 0x00..0x7E and 0x80..0xFE are finite; draw from
                # 0..125 and flip the sign bit at random via a second fill
                for t, k in ((lw.sh_w13, 5), (lw.sh_w2, 6)):
                    ops.fill_bytes(t, s + k, 0, 125)
                    sign = torch.empty_like(t)
                    ops.fill_bytes(sign, s + k + 100, 0, 1)
                    t.bitwise_or_(sign << 7)
                lw.sh_s13.fill_(121)
                lw.sh_s2.fill_(121)
            if lw.gate is not None:
                g.manual_seed(s + 7)
                lw.gate.copy_((torch.randn(lw.gate.shape, generator=g, device=self.device) * 0.02).to(torch.bfloat16))
                if lw.bias is not None:
                    lw.bias.copy_((torch.randn(lw.bias.shape, generator=g, device=self.device) * 0.01)
                                  .to(torch.bfloat16))
            if lw.tid2eid is not None:
                g.manual_seed(s + 8)
                lw.tid2eid.copy_(torch.randint(0, self.E, lw.tid2eid.shape, generator=g, device=self.device))
            lw.desc = None

    # --- kernel-facing -----------------------------------------------------------
    def desc(self, layer: int) -> ctypes.Array:
        lw = self.layers[layer]
        if lw.desc is None:
            lw.desc = ops.make_moe_desc(lw.w13, lw.s13, lw.w2, lw.s2, lw.sh_w13, lw.sh_s13, lw.sh_w2, lw.sh_s2)
        return lw.desc

    @property
    def dims(self) -> tuple:
        return (self.E_local, self.D, self.I, self.I_sh)

    def bytes_per_expert(self) -> int:
        return 3 * self.I * self.D // 2 + 3 * self.I * self.D // 32

    def total_bytes(self) -> int:
        n = 0
        for lw in self.layers:
            for t in (lw.w13, lw.s13, lw.w2, lw.s2, lw.sh_w13, lw.sh_s13, lw.sh_w2, lw.sh_s2, lw.gate, lw.bias,
                      lw.tid2eid):
                if t is not None:
                    n += t.numel() * t.element_size()
        return n

    # --- reference-facing format (engine.py:1084-1129, 1173-1285) ---------------
    def _load_expert_fp4_raw(self, layer_idx: int, eid: int):
        """(w1 int8 [I, D/2], s1 e8m0 [I, D/32], w3, s3, w2 int8 [D, I/2], s2 e8m0 [D, I/32]),
        row-major copies out of the tiled store (the kernel path never calls this)."""
        lw = self.layers[layer_idx]
        try:
            le = self._local(eid)
        except KeyError:
            return None
        e8 = torch.float8_e8m0fnu
        return (untile_rows(lw.w13[le, :, :, 0]).view(torch.int8), atoms_to_scales(lw.s13[le, :, :, 0]).view(e8),
                untile_rows(lw.w13[le, :, :, 1]).view(torch.int8), atoms_to_scales(lw.s13[le, :, :, 1]).view(e8),
                untile_rows(lw.w2[le]).view(torch.int8), atoms_to_scales(lw.s2[le]).view(e8))

    def _load_expert_weights(self, layer_idx: int, eid: int):
        """Reference triple format: ((data, scale, "fp4_gpu"), w3 entry, w2 entry)."""
        raw = self._load_expert_fp4_raw(layer_idx, eid)
        if raw is None:
            return None
        w1, s1, w3, s3, w2, s2 = raw
        return ((w1, s1, "fp4_gpu"), (w3, s3, "fp4_gpu"), (w2, s2, "fp4_gpu"))

    def loader(self):
        """A `load_expert_fn(layer, eid)` for FusedMoEFFN.forward; the kernel path
        recognises it and reads the store directly (no per-expert calls)."""
        store = self

        def load_expert_fn(layer_idx, eid):
            return store._load_expert_fp4_raw(layer_idx, eid)

        load_expert_fn.__hs_store__ = store
        return load_expert_fn
