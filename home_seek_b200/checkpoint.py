"""Reference-format safetensors checkpoint -> HBMExpertStore, streamed once.

Reference being replaced: `WeightLoader` (inference_engine/weight_loader.py:
48-125: the key -> file index from model.safetensors.index.json or a scan of
the *.safetensors files, mmap'd `safe_open` handles) together with the MoE
reads of the engine: routed experts `layers.{l}.ffn.experts.{e}.w{1,3,2}.
{weight,scale}` (engine.py:1084-1129; packed e2m1 int8 [I, D/2] / [D, I/2] and
UE8M0 [I, D/32] / [D, I/32] scales), the FP8 shared expert
`layers.{l}.ffn.shared_experts.w{1,3,2}.{weight,scale}` (engine.py:1743-1777;
e4m3 with 128x128 UE8M0 block scales) and the router `ffn.gate.{weight,scale,
bias,tid2eid}` (engine.py:1413-1415, 1586-1588; an e4m3 gate is dequantised
with its 128x128 block scales, weight_loader.py:22-32). The MTP layer's MoE
uses the prefix `mtp.0`.

The reference keeps the experts on pinned host memory (or mmap) and copies each
one to the GPU when a token routes to it; here every tensor is read once from
the mmap and written into the store's tiled layout on the device, where it
stays. Expert parallelism: `rank`/`world` load only that rank's routed experts
and its rows of the shared expert (the split of `ep.shard_store`).
"""
from __future__ import annotations

import json
import os
import re
from typing import Optional, Sequence

import torch

from .expert_store import HBMExpertStore

_EXPERT = re.compile(r"^(?P<prefix>.+)\.ffn\.experts\.(?P<eid>\d+)\.w1\.weight$")


class CheckpointIndex:
    """key -> safetensors file, as WeightLoader._build_index (weight_loader.py:62-80)."""

    def __init__(self, weight_dir: str):
        from safetensors import safe_open  # noqa: F401  (fail early when the package is missing)
        self.weight_dir = weight_dir
        self.weight_map: dict[str, str] = {}
        self._handles: dict[str, object] = {}
        idx = os.path.join(weight_dir, "model.safetensors.index.json")
        if os.path.exists(idx):
            with open(idx) as f:
                self.weight_map = dict(json.load(f)["weight_map"])
        else:
            for fname in sorted(os.listdir(weight_dir)):
                if fname.endswith(".safetensors"):
                    with self._open(fname) as h:
                        for k in h.keys():
                            self.weight_map[k] = fname
            self._handles.clear()

    def _open(self, fname: str):
        from safetensors import safe_open
        return safe_open(os.path.join(self.weight_dir, fname), framework="pt", device="cpu")

    def get(self, key: str) -> Optional[torch.Tensor]:
        fname = self.weight_map.get(key)
        if fname is None:
            return None
        h = self._handles.get(fname)
        if h is None:
            h = self._open(fname).__enter__()
            self._handles[fname] = h
        return h.get_tensor(key)

    def require(self, key: str) -> torch.Tensor:
        t = self.get(key)
        if t is None:
            raise KeyError(f"checkpoint has no tensor {key!r}")
        return t

    def prefixes(self) -> list[str]:
        """MoE layer prefixes that hold routed experts, in layer order (then mtp.*)."""
        found = {m.group("prefix") for k in self.weight_map if (m := _EXPERT.match(k))}

        def order(p: str):
            m = re.match(r"^layers\.(\d+)$", p)
            return (0, int(m.group(1)), p) if m else (1, 0, p)
        return sorted(found, key=order)

    def num_experts(self, prefix: str) -> int:
        ids = [int(m.group("eid")) for k in self.weight_map if (m := _EXPERT.match(k)) and m.group("prefix") == prefix]
        return max(ids) + 1 if ids else 0

    def close(self) -> None:
        for h in self._handles.values():
            h.__exit__(None, None, None)
        self._handles.clear()


def _ue8m0_bytes(scale: torch.Tensor, what: str) -> torch.Tensor:
    """Scale factors as UE8M0 bytes: 1-byte tensors as they are; wider floats
    (the reference's _ue8m0_to_f32 accepts either) must be powers of two."""
    if scale.element_size() == 1:
        return scale.contiguous().view(torch.uint8)
    f = scale.to(torch.float32)
    m, e = torch.frexp(f)
    if not bool(((m == 0.5) & (f > 0)).all()):
        raise ValueError(f"{what}: scale factors must be positive powers of two (UE8M0) for the FP4/FP8 kernels")
    return (e - 1 + 127).clamp(0, 254).to(torch.uint8)


def _dequant_block128(data: torch.Tensor, scale: Optional[torch.Tensor]) -> torch.Tensor:
    """e4m3 weight x 128x128 block scale -> bf16 (weight_loader.py:22-32)."""
    if data.dtype in (torch.bfloat16, torch.float32, torch.float16):
        return data.to(torch.bfloat16)
    x = data.to(torch.float32)
    if scale is not None:
        if scale.element_size() == 1:
            sf = (scale.contiguous().view(torch.uint8).to(torch.int32) << 23).view(torch.float32)
        else:
            sf = scale.to(torch.float32)
        sf = sf.repeat_interleave(128, 0).repeat_interleave(128, 1)[:x.shape[0], :x.shape[1]]
        x = x * sf
    return x.to(torch.bfloat16)


def load_expert_store(weight_dir: str, prefixes: Optional[Sequence[str]] = None, device="cuda",
                      rank: int = 0, world: int = 1, with_router: bool = True,
                      shared: str = "split") -> HBMExpertStore:
    """Read the MoE weights of `prefixes` (default: every `layers.{l}` with
    routed experts, in order; add "mtp.0" for the MTP layer) into a new store.

    Shapes come from the checkpoint: E from the expert ids, D and I from w1
    ([I, D/2] packed e2m1), I_sh from the shared expert's w1, the hash layers
    and top_k from `ffn.gate.tid2eid` [V, k]. Layer j of the store is
    prefixes[j]. With world > 1 the store holds rank's block of routed experts
    and its rows of the shared expert (ep.expert_range / ep.shared_slice), or
    the whole shared expert with shared="replicated" (ep.TokenShardedEP)."""
    from .ep import expert_range, shared_slice
    ck = CheckpointIndex(weight_dir)
    try:
        prefixes = list(prefixes) if prefixes is not None else [p for p in ck.prefixes() if p.startswith("layers.")]
        if not prefixes:
            raise ValueError(f"no routed experts found under {weight_dir}")
        p0 = prefixes[0]
        E = ck.num_experts(p0)
        w1 = ck.require(f"{p0}.ffn.experts.0.w1.weight")
        I, D = int(w1.shape[0]), int(w1.shape[1]) * 2
        sh = ck.get(f"{p0}.ffn.shared_experts.w1.weight")
        I_sh_full = int(sh.shape[0]) if sh is not None else 0
        tids = [ck.get(f"{p}.ffn.gate.tid2eid") for p in prefixes]
        hash_layers = 0
        while hash_layers < len(tids) and tids[hash_layers] is not None:
            hash_layers += 1
        if any(t is not None for t in tids[hash_layers:]):
            raise ValueError("hash-routed layers (ffn.gate.tid2eid) must come first")
        vocab, top_k = (int(tids[0].shape[0]), int(tids[0].shape[1])) if hash_layers else (129280, 6)
        off, held = expert_range(E, rank, world)
        if shared not in ("split", "replicated"):
            raise ValueError(f"shared must be 'split' or 'replicated', not {shared!r}")
        lo, hi = (shared_slice(I_sh_full, rank, world) if shared == "split" else (0, I_sh_full)) \
            if I_sh_full else (0, 0)
        store = HBMExpertStore(len(prefixes), E, D, I, (hi - lo) if I_sh_full else None, device=device,
                               with_router=with_router, hash_layers=hash_layers, vocab_size=vocab, top_k=top_k,
                               expert_offset=off, experts_held=held)
        for l, p in enumerate(prefixes):
            if ck.num_experts(p) != E:
                raise ValueError(f"{p}: {ck.num_experts(p)} experts, layer {p0} has {E}")
            for e in range(off, off + held):
                q = f"{p}.ffn.experts.{e}"
                t = [ck.require(f"{q}.{w}.{k}") for w in ("w1", "w3", "w2") for k in ("weight", "scale")]
                for j in (1, 3, 5):
                    t[j] = _ue8m0_bytes(t[j], f"{q} scale")
                store.set_expert(l, e, *t)
            if I_sh_full:
                q = f"{p}.ffn.shared_experts"
                sw1, ss1, sw3, ss3, sw2, ss2 = (ck.require(f"{q}.{w}.{k}") for w in ("w1", "w3", "w2")
                                                for k in ("weight", "scale"))
                u8 = lambda x: x.contiguous().view(torch.uint8)  # noqa: E731
                s13 = torch.stack([_ue8m0_bytes(ss1, q), _ue8m0_bytes(ss3, q)])[:, lo // 128:hi // 128]
                store.set_shared(l, torch.stack([u8(sw1)[lo:hi], u8(sw3)[lo:hi]]), s13,
                                 u8(sw2)[:, lo:hi].contiguous(), _ue8m0_bytes(ss2, q)[:, lo // 128:hi // 128])
            if with_router:
                gate = ck.get(f"{p}.ffn.gate.weight")
                if gate is not None:
                    store.set_router(l, _dequant_block128(gate, ck.get(f"{p}.ffn.gate.scale")),
                                     ck.get(f"{p}.ffn.gate.bias"))
            if l < hash_layers:
                store.layers[l].tid2eid.copy_(tids[l].to(torch.int64))
        return store
    finally:
        ck.close()
