"""Reference-format checkpoint -> HBMExpertStore.

A synthetic checkpoint with the reference's key names and dtypes (packed e2m1
int8 experts with float8_e8m0fnu scales, an e4m3 shared expert with 128x128
UE8M0 block scales, a bf16 router gate and bias, an e4m3 gate with block
scales, a hash layer's tid2eid), split over two safetensors files with an
index, must load into a store byte-identical to one filled tensor by tensor;
the reference-facing `_load_expert_fp4_raw` must return the checkpoint's own
bytes; an expert-parallel rank must load exactly `ep.shard_store`'s slice.
"""
from __future__ import annotations

import json

import pytest
import torch

from oracle import inputs as I

SHAPE = I.MoeShape(D=512, I=512, E=8, I_sh=512, K=6)  # the kernels' smallest D and I
LAYERS = 3  # layer 0 hash-routed, layer 1 bf16 gate, layer 2 e4m3 gate with block scales


def _tensors(shape=SHAPE):
    t = {}
    for l in range(LAYERS):
        p = f"layers.{l}.ffn"
        load = I.make_loader(shape, seed_base=1000 + 100 * l)
        for e in range(shape.E):
            w1, s1, w3, s3, w2, s2 = load(e)
            for name, w, s in (("w1", w1, s1), ("w3", w3, s3), ("w2", w2, s2)):
                t[f"{p}.experts.{e}.{name}.weight"] = torch.from_numpy(w.copy()).view(torch.int8)
                t[f"{p}.experts.{e}.{name}.scale"] = torch.from_numpy(s.copy()).view(torch.float8_e8m0fnu)
        w13, s13, w2, s2 = (torch.from_numpy(x.copy()) for x in I.shared_fp8(shape.D, shape.I_sh, seed=50 + l))
        s13 = s13.clone()
        s13[0, 1, 2] = 119  # distinct block scales
        s13[1, 3, 0] = 123
        for name, w, s in (("w1", w13[0], s13[0]), ("w3", w13[1], s13[1]), ("w2", w2, s2)):
            t[f"{p}.shared_experts.{name}.weight"] = w.contiguous().view(torch.float8_e4m3fn)
            t[f"{p}.shared_experts.{name}.scale"] = s.contiguous().view(torch.float8_e8m0fnu)
        gate, bias = I.router_weights(shape.E, shape.D, seed=60 + l)
        if l == 0:
            t[f"{p}.gate.tid2eid"] = I.tid2eid(100, shape.E, shape.K, seed=7)
            t[f"{p}.gate.weight"] = gate
        elif l == 1:
            t[f"{p}.gate.weight"] = gate
            t[f"{p}.gate.bias"] = bias
        else:
            g8 = (gate.float() * 64).to(torch.float8_e4m3fn)
            t[f"{p}.gate.weight"] = g8
            t[f"{p}.gate.scale"] = torch.full((1, shape.D // 128), 121, dtype=torch.uint8).view(torch.float8_e8m0fnu)
            t[f"{p}.gate.bias"] = bias
    return t


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    from safetensors.torch import save_file
    d = tmp_path_factory.mktemp("ckpt")
    t = _tensors()
    keys = sorted(t)
    half = len(keys) // 2
    wm = {}
    for fname, ks in (("model-00001-of-00002.safetensors", keys[:half]),
                      ("model-00002-of-00002.safetensors", keys[half:])):
        save_file({k: t[k] for k in ks}, str(d / fname))
        wm.update({k: fname for k in ks})
    with open(d / "model.safetensors.index.json", "w") as f:
        json.dump({"metadata": {"total_size": 0}, "weight_map": wm}, f)
    return str(d), t


def _expected_store(t, device="cpu"):
    from home_seek_b200.expert_store import HBMExpertStore
    st = HBMExpertStore(LAYERS, SHAPE.E, SHAPE.D, SHAPE.I, SHAPE.I_sh, device=device, hash_layers=1, vocab_size=100,
                        top_k=SHAPE.K)
    for l in range(LAYERS):
        p = f"layers.{l}.ffn"
        for e in range(SHAPE.E):
            st.set_expert(l, e, *(t[f"{p}.experts.{e}.{w}.{k}"].view(torch.uint8)
                                  for w in ("w1", "w3", "w2") for k in ("weight", "scale")))
        sw = [t[f"{p}.shared_experts.{w}.weight"].view(torch.uint8) for w in ("w1", "w3", "w2")]
        ss = [t[f"{p}.shared_experts.{w}.scale"].view(torch.uint8) for w in ("w1", "w3", "w2")]
        st.set_shared(l, torch.stack(sw[:2]), torch.stack(ss[:2]), sw[2], ss[2])
        gate = t[f"{p}.gate.weight"]
        if gate.dtype == torch.float8_e4m3fn:  # 128x128 blocks of 2^(121-127)
            gate = (gate.float() * 2.0 ** -6).to(torch.bfloat16)
        st.set_router(l, gate, t.get(f"{p}.gate.bias"))
    st.layers[0].tid2eid.copy_(t["layers.0.ffn.gate.tid2eid"])
    return st


def _store_tensors(st):
    out = []
    for lw in st.layers:
        for name in ("w13", "s13", "w2", "s2", "sh_w13", "sh_s13", "sh_w2", "sh_s2", "gate", "bias", "tid2eid"):
            out.append((name, getattr(lw, name)))
    return out


def test_checkpoint_loads_byte_identical_store(ckpt):
    from home_seek_b200.checkpoint import load_expert_store
    d, t = ckpt
    st = load_expert_store(d, device="cpu")
    ref = _expected_store(t)
    assert (st.num_layers, st.E, st.D, st.I, st.I_sh, st.K) == (LAYERS, SHAPE.E, SHAPE.D, SHAPE.I, SHAPE.I_sh,
                                                               SHAPE.K)
    for (name, a), (_, b) in zip(_store_tensors(st), _store_tensors(ref)):
        if a is None or b is None:
            assert a is None and b is None, name
        else:
            assert torch.equal(a, b), name
    # the reference-facing API returns the checkpoint's own tensors
    for l, e in ((0, 0), (1, 5), (2, 7)):
        raw = st._load_expert_fp4_raw(l, e)
        want = [t[f"layers.{l}.ffn.experts.{e}.{w}.{k}"] for w in ("w1", "w3", "w2") for k in ("weight", "scale")]
        for a, b in zip(raw, want):
            assert torch.equal(a.view(torch.uint8), b.view(torch.uint8))


def test_checkpoint_without_index_file(ckpt, tmp_path):
    """No index: the files are scanned (weight_loader.py:70-80)."""
    from safetensors.torch import save_file
    from home_seek_b200.checkpoint import load_expert_store
    _, t = ckpt
    save_file({k: v for k, v in t.items() if k.startswith("layers.1.")}, str(tmp_path / "a.safetensors"))
    st = load_expert_store(str(tmp_path), device="cpu")
    ref = _expected_store(t)
    assert st.num_layers == 1 and st.layers[0].tid2eid is None
    assert torch.equal(st.layers[0].w13, ref.layers[1].w13) and torch.equal(st.layers[0].gate, ref.layers[1].gate)


@pytest.mark.parametrize("rank", [0, 1])
def test_checkpoint_expert_parallel_rank_equals_shard(ckpt, rank):
    from home_seek_b200.checkpoint import load_expert_store
    from home_seek_b200.ep import shard_store
    d, t = ckpt
    st = load_expert_store(d, device="cpu", rank=rank, world=2)
    ref = shard_store(_expected_store(t), rank, 2)
    assert (st.expert_offset, st.E_local, st.I_sh) == (ref.expert_offset, ref.E_local, ref.I_sh)
    for (name, a), (_, b) in zip(_store_tensors(st), _store_tensors(ref)):
        if a is None or b is None:
            assert a is None and b is None, name
        else:
            assert torch.equal(a, b), name


def test_checkpoint_rejects_non_power_of_two_scales(ckpt, tmp_path):
    from safetensors.torch import save_file
    from home_seek_b200.checkpoint import load_expert_store
    _, t = ckpt
    bad = {k: v for k, v in t.items() if k.startswith("layers.1.")}
    k = "layers.1.ffn.experts.3.w2.scale"
    bad[k] = torch.full(bad[k].shape, 0.3, dtype=torch.float32)
    save_file(bad, str(tmp_path / "a.safetensors"))
    with pytest.raises(ValueError, match="powers of two"):
        load_expert_store(str(tmp_path), device="cpu")


@pytest.mark.gpu
def test_checkpoint_store_on_gpu_matches_oracle(ckpt):
    """The loaded store drives the kernels: layer 2 of the checkpoint through
    hs_moe_ffn_fp4 against the oracle on the checkpoint's own tensors."""
    from home_seek_b200 import ops
    from home_seek_b200.checkpoint import load_expert_store
    from oracle import moe as O
    d, t = ckpt
    st = load_expert_store(d, device="cuda")
    T = 5
    g = torch.Generator().manual_seed(3)
    idx = torch.stack([torch.randperm(SHAPE.E, generator=g)[:SHAPE.K] for _ in range(T)])
    w = torch.softmax(torch.randn(T, SHAPE.K, generator=g), -1)
    h = I.hidden(T, SHAPE.D, seed=4)
    out = ops.moe_ffn(st.desc(2), st.dims, h.cuda(), idx.cuda(), w.cuda(), use_shared=True)
    assert ops.check_status(torch.device("cuda")) == 0
    load = I.make_loader(SHAPE, seed_base=1000 + 200)
    p = "layers.2.ffn.shared_experts"
    sh = (torch.stack([t[f"{p}.w1.weight"], t[f"{p}.w3.weight"]]).view(torch.uint8).numpy(),
          torch.stack([t[f"{p}.w1.scale"], t[f"{p}.w3.scale"]]).view(torch.uint8).numpy(),
          t[f"{p}.w2.weight"].view(torch.uint8).numpy(), t[f"{p}.w2.scale"].view(torch.uint8).numpy())
    ref = O.moe_layer(h, idx, w, load, sh)
    err = float((out.float().cpu() - ref.float()).abs().max() / ref.float().abs().max())
    assert err <= 1e-2, err
