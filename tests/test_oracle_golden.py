"""The CPU oracle against golden vectors produced by the reference's own code
(tests/golden/make_golden.py), plus the reference's known-answer tests for the
FP4 / UE8M0 codecs and stable top-k."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import accept as A
from oracle import fp4 as F4
from oracle import inputs as I
from oracle import moe as O


def bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(a.astype(np.uint16).view(np.int16)).view(torch.bfloat16)


# --- known answers from the reference's tests --------------------------------

def test_e2m1_lut_and_nibble_order():
    # fused_moe.py:604-608 table; _fp4.py low nibble first (tests/test_fp4_experts.py:432-476)
    assert F4.E2M1_LUT.tolist() == [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                                    -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0]
    packed = np.array([[0x21, 0xF7]], dtype=np.uint8)
    assert F4.unpack_e2m1(packed).tolist() == [[0.5, 1.0, 6.0, -6.0]]


def test_ue8m0_known_answers():
    # tests/test_weight_loading_bug.py:234-255
    assert F4.e8m0_to_f32_shift(np.array([127, 128, 126], np.uint8)).tolist() == [1.0, 2.0, 0.5]
    t = F4.e8m0_to_f32_torch(np.array([0, 127, 255], np.uint8))
    ref = torch.tensor([0, 127, 255], dtype=torch.uint8).view(torch.float8_e8m0fnu).float().numpy()
    assert t[1] == 1.0 and t[0] == ref[0] and np.isnan(t[2]) and np.isnan(ref[2])


def test_e4m3_decode_matches_torch():
    b = np.arange(256, dtype=np.uint8)
    mine = F4.e4m3_to_f32(b)
    ref = torch.from_numpy(b).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(np.isnan(mine), np.isnan(ref))
    ok = ~np.isnan(ref)
    assert np.array_equal(mine[ok], ref[ok])


def test_per_group_scale_isolation():
    # tests/test_fp4_experts.py:598-631: one scale per 32 columns
    packed = np.full((1, 32), 0x22, dtype=np.uint8)  # all 1.0
    scale = np.array([[127, 129]], dtype=np.uint8)   # 1.0, 4.0
    w = F4.dequant_fp4(packed, scale).float().numpy()
    assert np.all(w[0, :32] == 1.0) and np.all(w[0, 32:] == 4.0)


def test_stable_topk_known_answer():
    # tests/test_tile_ops.py:30-37
    s = torch.tensor([[1.0, 5.0, 3.0, 7.0], [8.0, 2.0, 6.0, 4.0]])
    assert O.stable_topk(s, 2).tolist() == [[3, 1], [0, 2]]


# --- golden vectors from the reference ---------------------------------------

@pytest.mark.parametrize("name,T,D,E,seed", [("small", 5, 512, 16, 10), ("cfg0", 3, 4096, 256, 0),
                                             ("t24", 24, 4096, 256, 12)])
def test_router_matches_reference(golden, name, T, D, E, seed):
    h = I.hidden(T, D, seed=seed)
    gate, bias = I.router_weights(E, D, seed=seed + 1)
    idx, w, lb = O.router(h, gate, bias, 6, 1.5, return_logits=True)
    assert np.array_equal(idx.numpy(), golden[f"router_{name}_idx"])
    assert np.array_equal(w.numpy(), golden[f"router_{name}_w"])
    assert np.array_equal(lb.view(torch.int16).numpy().view(np.uint16), golden[f"router_{name}_logits"])
    assert np.allclose(w.sum(-1).numpy(), 1.5, atol=1e-5)  # tests/test_fixes.py:339-352


def test_router_ties_stable(golden):
    idx = golden["router_ties_idx"]
    # rows 5, 9, 20 of the gate are identical; when several are selected the
    # lower id must come first (stable sort)
    for row in idx.tolist():
        sel = [e for e in row if e in (5, 9, 20)]
        assert sel == sorted(sel)
    h = I.hidden(4, 512, seed=14)
    gate, bias = I.router_weights(32, 512, seed=15)
    gate = gate.clone()
    gate[9] = gate[5]
    gate[20] = gate[5]
    bias = bias.clone()
    bias[9] = bias[5]
    bias[20] = bias[5]
    i2, w2 = O.router(h, gate, bias)
    assert np.array_equal(i2.numpy(), idx)
    assert np.array_equal(w2.numpy(), golden["router_ties_w"])


def test_hash_matches_reference(golden):
    tid = I.tid2eid(1000, 256, 6, seed=3)
    ids = torch.from_numpy(golden["hash_ids"])
    e, w = O.hash_route(ids, tid, 6)
    assert np.array_equal(e.numpy(), golden["hash_eids"])
    assert np.array_equal(w.numpy(), golden["hash_w"])


@pytest.mark.parametrize("name", ["small_t1", "small_t3", "small_t5", "small_t24", "small_hash", "cfg0"])
def test_moe_matches_reference(golden, name):
    D, Iw, E, I_sh, K, T, seed = golden[f"moe_{name}_meta"].tolist()
    shape = I.MoeShape(D=D, I=Iw, E=E, I_sh=I_sh, K=K)
    h = I.hidden(T, D, seed=seed)
    idx = torch.from_numpy(golden[f"moe_{name}_idx"])
    w = torch.from_numpy(golden[f"moe_{name}_w"])
    load = I.make_loader(shape)
    sh = I.shared_fp8(D, I_sh, seed=seed + 2)
    routed = O.moe_routed(h, idx, w, load)
    assert np.array_equal(routed.view(torch.int16).numpy().view(np.uint16), golden[f"moe_{name}_routed"])
    full = routed + O.shared_expert(h, sh)
    assert np.array_equal(full.view(torch.int16).numpy().view(np.uint16), golden[f"moe_{name}_out"])


def test_greedy_accept_matches_reference(golden):
    logits = bf16(golden["accept_logits"]).float().numpy()
    ids = golden["accept_ids"]
    n, nxt, _ = A.greedy(logits, ids[:, 1:])
    assert np.array_equal(n, golden["accept_n"])
    assert np.array_equal(nxt, golden["accept_next"])
    assert set(golden["accept_n"].tolist()) == {0, 1, 2}


def test_permute_matches_reference(golden):
    idx = golden["perm_idx"]
    pos, p2e, cnt, n = O.permute_plan(idx, 8)
    assert np.array_equal(pos, golden["perm_pos"])
    x = bf16(golden["perm_x"])
    xe = O.expand(x, pos, idx.size)
    assert np.array_equal(xe.view(torch.int16).numpy().view(np.uint16), golden["perm_xe"])
    red = O.reduce(xe, torch.from_numpy(golden["perm_w"]), pos)
    assert np.array_equal(red.view(torch.int16).numpy().view(np.uint16), golden["perm_reduced"])


def test_rejection_oracle_properties():
    # no reference counterpart: check the distributional identity on a tiny vocab.
    # With p == q every draft is accepted and the bonus follows p.
    B, M, V = 4, 2, 64
    g = torch.Generator().manual_seed(3)
    tl = (torch.randn(B, M + 1, V, generator=g) * 3).to(torch.bfloat16).float().numpy()
    ids = np.zeros((B, M), dtype=np.int64)
    u = np.full((B, M + 1), 0.999, dtype=np.float32)
    n, tok = A.rejection(tl, tl, ids, u, 0.7)
    assert (n == M).all()
    # a rejected draft never resamples a token where q >= p
    dl = (torch.randn(B, M + 1, V, generator=g) * 3).to(torch.bfloat16).float().numpy()
    u2 = np.full((B, M + 1), 0.5, dtype=np.float32)
    ids2 = np.argmax(dl[:, :M], axis=-1)
    n2, tok2 = A.rejection(tl, dl, ids2, u2, 0.7)
    for b in range(B):
        if n2[b] < M:
            p = A._softmax64(tl[b, n2[b]].astype(np.float32) / np.float32(0.7))
            q = A._softmax64(dl[b, n2[b]].astype(np.float32) / np.float32(0.7))
            assert p[tok2[b]] > q[tok2[b]]


def test_mtp_decode_loop_matches_reference(golden):
    """oracle.mtp.decode_loop against the reference's own MTP loop (its
    _forward_layer, _mtp_generate_draft and _mtp_verify_batched on the seeded
    small model, attention off): the token stream, every iteration's decisions
    and every logits row an argmax was taken of, bit for bit."""
    from oracle import inputs as I
    from oracle import mtp as OM
    s = I.MTP_SMALL
    meta = golden["mtp_meta"]
    assert list(meta[:9]) == [s.D, s.I, s.E, s.I_sh, s.K, s.V, s.L, s.hash_layers, s.M]
    W = OM.weights_from_inputs(I.mtp_model(s), s.L, s.hash_layers, s.K, s.M)
    tokens, recs, lg = OM.decode_loop(W, int(meta[10]), int(meta[9]), s.L)
    assert np.array_equal(tokens, golden["mtp_tokens"])
    assert np.array_equal(recs, golden["mtp_records"])
    for k in ("main", "draft", "verify"):
        assert np.array_equal(lg[k].contiguous().view(torch.int16).numpy().view(np.uint16),
                              golden[f"mtp_logits_{k}"]), k
    assert {int(r[4]) for r in recs} == {0, 1, 2}  # rejections, one and two acceptances


def test_verify_state_oracle_matches_reference(golden):
    """oracle/verify_state.commit against the reference's _mtp_verify_batched
    state handling (engine.py:2443-2459, 2500-2538): KV caches trimmed to old +
    n_accept (restored at 0), compressed data and compressor states restored,
    position old + n_accept, for n_accept = 0, 1, 2 of 3 positions."""
    import copy

    from oracle import verify_state as VS
    for case in range(3):
        before = VS.scenario_states(seed=7 + case)
        after = copy.deepcopy(before)
        for l in after:
            VS.forward_mutation(after[l], [5, 9, 13], l)
        n, pos = (int(v) for v in golden[f"vs{case}_n"])
        assert n == case
        out, p = VS.commit(before, after, n, 3, 40)
        assert p == pos
        for l, st in out.items():
            assert np.array_equal(st["kv"].view(torch.int16).numpy().view(np.uint16), golden[f"vs{case}_kv{l}"])
            assert np.array_equal(st["cdata"].view(torch.int16).numpy().view(np.uint16), golden[f"vs{case}_cdata{l}"])
            assert np.array_equal(st["cidx"].numpy(), golden[f"vs{case}_cidx{l}"])
            assert st["comp"][0] == int(golden[f"vs{case}_acc{l}"][0])
            assert np.array_equal(st["comp"][1].numpy(), golden[f"vs{case}_kvs{l}"])
            assert np.array_equal(st["comp"][2].numpy(), golden[f"vs{case}_scs{l}"])
