"""hs_moe_layer_fp4: the MoE half of a decode layer (norm -> routing -> routed
FP4 + shared FP8 experts -> residual add) in one call must equal the unfused
chain hs_rms_norm -> hs_router_topk (or hs_hash_route) -> hs_moe_ffn_fp4 ->
residual add, bit for bit, in router and hash mode, in place, and split over
two expert-parallel ranks (within the partial-sum tolerance)."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

HS_DEV_BAD_TOKEN = 0x2


@pytest.fixture(scope="module")
def store():
    from home_seek_b200.expert_store import HBMExpertStore
    st = HBMExpertStore(1, 256, 4096, 2048, 2048, device="cuda", hash_layers=1, vocab_size=4096)
    st.fill_random(21)
    return st


def _rows(T, seed, scale=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(T, 4096, generator=g, device="cuda") * scale).to(torch.bfloat16)


def _norm_w(seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (1 + 0.05 * torch.randn(4096, generator=g, device="cuda")).to(torch.bfloat16)


def _add(h, y):
    return (h.float() + y.float()).to(torch.bfloat16)   # torch's bf16 add: one rounding of the f32 sum


@pytest.mark.parametrize("T", [1, 3, 8])
def test_router_layer_equals_unfused_chain(store, T):
    from home_seek_b200 import ops
    lw = store.layers[0]
    h = _rows(T, 100 + T, scale=3.0)
    nw = _norm_w(T)
    dup = 1 if T == 1 else 0
    x = ops.rms_norm(h, nw)
    idx, w = ops.router_topk(x, lw.gate, lw.bias, 6, 1.5)
    y = ops.moe_ffn(store.desc(0), store.dims, x, idx, w, dup_mode=dup)
    x2 = torch.empty_like(x)
    h2, idx2, w2 = ops.moe_layer(store.desc(0), store.dims, h, nw, lw.gate, lw.bias, 6, 1.5, dup_mode=dup,
                                 x_out=x2)
    assert ops.check_status(torch.device("cuda")) == 0
    assert torch.equal(x2, x)
    assert torch.equal(idx2, idx) and torch.equal(w2, w)
    assert torch.equal(h2, _add(h, y))
    # in place (h_out = h)
    hi = h.clone()
    ops.moe_layer(store.desc(0), store.dims, hi, nw, lw.gate, lw.bias, 6, 1.5, dup_mode=dup, h_out=hi)
    assert torch.equal(hi, h2)


@pytest.mark.parametrize("T", [1, 3])
def test_hash_layer_equals_unfused_chain(store, T):
    from home_seek_b200 import ops
    lw = store.layers[0]
    h = _rows(T, 200 + T)
    nw = _norm_w(50 + T)
    ids = torch.randint(0, 4096, (T,), generator=torch.Generator(device="cuda").manual_seed(T), device="cuda")
    dup = 1 if T == 1 else 0
    x = ops.rms_norm(h, nw)
    idx, w = ops.hash_route(ids, lw.tid2eid, 6)
    y = ops.moe_ffn(store.desc(0), store.dims, x, idx, w, dup_mode=dup)
    h2, idx2, w2 = ops.moe_layer(store.desc(0), store.dims, h, nw, None, None, 6, 1.5, dup_mode=dup, ids=ids,
                                 tid2eid=lw.tid2eid)
    assert ops.check_status(torch.device("cuda")) == 0
    assert torch.equal(idx2, idx.view(T, 6)) and torch.equal(w2, w.view(T, 6))
    assert torch.equal(h2, _add(h, y))


def test_hash_layer_bad_token_is_reported_and_skipped(store):
    from home_seek_b200 import ops
    lw = store.layers[0]
    h = _rows(2, 7)
    nw = _norm_w(7)
    ids = torch.tensor([5, 4096], device="cuda")     # the second id is outside the table
    h2, idx2, _ = ops.moe_layer(store.desc(0), store.dims, h, nw, None, None, 6, 1.5, ids=ids, tid2eid=lw.tid2eid)
    assert ops.check_status(torch.device("cuda")) & HS_DEV_BAD_TOKEN
    assert (idx2[1] == -1).all()
    x = ops.rms_norm(h, nw)
    idx, w = ops.hash_route(ids[:1], lw.tid2eid, 6)
    y = ops.moe_ffn(store.desc(0), store.dims, x[:1], idx, w)
    assert torch.equal(h2[0], _add(h[:1], y)[0])   # token 0 as if alone (token 1 gets the shared expert only)


def test_router_ties_go_to_the_lower_expert_id(store):
    """Equal scores (a duplicated gate row with an equal bias) select the lower
    id, as hs_router_topk (torch.sort(stable=True) in the reference): five
    experts are forced in by a large bias, and experts 7 and 9 tie for the
    sixth slot, which must go to 7."""
    from home_seek_b200 import ops
    lw = store.layers[0]
    gate = lw.gate.clone()
    bias = lw.bias.clone()
    for a in (3, 50, 90, 150, 220):
        bias[a] = 8.0
    gate[9] = gate[7]
    bias[7] = bias[9] = 6.0
    h = _rows(3, 9)
    nw = _norm_w(9)
    x = ops.rms_norm(h, nw)
    idx, w = ops.router_topk(x, gate, bias, 6, 1.5)
    _, idx2, w2 = ops.moe_layer(store.desc(0), store.dims, h, nw, gate, bias, 6, 1.5)
    assert torch.equal(idx2, idx) and torch.equal(w2, w)
    for row in idx.tolist():
        assert set(row) == {3, 50, 90, 150, 220, 7}, row


@pytest.mark.parametrize("T", [1, 3])
def test_layer_partials_over_two_ranks(store, T):
    from home_seek_b200 import ops
    from home_seek_b200.ep import shard_store
    lw = store.layers[0]
    h = _rows(T, 300 + T)
    nw = _norm_w(300 + T)
    dup = 1 if T == 1 else 0
    x = ops.rms_norm(h, nw)
    idx, w = ops.router_topk(x, lw.gate, lw.bias, 6, 1.5)
    y_ref = ops.moe_ffn(store.desc(0), store.dims, x, idx, w, dup_mode=dup)
    total = torch.zeros(2, T, 4096, dtype=torch.float32, device="cuda")
    for r in range(2):
        sh = shard_store(store, r, 2)
        p, idx_r, _ = ops.moe_layer(sh.desc(0), sh.dims, h, nw, lw.gate, lw.bias, 6, 1.5, dup_mode=dup,
                                    num_experts=256, expert_offset=sh.expert_offset, partials=True)
        assert torch.equal(idx_r, idx)
        total += p
    h2, none = ops.moe_combine_add_rms_norm(total, h, None)
    assert none is None and ops.check_status(torch.device("cuda")) == 0
    y = ops.moe_combine(total)
    assert torch.equal(h2, _add(h, y))
    rel = float((y.float() - y_ref.float()).abs().max() / y_ref.float().abs().max())
    assert rel <= 1e-2, rel
