"""The reference engine's MTP operator surface on the GPU (mtp.MTPEngine), driven
through the reference's own signatures:
  _mtp_generate_draft(last_hidden, num_draft, temperature, last_token_id)
      -> (draft_ids [1, M], M)                           (engine.py:2251-2336)
  _mtp_verify_batched(draft_ids, temperature, main_pred_id)
      -> (n_accept, bonus_logits [1, V])                 (engine.py:2431-2540)
  SharedExpertFFN.forward(h, w1, w3, w2, dtype)          (fused_moe.py:585)

At t = 0 the generate() loop written with these calls must reproduce the
reference's own run recorded in tests/golden/golden.npz (gen_mtp) decision by
decision. At t > 0 the sampled draft and bonus tokens must be the inverse-CDF
samples of the GPU's own logits for the supplied uniforms, and the
speculative-sampling acceptance must equal oracle.accept.rejection on the same
logits and uniforms.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import accept as A
from oracle import inputs as I
from oracle import moe as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def engine():
    from home_seek_b200.mtp import ModelShape, MoEPathModel, MTPEngine
    s = I.MTP_SMALL
    shape = ModelShape(num_layers=s.L, num_experts=s.E, hidden=s.D, inter=s.I, shared_inter=s.I_sh, vocab=s.V,
                       top_k=s.K, hash_layers=s.hash_layers, routed_scaling=1.5, num_draft=s.M)
    return MTPEngine(MoEPathModel(shape, device="cuda", weights=I.mtp_model(s)))


def test_greedy_loop_through_the_reference_signatures(engine, golden):
    meta = golden["mtp_meta"]
    iters, first, M = int(meta[9]), int(meta[10]), int(meta[8])
    next_id = torch.tensor([[first]], device="cuda")
    tokens = []
    for it in range(iters):
        last_h, next_id = engine.main_step(next_id)
        tokens.append(int(next_id))
        draft_ids, n_draft = engine._mtp_generate_draft(last_h, M, 0.0, last_token_id=next_id)
        assert n_draft == M and tuple(draft_ids.shape) == (1, M)
        n_acc, bonus_logits = engine._mtp_verify_batched(draft_ids, 0.0, main_pred_id=next_id)
        assert isinstance(n_acc, int) and tuple(bonus_logits.shape) == (1, engine.model.shape.vocab)
        rec = [int(v) for v in golden["mtp_records"][it]]
        assert [rec[1]] + [int(v) for v in draft_ids[0]] == rec[1:2 + M], it
        assert n_acc == rec[2 + M], it
        if n_acc > 0:  # engine.py:2893-2916
            tokens.extend(int(v) for v in draft_ids[0, :n_acc])
            next_id = engine.bonus_token(bonus_logits, 0.0)
            tokens.append(int(next_id))
        assert int(next_id) == rec[3 + M], it
    assert tokens == golden["mtp_tokens"].tolist()


def test_no_drafts_and_no_last_token(engine):
    assert engine._mtp_verify_batched(torch.empty(1, 0, dtype=torch.int64, device="cuda"), 0.0) == (0, None)
    assert engine._mtp_generate_draft(torch.zeros(1, 1, 1, 512, dtype=torch.bfloat16, device="cuda"), 0) == (None, 0)
    last_h, tok = engine.main_step(torch.tensor([[3]], device="cuda"))
    d, n = engine._mtp_generate_draft(last_h, 2, 0.0, last_token_id=None)  # zero embedding at step 0
    assert n == 2 and bool(((d >= 0) & (d < engine.model.shape.vocab)).all())


def _inverse_cdf(logits: torch.Tensor, t: float, u: float) -> int:
    n, tok = A.rejection(logits.float().cpu().numpy()[None, None], np.zeros((1, 0, logits.numel()), np.float32),
                         np.zeros((1, 0), np.int64), np.array([[u]], np.float32), t)
    return int(tok[0])


def test_temperature_draft_bonus_and_rejection_acceptance(engine):
    t = 0.7
    g = torch.Generator().manual_seed(21)
    next_id = torch.tensor([[41]], device="cuda")
    for it in range(12):
        u_main = torch.rand(1, generator=g)
        last_h, next_id = engine.main_step(next_id, t, u_main.cuda())
        u_d = torch.rand(2, generator=g)
        draft_ids, _ = engine._mtp_generate_draft(last_h, 2, t, last_token_id=next_id, uniform=u_d.cuda())
        q = engine._mtp_draft_logits
        for i in range(2):  # each draft token is the inverse-CDF sample of its own logits
            assert int(draft_ids[0, i]) == _inverse_cdf(q[i], t, float(u_d[i])), (it, i)
        u_v = torch.rand(3, generator=g)
        n, nxt = engine._mtp_verify_rejection(draft_ids, t, next_id, uniform=u_v.cuda())
        _, xv = engine._verify_forward(draft_ids, next_id)
        p = engine.model.logits(xv)
        n_o, tok_o = A.rejection(p.float().cpu().numpy()[None], q.float().cpu().numpy()[None],
                                 draft_ids.cpu().numpy(), u_v.numpy()[None], t)
        assert (n, int(nxt)) == (int(n_o[0]), int(tok_o[0])), it
        # the reference's own t > 0 verify compares argmaxes; its bonus is a sample
        n_g, bonus = engine._mtp_verify_batched(draft_ids, t, main_pred_id=next_id)
        u_b = torch.rand(1, generator=g)
        b = engine.bonus_token(bonus, t, u_b.cuda())
        assert int(b) == _inverse_cdf(bonus[0], t, float(u_b)), it
        next_id = nxt


def test_shared_expert_reference_signature_fp8_and_bf16_forms():
    from home_seek_b200.fused_moe import SharedExpertFFN
    from home_seek_b200.layout import fp8_block_dequant
    shape = I.SMALL
    w13, s13, w2, s2 = I.shared_fp8(shape.D, shape.I_sh, seed=2)
    t8 = lambda a: torch.from_numpy(np.ascontiguousarray(a)).view(torch.float8_e4m3fn).cuda()  # noqa: E731
    u8 = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    h = I.hidden(3, shape.D, seed=4)
    ffn = SharedExpertFFN(hidden_size=shape.D, intermediate_size=shape.I_sh)
    # the FP8 + block-scale form (what _get_shared_expert holds before load_fp8_weight)
    out_a = ffn.forward(h.cuda().unsqueeze(0), (t8(w13[0]), u8(s13[0])), (t8(w13[1]), u8(s13[1])),
                        (t8(w2), u8(s2)), torch.bfloat16)
    # the bf16 form load_fp8_weight returns (engine.py:1451/1469/1534 pass these)
    bf = [fp8_block_dequant(t8(a), u8(sc)) for a, sc in ((w13[0], s13[0]), (w13[1], s13[1]), (w2, s2))]
    out_b = ffn.forward(h.cuda().unsqueeze(0), *bf, torch.bfloat16)
    assert out_a.shape == (1, 3, shape.D) and torch.equal(out_a, out_b)
    ref = O.shared_expert(h, (w13, s13, w2, s2))
    rel = float((out_a[0].float().cpu() - ref.float()).abs().max() / ref.float().abs().max())
    assert rel <= 1e-2, rel
    # a bf16 weight that is not an FP8 block-scaled value cannot run on the FP8 kernel
    with pytest.raises(TypeError):
        ffn.forward(h.cuda().unsqueeze(0), bf[0] * 1.01, bf[1], bf[2], torch.bfloat16)


def test_fused_moe_accepts_the_reference_bf16_three_tuple_loader():
    """FusedMoEFFN.forward with the BF16 3-tuples the reference's T >= 2 path
    passes (_bf16_load, engine.py:1480-1486) gives the same bits as with the
    FP4 6-tuples they were dequantised from."""
    from home_seek_b200 import ops
    from home_seek_b200.fused_moe import FusedMoEFFN
    from oracle import fp4 as F
    shape = I.SMALL
    load = I.make_loader(shape)
    dev = torch.device("cuda")

    def six(layer, eid):
        w1, s1, w3, s3, w2, s2 = load(int(eid))
        c = lambda a: torch.from_numpy(a).view(torch.int8).to(dev)  # noqa: E731
        e = lambda a: torch.from_numpy(a).view(torch.float8_e8m0fnu).to(dev)  # noqa: E731
        return (c(w1), e(s1), c(w3), e(s3), c(w2), e(s2))

    def three(layer, eid):
        w1, s1, w3, s3, w2, s2 = load(int(eid))
        return tuple(F.dequant_fp4(a, sc).to(dev) for a, sc in ((w1, s1), (w3, s3), (w2, s2)))

    gate, bias = I.router_weights(shape.E, shape.D, seed=1)
    h = I.hidden(5, shape.D, seed=3).cuda()
    idx, w = ops.router_topk(h, gate.cuda(), bias.cuda(), shape.K, 1.5)
    ffn = FusedMoEFFN(num_experts=shape.E, intermediate_size=shape.I, hidden_size=shape.D)
    a = ffn.forward(h, idx, w, six, 0)
    b = ffn.forward(h, idx, w, three, 0)
    assert torch.equal(a, b)
    ref = O.moe_routed(h.cpu(), idx.cpu(), w.cpu(), load)
    rel = float((a.float().cpu() - ref.float()).abs().max() / ref.float().abs().max())
    assert rel <= 1e-2, rel
