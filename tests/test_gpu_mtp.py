"""MTP decode step on a small model shape: the GPU path (fused add+RMSNorm,
router / hash routing, MoE kernels, lm_head, greedy acceptance, device-side
bookkeeping) against the CPU restatement in oracle/mtp.py on the same
weights."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import accept as A
from oracle import mtp as OM

pytestmark = pytest.mark.gpu

TOL = 3e-2  # two MoE layers at <= 1e-2 each plus norms, relative to the max magnitude


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float().cpu(), b.float().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp(min=1e-30))


def _extract(m) -> OM.ModelWeights:
    """The GPU model's weights in the reference layouts the oracle consumes."""
    from home_seek_b200.layout import untile_rows
    st = m.store
    layers = []
    for l in range(m.shape.num_layers + 1):
        lw = st.layers[l]

        def load(e, l=l):
            return tuple(t.view(torch.uint8).cpu().numpy() for t in st._load_expert_fp4_raw(l, e))

        sh = None
        if lw.sh_w13 is not None:
            w13 = torch.stack([untile_rows(lw.sh_w13[:, :, 0]), untile_rows(lw.sh_w13[:, :, 1])]).cpu().numpy()
            s13 = lw.sh_s13[..., 0].permute(2, 0, 1).contiguous().cpu().numpy()
            sh = (w13, s13, untile_rows(lw.sh_w2).cpu().numpy(), lw.sh_s2[..., 0].contiguous().cpu().numpy())
        layers.append(OM.LayerWeights(load, sh,
                                      lw.gate.cpu() if lw.gate is not None else None,
                                      lw.bias.cpu() if lw.bias is not None else None,
                                      lw.tid2eid.cpu() if lw.tid2eid is not None else None))
    s = m.shape
    return OM.ModelWeights(layers, m.embed.cpu(), m.lm_head.cpu(), m.norm_w.cpu(), m.ln_w.cpu(), m.e_proj.cpu(),
                           m.h_proj.cpu(), m.enorm_w.cpu(), m.hnorm_w.cpu(), m.mtp_norm_w.cpu(), s.top_k,
                           s.hash_layers, s.routed_scaling, s.num_draft)


@pytest.fixture(scope="module")
def model():
    from home_seek_b200.mtp import ModelShape, MoEPathModel
    shape = ModelShape(num_layers=2, num_experts=16, hidden=512, inter=512, shared_inter=512, vocab=1024, top_k=6,
                       hash_layers=1, routed_scaling=1.5, num_draft=2)
    m = MoEPathModel(shape, device="cuda", seed=3)
    return m, _extract(m)


@pytest.mark.parametrize("ids", [[5], [5, 17, 300]])
def test_forward_and_logits_match_oracle(model, ids):
    m, W = model
    t = torch.tensor(ids, dtype=torch.int64)
    h, x = m.forward(t.cuda())
    ho, xo = OM.forward(W, t, m.shape.num_layers)
    assert _rel(h, ho) <= TOL, _rel(h, ho)
    assert _rel(x, xo) <= TOL, _rel(x, xo)
    lg, lgo = m.logits(x), OM.logits(W, xo)
    assert _rel(lg, lgo) <= TOL, _rel(lg, lgo)


def _near_argmax(lv: torch.Tensor, tok: int) -> bool:
    lv = lv.float()
    return float(lv[tok]) >= float(lv.max()) - TOL * float(lv.abs().max())


def test_draft_tokens_are_oracle_argmax(model):
    from home_seek_b200 import ops
    m, W = model
    h, x = m.forward(torch.tensor([5], device="cuda"))
    none = torch.empty(1, 0, dtype=torch.int64, device="cuda")
    _, main = ops.accept_greedy(m.logits(x).view(1, 1, -1), none)
    d = m.draft(h, main).cpu()
    prev, tok = h.cpu(), main.cpu()
    for i in range(m.shape.num_draft):
        prev, lgo = OM.draft_step(W, prev, tok, m.shape.num_layers)
        assert _near_argmax(lgo[0], int(d[i])), (i, int(d[i]), int(lgo[0].float().argmax()))
        tok = d[i:i + 1]


def test_iteration_bookkeeping_matches_greedy_acceptance(model):
    """One MTPDecoder iteration: the tokens it appends, its count, acceptance
    and next id follow oracle.accept.greedy on the logits of the same passes."""
    from home_seek_b200 import ops
    from home_seek_b200.mtp import MTPDecoder
    m, _ = model
    dec = MTPDecoder(m, max_tokens=64)
    dec.reset(5)
    dec.iteration()
    torch.cuda.synchronize()
    # the same passes again (the kernels are deterministic) to see the logits
    M = m.shape.num_draft
    h, x = m.forward(torch.tensor([5], device="cuda"))
    none = torch.empty(1, 0, dtype=torch.int64, device="cuda")
    _, main = ops.accept_greedy(m.logits(x).view(1, 1, -1), none)
    d = m.draft(h, main)
    _, xv = m.forward(torch.cat([main, d]))
    lv = m.logits(xv).view(1, M + 1, -1).float().cpu().numpy()
    n_o, nxt_o, _ = A.greedy(lv, d.view(1, M).cpu().numpy())
    n = int(n_o[0])
    want = [int(main)] + ([int(v) for v in d[:n].cpu()] + [int(nxt_o[0])] if n > 0 else [])
    cnt = int(dec.step_count)
    assert cnt == len(want)
    assert dec.step_tokens[:cnt].cpu().tolist() == want
    assert dec.tokens[:cnt].cpu().tolist() == want
    assert int(dec.accepted) == n and int(dec.count) == cnt
    assert int(dec.next_id) == (int(nxt_o[0]) if n > 0 else int(main))


def test_rms_norm_and_add_rms_norm_match_reference_formula():
    from home_seek_b200 import ops
    g = torch.Generator().manual_seed(11)
    for T, D in ((1, 4096), (3, 4096), (5, 512), (2, 8192)):
        h = (torch.randn(T, D, generator=g) * 3).to(torch.bfloat16)
        y = (torch.randn(T, D, generator=g) * 0.5).to(torch.bfloat16)
        w = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16)
        x = ops.rms_norm(h.cuda(), w.cuda()).cpu()
        xo = OM.rms_norm(h, w)
        # fixed-order sum vs torch's: at most one bf16 ulp apart, almost always equal
        ulp = (xo.float().abs() * 2.0 ** -7).clamp(min=1e-30)
        assert bool(((x.float() - xo.float()).abs() <= ulp).all())
        assert float((x == xo).float().mean()) >= 0.99
        hh, xx = ops.add_rms_norm(h.cuda(), y.cuda(), w.cuda())
        assert torch.equal(hh.cpu(), h + y)
        xo2 = OM.rms_norm(h + y, w)
        assert bool(((xx.cpu().float() - xo2.float()).abs() <= (xo2.float().abs() * 2.0 ** -7)).all())
        # in place on the residual stream
        hc = h.cuda().clone()
        ops.add_rms_norm(hc, y.cuda(), w.cuda(), h_out=hc)
        assert torch.equal(hc.cpu(), h + y)
