"""lm_head GEMV with the fused greedy decision (hs_lm_head_argmax) against
torch on the same bf16 inputs: the logits it computes (optionally written)
against an f64 reference rounded to bf16, its argmax against torch.argmax of
those logits (first index on ties, NaN maximal, -0 equal to +0), and the
acceptance it applies against oracle.accept.greedy (engine.py:2485-2497)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import accept as A

pytestmark = pytest.mark.gpu


def _ref_logits(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """bf16(x @ w.T) with the sum taken in f64 (the kernel sums in f32)."""
    return (x.double() @ w.double().t()).to(torch.bfloat16)


def _within_one_ulp(a: torch.Tensor, b: torch.Tensor) -> bool:
    """|a - b| <= one bf16 ulp of b, with an absolute floor of 2^-12 for
    logits near zero, where the f32 sum's cancellation error (~1e-7 of the
    terms) exceeds an ulp of the tiny result."""
    a, b = a.float(), b.float()
    ulp = (b.abs() * 2.0 ** -7).clamp(min=2.0 ** -12)
    return bool(((a - b).abs() <= ulp).all())


@pytest.mark.parametrize("T,D,V", [(1, 512, 1000), (3, 512, 1000), (16, 1024, 4096), (3, 4096, 129280)])
def test_logits_and_argmax_match_torch(T, D, V):
    from home_seek_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(T * 1000 + V)
    x = torch.randn(T, D, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(V, D, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    am, n, nxt, lg = ops.lm_head_argmax(x, w, want_logits=True)
    torch.cuda.synchronize()
    assert ops.check_status(x.device) == 0
    ref = _ref_logits(x, w)
    assert _within_one_ulp(lg, ref)
    # the fused argmax is torch.argmax of the logits the kernel computed, bit for bit
    assert torch.equal(am, lg.argmax(dim=-1))
    # and of the reference's logits wherever the top two are more than an ulp apart
    top2 = ref.float().topk(2, dim=-1).values
    clear = (top2[:, 0] - top2[:, 1]) > top2[:, 0].abs() * 2.0 ** -6
    assert torch.equal(am[clear], ref.argmax(dim=-1)[clear])
    assert int(n) == 0 and int(nxt) == int(am[0])
    # the same call without the logits write gives the same decisions
    am2, _, nxt2 = ops.lm_head_argmax(x, w)
    assert torch.equal(am2, am) and int(nxt2) == int(nxt)


def test_ties_nan_and_signed_zero_follow_torch_argmax():
    from home_seek_b200 import ops
    D, V = 512, 2000
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(4, D, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(V, D, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    lg0 = _ref_logits(x, w)
    best = int(lg0[0].float().argmax())
    # row 0: the best head row copied to a lower and a higher index -> the lowest wins
    lo, hi = (best // 2), min(V - 1, best + 700)
    w[lo] = w[best]
    w[hi] = w[best]
    # row 1: NaN logits at two indices -> the first NaN wins
    x[1, 7] = float("nan")
    # row 2: all-zero input -> every logit is +-0, argmax 0
    x[2].zero_()
    am, n, nxt, lg = ops.lm_head_argmax(x, w, want_logits=True)
    torch.cuda.synchronize()
    assert torch.equal(am, lg.argmax(dim=-1))
    assert int(am[0]) == min(lo, best)
    assert int(am[1]) == 0  # every logit of row 1 is NaN (x has a NaN): the first index
    assert int(am[2]) == 0
    # a NaN in one head row only: that row's index wins for every finite token row
    w2 = w.clone()
    w2[1234, 3] = float("nan")
    w2[1500, 9] = float("nan")
    am2 = ops.lm_head_argmax(x[3:4].contiguous(), w2)[0]
    assert int(am2[0]) == 1234


def test_fused_greedy_acceptance_matches_the_reference_loop():
    from home_seek_b200 import ops
    D, V = 512, 3000
    g = torch.Generator(device="cuda").manual_seed(9)
    x = torch.randn(3, D, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(V, D, generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    lg = ops.lm_head_argmax(x, w, want_logits=True)[3]
    am = lg.argmax(dim=-1).cpu().tolist()
    cases = [[(am[0] + 1) % V, am[1]], [am[0], (am[1] + 1) % V], [am[0], am[1]], [(am[0] + 5) % V, (am[1] + 5) % V]]
    for d in cases:
        ids = torch.tensor(d, dtype=torch.int64, device="cuda")
        a2, n, nxt = ops.lm_head_argmax(x, w, draft_ids=ids)
        n_o, nxt_o, _ = A.greedy(lg.float().cpu().numpy()[None], np.array([d], dtype=np.int64))
        assert int(n) == int(n_o[0]), (d, int(n), int(n_o[0]))
        assert int(nxt) == int(nxt_o[0]), (d, int(nxt), int(nxt_o[0]))
    assert ops.check_status(x.device) == 0
    # an out-of-range draft id stops the acceptance and is reported
    ids = torch.tensor([am[0], V + 3], dtype=torch.int64, device="cuda")
    _, n, nxt = ops.lm_head_argmax(x, w, draft_ids=ids)
    torch.cuda.synchronize()
    assert int(n) == 1 and int(nxt) == am[1]
    from home_seek_b200._lib import HS_DEV_BAD_DRAFT
    assert ops.check_status(x.device) & HS_DEV_BAD_DRAFT
