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


# --- vocabulary split over an expert-parallel group (hs_lm_head_argmax_ep) ---

_HDR = 256
_HEAD_CALLS, _HEAD_POISON = 3, 4
_EMPTY_KEY = (1 << 64) - 1


def _key(b16: int, v: int) -> int:
    """The kernel's ordered key of a bf16 logit (bits b16) at vocab index v."""
    if (b16 & 0x7FFF) > 0x7F80:
        ordv = 0x10000
    else:
        if b16 == 0x8000:
            b16 = 0
        ordv = (0x7FFF - (b16 & 0x7FFF)) if b16 & 0x8000 else 0x8000 + b16
    return (ordv << 32) | (~v & 0xFFFFFFFF)


def _key_region(world: int, D: int) -> int:
    """Byte offset of the lm_head key slots in an exchange buffer."""
    return _HDR + 2 * world * 2 * 8 * D * 4


class _I64View:
    """n 64-bit words at a raw device address, as an int64 tensor."""

    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<i8", "data": (ptr, False), "version": 3}


def _two_rank_buffers(D: int, limit_ns: int = 0):
    import ctypes
    from home_seek_b200 import _lib
    nb = _lib.load().hs_ep_buffer_bytes(2, D)
    bufs = []
    for _ in range(2):
        p = ctypes.c_void_p()
        _lib.call("hs_ep_buffer_alloc", nb, ctypes.byref(p))
        bufs.append(p.value)
    peers = _lib.HsEpPeers()
    peers.rank, peers.world = 0, 2
    peers.recv[0], peers.recv[1] = bufs
    peers.wait_limit_ns = limit_ns
    return bufs, peers


def _words(ptr: int, off: int, n: int) -> torch.Tensor:
    return torch.as_tensor(_I64View(ptr + off, n), device="cuda")


@pytest.mark.parametrize("T,with_drafts", [(1, False), (3, True)])
def test_vocab_split_head_equals_the_whole_head(T, with_drafts):
    """Rank 0 of a two-rank group streams its rows; rank 1's best keys (from
    the head kernel's own bf16 logits over rank 1's rows) are already in rank
    0's buffer, so the kernel's wait is satisfied without another kernel. The
    combined argmax and acceptance equal hs_lm_head_argmax on the whole head,
    and the key slots are emptied and the call counted afterwards."""
    from home_seek_b200 import _lib, ops
    D, V = 512, 5000
    g = torch.Generator(device="cuda").manual_seed(77 + T)
    x = torch.randn(T, D, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(V, D, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    drafts = None
    full = ops.lm_head_argmax(x, w)
    if with_drafts:  # the first draft right, the second wrong
        drafts = torch.stack([full[0][0], (full[0][1] + 1) % V]).to(torch.int64)
        full = ops.lm_head_argmax(x, w, draft_ids=drafts)
    bufs, peers = _two_rank_buffers(D)
    try:
        r1_0, r1_n = ops.vocab_rows(V, 1, 2)
        _, _, _, lg1 = ops.lm_head_argmax(x, w[r1_0:r1_0 + r1_n].contiguous(), want_logits=True)
        bits = lg1.view(torch.int16).cpu().numpy().astype(np.int64) & 0xFFFF
        keys = [max(_key(int(bits[t, j]), r1_0 + j) for j in range(r1_n)) for t in range(T)]
        slot0_src1 = _key_region(2, D) + (0 * 8 + 1) * 16 * 8
        _words(bufs[0], slot0_src1, T).copy_(torch.tensor([k - (1 << 64) if k >= 1 << 63 else k for k in keys],
                                                          dtype=torch.int64))
        out = ops.lm_head_argmax_ep(x, w, peers, draft_ids=drafts)
        torch.cuda.synchronize()
        assert ops.check_status(x.device) == 0
        for got, want in zip(out, full):
            assert torch.equal(got, want)
        region = _words(bufs[0], _key_region(2, D), 2 * 8 * 16).cpu()
        assert bool((region == -1).all())                          # every key slot empty again
        assert int(_words(bufs[0], 0, 8)[_HEAD_CALLS]) == 1
    finally:
        for b in bufs:
            _lib.call("hs_ep_buffer_free", b)


def test_vocab_split_head_wait_runs_out_and_poisons():
    """Nothing stores rank 1's keys: the bounded wait (50 ms) gives up with
    HS_DEV_TIMEOUT, the buffer is poisoned and the counter kept, and the next
    call reports the timeout at once without storing anything."""
    import time
    from home_seek_b200 import _lib, ops
    D, V, T = 512, 3000, 2
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(T, D, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(V, D, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    bufs, peers = _two_rank_buffers(D, limit_ns=50_000_000)
    try:
        st = ops.status_word(x.device)
        st.zero_()
        ops.lm_head_argmax_ep(x, w, peers)
        torch.cuda.synchronize()
        assert int(st.item()) & _lib.HS_DEV_TIMEOUT
        hdr = _words(bufs[0], 0, 8).cpu()
        assert int(hdr[_HEAD_POISON]) == 1 and int(hdr[_HEAD_CALLS]) == 0
        peer_keys = _words(bufs[1], _key_region(2, D), 2 * 8 * 16).cpu()
        st.zero_()
        t0 = time.perf_counter()
        ops.lm_head_argmax_ep(x, w, peers)
        torch.cuda.synchronize()
        assert time.perf_counter() - t0 < 0.04                      # refused, no second wait
        assert int(st.item()) & _lib.HS_DEV_TIMEOUT
        assert torch.equal(_words(bufs[1], _key_region(2, D), 2 * 8 * 16).cpu(), peer_keys)
    finally:
        st.zero_()
        for b in bufs:
            _lib.call("hs_ep_buffer_free", b)
