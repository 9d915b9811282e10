"""Expert parallelism on the CPU with two gloo ranks: the expert / shared-row
split (ep.expert_range, ep.shared_slice), id localisation (ep.localize) and the
group plumbing (ExpertParallel.all_reduce over torch.distributed) reproduce the
single-process layer. Each rank's partial sums come from the oracle (the CUDA
kernels need a GPU; tests/test_gpu_ep.py checks them), summed over the two
ranks, combined, and compared with oracle.moe.moe_layer on the full weights."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import inputs as I
from oracle import moe as O


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, T: int, out_q) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from home_seek_b200.ep import ExpertParallel, expert_range, localize, shared_slice
        shape = I.SMALL
        load = I.make_loader(shape)
        gate, bias = I.router_weights(shape.E, shape.D, seed=1)
        sh = I.shared_fp8(shape.D, shape.I_sh, seed=2)
        h = I.hidden(T, shape.D, seed=3 + T)
        idx, w = O.router(h, gate, bias)                       # identical on every rank
        off, held = expert_range(shape.E, rank, world)
        lo, hi = shared_slice(shape.I_sh, rank, world)
        loc = localize(idx, off, held)
        # this rank's partials: its experts (local ids -> global for the loader)
        routed = O.moe_routed_f32(h, torch.where(loc >= 0, loc + off, loc), w, load)
        w13, s13, w2, s2 = sh
        shared = O.shared_expert_f32(h, (w13[:, lo:hi], s13[:, lo // 128:hi // 128], w2[:, lo:hi],
                                         s2[:, lo // 128:hi // 128]))
        buf = torch.stack([routed, shared]).contiguous()
        ExpertParallel(rank, world).all_reduce(buf)
        out = O.ep_combine(buf[0], buf[1])
        ref = O.moe_layer(h, idx, w, load, sh)
        out_q.put((rank, out.float().numpy(), ref.float().numpy(), int((loc >= 0).sum())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("T", [1, 3])
def test_two_rank_expert_parallel_layer_matches_single_process(T):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, T, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort()
    (_, out0, ref, n0), (_, out1, _, n1) = res
    assert n0 + n1 == T * 6                 # every routed pair lands on exactly one rank
    assert np.array_equal(out0, out1)       # the group agrees
    rel = float(np.abs(out0 - ref).max() / max(np.abs(ref).max(), 1e-30))
    assert rel <= 1e-2, rel


def _sharded_rank_main(rank: int, world: int, port: int, T: int, out_q, skip_self: bool = False) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from home_seek_b200.ep import TokenShardedEP, expert_range, localize
        shape = I.SMALL
        load = I.make_loader(shape)
        gate, bias = I.router_weights(shape.E, shape.D, seed=1)
        sh = I.shared_fp8(shape.D, shape.I_sh, seed=2)
        h = I.hidden(T, shape.D, seed=30 + T)
        idx, w = O.router(h, gate, bias)
        lo, hi = rank * T // world, (rank + 1) * T // world     # this rank's token shard
        hl, il, wl = h[lo:hi], idx[lo:hi], w[lo:hi]
        off, held = expert_range(shape.E, rank, world)
        ep = TokenShardedEP(rank, world)
        d, hr, ir, wr = ep.dispatch(hl, il, wl, held, skip_self=skip_self)
        assert int(ir.max()) < held if ir.numel() else True
        # the received rows through this rank's experts (local ids -> global for the loader)
        y = O.moe_routed_f32(hr, torch.where(ir >= 0, ir + off, ir), wr, load)
        own = None
        if skip_self:
            # TokenShardedEP.moe's form: this rank's own experts on its own tokens,
            # run locally and added at this rank's place in the sum
            assert d.send_counts[rank] == 0 and d.recv_counts[rank] == 0
            loc = localize(il, off, held)
            own = O.moe_routed_f32(hl, torch.where(loc >= 0, loc + off, loc), wl, load)
        routed = ep.combine(d, y, hl.shape[0], own=own)
        out = O.ep_combine(routed, O.shared_expert_f32(hl, sh))
        ref = O.moe_layer(hl, il, wl, load, sh)
        ref_routed = O.moe_routed_f32(hl, il, wl, load)
        rr = float((routed - ref_routed).abs().max() / ref_routed.abs().max())
        out_q.put((rank, out.float().numpy(), ref.float().numpy(), rr, sum(d.send_counts), sum(d.recv_counts)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("skip_self", [False, True])
@pytest.mark.parametrize("T,world", [(5, 2), (8, 2), (9, 4)])
def test_token_sharded_dispatch_combine(T, world, skip_self):
    """Prefill-size expert parallelism with the tokens sharded: each rank sends
    its tokens' rows to the ranks holding their experts (gloo all-to-all), the
    receivers run their experts (the oracle here; the kernels on the GPU), the
    f32 results come back and are added per token in rank order: each rank's
    tokens come out as the single-process layer computes them. skip_self is
    TokenShardedEP.moe's form: nothing is sent to the rank itself, its own
    experts' term comes in through combine(own=...)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sharded_rank_main, args=(r, world, port, T, q, skip_self)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort()
    assert sum(r[4] for r in res) == sum(r[5] for r in res)   # every row sent is received
    for _, out, ref, rr, _, _ in res:
        assert rr <= 1e-5, rr                                # f32 sums: only the association differs
        rel = float(np.abs(out - ref).max() / max(np.abs(ref).max(), 1e-30))
        assert rel <= 1e-2, rel


def test_dispatch_lists():
    from home_seek_b200.ep import dispatch_lists
    idx = torch.tensor([[0, 5, -1], [6, 7, 2], [1, 1, 3], [9, -1, -1]])
    toks, ids = dispatch_lists(idx, 4, 2)           # rank 0: experts 0-3, rank 1: 4-7; id 9 goes nowhere
    assert [t.tolist() for t in toks] == [[0, 1, 2], [0, 1]]
    assert ids[0].tolist() == [[0, -1, -1], [-1, -1, 2], [1, 1, 3]]
    assert ids[1].tolist() == [[-1, 1, -1], [2, 3, -1]]


def test_expert_and_shared_splits():
    from home_seek_b200.ep import expert_range, localize, shared_slice
    assert [expert_range(256, r, 8) for r in (0, 7)] == [(0, 32), (224, 32)]
    assert shared_slice(2048, 3, 8) == (768, 1024)
    with pytest.raises(ValueError):
        shared_slice(2048, 0, 16)           # 128-row slices: below the kernels' 256-row granularity
    idx = torch.tensor([[0, 31, 32, 255, -1, 64]])
    assert localize(idx, 32, 32).tolist() == [[-1, -1, 0, -1, -1, -1]]
    assert localize(idx, 0, 32).tolist() == [[0, 31, -1, -1, -1, -1]]
