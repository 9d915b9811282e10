"""Expert parallelism on the GPU. On one GPU the group is emulated: the full
store is split with ep.shard_store, each shard's hs_moe_ffn_fp4_partials runs
on its localised ids, the shards' f32 partials are added (what the all-reduce
does) and hs_moe_combine must give the single-call output. With two or more
GPUs the same check runs over a real NCCL group (one process per GPU)."""
from __future__ import annotations

import os
import socket

import pytest
import torch

from oracle import inputs as I

pytestmark = pytest.mark.gpu

MOE_TOL = 1e-2


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float().cpu(), b.float().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp(min=1e-30))


def _full_store(device="cuda"):
    from home_seek_b200.expert_store import HBMExpertStore
    shape = I.SMALL
    st = HBMExpertStore(1, shape.E, shape.D, shape.I, shape.I_sh, device=device, with_router=False)
    load = I.make_loader(shape)
    for e in range(shape.E):
        st.set_expert(0, e, *load(e))
    st.set_shared(0, *I.shared_fp8(shape.D, shape.I_sh, seed=2))
    return st


@pytest.mark.parametrize("T", [1, 3, 24, 1024])  # 1024: segmented plan + token-major kernels on every shard
def test_emulated_two_rank_partials_combine_to_the_single_call(T):
    from home_seek_b200 import ops
    from home_seek_b200.ep import localize, shard_store
    shape = I.SMALL
    full = _full_store()
    gate, bias = I.router_weights(shape.E, shape.D, seed=1)
    h = I.hidden(T, shape.D, seed=5 + T).cuda()
    idx, w = ops.router_topk(h, gate.cuda(), bias.cuda(), shape.K, 1.5)
    dup = 1 if T == 1 else 0
    ref = ops.moe_ffn(full.desc(0), full.dims, h, idx, w, use_shared=True, dup_mode=dup)
    ref_f32 = torch.empty(T, shape.D, dtype=torch.float32, device="cuda")
    ops.moe_ffn(full.desc(0), full.dims, h, idx, w, use_shared=False, dup_mode=dup, out_f32=ref_f32)
    total = torch.zeros(2, T, shape.D, dtype=torch.float32, device="cuda")
    for r in range(2):
        sh = shard_store(full, r, 2)
        part = ops.moe_ffn_partials(sh.desc(0), sh.dims, h, localize(idx, sh.expert_offset, sh.E_local), w,
                                    use_shared=True, dup_mode=dup)
        total += part
    out = ops.moe_combine(total)
    assert ops.check_status(torch.device("cuda")) == 0
    assert _rel(out, ref) <= MOE_TOL, _rel(out, ref)
    assert _rel(total[0], ref_f32) <= 1e-3, _rel(total[0], ref_f32)   # routed f32 sums, before rounding
    # fused combine + residual add + norm equals the two-step form
    from oracle import mtp as OM
    res = torch.randn(T, shape.D, device="cuda").to(torch.bfloat16)
    nw = (1 + 0.1 * torch.randn(shape.D, device="cuda")).to(torch.bfloat16)
    h2, x2 = ops.moe_combine_add_rms_norm(total, res, nw)
    h3, x3 = ops.add_rms_norm(res, out, nw)
    assert torch.equal(h2, h3) and torch.equal(x2, x3)
    assert _rel(x2, OM.rms_norm((res.cpu() + out.cpu()), nw.cpu())) <= 2e-2


@pytest.mark.parametrize("T", [1, 3])
def test_emulated_eight_shards_full_shape_combine_to_the_single_call(T):
    """Eight expert-parallel shards of the full config-0 shape on one GPU:
    at T = 1 and 3 most shards hold few or none of the tokens' experts, so
    their gate/up phase is little more than their eighth of the shared
    expert and runs on fewer stream-K CTAs (at least four steps each). The
    shards' f32 partials, summed and combined, equal the single call within
    the MoE tolerance, and the routed sums within f32 association error."""
    from home_seek_b200 import ops
    from home_seek_b200.ep import localize, shard_store
    from home_seek_b200.expert_store import HBMExpertStore
    dev = torch.device("cuda")
    full = HBMExpertStore(1, 256, 4096, 2048, 2048, device=dev)
    full.fill_random(47)
    g = torch.Generator(device=dev).manual_seed(11 + T)
    h = (torch.randn(T, 4096, generator=g, device=dev) * 2).to(torch.bfloat16)
    gate = (torch.randn(256, 4096, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    bias = (torch.randn(256, generator=g, device=dev) * 0.1).to(torch.bfloat16)
    idx, w = ops.router_topk(h, gate, bias, 6, 1.5)
    dup = 1 if T == 1 else 0
    ref = ops.moe_ffn(full.desc(0), full.dims, h, idx, w, use_shared=True, dup_mode=dup)
    ref_f32 = torch.empty(T, 4096, dtype=torch.float32, device=dev)
    ops.moe_ffn(full.desc(0), full.dims, h, idx, w, use_shared=False, dup_mode=dup, out_f32=ref_f32)
    total = torch.zeros(2, T, 4096, dtype=torch.float32, device=dev)
    held = []
    for r in range(8):
        sh = shard_store(full, r, 8)
        loc = localize(idx, sh.expert_offset, sh.E_local)
        held.append(int((loc >= 0).sum()))
        total += ops.moe_ffn_partials(sh.desc(0), sh.dims, h, loc, w, use_shared=True, dup_mode=dup)
        del sh
    out = ops.moe_combine(total)
    assert ops.check_status(dev) == 0
    if T == 1:
        assert min(held) == 0, held  # some shard's phase is the shared slice alone
    assert _rel(out, ref) <= MOE_TOL, _rel(out, ref)
    assert _rel(total[0], ref_f32) <= 1e-3, _rel(total[0], ref_f32)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_rank(rank: int, world: int, port: int, q) -> None:
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        from home_seek_b200 import ops
        from home_seek_b200.ep import ExpertParallel, shard_store
        shape = I.SMALL
        full = _full_store(dev)
        gate, bias = I.router_weights(shape.E, shape.D, seed=1)
        h = I.hidden(3, shape.D, seed=9).to(dev)
        idx, w = ops.router_topk(h, gate.to(dev), bias.to(dev), shape.K, 1.5)
        ref = ops.moe_ffn(full.desc(0), full.dims, h, idx, w, use_shared=True)
        ep = ExpertParallel(rank, world)
        out = ep.moe(shard_store(full, rank, world), 0, h, idx, w, 0)
        torch.cuda.synchronize()
        q.put((rank, _rel(out, ref)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_nccl_expert_parallel_matches_single_gpu():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, rel in res:
        assert rel <= MOE_TOL, (rank, rel)


def _p2p_rank(rank: int, world: int, port: int, q) -> None:
    """One rank of a two-GPU group: four consecutive layer calls through the
    peer-memory exchange (both slots used twice) against the single-GPU layer
    call on the full store, and the ranks' results bit-identical."""
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    px = None
    try:
        from home_seek_b200 import ops
        from home_seek_b200.ep import PeerExchange, shard_store
        from home_seek_b200.expert_store import HBMExpertStore
        full = HBMExpertStore(2, 256, 4096, 2048, 2048, device=dev)
        full.fill_random(31)
        sh = shard_store(full, rank, world)
        px = PeerExchange(rank, world, 4096)
        g = torch.Generator(device=dev).manual_seed(4)
        h0 = (torch.randn(3, 4096, generator=g, device=dev) * 2).to(torch.bfloat16)
        nw = (1 + 0.05 * torch.randn(2, 4096, generator=g, device=dev)).to(torch.bfloat16)
        h_ep, h_ref = h0.clone(), h0.clone()
        worst = 0.0
        for call in range(4):
            l = call % 2
            lw = full.layers[l]
            ops.moe_layer(full.desc(l), full.dims, h_ref, nw[l], lw.gate, lw.bias, 6, 1.5, h_out=h_ref)
            ops.moe_layer_ep(sh.desc(l), sh.dims, h_ep, nw[l], lw.gate, lw.bias, 6, 1.5, px.peers,
                             num_experts=256, expert_offset=sh.expert_offset, h_out=h_ep)
            torch.cuda.synchronize()
            d = (h_ep.float() - h_ref.float()).abs().max().item() / h_ref.float().abs().max().item()
            worst = max(worst, d)
            h_ep.copy_(h_ref)  # next call from the same input on both paths
        chain_same = _chained_equals_unchained(sh, nw, px.peers, h0)
        # the vocabulary split lm_head over the same buffers: three calls (both
        # key slots used, one twice), each equal to the whole-head call
        head_same = True
        w = (torch.randn(129280, 4096, generator=torch.Generator(device=dev).manual_seed(8), device=dev)
             * 0.02).to(torch.bfloat16)
        for T in (3, 1, 3):
            x = torch.randn(T, 4096, generator=g, device=dev).to(torch.bfloat16)
            dist.broadcast(x, src=0)
            drafts = None
            if T == 3:
                am = ops.lm_head_argmax(x, w)[0]
                drafts = torch.stack([am[0], (am[1] + 1) % 129280])
            ref = ops.lm_head_argmax(x, w, draft_ids=drafts)
            got = ops.lm_head_argmax_ep(x, w, px.peers, draft_ids=drafts)
            torch.cuda.synchronize()
            head_same = head_same and all(torch.equal(a, b) for a, b in zip(got, ref))
        status = ops.check_status(dev)
        gathered = [torch.empty_like(h_ep) for _ in range(world)]
        dist.all_gather(gathered, h_ep)
        same = all(torch.equal(gathered[0], x) for x in gathered)
        q.put((rank, worst, status, same and head_same and chain_same))
    finally:
        if px is not None:
            px.close()
        dist.destroy_process_group()


def _chained_equals_unchained(sh, nw, peers, h0) -> bool:
    """Five layer calls chained (each exchange completed by the next call's
    route kernel, the last by ep_combine_pending) against the same five
    unchained calls, for T = 3, 1 and 8 (T rows of h0 repeated), use_shared
    alternating so the pending call's flag matters: bit-identical rows."""
    from home_seek_b200 import ops
    same = True
    for T in (3, 1, 8):
        hx = h0.repeat((T + h0.shape[0] - 1) // h0.shape[0], 1)[:T].contiguous()
        hu, hc = hx.clone(), hx.clone()
        plan = [(call % 2, call % 3 != 1) for call in range(5)]
        for l, us in plan:
            lw = sh.layers[l]
            ops.moe_layer_ep(sh.desc(l), sh.dims, hu, nw[l], lw.gate, lw.bias, 6, 1.5, peers, use_shared=us,
                             num_experts=256, expert_offset=sh.expert_offset, h_out=hu)
        pending = None
        for l, us in plan:
            lw = sh.layers[l]
            ops.moe_layer_ep_chained(sh.desc(l), sh.dims, hc, nw[l], lw.gate, lw.bias, 6, 1.5, peers,
                                     prev_pending=pending is not None, prev_use_shared=bool(pending),
                                     use_shared=us, num_experts=256, expert_offset=sh.expert_offset)
            pending = us
        ops.ep_combine_pending(peers, hc, use_shared=pending)
        torch.cuda.synchronize()
        same = same and torch.equal(hu, hc)
    return same


def test_chained_peer_exchange_single_rank_matches_unchained():
    """A one-rank peer-memory group: the chained layer calls (the exchange
    completed inside the next call's route kernel) give the unchained calls'
    rows bit for bit, and the call counter ends where the unchained calls
    leave it."""
    import ctypes
    from home_seek_b200 import _lib, ops
    from home_seek_b200.ep import shard_store
    from home_seek_b200.expert_store import HBMExpertStore
    dev = torch.device("cuda")
    full = HBMExpertStore(2, 256, 4096, 2048, 2048, device=dev)
    full.fill_random(37)
    sh = shard_store(full, 0, 1)
    buf = ctypes.c_void_p()
    _lib.call("hs_ep_buffer_alloc", _lib.load().hs_ep_buffer_bytes(1, 4096), ctypes.byref(buf))
    try:
        peers = _lib.HsEpPeers()
        peers.rank, peers.world = 0, 1
        peers.recv[0] = buf.value
        g = torch.Generator(device=dev).manual_seed(5)
        h0 = (torch.randn(3, 4096, generator=g, device=dev) * 2).to(torch.bfloat16)
        nw = (1 + 0.05 * torch.randn(2, 4096, generator=g, device=dev)).to(torch.bfloat16)
        ops.check_status(dev)
        assert _chained_equals_unchained(sh, nw, peers, h0)
        assert ops.check_status(dev) == 0
        hdr = torch.as_tensor(_DevView(buf.value, 4), device=dev).cpu().tolist()
        assert hdr[0] == 30 and hdr[2] == 0, hdr  # 3 T x (5 unchained + 5 chained) calls
    finally:
        torch.cuda.synchronize()
        _lib.call("hs_ep_buffer_free", buf.value)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_p2p_expert_parallel_layer_matches_single_gpu():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_p2p_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, worst, status, same in res:
        assert status == 0, (rank, status)
        assert same, rank
        # bf16(h + y) against the single-GPU call: y differs by f32 summation order only
        assert worst <= 2e-2, (rank, worst)


class _ThreadExchange:
    """In-process all-to-all between rank threads on one GPU (each rank on its
    own stream): a rank posts its input pieces, waits for every rank, gathers
    the pieces addressed to it, and waits again before the next exchange."""

    def __init__(self, world: int):
        import threading
        self.world = world
        self.bar = threading.Barrier(world, timeout=120)
        self.box = {}

    def for_rank(self, rank: int):
        def a2a(out, inp, out_splits, in_splits):
            torch.cuda.synchronize()
            self.box[rank] = list(torch.split(inp, in_splits))
            self.bar.wait()
            pieces = [self.box[s][rank] for s in range(self.world)]
            if out.numel():
                out.copy_(torch.cat(pieces))
            torch.cuda.synchronize()
            self.bar.wait()
        return a2a


@pytest.mark.parametrize("T", [6, 1024])   # 1024: the token-major kernels on the received rows
def test_emulated_token_sharded_two_ranks_match_the_single_call(T):
    """Prefill-size expert parallelism with sharded tokens (TokenShardedEP),
    two ranks emulated as threads on one GPU: each rank's tokens come out as
    the single-GPU call on the full store computes them."""
    import threading
    from home_seek_b200 import ops
    from home_seek_b200.ep import TokenShardedEP, shard_store
    shape = I.SMALL
    full = _full_store()
    gate, bias = I.router_weights(shape.E, shape.D, seed=1)
    h = I.hidden(T, shape.D, seed=70 + T).cuda()
    idx, w = ops.router_topk(h, gate.cuda(), bias.cuda(), shape.K, 1.5)
    ref = ops.moe_ffn(full.desc(0), full.dims, h, idx, w, use_shared=True)
    shards = [shard_store(full, r, 2, shared="replicated") for r in range(2)]
    for s in shards:
        s.desc(0)
    torch.cuda.synchronize()
    ex = _ThreadExchange(2)
    outs, errs = [None, None], []

    def run(r):
        try:
            with torch.cuda.stream(torch.cuda.Stream()):
                lo, hi = r * T // 2, (r + 1) * T // 2
                ep = TokenShardedEP(r, 2, all_to_all=ex.for_rank(r))
                outs[r] = ep.moe(shards[r], 0, h[lo:hi].contiguous(), idx[lo:hi].contiguous(), w[lo:hi].contiguous())
                torch.cuda.synchronize()
        except BaseException as e:  # noqa: BLE001
            errs.append(e)
            ex.bar.abort()

    th = [threading.Thread(target=run, args=(r,)) for r in range(2)]
    for t in th:
        t.start()
    for t in th:
        t.join(timeout=300)
    assert not errs, errs
    out = torch.cat(outs)
    assert ops.check_status(torch.device("cuda")) == 0
    assert _rel(out, ref) <= MOE_TOL, _rel(out, ref)


def _sharded_nccl_rank(rank: int, world: int, port: int, q) -> None:
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        from home_seek_b200 import ops
        from home_seek_b200.ep import TokenShardedEP, shard_store
        shape = I.SMALL
        full = _full_store(dev)
        gate, bias = I.router_weights(shape.E, shape.D, seed=1)
        T = 1024
        h = I.hidden(T, shape.D, seed=11).to(dev)
        idx, w = ops.router_topk(h, gate.to(dev), bias.to(dev), shape.K, 1.5)
        lo, hi = rank * T // world, (rank + 1) * T // world
        ref = ops.moe_ffn(full.desc(0), full.dims, h[lo:hi], idx[lo:hi], w[lo:hi], use_shared=True)
        out = TokenShardedEP(rank, world).moe(shard_store(full, rank, world, shared="replicated"), 0,
                                              h[lo:hi].contiguous(), idx[lo:hi].contiguous(), w[lo:hi].contiguous())
        torch.cuda.synchronize()
        q.put((rank, _rel(out, ref)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_nccl_token_sharded_expert_parallel_matches_single_gpu():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sharded_nccl_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, rel in res:
        assert rel <= MOE_TOL, (rank, rel)


def _sharded_c_rank(rank: int, world: int, port: int, q) -> None:
    """hs_ep_dispatch_combine (NcclTokenShardedEP) against TokenShardedEP on the
    same shards (identical bits) and the single-GPU call; uneven token shards."""
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    ep = None
    try:
        from home_seek_b200 import ops
        from home_seek_b200.ep import NcclTokenShardedEP, TokenShardedEP, shard_store
        shape = I.SMALL
        full = _full_store(dev)
        gate, bias = I.router_weights(shape.E, shape.D, seed=1)
        T = 1000
        h = I.hidden(T, shape.D, seed=13).to(dev)
        idx, w = ops.router_topk(h, gate.to(dev), bias.to(dev), shape.K, 1.5)
        cuts = {2: [0, 563, 1000], 4: [0, 250, 463, 750, 1000]}[world]  # uneven token shards
        lo, hi = cuts[rank], cuts[rank + 1]
        T_max = max(cuts[r + 1] - cuts[r] for r in range(world))
        st = shard_store(full, rank, world, shared="replicated")
        hl, il, wl = h[lo:hi].contiguous(), idx[lo:hi].contiguous(), w[lo:hi].contiguous()
        ref = ops.moe_ffn(full.desc(0), full.dims, hl, il, wl, use_shared=True)
        py = TokenShardedEP(rank, world).moe(st, 0, hl, il, wl)
        ep = NcclTokenShardedEP(rank, world, T_max)
        c1 = ep.moe(st, 0, hl, il, wl)
        c2 = ep.moe(st, 0, hl, il, wl)   # the workspace's second use
        torch.cuda.synchronize()
        q.put((rank, hi - lo, bool(torch.equal(c1, py)), bool(torch.equal(c2, py)), _rel(c1, ref)))
    finally:
        if ep is not None:
            ep.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_nccl_dispatch_combine_c_abi_matches_token_sharded_ep(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sharded_c_rank, args=(r, world, port, q), daemon=True) for r in range(world)]
    for p in procs:
        p.start()
    try:  # a rank that fails leaves its peers in NCCL waits: end them all
        res = sorted(q.get(timeout=150) for _ in procs)
        for p in procs:
            p.join(timeout=60)
            assert p.exitcode == 0
    finally:
        for p in procs:
            if p.is_alive():
                p.terminate()
    assert sum(r[1] for r in res) == 1000
    for rank, _, eq1, eq2, rel in res:
        assert eq1 and eq2, rank
        assert rel <= MOE_TOL, (rank, rel)


def test_dispatch_plan_matches_dispatch_lists():
    """hs_ep_dispatch_plan's lists (kernel) are dispatch_lists' with this rank's
    own list empty, and its own ids are localize's, on ids with -1 and ids past
    the group's experts."""
    from home_seek_b200.ep import dispatch_lists, dispatch_plan, localize
    g = torch.Generator().manual_seed(3)
    for T, world, epr in [(1, 2, 8), (37, 4, 8), (1500, 8, 32), (0, 2, 8)]:
        idx = torch.randint(-1, world * epr + 3, (T, 6), generator=g)
        for rank in range(world):
            counts, pos, own = dispatch_plan(idx.cuda(), epr, world, rank)
            counts, pos, own = counts.cpu(), pos.cpu(), own.cpu()
            toks, _ = dispatch_lists(idx, epr, world)
            for q in range(world):
                want = toks[q].tolist() if q != rank else []
                assert int(counts[q]) == len(want), (T, world, rank, q)
                got = [t for t in range(T) if int(pos[t, q]) >= 0]
                assert got == want
                assert [int(pos[t, q]) for t in got] == list(range(len(want)))
            if T:
                assert torch.equal(own, localize(idx, rank * epr, epr))


def test_nccl_dispatch_combine_single_rank_is_the_partials_call():
    """world = 1 (no exchange, no host synchronisation): the C-ABI call is
    hs_moe_ffn_fp4_partials on the tokens plus hs_moe_combine, bit for bit."""
    from home_seek_b200 import ops
    from home_seek_b200.ep import NcclTokenShardedEP
    shape = I.SMALL
    st = _full_store()
    gate, bias = I.router_weights(shape.E, shape.D, seed=1)
    ep = NcclTokenShardedEP(0, 1, 300)
    try:
        for T in (0, 1, 7, 300):
            h = I.hidden(max(T, 1), shape.D, seed=17)[:T].cuda().contiguous()
            if T:
                idx, w = ops.router_topk(h, gate.cuda(), bias.cuda(), shape.K, 1.5)
            else:
                idx = torch.zeros(0, shape.K, dtype=torch.int64, device="cuda")
                w = torch.zeros(0, shape.K, dtype=torch.float32, device="cuda")
            out = ep.moe(st, 0, h, idx, w)
            if T:
                parts = ops.moe_ffn_partials(st.desc(0), st.dims, h, idx, w, use_shared=True)
                assert torch.equal(out, ops.moe_combine(parts, use_shared=True)), T
    finally:
        ep.close()


class _DevView:
    """A raw device pointer as an int64 array torch can wrap (CUDA array interface)."""

    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<i8", "data": (ptr, False), "version": 3}


def test_peer_exchange_wait_runs_out_and_poisons_the_buffer():
    """Rank 0 of a two-rank peer-memory group whose rank 1 never runs (both
    receive buffers live on this GPU and nothing stores rank 1's rows): the
    combine's bounded wait runs out (a short limit), the call reports
    HS_DEV_TIMEOUT and leaves h untouched, and the next call on the poisoned
    buffer refuses at once with the same status instead of waiting again."""
    import ctypes
    import time
    from home_seek_b200 import _lib, ops
    from home_seek_b200.ep import shard_store
    from home_seek_b200.expert_store import HBMExpertStore
    dev = torch.device("cuda")
    full = HBMExpertStore(1, 256, 4096, 2048, 2048, device=dev)
    full.fill_random(41)
    sh = shard_store(full, 0, 2)
    lib = _lib.load()
    nb = lib.hs_ep_buffer_bytes(2, 4096)
    bufs = [ctypes.c_void_p(), ctypes.c_void_p()]
    for b in bufs:
        _lib.call("hs_ep_buffer_alloc", nb, ctypes.byref(b))
    try:
        peers = _lib.HsEpPeers()
        peers.rank, peers.world = 0, 2
        peers.recv[0], peers.recv[1] = bufs[0].value, bufs[1].value
        peers.wait_limit_ns = 50_000_000  # 50 ms
        g = torch.Generator(device=dev).manual_seed(8)
        h = (torch.randn(3, 4096, generator=g, device=dev)).to(torch.bfloat16)
        nw = (1 + 0.05 * torch.randn(4096, generator=g, device=dev)).to(torch.bfloat16)
        lw = full.layers[0]
        ops.check_status(dev)
        for call in range(2):
            h_out = torch.full_like(h, 7.0)
            t0 = time.monotonic()
            ops.moe_layer_ep(sh.desc(0), sh.dims, h, nw, lw.gate, lw.bias, 6, 1.5, peers, num_experts=256,
                             expert_offset=0, h_out=h_out)
            torch.cuda.synchronize()
            dt = time.monotonic() - t0
            st = ops.check_status(dev)
            assert st & _lib.HS_DEV_TIMEOUT, (call, st)
            assert bool((h_out == 7.0).all()), call  # nothing combined
            assert dt < 1.5, (call, dt)              # bounded by the 50 ms limit (first) or refused (second)
        # the call counter stayed at 0 and the poison word is set
        hdr = torch.as_tensor(_DevView(bufs[0].value, 4), device=dev).cpu().tolist()
        assert hdr[0] == 0 and hdr[2] != 0, hdr
    finally:
        torch.cuda.synchronize()
        for b in bufs:
            _lib.call("hs_ep_buffer_free", b.value)


def test_chained_peer_exchange_wait_runs_out_and_poisons_the_buffer():
    """The chained form of the check above: the first chained call leaves its
    exchange pending; the second call's route kernel waits for rank 1's rows
    (a 50 ms limit), reports HS_DEV_TIMEOUT, leaves h untouched and poisons the
    buffer; ep_combine_pending on it then refuses at once."""
    import ctypes
    import time
    from home_seek_b200 import _lib, ops
    from home_seek_b200.ep import shard_store
    from home_seek_b200.expert_store import HBMExpertStore
    dev = torch.device("cuda")
    full = HBMExpertStore(1, 256, 4096, 2048, 2048, device=dev)
    full.fill_random(43)
    sh = shard_store(full, 0, 2)
    lib = _lib.load()
    nb = lib.hs_ep_buffer_bytes(2, 4096)
    bufs = [ctypes.c_void_p(), ctypes.c_void_p()]
    for b in bufs:
        _lib.call("hs_ep_buffer_alloc", nb, ctypes.byref(b))
    try:
        peers = _lib.HsEpPeers()
        peers.rank, peers.world = 0, 2
        peers.recv[0], peers.recv[1] = bufs[0].value, bufs[1].value
        peers.wait_limit_ns = 50_000_000  # 50 ms
        g = torch.Generator(device=dev).manual_seed(9)
        h = (torch.randn(3, 4096, generator=g, device=dev)).to(torch.bfloat16)
        nw = (1 + 0.05 * torch.randn(4096, generator=g, device=dev)).to(torch.bfloat16)
        lw = full.layers[0]
        ops.check_status(dev)
        h_before = h.clone()
        for prev in (False, True):
            t0 = time.monotonic()
            ops.moe_layer_ep_chained(sh.desc(0), sh.dims, h, nw, lw.gate, lw.bias, 6, 1.5, peers,
                                     prev_pending=prev, num_experts=256, expert_offset=0)
            torch.cuda.synchronize()
            dt = time.monotonic() - t0
            st = ops.check_status(dev)
            assert bool(st & _lib.HS_DEV_TIMEOUT) == prev, (prev, st)
            assert dt < 1.5, (prev, dt)
            assert torch.equal(h, h_before), prev
        t0 = time.monotonic()
        ops.ep_combine_pending(peers, h)
        torch.cuda.synchronize()
        assert ops.check_status(dev) & _lib.HS_DEV_TIMEOUT
        assert time.monotonic() - t0 < 1.5
        assert torch.equal(h, h_before)
        hdr = torch.as_tensor(_DevView(bufs[0].value, 4), device=dev).cpu().tolist()
        assert hdr[0] == 0 and hdr[2] != 0, hdr
    finally:
        torch.cuda.synchronize()
        for b in bufs:
            _lib.call("hs_ep_buffer_free", b.value)
