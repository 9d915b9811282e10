"""Expert parallelism for the MoE layer.

Reference being replaced: `_forward_ffn_ep` (inference_engine/engine.py:1575-1709)
with its worker thread `_EPWorker` (inference_engine/parallel.py:189-290). The
reference keeps every token on every GPU, splits the routed experts of the layer
over the GPUs, runs each GPU on all tokens and adds the GPUs' bf16 outputs and
the shared expert on GPU 0.

Here one process per GPU (torch.distributed, NCCL over NVLink): rank r of n holds
the routed experts [r E/n, (r+1) E/n) of every layer and rows
[r I_sh/n, (r+1) I_sh/n) of the shared expert's intermediate dimension (an
exact split: each intermediate unit's SwiGLU lives on one rank, the down
projection is a sum over units). Every rank routes identically (replicated
router, deterministic kernels), runs `hs_moe_ffn_fp4_partials` on its experts,
which writes the UN-ROUNDED f32 routed and shared sums, and one all-reduce adds
the ranks' partials in f32; the combine then rounds exactly where the
single-GPU call rounds (bf16(bf16(routed) + bf16(shared))), fused with the
layer's residual add and the next norm. There is no token dispatch at decode
sizes: the tokens are already on every rank, so the only exchange is the
[2, T, D] f32 combine.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Callable, Optional

import torch

from . import _lib, ops
from .expert_store import HBMExpertStore


def expert_range(num_experts: int, rank: int, world: int) -> tuple[int, int]:
    """(offset, count) of the routed experts rank `rank` holds."""
    if num_experts % world:
        raise ValueError(f"{num_experts} experts do not split over {world} ranks")
    n = num_experts // world
    return rank * n, n


def shared_slice(shared_inter: int, rank: int, world: int) -> tuple[int, int]:
    """[lo, hi) of the shared expert's intermediate rows rank `rank` holds
    (a multiple of 256 wide: the kernels' shared-expert granularity)."""
    if shared_inter % (256 * world):
        raise ValueError(f"shared intermediate size {shared_inter} does not split into {world} x 256k")
    n = shared_inter // world
    return rank * n, (rank + 1) * n


def localize(topk_idx: torch.Tensor, offset: int, held: int) -> torch.Tensor:
    """Global expert ids -> this rank's local ids; experts held elsewhere -> -1
    (skipped by the kernels), as the reference's per-GPU `topk_per_gpu`
    (engine.py:1617-1622)."""
    inside = (topk_idx >= offset) & (topk_idx < offset + held)
    return torch.where(inside, topk_idx - offset, torch.full_like(topk_idx, -1))


class PeerExchange:
    """The receive buffers of the peer-memory exchange (hs_moe_layer_fp4_ep).

    Each rank's buffer is allocated by the library, its CUDA IPC handle is
    exchanged over the process group, and every other rank maps it, so a down
    phase can store its rows into all ranks' buffers over NVLink. Created
    collectively (every rank, same order); `close` is collective too and must
    run after all GPU work that uses the buffers has finished."""

    def __init__(self, rank: int, world: int, hidden: int, group=None):
        import torch.distributed as dist
        lib = _lib.load()
        nbytes = lib.hs_ep_buffer_bytes(world, hidden)
        if nbytes == 0:
            raise ValueError(f"no peer exchange for world={world}, hidden={hidden}")
        local = ctypes.c_void_p()
        _lib.call("hs_ep_buffer_alloc", nbytes, ctypes.byref(local))
        self.local = local.value
        hnd = (ctypes.c_uint8 * _lib.HS_IPC_HANDLE_BYTES)()
        _lib.call("hs_ipc_get_handle", self.local, hnd, _lib.HS_IPC_HANDLE_BYTES)
        handles = [None] * world
        dist.all_gather_object(handles, bytes(hnd), group=group)
        self.group = group
        self.mapped = []
        peers = _lib.HsEpPeers()
        peers.rank = rank
        peers.world = world
        for q in range(world):
            if q == rank:
                peers.recv[q] = self.local
                continue
            ptr = ctypes.c_void_p()
            buf = (ctypes.c_uint8 * _lib.HS_IPC_HANDLE_BYTES).from_buffer_copy(handles[q])
            _lib.call("hs_ipc_open_handle", buf, ctypes.byref(ptr))
            peers.recv[q] = ptr.value
            self.mapped.append(ptr.value)
        self.peers = peers
        dist.barrier(group=group)  # every rank has mapped every buffer before anyone stores

    def close(self) -> None:
        import torch.distributed as dist
        torch.cuda.synchronize()
        dist.barrier(group=self.group)  # no rank stores into a buffer that is going away
        for ptr in self.mapped:
            _lib.call("hs_ipc_close_handle", ptr)
        self.mapped = []
        dist.barrier(group=self.group)
        _lib.call("hs_ep_buffer_free", self.local)
        self.local = None


@dataclass
class ExpertParallel:
    """One rank's view of the expert-parallel group. `all_reduce` sums a tensor
    over the group in place (default: torch.distributed on `group`). With
    `peers` set (a PeerExchange), decode-size layers exchange their partial
    sums through NVLink peer memory inside the layer call instead."""
    rank: int
    world: int
    group: Optional[object] = None
    all_reduce: Optional[Callable[[torch.Tensor], None]] = None
    peers: Optional[PeerExchange] = None

    def __post_init__(self):
        if self.all_reduce is None:
            import torch.distributed as dist
            grp = self.group

            def _ar(t: torch.Tensor) -> None:
                dist.all_reduce(t, op=dist.ReduceOp.SUM, group=grp)

            self.all_reduce = _ar

    def partials(self, store: HBMExpertStore, layer: int, x: torch.Tensor, topk_idx: torch.Tensor,
                 topk_w: torch.Tensor, dup_mode: int, use_shared: bool = True,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """This rank's f32 partial sums [2, T, D] for normed rows x, summed over
        the group on return."""
        idx = localize(topk_idx, store.expert_offset, store.E_local)
        buf = ops.moe_ffn_partials(store.desc(layer), store.dims, x, idx, topk_w, use_shared=use_shared,
                                   dup_mode=dup_mode, out=out)
        self.all_reduce(buf)
        return buf

    def moe(self, store: HBMExpertStore, layer: int, x: torch.Tensor, topk_idx: torch.Tensor,
            topk_w: torch.Tensor, dup_mode: int, use_shared: bool = True) -> torch.Tensor:
        """The layer's MoE output [T, D] bf16 (same on every rank)."""
        buf = self.partials(store, layer, x, topk_idx, topk_w, dup_mode, use_shared)
        return ops.moe_combine(buf, use_shared=use_shared and store.I_sh > 0)


def shard_store(full: HBMExpertStore, rank: int, world: int, device=None, shared: str = "split") -> HBMExpertStore:
    """Rank `rank`'s slice of a full store: its routed experts, the replicated
    router, and its rows of the shared expert (shared="split", the decode
    scheme) or all of them (shared="replicated", the token-sharded prefill
    scheme of TokenShardedEP). For tests and for loading one set of weights
    onto an expert-parallel group."""
    from .layout import untile_rows
    if shared not in ("split", "replicated"):
        raise ValueError(f"shared must be 'split' or 'replicated', not {shared!r}")
    dev = torch.device(device) if device is not None else full.device
    off, held = expert_range(full.E, rank, world)
    if not full.I_sh:
        lo, hi = 0, 0
    elif shared == "split":
        lo, hi = shared_slice(full.I_sh, rank, world)
    else:
        lo, hi = 0, full.I_sh
    hash_layers = sum(1 for lw in full.layers if lw.tid2eid is not None)
    vocab = full.layers[0].tid2eid.shape[0] if hash_layers else 129280
    out = HBMExpertStore(full.num_layers, full.E, full.D, full.I, hi - lo if full.I_sh else None, device=dev,
                         with_router=full.layers[0].gate is not None, hash_layers=hash_layers, vocab_size=vocab,
                         top_k=full.K, expert_offset=off, experts_held=held)
    for l, (src, dst) in enumerate(zip(full.layers, out.layers)):
        s0 = full._local(off)
        for t_src, t_dst in ((src.w13, dst.w13), (src.s13, dst.s13), (src.w2, dst.w2), (src.s2, dst.s2)):
            t_dst.copy_(t_src[s0:s0 + held])
        if full.I_sh:
            # rows lo..hi of w1 / w3 (row tiles lo/128..), the same columns of w2
            w13 = untile_rows(src.sh_w13[:, :, 0]), untile_rows(src.sh_w13[:, :, 1])
            s13 = src.sh_s13[..., 0]                        # [I_sh/128][D/128][2] block scales
            w2 = untile_rows(src.sh_w2)                      # [D][I_sh]
            s2 = src.sh_s2[..., 0]                          # [D/128][I_sh/128]
            out.set_shared(l, torch.stack([w13[0][lo:hi], w13[1][lo:hi]]),
                           s13[lo // 128:hi // 128].permute(2, 0, 1), w2[:, lo:hi].contiguous(),
                           s2[:, lo // 128:hi // 128])
        if src.gate is not None:
            dst.gate.copy_(src.gate)
            if src.bias is not None:
                dst.bias.copy_(src.bias)
            else:
                dst.bias = None
        if src.tid2eid is not None:
            dst.tid2eid.copy_(src.tid2eid)
        dst.desc = None
    return out


@dataclass
class Dispatch:
    """Where one rank's tokens went: for every destination rank the local token
    indices sent there (ascending), and the row counts both ways."""
    tokens: list
    send_counts: list
    recv_counts: list


def dispatch_lists(topk_idx: torch.Tensor, experts_per_rank: int, world: int):
    """For every destination rank r: the tokens with at least one expert on r
    (ascending) and their ids localised to r (experts elsewhere -> -1). Ids
    outside [0, world * experts_per_rank) go nowhere (skipped)."""
    owner = torch.where(topk_idx >= 0, torch.div(topk_idx, experts_per_rank, rounding_mode="floor"),
                        torch.full_like(topk_idx, -1))
    toks, ids = [], []
    for r in range(world):
        m = owner == r
        t_r = m.any(1).nonzero().flatten()
        toks.append(t_r)
        ids.append(torch.where(m, topk_idx - r * experts_per_rank, torch.full_like(topk_idx, -1)).index_select(0, t_r))
    return toks, ids


class TokenShardedEP:
    """Expert parallelism for prefill-size calls with the tokens sharded over
    the ranks (the dispatch / combine scheme; the reference's own
    `_forward_ffn_ep`, engine.py:1575-1709, replicates the tokens instead).

    Rank r holds the routed experts [r E/n, (r+1) E/n) (shard_store or
    checkpoint.load_expert_store with rank/world) and the whole shared expert
    (shared="replicated"), and owns a shard of the tokens with their routing.
    `moe` sends each token's hidden row once to every other rank that holds
    one of its experts, with its ids localised to that rank and its weights
    (NCCL all-to-all of counts, rows, ids, weights); runs its own experts and
    the shared expert on its own tokens in one call and the routed FP4 kernels
    on the received rows (`hs_moe_ffn_fp4_partials`: un-rounded f32 sums);
    sends the f32 rows back, adds every rank's term per token in rank order
    (deterministic) and rounds as the single-GPU call does (bf16(bf16(routed)
    + bf16(shared)), `hs_moe_combine`). The host reads the counts (one
    synchronisation per call), as any all-to-all with data-dependent sizes
    does."""

    def __init__(self, rank: int, world: int, group=None,
                 all_to_all: Optional[Callable[[torch.Tensor, torch.Tensor, list, list], None]] = None):
        self.rank = rank
        self.world = world
        self.group = group
        if all_to_all is None:
            import torch.distributed as dist

            def _a2a(out, inp, out_splits, in_splits):
                dist.all_to_all_single(out, inp, out_splits, in_splits, group=group)
            all_to_all = _a2a
        self._a2a = all_to_all

    def dispatch(self, h: torch.Tensor, topk_idx: torch.Tensor, topk_w: torch.Tensor, experts_per_rank: int,
                 skip_self: bool = False):
        """-> (Dispatch, received rows [N, D], their local ids [N, K], weights [N, K]).
        skip_self: nothing is sent to this rank itself (its own experts run locally)."""
        toks, ids = dispatch_lists(topk_idx, experts_per_rank, self.world)
        if skip_self:
            toks[self.rank] = toks[self.rank][:0]
            ids[self.rank] = ids[self.rank][:0]
        send_counts = [int(t.numel()) for t in toks]
        order = torch.cat(toks)
        sc = torch.tensor(send_counts, dtype=torch.int64, device=h.device)
        rc = torch.empty_like(sc)
        self._a2a(rc, sc, [1] * self.world, [1] * self.world)
        recv_counts = [int(c) for c in rc.tolist()]
        n = sum(recv_counts)
        K = topk_idx.shape[1]
        h_recv = h.new_empty(n, h.shape[1])
        idx_recv = topk_idx.new_empty(n, K)
        w_recv = topk_w.new_empty(n, K)
        self._a2a(h_recv, h.index_select(0, order).contiguous(), recv_counts, send_counts)
        self._a2a(idx_recv, torch.cat(ids).contiguous(), recv_counts, send_counts)
        self._a2a(w_recv, topk_w.index_select(0, order).contiguous(), recv_counts, send_counts)
        return Dispatch(toks, send_counts, recv_counts), h_recv, idx_recv, w_recv

    def combine(self, d: Dispatch, y_recv: torch.Tensor, num_tokens: int,
                own: Optional[torch.Tensor] = None) -> torch.Tensor:
        """The received rows' f32 results back to their tokens: [T_local, D] f32,
        each token's rows added in rank order; `own` ([T_local, D] f32, zero
        where a token has no expert here) is this rank's term when its own
        experts ran locally (dispatch with skip_self)."""
        D = y_recv.shape[1]
        back = y_recv.new_empty(sum(d.send_counts), D)
        self._a2a(back, y_recv.contiguous(), d.send_counts, d.recv_counts)
        routed = torch.zeros(num_tokens, D, dtype=torch.float32, device=y_recv.device)
        off = 0
        for r, (t_r, c) in enumerate(zip(d.tokens, d.send_counts)):
            if r == self.rank and own is not None:
                routed += own
            elif c:
                routed.index_add_(0, t_r, back[off:off + c].float())
            off += c
        return routed

    def moe(self, store: HBMExpertStore, layer: int, h: torch.Tensor, topk_idx: torch.Tensor,
            topk_w: torch.Tensor, dup_mode: int = _lib.HS_DUP_LAST, use_shared: bool = True) -> torch.Tensor:
        """The MoE output [T_local, D] bf16 for this rank's tokens (normed rows h,
        global expert ids)."""
        T = h.shape[0]
        use_shared = use_shared and store.I_sh > 0
        d, h_r, idx_r, w_r = self.dispatch(h, topk_idx, topk_w, store.E_local, skip_self=True)
        # this rank's own experts and the shared expert on its own tokens: one call
        parts = None
        if T:
            own = localize(topk_idx, store.expert_offset, store.E_local)
            parts = ops.moe_ffn_partials(store.desc(layer), store.dims, h, own, topk_w, use_shared=use_shared,
                                         dup_mode=dup_mode)
        if h_r.shape[0]:
            y_r = ops.moe_ffn_partials(store.desc(layer), store.dims, h_r, idx_r, w_r, use_shared=False,
                                       dup_mode=dup_mode)[0]
        else:
            y_r = torch.empty(0, h.shape[1], dtype=torch.float32, device=h.device)
        routed = self.combine(d, y_r, T, own=parts[0] if parts is not None else None)
        if T == 0:  # no tokens of its own: the rank still took part in every exchange
            return h.new_empty(0, h.shape[1])
        parts[0].copy_(routed)
        return ops.moe_combine(parts, use_shared=use_shared)


def dispatch_plan(topk_idx: torch.Tensor, experts_per_rank: int, world: int, rank: int):
    """hs_ep_dispatch_plan on the device: (counts [world] int32, pos [T, world]
    int32, own_ids [T, K] int64) — rank q's list of this rank's tokens with an
    expert on q (ascending; empty for this rank), each token's place in it (or
    -1), and this rank's own ids localised (others -1). The same lists as
    dispatch_lists with skip_self."""
    dev = ops._check_cuda(topk_idx)
    topk_idx = topk_idx.to(torch.int64).contiguous()
    T, K = topk_idx.shape
    counts = torch.empty(world, dtype=torch.int32, device=dev)
    pos = torch.empty(T, world, dtype=torch.int32, device=dev)
    own = torch.empty(T, K, dtype=torch.int64, device=dev)
    ops._launch("hs_ep_dispatch_plan", topk_idx.data_ptr(), T, K, experts_per_rank, world, rank,
                counts.data_ptr(), pos.data_ptr(), own.data_ptr(), ops._stream(dev), extra=1 if T else 0)
    return counts, pos, own


class NcclTokenShardedEP:
    """TokenShardedEP as one C-ABI call (hs_ep_dispatch_combine): the plan,
    pack and combine are kernels, the exchanges NCCL send/recv on the caller's
    stream through a communicator of the library's own (created from a unique
    id that rank 0 makes and the torch process group hands round). Same
    arithmetic as TokenShardedEP.moe, so the outputs are identical; T_max
    (>= every rank's token count, the same on all ranks) sizes the workspace."""

    def __init__(self, rank: int, world: int, T_max: int, group=None, device: Optional[torch.device] = None):
        import torch.distributed as dist
        self.rank, self.world, self.T_max = rank, world, int(T_max)
        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        lib = _lib.load()
        uid = (ctypes.c_uint8 * _lib.HS_NCCL_UNIQUE_ID_BYTES)()
        if world > 1:
            if rank == 0:
                _lib.call("hs_ep_nccl_unique_id", ctypes.addressof(uid))
            obj = [bytes(uid)]
            dist.broadcast_object_list(obj, src=0, group=group)
            ctypes.memmove(uid, obj[0], len(obj[0]))
        elif world == 1:
            _lib.call("hs_ep_nccl_unique_id", ctypes.addressof(uid))
        self._comm = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            st = lib.hs_ep_nccl_comm_init(ctypes.addressof(uid), world, rank, ctypes.byref(self._comm))
        if st != 0:
            raise _lib.HsError("hs_ep_nccl_comm_init", st)

    def close(self) -> None:
        if self._comm:
            _lib.call("hs_ep_nccl_comm_destroy", self._comm)
            self._comm = ctypes.c_void_p()

    def moe(self, store: HBMExpertStore, layer: int, h: torch.Tensor, topk_idx: torch.Tensor,
            topk_w: torch.Tensor, dup_mode: int = _lib.HS_DUP_LAST, use_shared: bool = True,
            out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """The MoE output [T, D] bf16 of this rank's tokens (normed rows h,
        global expert ids), as TokenShardedEP.moe."""
        dev = self.device
        T, D = h.shape
        if T:
            ops._check_cuda(h, topk_idx, topk_w, out)
            if h.dtype != torch.bfloat16:
                raise TypeError("h must be bf16")
        topk_idx = topk_idx.to(torch.int64).contiguous()
        topk_w = topk_w.to(torch.float32).contiguous()
        K = topk_idx.shape[1] if topk_idx.dim() == 2 else 6
        _, Dd, I, I_sh = store.dims
        if out is None:
            out = torch.empty(T, D, dtype=torch.bfloat16, device=dev)
        lib = _lib.load()
        nb = lib.hs_ep_dispatch_combine_workspace_size(self.T_max, K, Dd, I, I_sh, self.world)
        ws = ops.workspace(dev, nb, "ep_nccl")
        ops._launch("hs_ep_dispatch_combine", self._comm, ctypes.addressof(store.desc(layer)), h.data_ptr(),
                    topk_idx.data_ptr(), topk_w.data_ptr(), T, self.T_max, K, int(use_shared and I_sh > 0),
                    int(dup_mode), out.data_ptr(), ws.data_ptr(), ws.numel(), ops.status_word(dev).data_ptr(),
                    ops._stream(dev), extra=4 if T else 1)
        return out
