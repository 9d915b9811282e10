"""MTP speculative decode (M=2 draft, fused T=3 verify, greedy acceptance) over
the MoE path of the DeepSeek-V4-Flash-shaped model, with every expert in HBM.

Reference: HomeSeekInferenceEngine.generate's decode loop
(inference_engine/engine.py:2809-2922), `_mtp_generate_draft`
(engine.py:2251-2336) and `_mtp_verify_batched` (engine.py:2431-2540).

What runs per layer here is the part of `_forward_layer` this build owns:
rms_norm -> router (or hash routing for layers < num_hash_layers) -> routed FP4
experts + FP8 shared expert -> residual add. At decode sizes (T <= 8) that is
one call, hs_moe_layer_fp4, of three launches: the norm runs in the routing
cluster and the residual add in the down phase's epilogue.
Attention and the MHC hyper-connections stay on the reference's PyTorch path
and are not part of this module; the layer body is therefore
h <- h + MoE(rms_norm(h)). The draft layer is the MTP block's projections
(e_proj(enorm(embed(tok))) + h_proj(hnorm(h))) followed by its own MoE.

Everything stays on the device between iterations: the accept/branch logic of
generate() (append n_acc drafts and the bonus token if n_acc > 0, else keep
the main-step token) is computed with tensor ops, so one iteration has no host
synchronisation and is captured as a single CUDA graph.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import TYPE_CHECKING, Optional

import torch

from . import ops
from ._lib import HS_DUP_LAST, HS_DUP_SUM
from .expert_store import HBMExpertStore

if TYPE_CHECKING:
    from .ep import ExpertParallel


@dataclass
class ModelShape:
    num_layers: int = 43
    num_experts: int = 256
    hidden: int = 4096
    inter: int = 2048
    shared_inter: int = 2048
    vocab: int = 129280
    top_k: int = 6
    hash_layers: int = 3
    routed_scaling: float = 1.5
    num_draft: int = 2

    @property
    def bytes_per_expert(self) -> int:
        return 3 * self.inter * self.hidden // 2 + 3 * self.inter * self.hidden // 32


class MoEPathModel:
    """Random-init weights of the full model shape on one GPU (layers 0..L-1 plus
    the MTP layer at index L in the same expert store)."""

    def __init__(self, shape: ModelShape, device: str | torch.device = "cuda", seed: int = 0,
                 ep: Optional["ExpertParallel"] = None, weights: Optional[dict] = None):
        """ep: expert parallelism (ep.py): this rank holds its block of routed
        experts and its rows of the shared expert; everything else (router,
        embeddings, norms, lm_head) is replicated and identical on every rank.
        weights: explicit tensors in the reference's formats instead of a
        random init (see load_weights)."""
        self.shape = s = shape
        self.device = dev = torch.device(device)
        self.ep = ep
        # under peer-memory expert parallelism, forward chains its layer calls
        # (each call's exchange completed by the next call's route kernel)
        self.chain_ep = True
        off, held, sh = 0, None, s.shared_inter
        if ep is not None:
            from .ep import expert_range, shared_slice
            off, held = expert_range(s.num_experts, ep.rank, ep.world)
            lo, hi = shared_slice(s.shared_inter, ep.rank, ep.world)
            sh = hi - lo
        self.store = HBMExpertStore(s.num_layers + 1, s.num_experts, s.hidden, s.inter, sh, device=dev,
                                    with_router=True, hash_layers=s.hash_layers, vocab_size=s.vocab,
                                    top_k=s.top_k, expert_offset=off, experts_held=held)
        if weights is not None:
            self.load_weights(weights)
        else:
            self.store.fill_random(seed)
            g = torch.Generator(device=dev)
            g.manual_seed(seed + 17)

            def randn(*shp, std):
                return (torch.randn(*shp, generator=g, device=dev) * std).to(torch.bfloat16)

            self.embed = randn(s.vocab, s.hidden, std=0.02)
            self.lm_head = randn(s.vocab, s.hidden, std=0.02)
            self.norm_w = (1.0 + randn(s.hidden, std=0.02).float()).to(torch.bfloat16)
            self.ln_w = (1.0 + randn(s.num_layers + 1, s.hidden, std=0.02).float()).to(torch.bfloat16)
            self.e_proj = randn(s.hidden, s.hidden, std=0.02)
            self.h_proj = randn(s.hidden, s.hidden, std=0.02)
            self.enorm_w = (1.0 + randn(s.hidden, std=0.02).float()).to(torch.bfloat16)
            self.hnorm_w = (1.0 + randn(s.hidden, std=0.02).float()).to(torch.bfloat16)
            self.mtp_norm_w = (1.0 + randn(s.hidden, std=0.02).float()).to(torch.bfloat16)
        for layer in range(s.num_layers + 1):
            self.store.desc(layer)  # encode TMA descriptors once

    def load_weights(self, w: dict) -> None:
        """Fill the model from tensors in the reference's formats: w["experts"][l]
        (eid -> FP4 6-tuple), w["shared"][l] (FP8 (w13, s13, w2, s2)) for the
        main layers, w["gate"][l], w["bias"][l], w["tid2eid"][l] for the hash
        layers, and the dense bf16 tensors embed, lm_head, norm_w, ln_w
        [L + 1, D], e_proj, h_proj, enorm_w, hnorm_w, mtp_norm_w. Layer L is the
        MTP layer (no shared expert is used there)."""
        s = self.shape
        dev = self.device
        st = self.store
        lo, hi = st.expert_offset, st.expert_offset + st.E_local
        for layer in range(s.num_layers + 1):
            load = w["experts"][layer]
            for e in range(lo, hi):
                st.set_expert(layer, e, *load(e))
            if layer < s.num_layers and st.I_sh:
                st.set_shared(layer, *w["shared"][layer])
            st.set_router(layer, w["gate"][layer].to(dev), w["bias"][layer].to(dev))
            tid = w["tid2eid"].get(layer)
            if tid is not None and st.layers[layer].tid2eid is not None:
                st.layers[layer].tid2eid.copy_(tid.to(dev))
        bf = lambda t: t.to(device=dev, dtype=torch.bfloat16).contiguous()  # noqa: E731
        self.embed, self.lm_head = bf(w["embed"]), bf(w["lm_head"])
        self.norm_w, self.ln_w = bf(w["norm_w"]), bf(w["ln_w"])
        self.e_proj, self.h_proj = bf(w["e_proj"]), bf(w["h_proj"])
        self.enorm_w, self.hnorm_w, self.mtp_norm_w = bf(w["enorm_w"]), bf(w["hnorm_w"]), bf(w["mtp_norm_w"])

    # --- one MoE layer (the part of _forward_layer / _forward_ffn this build owns)
    def moe(self, x: torch.Tensor, layer: int, ids: torch.Tensor) -> torch.Tensor:
        s = self.shape
        st = self.store
        lw = st.layers[layer]
        # T=1 decode follows the reference's M=1 path (duplicates summed,
        # engine.py:1388-1393); T>1 follows _forward_legacy (last weight wins)
        dup = HS_DUP_SUM if x.shape[0] == 1 else HS_DUP_LAST
        if layer < s.hash_layers and lw.tid2eid is not None:
            idx, w = ops.hash_route(ids, lw.tid2eid, s.top_k)
        elif x.shape[0] <= 8:
            # decode sizes: router + FFN in one call (routing and plan in one cluster)
            if self.ep is not None:  # f32 partial sums, summed over the ranks
                buf, _, _ = ops.moe_route_ffn(st.desc(layer), st.dims, x, lw.gate, lw.bias, s.top_k,
                                              s.routed_scaling, dup_mode=dup, expert_offset=st.expert_offset,
                                              partials=True)
                self.ep.all_reduce(buf)
                return buf
            out, _, _ = ops.moe_route_ffn(st.desc(layer), st.dims, x, lw.gate, lw.bias, s.top_k, s.routed_scaling,
                                          dup_mode=dup)
            return out
        else:
            idx, w = ops.router_topk(x, lw.gate, lw.bias, s.top_k, s.routed_scaling)
        if self.ep is not None:  # f32 partial sums, already summed over the ranks
            return self.ep.partials(st, layer, x, idx, w, dup)
        return ops.moe_ffn(st.desc(layer), st.dims, x, idx, w, use_shared=True, dup_mode=dup)

    def _layer_args(self, h: torch.Tensor, layer: int, ids: torch.Tensor):
        s = self.shape
        st = self.store
        lw = st.layers[layer]
        dup = HS_DUP_SUM if h.shape[0] == 1 else HS_DUP_LAST
        hashed = layer < s.hash_layers and lw.tid2eid is not None
        kw = {"ids": ids, "tid2eid": lw.tid2eid} if hashed else {}
        # the MTP block runs the routed experts only (engine.py:2087-2097)
        kw["use_shared"] = layer < s.num_layers
        gate, bias = (None, None) if hashed else (lw.gate, lw.bias)
        args = (st.desc(layer), st.dims, h, self.ln_w[layer], gate, bias, s.top_k, s.routed_scaling)
        return args, dup, kw

    def layer_chained(self, h: torch.Tensor, layer: int, ids: torch.Tensor, prev_shared: Optional[bool]) -> bool:
        """The layer call in the chained peer-memory form: h first receives the
        previous chained call's output (prev_shared: its use_shared, None when
        nothing is pending), then this layer's output is left pending. Returns
        this call's use_shared, for the next call or ep_combine_pending."""
        args, dup, kw = self._layer_args(h, layer, ids)
        ops.moe_layer_ep_chained(*args, self.ep.peers.peers, prev_pending=prev_shared is not None,
                                 prev_use_shared=bool(prev_shared), dup_mode=dup,
                                 num_experts=self.shape.num_experts, expert_offset=self.store.expert_offset, **kw)
        return bool(kw["use_shared"])

    def layer(self, h: torch.Tensor, layer: int, ids: torch.Tensor,
              h_out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """h + MoE(rms_norm(h, ln_w[layer])) for T <= 8 rows (into h_out when
        given, which may be h): one hs_moe_layer_fp4 call; under expert
        parallelism either hs_moe_layer_fp4_ep (the exchange through NVLink
        peer memory inside the call) or the partials form, an NCCL all-reduce
        and the combine + add."""
        s = self.shape
        st = self.store
        args, dup, kw = self._layer_args(h, layer, ids)
        if self.ep is not None and self.ep.peers is not None:  # exchange through peer memory in the call
            return ops.moe_layer_ep(*args, self.ep.peers.peers, dup_mode=dup, num_experts=s.num_experts,
                                    expert_offset=st.expert_offset, h_out=h_out, **kw)[0]
        if self.ep is not None:
            buf, _, _ = ops.moe_layer(*args, dup_mode=dup, num_experts=s.num_experts,
                                      expert_offset=st.expert_offset, partials=True, **kw)
            self.ep.all_reduce(buf)
            return ops.moe_combine_add_rms_norm(buf, h, None, h_out=h_out)[0]
        return ops.moe_layer(*args, dup_mode=dup, num_experts=s.num_experts, h_out=h_out, **kw)[0]

    def _add_norm(self, h: torch.Tensor, y: torch.Tensor, w: torch.Tensor, in_place: bool,
                  x_out: Optional[torch.Tensor] = None):
        """Residual add of the MoE output y (bf16, or [2, T, D] f32 partials under
        expert parallelism) fused with the next norm (h updated in place when
        in_place; the norm written into x_out when given)."""
        kw = {"h_out": h} if in_place else {}
        if x_out is not None:
            kw["x_out"] = x_out
        if self.ep is not None:
            return ops.moe_combine_add_rms_norm(y, h, w, **kw)
        return ops.add_rms_norm(h, y, w, **kw)

    def forward(self, ids: torch.Tensor):
        """All layers for tokens `ids`: returns (h, x) with h the residual stream
        after the last layer and x = rms_norm(h, final norm). At T <= 8 each
        layer is one hs_moe_layer_fp4 call updating h in place (under
        peer-memory expert parallelism chained: each call's exchange completed
        by the next call); above, each layer's residual add is fused with the
        next layer's input norm."""
        L = self.shape.num_layers
        h = self.embed[ids]
        if ids.shape[0] <= 8 and self.chain_ep and self.ep is not None and self.ep.peers is not None:
            pending = None
            for layer in range(L):
                pending = self.layer_chained(h, layer, ids, pending)
            if pending is not None:
                ops.ep_combine_pending(self.ep.peers.peers, h, use_shared=pending)
            return h, ops.rms_norm(h, self.norm_w)
        if ids.shape[0] <= 8:
            for layer in range(L):
                self.layer(h, layer, ids, h_out=h)
            return h, ops.rms_norm(h, self.norm_w)
        x = ops.rms_norm(h, self.ln_w[0])
        for layer in range(L):
            y = self.moe(x, layer, ids)
            w_next = self.ln_w[layer + 1] if layer + 1 < L else self.norm_w
            h, x = self._add_norm(h, y, w_next, in_place=True, x_out=x)
        return h, x

    def logits(self, x_normed: torch.Tensor) -> torch.Tensor:
        """lm_head over rows that already carry the final norm (forward's x):
        the bf16 logits, written out (the sampling paths need them)."""
        return ops.lm_head_argmax(x_normed, self.lm_head, want_logits=True)[3]

    def greedy(self, x_normed: torch.Tensor, draft_ids: Optional[torch.Tensor] = None):
        """lm_head + argmax in one kernel (the logits never leave the chip):
        returns (argmax [T], n_accept [1], next_token [1]); with draft_ids the
        verify pass's greedy acceptance (engine.py:2485-2497). Under expert
        parallelism over peer memory the vocabulary is split over the group
        as well (every rank streams 1/n of the head; the same results)."""
        if self.ep is not None and self.ep.peers is not None:
            return ops.lm_head_argmax_ep(x_normed, self.lm_head, self.ep.peers.peers, draft_ids=draft_ids)
        return ops.lm_head_argmax(x_normed, self.lm_head, draft_ids=draft_ids)

    def draft(self, h_last: torch.Tensor, tok: torch.Tensor) -> torch.Tensor:
        """_mtp_generate_draft at t=0 (engine.py:2251-2336) on the MoE path: M steps."""
        s = self.shape
        L = s.num_layers
        prev = h_last
        out = []
        t = tok
        for _ in range(s.num_draft):
            e = ops.rms_norm(self.embed[t], self.enorm_w) @ self.e_proj.t()
            hc = ops.rms_norm(prev, self.hnorm_w) @ self.h_proj.t() + e
            hm = self.layer(hc, L, t)
            xm = ops.rms_norm(hm, self.mtp_norm_w)
            t = self.greedy(xm)[2]
            out.append(t)
            prev = hm
        return torch.cat(out)


class MTPDecoder:
    """Device-resident MTP decode loop. state: next_id [1], out buffer of tokens."""

    def __init__(self, model: MoEPathModel, max_tokens: int = 4096):
        self.m = model
        dev = model.device
        M = model.shape.num_draft
        self.next_id = torch.zeros(1, dtype=torch.int64, device=dev)
        self.tokens = torch.zeros(max_tokens + M + 2, dtype=torch.int64, device=dev)
        self.count = torch.zeros(1, dtype=torch.int64, device=dev)
        self.step_tokens = torch.zeros(M + 2, dtype=torch.int64, device=dev)
        self.step_count = torch.zeros(1, dtype=torch.int64, device=dev)
        self.accepted = torch.zeros(1, dtype=torch.int64, device=dev)
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self._ar = torch.arange(M + 2, device=dev)

    def iteration(self) -> None:
        """One generate() iteration: main T=1 step, M-token draft, fused T=1+M verify, accept."""
        m = self.m
        M = m.shape.num_draft
        h, x = m.forward(self.next_id)                                # main step, T=1
        main_pred = m.greedy(x)[2]
        d = m.draft(h, main_pred)                                     # M drafts
        ids = torch.cat([main_pred, d])                               # combined_ids
        _, xv = m.forward(ids)                                        # fused verify, T=1+M
        _, n_acc, bonus = m.greedy(xv, draft_ids=d)                   # lm_head + greedy acceptance
        n = n_acc.to(torch.int64)
        # tokens of this iteration: main_pred, then d[:n], then bonus if n > 0
        cand = torch.cat([main_pred, d, bonus])                       # [M + 2]
        take = torch.where(self._ar <= n, cand, torch.zeros_like(cand))
        # bonus sits right after the n accepted drafts
        take = torch.where(self._ar == n + 1, bonus.expand(M + 2), take)
        cnt = torch.where(n > 0, n + 2, torch.ones_like(n))
        self.step_tokens.copy_(take)
        self.step_count.copy_(cnt)
        pos = self.count + self._ar
        keep = self._ar < cnt
        self.tokens.index_put_((pos.clamp(max=self.tokens.numel() - 1),), torch.where(keep, take, self.tokens[
            pos.clamp(max=self.tokens.numel() - 1)]))
        self.count.add_(cnt)
        self.accepted.add_(n)
        self.next_id.copy_(torch.where(n > 0, bonus, main_pred))

    def capture(self, warmup: int = 1) -> None:
        s = torch.cuda.Stream(self.next_id.device)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(warmup):
                self.iteration()
        torch.cuda.current_stream().wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        # capture on the warm-up stream: the per-stream workspaces it allocated
        # (zero-filled once) are reused, so no fill is captured into the graph
        with torch.cuda.graph(self.graph, stream=s):
            self.iteration()

    def replay(self) -> None:
        if self.graph is None:
            self.iteration()
        else:
            self.graph.replay()

    def reset(self, token: int) -> None:
        self.next_id.fill_(token)
        self.count.zero_()
        self.accepted.zero_()


class MTPEngine:
    """The reference engine's MTP methods over the MoE path, with the
    reference's names, arguments and returns (HomeSeekInferenceEngine,
    inference_engine/engine.py): `_mtp_generate_draft` (engine.py:2251-2336),
    `_mtp_verify_batched` (engine.py:2431-2540) and the main decode step of
    generate() (engine.py:2811-2853). Hidden states carry hc_mult = 1 (the
    MHC streams are on the attention path this build does not own): [1, 1, 1,
    D] or [1, D].

    Temperature: the reference draws draft and bonus tokens with
    torch.multinomial; here they are drawn by inverse CDF from a supplied
    uniform (ops.sample), so a run is reproducible given the uniforms (drawn
    with torch.rand on the device when none are given). Verification compares
    argmaxes as the reference does at any temperature;
    `_mtp_verify_rejection` is the speculative-sampling acceptance (accept d_i
    iff u_i < p_i(d_i) / q_i(d_i)), which the reference does not have.
    """

    def __init__(self, model: MoEPathModel):
        self.model = model
        self._global_pos = 0
        self._mtp_draft_logits: Optional[torch.Tensor] = None  # [M, V] of the last sampled draft

    def _ids(self, t: torch.Tensor) -> torch.Tensor:
        return t.reshape(-1).to(device=self.model.device, dtype=torch.int64)

    def main_step(self, next_id: torch.Tensor, temperature: float = 0.0, uniform: Optional[torch.Tensor] = None):
        """One decode step of generate() (engine.py:2811-2853): forward the token,
        final norm, lm_head, argmax (t = 0) or a sample (t > 0). Returns
        (last hidden [1, 1, 1, D], next token [1, 1])."""
        m = self.model
        h, x = m.forward(self._ids(next_id)[-1:])
        if temperature > 0:
            u = uniform if uniform is not None else torch.rand(1, device=m.device)
            tok = ops.sample(m.logits(x), temperature, u)
        else:
            tok = m.greedy(x)[2]
        return h.view(1, 1, 1, -1), tok.view(1, 1)

    def _mtp_generate_draft(self, last_hidden: torch.Tensor, num_draft: int = 3, temperature: float = 0.6,
                            last_token_id: Optional[torch.Tensor] = None, uniform: Optional[torch.Tensor] = None):
        """engine.py:2251-2336: num_draft autoregressive MTP steps from the main
        model's last hidden state. Step i: e = e_proj(enorm(embed(tok_i))) (a
        zero embedding when step 0 has no last token), h = h_proj(hnorm(prev))
        + e, the MTP block (its routed experts, engine.py:2036-2107), its head
        norm, lm_head, then argmax (t = 0) or a sample with uniform[i] (t > 0).
        Returns (draft_ids [1, num_draft] int64, num_draft), or (None, 0)."""
        m = self.model
        if num_draft < 1:
            return None, 0
        s = m.shape
        prev = last_hidden.reshape(-1, s.hidden)[-1:].to(torch.bfloat16).contiguous()
        dev = prev.device
        if temperature > 0 and uniform is None:
            uniform = torch.rand(num_draft, device=dev)
        toks, rows = [], []
        for step in range(num_draft):
            if step == 0 and last_token_id is not None:
                tok = self._ids(last_token_id)[-1:]
            elif step > 0:
                tok = toks[-1]
            else:
                tok = None
            e_in = m.embed[tok] if tok is not None else torch.zeros(1, s.hidden, dtype=torch.bfloat16, device=dev)
            e = ops.rms_norm(e_in, m.enorm_w) @ m.e_proj.t()
            hc = ops.rms_norm(prev, m.hnorm_w) @ m.h_proj.t() + e
            prev = m.layer(hc, s.num_layers, tok if tok is not None else torch.zeros(1, dtype=torch.int64, device=dev))
            xm = ops.rms_norm(prev, m.mtp_norm_w)
            if temperature > 0:
                lg = m.logits(xm)
                rows.append(lg)
                t = ops.sample(lg, temperature, uniform.reshape(-1)[step:step + 1])
            else:
                t = m.greedy(xm)[2]
            toks.append(t)
        self._mtp_draft_logits = torch.cat(rows) if rows else None
        return torch.cat(toks).view(1, num_draft), num_draft

    def _verify_forward(self, draft_ids: torch.Tensor, main_pred_id: Optional[torch.Tensor]):
        ids = self._ids(draft_ids)
        if main_pred_id is not None:
            ids = torch.cat([self._ids(main_pred_id)[-1:], ids])
        return ids, self.model.forward(ids)[1]

    def _mtp_verify_batched(self, draft_ids: torch.Tensor, temperature: float = 0.6,
                            main_pred_id: Optional[torch.Tensor] = None):
        """engine.py:2431-2540: one fused forward over [main_pred, drafts]; logits[i]
        predicts the token after combined[i]; accept combined[i + 1] while
        argmax(logits[i]) equals it. Returns (n_accept: int, bonus_logits
        [1, V] bf16 = logits[n_accept]), or (0, None) with no drafts. The
        decision is hs_lm_head_argmax's fused greedy loop; reading n_accept is
        the one host synchronisation the reference's int return implies."""
        if not isinstance(draft_ids, torch.Tensor) or draft_ids.shape[-1] == 0:
            return 0, None
        m = self.model
        ids, xv = self._verify_forward(draft_ids, main_pred_id)
        _, n, _, lg = ops.lm_head_argmax(xv, m.lm_head, draft_ids=ids[1:], want_logits=True)
        n_accept = int(n)
        pos = self._global_pos
        self._global_pos = pos + n_accept  # engine.py:2518
        return n_accept, lg[n_accept:n_accept + 1]

    def _mtp_verify_rejection(self, draft_ids: torch.Tensor, temperature: float, main_pred_id: torch.Tensor,
                              uniform: Optional[torch.Tensor] = None):
        """Speculative-sampling acceptance of the last sampled draft (Leviathan et
        al. 2023): target p_i = softmax(verify logits[i] / t), draft q_i =
        softmax(draft logits[i] / t); accept d_i iff u_i < p_i(d_i) / q_i(d_i);
        at the first rejection sample from normalise(max(0, p_i - q_i)), else
        the bonus from p_M, with u_M. Returns (n_accept: int, next token [1, 1])."""
        m = self.model
        q = self._mtp_draft_logits
        M = self._ids(draft_ids).numel()
        if q is None or q.shape[0] != M:
            raise ValueError("_mtp_verify_rejection needs the draft logits of a sampled draft (temperature > 0)")
        _, xv = self._verify_forward(draft_ids, main_pred_id)
        p = m.logits(xv)
        u = uniform if uniform is not None else torch.rand(M + 1, device=m.device)
        n, nxt = ops.accept_rejection(p.view(1, M + 1, -1), q.view(1, M, -1), self._ids(draft_ids).view(1, M),
                                      u.view(1, M + 1), temperature)
        n_accept = int(n[0])
        self._global_pos += n_accept
        return n_accept, nxt.view(1, 1)

    def bonus_token(self, bonus_logits: torch.Tensor, temperature: float = 0.0,
                    uniform: Optional[torch.Tensor] = None) -> torch.Tensor:
        """generate()'s next token from the verify's bonus logits (engine.py:
        2905-2913): argmax at t = 0, a sample from softmax(bonus / t) above."""
        if temperature > 0:
            u = uniform if uniform is not None else torch.rand(1, device=bonus_logits.device)
            return ops.sample(bonus_logits.reshape(1, -1).contiguous(), temperature, u).view(1, 1)
        return bonus_logits.reshape(1, -1).argmax(dim=-1, keepdim=True)
