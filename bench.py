"""Benchmark: MTP-verified decode tok/s (bs=1) on the 43-layer DeepSeek-V4-Flash
shaped model's MoE path, plus the FP4 MoE layer's HBM roofline fraction.

One step = one iteration of generate()'s MTP loop (engine.py:2809-2922): the
main T=1 forward through 43 MoE layers, the M=2 MTP draft, the fused T=3
verify forward through 43 MoE layers, lm_head and greedy acceptance. Weights
are random-init in the reference's formats (FP4 e2m1 + UE8M0 routed experts,
FP8 e4m3 shared experts, bf16 router/embed/head), all resident in HBM.
Attention/MHC are the reference's PyTorch path and are not part of this
build's step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line (rank 0). N > 1 (torchrun) runs one full replica per GPU
(the MoE path is replicated per sequence; value = all ranks' tokens / max
time over ranks).
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import threading
import sys
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "MTP-verified decode tok/s (bs=1); FP4 MoE layer HBM TB/s vs ~8 TB/s peak"
UNIT = "tok/s"


def _peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def _traffic_from_profile():
    """dram bytes per MoE FFN call from the committed ncu summary, if any."""
    f = REPO / "profiles" / "moe_layer_cfg0_t3.md"
    if not f.exists():
        return None
    m = re.search(r"traffic_bytes_per_call:\s*([0-9.eE+]+)", f.read_text())
    return float(m.group(1)) if m else None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []          # (monotonic time, csv line)
        self.t0 = self.t1 = None
        self.reader = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.monotonic(), line))

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "50", "-i", str(self.gpu)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.reader = threading.Thread(target=self._read, daemon=True)
            self.reader.start()
            deadline = time.monotonic() + 5.0
            while not self.lines and time.monotonic() < deadline:  # sampler is up before timing starts
                time.sleep(0.01)
        except Exception:
            self.proc = None
        self.t0 = time.monotonic()
        return self

    def __exit__(self, *a):
        self.t1 = time.monotonic()
        if self.proc is not None:
            time.sleep(0.06)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            if self.reader is not None:
                self.reader.join(timeout=2)

    def summary(self):
        if not self.lines:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        # samples taken while the timed region ran (widened to the nearest
        # samples around it when the region is shorter than the interval)
        inside = [l for t, l in self.lines if self.t0 <= t <= self.t1]
        if len(inside) < 3:
            inside = [l for t, l in self.lines if self.t0 - 0.1 <= t <= self.t1 + 0.1] or [self.lines[-1][1]]
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in inside:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------------------------------- CPU
def _reference_modules():
    """The reference's own modules from baseline/_ref (pip-installed there from
    its source tree, --no-deps), or None when that install is absent."""
    ref = REPO / "baseline" / "_ref"
    if not (ref / "home_seek").is_dir():
        return None
    if str(ref) not in sys.path:
        sys.path.insert(0, str(ref))
    try:
        from home_seek.fused_moe import FusedMoEFFN, SharedExpertFFN
        from home_seek.inference_engine.weight_loader import load_fp8_weight
        from home_seek.router import compute_expert_affinity_with_bias
    except Exception:  # noqa: BLE001 (an unusable install falls back to the port)
        return None
    return FusedMoEFFN, SharedExpertFFN, load_fp8_weight, compute_expert_affinity_with_bias


def cpu_sample(threads: int | None = None):
    """The reference's CPU path timed on a bounded sample: one T=3 verify MoE
    layer and one T=1 decode MoE layer at config-0 shapes (router, routed FP4
    experts, FP8 shared expert, bf16 add) and one lm_head GEMV, extrapolated to
    the 43-layer MTP iteration. Runs the reference's own code from baseline/_ref
    (compute_expert_affinity_with_bias, FusedMoEFFN(use_triton=False).forward,
    SharedExpertFFN(use_triton=False).forward + load_fp8_weight: kind
    "reference"), else the oracle's restatement of it (kind "port"). Weights
    come from the seeded generators of oracle/inputs.py, outside the timed
    region. Returns (tok_per_s, detail)."""
    import torch
    n = threads or os.cpu_count() or 1
    torch.set_num_threads(n)
    route, layer, h3, h1, head, kind = _cpu_setup()
    t0 = time.perf_counter()
    i3, w3 = route(h3)
    layer(h3, i3, w3)
    t1 = time.perf_counter()
    i1, w1 = route(h1)
    layer(h1, i1, w1)
    t2 = time.perf_counter()
    _ = torch.matmul(h1, head.t())
    t3 = time.perf_counter()
    t_verify, t_main, t_head = t1 - t0, t2 - t1, t3 - t2
    L = 43
    t_iter = L * (t_main + t_verify) + 2 * t_main + 4 * t_head
    return 1.0 / t_iter, {"t_layer_T3_s": t_verify, "t_layer_T1_s": t_main, "t_lm_head_s": t_head, "cores": n,
                          "t_iter_s": t_iter, "kind": kind}


_CPU_SETUP = None


def _cpu_setup():
    """Inputs and callables of the CPU sample, built once per process (the
    weight generation stays out of every timed step)."""
    global _CPU_SETUP
    if _CPU_SETUP is not None:
        return _CPU_SETUP
    import numpy as np
    import torch
    from oracle import inputs as I
    shape = I.CONFIG0
    gate, bias = I.router_weights(256, 4096, seed=1)
    w13, s13, w2, s2 = I.shared_fp8(4096, 2048, seed=2)
    load = I.make_loader(shape)
    h3, h1 = I.hidden(3, 4096, seed=0), I.hidden(1, 4096, seed=5)
    head = (torch.randn(129280, 4096, generator=torch.Generator().manual_seed(9)) * 0.02).to(torch.bfloat16)
    mods = _reference_modules()
    if mods is not None:
        FusedMoEFFN, SharedExpertFFN, load_fp8_weight, router = mods
        kind = "reference"
        t8 = lambda a: torch.from_numpy(np.ascontiguousarray(a)).view(torch.float8_e4m3fn)  # noqa: E731
        u8 = lambda a: torch.from_numpy(np.ascontiguousarray(a))  # noqa: E731
        sw = (load_fp8_weight(t8(w13[0]), u8(s13[0])), load_fp8_weight(t8(w13[1]), u8(s13[1])),
              load_fp8_weight(t8(w2), u8(s2)))
        ffn = FusedMoEFFN(num_experts=256, intermediate_size=2048, hidden_size=4096, use_triton=False)
        shf = SharedExpertFFN(hidden_size=4096, intermediate_size=2048, use_triton=False)

        def ref_load(layer, eid):
            a, sa, b, sb, c, sc = load(int(eid))
            i8 = lambda x: torch.from_numpy(x).view(torch.int8)  # noqa: E731
            e8 = lambda x: torch.from_numpy(x).view(torch.float8_e8m0fnu)  # noqa: E731
            return (i8(a), e8(sa), i8(b), e8(sb), i8(c), e8(sc))

        def route(h):
            return router(h, gate, bias, top_k=6, routed_scaling_factor=1.5)

        def layer(h, idx, w):  # engine.py:1480-1536: routed + shared, bf16 add
            return ffn.forward(h, idx, w, ref_load, 5) + shf.forward(h.unsqueeze(0), *sw, torch.bfloat16)[0]
    else:
        from oracle import moe as O
        kind = "port"
        sh = (w13, s13, w2, s2)

        def route(h):
            return O.router(h, gate, bias)

        def layer(h, idx, w):
            return O.moe_layer(h, idx, w, load, sh)
    i3, w3 = route(h3)
    i1, w1 = route(h1)
    for e in set(i3.flatten().tolist()) | set(i1.flatten().tolist()):
        load(int(e))  # generate the sample's weights outside the timed region
    _CPU_SETUP = (route, layer, h3, h1, head, kind)
    return _CPU_SETUP


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    for _ in range(args.warmup):
        cpu_sample()
    vals, det = [], None
    for _ in range(args.steps):
        v, det = cpu_sample()
        vals.append(v)
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * det["t_iter_s"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "config1 MTP iteration, MoE path, extrapolated from one T=3 + one T=1 MoE layer "
                               "and one lm_head GEMV per step", "model": "DeepSeek-V4-Flash-shape 43L",
                   "global_batch": 1, "seq_len": 3, "parallelism": "cpu"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": det["cores"], "kind": det["kind"],
                         "sample": "per step: 1 verify MoE layer (T=3) + 1 decode MoE layer (T=1) + 1 lm_head "
                                   "GEMV at config-0 shapes; x43 layers + 2 draft layers + 4 heads"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------------------- GPU
def _graph_time_per_call(enqueue, n_calls: int, replays: int = 5) -> float:
    """Capture `enqueue()` (n_calls MoE calls back to back, as in a layer loop)
    in one CUDA graph and time its replays with CUDA events: ms per call with
    no host launch cost in the timed region."""
    import torch
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        enqueue()  # warm-up: workspaces, descriptors, function attributes
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):  # the warm-up's workspaces, no captured fill
        enqueue()
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(replays):
        graph.replay()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / (replays * n_calls)
    del graph
    return ms


def moe_roofline(model, reps: int = 43):
    """Time the MoE half of a routed layer at T=3 (the verify shape) as the
    model step runs it, hs_moe_layer_fp4 (norm + routing + FFN + residual add),
    over distinct layers replayed from a CUDA graph. Algorithmic bytes per call:
    the touched experts' FP4 bytes + the FP8 shared expert + the router gate +
    activations (under expert parallelism: this rank's experts and shared rows,
    the partials call, the all-reduce and the combine)."""
    import torch
    from home_seek_b200 import ops
    s = model.shape
    dev = model.device
    g = torch.Generator(device=dev)
    g.manual_seed(123)
    L = s.num_layers
    calls = []
    for l in range(s.hash_layers, L):
        h = (torch.randn(3, s.hidden, generator=g, device=dev)).to(torch.bfloat16)
        lw = model.store.layers[l]
        idx, w = ops.router_topk(ops.rms_norm(h, model.ln_w[l]), lw.gate, lw.bias, s.top_k, s.routed_scaling)
        calls.append((l, h, idx, torch.empty_like(h)))
    st = model.store

    def layer_call(l, h, h_out):
        lw = st.layers[l]
        if model.ep is None:
            ops.moe_layer(st.desc(l), st.dims, h, model.ln_w[l], lw.gate, lw.bias, s.top_k, s.routed_scaling,
                          h_out=h_out)
            return
        if model.ep.peers is not None:
            ops.moe_layer_ep(st.desc(l), st.dims, h, model.ln_w[l], lw.gate, lw.bias, s.top_k, s.routed_scaling,
                             model.ep.peers.peers, num_experts=s.num_experts, expert_offset=st.expert_offset,
                             h_out=h_out)
            return
        buf = ops.moe_layer(st.desc(l), st.dims, h, model.ln_w[l], lw.gate, lw.bias, s.top_k, s.routed_scaling,
                            num_experts=s.num_experts, expert_offset=st.expert_offset, partials=True)[0]
        model.ep.all_reduce(buf)
        ops.moe_combine_add_rms_norm(buf, h, None, h_out=h_out)

    lo, hi = st.expert_offset, st.expert_offset + st.E_local
    uniq = [len({e for e in c[2].flatten().tolist() if lo <= e < hi}) for c in calls]
    per_call = _graph_time_per_call(lambda: [layer_call(l, h, ho) for (l, h, idx, ho) in calls], len(calls))
    # the main pass's shape too (T = 1), for the record
    calls1 = [(l, h[:1].contiguous(), idx, torch.empty_like(h[:1])) for (l, h, idx, ho) in calls]
    per_call_t1 = _graph_time_per_call(lambda: [layer_call(l, h, ho) for (l, h, idx, ho) in calls1], len(calls1))
    ms = [per_call] * len(calls)
    shared = 3 * st.I_sh * s.hidden + 3 * (st.I_sh // 128) * (s.hidden // 128)
    # h in, normed rows (x8) and activations, h out, idx/w, norm weight, router gate and bias
    act = 3 * s.hidden * 2 * 3 + 12 * 3 * 2 + s.hidden * 2 + s.num_experts * s.hidden * 2 + 512
    bytes_ = [u * s.bytes_per_expert + shared + act for u in uniq]
    gbs = [b / (m * 1e-3) / 1e9 for b, m in zip(bytes_, ms)]
    return {"avg_ms": statistics.mean(ms), "avg_bytes": statistics.mean(bytes_), "avg_gbs": statistics.mean(gbs),
            "avg_unique_experts": statistics.mean(uniq), "t1_ms": per_call_t1}


def run_moe_only(args):
    """MoE FFN microbenchmark for profiling: one (or a few) random-init layers
    of the config-0 shape, T tokens routed by the layer's own router,
    hs_moe_ffn_fp4 timed with CUDA events (prints one JSON line)."""
    import torch
    from home_seek_b200 import ops
    from home_seek_b200.expert_store import HBMExpertStore
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    store = HBMExpertStore(args.layers, 256, 4096, 2048, 2048, device=dev)
    store.fill_random(7)
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    calls = []
    for l in range(args.layers):
        for _ in range(max(1, args.reps // args.layers)):
            h = torch.randn(args.T, 4096, generator=g, device=dev).to(torch.bfloat16)
            idx, w = ops.router_topk(h, store.layers[l].gate, store.layers[l].bias, 6, 1.5)
            calls.append((l, h, idx, w))
    dup = 1 if args.T == 1 else 0

    nw = (1 + 0.02 * torch.randn(args.layers, 4096, generator=g, device=dev)).to(torch.bfloat16)
    h_out = torch.empty(args.T, 4096, dtype=torch.bfloat16, device=dev)

    def call(l, h, idx, w):
        lw = store.layers[l]
        if args.layer:  # norm + router + FFN + residual add (what the model step runs at T <= 8)
            return ops.moe_layer(store.desc(l), store.dims, h, nw[l], lw.gate, lw.bias, 6, 1.5, dup_mode=dup,
                                 h_out=h_out)[0]
        if args.fused:  # router folded into the call
            return ops.moe_route_ffn(store.desc(l), store.dims, h, lw.gate, lw.bias, 6, 1.5, dup_mode=dup)[0]
        return ops.moe_ffn(store.desc(l), store.dims, h, idx, w, dup_mode=dup)

    for c in calls[:3]:
        call(*c)
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in calls]
    for c, (a, b) in zip(calls, ev):
        a.record()
        call(*c)
        b.record()
    torch.cuda.synchronize()
    ms = [a.elapsed_time(b) for a, b in ev]
    # the same calls replayed from one CUDA graph (no host launch cost; with
    # layers > 1 consecutive calls stream different weights, as in the model)
    graph_ms = _graph_time_per_call(lambda: [call(*c) for c in calls], len(calls))
    uniq = [len(set(c[2].flatten().tolist())) for c in calls]
    shared = 3 * 2048 * 4096 + 3 * 16 * 32
    routed_in = args.fused or args.layer
    byts = [u * 13_369_344 + shared + args.T * 4096 * 4 + 24 * args.T + (256 * 4096 * 2 + 512 if routed_in else 0)
            + (args.T * 4096 * 2 + 4096 * 2 if args.layer else 0) for u in uniq]
    peak, kind = _peaks()
    gbs = statistics.mean(b / (m * 1e-3) / 1e9 for b, m in zip(byts, ms))
    graph_gbs = statistics.mean(byts) / (graph_ms * 1e-3) / 1e9
    print(json.dumps({"mode": "moe", "fused_router": bool(routed_in), "layer_call": bool(args.layer), "T": args.T,
                      "layers": args.layers,
                      "calls": len(calls),
                      "avg_us": 1000 * statistics.mean(ms), "min_us": 1000 * min(ms),
                      "graph_us": 1000 * graph_ms, "graph_frac": graph_gbs / peak,
                      "avg_unique_experts": statistics.mean(uniq), "avg_bytes": statistics.mean(byts),
                      "gbs": gbs, "frac": gbs / peak, "peak": peak, "peak_kind": kind}), flush=True)
    return 0


def run_moe_ep(args):
    """Config 3, the MoE half: an 8192-token prompt (T tokens, sharded T/n per
    rank) through `args.layers` layers of the config-0 shape (43 = the model)
    with token-sharded expert parallelism over the torchrun ranks: each rank
    holds its 256/n routed experts of every layer and the whole shared expert
    (random init), and every layer call dispatches rows to the experts' ranks
    and combines the results (--ep-impl torch: TokenShardedEP, torch.distributed
    all-to-all; c: hs_ep_dispatch_combine, one C-ABI call over NCCL). One pass
    calls every layer once; `reps` passes are timed (after one untimed pass).
    Prints the ms per layer call and per pass, the max over ranks of CUDA event
    time. Attention is not in this build's step."""
    import datetime
    import torch
    import torch.distributed as dist
    from home_seek_b200 import ops
    from home_seek_b200.ep import TokenShardedEP, expert_range
    from home_seek_b200.expert_store import HBMExpertStore
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        off, held = expert_range(256, rank, world)
        store = HBMExpertStore(args.layers, 256, 4096, 2048, 2048, device=dev, expert_offset=off, experts_held=held)
        store.fill_random(7 + rank)
        for l in range(args.layers):  # one router for the whole group
            g = torch.Generator(device=dev).manual_seed(100 + l)
            store.layers[l].gate.copy_((torch.randn(256, 4096, generator=g, device=dev) * 0.02).to(torch.bfloat16))
        Tl = args.T // world
        g = torch.Generator(device=dev).manual_seed(5 + rank)
        calls = []
        for l in range(args.layers):  # one pass: every layer once, its own rows and routing
            h = torch.randn(Tl, 4096, generator=g, device=dev).to(torch.bfloat16)
            idx, w = ops.router_topk(h, store.layers[l].gate, store.layers[l].bias, 6, 1.5)
            calls.append((l, h, idx, w))
        if args.ep_impl == "c":
            from home_seek_b200.ep import NcclTokenShardedEP
            ep = NcclTokenShardedEP(rank, world, Tl)
        else:
            ep = TokenShardedEP(rank, world)
        for c in calls:  # untimed pass
            ep.moe(store, c[0], c[1], c[2], c[3])
        torch.cuda.synchronize()
        dist.barrier()
        flag = torch.ones(1, device=dev)
        dist.all_reduce(flag)  # a common start on the device
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        passes = max(args.reps // max(args.layers, 1), 1)
        a.record()
        for _ in range(passes):
            for c in calls:
                ep.moe(store, c[0], c[1], c[2], c[3])
        b.record()
        torch.cuda.synchronize()
        ms = torch.tensor([a.elapsed_time(b) / passes], device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        if args.ep_impl == "c":
            ep.close()
        if rank == 0:
            print(json.dumps({"mode": "moe-ep", "T": Tl * world, "tokens_per_rank": Tl, "world": world,
                              "layers": args.layers, "passes": passes, "ms_per_pass": float(ms.item()),
                              "ms_per_layer": float(ms.item()) / args.layers,
                              "tokens_per_s": Tl * world / (float(ms.item()) * 1e-3),
                              "ep_impl": args.ep_impl,
                              "scheme": "token-sharded dispatch/combine (" + (
                                  "hs_ep_dispatch_combine: NCCL send/recv inside the C-ABI call)"
                                  if args.ep_impl == "c" else "torch.distributed all-to-all)")}), flush=True)
        return 0
    finally:
        dist.destroy_process_group()


def run_accept(args):
    """Config 4: batched speculative acceptance on [64, 3, 129280] bf16 logits
    (target and draft ~N(0, 3^2), t = 0.7, fp32 uniforms [64, 3] from seed 1),
    greedy (hs_accept_greedy, reads the target: 49.6 MB) and rejection sampling
    (hs_accept_rejection, algorithmic bytes 2 x 64 x 3 x V x 2 = 99.3 MB).
    Inputs are smaller than L2, so a 256 MB buffer is written between timed
    calls (outside the events). Prints one JSON line (not the driver's line)."""
    import torch
    from home_seek_b200 import ops
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, M, V, t = 64, 2, 129280, 0.7
    # the config-4 inputs (the same seeds and draws as the parity tests' fixture)
    g = torch.Generator().manual_seed(101)
    target = (torch.randn(B, M + 1, V, generator=g) * 3.0).to(torch.bfloat16)
    draft = (torch.randn(B, M + 1, V, generator=g) * 3.0).to(torch.bfloat16)
    u = torch.rand(B, M + 1, generator=torch.Generator().manual_seed(1))
    q = torch.softmax(draft[:, :M].float() / t, dim=-1)
    ids = torch.multinomial(q.reshape(B * M, V), 1, generator=torch.Generator().manual_seed(2)).reshape(B, M)
    target, draft, ids, u = target.to(dev), draft.to(dev), ids.to(dev), u.to(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    peak, kind = _peaks()

    def timed(fn, reps):
        for _ in range(3):
            fn()
        ms = []
        for _ in range(reps):
            flush.fill_(1)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            ms.append(a.elapsed_time(b))
        return statistics.median(ms)

    g_ms = timed(lambda: ops.accept_greedy(target, ids), args.reps)
    r_ms = timed(lambda: ops.accept_rejection(target, draft, ids, u, t), args.reps)
    g_bytes = B * (M + 1) * V * 2
    r_bytes = 2 * B * (M + 1) * V * 2 + B * (M + 1) * 4
    out = {"mode": "accept", "config": "config4: B=64, M=2, V=129280, t=0.7", "reps": args.reps,
           "l2": "256 MB written between timed calls",
           "greedy_us": 1000 * g_ms, "greedy_bytes": g_bytes, "greedy_gbs": g_bytes / (g_ms * 1e-3) / 1e9,
           "rejection_us": 1000 * r_ms, "rejection_bytes": r_bytes, "rejection_gbs": r_bytes / (r_ms * 1e-3) / 1e9,
           "peak_gbs": peak, "peak_kind": kind}
    out["greedy_frac"] = out["greedy_gbs"] / peak
    out["rejection_frac"] = out["rejection_gbs"] / peak
    print(json.dumps(out), flush=True)
    return 0


def run_head(args):
    """The lm_head GEMV with the fused argmax (hs_lm_head_argmax) at the model's
    shape: x [T, 4096] bf16, head [129280, 4096] bf16 (1.06 GB, larger than L2),
    T = args.T; against cuBLAS (torch.matmul) + torch.argmax, the path it
    replaces. Prints one JSON line (not the driver's line)."""
    import torch
    from home_seek_b200 import ops
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    V, D, T = 129280, 4096, args.T
    g = torch.Generator(device=dev).manual_seed(3)
    head = (torch.randn(V, D, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    x = torch.randn(T, D, generator=g, device=dev).to(torch.bfloat16)
    peak, kind = _peaks()

    def timed(fn, reps):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps

    ours = timed(lambda: ops.lm_head_argmax(x, head), args.reps)
    base = timed(lambda: (x @ head.t()).argmax(dim=-1), args.reps)
    nbytes = V * D * 2 + T * D * 2
    am = ops.lm_head_argmax(x, head)[0]
    same = bool(torch.equal(am, (x @ head.t()).argmax(dim=-1)))
    print(json.dumps({"mode": "head", "T": T, "reps": args.reps, "us": 1000 * ours, "bytes": nbytes,
                      "gbs": nbytes / (ours * 1e-3) / 1e9, "frac": nbytes / (ours * 1e-3) / 1e9 / peak,
                      "cublas_argmax_us": 1000 * base, "argmax_equal_to_cublas": same, "peak_gbs": peak,
                      "peak_kind": kind}), flush=True)
    return 0


def run_ours(args):
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    from home_seek_b200 import ops
    from home_seek_b200.mtp import ModelShape, MoEPathModel, MTPDecoder
    shape = ModelShape(num_layers=args.layers)
    ep = None
    if world > 1:
        # one decode stream over an expert-parallel group: every rank holds
        # 1/world of the routed experts and of the shared expert (ep.py)
        from home_seek_b200.ep import ExpertParallel, PeerExchange
        ep = ExpertParallel(rank, world)
        # decode-size layers exchange their partial sums through NVLink peer
        # memory inside the layer call (HS_EP_TRANSPORT=nccl: NCCL all-reduce)
        if os.environ.get("HS_EP_TRANSPORT", "p2p") == "p2p":
            ep.peers = PeerExchange(rank, world, shape.hidden)
    model = MoEPathModel(shape, device=dev, seed=0, ep=ep)
    # HS_EP_CHAIN=0: each peer-memory layer call completes its own exchange
    # (a combine kernel per call) instead of the next call's route kernel
    model.chain_ep = os.environ.get("HS_EP_CHAIN", "1") != "0"
    dec = MTPDecoder(model, max_tokens=(args.steps + args.warmup + 8) * (shape.num_draft + 2))
    dec.reset(token=1234)
    before = ops.launches
    dec.iteration()  # eager iteration: counts this library's kernels per iteration
    launches_per_iter = ops.launches - before
    dec.capture(warmup=1)
    dec.reset(token=1234)
    for _ in range(args.warmup):
        dec.replay()
    torch.cuda.synchronize()
    dec.count.zero_()
    dec.accepted.zero_()

    def device_barrier():
        """Every rank's next event fires when a one-element all-reduce has
        completed on the device, i.e. at the same moment on every rank (a host
        barrier alone leaves each rank's start at its own host wake-up time).
        The caller records its start event right after this, with no host
        synchronisation in between."""
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
            flag = torch.ones(1, device=dev)
            dist.all_reduce(flag)

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # the sampler is started (its first sample read) before the barrier: its
    # start-up time differs between ranks and must not end up inside a window
    with ClockSampler(local if not os.environ.get("CUDA_VISIBLE_DEVICES") else
                      int(os.environ["CUDA_VISIBLE_DEVICES"].split(",")[local])
                      if os.environ["CUDA_VISIBLE_DEVICES"].split(",")[local].isdigit() else local) as clk:
        device_barrier()
        start.record()
        for _ in range(args.steps):
            dec.replay()
        end.record()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = start.elapsed_time(end)
    tokens = int(dec.count.item())
    accepted = int(dec.accepted.item())
    t = torch.tensor([ms, float(tokens)], device=dev, dtype=torch.float64)
    if world > 1:  # one stream: every rank produced the same tokens; time = slowest rank
        tmax = t.clone()
        dist.all_reduce(tmax[:1], op=dist.ReduceOp.MAX)
        ms = float(tmax[0])
    tokens_all = float(tokens)
    value = tokens_all / (ms * 1e-3)

    # e2e through the public loop with host buffers: H2D of the step's input
    # token, D2H of the produced tokens and their count, every step
    host_in = torch.empty(1, dtype=torch.int64, pin_memory=True)
    host_tok = torch.empty(shape.num_draft + 2, dtype=torch.int64, pin_memory=True)
    host_cnt = torch.empty(1, dtype=torch.int64, pin_memory=True)
    host_in.fill_(4321)
    dec.count.zero_()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_tokens = 0
    device_barrier()
    e0.record()
    for _ in range(args.steps):
        dec.next_id.copy_(host_in, non_blocking=True)
        dec.replay()
        host_tok.copy_(dec.step_tokens, non_blocking=True)
        host_cnt.copy_(dec.step_count, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        c = int(host_cnt[0])
        e_tokens += c
        host_in[0] = host_tok[c - 1]
    e1.record()
    torch.cuda.synchronize()
    e_ms = e0.elapsed_time(e1)
    et = torch.tensor([e_ms, float(e_tokens)], device=dev, dtype=torch.float64)
    if world > 1:
        emax = et.clone()
        dist.all_reduce(emax[:1], op=dist.ReduceOp.MAX)
        e_ms = float(emax[0])
    e2e = {"value": float(e_tokens) / (e_ms * 1e-3), "unit": UNIT, "h2d_bytes_per_step": 8,
           "d2h_bytes_per_step": 8 * (shape.num_draft + 2) + 8}

    roof = moe_roofline(model)  # every rank (expert parallelism runs collectives)
    status = ops.check_status(dev)
    if world > 1:
        dev_graph = dec.graph
        dec.graph = None
        del dev_graph
        dist.barrier()
        if ep.peers is not None:
            ep.peers.close()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    peak, peak_kind = _peaks()
    achieved = roof["avg_gbs"]
    cpu_v, cpu_d = cpu_sample() if not args.no_cpu else (None, {"cores": 0})
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "config1: MTP decode iteration (main T=1 + M=2 draft + fused T=3 verify + greedy "
                               "accept) over the 43-layer MoE path, bs=1",
                   "model": "DeepSeek-V4-Flash-shape 43L+MTP, 256 FP4 experts top-6 + FP8 shared, random init",
                   "global_batch": 1, "seq_len": 3,
                   "parallelism": (f"expert-parallel x{world} (1/{world} of the routed and shared experts per GPU, "
                                   + ("f32 partials stored into every rank's buffer over NVLink by the down phase"
                                      + (", summed by the next layer call's route kernel)" if model.chain_ep
                                         else ", summed by a combine kernel)")
                                      if ep is not None and ep.peers is not None else
                                      "f32 partials all-reduced over NCCL)")) if world > 1 else "single GPU",
                   "attention": "not in this build's step (reference PyTorch path)",
                   "l2": "inputs larger than L2: ~16 GB of distinct expert weights streamed per iteration",
                   "acceptance_rate": accepted / max(1, args.steps * shape.num_draft), "status_word": status},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": _traffic_from_profile(),
                     "kernel": "hs_moe_layer_fp4 at T=3 (norm+route+plan, gate/up, down+residual launches)",
                     "peak_kind": peak_kind, "avg_ms": roof["avg_ms"], "t1_layer_ms": roof["t1_ms"],
                     "avg_bytes": roof["avg_bytes"],
                     "avg_unique_experts": roof["avg_unique_experts"]},
        "cpu_baseline": {"value": cpu_v, "unit": UNIT, "cores": cpu_d["cores"], "kind": cpu_d.get("kind", "port"),
                         "sample": "one T=3 + one T=1 MoE layer and one lm_head GEMV at config-0 shapes, "
                                   "extrapolated to 43 layers + 2 draft layers + 4 heads"},
        "e2e": e2e,
        "gpu_launches": launches_per_iter * args.steps,
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=43)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--mode", default="decode", choices=["decode", "moe", "moe-ep", "accept", "head"],
                    help="moe: MoE FFN microbenchmark only (profiling; not the driver's line); moe-ep: "
                         "prefill-size MoE with the tokens sharded over the torchrun ranks (TokenShardedEP); "
                         "accept: config-4 acceptance kernels; head: lm_head GEMV + fused argmax")
    ap.add_argument("--T", type=int, default=3, help="tokens per MoE call in --mode moe")
    ap.add_argument("--ep-impl", default="torch", choices=["torch", "c"],
                    help="--mode moe-ep: TokenShardedEP (torch) or hs_ep_dispatch_combine (c)")
    ap.add_argument("--reps", type=int, default=20, help="MoE calls timed in --mode moe")
    ap.add_argument("--fused", action="store_true", help="--mode moe: router folded into the call (T <= 8)")
    ap.add_argument("--layer", action="store_true",
                    help="--mode moe: the layer call, norm + router + FFN + residual add (T <= 8)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.mode == "moe":
        return run_moe_only(args)
    if args.mode == "moe-ep":
        return run_moe_ep(args)
    if args.mode == "accept":
        return run_accept(args)
    if args.mode == "head":
        return run_head(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
