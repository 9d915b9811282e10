"""Phase timeline of the decode layer call, from the tracing build.

`python -m home_seek_b200.build --trace` compiles libhs_ext_trace.so: the same
kernels, with every phase boundary of the token-mode layer call
(hs_moe_layer_fp4: route kernel, gate/up, down, and under expert parallelism
the peer-exchange combine) stamped with %globaltimer into a device array
(csrc/hs_trace.cuh). `HS_TRACE=1 python -m home_seek_b200.trace --T 1 3 8`
replays `layers` layer calls of the config-0 shape from one CUDA graph and
prints, per phase, the min / median / max over the CTAs of the time after the
route kernel left its wait for the previous call (median over the calls).
The stamps cost a few percent; time the normal build with bench.py.
"""
from __future__ import annotations

import argparse
import ctypes
import os
import statistics
from typing import Optional

import torch

# (name, kernel, event, CTAs or None = all) of every printed phase
PHASES = [
    ("route entry", 0, 0, "route"), ("route rows in", 0, 2, "route"), ("route norm done", 0, 3, "route"),
    ("route keys gathered", 0, 4, "route"), ("route others done", 0, 5, "others"),
    ("route CTA 0 top-k done", 0, 6, "rank0"), ("route CTA 0 plan counted", 0, 7, "rank0"),
    ("route CTA 0 done", 0, 5, "rank0"),
    ("gate/up wait over", 1, 1, None), ("gate/up first TMA", 1, 2, None), ("gate/up first MMA", 1, 3, None),
    ("gate/up first acc", 1, 6, None), ("gate/up last copy issued", 3, 4, None), ("gate/up last MMA", 1, 4, None),
    ("gate/up MMA warp done", 3, 3, None), ("gate/up last ticket", 3, 0, None), ("gate/up peer sums", 1, 7, None),
    ("gate/up last acc", 3, 1, None), ("gate/up epilogue done", 3, 2, None), ("gate/up done", 1, 5, None), ("down entry", 2, 0, None), ("down first weights", 2, 2, None),
    ("down started", 2, 1, None), ("down first MMA", 2, 3, None), ("down last MMA", 2, 4, None),
    ("down cluster sync", 2, 7, None), ("down done", 2, 5, None),
    ("combine started", 4, 1, None), ("combine rows in", 4, 2, None), ("combine done", 4, 3, None),
]
SLOTS, KERNELS, CTAS, EVENTS = 32, 5, 296, 8


class _View:
    def __init__(self, ptr: int, n: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False), "version": 3}


def buffers(device: torch.device):
    """(stamps [32, 5, 296, 8] int64, calls [1] int32) of the loaded tracing library."""
    from . import _lib
    lib = _lib.load()
    p0, p1 = lib.hs_trace_buffer(0), lib.hs_trace_buffer(1)
    if not p0 or not p1:
        raise RuntimeError("the loaded library is not the tracing build: set HS_TRACE=1 and build with --trace")
    stamps = torch.as_tensor(_View(p0, SLOTS * KERNELS * CTAS * EVENTS, "<i8"), device=device)
    calls = torch.as_tensor(_View(p1, 1, "<i4"), device=device)
    return stamps.view(SLOTS, KERNELS, CTAS, EVENTS), calls


def phases(X: torch.Tensor, ncalls: int) -> dict:
    """Per phase: (min, median, max) over CTAs in us after the route kernel's
    wait, the median over calls 1 .. ncalls-2 (the first and last excluded)."""
    out = {}
    for name, k, e, which in PHASES:
        per_call = []
        for i in range(1, max(ncalls - 1, 1)):
            r0 = int(X[i, 0, 0, 1])
            if r0 == 0:
                continue
            if which == "rank0":
                cs = [0]
            elif which == "others":
                cs = range(1, 16)
            elif which == "route":
                cs = range(16)
            else:
                cs = range(CTAS)
            v = [(int(X[i, k, c, e]) - r0) / 1000 for c in cs if int(X[i, k, c, e]) > 0]
            if v:
                per_call.append((min(v), statistics.median(v), max(v)))
        if per_call:
            out[name] = tuple(statistics.median(p[j] for p in per_call) for j in range(3))
    if ncalls > 2:
        nxt = [(int(X[i + 1, 0, 0, 1]) - int(X[i, 0, 0, 1])) / 1000 for i in range(1, ncalls - 1)]
        out["next call's route wait over"] = (statistics.median(nxt),) * 3
    return out


def run(T_values, layers: int = 8, device: Optional[torch.device] = None) -> dict:
    from . import ops
    from .expert_store import HBMExpertStore
    dev = device or torch.device("cuda", torch.cuda.current_device())
    stamps, calls = buffers(dev)
    store = HBMExpertStore(layers, 256, 4096, 2048, 2048, device=dev)
    store.fill_random(7)
    g = torch.Generator(device=dev).manual_seed(5)
    nw = (1 + 0.02 * torch.randn(layers, 4096, generator=g, device=dev)).to(torch.bfloat16)
    res = {}
    for T in T_values:
        hs = [torch.randn(T, 4096, generator=g, device=dev).to(torch.bfloat16) for _ in range(layers)]
        h_out = torch.empty(T, 4096, dtype=torch.bfloat16, device=dev)

        def step():
            for l in range(layers):
                lw = store.layers[l]
                ops.moe_layer(store.desc(l), store.dims, hs[l], nw[l], lw.gate, lw.bias, 6, 1.5,
                              dup_mode=1 if T == 1 else 0, h_out=h_out)
        for _ in range(3):
            step()
        torch.cuda.synchronize()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            step()
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        stamps.zero_()
        calls.zero_()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        graph.replay()
        b.record()
        torch.cuda.synchronize()
        n = min(int(calls.item()), SLOTS)
        raw = stamps[:n].cpu()
        res[T] = {"us_per_call": a.elapsed_time(b) * 1000 / layers, "phases": phases(raw, n), "stamps": raw}
    return res


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--T", type=int, nargs="+", default=[1, 3, 8])
    ap.add_argument("--layers", type=int, default=8)
    args = ap.parse_args()
    if os.environ.get("HS_TRACE") != "1":
        raise SystemExit("set HS_TRACE=1 (the tracing build, python -m home_seek_b200.build --trace)")
    for T, r in run(args.T, args.layers).items():
        print(f"T={T}: {r['us_per_call']:.1f} us per layer call (tracing build); us after the route kernel's wait, "
              "min / median / max over CTAs")
        for name, (lo, med, hi) in r["phases"].items():
            print(f"  {name:28s} {lo:8.2f} {med:8.2f} {hi:8.2f}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
