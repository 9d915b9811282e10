"""hs_moe_ffn_fp4_noalloc: the MoE call for callers that cannot allocate device
memory when they call (plugin hosts whose enqueue path forbids allocation,
latency-critical loops where cudaMalloc/cudaFree would synchronise the
device). It uses a fixed scratch array inside the library instead of a
caller workspace; this test checks it through the C ABI against the
workspace-taking hs_moe_ffn_fp4 on two calls in a row. Both entry points run
the same deterministic kernels (fixed-order reductions, the same schedule),
so the outputs must be bit-identical, not merely within the MoE tolerance.
The file name sorts last so a stop-at-first-failure run has already run
every other test."""
from __future__ import annotations

import ctypes

import pytest
import torch

from oracle import inputs as I

pytestmark = pytest.mark.gpu


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float().cpu(), b.float().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp(min=1e-30))


def _noalloc(lib, store, h, idx, w, out):
    st = torch.cuda.current_stream().cuda_stream
    return lib.hs_moe_ffn_fp4_noalloc(ctypes.addressof(store.desc(0)), h.data_ptr(), idx.data_ptr(), w.data_ptr(),
                                      h.shape[0], idx.shape[1], 1, 0, out.data_ptr(), None, None, st)


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    from home_seek_b200 import _lib, ops
    from home_seek_b200.expert_store import HBMExpertStore

    lib = _lib.load()
    shape = I.SMALL
    gate, bias = I.router_weights(shape.E, shape.D, seed=31)
    store = HBMExpertStore(1, shape.E, shape.D, shape.I, shape.I_sh, device="cuda", with_router=False)
    load = I.make_loader(shape)
    for e in range(shape.E):
        store.set_expert(0, e, *load(e))
    store.set_shared(0, *I.shared_fp8(shape.D, shape.I_sh, seed=32))

    for call, T in enumerate((3, 5)):  # two calls in a row through the shared scratch
        h = I.hidden(T, shape.D, seed=40 + call).cuda()
        idx, w = ops.router_topk(h, gate.cuda(), bias.cuda(), shape.K, 1.5)
        ref = ops.moe_ffn(store.desc(0), store.dims, h, idx, w, use_shared=True)
        out = torch.empty_like(ref)
        assert _noalloc(lib, store, h, idx, w, out) == 0
        torch.cuda.synchronize()
        assert torch.equal(out, ref), (call, _rel(out, ref))


def test_noalloc_rejects_sizes_beyond_its_scratch():
    from home_seek_b200 import _lib
    from home_seek_b200.expert_store import HBMExpertStore

    lib = _lib.load()
    store = HBMExpertStore(1, 16, 4096, 2048, 2048, device="cuda", with_router=False)
    # 64 tokens x top-6 at D = 4096 needs more than the fixed scratch holds
    assert lib.hs_moe_workspace_size(64, 6, 4096, 2048, 2048) > _lib.HS_MOE_NOALLOC_BYTES
    h = torch.zeros(64, 4096, dtype=torch.bfloat16, device="cuda")
    idx = torch.zeros(64, 6, dtype=torch.int64, device="cuda")
    w = torch.zeros(64, 6, dtype=torch.float32, device="cuda")
    out = torch.empty_like(h)
    assert _noalloc(lib, store, h, idx, w, out) == 3  # HS_ERR_WORKSPACE, nothing launched
