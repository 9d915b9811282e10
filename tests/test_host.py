"""Host-side logic on the CPU: the expert store's tiled layout and its
reference-format copies, the loader protocol, and expert-id localisation for sharded stores."""
from __future__ import annotations

import numpy as np
import torch

from oracle import inputs as I


def test_store_layout_and_reference_format():
    from home_seek_b200.expert_store import HBMExpertStore
    sh = I.SMALL
    st = HBMExpertStore(2, sh.E, sh.D, sh.I, sh.I_sh, device="cpu", hash_layers=1, vocab_size=100)
    w = I.expert_fp4(5, sh.D, sh.I)
    st.set_expert(1, 5, *w)
    raw = st._load_expert_fp4_raw(1, 5)
    assert raw[0].dtype == torch.int8 and raw[1].dtype == torch.float8_e8m0fnu
    assert raw[0].shape == (sh.I, sh.D // 2) and raw[4].shape == (sh.D, sh.I // 2)
    for got, want in zip(raw, w):
        assert np.array_equal(got.view(torch.uint8).numpy(), want)
    # the store keeps tiles: tile (row tile 1, k chunk 2) of w3 is one contiguous block
    tile = st.layers[1].w13[5, 1, 2, 1]
    assert tile.is_contiguous() and tile.shape == (128, 64)
    assert np.array_equal(tile.numpy(), w[2][128:256, 128:192])
    trip = st._load_expert_weights(1, 5)
    assert [e[2] for e in trip] == ["fp4_gpu"] * 3
    assert st.layers[0].tid2eid is not None and st.layers[1].tid2eid is None
    assert st.bytes_per_expert() == 3 * sh.I * sh.D // 2 + 3 * sh.I * sh.D // 32


def test_config0_expert_bytes():
    from home_seek_b200.mtp import ModelShape
    # B_exp = 3 * I * D * (1/2 + 1/32), engine.py:152 (I*D*51/32)
    assert ModelShape().bytes_per_expert == 13_369_344 == 2048 * 4096 * 51 // 32


def test_loader_protocol_and_localise():
    from home_seek_b200.expert_store import HBMExpertStore
    from home_seek_b200.fused_moe import _localise, _e8m0_bytes
    sh = I.SMALL
    st = HBMExpertStore(1, sh.E, sh.D, sh.I, None, device="cpu", with_router=False, expert_offset=8,
                        experts_held=8)
    fn = st.loader()
    assert fn.__hs_store__ is st
    assert fn(0, 3) is None and fn(0, 9) is not None
    idx = torch.tensor([[0, 8, 15, 16, -1]])
    assert _localise(idx, 8, 8).tolist() == [[-1, 0, 7, -1, -1]]
    s = torch.tensor([1.0, 2.0, 0.5, 2.0 ** -9], dtype=torch.float32)
    assert _e8m0_bytes(s).tolist() == [127, 128, 126, 118]


def test_scale_atom_layout_roundtrip_and_formula():
    from home_seek_b200.layout import atoms_to_scales, block_scales_to_atoms, scales_to_atoms
    g = torch.Generator().manual_seed(0)
    s = torch.randint(0, 256, (256, 64), generator=g, dtype=torch.uint8)
    a = scales_to_atoms(s)
    assert a.shape == (2, 16, 512)
    assert torch.equal(atoms_to_scales(a), s)
    # byte m0*16 + m1*4 + j of atom (ra, ka) = s[128*ra + 32*m1 + m0][4*ka + j]
    for ra, ka, m0, m1, j in [(0, 0, 0, 0, 0), (1, 3, 31, 3, 3), (0, 7, 5, 2, 1), (1, 15, 17, 1, 2)]:
        assert a[ra, ka, m0 * 16 + m1 * 4 + j] == s[128 * ra + 32 * m1 + m0, 4 * ka + j]
    b = torch.tensor([[121, 120]], dtype=torch.uint8)
    ab = block_scales_to_atoms(b)
    assert ab.shape == (1, 2, 512) and (ab[0, 0] == 121).all() and (ab[0, 1] == 120).all()


def test_fp4_and_fp8_block_forms_recovered_from_bf16_losslessly():
    """layout.fp4_block_from_bf16 / fp8_block_from_bf16 invert the reference's
    dequantisations (fused_moe.py:672-735, weight_loader.py:22-32) exactly,
    and refuse bf16 weights that are not such values."""
    import pytest
    import torch
    from home_seek_b200.layout import fp4_block_from_bf16, fp8_block_dequant, fp8_block_from_bf16
    from oracle import fp4 as F
    from oracle import inputs as I
    w1, s1, *_ = I.expert_fp4(5, 512, 512)
    bf = F.dequant_fp4(w1, s1)
    p, s = fp4_block_from_bf16(bf)
    assert torch.equal(F.dequant_fp4(p.numpy(), s.numpy()), bf)
    with pytest.raises(TypeError):
        fp4_block_from_bf16((bf.float() * 1.1).to(torch.bfloat16))
    w13, s13, _, _ = I.shared_fp8(512, 512, seed=2)
    d8 = torch.from_numpy(w13[0])
    b8 = fp8_block_dequant(d8, torch.from_numpy(s13[0]))
    assert torch.equal(b8, F.dequant_fp8_block(w13[0], s13[0]))
    q, k = fp8_block_from_bf16(b8)
    assert torch.equal(fp8_block_dequant(q, k), b8)
    with pytest.raises(TypeError):
        fp8_block_from_bf16((b8.float() * 1.01).to(torch.bfloat16))


def test_vocab_rows_tile_the_vocabulary():
    """ops.vocab_rows: the ranks' head rows are disjoint, cover [0, V) in rank
    order, start on 128-row tiles and differ by at most one tile."""
    from home_seek_b200 import ops
    for V in (129280, 1000, 128, 5000, 257):
        for world in (1, 2, 3, 4, 8):
            parts = [ops.vocab_rows(V, r, world) for r in range(world)]
            pos = 0
            for row0, rows in parts:
                assert row0 == pos and row0 % 128 == 0
                pos += rows
            assert pos == V
            tiles = [(r + 127) // 128 for _, r in parts]
            assert max(tiles) - min(tiles) <= 1


def test_ep_dispatch_combine_workspace_sizes():
    """The C-ABI exchange's workspace: grows with T_max and the group, and bad
    arguments give 0 (the call then refuses with HS_ERR_BAD_SHAPE)."""
    from home_seek_b200 import _lib
    lib = _lib.load()
    size = lib.hs_ep_dispatch_combine_workspace_size
    s1 = size(1024, 6, 4096, 2048, 2048, 2)
    assert s1 > 2 * 1024 * 4096 * 2           # the rows sent and received
    assert size(2048, 6, 4096, 2048, 2048, 2) > s1
    assert size(1024, 6, 4096, 2048, 2048, 8) > s1
    assert size(1024, 6, 4096, 2048, 2048, 1) > 0
    assert size(-1, 6, 4096, 2048, 2048, 2) == 0
    assert size(70000, 6, 4096, 2048, 2048, 2) == 0
    assert size(1024, 6, 4096, 2048, 2048, 9) == 0
    assert lib.hs_ep_dispatch_plan(None, 3, 6, 32, 9, 0, None, None, None, None) == 1   # world 9: bad shape
    assert lib.hs_ep_dispatch_plan(None, 3, 6, 32, 2, 0, None, None, None, None) == 2   # NULL outputs


def test_trace_phases_from_stamps():
    """home_seek_b200.trace.phases on a synthetic stamp array: times are per
    call relative to the route kernel's wait (kernel 0, CTA 0, event 1), CTAs
    without a stamp are ignored, and the first and last calls are left out."""
    import torch
    from home_seek_b200 import trace
    X = torch.zeros(5, trace.KERNELS, trace.CTAS, trace.EVENTS, dtype=torch.int64)
    for i in range(5):
        base = 1_000_000 * (i + 1)
        X[i, 0, 0, 1] = base                            # route wait over
        X[i, 0, :16, 0] = base - 1500                   # route entry
        X[i, 1, :10, 1] = base + torch.arange(10) * 100 + 9000   # gate/up wait: 9.0 .. 9.9 us
        X[i, 2, :256, 5] = base + 60_000                # down done at 60 us
    ph = trace.phases(X, 5)
    assert ph["route entry"] == (-1.5, -1.5, -1.5)
    lo, med, hi = ph["gate/up wait over"]
    assert abs(lo - 9.0) < 1e-9 and abs(hi - 9.9) < 1e-9 and abs(med - 9.45) < 1e-9
    assert ph["down done"] == (60.0, 60.0, 60.0)
    assert ph["next call's route wait over"][0] == 1000.0
    assert "combine done" not in ph                     # no stamps, no phase
