"""Verify-state snapshot / restore on the device (hs_verify_state_snapshot /
hs_verify_state_commit through verify_state.VerifyState) against the
reference's _mtp_verify_batched state handling (engine.py:2443-2459,
2500-2538), recorded in tests/golden/golden.npz for n_accept = 0, 1, 2 of 3
positions: the same seeded states and the same mocked forward
(oracle/verify_state.forward_mutation) applied to device buffers, then the
device commit with n_accept in device memory must leave exactly the
reference's states and position. The whole sequence also runs inside one
CUDA graph."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import verify_state as VS

pytestmark = pytest.mark.gpu


def _bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)


class _DeviceLayer:
    """One layer's states in device buffers: KV and compressed rows as append
    buffers (the compressed index too), the compressor state as copy regions."""

    def __init__(self, st: dict, dev, ids: list, layer: int):
        from home_seek_b200.verify_state import AppendBuffer
        kv = st["kv"][0]
        d = kv.shape[-1]
        # the rows the mocked forward appends, made before any graph capture
        self.rows_kv = VS.forward_rows(ids, layer, d).to(dev)
        self.rows_c = VS.forward_rows(ids[:1], layer + 100, d).to(dev)
        self.T, self.layer = len(ids), layer
        self.kv = AppendBuffer(64, kv.shape[1:], torch.bfloat16, dev, kv.to(dev))
        cd = st["cdata"][0]
        self.cdata = AppendBuffer(64, cd.shape[1:], torch.bfloat16, dev, cd.to(dev))
        self.cidx = AppendBuffer(64, (), torch.int64, dev, st["cidx"].to(dev))
        acc, kvs, scs = st["comp"]
        self.acc = torch.tensor([acc, 0], dtype=torch.int64, device=dev)  # 16 bytes
        self.kvs = kvs.to(dev).contiguous()
        self.scs = scs.to(dev).contiguous()

    def register(self, vs) -> None:
        vs.add_append(self.kv.length, keep_accepted=True)      # KV cache: old + n_accept
        vs.add_append(self.cdata.length, keep_accepted=False)  # compressed KV: restored
        vs.add_append(self.cidx.length, keep_accepted=False)
        for t in (self.acc, self.kvs, self.scs):                # compressor: restored
            vs.add_copy(t)

    def forward(self) -> None:
        """oracle/verify_state.forward_mutation on the device buffers."""
        self.kv.append(self.rows_kv)
        self.cdata.append(self.rows_c)
        last = self.cidx.data[(self.cidx.length - 1).clamp(min=0)]
        self.cidx.append(last + 4)
        self.acc[0] += self.T
        self.kvs.add_(1 + self.layer)
        self.scs.mul_(0.5)


def _check(layers: dict, pos, golden, case: int) -> None:
    n, p = (int(v) for v in golden[f"vs{case}_n"])
    assert int(pos.length) == p
    for l, dl in layers.items():
        assert torch.equal(dl.kv.view().cpu(), _bf16(golden[f"vs{case}_kv{l}"])[0]), (case, l)
        assert torch.equal(dl.cdata.view().cpu(), _bf16(golden[f"vs{case}_cdata{l}"])[0]), (case, l)
        assert dl.cidx.view().cpu().tolist() == golden[f"vs{case}_cidx{l}"].tolist()
        assert int(dl.acc[0]) == int(golden[f"vs{case}_acc{l}"][0])
        assert torch.equal(dl.kvs.cpu(), torch.from_numpy(golden[f"vs{case}_kvs{l}"]))
        assert torch.equal(dl.scs.cpu(), torch.from_numpy(golden[f"vs{case}_scs{l}"]))


@pytest.mark.parametrize("graph", [False, True])
def test_device_snapshot_commit_matches_reference(golden, graph):
    from home_seek_b200.verify_state import AppendBuffer, VerifyState
    dev = torch.device("cuda")
    for case in range(3):
        before = VS.scenario_states(seed=7 + case)
        layers = {l: _DeviceLayer(st, dev, [5, 9, 13], l) for l, st in before.items()}
        pos = AppendBuffer(1, (), torch.int64, dev)   # the position as a count
        pos.length.fill_(40)
        vs = VerifyState(dev)
        for dl in layers.values():
            dl.register(vs)
        vs.add_append(pos.length, keep_accepted=True)
        n_acc = torch.tensor([int(golden[f"vs{case}_n"][0])], dtype=torch.int32, device=dev)

        def step():
            vs.snapshot()
            for dl in layers.values():
                dl.forward()
            pos.length.add_(1)   # the verify advances the position (engine.py:2467)
            vs.commit(n_acc, 3)

        if graph:
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            g = torch.cuda.CUDAGraph()
            vs._device_table()  # the table is uploaded before the capture
            with torch.cuda.graph(g, stream=s):
                step()
            g.replay()
        else:
            step()
        torch.cuda.synchronize()
        _check(layers, pos, golden, case)


def test_commit_keeps_everything_when_all_positions_are_accepted():
    from home_seek_b200.verify_state import AppendBuffer, VerifyState
    dev = torch.device("cuda")
    kv = AppendBuffer(16, (8,), torch.bfloat16, dev, torch.ones(3, 8, dtype=torch.bfloat16, device=dev))
    st = torch.arange(8, dtype=torch.float32, device=dev)
    vs = VerifyState(dev)
    vs.add_append(kv.length)
    vs.add_copy(st)
    vs.snapshot()
    kv.append(torch.zeros(3, 8, dtype=torch.bfloat16, device=dev))
    st.mul_(2)
    vs.commit(torch.tensor([3], dtype=torch.int32, device=dev), 3)
    torch.cuda.synchronize()
    assert int(kv.length) == 6 and torch.equal(st.cpu(), torch.arange(8, dtype=torch.float32) * 2)
