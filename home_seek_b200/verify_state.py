"""Verify-state snapshot and restore on the device.

Reference being replaced: the state handling around the fused verify forward
of `_mtp_verify_batched` (inference_engine/engine.py:2443-2459, 2500-2538).
Before the forward the reference clones every layer's `kv_latent_cache`,
`compressed_kv_data` / `compressed_kv_idx` and compressor state (`accumulated`,
`kv_state`, `score_state`); after it, unless every position was accepted, each
KV cache is trimmed to its old length + n_accept, the compressed data and the
compressor states are put back, and the position becomes old + n_accept
(with n_accept = 0 the KV caches go back to their snapshots, which is the same
trim). Every step therefore copies O(context) bytes and allocates fresh tensors.

Here the states live in preallocated device buffers registered once:
  * `AppendBuffer` (a KV cache, the position, any append-only state): rows in a
    buffer of fixed capacity and a device entry count; a snapshot records the
    count and a commit sets it to saved + n_accept (`keep_accepted`) or back to
    saved. No bytes move.
  * copy regions (states the forward rewrites in place): copied into a shadow
    by the snapshot and back by the commit.
`VerifyState.snapshot()` and `VerifyState.commit(n_accept)` are one launch each
(hs_verify_state_snapshot / hs_verify_state_commit) over a device table of all
regions; the commit reads n_accept from device memory (the acceptance kernel's
output), so an MTP iteration with its state handling needs no host
synchronisation and can be captured in one CUDA graph.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib
from .ops import _check_cuda, _stream


class AppendBuffer:
    """Append-only rows (a KV latent cache) in a buffer of fixed capacity with
    a device entry count `length` (int64 [1])."""

    def __init__(self, capacity: int, row_shape: tuple, dtype: torch.dtype, device, init: Optional[torch.Tensor] = None):
        self.data = torch.zeros(capacity, *row_shape, dtype=dtype, device=device)
        self.length = torch.zeros(1, dtype=torch.int64, device=device)
        if init is not None and init.shape[0]:
            self.data[: init.shape[0]].copy_(init)
            self.length.fill_(init.shape[0])
        self._ar = torch.arange(capacity, device=device)

    def append(self, rows: torch.Tensor) -> None:
        """Write rows at [length, length + n) and advance length, on the device
        (no host synchronisation). Rows past the capacity are dropped."""
        n = rows.shape[0]
        pos = (self.length + self._ar[:n]).clamp(max=self.data.shape[0] - 1)
        self.data.index_copy_(0, pos, rows.to(self.data.dtype))
        self.length.add_(n)

    def view(self) -> torch.Tensor:
        """The valid rows (reads the length: a host synchronisation)."""
        return self.data[: int(self.length)]


class hs_state_region(ctypes.Structure):
    _fields_ = [("live", ctypes.c_void_p), ("shadow", ctypes.c_void_p), ("bytes", ctypes.c_int64),
                ("length", ctypes.c_void_p), ("saved_length", ctypes.c_int64), ("keep_accepted", ctypes.c_int32),
                ("reserved", ctypes.c_int32)]


class VerifyState:
    """The states a verify pass may roll back, as one device table."""

    def __init__(self, device):
        self.device = torch.device(device)
        self._regions: list = []
        self._keep: list = []       # tensors the table points into
        self._table: Optional[torch.Tensor] = None
        self._max_bytes = 0

    def add_append(self, length: torch.Tensor, keep_accepted: bool = True) -> None:
        """An append-only state by its device entry count (int64 [1]):
        keep_accepted = True keeps saved + n_accept entries after a partial
        acceptance (KV caches, the position), False rolls back to saved."""
        _check_cuda(length)
        if length.dtype != torch.int64 or length.numel() != 1:
            raise TypeError("length must be one int64 on the device")
        self._regions.append(hs_state_region(None, None, 0, length.data_ptr(), 0, int(bool(keep_accepted)), 0))
        self._keep.append(length)
        self._table = None

    def add_copy(self, state: torch.Tensor) -> None:
        """A state the forward rewrites in place: saved to a shadow by the
        snapshot and put back by the commit (contiguous, a multiple of 16 bytes)."""
        _check_cuda(state)
        nbytes = state.numel() * state.element_size()
        if nbytes % 16 or state.data_ptr() % 16:
            raise ValueError("copy regions must be 16-byte aligned and a multiple of 16 bytes")
        shadow = torch.empty_like(state)
        self._regions.append(hs_state_region(state.data_ptr(), shadow.data_ptr(), nbytes, None, 0, 0, 0))
        self._keep += [state, shadow]
        self._max_bytes = max(self._max_bytes, nbytes)
        self._table = None

    def _device_table(self) -> torch.Tensor:
        if self._table is None:
            arr = (hs_state_region * len(self._regions))(*self._regions)
            raw = torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8)
            self._table = raw.to(self.device)
        return self._table

    def snapshot(self) -> None:
        """Record every append count and copy every copy region to its shadow
        (one launch, on the current stream)."""
        t = self._device_table()
        _lib.call("hs_verify_state_snapshot", t.data_ptr(), len(self._regions), self._max_bytes,
                  _stream(self.device))

    def commit(self, n_accept: torch.Tensor, t_total: int) -> None:
        """After the verify: with n_accept (device int32) < t_total, append
        counts become saved + n_accept (or saved) and copy regions are put
        back; with everything accepted nothing changes (engine.py:2500-2538)."""
        _check_cuda(n_accept)
        if n_accept.dtype != torch.int32:
            raise TypeError("n_accept must be int32 on the device")
        t = self._device_table()
        _lib.call("hs_verify_state_commit", t.data_ptr(), len(self._regions), self._max_bytes,
                  n_accept.data_ptr(), int(t_total), _stream(self.device))
