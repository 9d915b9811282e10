"""Scale-factor layout of the HBM expert store.

The kernels feed UE8M0 scales to the tensor cores' scale-factor memory with
one 32x128-bit copy per 128 rows x 128 columns. The store therefore keeps
every scale matrix s[R][KB] (one byte per row and 32-column block) as atoms of
512 bytes: atom (ra, ka) holds rows 128*ra .. 128*ra+127 and blocks 4*ka ..
4*ka+3, byte m0*16 + m1*4 + j = s[128*ra + 32*m1 + m0][4*ka + j]. Each 32-bit
word then holds one row's four consecutive block scales (the tensor memory
word), and the 16-byte line m0 holds rows m0, m0+32, m0+64, m0+96.
"""
from __future__ import annotations

import torch


def scales_to_atoms(s: torch.Tensor) -> torch.Tensor:
    """[R, KB] uint8 (R % 128 == 0, KB % 4 == 0) -> [R/128, KB/4, 512]."""
    R, KB = s.shape
    if R % 128 or KB % 4:
        raise ValueError(f"scale matrix {tuple(s.shape)} is not a whole number of 128x4 atoms")
    v = s.reshape(R // 128, 4, 32, KB // 4, 4)            # (ra, m1, m0, ka, j)
    return v.permute(0, 3, 2, 1, 4).reshape(R // 128, KB // 4, 512).contiguous()


def atoms_to_scales(a: torch.Tensor) -> torch.Tensor:
    """[R/128, KB/4, 512] -> [R, KB] (inverse of scales_to_atoms)."""
    ra, ka, _ = a.shape
    v = a.reshape(ra, ka, 32, 4, 4).permute(0, 3, 2, 1, 4)  # (ra, m1, m0, ka, j)
    return v.reshape(ra * 128, ka * 4).contiguous()


def block_scales_to_atoms(b: torch.Tensor) -> torch.Tensor:
    """128x128 block scales [..., R/128, K/128] -> atoms [..., R/128, K/128, 512]
    (a 128x128 block is exactly one atom, so every byte is the block's scale)."""
    return b.unsqueeze(-1).expand(*b.shape, 512).contiguous()
