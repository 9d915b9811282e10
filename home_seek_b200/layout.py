"""Weight and scale layouts of the HBM expert store.

Weight tiles. The kernels stream 128-row x 128-column tiles. The store keeps
each expert's packed e2m1 matrices tiled so that every tile is contiguous in
HBM (8 KB of packed FP4, rows of 64 bytes) and the tiles one pipeline stage
reads are adjacent: one TMA fetches 16 KB of consecutive bytes.
  w13 [E][I/128][D/128][2][128][64]   w1 tile then w3 tile of (row tile, k chunk)
  w2  [E][D/128][I/128][128][64]      consecutive k chunks adjacent
  sh_w13 [I_sh/128][D/128][2][128][128]  (e4m3, one byte per value)
  sh_w2  [D/128][I_sh/128][128][128]

Scale-factor atoms. The kernels feed UE8M0 scales to the tensor cores'
scale-factor memory with one 32x128-bit copy per 128 rows x 128 columns. Every
scale matrix s[R][KB] (one byte per row and 32-column block) is kept as atoms
of 512 bytes: atom (ra, ka) holds rows 128*ra .. 128*ra+127 and blocks 4*ka ..
4*ka+3, byte m0*16 + m1*4 + j = s[128*ra + 32*m1 + m0][4*ka + j]. Each 32-bit
word then holds one row's four consecutive block scales (the tensor memory
word), and the 16-byte line m0 holds rows m0, m0+32, m0+64, m0+96. The atoms a
stage needs are adjacent too:
  s13 [E][I/128][D/128][2][512], s2 [E][D/128][I/128][512],
  sh_s13 [I_sh/128][D/128][2][512], sh_s2 [D/128][I_sh/128][512].
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


def tile_rows(w: torch.Tensor, row_bytes: int) -> torch.Tensor:
    """[R, C] bytes -> [R/128, C/row_bytes, 128, row_bytes]: 128-row tiles of
    row_bytes columns, each tile contiguous."""
    R, C = w.shape
    if R % 128 or C % row_bytes:
        raise ValueError(f"matrix {tuple(w.shape)} is not a whole number of 128 x {row_bytes} tiles")
    return w.reshape(R // 128, 128, C // row_bytes, row_bytes).permute(0, 2, 1, 3).contiguous()


def untile_rows(t: torch.Tensor) -> torch.Tensor:
    """Inverse of tile_rows: [RT, CT, 128, rb] -> [RT*128, CT*rb]."""
    RT, CT, r, rb = t.shape
    return t.permute(0, 2, 1, 3).reshape(RT * r, CT * rb).contiguous()
