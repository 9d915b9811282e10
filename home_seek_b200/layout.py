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


def fp8_block_dequant(data: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """e4m3 [R, C] with UE8M0 128x128 block scales [R/128, C/128] -> bf16: the
    value load_fp8_weight gives (weight_loader.py:22-32, exact: an e4m3 value
    times a power of two fits bf16)."""
    R, C = data.shape
    v = data.view(torch.float8_e4m3fn).float()
    e = scale.contiguous().view(torch.uint8).to(torch.int32)
    f = torch.ldexp(torch.ones_like(e, dtype=torch.float32), e - 127)
    f = f.repeat_interleave(128, 0)[:R].repeat_interleave(128, 1)[:, :C]
    return (v * f).to(torch.bfloat16)


def fp8_block_from_bf16(w: torch.Tensor):
    """Inverse of fp8_block_dequant for weights that came from it: bf16 [R, C]
    -> (e4m3 bytes [R, C] uint8, UE8M0 block scales [R/128, C/128] uint8).

    Per 128x128 block the scale is the smallest power of two 2^k with max|w| /
    2^k <= 448; every w / 2^k is then an e4m3 value exactly (an e4m3 value
    times 2^(k0 - k) with k <= k0 keeps its three mantissa bits). Raises
    TypeError when a block has a value that no e4m3 x 2^k represents (a bf16
    weight that did not come from an FP8 block-scaled one)."""
    R, C = w.shape
    if R % 128 or C % 128:
        raise TypeError(f"FP8 block form needs 128-multiple shapes, got {tuple(w.shape)}")
    f = w.float()
    blk = f.abs().reshape(R // 128, 128, C // 128, 128).amax(dim=(1, 3))
    k = torch.ceil(torch.log2(torch.clamp(blk, min=2.0 ** -100) / 448.0)).to(torch.int32).clamp(-127, 127)
    k = torch.where(blk == 0, torch.full_like(k, -6), k)
    mul = torch.ldexp(torch.ones_like(k, dtype=torch.float32), -k).repeat_interleave(128, 0).repeat_interleave(128, 1)
    q = (f * mul).to(torch.float8_e4m3fn)
    if not torch.equal(q.float() / mul, f):
        raise TypeError("bf16 weight is not an FP8 (e4m3, 128x128 power-of-two block scale) value")
    return q.view(torch.uint8), (k + 127).to(torch.uint8)


_E2M1_MAG = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)


def fp4_block_from_bf16(w: torch.Tensor):
    """bf16 [R, C] that came from packed e2m1 with one UE8M0 scale per 32
    columns (load_fp4_weight / the reference's BF16 expert cache,
    fused_moe.py:672-735) -> (packed e2m1 [R, C/2] uint8, low nibble = even
    column; UE8M0 scales [R, C/32] uint8).

    Per 32-column block the scale is 2^k with k = ceil(log2(max|w| / 6)); every
    w / 2^k is then an e2m1 value (an e2m1 value m times 2^s, with s fixed by
    how far the block's largest value sits below 6, stays in the e2m1 set), so
    the conversion is lossless; the scale byte may differ from the one the
    weights were made with, the products do not. Raises TypeError for a value
    no e2m1 x 2^k represents."""
    R, C = w.shape
    if C % 32:
        raise TypeError(f"FP4 block form needs a multiple of 32 columns, got {C}")
    f = w.float().reshape(R, C // 32, 32)
    blk = f.abs().amax(-1)
    k = torch.ceil(torch.log2(torch.clamp(blk, min=2.0 ** -120) / 6.0)).to(torch.int32).clamp(-127, 127)
    k = torch.where(blk == 0, torch.full_like(k, -127), k)
    q = f * torch.ldexp(torch.ones_like(k, dtype=torch.float32), -k).unsqueeze(-1)
    mag = torch.tensor(_E2M1_MAG, dtype=torch.float32, device=w.device)
    code = torch.searchsorted(mag, q.abs().contiguous()).clamp(max=7)
    if not torch.equal(mag[code], q.abs()):
        raise TypeError("bf16 weight is not an FP4 (e2m1, 32-column power-of-two block scale) value")
    code = code | (torch.signbit(q).to(torch.int64) << 3)
    code = code.reshape(R, C).to(torch.uint8)
    packed = code[:, 0::2] | (code[:, 1::2] << 4)
    return packed.contiguous(), (k + 127).to(torch.uint8).contiguous()
