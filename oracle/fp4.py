"""FP4 (e2m1) / FP8 (e4m3) / UE8M0 decoding on the CPU (numpy + torch).

Follows:
  - home_seek/_fp4.py:72-95 (unpack_from_e2m1fn_x2): low nibble -> even column,
    e2m1 values {0, .5, 1, 1.5, 2, 3, 4, 6} with a sign bit;
  - home_seek/fused_moe.py:604-608 (_FP4_LUT), the same table;
  - home_seek/fused_moe.py:687-691 (CPU branch of triton_dequantize_fp4_to_bf16):
    value * float(scale) rounded to bf16, one scale per 32 columns;
  - home_seek/inference_engine/weight_loader.py:14-32 (_ue8m0_to_f32,
    load_fp8_weight): e4m3 * 2^(s-127) over 128x128 blocks, shift semantics;
  - torch's float8_e8m0fnu -> float conversion for the FP4 path
    (0 -> 2^-127, 255 -> NaN).
"""
from __future__ import annotations

import numpy as np
import torch

E2M1_LUT = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                     -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=np.float32)


def unpack_e2m1(packed: np.ndarray) -> np.ndarray:
    """[..., K/2] uint8 -> [..., K] float32, low nibble first (_fp4.py:72-95)."""
    p = np.asarray(packed).view(np.uint8)
    lo = E2M1_LUT[p & 0x0F]
    hi = E2M1_LUT[(p >> 4) & 0x0F]
    return np.stack([lo, hi], axis=-1).reshape(*p.shape[:-1], p.shape[-1] * 2)


def e8m0_to_f32_torch(s: np.ndarray) -> np.ndarray:
    """UE8M0 bytes -> float32 the way torch converts float8_e8m0fnu."""
    s = np.asarray(s).view(np.uint8).astype(np.uint32)
    bits = np.where(s == 0, np.uint32(0x00400000), s << np.uint32(23))
    bits = np.where(s == 255, np.uint32(0x7FC00000), bits)
    return bits.astype(np.uint32).view(np.float32)


def e8m0_to_f32_shift(s: np.ndarray) -> np.ndarray:
    """UE8M0 bytes -> float32 by a 23-bit shift (weight_loader.py:14-19)."""
    s = np.asarray(s).view(np.uint8).astype(np.uint32)
    return (s << np.uint32(23)).astype(np.uint32).view(np.float32)


def dequant_fp4(packed: np.ndarray, scale: np.ndarray) -> torch.Tensor:
    """Packed e2m1 [N, K/2] + UE8M0 [N, K/32] -> bf16 [N, K] (fused_moe.py:687-691)."""
    v = unpack_e2m1(packed)
    sf = np.repeat(e8m0_to_f32_torch(scale), 32, axis=1)
    return torch.from_numpy(np.ascontiguousarray(v * sf)).to(torch.bfloat16)


def e4m3_to_f32(b: np.ndarray) -> np.ndarray:
    """e4m3fn bytes -> float32 (exact; 0x7F / 0xFF are NaN)."""
    b = np.asarray(b).view(np.uint8).astype(np.int32)
    sign = np.where(b & 0x80, -1.0, 1.0).astype(np.float32)
    e = (b >> 3) & 0xF
    m = (b & 0x7).astype(np.float32)
    sub = m / 8.0 * np.float32(2.0 ** -6)
    norm = (1.0 + m / 8.0) * np.power(np.float32(2.0), (e - 7).astype(np.float32))
    v = np.where(e == 0, sub, norm).astype(np.float32) * sign
    v = np.where((b & 0x7F) == 0x7F, np.float32(np.nan), v)
    return v.astype(np.float32)


def dequant_fp8_block(w: np.ndarray, scale: np.ndarray, block: int = 128) -> torch.Tensor:
    """e4m3 [N, K] + UE8M0 [N/128, K/128] -> bf16 [N, K] (weight_loader.py:22-32, _fp4.py:98-110)."""
    v = e4m3_to_f32(w)
    sf = e8m0_to_f32_shift(scale)
    sf = np.repeat(np.repeat(sf, block, axis=0), block, axis=1)[: v.shape[0], : v.shape[1]]
    return torch.from_numpy(np.ascontiguousarray(v * sf)).to(torch.bfloat16)
