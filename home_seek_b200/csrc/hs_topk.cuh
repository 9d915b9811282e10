// Router arithmetic shared by the router kernels (csrc/hs_router.cu) and the
// fused route + plan kernel of the MoE layer (csrc/hs_moe.cu), so both give
// bit-identical logits and selections. Reference: home_seek/router.py:22-36.
#pragma once

#include "hs_common.cuh"

namespace hs {
namespace router {

constexpr int kKSplitCols = 512;  // logits: columns per k-split along D
constexpr int kWarps = 4;         // 128 columns per warp per k-split

// One warp: 16 experts (rows g and g+8 of the m16n8k16 A fragment) x 8 tokens
// (columns) over the 128 columns [kw, kw + 128), bf16 MMA with f32
// accumulation. Thread c owns logical columns 8c..8c+7 of every 32-column
// group on both operands, so the MMA sums exactly the same products. alo/ahi
// point at the two experts' rows, brow at this thread's token row (tv = false:
// a padding token, read as zeros). Works on global or shared memory.
__device__ __forceinline__ void logit_chunk(const __nv_bfloat16* alo, const __nv_bfloat16* ahi,
                                            const __nv_bfloat16* brow, bool tv, int kw, float (&acc)[4]) {
  const int c = threadIdx.x & 3;
#pragma unroll
  for (int j = 0; j < 4; ++j) acc[j] = 0.f;
#pragma unroll
  for (int k = 0; k < kKSplitCols / kWarps; k += 32) {
    const int kk = kw + k + 8 * c;
    const uint4 al = *reinterpret_cast<const uint4*>(alo + kk);
    const uint4 ah = *reinterpret_cast<const uint4*>(ahi + kk);
    uint4 bv = make_uint4(0u, 0u, 0u, 0u);
    if (tv) bv = *reinterpret_cast<const uint4*>(brow + kk);
    mma_bf16(acc, al.x, ah.x, al.y, ah.y, bv.x, bv.y);
    mma_bf16(acc, al.z, ah.z, al.w, ah.w, bv.z, bv.w);
  }
}

// The four 128-column quarters [kw + 128 q, kw + 128 q + 128) of one k-split
// at once: quarter q's accumulator gets exactly logit_chunk's MMAs in
// logit_chunk's order, but the four quarters' MMAs alternate, so four
// independent accumulator chains are in flight instead of one.
__device__ __forceinline__ void logit_chunk4(const __nv_bfloat16* alo, const __nv_bfloat16* ahi,
                                             const __nv_bfloat16* brow, bool tv, int kw, float (&acc)[4][4]) {
  const int c = threadIdx.x & 3;
#pragma unroll
  for (int q = 0; q < 4; ++q)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[q][j] = 0.f;
#pragma unroll
  for (int k = 0; k < kKSplitCols / kWarps; k += 32) {
    uint4 al[4], ah[4], bv[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int kk = kw + q * (kKSplitCols / kWarps) + k + 8 * c;
      al[q] = *reinterpret_cast<const uint4*>(alo + kk);
      ah[q] = *reinterpret_cast<const uint4*>(ahi + kk);
      bv[q] = tv ? *reinterpret_cast<const uint4*>(brow + kk) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) mma_bf16(acc[q], al[q].x, ah[q].x, al[q].y, ah[q].y, bv[q].x, bv[q].y);
#pragma unroll
    for (int q = 0; q < 4; ++q) mma_bf16(acc[q], al[q].z, ah[q].z, al[q].w, ah[q].w, bv[q].z, bv[q].w);
  }
}

__device__ __forceinline__ uint64_t score_key(float s, int e) {
  const uint32_t hi = isnan(s) ? 0xffffffffu : __float_as_uint(s);  // s >= 0 (or NaN)
  return (static_cast<uint64_t>(hi) << 32) | static_cast<uint64_t>(0xffffffffu - static_cast<uint32_t>(e));
}

// One warp selects the top-K experts of one token. PER = experts per lane
// (compile-time, so scores and keys stay in registers).
template <int PER, bool kShared>
__device__ __forceinline__ void topk_token(const float* __restrict__ partial, int ksplit, int T, int E, int t,
                                           const __nv_bfloat16* __restrict__ bias, int K, float scaling,
                                           int64_t* __restrict__ idx_out, float* __restrict__ w_out,
                                           __nv_bfloat16* __restrict__ logits_out) {
  const int lane = threadIdx.x & 31;
  float sc[PER];
  uint64_t key[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane + 32 * i;
    key[i] = 0ull;
    sc[i] = 0.f;
    if (e < E) {
      // all k-split partials are loaded before the in-order sum (independent loads)
      float pv[16];
#pragma unroll
      for (int s = 0; s < 16; ++s) {
        const float* src = partial + (static_cast<int64_t>(s) * T + t) * E + e;
        pv[s] = s < ksplit ? (kShared ? *src : __ldcg(src)) : 0.f;
      }
      float l = 0.f;
#pragma unroll
      for (int s = 0; s < 16; ++s)
        if (s < ksplit) l += pv[s];
      float lb = round_bf16(l);
      if (bias) lb = round_bf16(lb + __bfloat162float(bias[e]));
      if (logits_out) logits_out[static_cast<int64_t>(t) * E + e] = __float2bfloat16_rn(lb);
      const float sp = lb > 20.f ? lb : log1pf(expf(lb));
      sc[i] = sqrtf(sp);
      key[i] = score_key(sc[i], e);
    }
  }
  float wsum = 0.f;
  float wsel = 0.f;  // lane r keeps the r-th selected score
  int esel = 0;
  for (int r = 0; r < K; ++r) {
    uint64_t best = 0ull;
#pragma unroll
    for (int i = 0; i < PER; ++i) best = key[i] > best ? key[i] : best;
    uint64_t wb = best;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const uint64_t other = __shfl_xor_sync(0xffffffffu, wb, o);
      wb = other > wb ? other : wb;
    }
    const int e = static_cast<int>(0xffffffffu - static_cast<uint32_t>(wb & 0xffffffffull));
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (key[i] == wb) {
        s = sc[i];
        key[i] = 0ull;
      }
    s = __shfl_sync(0xffffffffu, s, e & 31);
    wsum += s;  // same order on every lane: selection order
    if (lane == r) {
      wsel = s;
      esel = e;
    }
  }
  const float denom = fmaxf(wsum, 1e-20f);
  if (lane < K) {
    idx_out[static_cast<int64_t>(t) * K + lane] = esel;
    w_out[static_cast<int64_t>(t) * K + lane] = (wsel / denom) * scaling;
  }
}

template <bool kShared = false>
__device__ __forceinline__ void topk_dispatch(const float* partial, int ksplit, int T, int E, int t,
                                              const __nv_bfloat16* bias, int K, float scaling, int64_t* idx_out,
                                              float* w_out, __nv_bfloat16* logits_out) {
  const int per = (E + 31) / 32;
  if (per <= 1)
    topk_token<1, kShared>(partial, ksplit, T, E, t, bias, K, scaling, idx_out, w_out, logits_out);
  else if (per <= 2)
    topk_token<2, kShared>(partial, ksplit, T, E, t, bias, K, scaling, idx_out, w_out, logits_out);
  else if (per <= 4)
    topk_token<4, kShared>(partial, ksplit, T, E, t, bias, K, scaling, idx_out, w_out, logits_out);
  else if (per <= 8)
    topk_token<8, kShared>(partial, ksplit, T, E, t, bias, K, scaling, idx_out, w_out, logits_out);
  else if (per <= 16)
    topk_token<16, kShared>(partial, ksplit, T, E, t, bias, K, scaling, idx_out, w_out, logits_out);
  else
    topk_token<32, kShared>(partial, ksplit, T, E, t, bias, K, scaling, idx_out, w_out, logits_out);
}

}  // namespace router
}  // namespace hs
