// RMSNorm, the residual add fused with the next RMSNorm, and the MoE combine of
// f32 partial sums (expert parallelism) fused with both, sm_100a.
//
// Reference being replaced: home_seek/utils.py:6-9 (rms_norm, applied before
// every FFN at inference_engine/engine.py:2679 and before the logits at
// engine.py:2482) and the residual add that closes each layer
// (engine.py:2685). In the decode loop the residual add of layer l and the
// norm that opens layer l+1 touch the same row, so one launch does both.
//
// Numerics follow the reference operation by operation, in f32:
//   h' = bf16(h + y)                      (bf16 + bf16 computed in f32)
//   var = sum(f32(x)^2) / D               (each square rounded, then summed)
//   out = bf16(f32(w) * (f32(x) * (1 / sqrt(var + eps))))
// The sum runs in a fixed order (per-thread, then a fixed shuffle tree, then
// warps in order), so results are deterministic; the reference's reduction
// order differs, which can move var by an ulp.
#include <algorithm>

#include "hs_common.cuh"

namespace hs {
namespace norm {

constexpr int kThreads = kNormThreads;
constexpr int kMaxVec = kNormMaxVec;  // 8 bf16 per vector: D <= kThreads * 8 * kMaxVec = 8192

// The MoE output from un-rounded f32 partial sums (already summed over
// expert-parallel ranks): bf16(bf16(routed) + bf16(shared)), the rounding the
// single-GPU kernel applies (engine.py:1530-1536).
__device__ __forceinline__ void combine8(const float* r, const float* sh, int64_t off, bool use_shared, float (&o)[8]) {
  const float4 r0 = reinterpret_cast<const float4*>(r + off)[0], r1 = reinterpret_cast<const float4*>(r + off)[1];
  const float rv[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
  float sv[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (use_shared) {
    const float4 s0 = reinterpret_cast<const float4*>(sh + off)[0], s1 = reinterpret_cast<const float4*>(sh + off)[1];
    sv[0] = s0.x, sv[1] = s0.y, sv[2] = s0.z, sv[3] = s0.w, sv[4] = s1.x, sv[5] = s1.y, sv[6] = s1.z, sv[7] = s1.w;
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) o[k] = round_bf16(round_bf16(rv[k]) + (use_shared ? round_bf16(sv[k]) : 0.f));
}

// One CTA per row. kMode 0: normalise h. 1: h_out = bf16(h + y), normalised.
// 2: y is the MoE combine of f32 partials (r, sh); h_out = bf16(h + y),
// normalised. h_out may alias h (every element is read and written by the same
// thread).
template <int kMode>
__global__ void __launch_bounds__(kThreads) add_norm_kernel(const __nv_bfloat16* h, const __nv_bfloat16* y,
                                                            const float* r, const float* sh, int use_shared,
                                                            const __nv_bfloat16* __restrict__ w, float eps, int D,
                                                            __nv_bfloat16* h_out, __nv_bfloat16* __restrict__ x_out) {
  pdl_trigger();
  pdl_wait();
  const int64_t row = static_cast<int64_t>(blockIdx.x) * D;
  const int nv = D / 8;
  const uint4* hr = reinterpret_cast<const uint4*>(h + row);
  float v[kMaxVec][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int j = threadIdx.x + i * kThreads;
    if (j < nv) {
      bf16x8_unpack(hr[j], v[i]);
      if (kMode != 0) {
        float g[8];
        if (kMode == 1)
          bf16x8_unpack(reinterpret_cast<const uint4*>(y + row)[j], g);
        else
          combine8(r, sh, row + 8 * static_cast<int64_t>(j), use_shared != 0, g);
#pragma unroll
        for (int k = 0; k < 8; ++k) v[i][k] = round_bf16(__fadd_rn(v[i][k], g[k]));
        reinterpret_cast<uint4*>(h_out + row)[j] = bf16x8_pack(v[i]);
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) ss = __fadd_rn(ss, __fmul_rn(v[i][k], v[i][k]));
    }
  }
  if (kMode != 0 && x_out == nullptr) return;  // the residual add alone (uniform over the CTA)
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
  __shared__ float part[kThreads / 32];
  __shared__ float rinv;
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int i = 0; i < kThreads / 32; ++i) tot = __fadd_rn(tot, part[i]);
    const float var = __fdiv_rn(tot, static_cast<float>(D));
    rinv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(var, eps)));
  }
  __syncthreads();
  const float ri = rinv;
  const uint4* wr = reinterpret_cast<const uint4*>(w);
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int j = threadIdx.x + i * kThreads;
    if (j < nv) {
      float wf[8], o[8];
      bf16x8_unpack(wr[j], wf);
#pragma unroll
      for (int k = 0; k < 8; ++k) o[k] = __fmul_rn(wf[k], __fmul_rn(v[i][k], ri));
      reinterpret_cast<uint4*>(x_out + row)[j] = bf16x8_pack(o);
    }
  }
}

static int launch(int mode, const void* h, const void* y, const float* r, const float* sh, int use_shared,
                  const void* w, float eps, int64_t T, int64_t D, void* h_out, void* x_out, void* stream) {
  if (T < 0 || D < 8 || D % 8 != 0 || D > kThreads * 8 * kMaxVec || T > (1 << 24)) return HS_ERR_BAD_SHAPE;
  if (T == 0) return HS_OK;
  // modes 1 and 2 may leave out the norm (w and x_out both NULL): the add alone
  const bool no_norm = mode != 0 && !w && !x_out;
  if (!h || (!no_norm && (!w || !x_out)) || (mode != 0 && !h_out) || (mode == 1 && !y) ||
      (mode == 2 && (!r || (use_shared && !sh))))
    return HS_ERR_BAD_ARGUMENT;
  if (!aligned16(h) || (w && !aligned16(w)) || (x_out && !aligned16(x_out)) || (h_out && !aligned16(h_out)) || (y && !aligned16(y)) ||
      (r && !aligned16(r)) || (sh && !aligned16(sh)))
    return HS_ERR_ALIGN;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const auto* hb = static_cast<const __nv_bfloat16*>(h);
  const auto* yb = static_cast<const __nv_bfloat16*>(y);
  const auto* wb = static_cast<const __nv_bfloat16*>(w);
  auto* ho = static_cast<__nv_bfloat16*>(h_out);
  auto* xo = static_cast<__nv_bfloat16*>(x_out);
  const dim3 grid(static_cast<unsigned>(T)), block(kThreads);
  const int Di = static_cast<int>(D);
  if (mode == 0)
    HS_CUDA_CHECK(launch_pdl(add_norm_kernel<0>, grid, block, 0, st, hb, yb, r, sh, use_shared, wb, eps, Di, ho, xo));
  else if (mode == 1)
    HS_CUDA_CHECK(launch_pdl(add_norm_kernel<1>, grid, block, 0, st, hb, yb, r, sh, use_shared, wb, eps, Di, ho, xo));
  else
    HS_CUDA_CHECK(launch_pdl(add_norm_kernel<2>, grid, block, 0, st, hb, yb, r, sh, use_shared, wb, eps, Di, ho, xo));
  return check_launch();
}

__global__ void __launch_bounds__(kThreads) combine_kernel(const float* __restrict__ r, const float* __restrict__ sh,
                                                           int use_shared, int64_t n8, __nv_bfloat16* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  for (int64_t j = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; j < n8;
       j += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float o[8];
    combine8(r, sh, 8 * j, use_shared != 0, o);
    reinterpret_cast<uint4*>(out)[j] = bf16x8_pack(o);
  }
}

}  // namespace norm
}  // namespace hs

extern "C" int hs_rms_norm(const void* x, const void* w, float eps, int64_t T, int64_t D, void* out, void* stream) {
  return hs::norm::launch(0, x, nullptr, nullptr, nullptr, 0, w, eps, T, D, nullptr, out, stream);
}

extern "C" int hs_add_rms_norm(const void* h, const void* y, const void* w, float eps, int64_t T, int64_t D,
                               void* h_out, void* x_out, void* stream) {
  return hs::norm::launch(1, h, y, nullptr, nullptr, 0, w, eps, T, D, h_out, x_out, stream);
}

extern "C" int hs_moe_combine(const float* routed_f32, const float* shared_f32, int use_shared, int64_t T, int64_t D,
                              void* out, void* stream) {
  using namespace hs;
  if (T < 0 || D < 8 || D % 8 != 0) return HS_ERR_BAD_SHAPE;
  if (T == 0) return HS_OK;
  if (!routed_f32 || !out || (use_shared && !shared_f32)) return HS_ERR_BAD_ARGUMENT;
  if (!aligned16(routed_f32) || !aligned16(out) || (shared_f32 && !aligned16(shared_f32))) return HS_ERR_ALIGN;
  const int64_t n8 = T * D / 8;
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>((n8 + hs::norm::kThreads - 1) / hs::norm::kThreads, 1184));
  HS_CUDA_CHECK(launch_pdl(hs::norm::combine_kernel, dim3(grid), dim3(hs::norm::kThreads), 0,
                           static_cast<cudaStream_t>(stream), routed_f32, shared_f32, use_shared, n8,
                           static_cast<__nv_bfloat16*>(out)));
  return check_launch();
}

extern "C" int hs_moe_combine_add_rms_norm(const float* routed_f32, const float* shared_f32, int use_shared,
                                           const void* h, const void* w, float eps, int64_t T, int64_t D,
                                           void* h_out, void* x_out, void* stream) {
  return hs::norm::launch(2, h, nullptr, routed_f32, shared_f32, use_shared, w, eps, T, D, h_out, x_out, stream);
}
