// Router (sqrt-softplus + bias, stable top-k) and hash routing, sm_100a.
//
// Reference being replaced: home_seek/router.py:22-36
// (compute_expert_affinity_with_bias) and router.py:10-19
// (compute_expert_affinity), reached from inference_engine/engine.py:1025-1031;
// hash routing at engine.py:1018-1023.
//
// Numerics follow the reference operation by operation:
//   logits = bf16(sum_k h[k] * gate[e][k])  (f32 accumulate, one rounding)
//   logits = bf16(f32(logits) + f32(bias))  (the bf16 add rounds again)
//   s = sqrt(softplus(f32(logits)))         (softplus threshold 20 as torch)
//   top-k by s, ties to the lower expert id (torch.sort(stable=True))
//   w = s / max(sum(s), 1e-20) * routed_scaling
// Because s is a strictly increasing function of the bf16 logit (apart from
// the far negative tail where exp underflows), the selected indices equal the
// reference's whenever the bf16 logits agree; the only source of difference is
// the order of the f32 sum inside the GEMV, which can move a logit that sits
// on a bf16 rounding boundary by one bf16 ulp.
//
// Kernel 1 (logits): CTA = 16 experts x up to 8 tokens x D/ksplit columns,
// warp MMA m16n8k16 bf16 with f32 accumulate, the 4 warps reduced in a fixed
// order, partial sums written per k-split (deterministic, no atomics).
// Kernel 2 (top-k): one warp per token sums the k-split partials in order,
// applies the roundings/transcendentals and selects by warp-shuffle arg-max.
#include "hs_common.cuh"

namespace hs {
namespace router {

constexpr int kKSplitCols = 512;  // columns per CTA along D
constexpr int kWarps = 4;         // 128 columns per warp per CTA
constexpr int kFusedTopkTokens = 64;  // T <= this: top-k runs in the last logits CTA

struct TopkArgs {
  const __nv_bfloat16* bias;
  int K;
  float scaling;
  int64_t* idx_out;
  float* w_out;
  __nv_bfloat16* logits_out;
  uint32_t* counter;  // nullptr: a separate top-k launch follows
};

__device__ __forceinline__ void topk_dispatch(const float* partial, int ksplit, int T, int E, int t,
                                              const __nv_bfloat16* bias, int K, float scaling, int64_t* idx_out,
                                              float* w_out, __nv_bfloat16* logits_out);

__global__ void __launch_bounds__(kWarps * 32) logits_kernel(const __nv_bfloat16* __restrict__ h,
                                                             const __nv_bfloat16* __restrict__ gate, int T, int D,
                                                             int E, float* __restrict__ partial, TopkArgs ta) {
  pdl_trigger();  // the plan kernel may start its prologue
  pdl_wait();     // the hidden rows (and everything earlier) are complete
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int e0 = blockIdx.x * 16;
  const int ks = blockIdx.y;
  const int t0 = blockIdx.z * 8;
  const int kw = ks * kKSplitCols + warp * (kKSplitCols / kWarps);
  const __nv_bfloat16* alo = gate + static_cast<int64_t>(e0 + g) * D;
  const __nv_bfloat16* ahi = gate + static_cast<int64_t>(e0 + g + 8) * D;
  const bool tv = (t0 + g) < T;
  const __nv_bfloat16* brow = h + static_cast<int64_t>(tv ? t0 + g : 0) * D;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int k = 0; k < kKSplitCols / kWarps; k += 32) {
    // thread c owns logical columns 8c..8c+7 of this 32-column group on both
    // operands, so the MMA sums exactly the same products.
    const int kk = kw + k + 8 * c;
    const uint4 al = *reinterpret_cast<const uint4*>(alo + kk);
    const uint4 ah = *reinterpret_cast<const uint4*>(ahi + kk);
    uint4 bv = make_uint4(0u, 0u, 0u, 0u);
    if (tv) bv = *reinterpret_cast<const uint4*>(brow + kk);
    mma_bf16(acc, al.x, ah.x, al.y, ah.y, bv.x, bv.y);
    mma_bf16(acc, al.z, ah.z, al.w, ah.w, bv.z, bv.w);
  }
  __shared__ float red[kWarps][32][4];
#pragma unroll
  for (int j = 0; j < 4; ++j) red[warp][lane][j] = acc[j];
  __syncthreads();
  if (warp == 0) {
    float s[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) s[j] = ((red[0][lane][j] + red[1][lane][j]) + red[2][lane][j]) + red[3][lane][j];
    // C layout: rows (experts) g / g+8, columns (tokens) 2c, 2c+1
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = e0 + g + ((j & 2) ? 8 : 0);
      const int t = t0 + 2 * c + (j & 1);
      if (t < T) partial[(static_cast<int64_t>(ks) * T + t) * E + e] = s[j];
    }
  }
  if (ta.counter == nullptr) return;
  // Last CTA to finish runs the top-k for every token (small T only). The
  // ticket is an atomic on a workspace counter that the last CTA resets; no
  // CTA ever waits for another.
  __shared__ int last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t total = gridDim.x * gridDim.y * gridDim.z;
    last = atomicAdd(ta.counter, 1u) == total - 1u;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  const int ksplit = gridDim.y;
  for (int t = warp; t < T; t += kWarps)
    topk_dispatch(partial, ksplit, T, E, t, ta.bias, ta.K, ta.scaling, ta.idx_out, ta.w_out, ta.logits_out);
  if (threadIdx.x == 0) *ta.counter = 0u;
}

__device__ __forceinline__ uint64_t score_key(float s, int e) {
  const uint32_t hi = isnan(s) ? 0xffffffffu : __float_as_uint(s);  // s >= 0 (or NaN)
  return (static_cast<uint64_t>(hi) << 32) | static_cast<uint64_t>(0xffffffffu - static_cast<uint32_t>(e));
}

// One warp selects the top-K experts of one token. PER = experts per lane
// (compile-time, so scores and keys stay in registers).
template <int PER>
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
      for (int s = 0; s < 16; ++s) pv[s] = s < ksplit ? __ldcg(partial + (static_cast<int64_t>(s) * T + t) * E + e) : 0.f;
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

__device__ __forceinline__ void topk_dispatch(const float* partial, int ksplit, int T, int E, int t,
                                              const __nv_bfloat16* bias, int K, float scaling, int64_t* idx_out,
                                              float* w_out, __nv_bfloat16* logits_out) {
  const int per = (E + 31) / 32;
  if (per <= 1)
    topk_token<1>(partial, ksplit, T, E, t, bias, K, scaling, idx_out, w_out, logits_out);
  else if (per <= 2)
    topk_token<2>(partial, ksplit, T, E, t, bias, K, scaling, idx_out, w_out, logits_out);
  else if (per <= 4)
    topk_token<4>(partial, ksplit, T, E, t, bias, K, scaling, idx_out, w_out, logits_out);
  else if (per <= 8)
    topk_token<8>(partial, ksplit, T, E, t, bias, K, scaling, idx_out, w_out, logits_out);
  else if (per <= 16)
    topk_token<16>(partial, ksplit, T, E, t, bias, K, scaling, idx_out, w_out, logits_out);
  else
    topk_token<32>(partial, ksplit, T, E, t, bias, K, scaling, idx_out, w_out, logits_out);
}

__global__ void __launch_bounds__(128) topk_kernel(const float* __restrict__ partial, int ksplit, int T, int E,
                                                   const __nv_bfloat16* __restrict__ bias, int K, float scaling,
                                                   int64_t* __restrict__ idx_out, float* __restrict__ w_out,
                                                   __nv_bfloat16* __restrict__ logits_out) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x * 4 + (threadIdx.x >> 5);
  if (t >= T) return;
  topk_dispatch(partial, ksplit, T, E, t, bias, K, scaling, idx_out, w_out, logits_out);
}

__global__ void hash_kernel(const int64_t* __restrict__ ids, int T, const int64_t* __restrict__ tid2eid, int64_t V,
                            int K, float w, int64_t* __restrict__ idx_out, float* __restrict__ w_out, int32_t* status) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= T * K) return;
  const int t = i / K, j = i - t * K;
  const int64_t id = ids[t];
  int64_t e = -1;
  if (id < 0 || id >= V)
    report(status, HS_DEV_BAD_TOKEN);
  else
    e = tid2eid[id * K + j];
  idx_out[i] = e;
  w_out[i] = w;
}

}  // namespace router
}  // namespace hs

using namespace hs;
using namespace hs::router;

extern "C" size_t hs_router_workspace_size(int64_t T, int64_t D, int64_t E) {
  if (T < 0 || D < kKSplitCols || E < 1) return 0;
  return static_cast<size_t>(D / kKSplitCols) * T * E * sizeof(float) + 512;
}

extern "C" int hs_router_topk(const void* hidden, const void* gate, const void* bias, int64_t T, int64_t D, int64_t E,
                              int64_t top_k, float routed_scaling, int64_t* topk_idx, float* topk_w, void* logits_out,
                              void* workspace, size_t workspace_bytes, void* stream) {
  if (T < 0 || D % kKSplitCols != 0 || D < kKSplitCols || D > 16 * kKSplitCols || E % 16 != 0 || E < 16 ||
      E > 1024 || top_k < 1 || top_k > 16 || top_k > E)
    return HS_ERR_BAD_SHAPE;
  if (T == 0) return HS_OK;
  if (T > 65535 * 8) return HS_ERR_BAD_SHAPE;
  if (!hidden || !gate || !topk_idx || !topk_w || !workspace) return HS_ERR_BAD_ARGUMENT;
  if (!aligned16(hidden) || !aligned16(gate)) return HS_ERR_ALIGN;
  if (workspace_bytes < hs_router_workspace_size(T, D, E)) return HS_ERR_WORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int ksplit = static_cast<int>(D / kKSplitCols);
  // workspace: [0, 256) counter (zero at rest), then the k-split partials
  uint32_t* counter = static_cast<uint32_t*>(workspace);
  float* partial = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + 256);
  const bool fused = T <= kFusedTopkTokens;
  TopkArgs ta{static_cast<const __nv_bfloat16*>(bias), static_cast<int>(top_k), routed_scaling, topk_idx, topk_w,
              static_cast<__nv_bfloat16*>(logits_out), fused ? counter : nullptr};
  dim3 g1(static_cast<unsigned>(E / 16), static_cast<unsigned>(ksplit), static_cast<unsigned>((T + 7) / 8));
  HS_CUDA_CHECK(launch_pdl(logits_kernel, g1, dim3(kWarps * 32), 0, st, static_cast<const __nv_bfloat16*>(hidden),
                           static_cast<const __nv_bfloat16*>(gate), static_cast<int>(T), static_cast<int>(D),
                           static_cast<int>(E), partial, ta));
  int rc = check_launch();
  if (rc || fused) return rc;
  HS_CUDA_CHECK(launch_pdl(topk_kernel, dim3(static_cast<unsigned>((T + 3) / 4)), dim3(128), 0, st,
                           static_cast<const float*>(partial), ksplit, static_cast<int>(T), static_cast<int>(E),
                           static_cast<const __nv_bfloat16*>(bias), static_cast<int>(top_k), routed_scaling, topk_idx,
                           topk_w, static_cast<__nv_bfloat16*>(logits_out)));
  return check_launch();
}

extern "C" int hs_hash_route(const int64_t* input_ids, int64_t T, const int64_t* tid2eid, int64_t V, int64_t top_k,
                             int64_t* topk_idx, float* topk_w, int32_t* dev_status, void* stream) {
  if (T < 0 || V < 1 || top_k < 1 || top_k > 64) return HS_ERR_BAD_SHAPE;
  if (T == 0) return HS_OK;
  if (!input_ids || !tid2eid || !topk_idx || !topk_w) return HS_ERR_BAD_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int n = static_cast<int>(T * top_k);
  // torch.full(..., 1.0 / k) with a float32 default dtype
  const float w = static_cast<float>(1.0 / static_cast<double>(top_k));
  HS_CUDA_CHECK(launch_pdl(hash_kernel, dim3((n + 255) / 256), dim3(256), 0, st, input_ids, static_cast<int>(T),
                           tid2eid, V, static_cast<int>(top_k), w, topk_idx, topk_w, dev_status));
  return check_launch();
}
