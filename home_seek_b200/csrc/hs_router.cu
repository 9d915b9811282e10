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
#include "hs_topk.cuh"

namespace hs {
namespace router {

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
  const bool tv = (t0 + g) < T;
  float acc[4];
  logit_chunk(gate + static_cast<int64_t>(e0 + g) * D, gate + static_cast<int64_t>(e0 + g + 8) * D,
              h + static_cast<int64_t>(tv ? t0 + g : 0) * D, tv, kw, acc);
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
