// hs_ep.cu — expert parallelism with the tokens sharded over the ranks, as
// one C-ABI call over NCCL (hs_ep_dispatch_combine).
//
// The reference's expert parallelism (_forward_ffn_ep, engine.py:1575-1709)
// keeps every token on every GPU, runs each GPU's experts and adds the GPUs'
// bf16 outputs. Here each rank owns a shard of the tokens and the routed
// experts [r E_l, (r + 1) E_l) of a store built for it (E_l = the descriptor's
// E), plus the whole shared expert, and one call does the exchange:
//   1. ep_plan_kernel: for every other rank q, the tokens with at least one
//      expert on q (ascending), each token's place in q's list, the counts,
//      and this rank's own ids (the ids it holds, localised; others -1);
//   2. ep_pack_kernel: the rows, ids (localised to the destination) and
//      weights, destination by destination;
//   3. NCCL: the counts (one int32 per peer each way), read on the host: the
//      call's one synchronisation, as any exchange with data-dependent sizes;
//   4. NCCL: the rows, ids and weights (grouped send/recv);
//   5. hs_moe_ffn_fp4_partials on the own tokens (own experts + the shared
//      expert) and on the received rows (routed only): un-rounded f32 sums;
//   6. NCCL: the received rows' f32 sums back to their ranks;
//   7. ep_combine_kernel: every token's terms added in rank order (the own
//      term at this rank's place), then bf16(bf16(routed) + bf16(shared)), the
//      single-GPU call's rounding.
// The arithmetic is ep.TokenShardedEP.moe's step for step, so the two give
// identical bits. NCCL is resolved at run time (libnccl.so.2, the copy the
// process already loaded if any); without it the calls return
// HS_ERR_UNSUPPORTED.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <vector>

#include "hs_common.cuh"
#include "hs_ext.h"

namespace hs {
namespace ep {

constexpr int kPlanThreads = 1024;
constexpr int kMaxTokens = 65535;  // per rank: the plan's packed 16-bit counters

// The ranks (other than `self`) holding an expert of token t, as a bit mask,
// and this rank's own localised ids of the token.
__device__ __forceinline__ uint32_t token_mask(const int64_t* idx, int t, int K, int64_t El, int W, int self,
                                               int64_t* own_ids) {
  uint32_t m = 0;
  for (int k = 0; k < K; ++k) {
    const int64_t id = idx[static_cast<int64_t>(t) * K + k];
    int64_t own = -1;
    if (id >= 0 && id < El * W) {
      const int r = static_cast<int>(id / El);
      if (r == self)
        own = id - static_cast<int64_t>(self) * El;
      else
        m |= 1u << r;
    }
    if (own_ids) own_ids[static_cast<int64_t>(t) * K + k] = own;
  }
  return m;
}

// One CTA: counts[q] and pos[t][q] (the token's place in rank q's list, or
// -1) for every rank q; own_ids. Thread i takes a contiguous run of tokens;
// per-rank counts travel as 16-bit fields of two 64-bit words (ranks 0-3, 4-7)
// through one block-wide exclusive scan.
__global__ void __launch_bounds__(kPlanThreads) ep_plan_kernel(const int64_t* __restrict__ idx, int T, int K,
                                                               int64_t El, int W, int self, int32_t* counts,
                                                               int32_t* pos, int64_t* own_ids) {
  __shared__ uint64_t wsum[2][kPlanThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (T + kPlanThreads - 1) / kPlanThreads;
  const int t0 = min(T, tid * per), t1 = min(T, t0 + per);
  uint64_t c0 = 0, c1 = 0;
  for (int t = t0; t < t1; ++t) {
    const uint32_t m = token_mask(idx, t, K, El, W, self, own_ids);
#pragma unroll
    for (int r = 0; r < 8; ++r)
      if ((m >> r) & 1u) {
        if (r < 4)
          c0 += 1ull << (16 * r);
        else
          c1 += 1ull << (16 * (r - 4));
      }
  }
  // inclusive warp scan, then the warps' totals
  uint64_t i0 = c0, i1 = c1;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint64_t v0 = __shfl_up_sync(0xffffffffu, i0, o), v1 = __shfl_up_sync(0xffffffffu, i1, o);
    if (lane >= o) {
      i0 += v0;
      i1 += v1;
    }
  }
  if (lane == 31) {
    wsum[0][warp] = i0;
    wsum[1][warp] = i1;
  }
  __syncthreads();
  if (warp == 0) {
    uint64_t w0 = wsum[0][lane], w1 = wsum[1][lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint64_t v0 = __shfl_up_sync(0xffffffffu, w0, o), v1 = __shfl_up_sync(0xffffffffu, w1, o);
      if (lane >= o) {
        w0 += v0;
        w1 += v1;
      }
    }
    wsum[0][lane] = w0;  // inclusive over warps
    wsum[1][lane] = w1;
  }
  __syncthreads();
  const uint64_t b0 = (warp ? wsum[0][warp - 1] : 0ull) + i0 - c0;  // exclusive base of this thread
  const uint64_t b1 = (warp ? wsum[1][warp - 1] : 0ull) + i1 - c1;
  if (tid == 0)
    for (int r = 0; r < W; ++r)
      counts[r] = static_cast<int32_t>(((r < 4 ? wsum[0][31] : wsum[1][31]) >> (16 * (r & 3))) & 0xffffu);
  int run[8];
#pragma unroll
  for (int r = 0; r < 8; ++r) run[r] = static_cast<int>(((r < 4 ? b0 : b1) >> (16 * (r & 3))) & 0xffffu);
  for (int t = t0; t < t1; ++t) {
    const uint32_t m = token_mask(idx, t, K, El, W, self, nullptr);
#pragma unroll
    for (int r = 0; r < 8; ++r)
      if (r < W) pos[static_cast<int64_t>(t) * W + r] = ((m >> r) & 1u) ? run[r]++ : -1;
  }
}

// Rank q's first row in the send buffer (ranks in order, this rank's own list
// empty).
__device__ __forceinline__ int64_t send_base(const int32_t* counts, int q, int self) {
  int64_t o = 0;
  for (int r = 0; r < q; ++r)
    if (r != self) o += counts[r];
  return o;
}

// Block t: token t's row, ids (localised to the destination) and weights to
// every rank in its list.
__global__ void __launch_bounds__(256) ep_pack_kernel(const __nv_bfloat16* __restrict__ h,
                                                      const int64_t* __restrict__ idx, const float* __restrict__ w,
                                                      int K, int D, int64_t El, int W, int self,
                                                      const int32_t* __restrict__ counts,
                                                      const int32_t* __restrict__ pos, __nv_bfloat16* send_rows,
                                                      int64_t* send_ids, float* send_w) {
  const int t = blockIdx.x;
  const int nv = D / 8;
  for (int q = 0; q < W; ++q) {
    const int p = pos[static_cast<int64_t>(t) * W + q];
    if (p < 0) continue;
    const int64_t row = send_base(counts, q, self) + p;
    const uint4* src = reinterpret_cast<const uint4*>(h + static_cast<int64_t>(t) * D);
    uint4* dst = reinterpret_cast<uint4*>(send_rows + row * D);
    for (int v = threadIdx.x; v < nv; v += blockDim.x) dst[v] = src[v];
    if (threadIdx.x < K) {
      const int64_t id = idx[static_cast<int64_t>(t) * K + threadIdx.x];
      const int64_t lo = static_cast<int64_t>(q) * El;
      send_ids[row * K + threadIdx.x] = (id >= lo && id < lo + El) ? id - lo : -1;
      send_w[row * K + threadIdx.x] = w[static_cast<int64_t>(t) * K + threadIdx.x];
    }
  }
}

// out[t][d] = bf16(bf16(routed) + bf16(shared)), routed = the terms of every
// rank in order from 0 (this rank's own sum at its place, a peer's only where
// the token was sent there), accumulated from 0 in f32.
__global__ void __launch_bounds__(256) ep_combine_kernel(const float* __restrict__ own_r,
                                                         const float* __restrict__ own_s,
                                                         const float* __restrict__ back,
                                                         const int32_t* __restrict__ counts,
                                                         const int32_t* __restrict__ pos, int T, int D, int W,
                                                         int self, int use_shared, __nv_bfloat16* out) {
  __shared__ int64_t base[8];
  if (threadIdx.x < 8) base[threadIdx.x] = threadIdx.x < W ? send_base(counts, threadIdx.x, self) : 0;
  __syncthreads();
  const int64_t n4 = static_cast<int64_t>(T) * D / 4;
  const int d4n = D / 4;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / d4n;
    const int64_t d4 = i - t * d4n;
    float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int q = 0; q < W; ++q) {
      float4 v;
      if (q == self) {
        v = reinterpret_cast<const float4*>(own_r)[i];
      } else {
        const int p = pos[t * W + q];
        if (p < 0) continue;
        v = reinterpret_cast<const float4*>(back)[(base[q] + p) * d4n + d4];
      }
      r.x += v.x;
      r.y += v.y;
      r.z += v.z;
      r.w += v.w;
    }
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    if (use_shared) s = reinterpret_cast<const float4*>(own_s)[i];
    const float rr[4] = {r.x, r.y, r.z, r.w}, ss[4] = {s.x, s.y, s.z, s.w};
    __nv_bfloat16 y[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float o = round_bf16(rr[k]);
      if (use_shared) o += round_bf16(ss[k]);
      y[k] = __float2bfloat16_rn(o);
    }
    reinterpret_cast<uint2*>(out)[i] =
        make_uint2(static_cast<uint32_t>(__bfloat16_as_ushort(y[0])) | (static_cast<uint32_t>(__bfloat16_as_ushort(y[1])) << 16),
                   static_cast<uint32_t>(__bfloat16_as_ushort(y[2])) | (static_cast<uint32_t>(__bfloat16_as_ushort(y[3])) << 16));
  }
}

// ---------------------------------------------------------------------------
// NCCL, resolved at run time
// ---------------------------------------------------------------------------
struct Nccl {
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRank) comm_init_rank = nullptr;
  decltype(&ncclCommDestroy) comm_destroy = nullptr;
  decltype(&ncclCommCount) comm_count = nullptr;
  decltype(&ncclCommUserRank) comm_user_rank = nullptr;
  decltype(&ncclGroupStart) group_start = nullptr;
  decltype(&ncclGroupEnd) group_end = nullptr;
  decltype(&ncclSend) send = nullptr;
  decltype(&ncclRecv) recv = nullptr;
  bool ok = false;
};

static const Nccl* nccl() {
  static const Nccl api = [] {
    Nccl a;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // the copy already in the process, if any
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW);
    if (!h) return a;
#define HS_NCCL_SYM(field, name) a.field = reinterpret_cast<decltype(a.field)>(dlsym(h, #name))
    HS_NCCL_SYM(get_unique_id, ncclGetUniqueId);
    HS_NCCL_SYM(comm_init_rank, ncclCommInitRank);
    HS_NCCL_SYM(comm_destroy, ncclCommDestroy);
    HS_NCCL_SYM(comm_count, ncclCommCount);
    HS_NCCL_SYM(comm_user_rank, ncclCommUserRank);
    HS_NCCL_SYM(group_start, ncclGroupStart);
    HS_NCCL_SYM(group_end, ncclGroupEnd);
    HS_NCCL_SYM(send, ncclSend);
    HS_NCCL_SYM(recv, ncclRecv);
#undef HS_NCCL_SYM
    a.ok = a.get_unique_id && a.comm_init_rank && a.comm_destroy && a.comm_count && a.comm_user_rank &&
           a.group_start && a.group_end && a.send && a.recv;
    return a;
  }();
  return api.ok ? &api : nullptr;
}

#define HS_NCCL_CHECK(expr)            \
  do {                                 \
    if ((expr) != ncclSuccess) return HS_ERR_NCCL; \
  } while (0)

// Workspace regions (256-byte aligned), from the same arguments on every rank.
struct Layout {
  size_t counts, rcounts, pos, own_ids, send_rows, send_ids, send_w, recv_rows, recv_ids, recv_w, own_r, own_s,
      y_recv, back, moe, moe_bytes, total;
};

static Layout layout(int64_t T_max, int64_t K, int64_t D, int64_t I, int64_t I_sh, int64_t W) {
  Layout l{};
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o += (bytes + 255) & ~static_cast<size_t>(255);
    return at;
  };
  const int64_t cap = T_max * (W - 1);  // rows sent (or received) at most: once per token and peer
  l.counts = take(sizeof(int32_t) * 8);
  l.rcounts = take(sizeof(int32_t) * 8);
  l.pos = take(sizeof(int32_t) * T_max * W);
  l.own_ids = take(sizeof(int64_t) * T_max * K);
  l.send_rows = take(2 * cap * D);
  l.send_ids = take(sizeof(int64_t) * cap * K);
  l.send_w = take(sizeof(float) * cap * K);
  l.recv_rows = take(2 * cap * D);
  l.recv_ids = take(sizeof(int64_t) * cap * K);
  l.recv_w = take(sizeof(float) * cap * K);
  l.own_r = take(sizeof(float) * T_max * D);
  l.own_s = take(sizeof(float) * T_max * D);
  l.y_recv = take(sizeof(float) * cap * D);
  l.back = take(sizeof(float) * cap * D);
  l.moe_bytes = std::max(hs_moe_workspace_size(std::max<int64_t>(T_max, 1), K, D, I, I_sh),
                         hs_moe_workspace_size(std::max<int64_t>(cap, 1), K, D, I, I_sh));
  l.moe = take(l.moe_bytes);
  l.total = o;
  return l;
}

static int plan_launch(const int64_t* idx, int64_t T, int64_t K, int64_t El, int W, int self, int32_t* counts,
                       int32_t* pos, int64_t* own_ids, cudaStream_t st) {
  if (T == 0) {
    HS_CUDA_CHECK(cudaMemsetAsync(counts, 0, sizeof(int32_t) * W, st));
    return HS_OK;
  }
  ep_plan_kernel<<<1, kPlanThreads, 0, st>>>(idx, static_cast<int>(T), static_cast<int>(K), El, W, self, counts,
                                             pos, own_ids);
  return check_launch();
}

}  // namespace ep
}  // namespace hs

using namespace hs;
using namespace hs::ep;

extern "C" int hs_ep_nccl_unique_id(void* id_out) {
  const Nccl* nc = nccl();
  if (!nc) return HS_ERR_UNSUPPORTED;
  if (!id_out) return HS_ERR_BAD_ARGUMENT;
  ncclUniqueId id;
  HS_NCCL_CHECK(nc->get_unique_id(&id));
  memcpy(id_out, &id, sizeof(id));
  return HS_OK;
}

extern "C" int hs_ep_nccl_comm_init(const void* id, int32_t world, int32_t rank, void** comm) {
  const Nccl* nc = nccl();
  if (!nc) return HS_ERR_UNSUPPORTED;
  if (!id || !comm) return HS_ERR_BAD_ARGUMENT;
  if (world < 1 || world > HS_EP_MAX_RANKS || rank < 0 || rank >= world) return HS_ERR_BAD_SHAPE;
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  ncclComm_t c = nullptr;
  HS_NCCL_CHECK(nc->comm_init_rank(&c, world, uid, rank));
  *comm = c;
  return HS_OK;
}

extern "C" int hs_ep_nccl_comm_destroy(void* comm) {
  const Nccl* nc = nccl();
  if (!nc) return HS_ERR_UNSUPPORTED;
  if (!comm) return HS_OK;
  HS_NCCL_CHECK(nc->comm_destroy(static_cast<ncclComm_t>(comm)));
  return HS_OK;
}

extern "C" int hs_ep_dispatch_plan(const int64_t* topk_idx, int64_t T, int64_t top_k, int64_t experts_per_rank,
                                   int32_t world, int32_t rank, int32_t* counts, int32_t* pos, int64_t* own_ids,
                                   void* stream) {
  if (T < 0 || T > kMaxTokens || top_k < 1 || top_k > 16 || experts_per_rank < 1 || world < 1 ||
      world > HS_EP_MAX_RANKS || rank < 0 || rank >= world)
    return HS_ERR_BAD_SHAPE;
  if (!counts || (T > 0 && (!topk_idx || !pos))) return HS_ERR_BAD_ARGUMENT;
  return plan_launch(topk_idx, T, top_k, experts_per_rank, world, rank, counts, pos, own_ids,
                     static_cast<cudaStream_t>(stream));
}

extern "C" size_t hs_ep_dispatch_combine_workspace_size(int64_t T_max, int64_t top_k, int64_t D, int64_t I,
                                                        int64_t I_sh, int32_t world) {
  if (T_max < 0 || T_max > kMaxTokens || top_k < 1 || world < 1 || world > HS_EP_MAX_RANKS) return 0;
  return layout(T_max, top_k, D, I, I_sh, world).total;
}

extern "C" int hs_ep_dispatch_combine(void* comm, const void* desc, const void* hidden, const int64_t* topk_idx,
                                      const float* topk_w, int64_t T, int64_t T_max, int64_t top_k, int use_shared,
                                      int dup_mode, void* out, void* workspace, size_t workspace_bytes,
                                      int32_t* dev_status, void* stream) {
  const Nccl* nc = nccl();
  if (!nc) return HS_ERR_UNSUPPORTED;
  if (!comm || !workspace) return HS_ERR_BAD_ARGUMENT;
  ncclComm_t c = static_cast<ncclComm_t>(comm);
  int W = 0, self = 0;
  HS_NCCL_CHECK(nc->comm_count(c, &W));
  HS_NCCL_CHECK(nc->comm_user_rank(c, &self));
  int64_t El = 0, D = 0, I = 0, I_sh = 0;
  int st = moe_desc_dims(desc, &El, &D, &I, &I_sh);
  if (st) return st;
  // arguments every rank passes alike: a mismatch is returned before any exchange
  if (W < 1 || W > HS_EP_MAX_RANKS || T_max < 0 || T_max > kMaxTokens || top_k < 1 || top_k > 16)
    return HS_ERR_BAD_SHAPE;
  const Layout L = layout(T_max, top_k, D, I, I_sh, W);
  if (workspace_bytes < L.total) return HS_ERR_WORKSPACE;
  // this rank's own arguments: a bad one makes the rank take part with no tokens
  // (the peers' exchanges still complete) and return the error afterwards
  int local = HS_OK;
  if (T < 0 || T > T_max) local = HS_ERR_BAD_SHAPE;
  else if (T > 0 && (!hidden || !topk_idx || !topk_w || !out)) local = HS_ERR_BAD_ARGUMENT;
  else if (T > 0 && (!aligned16(hidden) || !aligned16(out))) local = HS_ERR_ALIGN;
  const int64_t Tl = local ? 0 : T;
  use_shared = use_shared && I_sh > 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int32_t* counts = reinterpret_cast<int32_t*>(ws + L.counts);
  int32_t* rcounts = reinterpret_cast<int32_t*>(ws + L.rcounts);
  int32_t* pos = reinterpret_cast<int32_t*>(ws + L.pos);
  int64_t* own_ids = reinterpret_cast<int64_t*>(ws + L.own_ids);
  __nv_bfloat16* send_rows = reinterpret_cast<__nv_bfloat16*>(ws + L.send_rows);
  int64_t* send_ids = reinterpret_cast<int64_t*>(ws + L.send_ids);
  float* send_w = reinterpret_cast<float*>(ws + L.send_w);
  __nv_bfloat16* recv_rows = reinterpret_cast<__nv_bfloat16*>(ws + L.recv_rows);
  int64_t* recv_ids = reinterpret_cast<int64_t*>(ws + L.recv_ids);
  float* recv_w = reinterpret_cast<float*>(ws + L.recv_w);
  float* own_r = reinterpret_cast<float*>(ws + L.own_r);
  float* own_s = reinterpret_cast<float*>(ws + L.own_s);
  float* y_recv = reinterpret_cast<float*>(ws + L.y_recv);
  float* back = reinterpret_cast<float*>(ws + L.back);
  void* moe_ws = ws + L.moe;

  // 1-2. plan and pack
  if ((st = plan_launch(topk_idx, Tl, top_k, El, W, self, counts, pos, own_ids, s))) return st;
  if (Tl > 0 && W > 1) {
    ep_pack_kernel<<<static_cast<unsigned>(Tl), 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(hidden), topk_idx, topk_w, static_cast<int>(top_k), static_cast<int>(D),
        El, W, self, counts, pos, send_rows, send_ids, send_w);
    if ((st = check_launch())) return st;
  }
  // 3. the counts both ways, on the host
  std::vector<int32_t> sc(W, 0), rc(W, 0);
  if (W > 1) {
    HS_NCCL_CHECK(nc->group_start());
    for (int p = 0; p < W; ++p) {
      if (p == self) continue;
      HS_NCCL_CHECK(nc->send(counts + p, 1, ncclInt32, p, c, s));
      HS_NCCL_CHECK(nc->recv(rcounts + p, 1, ncclInt32, p, c, s));
    }
    HS_NCCL_CHECK(nc->group_end());
    HS_CUDA_CHECK(cudaMemcpyAsync(sc.data(), counts, sizeof(int32_t) * W, cudaMemcpyDeviceToHost, s));
    HS_CUDA_CHECK(cudaMemcpyAsync(rc.data(), rcounts, sizeof(int32_t) * W, cudaMemcpyDeviceToHost, s));
    HS_CUDA_CHECK(cudaStreamSynchronize(s));
    sc[self] = 0;
    rc[self] = 0;
  }
  std::vector<int64_t> so(W + 1, 0), ro(W + 1, 0);
  for (int p = 0; p < W; ++p) {
    so[p + 1] = so[p] + sc[p];
    ro[p + 1] = ro[p] + rc[p];
  }
  const int64_t n_recv = ro[W];
  if (n_recv > T_max * (W - 1)) return HS_ERR_BAD_SHAPE;  // a peer holds more than T_max tokens
  const int64_t K = top_k;
  // 4. rows, ids and weights to their ranks
  if (W > 1) {
    HS_NCCL_CHECK(nc->group_start());
    for (int p = 0; p < W; ++p) {
      if (p == self) continue;
      HS_NCCL_CHECK(nc->send(send_rows + so[p] * D, static_cast<size_t>(sc[p] * D), ncclBfloat16, p, c, s));
      HS_NCCL_CHECK(nc->recv(recv_rows + ro[p] * D, static_cast<size_t>(rc[p] * D), ncclBfloat16, p, c, s));
      HS_NCCL_CHECK(nc->send(send_ids + so[p] * K, static_cast<size_t>(sc[p] * K), ncclInt64, p, c, s));
      HS_NCCL_CHECK(nc->recv(recv_ids + ro[p] * K, static_cast<size_t>(rc[p] * K), ncclInt64, p, c, s));
      HS_NCCL_CHECK(nc->send(send_w + so[p] * K, static_cast<size_t>(sc[p] * K), ncclFloat32, p, c, s));
      HS_NCCL_CHECK(nc->recv(recv_w + ro[p] * K, static_cast<size_t>(rc[p] * K), ncclFloat32, p, c, s));
    }
    HS_NCCL_CHECK(nc->group_end());
  }
  // 5. this rank's experts: own tokens (with the shared expert), received rows
  if (Tl > 0 &&
      (st = hs_moe_ffn_fp4_partials(desc, hidden, own_ids, topk_w, Tl, K, use_shared, dup_mode, own_r,
                                    use_shared ? own_s : nullptr, moe_ws, L.moe_bytes, dev_status, stream)))
    return st;
  if (n_recv > 0 &&
      (st = hs_moe_ffn_fp4_partials(desc, recv_rows, recv_ids, recv_w, n_recv, K, 0, dup_mode, y_recv, nullptr,
                                    moe_ws, L.moe_bytes, dev_status, stream)))
    return st;
  // 6. the received rows' sums back to their ranks
  if (W > 1) {
    HS_NCCL_CHECK(nc->group_start());
    for (int p = 0; p < W; ++p) {
      if (p == self) continue;
      HS_NCCL_CHECK(nc->send(y_recv + ro[p] * D, static_cast<size_t>(rc[p] * D), ncclFloat32, p, c, s));
      HS_NCCL_CHECK(nc->recv(back + so[p] * D, static_cast<size_t>(sc[p] * D), ncclFloat32, p, c, s));
    }
    HS_NCCL_CHECK(nc->group_end());
  }
  // 7. every token's terms in rank order, rounded as the single-GPU call
  if (Tl > 0) {
    const int64_t n4 = Tl * D / 4;
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>((n4 + 255) / 256, 148 * 8));
    ep_combine_kernel<<<grid, 256, 0, s>>>(own_r, own_s, back, counts, pos, static_cast<int>(Tl),
                                           static_cast<int>(D), W, self, use_shared,
                                           static_cast<__nv_bfloat16*>(out));
    if ((st = check_launch())) return st;
  }
  return local;
}
