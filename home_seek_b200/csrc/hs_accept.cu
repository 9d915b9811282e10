// Speculative-decode acceptance over 129280-wide logits, sm_100a.
//
// Reference being replaced: the greedy loop inside
// HomeSeekInferenceEngine._mtp_verify_batched (inference_engine/engine.py:
// 2485-2497) and the bonus token choice in generate() (engine.py:2908-2913).
// The reference has no rejection sampling; hs_accept_rejection implements
// standard speculative sampling (Leviathan et al. 2023, "Fast Inference from
// Transformers via Speculative Decoding"; Chen et al. 2023).
//
// One thread-block cluster of 8 CTAs per sequence: each CTA streams one eighth
// of every logits row of the sequence (16-byte loads, four in flight per
// thread, HBM-bound), each warp reduces its part of every row, one barrier
// and a fixed-order reduction over the warps follow, and the cluster combines
// the 8 partial results through distributed shared memory in rank order
// (deterministic). Greedy folds each 16-byte chunk with the packed
// NaN-propagating bf16 max and locates an index only in a chunk that beats the
// running maximum; rejection sampling evaluates the softmax as
// 2^((x - max) * log2(e) / t), one fused multiply-add and one ex2 per value.
// The only waits are hardware cluster barriers.
#include <cooperative_groups.h>

#include "hs_common.cuh"

namespace cg = cooperative_groups;

namespace hs {
namespace accept {

constexpr int kCluster = 8;
constexpr int kThreads = 256;
constexpr int kMaxRows = 16;

// torch.argmax: first maximal index, NaN counts as maximal.
__device__ __forceinline__ bool better(float v1, int i1, float v2, int i2) {
  const bool n1 = isnan(v1), n2 = isnan(v2);
  if (n1 || n2) {
    if (n1 && n2) return i1 < i2;
    return n1;
  }
  return v1 > v2 || (v1 == v2 && i1 < i2);
}

__device__ __forceinline__ void slice_of(int V, int rank, int& lo, int& hi) {
  const int per = ((V + kCluster * 8 - 1) / (kCluster * 8)) * 8;
  lo = min(V, rank * per);
  hi = min(V, lo + per);
}

__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__device__ __forceinline__ __nv_bfloat162 as_bf162(uint32_t w) {
  return *reinterpret_cast<const __nv_bfloat162*>(&w);
}

constexpr int kBatch = 4;  // 16-byte chunks each thread has in flight per row

// One thread's chunk u of a batch: chunk index i0 + u * blockDim.x.
__device__ __forceinline__ void argmax_chunk(const uint4& q, int base, float& v, int& ix) {
  const __nv_bfloat162 m2 =
      __hmax2_nan(__hmax2_nan(as_bf162(q.x), as_bf162(q.y)), __hmax2_nan(as_bf162(q.z), as_bf162(q.w)));
  const float cm = __bfloat162float(__hmax_nan(m2.x, m2.y));
  const bool nan_chunk = isnan(cm);
  if (cm > v || (nan_chunk && !isnan(v)) || ix == 0x7fffffff) {  // (the first chunk: a row of -inf)
    // the chunk wins: its first element equal to the folded maximum (the first
    // NaN when it holds one; -0 and +0 compare equal)
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
    int j = 7;
#pragma unroll
    for (int e = 7; e >= 0; --e) {
      const float x = (e & 1) ? bf16hi(w[e >> 1]) : bf16lo(w[e >> 1]);
      j = (nan_chunk ? isnan(x) : x == cm) ? e : j;
    }
    v = cm;
    ix = base + j;
  }
}

// Warp-level arg-max of one row slice [lo, hi): every lane gets the warp's
// (value, first index). Each thread scans its 16-byte chunks in ascending
// index order, kBatch loads in flight at a time, and keeps (value, first
// index); a chunk's eight values are first folded with the packed
// NaN-propagating bf16 max, and only a chunk whose maximum beats the running
// value (greater, or NaN over a number), and the thread's first chunk, are
// scanned element by element, so equal values keep the earlier index and the
// first NaN wins, as torch.argmax.
__device__ void warp_argmax(const __nv_bfloat16* __restrict__ row, int lo, int hi, float& v, int& ix) {
  v = -INFINITY;
  ix = 0x7fffffff;
  // 8 bf16 per 16-byte load; lo is a multiple of 8 and rows are 16-byte aligned
  const int nvec = (hi - lo) / 8;
  const uint4* p = reinterpret_cast<const uint4*>(row + lo);
  const int bd = static_cast<int>(blockDim.x);
  for (int i0 = threadIdx.x; i0 < nvec; i0 += kBatch * bd) {
    uint4 q[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u)
      if (i0 + u * bd < nvec) q[u] = __ldcs(p + i0 + u * bd);
#pragma unroll
    for (int u = 0; u < kBatch; ++u)
      if (i0 + u * bd < nvec) argmax_chunk(q[u], lo + 8 * (i0 + u * bd), v, ix);
  }
  for (int k = lo + nvec * 8 + threadIdx.x; k < hi; k += bd) {
    const float a = __bfloat162float(row[k]);
    if (better(a, k, v, ix)) {
      v = a;
      ix = k;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, ix, o);
    if (better(v2, i2, v, ix)) {
      v = v2;
      ix = i2;
    }
  }
}

__global__ void __cluster_dims__(kCluster, 1, 1) __launch_bounds__(kThreads)
    greedy_kernel(const __nv_bfloat16* __restrict__ logits, int T, int V, const int64_t* __restrict__ draft_ids,
                  int32_t* __restrict__ n_acc, int64_t* __restrict__ next_tok, int64_t* __restrict__ argmax_out) {
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = static_cast<int>(cluster.block_rank());
  const int b = blockIdx.x / kCluster;
  __shared__ float pv[kMaxRows];
  __shared__ int pi[kMaxRows];
  __shared__ float wv[kMaxRows][kThreads / 32];
  __shared__ int wi[kMaxRows][kThreads / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int lo, hi;
  slice_of(V, rank, lo, hi);
  // every row's warp results first, then one barrier and the CTA reduction
  for (int i = 0; i < T; ++i) {
    float v;
    int ix;
    warp_argmax(logits + (static_cast<int64_t>(b) * T + i) * V, lo, hi, v, ix);
    if (lane == 0) {
      wv[i][warp] = v;
      wi[i][warp] = ix;
    }
  }
  __syncthreads();
  if (threadIdx.x < T) {
    const int i = threadIdx.x;
    float v = wv[i][0];
    int ix = wi[i][0];
    for (int w2 = 1; w2 < kThreads / 32; ++w2)
      if (better(wv[i][w2], wi[i][w2], v, ix)) {
        v = wv[i][w2];
        ix = wi[i][w2];
      }
    pv[i] = v;
    pi[i] = ix;
  }
  cluster.sync();
  if (rank == 0 && warp == 0) {
    // lane (row i, rank r): all remote loads at once, then the 8 ranks of a
    // row combined with shuffles (the (value, first index) order does not
    // depend on the combining order)
    __shared__ int am[kMaxRows];
    for (int i0 = 0; i0 < T; i0 += 32 / kCluster) {
      const int i = i0 + lane / kCluster, r = lane % kCluster;
      float v = -INFINITY;
      int ix = 0x7fffffff;
      if (i < T) {
        v = cluster.map_shared_rank(pv, r)[i];
        ix = cluster.map_shared_rank(pi, r)[i];
      }
#pragma unroll
      for (int o = kCluster / 2; o > 0; o >>= 1) {
        const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
        const int i2 = __shfl_xor_sync(0xffffffffu, ix, o);
        if (i2 != 0x7fffffff && (ix == 0x7fffffff || better(v2, i2, v, ix))) {
          v = v2;
          ix = i2;
        }
      }
      if (i < T && r == 0) {
        am[i] = ix;
        if (argmax_out) argmax_out[static_cast<int64_t>(b) * T + i] = ix;
      }
    }
    __syncwarp();
    if (lane == 0) {
      int n = 0;
      while (n < T - 1 && static_cast<int64_t>(am[n]) == draft_ids[static_cast<int64_t>(b) * (T - 1) + n]) ++n;
      n_acc[b] = n;
      next_tok[b] = am[n];
    }
  }
  cluster.sync();
}

// ---------------------------------------------------------------------------
// rejection sampling
// ---------------------------------------------------------------------------
struct MS {
  float m, s;
};

// The softmax of x / t is evaluated as 2^((x - m) * c) with c = log2(e) / t:
// one fused multiply-add and one ex2 per element. A pair (m, s) holds a
// slice's largest logit m and s = sum 2^((x - m) * c).
__device__ __forceinline__ float ex2(float y) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(y));
  return r;
}

__device__ __forceinline__ MS ms_combine(MS a, MS b, float c) {
  if (a.m == -INFINITY) return b;
  if (b.m == -INFINITY) return a;
  const float m = fmaxf(a.m, b.m);
  return MS{m, a.s * ex2((a.m - m) * c) + b.s * ex2((b.m - m) * c)};
}

// Warp-level (m, s) of a row slice (every lane gets the warp's pair). Two
// passes over the thread's chunks (kBatch loads in flight): the largest logit
// (packed bf16 max, NaN propagating), then the branch-free sum of
// 2^((x - m) * c).
__device__ MS warp_ms(const __nv_bfloat16* __restrict__ row, int lo, int hi, float c) {
  const int nvec = (hi - lo) / 8;
  const uint4* p = reinterpret_cast<const uint4*>(row + lo);
  const int bd = static_cast<int>(blockDim.x);
  __nv_bfloat162 mx2 = __float2bfloat162_rn(-INFINITY);
  for (int i0 = threadIdx.x; i0 < nvec; i0 += kBatch * bd) {
    uint4 q[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u)
      if (i0 + u * bd < nvec) q[u] = __ldcg(p + i0 + u * bd);
#pragma unroll
    for (int u = 0; u < kBatch; ++u)
      if (i0 + u * bd < nvec)
        mx2 = __hmax2_nan(mx2, __hmax2_nan(__hmax2_nan(as_bf162(q[u].x), as_bf162(q[u].y)),
                                           __hmax2_nan(as_bf162(q[u].z), as_bf162(q[u].w))));
  }
  float mx = __bfloat162float(__hmax_nan(mx2.x, mx2.y));
  for (int k = lo + nvec * 8 + threadIdx.x; k < hi; k += bd) {
    const float x = __bfloat162float(row[k]);
    mx = isnan(x) || x > mx ? x : mx;
  }
  MS acc{-INFINITY, 0.f};
  if (mx != -INFINITY) {
    const float mc = mx * c;
    float sum = 0.f;
    for (int i0 = threadIdx.x; i0 < nvec; i0 += kBatch * bd) {
      uint4 q[kBatch];
#pragma unroll
      for (int u = 0; u < kBatch; ++u)
        if (i0 + u * bd < nvec) q[u] = __ldcg(p + i0 + u * bd);
#pragma unroll
      for (int u = 0; u < kBatch; ++u)
        if (i0 + u * bd < nvec) {
          const uint32_t w[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            sum += ex2(fmaf(bf16lo(w[j]), c, -mc));
            sum += ex2(fmaf(bf16hi(w[j]), c, -mc));
          }
        }
    }
    for (int k = lo + nvec * 8 + threadIdx.x; k < hi; k += bd) sum += ex2(fmaf(__bfloat162float(row[k]), c, -mc));
    acc = MS{mx, sum};
  }
  for (int o = 16; o > 0; o >>= 1) {
    MS other{__shfl_xor_sync(0xffffffffu, acc.m, o), __shfl_xor_sync(0xffffffffu, acc.s, o)};
    acc = ms_combine(acc, other, c);
  }
  return acc;
}

struct Bcast {
  int n_acc;
  int row;       // target row sampled from
  int residual;  // 1: max(0, p - q), 0: p
  float mt, ist, md, isd;  // row maxima and 1 / row sums
};

__device__ __forceinline__ float resid_of(float xt, float xd, float c, const Bcast& bc) {
  const float p = ex2((xt - bc.mt) * c) * bc.ist;
  if (!bc.residual) return p;
  const float q = ex2((xd - bc.md) * c) * bc.isd;
  return fmaxf(0.f, p - q);
}

// The sampled distribution at k .. k + 7 (values past `end` are 0): p, or
// max(0, p - q) at a rejection. k is a multiple of 8, so a whole group is
// one 16-byte load of each row.
__device__ __forceinline__ void resid8(const __nv_bfloat16* tr, const __nv_bfloat16* dr, int k, int end, float c,
                                       const Bcast& bc, float (&rv)[8]) {
  if (k + 8 <= end) {
    const uint4 a = __ldcg(reinterpret_cast<const uint4*>(tr + k));
    const uint4 b = bc.residual ? __ldcg(reinterpret_cast<const uint4*>(dr + k)) : make_uint4(0u, 0u, 0u, 0u);
    const uint32_t wa[4] = {a.x, a.y, a.z, a.w}, wb[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      rv[2 * j] = resid_of(bf16lo(wa[j]), bf16lo(wb[j]), c, bc);
      rv[2 * j + 1] = resid_of(bf16hi(wa[j]), bf16hi(wb[j]), c, bc);
    }
    return;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j)
    rv[j] = k + j < end ? resid_of(__bfloat162float(tr[k + j]), bc.residual ? __bfloat162float(dr[k + j]) : 0.f, c, bc)
                        : 0.f;
}

__global__ void __cluster_dims__(kCluster, 1, 1) __launch_bounds__(kThreads)
    rejection_kernel(const __nv_bfloat16* __restrict__ target, const __nv_bfloat16* __restrict__ draft, int M,
                     int draft_rows, int V, const int64_t* __restrict__ draft_ids, const float* __restrict__ u,
                     float t, int32_t* __restrict__ n_acc, int64_t* __restrict__ next_tok, int32_t* status) {
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = static_cast<int>(cluster.block_rank());
  const int b = blockIdx.x / kCluster;
  __shared__ MS tms[kMaxRows], dms[kMaxRows];
  __shared__ float tz[kMaxRows], dz[kMaxRows];  // z at the draft id (if in slice)
  __shared__ Bcast bc;
  __shared__ float csum;  // this CTA's slice mass
  __shared__ int clast;   // last index with positive mass in this slice
  __shared__ float tsum[kThreads];
  __shared__ int found;
  int lo, hi;
  slice_of(V, rank, lo, hi);
  const float c = 1.4426950408889634f / t;  // log2(e) / t
  const __nv_bfloat16* trow0 = target + static_cast<int64_t>(b) * (M + 1) * V;
  const __nv_bfloat16* drow0 = draft + static_cast<int64_t>(b) * draft_rows * V;

  // every row's warp pairs first (target rows 0..M, then draft rows), one
  // barrier, then thread i combines row i over the warps in warp order
  __shared__ MS wms[2 * kMaxRows][kThreads / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = 0; i <= 2 * M; ++i) {
    const __nv_bfloat16* row = i <= M ? trow0 + static_cast<int64_t>(i) * V : drow0 + static_cast<int64_t>(i - M - 1) * V;
    const MS r = warp_ms(row, lo, hi, c);
    if (lane == 0) wms[i][warp] = r;
  }
  __syncthreads();
  if (threadIdx.x <= 2 * M) {
    const int i = threadIdx.x;
    MS acc = wms[i][0];
    for (int w = 1; w < kThreads / 32; ++w) acc = ms_combine(acc, wms[i][w], c);
    if (i <= M)
      tms[i] = acc;
    else
      dms[i - M - 1] = acc;
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < M; ++i) {
      const int64_t d = draft_ids[static_cast<int64_t>(b) * M + i];
      tz[i] = NAN;
      dz[i] = NAN;
      if (d >= lo && d < hi) {
        tz[i] = __bfloat162float(trow0[static_cast<int64_t>(i) * V + d]);
        dz[i] = __bfloat162float(drow0[static_cast<int64_t>(i) * V + d]);
      }
    }
  }
  cluster.sync();
  // rank 0 gathers every rank's row pairs (lane r reads rank r: the remote
  // loads run in parallel), then thread 0 combines them in rank order
  __shared__ MS gT[kCluster][kMaxRows], gD[kCluster][kMaxRows];
  __shared__ float gzt[kCluster][kMaxRows], gzd[kCluster][kMaxRows];
  if (rank == 0 && warp == 0 && lane < kCluster) {
    const MS* rt = cluster.map_shared_rank(tms, lane);
    const MS* rd = cluster.map_shared_rank(dms, lane);
    const float* rtz = cluster.map_shared_rank(tz, lane);
    const float* rdz = cluster.map_shared_rank(dz, lane);
    for (int i = 0; i <= M; ++i) gT[lane][i] = rt[i];
    for (int i = 0; i < M; ++i) {
      gD[lane][i] = rd[i];
      gzt[lane][i] = rtz[i];
      gzd[lane][i] = rdz[i];
    }
  }
  if (rank == 0) __syncwarp();
  if (rank == 0 && threadIdx.x == 0) {
    MS T_[kMaxRows], D_[kMaxRows];
    float zt[kMaxRows], zd[kMaxRows];
    for (int i = 0; i <= M; ++i) {
      T_[i] = MS{-INFINITY, 0.f};
      D_[i] = MS{-INFINITY, 0.f};
      zt[i] = NAN;
      zd[i] = NAN;
    }
    for (int r = 0; r < kCluster; ++r) {
      for (int i = 0; i <= M; ++i) T_[i] = ms_combine(T_[i], gT[r][i], c);
      for (int i = 0; i < M; ++i) {
        D_[i] = ms_combine(D_[i], gD[r][i], c);
        if (!isnan(gzt[r][i])) {
          zt[i] = gzt[r][i];
          zd[i] = gzd[r][i];
        }
      }
    }
    int n = 0;
    for (; n < M; ++n) {
      const int64_t d = draft_ids[static_cast<int64_t>(b) * M + n];
      if (d < 0 || d >= V) {
        report(status, HS_DEV_BAD_DRAFT);
        break;
      }
      const float p = ex2((zt[n] - T_[n].m) * c) / T_[n].s;
      const float q = ex2((zd[n] - D_[n].m) * c) / D_[n].s;
      const float uu = u[static_cast<int64_t>(b) * (M + 1) + n];
      if (!(uu < p / q)) break;
    }
    bc.n_acc = n;
    bc.row = n;
    bc.residual = n < M ? 1 : 0;
    bc.mt = T_[n].m;
    bc.ist = 1.f / T_[n].s;
    bc.md = n < M ? D_[n].m : 0.f;
    bc.isd = n < M ? 1.f / D_[n].s : 1.f;
  }
  cluster.sync();
  const Bcast B = *cluster.map_shared_rank(&bc, 0);
  const __nv_bfloat16* tr = trow0 + static_cast<int64_t>(B.row) * V;
  const __nv_bfloat16* dr = drow0 + static_cast<int64_t>(B.row < draft_rows ? B.row : 0) * V;
  // Thread i owns one contiguous chunk of the slice; chunk sums are combined
  // by thread 0 in thread order, so the CTA total and the exclusive prefixes
  // come from the same sequence of additions.
  // (chunks are a multiple of 8 values, so each starts 16-byte aligned and is
  // read with vector loads)
  const int len = hi - lo;
  const int chunk = (len + 8 * static_cast<int>(blockDim.x) - 1) / (8 * static_cast<int>(blockDim.x)) * 8;
  const int k0 = min(hi, lo + static_cast<int>(threadIdx.x) * chunk), k1 = min(hi, k0 + chunk);
  float ts = 0.f;
  int tl = -1;
  for (int k = k0; k < k1; k += 8) {
    float rv[8];
    resid8(tr, dr, k, k1, c, B, rv);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      ts += rv[j];
      if (rv[j] > 0.f) tl = k + j;
    }
  }
  tsum[threadIdx.x] = ts;
  for (int o = 16; o > 0; o >>= 1) tl = max(tl, __shfl_xor_sync(0xffffffffu, tl, o));
  __shared__ int wl[kThreads / 32];
  if ((threadIdx.x & 31) == 0) wl[threadIdx.x >> 5] = tl;
  __syncthreads();
  if (threadIdx.x == 0) {
    float x = 0.f;
    for (int i = 0; i < static_cast<int>(blockDim.x); ++i) {
      const float y = tsum[i];
      tsum[i] = x;  // exclusive prefix within the CTA
      x += y;
    }
    csum = x;
    int m = -1;
    for (int i = 0; i < static_cast<int>(blockDim.x / 32); ++i) m = max(m, wl[i]);
    clast = m;
    found = 0x7fffffff;
  }
  cluster.sync();
  // every rank's slice mass and last positive index, read once per CTA (lane
  // r of warp 0 reads rank r), then the prefix over the cluster in rank order
  __shared__ float rsum[kCluster];
  __shared__ int rlast[kCluster];
  if (warp == 0 && lane < kCluster) {
    rsum[lane] = *cluster.map_shared_rank(&csum, lane);
    rlast[lane] = *cluster.map_shared_rank(&clast, lane);
  }
  __syncthreads();
  float pre = 0.f, tot = 0.f;
  int last = -1;
  for (int r = 0; r < kCluster; ++r) {
    const float s = rsum[r];
    if (r < rank) pre += s;
    tot += s;
    last = max(last, rlast[r]);
  }
  const float tau = u[static_cast<int64_t>(b) * (M + 1) + M] * tot;
  if (tau >= pre && tau < pre + csum) {
    float x = pre + tsum[threadIdx.x];
    bool done = false;
    for (int k = k0; k < k1 && !done; k += 8) {
      float rv[8];
      resid8(tr, dr, k, k1, c, B, rv);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        x += rv[j];
        if (!done && rv[j] > 0.f && x > tau) {
          atomicMin(&found, k + j);
          done = true;
        }
      }
    }
  }
  cluster.sync();
  if (rank == 0 && warp == 0) {
    int best = lane < kCluster ? *cluster.map_shared_rank(&found, lane) : 0x7fffffff;
    best = __reduce_min_sync(0xffffffffu, best);
    if (lane == 0) {
      next_tok[b] = best != 0x7fffffff ? best : (last >= 0 ? last : 0);
      n_acc[b] = B.n_acc;
    }
  }
  cluster.sync();
}

}  // namespace accept
}  // namespace hs

using namespace hs;
using namespace hs::accept;

extern "C" int hs_accept_greedy(const void* logits, int64_t B, int64_t T, int64_t V, const int64_t* draft_ids,
                                int32_t* n_accept, int64_t* next_token, int64_t* argmax_out, int32_t* dev_status,
                                void* stream) {
  (void)dev_status;
  if (B < 0 || T < 1 || T > kMaxRows || V < 64 || (V * 2) % 16 != 0) return HS_ERR_BAD_SHAPE;
  if (B == 0) return HS_OK;
  if (B * kCluster > 0x7fffffff) return HS_ERR_BAD_SHAPE;
  if (!logits || !n_accept || !next_token || (T > 1 && !draft_ids)) return HS_ERR_BAD_ARGUMENT;
  if (!aligned16(logits)) return HS_ERR_ALIGN;
  greedy_kernel<<<static_cast<unsigned>(B * kCluster), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(logits), static_cast<int>(T), static_cast<int>(V), draft_ids, n_accept,
      next_token, argmax_out);
  return check_launch();
}

extern "C" int hs_accept_rejection(const void* target_logits, const void* draft_logits, int64_t B, int64_t M,
                                   int64_t draft_rows, int64_t V, const int64_t* draft_ids, const float* uniform,
                                   float temperature, int32_t* n_accept, int64_t* next_token, int32_t* dev_status,
                                   void* stream) {
  if (B < 0 || M < 0 || M + 1 > kMaxRows || draft_rows < M || V < 64 || (V * 2) % 16 != 0) return HS_ERR_BAD_SHAPE;
  if (B == 0) return HS_OK;
  if (!target_logits || !n_accept || !next_token || (M > 0 && (!draft_logits || !draft_ids)))
    return HS_ERR_BAD_ARGUMENT;
  if (!(temperature > 0.f))
    return hs_accept_greedy(target_logits, B, M + 1, V, draft_ids, n_accept, next_token, nullptr, dev_status, stream);
  if (!uniform) return HS_ERR_BAD_ARGUMENT;
  if (!aligned16(target_logits) || (draft_logits && !aligned16(draft_logits))) return HS_ERR_ALIGN;
  rejection_kernel<<<static_cast<unsigned>(B * kCluster), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(target_logits), static_cast<const __nv_bfloat16*>(draft_logits),
      static_cast<int>(M), static_cast<int>(draft_rows), static_cast<int>(V), draft_ids, uniform, temperature,
      n_accept, next_token, dev_status);
  return check_launch();
}
