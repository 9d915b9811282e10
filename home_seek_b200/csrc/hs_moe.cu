// Routed FP4 expert FFN + fused FP8 shared expert on the 5th-generation tensor
// cores (tcgen05, TMEM accumulators, TMA), sm_100a.
//
// Reference being replaced: FusedMoEFFN._forward_legacy
// (home_seek/fused_moe.py:458-551), which dequantises every touched expert to
// BF16 (fused_moe.py:672-735), concatenates the weights (fused_moe.py:515-517)
// and runs three cuBLAS GEMMs; SharedExpertFFN.forward + fused_expert_ffn_pt
// (fused_moe.py:383-392, 573-598) for the shared expert; and the bf16 add of
// the two at inference_engine/engine.py:1530-1536.
//
// Design (B200-first):
//   * Weights never pass through registers. TMA loads 128x128 tiles of packed
//     e2m1 straight into 128B-swizzled shared memory (data type 16U4_ALIGN16B,
//     the layout kind::mxf8f6f4 reads), the UE8M0 scales (stored by the expert
//     store in the tcgen05 scale-factor atom layout, 512 B per 128 rows x 128
//     columns) go to TMEM with one tcgen05.cp, and tcgen05.mma.kind::mxf8f6f4
//     .block_scale multiplies them with the activations, accumulating f32 in
//     TMEM. The FP8 shared expert runs through the same MMA with E4M3 weights.
//   * Activations are bf16 in the reference. Each bf16 value v (8 significant
//     bits) is split into two e4m3 values hi = e4m3(v * 2^e), lo = e4m3(v * 2^e
//     - hi) that sum back to v * 2^e exactly (down to 2^-9 of the row maximum
//     scaled to [128, 256)); the power-of-two prescale 2^e is undone by the
//     MMA's B scale factor. The N dimension of one MMA carries the hi and lo
//     rows of up to 8*NT tokens, so every weight is read once.
//   * plan    one CTA builds the expert-major pair list (deterministic counting
//             sort); T more CTAs convert their token's row to the hi/lo pair
//             rows (one per (token, expert) pair and one for the shared expert).
//   * gateup  one CTA per (chunk of <= 8*NT pairs of one expert, 128 rows of
//             I): warp 4 issues TMA, warp 5 issues tcgen05.cp + tcgen05.mma,
//             warps 0-3 read the TMEM accumulators (gate and up), apply the
//             reference's roundings and SwiGLU, multiply by the bf16 routing
//             weight and write the activation as hi/lo e4m3 rows.
//   * down    one CTA per (chunk, 128 rows of D): same pipeline over w2; the
//             f32 partial rows are reduced per token in ascending expert order
//             by the last CTA to finish each 128-row slice of D (a ticket on a
//             counter; no CTA waits for another), rounded once to bf16 and
//             added to the bf16 shared-expert output.
#include <algorithm>
#include <atomic>
#include <mutex>

#include <cuda_fp8.h>

#include "hs_common.cuh"
#include "hs_tcgen05.cuh"

namespace hs {
namespace moe {

constexpr int kM = 128;                 // weight rows per unit (UMMA M)
constexpr int kBoxBytes = kM * 128;     // one 128x128 weight tile in shared memory
constexpr int kStages = 3;
constexpr int kThreads = 192;           // warps 0-3 epilogue, warp 4 TMA, warp 5 MMA
constexpr int kTmemCols = 256;
constexpr int kAccUp = 64;              // TMEM column of the up accumulator
constexpr int kSfaCol = 128;            // 8 columns per stage (2 boxes x 4)
constexpr int kSfbCol = 192;
constexpr int kMaxNT = 3;               // n-tiles of 8 pairs (N = 16 * NT)
constexpr int kPlanThreads = 512;
constexpr int kLocalPairs = 4096;       // T*K up to this: token CTAs place their own rows
constexpr uint32_t kDescMagic = 0x48534d32u;  // "HSM2"

struct __align__(64) Desc {
  CUtensorMap tm_w13;   // e2m1 [E*2*I rows][D], 16U4_ALIGN16B, box 128 x 128, swizzle 128B
  CUtensorMap tm_w2;    // e2m1 [E*D rows][I]
  CUtensorMap tm_sw13;  // e4m3 [2*I_sh rows][D], uint8, box 128 x 128
  CUtensorMap tm_sw2;   // e4m3 [D rows][I_sh]
  const uint8_t* s13a;  // [E][2][I/128][D/128][512] scale-factor atoms
  const uint8_t* s2a;   // [E][D/128][I/128][512]
  const uint8_t* sh_s13a;  // [2][I_sh/128][D/128][512]
  const uint8_t* sh_s2a;   // [D/128][I_sh/128][512]
  int32_t E, D, I, I_sh;
  int32_t has_shared;
  uint32_t magic;
};
static_assert(sizeof(Desc) <= HS_MOE_DESC_BYTES, "descriptor blob too small");

struct CallMaps {
  CUtensorMap tm_x8;    // [2*P_max rows][D] e4m3 hi rows then lo rows, box 128 x 8
  CUtensorMap tm_act8;  // [2*P_max rows][I_act]
};

// Device views into the caller's workspace.
struct Plan {
  int32_t* hdr;           // [0] routed chunks, [1] slots, [2] routed pairs
  int32_t* chunk_expert;  // [C_max]
  int32_t* chunk_pair0;   // [C_max] first pair index (global)
  int32_t* chunk_np;      // [C_max]
  int32_t* pair_token;    // [P_max]
  float* pair_wb;         // [P_max] bf16-rounded routing weight
  int32_t* pair_q;        // [P_max] power-of-two prescale of the activation
  uint8_t* sb1;           // [P_max] UE8M0 B scale of the gate/up MMA (undoes 2^e)
  uint8_t* sb2;           // [P_max] UE8M0 B scale of the down MMA (undoes 2^q)
  int32_t* tok_e;         // [T] power-of-two prescale of the hidden row
  int32_t* tok_pos;       // [T][K] ascending routed pair positions, -1 padded
  uint32_t* dcount;       // [D/128] finalize tickets, reset by the plan kernel
  uint8_t* x8;            // [2][P_max][D] e4m3 hi / lo
  uint8_t* act8;          // [2][P_max][I_act] e4m3 hi / lo
  float* out_part;        // [P_max][D]
};

struct Geometry {
  int64_t T, K, D, I, I_sh, I_act, P_max, C_max;
  size_t off_hdr, off_chunk, off_pair, off_sb, off_tok, off_tokpos, off_dcount, off_x8, off_act8, off_out, total;
};

static size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

static int64_t ntiles(int64_t T) {
  int64_t nt = (T + 7) / 8;
  return std::max<int64_t>(1, std::min<int64_t>(nt, kMaxNT));
}

static Geometry geometry(int64_t T, int64_t K, int64_t D, int64_t I, int64_t I_sh) {
  Geometry g{};
  g.T = T;
  g.K = K;
  g.D = D;
  g.I = I;
  g.I_sh = I_sh;
  g.I_act = std::max(I, I_sh);
  const int64_t CH = 8 * ntiles(T);
  const int64_t Pr = T * K;
  g.P_max = T + Pr;
  g.C_max = Pr / CH + std::min<int64_t>(Pr, 1024) + 1;
  size_t o = 0;
  g.off_hdr = o;
  o = align_up(o + 16 * sizeof(int32_t), 256);
  g.off_chunk = o;
  o = align_up(o + 3 * g.C_max * sizeof(int32_t), 256);
  g.off_pair = o;
  o = align_up(o + 3 * g.P_max * sizeof(int32_t), 256);
  g.off_sb = o;
  o = align_up(o + 2 * g.P_max, 256);
  g.off_tok = o;
  o = align_up(o + T * sizeof(int32_t), 256);
  g.off_tokpos = o;
  o = align_up(o + T * K * sizeof(int32_t), 256);
  g.off_dcount = o;
  o = align_up(o + (D / kM + 1) * sizeof(uint32_t), 256);
  g.off_x8 = o;
  o = align_up(o + 2 * g.P_max * D, 256);
  g.off_act8 = o;
  o = align_up(o + 2 * g.P_max * g.I_act, 256);
  g.off_out = o;
  o = align_up(o + g.P_max * D * sizeof(float), 256);
  g.total = o;
  return g;
}

static Plan plan_views(const Geometry& g, void* ws) {
  uint8_t* b = static_cast<uint8_t*>(ws);
  Plan p;
  p.hdr = reinterpret_cast<int32_t*>(b + g.off_hdr);
  p.chunk_expert = reinterpret_cast<int32_t*>(b + g.off_chunk);
  p.chunk_pair0 = p.chunk_expert + g.C_max;
  p.chunk_np = p.chunk_pair0 + g.C_max;
  p.pair_token = reinterpret_cast<int32_t*>(b + g.off_pair);
  p.pair_wb = reinterpret_cast<float*>(p.pair_token + g.P_max);
  p.pair_q = reinterpret_cast<int32_t*>(p.pair_wb + g.P_max);
  p.sb1 = b + g.off_sb;
  p.sb2 = p.sb1 + g.P_max;
  p.tok_e = reinterpret_cast<int32_t*>(b + g.off_tok);
  p.tok_pos = reinterpret_cast<int32_t*>(b + g.off_tokpos);
  p.dcount = reinterpret_cast<uint32_t*>(b + g.off_dcount);
  p.x8 = b + g.off_x8;
  p.act8 = b + g.off_act8;
  p.out_part = reinterpret_cast<float*>(b + g.off_out);
  return p;
}

// ---------------------------------------------------------------------------
// plan kernel
// ---------------------------------------------------------------------------
// Internal duplicate mode for the standalone permute: every valid (t, j) gets
// its own position.
constexpr int kDupKeepAll = 2;
constexpr int32_t kBadId = 0x7fffffff;  // expert id >= E (skipped and reported)

struct PermuteOut {
  int32_t* pos_to_expert;  // [T*K] or nullptr
  int32_t* expert_count;   // [E] or nullptr
  int32_t* num_pos;        // [1] or nullptr
};

struct PlanArgs {
  const int64_t* topk_idx;
  const float* topk_w;
  const __nv_bfloat16* hidden;  // nullptr for the standalone permute
  int T, K, E, D, CH, dup_mode, pos_offset, sort_tok, n_dcount;
  int64_t P_max;
  int local_rows;  // token CTAs write their routed pair rows themselves
  PermuteOut po;
  int32_t* status;
};

// Power-of-two prescale for an activation aw = bf16(a * wb), |a| <= 100:
// |aw| * 2^q <= 256 so the e4m3 split never saturates.
__device__ __forceinline__ int act_prescale(float wb) {
  const float m = fabsf(wb);
  if (!(m > 0.f) || !isfinite(m)) return 0;
  int ex;
  frexpf(m, &ex);
  return max(-100, min(100, 1 - ex));
}

__device__ __forceinline__ int32_t clamp_id(int64_t v, int E) {
  return v < 0 ? -1 : (v >= E ? kBadId : static_cast<int32_t>(v));
}

// Expert of pair l = t*K + j after the duplicate rule, or -1; *wsum receives
// the weight the pair carries. `row` is token t's K ids (clamped). Every CTA
// evaluates the same function, so positions computed anywhere agree.
__device__ __forceinline__ int pair_expert(const int32_t* row, const float* wrow, int j, int K, int dup_mode,
                                           float* wsum) {
  const int e = row[j];
  if (e < 0 || e == kBadId) return -1;
  if (dup_mode == kDupKeepAll) {
    if (wsum) *wsum = wrow ? wrow[j] : 1.f;
  } else if (dup_mode == HS_DUP_SUM) {
    for (int jj = 0; jj < j; ++jj)
      if (row[jj] == e) return -1;
    float s = 0.f;
    for (int jj = j; jj < K; ++jj)
      if (row[jj] == e) s += wrow ? wrow[jj] : 1.f;
    if (wsum) *wsum = s;
  } else {
    for (int jj = j + 1; jj < K; ++jj)
      if (row[jj] == e) return -1;
    if (wsum) *wsum = wrow ? wrow[j] : 1.f;
  }
  return e;
}

// hi/lo e4m3 split of 16 consecutive bf16 values scaled by 2^e.
__device__ __forceinline__ void split16(const __nv_bfloat16* src, float sc, uint4& hi, uint4& lo) {
  const uint4 a = reinterpret_cast<const uint4*>(src)[0];
  const uint4 b = reinterpret_cast<const uint4*>(src)[1];
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  uint32_t h[4] = {0, 0, 0, 0}, l[4] = {0, 0, 0, 0};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float v0 = __uint_as_float(w[i] << 16) * sc;
    const float v1 = __uint_as_float(w[i] & 0xffff0000u) * sc;
    const __nv_fp8x2_storage_t hp = __nv_cvt_float2_to_fp8x2(make_float2(v0, v1), __NV_SATFINITE, __NV_E4M3);
    const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(hp, __NV_E4M3);
    const float2 hf = __half22float2(*reinterpret_cast<const __half2*>(&hr));
    const __nv_fp8x2_storage_t lp =
        __nv_cvt_float2_to_fp8x2(make_float2(v0 - hf.x, v1 - hf.y), __NV_SATFINITE, __NV_E4M3);
    h[i >> 1] |= static_cast<uint32_t>(hp) << (16 * (i & 1));
    l[i >> 1] |= static_cast<uint32_t>(lp) << (16 * (i & 1));
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// Block 0 builds the routing plan; blocks 1..T (MoE call only) convert one
// token row each into its shared-expert row and, when local_rows is set, its
// routed pair rows (positions recomputed locally from the same counts).
__global__ void __launch_bounds__(kPlanThreads) plan_kernel(PlanArgs A, Plan P) {
  extern __shared__ int32_t sm[];
  const int tid = threadIdx.x;
  const int T = A.T, K = A.K, E = A.E;
  const int npairs = T * K;
  const bool cache_idx = npairs <= kLocalPairs;
  int32_t* sidx = sm;  // [npairs] clamped ids (when cached)
  int32_t* rest = sm + (cache_idx ? npairs : 0);
  if (cache_idx) {
    for (int l = tid; l < npairs; l += blockDim.x) sidx[l] = clamp_id(A.topk_idx[l], E);
    __syncthreads();
  }

  if (blockIdx.x > 0) {
    // ---- token row: prescale, hi/lo split, rows for its pairs ----
    const int t = blockIdx.x - 1;
    const __nv_bfloat16* h = A.hidden + static_cast<int64_t>(t) * A.D;
    float mx = 0.f;
    for (int k = tid; k < A.D; k += blockDim.x) mx = fmaxf(mx, fabsf(__bfloat162float(h[k])));
    __shared__ float red[kPlanThreads / 32];
    __shared__ int rows[17];
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((tid & 31) == 0) red[tid >> 5] = mx;
    int nrows = 1;
    if (A.local_rows && cache_idx) {
      nrows = 1 + K;
      if (tid < 32) {
        // warp 0: for each of my K entries count the valid pairs with a smaller
        // expert (its expert's base) and with the same expert on an earlier
        // token (its rank): the position block 0 assigns.
        for (int j = 0; j < K; ++j) {
          const int e = pair_expert(sidx + t * K, nullptr, j, K, A.dup_mode, nullptr);
          int base = 0, rank = 0;
          if (e >= 0) {
            for (int m = tid; m < npairs; m += 32) {
              const int tm = m / K;
              const int e2 = pair_expert(sidx + tm * K, nullptr, m - tm * K, K, A.dup_mode, nullptr);
              if (e2 < 0) continue;
              base += e2 < e;
              rank += (e2 == e) && (tm < t);
            }
          }
          for (int o = 16; o > 0; o >>= 1) {
            base += __shfl_xor_sync(0xffffffffu, base, o);
            rank += __shfl_xor_sync(0xffffffffu, rank, o);
          }
          if (tid == 0) rows[1 + j] = e >= 0 ? A.pos_offset + base + rank : -1;
        }
      }
    }
    __syncthreads();
    if (tid == 0) {
      float v = 0.f;
      for (int i = 0; i < static_cast<int>(blockDim.x / 32); ++i) v = fmaxf(v, red[i]);
      int e = 0;
      if (v > 0.f && isfinite(v)) {
        int ex;
        frexpf(v, &ex);
        e = max(-100, min(100, 8 - ex));
      }
      P.tok_e[t] = e;
      red[0] = static_cast<float>(e);
      rows[0] = t;  // shared-expert row
    }
    __syncthreads();
    const int e = static_cast<int>(red[0]);
    const float sc = exp2i(e);
    uint8_t* hi_plane = P.x8;
    uint8_t* lo_plane = P.x8 + A.P_max * A.D;
    for (int k16 = tid; k16 < A.D / 16; k16 += blockDim.x) {
      uint4 hv, lv;
      split16(h + 16 * k16, sc, hv, lv);
      for (int r = 0; r < nrows; ++r) {
        const int p = rows[r];
        if (p < 0) continue;
        reinterpret_cast<uint4*>(hi_plane + static_cast<int64_t>(p) * A.D)[k16] = hv;
        reinterpret_cast<uint4*>(lo_plane + static_cast<int64_t>(p) * A.D)[k16] = lv;
      }
    }
    if (tid < nrows && rows[tid] >= 0) P.sb1[rows[tid]] = static_cast<uint8_t>(127 - e);
    return;
  }

  // ---- routing plan (block 0) ----
  int32_t* hist = rest;              // [E]
  int32_t* base = hist + E;          // [E+1]
  int32_t* cursor = base + E + 1;    // [E]
  int32_t* cbase = cursor + E;       // [E+1]
  int32_t* wcnt = cbase + E + 1;     // [nwarps][E]
  const int nwarps = blockDim.x / 32;
  const int warp = tid >> 5, lane = tid & 31;

  // expert of pair l (ids from shared memory when cached, else global)
  auto expert_of = [&](int l, float* wsum) -> int {
    const int t = l / K, j = l - t * K;
    const float* wrow = A.topk_w ? A.topk_w + static_cast<int64_t>(t) * K : nullptr;
    int32_t rowbuf[16];
    const int32_t* row;
    if (cache_idx) {
      row = sidx + t * K;
    } else {
      for (int jj = 0; jj < K; ++jj) rowbuf[jj] = clamp_id(A.topk_idx[static_cast<int64_t>(t) * K + jj], E);
      row = rowbuf;
    }
    if (row[j] == kBadId) report(A.status, HS_DEV_BAD_EXPERT);
    return pair_expert(row, wrow, j, K, A.dup_mode, wsum);
  };

  for (int e = tid; e < E; e += blockDim.x) {
    hist[e] = 0;
    cursor[e] = 0;
  }
  for (int i = tid; i < A.n_dcount; i += blockDim.x) P.dcount[i] = 0u;
  __syncthreads();
  for (int l = tid; l < npairs; l += blockDim.x) {
    const int e = expert_of(l, nullptr);
    if (e >= 0) atomicAdd(&hist[e], 1);
  }
  __syncthreads();
  if (warp == 0) {
    int run = 0, crun = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int e = e0 + lane;
      const int hh = e < E ? hist[e] : 0;
      const int c = (hh + A.CH - 1) / A.CH;
      int x = hh, y = c;
      for (int o = 1; o < 32; o <<= 1) {
        const int xv = __shfl_up_sync(0xffffffffu, x, o);
        const int yv = __shfl_up_sync(0xffffffffu, y, o);
        if (lane >= o) {
          x += xv;
          y += yv;
        }
      }
      if (e < E) {
        base[e] = run + x - hh;
        cbase[e] = crun + y - c;
      }
      run += __shfl_sync(0xffffffffu, x, 31);
      crun += __shfl_sync(0xffffffffu, y, 31);
    }
    if (lane == 0) {
      base[E] = run;
      cbase[E] = crun;
    }
  }
  __syncthreads();
  int my_slots = 0;
  for (int e = tid; e < E; e += blockDim.x) {
    const int hh = hist[e];
    my_slots += hh > 0;
    int cb = cbase[e];
    for (int c = 0; c * A.CH < hh; ++c, ++cb) {
      P.chunk_expert[cb] = e;
      P.chunk_pair0[cb] = A.pos_offset + base[e] + c * A.CH;
      P.chunk_np[cb] = min(A.CH, hh - c * A.CH);
    }
  }
  for (int o = 16; o > 0; o >>= 1) my_slots += __shfl_xor_sync(0xffffffffu, my_slots, o);
  if (lane == 0) wcnt[warp] = my_slots;
  __syncthreads();
  if (tid == 0) {
    int slots = 0;
    for (int w = 0; w < nwarps; ++w) slots += wcnt[w];
    P.hdr[0] = cbase[E];
    P.hdr[1] = slots;
    P.hdr[2] = base[E];
    if (A.po.num_pos) *A.po.num_pos = base[E];
  }
  __syncthreads();
  if (A.po.expert_count)
    for (int e = tid; e < E; e += blockDim.x) A.po.expert_count[e] = hist[e];
  if (A.po.pos_to_expert)
    for (int p = base[E] + tid; p < npairs; p += blockDim.x) A.po.pos_to_expert[p] = -1;
  for (int t = tid; t < A.pos_offset; t += blockDim.x) {  // shared-expert pairs
    P.pair_token[t] = t;
    P.pair_wb[t] = 1.f;
    P.pair_q[t] = 0;
    P.sb2[t] = 127;
  }
  // stable positions, tile by tile (warp-major = pair order)
  const int tile = blockDim.x;
  for (int l0 = 0; l0 < npairs; l0 += tile) {
    const int l = l0 + tid;
    float wsum = 0.f;
    const int e = l < npairs ? expert_of(l, &wsum) : -1;
    const unsigned msk = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(msk & ((1u << lane) - 1u));
    for (int x = lane; x < E; x += 32) wcnt[warp * E + x] = 0;
    __syncwarp();
    if (e >= 0 && rank == 0) wcnt[warp * E + e] = __popc(msk);
    __syncthreads();
    for (int x = tid; x < E; x += blockDim.x) {
      int run = cursor[x];
      for (int w = 0; w < nwarps; ++w) {
        const int c = wcnt[w * E + x];
        wcnt[w * E + x] = run;
        run += c;
      }
      cursor[x] = run;
    }
    __syncthreads();
    if (l < npairs) {
      const int t = l / K;
      int pos = -1;
      if (e >= 0) {
        pos = A.pos_offset + base[e] + wcnt[warp * E + e] + rank;
        const float wb = round_bf16(wsum);
        const int q = act_prescale(wb);
        P.pair_token[pos] = t;
        P.pair_wb[pos] = wb;
        P.pair_q[pos] = q;
        P.sb2[pos] = static_cast<uint8_t>(127 - q);
        if (A.po.pos_to_expert) A.po.pos_to_expert[pos] = e;
      }
      P.tok_pos[l] = pos;
    }
    __syncthreads();
  }
  if (!A.sort_tok) return;
  for (int t = tid; t < T; t += blockDim.x) {
    int32_t* row = P.tok_pos + static_cast<int64_t>(t) * K;
    for (int a = 1; a < K; ++a) {
      const int v = row[a];
      const uint32_t kv = static_cast<uint32_t>(v);  // -1 sorts last
      int b = a - 1;
      while (b >= 0 && static_cast<uint32_t>(row[b]) > kv) {
        row[b + 1] = row[b];
        --b;
      }
      row[b + 1] = v;
    }
  }
}

// Routed pair rows when T*K is too large for per-token position recomputation:
// one CTA per routed pair copies its token's hi/lo rows (written by the plan).
__global__ void __launch_bounds__(256) gather_kernel(Plan P, int T, int64_t P_max, int D) {
  const int64_t p = T + static_cast<int64_t>(blockIdx.x);
  if (p >= T + P.hdr[2]) return;
  const int t = P.pair_token[p];
  const uint4* hs = reinterpret_cast<const uint4*>(P.x8 + static_cast<int64_t>(t) * D);
  const uint4* ls = reinterpret_cast<const uint4*>(P.x8 + (P_max + t) * D);
  uint4* hd = reinterpret_cast<uint4*>(P.x8 + p * D);
  uint4* ld = reinterpret_cast<uint4*>(P.x8 + (P_max + p) * D);
  for (int i = threadIdx.x; i < D / 16; i += blockDim.x) {
    hd[i] = hs[i];
    ld[i] = ls[i];
  }
  if (threadIdx.x == 0) P.sb1[p] = P.sb1[t];
}

// ---------------------------------------------------------------------------
// tcgen05 units
// ---------------------------------------------------------------------------
struct UnitArgs {
  Plan P;
  int T, K, CH;
  int64_t P_max;
  int n_sh_chunks;  // shared-expert chunks (0 when the shared expert is off)
  int use_shared;
  __nv_bfloat16* out;
  float* out_f32;
  int32_t* status;
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~static_cast<uintptr_t>(1023));
}

template <int NT, int BOXES>
struct SmemLayout {
  static constexpr int kA = 2 * kBoxBytes;             // two weight boxes per stage
  static constexpr int kB = BOXES * 2 * NT * 1024;     // hi and lo atoms per k-box
  static constexpr int kSF = 2 * 512;                  // two scale atoms per stage
  static constexpr int kStage = kA + kB + kSF;
  // three stages when two CTAs still fit on an SM (2 x 113 KB), else two
  static constexpr int kNumStages = (1024 + kStages * kStage + 768 <= 113 * 1024) ? kStages : 2;
  static constexpr int kBytes = 1024 + kNumStages * kStage + 512 + 256;
};

struct Bars {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t accum;
  uint32_t tmem;
  int32_t last;
};

// out[t][tile rows] = bf16( bf16(sum of the token's routed partial rows in
// ascending expert order) + bf16(shared-expert row) ), for every token.
__device__ __noinline__ void finalize_tile(const UnitArgs& a, int D, int tile) {
  for (int i = threadIdx.x; i < a.T * kM; i += blockDim.x) {
    const int t = i / kM;
    const int dd = tile * kM + (i - t * kM);
    const int32_t* pos = a.P.tok_pos + static_cast<int64_t>(t) * a.K;
    float r = 0.f;
    for (int j = 0; j < a.K; ++j) {
      const int p = pos[j];
      if (p < 0) break;
      r += __ldcg(a.P.out_part + static_cast<int64_t>(p) * D + dd);
    }
    if (a.out_f32) a.out_f32[static_cast<int64_t>(t) * D + dd] = r;
    float o = round_bf16(r);
    if (a.use_shared) o += round_bf16(__ldcg(a.P.out_part + static_cast<int64_t>(t) * D + dd));
    a.out[static_cast<int64_t>(t) * D + dd] = __float2bfloat16_rn(o);
  }
}

// One unit on the tensor cores. kDown = false: gate/up (A boxes = w1 and w3,
// one 128-column k-box per stage); kDown = true: down (A boxes = two k-boxes
// of w2). kFP8 selects the shared expert's E4M3 weights.
template <bool kDown, bool kFP8, int NT>
__device__ __forceinline__ void run_unit(const Desc& d, const CallMaps& cm, const UnitArgs& a, int e, int pair0,
                                         int np, int tile) {
  constexpr int BOXES = kDown ? 2 : 1;
  using L = SmemLayout<NT, BOXES>;
  constexpr int S_ = L::kNumStages;
  constexpr int N = 16 * NT;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = align1024(smem_raw);
  uint8_t* stages = base;
  uint8_t* sfb = base + S_ * L::kStage;
  Bars* bars = reinterpret_cast<Bars*>(sfb + 512);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D = d.D;
  const int Iu = kFP8 ? d.I_sh : d.I;
  const int nk = kDown ? Iu / 256 : D / 128;
  const uint32_t tx_box = kFP8 ? kBoxBytes : kBoxBytes / 2;  // packed e2m1 counts half
  const uint32_t tx = 2 * tx_box + L::kB + L::kSF;
  const uint8_t* sbv = kDown ? a.P.sb2 : a.P.sb1;

  // ---- setup: barriers, TMEM, B scale factors ----
  if (threadIdx.x == 0) {
    for (int i = 0; i < S_; ++i) {
      mbar_init(&bars->full[i], 1);
      mbar_init(&bars->empty[i], 1);
    }
    mbar_init(&bars->accum, 1);
    bars->last = 0;
    fence_mbar_init();
  }
  if (warp == 0) tc5::tmem_alloc(&bars->tmem, kTmemCols);
  if (threadIdx.x < 128) {
    // SFB atom: word (m0, m1) = scale of B row n = m0 + 32*m1 in all 4 k-blocks
    const int m0 = threadIdx.x >> 2, m1 = threadIdx.x & 3;
    const int n = m0 + 32 * m1;
    uint32_t b = 127u;
    if (n < N) {
      const int r = n % (8 * NT);
      if (r < np) b = sbv[pair0 + r];
    }
    *reinterpret_cast<uint32_t*>(sfb + m0 * 16 + m1 * 4) = b * 0x01010101u;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  tc5::fence_before_sync();
  __syncthreads();
  tc5::fence_after_sync();
  const uint32_t tmem = bars->tmem;

  if (warp == 4) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      const CUtensorMap* wm = kDown ? (kFP8 ? &d.tm_sw2 : &d.tm_w2) : (kFP8 ? &d.tm_sw13 : &d.tm_w13);
      const CUtensorMap* bm = kDown ? &cm.tm_act8 : &cm.tm_x8;
      int ya = 0, yb = 0;
      if (!kDown) {
        ya = kFP8 ? tile * kM : (2 * e) * d.I + tile * kM;
        yb = kFP8 ? d.I_sh + tile * kM : (2 * e + 1) * d.I + tile * kM;
      } else {
        ya = yb = kFP8 ? tile * kM : e * D + tile * kM;
      }
      for (int kc = 0; kc < nk; ++kc) {
        const int st = kc % S_;
        if (kc >= S_ && !mbar_wait(&bars->empty[st], ((kc / S_) - 1) & 1)) {
          report(a.status, HS_DEV_TIMEOUT);
          break;
        }
        uint8_t* S = stages + st * L::kStage;
        uint8_t* Bs = S + L::kA;
        uint8_t* SF = Bs + L::kB;
        mbar_arrive_expect_tx(&bars->full[st], tx);
        const int xa = kDown ? kc * 256 : kc * 128;
        tma_load_2d(S, wm, &bars->full[st], xa, ya);
        tma_load_2d(S + kBoxBytes, wm, &bars->full[st], kDown ? xa + 128 : xa, yb);
        for (int b = 0; b < BOXES; ++b)
          for (int pl = 0; pl < 2; ++pl)
            for (int nt = 0; nt < NT; ++nt)
              tma_load_2d(Bs + ((b * 2 + pl) * NT + nt) * 1024, bm, &bars->full[st], xa + b * 128,
                          static_cast<int>(pl * a.P_max) + pair0 + 8 * nt);
        for (int i = 0; i < 2; ++i) {
          const uint8_t* atom;
          if (!kDown) {
            atom = kFP8 ? d.sh_s13a + ((static_cast<int64_t>(i) * (d.I_sh / kM) + tile) * (D / kM) + kc) * 512
                        : d.s13a + (((static_cast<int64_t>(e) * 2 + i) * (d.I / kM) + tile) * (D / kM) + kc) * 512;
          } else {
            atom = kFP8 ? d.sh_s2a + (static_cast<int64_t>(tile) * (d.I_sh / kM) + kc * 2 + i) * 512
                        : d.s2a + ((static_cast<int64_t>(e) * (D / kM) + tile) * (d.I / kM) + kc * 2 + i) * 512;
          }
          bulk_load(SF + i * 512, atom, 512, &bars->full[st]);
        }
      }
    }
  } else if (warp == 5) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      tc5::cp_sf_32x128b(tmem + kSfbCol, tc5::sdesc_sf(smem_u32(sfb)));
      const uint32_t afmt = kFP8 ? 0u : 5u;
      for (int kc = 0; kc < nk; ++kc) {
        const int st = kc % S_;
        if (!mbar_wait(&bars->full[st], (kc / S_) & 1)) {
          report(a.status, HS_DEV_TIMEOUT);
          break;
        }
        tc5::fence_after_sync();
        uint8_t* S = stages + st * L::kStage;
        const uint32_t sA = smem_u32(S), sB = smem_u32(S + L::kA), sSF = smem_u32(S + L::kA + L::kB);
        const uint32_t sfa0 = tmem + kSfaCol + st * 8;
        tc5::cp_sf_32x128b(sfa0, tc5::sdesc_sf(sSF));
        tc5::cp_sf_32x128b(sfa0 + 4, tc5::sdesc_sf(sSF + 512));
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const uint64_t ad = tc5::sdesc_sw128(sA + i * kBoxBytes);
          const uint64_t bd = tc5::sdesc_sw128(sB + (kDown ? i * 2 * NT * 1024 : 0));
          const uint32_t dcol = tmem + (kDown ? 0 : (i ? kAccUp : 0));
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t id = tc5::idesc_mxf8f6f4(afmt, N, j, j);
            const uint32_t acc = (kc > 0 || j > 0 || (kDown && i > 0)) ? 1u : 0u;
            tc5::mma_mxf8f6f4(dcol, ad + 2 * j, bd + 2 * j, id, acc, (sfa0 + 4 * i) | (static_cast<uint32_t>(j) << 30),
                              (tmem + kSfbCol) | (static_cast<uint32_t>(j) << 30));
          }
        }
        tc5::commit(&bars->empty[st]);
      }
      tc5::commit(&bars->accum);
    }
  } else {
    // ---------------- epilogue (warps 0-3, TMEM lanes 32w..32w+31) ----------------
    const int row = 32 * warp + lane;  // weight row within the tile
    if (!mbar_wait(&bars->accum, 0)) report(a.status, HS_DEV_TIMEOUT);
    tc5::fence_after_sync();
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(32 * warp) << 16);
    float c0[N];
#pragma unroll
    for (int q = 0; q < NT; ++q) {
      float v[16];
      tc5::ld_32x32b_x16(lane_base + q * 16, v);
#pragma unroll
      for (int i = 0; i < 16; ++i) c0[q * 16 + i] = v[i];
    }
    if (!kDown) {
      float c1[N];
#pragma unroll
      for (int q = 0; q < NT; ++q) {
        float v[16];
        tc5::ld_32x32b_x16(lane_base + kAccUp + q * 16, v);
#pragma unroll
        for (int i = 0; i < 16; ++i) c1[q * 16 + i] = v[i];
      }
      tc5::wait_ld();
      const int64_t I_act = max(d.I, d.has_shared ? d.I_sh : 0);
      uint8_t* hi_plane = a.P.act8;
      uint8_t* lo_plane = a.P.act8 + a.P_max * I_act;
      const int col = tile * kM + row;
#pragma unroll
      for (int r = 0; r < 8 * NT; ++r) {
        if (r < np) {
          const int p = pair0 + r;
          // reference: gate/up rounded to bf16, SwiGLU with clamp 10 in f32,
          // rounded to bf16, times the bf16 routing weight, rounded to bf16
          const float gf = round_bf16(c0[r] + c0[8 * NT + r]);
          const float uf = round_bf16(c1[r] + c1[8 * NT + r]);
          const float gc = gf > 10.f ? 10.f : gf;
          const float uc = uf > 10.f ? 10.f : (uf < -10.f ? -10.f : uf);
          const float sig = 1.f / (1.f + expf(-gc));
          float av = round_bf16((gc * sig) * uc);
          if (!kFP8) av = round_bf16(av * a.P.pair_wb[p]);
          const float v = av * exp2i(a.P.pair_q[p]);
          const __nv_fp8_storage_t hb = __nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
          const __half_raw hr = __nv_cvt_fp8_to_halfraw(hb, __NV_E4M3);
          const float hf = __half2float(*reinterpret_cast<const __half*>(&hr));
          const __nv_fp8_storage_t lb = __nv_cvt_float_to_fp8(v - hf, __NV_SATFINITE, __NV_E4M3);
          hi_plane[static_cast<int64_t>(p) * I_act + col] = hb;
          lo_plane[static_cast<int64_t>(p) * I_act + col] = lb;
        }
      }
    } else {
      tc5::wait_ld();
#pragma unroll
      for (int r = 0; r < 8 * NT; ++r) {
        if (r < np) {
          const int p = pair0 + r;
          a.P.out_part[static_cast<int64_t>(p) * D + tile * kM + row] = c0[r] + c0[8 * NT + r];
        }
      }
    }
  }

  // ---- teardown: every tcgen05 op has completed (accum barrier / ld waits) ----
  tc5::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc5::fence_after_sync();
    tc5::tmem_dealloc(tmem, kTmemCols);
  }

  if (kDown) {
    // ---- finalize this 128-row slice of D if this CTA is the last one on it ----
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      const uint32_t total = static_cast<uint32_t>(a.n_sh_chunks + a.P.hdr[0]);
      bars->last = atomicAdd(&a.P.dcount[tile], 1u) == total - 1u;
    }
    __syncthreads();
    if (bars->last) {
      __threadfence();
      finalize_tile(a, D, tile);
    }
  }
}

template <bool kDown, int NT>
__global__ void __launch_bounds__(kThreads) unit_kernel(const __grid_constant__ Desc d,
                                                           const __grid_constant__ CallMaps cm, UnitArgs a) {
  int u = blockIdx.x;
  const int tiles_sh = kDown ? d.D / kM : (d.has_shared ? d.I_sh / kM : 0);
  const int tiles = kDown ? d.D / kM : d.I / kM;
  const int n_sh_units = a.n_sh_chunks * tiles_sh;
  if (u < n_sh_units) {
    const int c = u / tiles_sh;
    const int tile = u - c * tiles_sh;
    const int pair0 = c * a.CH;
    run_unit<kDown, true, NT>(d, cm, a, 0, pair0, min(a.CH, a.T - pair0), tile);
    return;
  }
  u -= n_sh_units;
  const int c = u / tiles;
  const int tile = u - c * tiles;
  if (c >= a.P.hdr[0]) {
    // no unit at all (every pair skipped, no shared expert): the first chunk
    // slot of each tile writes the all-zero result
    if (kDown && c == 0 && a.n_sh_chunks == 0) finalize_tile(a, d.D, tile);
    return;
  }
  run_unit<kDown, false, NT>(d, cm, a, a.P.chunk_expert[c], a.P.chunk_pair0[c], a.P.chunk_np[c], tile);
}

// ---------------------------------------------------------------------------
// standalone permute gather and unpermute (R10)
// ---------------------------------------------------------------------------
// Block l copies x[t] into row token_topk_to_pos[l] (if valid) and zero-fills
// row l when l >= num_pos, matching expand_to_fused's zero-initialised output.
__global__ void expand_kernel(const __nv_bfloat16* __restrict__ x, const int32_t* __restrict__ tok_pos, int K, int D,
                              const int32_t* __restrict__ num_pos, __nv_bfloat16* __restrict__ xe) {
  const int l = blockIdx.x;
  const int p = tok_pos[l];
  if (p >= 0) {
    const __nv_bfloat16* src = x + static_cast<int64_t>(l / K) * D;
    __nv_bfloat16* dst = xe + static_cast<int64_t>(p) * D;
    for (int k = threadIdx.x; k < D; k += blockDim.x) dst[k] = src[k];
  }
  if (l >= *num_pos) {
    __nv_bfloat16* dst = xe + static_cast<int64_t>(l) * D;
    for (int k = threadIdx.x; k < D; k += blockDim.x) dst[k] = __float2bfloat16_rn(0.f);
  }
}

__global__ void unpermute_kernel(const __nv_bfloat16* __restrict__ xe, int64_t n_rows, int D,
                                 const int32_t* __restrict__ pos, const float* __restrict__ w, int T, int K,
                                 __nv_bfloat16* __restrict__ out) {
  const int t = blockIdx.y;
  const int d = blockIdx.x * blockDim.x + threadIdx.x;
  if (d >= D) return;
  float acc = 0.f;
  for (int j = 0; j < K; ++j) {
    const int p = pos[t * K + j];
    if (p < 0 || p >= n_rows) continue;
    const float s = w ? w[t * K + j] : 1.f;
    // separate multiply and add (no contraction), as reduce_fused computes it
    acc = __fadd_rn(__fmul_rn(__bfloat162float(xe[static_cast<int64_t>(p) * D + d]), s), acc);
  }
  out[static_cast<int64_t>(t) * D + d] = __float2bfloat16_rn(acc);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2D map: `cols` elements per row, row pitch `pitch` bytes, box cols x rows, 128B swizzle.
static int make_map(CUtensorMap* m, const void* base, CUtensorMapDataType dt, uint64_t cols, uint64_t rows,
                    uint64_t pitch, uint32_t box_cols, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return HS_ERR_UNSUPPORTED;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {pitch};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_cuda_error(static_cast<int>(r));
    return HS_ERR_CUDA;
  }
  return HS_OK;
}

static bool dim_ok(int64_t v, int64_t mult, int64_t lo, int64_t hi) { return v % mult == 0 && v >= lo && v <= hi; }
static bool aligned32(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 31u) == 0; }

template <bool kDown, int NT>
static int launch_units(const Desc& d, const CallMaps& cm, const UnitArgs& a, int64_t units, cudaStream_t st) {
  constexpr int bytes = SmemLayout<NT, kDown ? 2 : 1>::kBytes;
  static std::atomic<uint64_t> done{0};
  int dev = 0;
  HS_CUDA_CHECK(cudaGetDevice(&dev));
  const uint64_t bit = 1ull << (dev & 63);
  if (!(done.load() & bit)) {
    HS_CUDA_CHECK(cudaFuncSetAttribute(unit_kernel<kDown, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    done.fetch_or(bit);
  }
  unit_kernel<kDown, NT><<<static_cast<unsigned>(units), kThreads, bytes, st>>>(d, cm, a);
  return check_launch();
}

template <bool kDown>
static int launch_nt(int NT, const Desc& d, const CallMaps& cm, const UnitArgs& a, int64_t units, cudaStream_t st) {
  switch (NT) {
    case 1:
      return launch_units<kDown, 1>(d, cm, a, units, st);
    case 2:
      return launch_units<kDown, 2>(d, cm, a, units, st);
    default:
      return launch_units<kDown, 3>(d, cm, a, units, st);
  }
}

static int plan_smem(int E, int npairs) {
  return static_cast<int>(((npairs <= kLocalPairs ? npairs : 0) + 4 * E + 2 + (kPlanThreads / 32) * E) *
                          sizeof(int32_t));
}

static int launch_plan(const PlanArgs& pa, const Plan& P, int grid, cudaStream_t st) {
  const int smem = plan_smem(pa.E, pa.T * pa.K);
  if (smem > 200 * 1024) return HS_ERR_BAD_SHAPE;
  static std::atomic<uint64_t> done{0};
  int dev = 0;
  HS_CUDA_CHECK(cudaGetDevice(&dev));
  const uint64_t bit = 1ull << (dev & 63);
  if (!(done.load() & bit)) {
    HS_CUDA_CHECK(cudaFuncSetAttribute(plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    done.fetch_or(bit);
  }
  plan_kernel<<<grid, kPlanThreads, smem, st>>>(pa, P);
  return check_launch();
}

}  // namespace moe
}  // namespace hs

using namespace hs;
using namespace hs::moe;

extern "C" int hs_moe_make_desc(const hs_moe_weights* w, void* desc_out, size_t desc_bytes) {
  if (!w || !desc_out) return HS_ERR_BAD_ARGUMENT;
  if (desc_bytes < sizeof(Desc)) return HS_ERR_BAD_ARGUMENT;
  if (!dim_ok(w->D, 512, 512, 8192) || !dim_ok(w->I, 512, 512, 8192) || w->E < 1 || w->E > 1024)
    return HS_ERR_BAD_SHAPE;
  if (!w->w13 || !w->s13 || !w->w2 || !w->s2) return HS_ERR_BAD_ARGUMENT;
  if (!aligned32(w->w13) || !aligned32(w->w2) || !aligned16(w->s13) || !aligned16(w->s2)) return HS_ERR_ALIGN;
  Desc d;
  memset(&d, 0, sizeof(d));
  d.E = static_cast<int32_t>(w->E);
  d.D = static_cast<int32_t>(w->D);
  d.I = static_cast<int32_t>(w->I);
  d.has_shared = w->sh_w13 != nullptr;
  int st;
  const uint64_t E = w->E, D = w->D, I = w->I;
  if ((st = make_map(&d.tm_w13, w->w13, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, D, E * 2 * I, D / 2, 128, kM)))
    return st;
  if ((st = make_map(&d.tm_w2, w->w2, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, I, E * D, I / 2, 128, kM))) return st;
  d.s13a = static_cast<const uint8_t*>(w->s13);
  d.s2a = static_cast<const uint8_t*>(w->s2);
  if (d.has_shared) {
    if (!dim_ok(w->I_sh, 256, 256, 8192)) return HS_ERR_BAD_SHAPE;
    if (!w->sh_s13 || !w->sh_w2 || !w->sh_s2) return HS_ERR_BAD_ARGUMENT;
    if (!aligned16(w->sh_w13) || !aligned16(w->sh_w2) || !aligned16(w->sh_s13) || !aligned16(w->sh_s2))
      return HS_ERR_ALIGN;
    d.I_sh = static_cast<int32_t>(w->I_sh);
    const uint64_t Ish = w->I_sh;
    if ((st = make_map(&d.tm_sw13, w->sh_w13, CU_TENSOR_MAP_DATA_TYPE_UINT8, D, 2 * Ish, D, 128, kM))) return st;
    if ((st = make_map(&d.tm_sw2, w->sh_w2, CU_TENSOR_MAP_DATA_TYPE_UINT8, Ish, D, Ish, 128, kM))) return st;
    d.sh_s13a = static_cast<const uint8_t*>(w->sh_s13);
    d.sh_s2a = static_cast<const uint8_t*>(w->sh_s2);
  }
  d.magic = kDescMagic;
  memset(desc_out, 0, desc_bytes);
  memcpy(desc_out, &d, sizeof(d));
  return HS_OK;
}

extern "C" size_t hs_moe_workspace_size(int64_t T, int64_t top_k, int64_t D, int64_t I, int64_t I_sh) {
  if (T < 0 || top_k < 1) return 0;
  return geometry(T, top_k, D, I, I_sh).total;
}

extern "C" int hs_moe_ffn_fp4(const void* desc, const void* hidden, const int64_t* topk_idx, const float* topk_w,
                              int64_t T, int64_t top_k, int use_shared, int dup_mode, void* out, float* out_f32,
                              void* workspace, size_t workspace_bytes, int32_t* dev_status, void* stream) {
  if (!desc) return HS_ERR_BAD_ARGUMENT;
  Desc d;
  memcpy(&d, desc, sizeof(d));
  if (d.magic != kDescMagic) return HS_ERR_BAD_ARGUMENT;
  if (T < 0 || top_k < 1 || top_k > 16) return HS_ERR_BAD_SHAPE;
  if (T == 0) return HS_OK;
  if (T > (1 << 20)) return HS_ERR_BAD_SHAPE;
  if (!hidden || !topk_idx || !topk_w || !out || !workspace) return HS_ERR_BAD_ARGUMENT;
  if (dup_mode != HS_DUP_LAST && dup_mode != HS_DUP_SUM) return HS_ERR_BAD_ARGUMENT;
  if (!aligned16(hidden) || !aligned16(out) || !aligned16(workspace) || (out_f32 && !aligned16(out_f32)))
    return HS_ERR_ALIGN;
  use_shared = (use_shared && d.has_shared) ? 1 : 0;
  if (!d.has_shared) d.I_sh = 0;
  const Geometry g = geometry(T, top_k, d.D, d.I, d.has_shared ? d.I_sh : 0);
  if (workspace_bytes < g.total) return HS_ERR_WORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const Plan P = plan_views(g, workspace);
  const int NT = static_cast<int>(ntiles(T));
  const int CH = 8 * NT;
  const int64_t npairs = T * top_k;
  const bool local_rows = npairs <= kLocalPairs;

  CallMaps cm;
  int rc;
  if ((rc = make_map(&cm.tm_x8, P.x8, CU_TENSOR_MAP_DATA_TYPE_UINT8, d.D, 2 * g.P_max, d.D, 128, 8))) return rc;
  if ((rc = make_map(&cm.tm_act8, P.act8, CU_TENSOR_MAP_DATA_TYPE_UINT8, g.I_act, 2 * g.P_max, g.I_act, 128, 8)))
    return rc;

  PlanArgs pa;
  pa.topk_idx = topk_idx;
  pa.topk_w = topk_w;
  pa.hidden = static_cast<const __nv_bfloat16*>(hidden);
  pa.T = static_cast<int>(T);
  pa.K = static_cast<int>(top_k);
  pa.E = d.E;
  pa.D = d.D;
  pa.CH = CH;
  pa.dup_mode = dup_mode;
  pa.pos_offset = static_cast<int>(T);
  pa.sort_tok = 1;
  pa.n_dcount = d.D / kM;
  pa.P_max = g.P_max;
  pa.local_rows = local_rows ? 1 : 0;
  pa.po = PermuteOut{nullptr, nullptr, nullptr};
  pa.status = dev_status;
  if ((rc = launch_plan(pa, P, 1 + static_cast<int>(T), st))) return rc;
  if (!local_rows) {
    gather_kernel<<<static_cast<unsigned>(npairs), 256, 0, st>>>(P, static_cast<int>(T), g.P_max, d.D);
    if ((rc = check_launch())) return rc;
  }

  UnitArgs a;
  a.P = P;
  a.T = static_cast<int>(T);
  a.K = static_cast<int>(top_k);
  a.CH = CH;
  a.P_max = g.P_max;
  a.n_sh_chunks = use_shared ? static_cast<int>((T + CH - 1) / CH) : 0;
  a.use_shared = use_shared;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.out_f32 = out_f32;
  a.status = dev_status;
  const int64_t gu_units = static_cast<int64_t>(a.n_sh_chunks) * (use_shared ? d.I_sh / kM : 0) +
                           g.C_max * (d.I / kM);
  const int64_t dn_units = (static_cast<int64_t>(a.n_sh_chunks) + g.C_max) * (d.D / kM);
  if (gu_units > 0x7fffffff || dn_units > 0x7fffffff) return HS_ERR_BAD_SHAPE;
  if ((rc = launch_nt<false>(NT, d, cm, a, gu_units, st))) return rc;
  return launch_nt<true>(NT, d, cm, a, dn_units, st);
}

extern "C" size_t hs_moe_permute_workspace_size(int64_t T, int64_t top_k, int64_t E) {
  (void)E;
  if (T < 0 || top_k < 1) return 0;
  return geometry(T, top_k, 0, 0, 0).total;
}

extern "C" int hs_moe_permute(const int64_t* topk_idx, int64_t T, int64_t top_k, int64_t E, const void* x, int64_t D,
                              int32_t* token_topk_to_pos, int32_t* pos_to_expert, int32_t* expert_count,
                              int32_t* num_pos, void* x_expanded, void* workspace, size_t workspace_bytes,
                              int32_t* dev_status, void* stream) {
  if (T < 0 || top_k < 1 || top_k > 16 || E < 1 || E > 1024) return HS_ERR_BAD_SHAPE;
  if (!topk_idx || !token_topk_to_pos || !num_pos || !workspace) return HS_ERR_BAD_ARGUMENT;
  if (x_expanded && (!x || D < 1)) return HS_ERR_BAD_ARGUMENT;
  const Geometry g = geometry(T, top_k, 0, 0, 0);
  if (workspace_bytes < g.total) return HS_ERR_WORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Plan P = plan_views(g, workspace);
  P.tok_pos = token_topk_to_pos;  // unsorted, k order
  if (T == 0) {
    HS_CUDA_CHECK(cudaMemsetAsync(num_pos, 0, sizeof(int32_t), st));
    if (expert_count) HS_CUDA_CHECK(cudaMemsetAsync(expert_count, 0, E * sizeof(int32_t), st));
    return HS_OK;
  }
  PlanArgs pa;
  pa.topk_idx = topk_idx;
  pa.topk_w = nullptr;
  pa.hidden = nullptr;
  pa.T = static_cast<int>(T);
  pa.K = static_cast<int>(top_k);
  pa.E = static_cast<int>(E);
  pa.D = 0;
  pa.CH = 1 << 30;
  pa.dup_mode = kDupKeepAll;
  pa.pos_offset = 0;
  pa.sort_tok = 0;
  pa.n_dcount = 0;
  pa.P_max = g.P_max;
  pa.local_rows = 0;
  pa.po = PermuteOut{pos_to_expert, expert_count, num_pos};
  pa.status = dev_status;
  int rc = launch_plan(pa, P, 1, st);
  if (rc) return rc;
  if (x_expanded) {
    expand_kernel<<<static_cast<unsigned>(T * top_k), 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(x), token_topk_to_pos, static_cast<int>(top_k), static_cast<int>(D),
        num_pos, static_cast<__nv_bfloat16*>(x_expanded));
    rc = check_launch();
  }
  return rc;
}

extern "C" int hs_moe_unpermute(const void* x_expanded, int64_t num_expanded, int64_t D,
                                const int32_t* token_topk_to_pos, const float* topk_w, int64_t T, int64_t top_k,
                                void* out_bf16, void* stream) {
  if (T < 0 || top_k < 1 || D < 1 || num_expanded < 0) return HS_ERR_BAD_SHAPE;
  if (T == 0) return HS_OK;
  if (!x_expanded || !token_topk_to_pos || !out_bf16) return HS_ERR_BAD_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  dim3 grid(static_cast<unsigned>((D + 255) / 256), static_cast<unsigned>(T));
  unpermute_kernel<<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x_expanded), num_expanded,
                                         static_cast<int>(D), token_topk_to_pos, topk_w, static_cast<int>(T),
                                         static_cast<int>(top_k), static_cast<__nv_bfloat16*>(out_bf16));
  return check_launch();
}

// ---------------------------------------------------------------------------
// No-allocation variant
// ---------------------------------------------------------------------------
// For callers that cannot allocate device memory when they call (plugin hosts
// whose enqueue path forbids it, code inside a CUDA-graph stream capture where
// cudaMalloc is not permitted, loops where cudaMalloc/cudaFree would
// synchronise the device): the scratch lives in this file-scope device array.
// Every GPU that loads the library holds it until the process exits, and
// every call shares it, so calls that overlap on the GPU race. The plan kernel
// clears the finalize counters at the start of each call; nothing else in the
// scratch needs to start at zero.
static __device__ __align__(256) uint8_t g_moe_noalloc_scratch[HS_MOE_NOALLOC_BYTES];

// Device address of the scratch array per device, looked up once per device
// with that device current (the array's name is only a host-side stand-in).
static void* noalloc_scratch_ptr(int* status) {
  static std::mutex mu;
  static void* ptrs[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    set_last_cuda_error(static_cast<int>(e));
    *status = HS_ERR_CUDA;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_moe_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      set_last_cuda_error(static_cast<int>(e));
      *status = HS_ERR_CUDA;
      return nullptr;
    }
    ptrs[dev] = p;
  }
  *status = HS_OK;
  return ptrs[dev];
}

extern "C" int hs_moe_ffn_fp4_noalloc(const void* desc, const void* hidden, const int64_t* topk_idx,
                                      const float* topk_w, int64_t T, int64_t top_k, int use_shared, int dup_mode,
                                      void* out, float* out_f32, int32_t* dev_status, void* stream) {
  if (!desc) return HS_ERR_BAD_ARGUMENT;
  Desc d;
  memcpy(&d, desc, sizeof(d));
  if (d.magic != kDescMagic) return HS_ERR_BAD_ARGUMENT;
  if (T < 0 || top_k < 1 || top_k > 16) return HS_ERR_BAD_SHAPE;
  if (hs_moe_workspace_size(T, top_k, d.D, d.I, d.has_shared ? d.I_sh : 0) > HS_MOE_NOALLOC_BYTES)
    return HS_ERR_WORKSPACE;
  int st = HS_OK;
  void* scratch = noalloc_scratch_ptr(&st);
  if (st != HS_OK) return st;
  return hs_moe_ffn_fp4(desc, hidden, topk_idx, topk_w, T, top_k, use_shared, dup_mode, out, out_f32, scratch,
                        HS_MOE_NOALLOC_BYTES, dev_status, stream);
}
