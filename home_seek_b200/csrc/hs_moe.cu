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
//   * Weights never pass through registers. The expert store keeps every
//     128x128 weight tile contiguous and the two tiles a pipeline stage needs
//     (w1 and w3 of one k-step, or two consecutive k-steps of w2) adjacent, so
//     one TMA per stage streams 16 KB of consecutive packed e2m1 straight into
//     128B-swizzled shared memory (data type 16U4_ALIGN16B, the layout
//     kind::mxf8f6f4 reads); the UE8M0 scales (stored in the tcgen05
//     scale-factor atom layout, 512 B per 128 rows x 128 columns, the stage's
//     two atoms adjacent) arrive with one 1 KB bulk copy and go to TMEM with
//     tcgen05.cp, and tcgen05.mma.kind::mxf8f6f4
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

#include <cooperative_groups.h>
#include <cuda_fp8.h>

#include "hs_common.cuh"
#include "hs_tcgen05.cuh"
#include "hs_topk.cuh"
#include "hs_trace.cuh"

namespace cg = cooperative_groups;

namespace hs {
namespace moe {

constexpr int kM = 128;                 // weight rows per unit (UMMA M)
constexpr int kBoxBytes = kM * 128;     // one 128x128 weight tile in shared memory
constexpr int kThreads = 192;           // warps 0-3 epilogue, warp 4 TMA, warp 5 MMA
constexpr int kAccUp = 48;              // TMEM column of the up accumulator within a buffer (N <= 48)
constexpr int kMaxNT = 3;               // n-tiles of 8 pairs (N = 16 * NT)
constexpr int kPlanThreads = 512;
constexpr int kLocalPairs = 4096;       // T*K up to this: token CTAs place their own rows
constexpr int kFastPlanPairs = 1024;    // T*K up to this: block 0 uses the direct-count plan
constexpr uint32_t kDescMagic = 0x48534d33u;  // "HSM3" (tiled weights)
constexpr int kTokMax = 8;              // T <= this: token mode (activation rows per token, not per pair)
constexpr int kInlineCombineMax = 64;   // T above this: the down phase's outputs are combined by a separate grid
constexpr int kTokChunks = 128;         // token mode: at most T*K <= 8*16 routed chunks
constexpr int kSegPairs = 1024;         // segmented plan: pairs per counting CTA
constexpr int kSegMaxE = 256;           // segmented plan: experts per call at most
constexpr int kSegTicket = 15;          // plan header word: the counting CTAs' ticket (left at 0)
constexpr int kCtasPerSm = 2;           // MoE CTAs resident per SM (two independent MMA streams)
constexpr int kSmemPerCta = 115712;     // (228 KB per SM - 1 KB reserved per CTA) / 2
constexpr int kTokDownPad = 256;        // token-mode down kernel: read-only slack after its last stage


struct __align__(64) Desc {
  // Weight tiles as rows of 128 values: [tiles * 128 rows][128], box 128 x 256
  // (two adjacent tiles), 128B swizzle.
  CUtensorMap tm_w13;   // e2m1 [E][I/128][D/128][w1, w3][128][128], 16U4_ALIGN16B
  CUtensorMap tm_w2;    // e2m1 [E][D/128][I/128][128][128]
  CUtensorMap tm_sw13;  // e4m3 [I_sh/128][D/128][w1, w3][128][128], uint8
  CUtensorMap tm_sw2;   // e4m3 [D/128][I_sh/128][128][128]
  const uint8_t* s13a;  // [E][I/128][D/128][2][512] scale-factor atoms
  const uint8_t* s2a;   // [E][D/128][I/128][512]
  const uint8_t* sh_s13a;  // [I_sh/128][D/128][2][512]
  const uint8_t* sh_s2a;   // [D/128][I_sh/128][512]
  // the same weights as plain bytes (L2 prefetch)
  const uint8_t* w13;
  const uint8_t* w2;
  const uint8_t* sh_w13;
  const uint8_t* sh_w2;
  int32_t E, D, I, I_sh;
  int32_t has_shared;
  uint32_t magic;
};
static_assert(sizeof(Desc) <= HS_MOE_DESC_BYTES, "descriptor blob too small");

struct CallMaps {
  CUtensorMap tm_x8;    // [2 (hi, lo)][P_max rows][D] e4m3, box 128 x 8*NT x 2
  CUtensorMap tm_act8;  // [2][P_max rows][I_act]
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
  uint8_t* act8;          // [2][P_max][I_act] e4m3 hi / lo; token mode [2][(1 + C_max) * 8][I_act]
  float* out_part;        // [P_max][D]
  float* ctab_wb;         // token mode: [C_max][8] routing weight of (chunk, token), 0 if not routed
  // token mode: the down MMA's B scale factors of the activation rows, as
  // scale-atom images: [1 + C_max slots][I_act / 128 k-tiles][256 bytes];
  // byte n * 16 + j is the UE8M0 scale of B row n (hi rows 0-7 = tokens, lo
  // rows 8-15) over the k-tile's 32-column block j, i.e. lines 0-15 of a
  // 512-byte atom (an N = 16 MMA never reads the rows above 15)
  uint8_t* act_img;
};

struct Geometry {
  int64_t T, K, D, I, I_sh, I_act, P_max, C_max;
  int64_t U_gu, U_dn;      // upper bounds on gate/up and down units
  int G;                   // persistent CTAs
  int aligned;             // unit-aligned schedule (no partial slots)
  int64_t slot_floats;     // floats per partial slot (gate/up, the larger)
  int64_t act_rows;        // rows per activation plane
  size_t off_hdr, off_chunk, off_pair, off_sb, off_tok, off_tokpos, off_dcount, off_x8, off_act8, off_out,
      off_ucount, off_part, off_ctab, off_img, off_seg, total;
};

static size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

static int64_t ntiles(int64_t T) {
  int64_t nt = (T + 7) / 8;
  return std::max<int64_t>(1, std::min<int64_t>(nt, kMaxNT));
}

static Geometry geometry(int64_t T, int64_t K, int64_t D, int64_t I, int64_t I_sh, int G = 148) {
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
  g.act_rows = T <= kTokMax ? std::max<int64_t>(g.P_max, 8 * (1 + g.C_max)) : g.P_max;
  g.off_act8 = o;
  o = align_up(o + 2 * g.act_rows * g.I_act, 256);
  g.off_out = o;
  o = align_up(o + g.P_max * D * sizeof(float), 256);
  // stream-K state: per-unit tickets and partial accumulator slots
  const int64_t n_sh = (T + CH - 1) / CH;
  g.U_gu = g.C_max * (I / kM) + n_sh * (I_sh / kM);
  g.U_dn = (g.C_max + n_sh) * (D / kM);
  g.G = G;
  g.aligned = 0;
  g.slot_floats = 2 * kM * 8 * ntiles(T);
  g.off_ucount = o;
  o = align_up(o + (g.U_gu + g.U_dn) * sizeof(uint32_t), 256);
  g.off_part = o;
  o = align_up(o + 2 * static_cast<int64_t>(G) * g.slot_floats * sizeof(float), 256);
  g.off_ctab = o;
  o = align_up(o + g.C_max * 8 * sizeof(float), 256);
  g.off_img = o;
  if (T <= kTokMax) o = align_up(o + (1 + g.C_max) * (g.I_act / kM) * 256, 256);
  // segmented plan: per-pair ranks, per-segment offsets, expert bases
  g.off_seg = o;
  o = align_up(o + (Pr + ((Pr + kSegPairs - 1) / kSegPairs) * kSegMaxE + kSegMaxE) * sizeof(int32_t), 256);
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
  p.ctab_wb = reinterpret_cast<float*>(b + g.off_ctab);
  p.act_img = b + g.off_img;
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
  int tok_mode;    // T <= kTokMax: per-(chunk, token) tables instead of per-pair rows
  int64_t n_ctab;  // token mode: table entries to clear (C_max * 8)
  PermuteOut po;
  int32_t* status;
  uint32_t* ucount;  // stream-K unit tickets to clear (all plan CTAs share the work)
  int64_t n_ucount;
  // segmented plan (plan_seg_kernel ran first; nullptr: off): a pair's rank
  // among its expert's pairs in its segment, [segment][E] offsets of the
  // segments, [E] first position of each expert (without pos_offset)
  const int32_t* seg_lrank;
  const int32_t* seg_off;
  const int32_t* seg_base;
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

// Row prescale exponent of a token row with max |x| = mx: the row times
// 2^e has its largest magnitude in [2^7, 2^8) for the hi/lo e4m3 split.
__device__ __forceinline__ int row_prescale(float mx) {
  if (!(mx > 0.f) || !isfinite(mx)) return 0;
  int ex;
  frexpf(mx, &ex);
  return max(-100, min(100, 8 - ex));
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

// hi/lo e4m3 split of 16 consecutive bf16 values (two uint4) scaled by 2^e.
__device__ __forceinline__ void split16(const uint4& a, const uint4& b, float sc, uint4& hi, uint4& lo) {
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

// Segmented plan for calls with many pairs (a stable counting sort of the
// pairs by expert, the order the single-CTA plan below produces). CTA s ranks
// the pairs of segment s (kSegPairs consecutive pairs) among the segment's
// pairs of the same expert (warp match + per-warp counts) and publishes the
// segment's per-expert counts; the last CTA to finish (a ticket in the plan
// header, reset for the next call) turns the counts into per-segment offsets
// and expert bases and writes the chunk table and the header. The token CTAs
// of plan_kernel then place their own pairs: position = T + base[e] +
// offset[segment][e] + rank.
__global__ void __launch_bounds__(kSegPairs) plan_seg_kernel(PlanArgs A, Plan P, int32_t* lrank, int32_t* segoff,
                                                            int32_t* ebase) {
  __shared__ int32_t wc[kSegPairs / 32][kSegMaxE];
  __shared__ int32_t hist[kSegMaxE];
  __shared__ int32_t base[kSegMaxE + 1];
  __shared__ int32_t cbase[kSegMaxE + 1];
  __shared__ int32_t slots;
  __shared__ int last;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = A.K, E = A.E;
  const int npairs = A.T * K;
  pdl_wait();
  pdl_trigger();
  const int l = blockIdx.x * kSegPairs + tid;
  int e = -1;
  if (l < npairs) {
    const int t = l / K, j = l - t * K;
    int32_t row[16];
    for (int jj = 0; jj < K; ++jj) row[jj] = clamp_id(A.topk_idx[static_cast<int64_t>(t) * K + jj], E);
    if (row[j] == kBadId) report(A.status, HS_DEV_BAD_EXPERT);
    e = pair_expert(row, nullptr, j, K, A.dup_mode, nullptr);
  }
  for (int x = lane; x < E; x += 32) wc[warp][x] = 0;
  __syncwarp();
  const unsigned msk = __match_any_sync(0xffffffffu, e);
  const int rank = __popc(msk & ((1u << lane) - 1u));
  if (e >= 0 && rank == 0) wc[warp][e] = __popc(msk);
  __syncthreads();
  if (tid < E) {
    int run = 0;
    for (int w = 0; w < kSegPairs / 32; ++w) {
      const int c = wc[w][tid];
      wc[w][tid] = run;
      run += c;
    }
    segoff[static_cast<int64_t>(blockIdx.x) * E + tid] = run;
  }
  __syncthreads();
  if (e >= 0) lrank[l] = wc[warp][e] + rank;
  __threadfence();
  __syncthreads();
  if (tid == 0) last = atomicAdd(reinterpret_cast<unsigned int*>(P.hdr + kSegTicket), 1u) == gridDim.x - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  // ---- last CTA: offsets of every segment per expert ----
  // thread (part, e) scans segments [part * per, (part + 1) * per) of expert e
  const int nseg = gridDim.x;
  const int parts = kSegPairs / E;
  const int per = (nseg + parts - 1) / parts;
  const int pe = tid % E, part = tid / E;
  int32_t* ps = &wc[0][0];  // [parts][E] partial sums
  if (part < parts) {
    int sum = 0;
    for (int sg = part * per; sg < min(nseg, (part + 1) * per); ++sg) sum += __ldcg(segoff + static_cast<int64_t>(sg) * E + pe);
    ps[part * E + pe] = sum;
  }
  __syncthreads();
  if (tid < E) {
    int run = 0;
    for (int pp = 0; pp < parts; ++pp) {
      const int c = ps[pp * E + tid];
      ps[pp * E + tid] = run;
      run += c;
    }
    hist[tid] = run;
  }
  if (tid == 0) slots = 0;
  __syncthreads();
  if (part < parts) {
    int run = ps[part * E + pe];
    for (int sg = part * per; sg < min(nseg, (part + 1) * per); ++sg) {
      int32_t* q = segoff + static_cast<int64_t>(sg) * E + pe;
      const int c = __ldcg(q);
      *q = run;
      run += c;
    }
  }
  // ---- expert bases and chunk bases (exclusive scans over experts) ----
  if (warp == 0) {
    int run = 0, crun = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int x0 = e0 + lane;
      const int hh = x0 < E ? hist[x0] : 0;
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
      if (x0 < E) {
        base[x0] = run + x - hh;
        cbase[x0] = crun + y - c;
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
  if (tid < E) {
    const int hh = hist[tid];
    ebase[tid] = base[tid];
    if (hh > 0) atomicAdd(&slots, 1);
    int cb = cbase[tid];
    for (int c = 0; c * A.CH < hh; ++c, ++cb) {
      P.chunk_expert[cb] = tid;
      P.chunk_pair0[cb] = A.pos_offset + base[tid] + c * A.CH;
      P.chunk_np[cb] = min(A.CH, hh - c * A.CH);
    }
  }
  __syncthreads();
  if (tid == 0) {
    P.hdr[0] = cbase[E];
    P.hdr[1] = slots;
    P.hdr[2] = base[E];
    P.hdr[kSegTicket] = 0;
  }
}

// Block 0 builds the routing plan; blocks 1..T (MoE call only) convert one
// token row each into its shared-expert row and, when local_rows is set, its
// routed pair rows (positions recomputed locally from the same counts).
__global__ void __launch_bounds__(kPlanThreads) plan_kernel(PlanArgs A, Plan P) {
  extern __shared__ int32_t sm[];
  const int tid = threadIdx.x;
  const int T = A.T, K = A.K, E = A.E;
  const int npairs = T * K;
  const bool cache_idx = npairs <= kLocalPairs && !A.seg_lrank;
  pdl_trigger();  // the MoE kernels may start their prologues
  pdl_wait();     // router outputs (and everything earlier) are complete
  // token CTAs: thread k16 holds values 16*k16 .. 16*k16+15 of the row in
  // registers (D <= 16 * kPlanThreads), loaded first so the load overlaps the
  // routing reads below; then the max and the split run from registers
  const bool holds = blockIdx.x > 0 && tid < A.D / 16;
  uint4 va = make_uint4(0u, 0u, 0u, 0u), vb = va;
  if (holds) {
    const uint4* hrow = reinterpret_cast<const uint4*>(A.hidden + static_cast<int64_t>(blockIdx.x - 1) * A.D);
    va = hrow[2 * tid];
    vb = hrow[2 * tid + 1];
  }
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + tid; i < A.n_ucount;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    A.ucount[i] = 0u;
  int32_t* sidx = sm;  // [npairs] clamped ids (when cached)
  int32_t* rest = sm + (cache_idx ? npairs : 0);
  if (cache_idx) {
    for (int l = tid; l < npairs; l += blockDim.x) sidx[l] = clamp_id(A.topk_idx[l], E);
    __syncthreads();
  }

  // expert of every pair after the duplicate rule (-1 = skipped), when cached
  int32_t* sval = rest;                          // [npairs]
  rest = rest + (cache_idx ? npairs : 0);
  if (cache_idx) {
    for (int l = tid; l < npairs; l += blockDim.x) {
      const int t = l / K;
      if (blockIdx.x == 0 && sidx[l] == kBadId) report(A.status, HS_DEV_BAD_EXPERT);
      sval[l] = pair_expert(sidx + t * K, nullptr, l - t * K, K, A.dup_mode, nullptr);
    }
    __syncthreads();
  }

  if (blockIdx.x > 0) {
    // ---- token row: prescale, hi/lo split, rows for its pairs ----
    const int t = blockIdx.x - 1;
    const int warp = tid >> 5, lane = tid & 31;
    float mx = 0.f;
    {
      const uint32_t w[8] = {va.x, va.y, va.z, va.w, vb.x, vb.y, vb.z, vb.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
        mx = fmaxf(mx, fmaxf(fabsf(__uint_as_float(w[i] << 16)), fabsf(__uint_as_float(w[i] & 0xffff0000u))));
    }
    __shared__ float red[kPlanThreads / 32];
    __shared__ int rows[17];
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[warp] = mx;
    int nrows = 1;
    if (A.local_rows && cache_idx && !A.tok_mode) {
      nrows = 1 + K;
      // warp j places this token's entry j: its position is the number of
      // valid pairs with a smaller expert plus the number with the same
      // expert on earlier tokens, exactly as block 0 assigns it
      if (warp < K) {
        const int e = sval[t * K + warp];
        int base = 0, rank = 0;
        if (e >= 0)
          for (int m = lane; m < npairs; m += 32) {
            const int e2 = sval[m];
            base += (e2 >= 0) & (e2 < e);
            rank += (e2 == e) & (m < t * K);
          }
        for (int o = 16; o > 0; o >>= 1) {
          base += __shfl_xor_sync(0xffffffffu, base, o);
          rank += __shfl_xor_sync(0xffffffffu, rank, o);
        }
        if (lane == 0) rows[1 + warp] = e >= 0 ? A.pos_offset + base + rank : -1;
      }
    }
    if (A.seg_lrank) {
      // segmented plan: lane j of warp 0 places this token's pair j from the
      // counts plan_seg_kernel left (the expert's base, the segment's offset,
      // the pair's rank in its segment), records the pair and the token's
      // sorted positions; the token's rows then go to all its positions
      nrows = 1 + K;
      if (warp == 0) {
        int pos = -1;
        if (lane < K) {
          int32_t row[16];
          for (int jj = 0; jj < K; ++jj) row[jj] = clamp_id(A.topk_idx[static_cast<int64_t>(t) * K + jj], E);
          const float* wrow = A.topk_w ? A.topk_w + static_cast<int64_t>(t) * K : nullptr;
          float wsum = 0.f;
          const int e = pair_expert(row, wrow, lane, K, A.dup_mode, &wsum);
          if (e >= 0) {
            const int l = t * K + lane;
            pos = A.pos_offset + __ldcg(A.seg_base + e) +
                  __ldcg(A.seg_off + static_cast<int64_t>(l / kSegPairs) * E + e) + __ldcg(A.seg_lrank + l);
            const float wb = round_bf16(wsum);
            const int q = act_prescale(wb);
            P.pair_token[pos] = t;
            P.pair_wb[pos] = wb;
            P.pair_q[pos] = q;
            P.sb2[pos] = static_cast<uint8_t>(127 - q);
          }
        }
        int nvalid = 0, rank = 0;
        for (int j = 0; j < K; ++j) {
          const int p2 = __shfl_sync(0xffffffffu, pos, j);
          nvalid += p2 >= 0;
          rank += (p2 >= 0) & (pos >= 0) & (p2 < pos);
        }
        if (lane < K) {
          if (pos >= 0) P.tok_pos[static_cast<int64_t>(t) * K + rank] = pos;
          if (lane >= nvalid) P.tok_pos[static_cast<int64_t>(t) * K + lane] = -1;
          rows[1 + lane] = pos;
        }
        if (lane == 0) {  // the token's shared-expert pair
          P.pair_token[t] = t;
          P.pair_wb[t] = 1.f;
          P.pair_q[t] = 0;
          P.sb2[t] = 127;
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
    if (holds) {
      uint4 hv, lv;
      split16(va, vb, sc, hv, lv);
      for (int r = 0; r < nrows; ++r) {
        const int p = rows[r];
        if (p < 0) continue;
        reinterpret_cast<uint4*>(hi_plane + static_cast<int64_t>(p) * A.D)[tid] = hv;
        reinterpret_cast<uint4*>(lo_plane + static_cast<int64_t>(p) * A.D)[tid] = lv;
      }
    }
    if (tid < nrows && rows[tid] >= 0) P.sb1[rows[tid]] = static_cast<uint8_t>(127 - e);
    return;
  }

  if (A.seg_lrank) {  // plan_seg_kernel built the plan
    for (int i = tid; i < A.n_dcount; i += blockDim.x) P.dcount[i] = 0u;
    return;
  }

  // ---- routing plan, small pair counts: three phases of independent counts ----
  if (cache_idx && npairs <= kFastPlanPairs) {
    int32_t* spos = rest;            // [npairs] position (or -1)
    int32_t* scnt = spos + npairs;   // [npairs] pair count of the expert (leaders only)
    float* swb = reinterpret_cast<float*>(scnt + npairs);  // [npairs] bf16 routing weight
    int32_t* sq = reinterpret_cast<int32_t*>(swb + npairs);  // [npairs] activation prescale
    __shared__ int tot[4];           // chunks, slots, pairs
    if (tid < 4) tot[tid] = 0;
    for (int i = tid; i < A.n_dcount; i += blockDim.x) P.dcount[i] = 0u;
    for (int64_t i = tid; i < A.n_ctab; i += blockDim.x) {
      P.ctab_wb[i] = 0.f;
    }
    if (A.po.expert_count)
      for (int x = tid; x < E; x += blockDim.x) A.po.expert_count[x] = 0;
    for (int t = tid; t < A.pos_offset; t += blockDim.x) {  // shared-expert pairs
      P.pair_token[t] = t;
      P.pair_wb[t] = 1.f;
      P.pair_q[t] = 0;
      P.sb2[t] = 127;
    }
    __syncthreads();
    for (int l = tid; l < npairs; l += blockDim.x) {
      const int e = sval[l];
      int pos = -1, cnt = 0;
      if (e >= 0) {
        int less = 0, before = 0;
        for (int m = 0; m < npairs; ++m) {
          const int e2 = sval[m];
          less += (e2 >= 0) & (e2 < e);
          before += (e2 == e) & (m < l);
          cnt += (e2 == e);
        }
        pos = A.pos_offset + less + before;
        const int t = l / K;
        float wsum = 0.f;
        pair_expert(sidx + t * K, A.topk_w ? A.topk_w + static_cast<int64_t>(t) * K : nullptr, l - t * K, K,
                    A.dup_mode, &wsum);
        const float wb = round_bf16(wsum);
        const int q = act_prescale(wb);
        P.pair_token[pos] = t;
        P.pair_wb[pos] = wb;
        P.pair_q[pos] = q;
        P.sb2[pos] = static_cast<uint8_t>(127 - q);
        swb[l] = wb;
        sq[l] = q;
        if (A.po.pos_to_expert) A.po.pos_to_expert[pos - A.pos_offset] = e;
        if (before == 0) {
          atomicAdd(&tot[0], (cnt + A.CH - 1) / A.CH);
          atomicAdd(&tot[1], 1);
          if (A.po.expert_count) A.po.expert_count[e] = cnt;
        }
        atomicAdd(&tot[2], 1);
      }
      spos[l] = pos;
      scnt[l] = 0;
      if (e >= 0) {
        int before = 0;
        for (int m = 0; m < l; ++m) before += sval[m] == e;
        scnt[l] = before == 0 ? cnt : 0;  // only the expert's first pair keeps the count
      }
    }
    __syncthreads();
    for (int l = tid; l < npairs; l += blockDim.x) {
      const int e = sval[l];
      const int pos = spos[l];
      if (e >= 0) {
        // the expert's first pair (the only one with a count) writes its chunks
        if (scnt[l] > 0) {
          int cb = 0;
          for (int m = 0; m < npairs; ++m) {
            const int e2 = sval[m];
            if (scnt[m] > 0 && e2 < e) cb += (scnt[m] + A.CH - 1) / A.CH;
          }
          const int cnt = scnt[l];
          const int first = pos;  // the leader holds the expert's first position
          for (int ck = 0; ck * A.CH < cnt; ++ck, ++cb) {
            P.chunk_expert[cb] = e;
            P.chunk_pair0[cb] = first + ck * A.CH;
            P.chunk_np[cb] = min(A.CH, cnt - ck * A.CH);
          }
        }
        if (A.tok_mode) {
          // one chunk per expert (at most T <= 8 pairs): its index is the
          // number of distinct experts below e; record (weight, scale) of this token
          int cb = 0;
          for (int m = 0; m < npairs; ++m) cb += (scnt[m] > 0) & (sval[m] < e);
          const int t = l / K;
          P.ctab_wb[cb * 8 + t] = swb[l];
        }
      }
      if (A.sort_tok) {
        // rank among the token's valid pairs by position (= by expert id)
        const int t = l / K;
        int nvalid = 0, rank = 0;
        for (int j = 0; j < K; ++j) {
          const int p2 = spos[t * K + j];
          nvalid += p2 >= 0;
          rank += (p2 >= 0) & (pos >= 0) & (p2 < pos);
        }
        if (pos >= 0) P.tok_pos[t * K + rank] = pos;
        const int j = l - t * K;
        if (j >= nvalid) P.tok_pos[t * K + j] = -1;
      } else {
        P.tok_pos[l] = pos;
      }
    }
    if (tid == 0) {
      P.hdr[0] = tot[0];
      P.hdr[1] = tot[1];
      P.hdr[2] = tot[2];
      if (A.po.num_pos) *A.po.num_pos = tot[2];
    }
    if (A.po.pos_to_expert) {
      __syncthreads();
      for (int p2 = tot[2] + tid; p2 < npairs; p2 += blockDim.x) A.po.pos_to_expert[p2] = -1;
    }
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
  pdl_trigger();
  pdl_wait();
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
// Fused norm + route + plan (token mode, T <= 8): one thread-block cluster of
// E/16 CTAs replaces the layer's RMSNorm, the router's two phases (or the hash
// lookup) and the plan kernel. CTA r stages the gate rows of experts
// [16r, 16r+16) and the norm weight with bulk copies (before the PDL wait:
// they do not depend on the previous kernel), then the T rows. When a norm
// weight is given the rows are the residual stream h and every CTA normalises
// them (utils.py:6-9, the sums in the order of the standalone norm kernel, so
// both give identical rows); otherwise they arrive normed. CTA r computes the
// logits of its 16 experts with the router's own arithmetic (logit_chunk, the
// same k-split order), their scores and selection keys, and sends the keys to
// CTA 0 through distributed shared memory; CTA 0 runs the router's top-k
// (identical selections and weights) or reads the hash table
// (engine.py:1018-1023), and builds the token-mode plan; every CTA writes its
// slice of the normed rows and of their hi/lo split.
// Reference: router.py:22-36 (routing), fused_moe.py:458-517 (the union of
// experts the FFN runs).
// ---------------------------------------------------------------------------
constexpr int kRouteThreads = kNormThreads;  // the norm's thread layout (256)
constexpr int kRouteMaxD = 4096;  // 16 gate rows + 8 token rows of D in shared memory

struct RouteArgs {
  const __nv_bfloat16* x;       // [T][D] rows: the residual stream (norm_w given) or normed rows
  const __nv_bfloat16* norm_w;  // [D] RMSNorm weight, or nullptr (rows already normed)
  float eps;
  __nv_bfloat16* x_out;         // [T][D] normed rows, or nullptr
  const __nv_bfloat16* gate;    // [E_router][D] (router mode)
  const __nv_bfloat16* bias;    // [E_router] or nullptr
  const int64_t* ids;           // [T] token ids (hash mode)
  const int64_t* tid2eid;       // [V][K]: hash mode when not nullptr
  int64_t V;
  int T, D, E, K;               // E = router experts (E/16 CTAs)
  float scaling;                // routed scaling factor (router mode) or the weight 1/K (hash mode)
  int dup_mode;
  int offset, held;             // this store holds routed experts [offset, offset + held)
  int64_t* idx_out;             // [T][K] global expert ids
  float* w_out;                 // [T][K]
  uint32_t* ucount;             // tickets to clear
  int64_t n_ucount;
  int64_t n_ctab;               // token tables to clear (C_max * 8)
  int64_t P_max;                // x8 plane stride in rows
  int32_t* status;
  // chained expert parallelism: before routing, complete the previous call's
  // peer-memory exchange into the rows (h <- h + bf16(bf16(routed) [+
  // bf16(shared)]), in place in h_chain and in every CTA's row buffer)
  uint8_t* ep_buf;              // this rank's exchange buffer, or nullptr (no chain)
  __nv_bfloat16* h_chain;       // [T][D] the residual rows (x, written in place)
  int ep_world, chain_shared;
  uint64_t wait_ns;
};

// Shared memory of the route kernel. Gate and token rows are stored with a
// 64-byte pad per row, so consecutive rows start in opposite halves of the
// banks and the MMA fragment loads (8 rows x 16 bytes per quarter warp) are
// conflict-free.
struct RouteSmem {
  static constexpr int stride(int D) { return D + 32; }  // bf16 elements per stored row
  static constexpr size_t gw(int) { return 0; }
  static constexpr size_t xs(int D) { return static_cast<size_t>(16) * stride(D) * 2; }
  static constexpr size_t nw(int D) { return xs(D) + static_cast<size_t>(8) * stride(D) * 2; }
  static constexpr size_t red(int D) { return nw(D) + static_cast<size_t>(D) * 2; }  // [split <= 8][lane][4] f32
  static constexpr size_t keys(int D) { return red(D) + 8 * 32 * 4 * 4; }            // CTA 0: [token][expert] u32
  static constexpr size_t top(int D) { return keys(D) + 8 * 256 * 4; }
  static constexpr size_t bar(int D) { return top(D) + 8 * 16 * (8 + 4) + 32 + 32 + 64 + 32 + 256 + 256; }
  static constexpr size_t bytes(int D) { return bar(D) + 16; }
};
static_assert(RouteSmem::bytes(kRouteMaxD) <= 232448, "route kernel shared memory");

// Selection key of a score: the score's bits plus one (scores are >= 0, so
// bit order is value order; 0 marks a taken or absent expert), NaN above all.
// Ties go to the lower expert id, as the router's 64-bit keys order them.
__device__ __forceinline__ uint32_t score_key32(float s) {
  return isnan(s) ? 0xffffffffu : __float_as_uint(s) + 1u;
}
__device__ __forceinline__ float key32_score(uint32_t k) {
  return __uint_as_float(k == 0xffffffffu ? k : k - 1u);
}

__global__ void __launch_bounds__(kRouteThreads, 1) route_plan_kernel(RouteArgs A, Plan P,
                                                                      const __grid_constant__ Desc d) {
  extern __shared__ __align__(128) uint8_t rs[];
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = static_cast<int>(cluster.block_rank());
  const int ncta = static_cast<int>(cluster.num_blocks());
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int T = A.T, D = A.D, E = A.E, K = A.K;
  const bool hash = A.tid2eid != nullptr;
  const bool norm = A.norm_w != nullptr;
  const int RS = RouteSmem::stride(D);
  __nv_bfloat16* gw = reinterpret_cast<__nv_bfloat16*>(rs + RouteSmem::gw(D));
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(rs + RouteSmem::xs(D));
  __nv_bfloat16* nw = reinterpret_cast<__nv_bfloat16*>(rs + RouteSmem::nw(D));
  float* red = reinterpret_cast<float*>(rs + RouteSmem::red(D));
  uint32_t* keys = reinterpret_cast<uint32_t*>(rs + RouteSmem::keys(D));
  int64_t* sI = reinterpret_cast<int64_t*>(rs + RouteSmem::top(D));  // [T][K] selections
  float* sW = reinterpret_cast<float*>(sI + 8 * 16);                 // [T][K] weights
  uint32_t* emask = reinterpret_cast<uint32_t*>(sW + 8 * 16);         // 256-bit expert bitmap (CTA 0)
  int* rowe = reinterpret_cast<int*>(emask + 8);                      // [8] row prescale exponents
  float* biasv = reinterpret_cast<float*>(rowe + 8);                  // [16] this CTA's biases
  float* wpart = biasv + 16 + 8;                                      // [8 warps][8 rows] sums of squares
  float* wmax = wpart + 64;                                           // [8 warps][8 rows] max |x|
  uint64_t* bar = reinterpret_cast<uint64_t*>(rs + RouteSmem::bar(D));
  const int e0 = rank * 16;
  const uint32_t rowb = static_cast<uint32_t>(D) * 2;
  const int nv = D / 8;  // 16-byte vectors per row
  // CTAs that write the hi/lo split of the rows (and need each row's prescale
  // exponent): every rank but 0 (rank 1 also takes rank 0's slice)
  const bool split_rows = rank != 0 || ncta == 1;

  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  HS_TRACE_SLOT_ROUTE(hs_tslot);
  if (tid == 0) HS_STAMP(hs_tslot, ::hs::trace::kRoute, rank, 0);
  const bool chain = A.ep_buf != nullptr;
  // the chained exchange stores into every CTA's row buffer: each CTA arrives
  // once it runs and waits for the others before the first such store
  if (chain) asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  if (tid == 0) {  // parameters do not depend on the previous kernel: start them now
    mbar_arrive_expect_tx(bar, rowb * ((hash ? 0 : 16) + (norm ? 1 : 0) + (chain ? 0 : T)));
    if (!hash)
      for (int r = 0; r < 16; ++r) bulk_load(gw + r * RS, A.gate + static_cast<int64_t>(e0 + r) * D, rowb, bar);
    if (norm) bulk_load(nw, A.norm_w, rowb, bar);
  }
  if (tid < 16) biasv[tid] = (!hash && A.bias) ? __bfloat162float(A.bias[e0 + tid]) : 0.f;
  pdl_trigger();
  pdl_wait();  // the rows (and everything earlier) are complete
  if (tid == 0) HS_STAMP(hs_tslot, ::hs::trace::kRoute, rank, 1);
  if (chain) {
    // The previous call's exchange: this CTA sums every rank's routed and
    // shared rows of its column slice (ranks in order from 0: identical bits
    // on every rank, the same as ep_combine_kernel), adds the residual, writes
    // the rows in place and into every cluster CTA's row buffer, and empties
    // the entries. Each entry is its own arrival flag; the wait is bounded and
    // a wait that runs out poisons the buffer, as in ep_combine_kernel.
    volatile uint64_t* hdr = reinterpret_cast<volatile uint64_t*>(A.ep_buf);
    const int slot = static_cast<int>(hdr[0] & 1u);
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
    bool bad = hdr[epx::kPoison] != 0u;
    if (bad && tid == 0) report(A.status, HS_DEV_TIMEOUT);
    const int cols = D / ncta, c0 = rank * cols, n4 = cols / 4;
    for (int u = tid; u < T * n4; u += kRouteThreads) {
      const int t = u / n4, c = c0 + 4 * (u - t * n4);
      const int64_t o = static_cast<int64_t>(t) * D + c;
      if (bad) {  // the call failed: zero rows (finite, routed like any rows) instead of stale shared memory
        for (int q = 0; q < ncta; ++q)
          *reinterpret_cast<uint2*>(cluster.map_shared_rank(xs, q) + t * RS + c) = make_uint2(0u, 0u);
        continue;
      }
      uint4 vr[HS_EP_MAX_RANKS], vs[HS_EP_MAX_RANKS];
#pragma unroll
      for (int q = 0; q < HS_EP_MAX_RANKS; ++q)
        if (q < A.ep_world) {
          vr[q] = ld_volatile_u4(epx::rows(A.ep_buf, slot, A.ep_world, q, 0, D) + o);
          vs[q] = ld_volatile_u4(epx::rows(A.ep_buf, slot, A.ep_world, q, 1, D) + o);
        }
      auto empty = [](const uint4& v) {
        return v.x == epx::kEmpty || v.y == epx::kEmpty || v.z == epx::kEmpty || v.w == epx::kEmpty;
      };
#pragma unroll
      for (int q = 0; q < HS_EP_MAX_RANKS; ++q) {
        if (q >= A.ep_world || bad) continue;
        if (empty(vr[q]) || empty(vs[q])) {
          const float* pr = epx::rows(A.ep_buf, slot, A.ep_world, q, 0, D) + o;
          const float* ps = epx::rows(A.ep_buf, slot, A.ep_world, q, 1, D) + o;
          const uint64_t w0 = globaltimer_ns();
          for (uint32_t it = 1; empty(vr[q]) || empty(vs[q]); ++it) {
            vr[q] = ld_volatile_u4(pr);
            vs[q] = ld_volatile_u4(ps);
            if ((it & 63u) == 0 && (globaltimer_ns() - w0 > A.wait_ns || hdr[epx::kPoison] != 0u)) {
              report(A.status, HS_DEV_TIMEOUT);
              hdr[epx::kPoison] = 1u;
              __threadfence();
              bad = true;
              break;
            }
          }
        }
      }
      if (bad) {
        for (int q = 0; q < ncta; ++q)
          *reinterpret_cast<uint2*>(cluster.map_shared_rank(xs, q) + t * RS + c) = make_uint2(0u, 0u);
        continue;
      }
      float r[4] = {0.f, 0.f, 0.f, 0.f}, sh[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int q = 0; q < HS_EP_MAX_RANKS; ++q)
        if (q < A.ep_world) {
          const uint32_t a4[4] = {vr[q].x, vr[q].y, vr[q].z, vr[q].w}, b4[4] = {vs[q].x, vs[q].y, vs[q].z, vs[q].w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            r[j] += __uint_as_float(a4[j]);
            sh[j] += __uint_as_float(b4[j]);
          }
          const uint4 e = make_uint4(epx::kEmpty, epx::kEmpty, epx::kEmpty, epx::kEmpty);
          st_volatile_u4(epx::rows(A.ep_buf, slot, A.ep_world, q, 0, D) + o, e);
          st_volatile_u4(epx::rows(A.ep_buf, slot, A.ep_world, q, 1, D) + o, e);
        }
      const uint2 hv = *reinterpret_cast<const uint2*>(A.h_chain + o);
      const uint32_t hw[2] = {hv.x, hv.y};
      uint32_t ow[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float y0 = round_bf16(r[2 * j]), y1 = round_bf16(r[2 * j + 1]);
        if (A.chain_shared) {
          y0 += round_bf16(sh[2 * j]);
          y1 += round_bf16(sh[2 * j + 1]);
        }
        const float b0 = __bfloat162float(__float2bfloat16_rn(y0)), b1 = __bfloat162float(__float2bfloat16_rn(y1));
        const uint32_t lo = __bfloat16_as_ushort(__float2bfloat16_rn(__fadd_rn(__uint_as_float(hw[j] << 16), b0)));
        const uint32_t hi =
            __bfloat16_as_ushort(__float2bfloat16_rn(__fadd_rn(__uint_as_float(hw[j] & 0xffff0000u), b1)));
        ow[j] = lo | (hi << 16);
      }
      const uint2 out = make_uint2(ow[0], ow[1]);
      *reinterpret_cast<uint2*>(A.h_chain + o) = out;
      for (int q = 0; q < ncta; ++q)
        *reinterpret_cast<uint2*>(cluster.map_shared_rank(xs, q) + t * RS + c) = out;
    }
    cluster.sync();  // every CTA's rows complete (and every poison store seen)
    if (rank == 0 && tid == 0 && hdr[epx::kPoison] == 0u) hdr[0] = hdr[0] + 1u;
  } else if (tid == 0) {
    for (int t = 0; t < T; ++t) bulk_load(xs + t * RS, A.x + static_cast<int64_t>(t) * D, rowb, bar);
  }
  // clear this kernel's share of the tickets and token tables meanwhile
  for (int64_t i = static_cast<int64_t>(rank) * kRouteThreads + tid; i < A.n_ucount;
       i += static_cast<int64_t>(ncta) * kRouteThreads)
    A.ucount[i] = 0u;
  for (int64_t i = static_cast<int64_t>(rank) * kRouteThreads + tid; i < A.n_ctab;
       i += static_cast<int64_t>(ncta) * kRouteThreads) {
    P.ctab_wb[i] = 0.f;
  }
  if (rank == 0) {
    if (tid < 8) emask[tid] = 0u;
    if (hash && tid < T * K) {  // hash routing: tid2eid[id], weight 1/K (engine.py:1018-1023)
      const int t = tid / K, j = tid - t * K;
      const int64_t id = A.ids[t];
      int64_t e = -1;
      if (id < 0 || id >= A.V)
        report(A.status, HS_DEV_BAD_TOKEN);
      else
        e = A.tid2eid[id * K + j];
      const float hw = A.scaling;  // hash mode: the host passes 1/K
      A.idx_out[tid] = e;
      A.w_out[tid] = hw;
      if (e >= E) {
        report(A.status, HS_DEV_BAD_EXPERT);
        e = -1;
      }
      sI[tid] = e;
      sW[tid] = hw;
    }
  }
  bool ok = mbar_wait(bar, 0);
  if (!ok) {  // report, and let the copies land before the shared memory is reused or released
    report(A.status, HS_DEV_TIMEOUT);
    (void)mbar_wait(bar, 0);
  }
  ok = __syncthreads_and(ok) != 0;  // uniform over the CTA (barriers follow)
  if (tid == 0) HS_STAMP(hs_tslot, ::hs::trace::kRoute, rank, 2);

  // ---- RMSNorm of every row (the standalone norm kernel's summation order),
  // and each normed row's max |x| for its prescale exponent; rows in groups
  // of four so their load, add and shuffle chains overlap ----
  if (norm && ok) {
    for (int t0 = 0; t0 < T; t0 += 4) {
      float ss[4] = {0.f, 0.f, 0.f, 0.f};
      for (int j = tid; j < nv; j += kRouteThreads) {
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (t0 + q < T) {
            float v[8];
            bf16x8_unpack(reinterpret_cast<const uint4*>(xs + (t0 + q) * RS)[j], v);
#pragma unroll
            for (int k = 0; k < 8; ++k) ss[q] = __fadd_rn(ss[q], __fmul_rn(v[k], v[k]));
          }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int q = 0; q < 4; ++q) ss[q] = __fadd_rn(ss[q], __shfl_xor_sync(0xffffffffu, ss[q], o));
      if (lane == 0)
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (t0 + q < T) wpart[warp * 8 + t0 + q] = ss[q];
    }
    __syncthreads();
    // 1 / rms of row t in lane t of every warp: each warp adds the warps'
    // partials itself, so no second barrier
    float ri_l = 0.f;
    if (lane < T) {
      float tot = 0.f;
      for (int w = 0; w < kRouteThreads / 32; ++w) tot = __fadd_rn(tot, wpart[w * 8 + lane]);
      const float var = __fdiv_rn(tot, static_cast<float>(D));
      ri_l = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(var, A.eps)));
    }
    const uint4* wv = reinterpret_cast<const uint4*>(nw);
    for (int t0 = 0; t0 < T; t0 += 4) {
      float mx[4] = {0.f, 0.f, 0.f, 0.f}, rq[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) rq[q] = __shfl_sync(0xffffffffu, ri_l, (t0 + q) & 31);
      for (int j = tid; j < nv; j += kRouteThreads) {
        float wf[8];
        bf16x8_unpack(wv[j], wf);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (t0 + q < T) {
            uint4* row = reinterpret_cast<uint4*>(xs + (t0 + q) * RS);
            float v[8];
            bf16x8_unpack(row[j], v);
#pragma unroll
            for (int k = 0; k < 8; ++k) v[k] = __fmul_rn(wf[k], __fmul_rn(v[k], rq[q]));
            const uint4 pk = bf16x8_pack(v);
            row[j] = pk;
            if (split_rows) {
              bf16x8_unpack(pk, v);
#pragma unroll
              for (int k = 0; k < 8; ++k) mx[q] = fmaxf(mx[q], fabsf(v[k]));
            }
          }
      }
      if (split_rows) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
          for (int q = 0; q < 4; ++q) mx[q] = fmaxf(mx[q], __shfl_xor_sync(0xffffffffu, mx[q], o));
        if (lane == 0)
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if (t0 + q < T) wmax[warp * 8 + t0 + q] = mx[q];
      }
    }
    __syncthreads();
    if (split_rows && tid < T) {
      float mx = 0.f;
      for (int w = 0; w < kRouteThreads / 32; ++w) mx = fmaxf(mx, wmax[w * 8 + tid]);
      rowe[tid] = row_prescale(mx);
    }
  } else if (split_rows && warp < T) {  // rows arrive normed: the prescale from them, one warp per token
    const uint4* row = reinterpret_cast<const uint4*>(xs + warp * RS);
    float mx = 0.f;
    for (int v = lane; v < nv; v += 32) {
      float f[8];
      bf16x8_unpack(row[v], f);
#pragma unroll
      for (int i = 0; i < 8; ++i) mx = fmaxf(mx, fabsf(f[i]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) rowe[warp] = row_prescale(mx);
  }

  if (tid == 0) HS_STAMP(hs_tslot, ::hs::trace::kRoute, rank, 3);
  // ---- logits: warp s sums the four 128-column quarters of k-split s in order ----
  const int nsplit = D / router::kKSplitCols;
  if (!hash && ok && warp < nsplit) {
    const int g = lane >> 2;
    float acc[4][4], s4[4];
    router::logit_chunk4(gw + g * RS, gw + (g + 8) * RS, xs + (g < T ? g : 0) * RS, g < T,
                         warp * router::kKSplitCols, acc);
#pragma unroll
    for (int j = 0; j < 4; ++j) s4[j] = ((acc[0][j] + acc[1][j]) + acc[2][j]) + acc[3][j];
#pragma unroll
    for (int j = 0; j < 4; ++j) red[(warp * 32 + lane) * 4 + j] = s4[j];
  }
  __syncthreads();
  // (expert, token) of the 16 x 8 fragment: the logit (k-splits in order), its
  // score sqrt(softplus(bf16(bf16(l) + bias))) and selection key, to CTA 0
  if (!hash && tid < 128) {
    const int ln = tid & 31, j = tid >> 5;
    const int el = (ln >> 2) + ((j & 2) ? 8 : 0), t = 2 * (ln & 3) + (j & 1);
    float l = 0.f;
    for (int sp = 0; sp < nsplit; ++sp) l += red[(sp * 32 + ln) * 4 + j];
    float lb = round_bf16(l);
    if (A.bias) lb = round_bf16(lb + biasv[el]);
    const float sp = lb > 20.f ? lb : log1pf(expf(lb));
    const float sc = sqrtf(sp);
    if (t < T) cluster.map_shared_rank(keys, 0)[t * 256 + e0 + el] = score_key32(sc);
  }
  cluster.sync();
  if (tid == 0) HS_STAMP(hs_tslot, ::hs::trace::kRoute, rank, 4);

  // ---- the normed rows and their hi/lo e4m3 split, column slice by slice: off
  // CTA 0's critical path (rank 1 also takes rank 0's slice) ----
  if (split_rows) {
    const int cols = D / ncta;
    for (int sl = (rank == 1 ? 0 : rank); sl <= rank; ++sl) {
      const int c16 = sl * cols / 16;
      for (int i = tid; i < T * (cols / 16); i += kRouteThreads) {
        const int t = i / (cols / 16), k16 = c16 + (i - t * (cols / 16));
        const uint4* src = reinterpret_cast<const uint4*>(xs + t * RS);
        uint4 hv, lv;
        split16(src[2 * k16], src[2 * k16 + 1], exp2i(rowe[t]), hv, lv);
        reinterpret_cast<uint4*>(P.x8 + static_cast<int64_t>(t) * D)[k16] = hv;
        reinterpret_cast<uint4*>(P.x8 + (A.P_max + t) * D)[k16] = lv;
        if (A.x_out) {
          uint4* xo = reinterpret_cast<uint4*>(A.x_out + static_cast<int64_t>(t) * D);
          xo[2 * k16] = src[2 * k16];
          xo[2 * k16 + 1] = src[2 * k16 + 1];
        }
      }
    }
    if ((rank == 1 || ncta == 1) && tid < T) {
      P.sb1[tid] = static_cast<uint8_t>(127 - rowe[tid]);
      P.tok_e[tid] = rowe[tid];
    }
    if (rank != 0) {
      if (tid == 0) HS_STAMP(hs_tslot, ::hs::trace::kRoute, rank, 5);
      return;
    }
  }

  // ---- CTA 0: the router's top-k selection from the gathered keys ----
  if (!hash && warp < T) {
    const int t = warp;
    uint32_t key[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = lane + 32 * i;
      key[i] = e < E ? keys[t * 256 + e] : 0u;
    }
    float wsum = 0.f, wsel = 0.f;
    int esel = 0;
#pragma unroll 1
    for (int r = 0; r < K; ++r) {
      // this lane's best (the lowest id among equal keys), then the warp's
      uint32_t best = 0u;
      int be = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (key[i] > best) {
          best = key[i];
          be = lane + 32 * i;
        }
      const uint32_t m = __reduce_max_sync(0xffffffffu, best);
      const int e = __reduce_min_sync(0xffffffffu, (best == m && m != 0u) ? be : 0x7fffffff);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (lane + 32 * i == e) key[i] = 0u;
      const float s = key32_score(m);
      wsum += s;  // selection order, as the router
      if (lane == r) {
        wsel = s;
        esel = e;
      }
    }
    const float denom = fmaxf(wsum, 1e-20f);
    if (lane < K) {
      const float wv = (wsel / denom) * A.scaling;
      sI[t * K + lane] = esel;
      sW[t * K + lane] = wv;
      A.idx_out[t * K + lane] = esel;
      A.w_out[t * K + lane] = wv;
    }
  }
  __syncthreads();
  if (tid == 0) HS_STAMP(hs_tslot, ::hs::trace::kRoute, 0, 6);

  // ---- CTA 0: the token-mode plan, one thread per (token, slot) pair ----
  // (compact loops: this code runs once per call on one SM, so its
  // instructions are fetched cold; fewer of them beat unrolled selections)
  const int npairs = T * K;
  int le = -1;
  float ws = 0.f;
  if (tid < npairs) {
    const int t = tid / K, j = tid - t * K;
    auto local = [&](int jj) {
      const int64_t e = sI[t * K + jj] - A.offset;
      return (e < 0 || e >= A.held) ? -1 : static_cast<int>(e);
    };
    le = local(j);
    if (le >= 0) {
      bool dropped = false;
      if (A.dup_mode == HS_DUP_SUM) {  // the first slot of an expert carries the summed weight
#pragma unroll 1
        for (int jj = 0; jj < j; ++jj)
          if (local(jj) == le) dropped = true;
        if (!dropped)
#pragma unroll 1
          for (int jj = j; jj < K; ++jj)
            if (local(jj) == le) ws += sW[t * K + jj];
      } else {  // the last slot of an expert wins
#pragma unroll 1
        for (int jj = j + 1; jj < K; ++jj)
          if (local(jj) == le) dropped = true;
        ws = sW[t * K + j];
      }
      if (dropped) le = -1;
    }
    if (le >= 0) atomicOr(&emask[le >> 5], 1u << (le & 31));
  }
  __syncthreads();
  if (tid == 0) HS_STAMP(hs_tslot, ::hs::trace::kRoute, 0, 7);
  uint32_t em[8];
#pragma unroll
  for (int w = 0; w < 8; ++w) em[w] = emask[w];
  if (tid < npairs && le >= 0) {
    const int t = tid / K;
    int cb = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const uint32_t ew = em[w];
      const uint32_t m = w < (le >> 5) ? ew : (w == (le >> 5) ? (ew & ((1u << (le & 31)) - 1u)) : 0u);
      cb += __popc(m);
    }
    const float wb = round_bf16(ws);
    P.ctab_wb[cb * 8 + t] = wb;
    P.chunk_expert[cb] = le;
    P.chunk_pair0[cb] = 0;
    P.chunk_np[cb] = 0;
  }
  if (tid == 0) {
    int C = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) C += __popc(em[w]);
    P.hdr[0] = C;
    P.hdr[1] = C;
    P.hdr[2] = 0;
    HS_STAMP(hs_tslot, ::hs::trace::kRoute, 0, 5);
    HS_TRACE_NEXT_CALL();
  }
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
  float* shared_f32;     // partials mode: the shared expert's f32 output (or nullptr)
  int partials;          // 1: write un-rounded f32 routed / shared sums only (no bf16 out)
  // token-mode down phase: the layer's residual add, resid_out = bf16(resid +
  // out) (engine.py:2685; resid_out may alias resid); out may then be nullptr
  const __nv_bfloat16* resid;
  __nv_bfloat16* resid_out;
  int32_t* status;
  // stream-K schedule
  int G;                 // persistent CTAs (kCtasPerSm per SM)
  int aligned;           // 1: CTA boundaries on unit boundaries (many units), 0: split units
  uint32_t* ucount;      // [U_max] per-unit tickets, cleared by the plan kernel
  float* part;           // [(U_max + G)][slot] partial accumulators
  int64_t act_rows;      // rows per activation plane (P_max, or (1 + C_max) * 8 in token mode)
  int ncl;               // token-mode down phase on clusters: CTAs per cluster (one cluster per tile)
  // schedule weight of a shared-expert k-step against a routed one: 2 when
  // both stream from HBM (FP8 is twice the bytes of FP4), 1 when the shared
  // expert was brought into L2 beforehand (token mode) and a step costs the
  // same MMA issue time either way
  int w_sh;
  // non-token mode, many tokens: the down phase only writes the per-pair rows
  // and combine_rows_kernel sums them afterwards over the whole grid (the
  // in-kernel per-tile finalize is one CTA per 128-row tile of D)
  int ext_combine;
  // expert parallelism over peer memory (hs_moe_layer_fp4_ep): the cluster
  // down epilogue stores this rank's rows into every rank's receive buffer
  int ep_rank, ep_world;  // ep_world 0: off
  uint8_t* ep_recv[HS_EP_MAX_RANKS];
};

template <int NT, int BOXES, int NBSF = 1>
struct SmemLayout {
  static constexpr int kA = 2 * kBoxBytes;             // two weight boxes per stage
  static constexpr int kB = BOXES * 2 * NT * 1024;     // hi and lo atoms per k-box
  static constexpr int kSF = 2 * 512 + NBSF * 512;     // two A scale atoms + NBSF B scale atoms
  static constexpr int kStage = kA + kB + kSF;
  static constexpr int kBarBytes = 256;
  static constexpr int kFit = (kSmemPerCta - kBarBytes) / kStage;
  static constexpr int kNumStages = kFit < 4 ? kFit : 4;
  static constexpr int kBytes = kNumStages * kStage + kBarBytes;  // stages at the 1024-aligned base
};

struct Bars {
  uint64_t full[4];
  uint64_t empty[4];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t mma_done;
  uint64_t pub;  // stream-K: the epilogue's partial rows of a split unit are stored (128 arrivals)
  uint32_t tmem;
  int32_t flag;
  int32_t issued, consumed;  // TMA stages issued by the producer / consumed by the MMA issuer
};

constexpr int64_t kMinW = 4;  // least weight per CTA of a stream-K phase (above: fewer CTAs)
constexpr int kFinishNlMaxT = 4;  // token mode: T up to this takes the warmed, non-inlined activation epilogue

// Stream-K schedule over one phase. Units (chunk x 128-row tile) are laid end
// to end as k-steps, shared-expert units first; a step of an FP8 unit weighs
// 2 (twice the bytes of an FP4 step). CTA c owns steps [lo(c), lo(c+1)).
struct Sched {
  int64_t n_sh_units, n_rt_units, U;
  int nk_sh, nk_rt, w_sh;
  int64_t S_sh, S, W_sh, W;
  int G, aligned;

  __device__ __forceinline__ int64_t ustart(int64_t u) const {
    return u < n_sh_units ? u * nk_sh : S_sh + (u - n_sh_units) * nk_rt;
  }
  __device__ __forceinline__ int unk(int64_t u) const { return u < n_sh_units ? nk_sh : nk_rt; }
  __device__ __forceinline__ int64_t unit_of(int64_t s) const {
    return s < S_sh ? s / nk_sh : n_sh_units + (s - S_sh) / nk_rt;
  }
  // first step at or after weight position w
  __device__ __forceinline__ int64_t step_at(int64_t w) const {
    if (w <= W_sh) return (w + w_sh - 1) / w_sh;
    return S_sh + (w - W_sh);
  }
  // weight position where step s starts
  __device__ __forceinline__ int64_t wpos(int64_t s) const {
    return s < S_sh ? s * w_sh : W_sh + (s - S_sh);
  }
  __device__ __forceinline__ int64_t lo(int c) const {
    if (c >= G) return S;
    if (aligned) return ustart(udiv(U * c, G));
    return step_at(udiv(W * c, G));
  }
  // The CTA whose range holds step s: the largest c with lo(c) <= s. With
  // lo(c) = step_at(floor(W c / G)), lo(c) <= s <=> floor(W c / G) <= wpos(s)
  // <=> c <= (G (wpos(s) + 1) - 1) / W (and likewise over units when aligned).
  __device__ __forceinline__ int cta_of(int64_t s) const {
    const int64_t c = aligned ? udiv(static_cast<int64_t>(G) * (unit_of(s) + 1) - 1, U)
                              : udiv(static_cast<int64_t>(G) * (wpos(s) + 1) - 1, W);
    return c < G - 1 ? static_cast<int>(c) : G - 1;
  }
  // non-negative division, 32-bit when both operands fit
  __device__ __forceinline__ static int64_t udiv(int64_t a, int64_t b) {
    if (((a | b) >> 32) == 0) return static_cast<uint32_t>(a) / static_cast<uint32_t>(b);
    return a / b;
  }
};

__device__ __forceinline__ int64_t min64(int64_t x, int64_t y) { return x < y ? x : y; }

__device__ __forceinline__ Sched make_sched(const Desc& d, const UnitArgs& a, bool down) {
  Sched s;
  const int tiles_sh = down ? d.D / kM : (d.has_shared ? d.I_sh / kM : 0);
  const int tiles_rt = down ? d.D / kM : d.I / kM;
  s.n_sh_units = static_cast<int64_t>(a.n_sh_chunks) * tiles_sh;
  s.n_rt_units = static_cast<int64_t>(__ldcg(a.P.hdr)) * tiles_rt;
  s.U = s.n_sh_units + s.n_rt_units;
  s.nk_sh = down ? (d.has_shared ? d.I_sh / 256 : 1) : d.D / 128;
  s.nk_rt = down ? d.I / 256 : d.D / 128;
  s.w_sh = a.w_sh;
  s.S_sh = s.n_sh_units * s.nk_sh;
  s.S = s.S_sh + s.n_rt_units * s.nk_rt;
  s.W_sh = s.S_sh * s.w_sh;
  s.W = s.W_sh + s.n_rt_units * s.nk_rt;
  // A unit's finisher sums the partial rows of every other CTA on it, one L2
  // round trip per few CTAs; with little work in the phase (an expert-parallel
  // rank whose only unit is its slice of the shared expert) spreading it over
  // all CTAs would split a 32-step unit over ~70 CTAs. The steps go to the
  // first W / kMinW CTAs instead (at least kMinW weight each), the rest idle.
  s.G = a.G;
  if (!a.aligned && s.W < static_cast<int64_t>(a.G) * kMinW)
    s.G = static_cast<int>(s.W / kMinW > 1 ? s.W / kMinW : 1);
  s.aligned = a.aligned;
  return s;
}

struct UnitInfo {
  int shared, e, pair0, np, tile, chunk;
};

__device__ __forceinline__ UnitInfo unit_info(const Desc& d, const UnitArgs& a, const Sched& s, int64_t u, bool down) {
  UnitInfo r;
  const int tiles_sh = down ? d.D / kM : (d.has_shared ? d.I_sh / kM : 1);
  const int tiles_rt = down ? d.D / kM : d.I / kM;
  if (u < s.n_sh_units) {
    const int c = static_cast<int>(u / tiles_sh);
    r.shared = 1;
    r.chunk = c;
    r.tile = static_cast<int>(u - static_cast<int64_t>(c) * tiles_sh);
    r.e = 0;
    r.pair0 = c * a.CH;
    r.np = min(a.CH, a.T - r.pair0);
  } else {
    const int64_t uu = u - s.n_sh_units;
    const int c = static_cast<int>(uu / tiles_rt);
    r.shared = 0;
    r.chunk = c;
    r.tile = static_cast<int>(uu - static_cast<int64_t>(c) * tiles_rt);
    // through L2: after the route kernel the plan may come from a grid that is
    // still running (a counter hand-off, not grid completion)
    r.e = __ldcg(a.P.chunk_expert + c);
    r.pair0 = __ldcg(a.P.chunk_pair0 + c);
    r.np = __ldcg(a.P.chunk_np + c);
  }
  return r;
}

// out[t][tile rows] = bf16( bf16(sum of the token's routed partial rows in
// ascending expert order) + bf16(shared-expert row) ), for every token; run
// by the 128 epilogue threads.
// Positions are ascending with -1 padding at the end; all K loads of a row
// are issued before the in-order sum, so they overlap.
__device__ __forceinline__ void finalize_tile(const UnitArgs& a, int D, int tile, int tid, int nthr) {
  for (int i = tid; i < a.T * kM; i += nthr) {
    const int t = i / kM;
    const int dd = tile * kM + (i - t * kM);
    const int32_t* pos = a.P.tok_pos + static_cast<int64_t>(t) * a.K;
    int p[16];
    float v[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) p[j] = j < a.K ? __ldcg(pos + j) : -1;
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = p[j] >= 0 ? __ldcg(a.P.out_part + static_cast<int64_t>(p[j]) * D + dd) : 0.f;
    float r = 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (p[j] >= 0) r += v[j];
    const int64_t o_i = static_cast<int64_t>(t) * D + dd;
    const float sh = a.use_shared ? __ldcg(a.P.out_part + o_i) : 0.f;  // the shared pair row of token t
    if (a.out_f32) a.out_f32[o_i] = r;
    if (a.partials) {
      if (a.shared_f32) a.shared_f32[o_i] = sh;
      continue;
    }
    float o = round_bf16(r);
    if (a.use_shared) o += round_bf16(sh);
    a.out[o_i] = __float2bfloat16_rn(o);
  }
}

// finalize_tile over the whole output, eight elements per thread and the
// same per-element order: out[t][d] from the token's per-pair rows (positions
// ascending) and its shared-expert row. Runs after the down phase.
__global__ void __launch_bounds__(256) combine_rows_kernel(UnitArgs a, int D) {
  pdl_trigger();
  pdl_wait();
  const int64_t nv = static_cast<int64_t>(a.T) * (D / 8);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < nv;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(i / (D / 8));
    const int dd = static_cast<int>(i - static_cast<int64_t>(t) * (D / 8)) * 8;
    float r[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < a.K; ++j) {
      const int p = __ldcg(a.P.tok_pos + static_cast<int64_t>(t) * a.K + j);
      if (p < 0) continue;
      const float4* src = reinterpret_cast<const float4*>(a.P.out_part + static_cast<int64_t>(p) * D + dd);
      const float4 v0 = __ldcg(src), v1 = __ldcg(src + 1);
      r[0] += v0.x, r[1] += v0.y, r[2] += v0.z, r[3] += v0.w;
      r[4] += v1.x, r[5] += v1.y, r[6] += v1.z, r[7] += v1.w;
    }
    const int64_t o_i = static_cast<int64_t>(t) * D + dd;
    float sh[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (a.use_shared) {
      const float4* src = reinterpret_cast<const float4*>(a.P.out_part + o_i);  // the token's shared row
      const float4 v0 = __ldcg(src), v1 = __ldcg(src + 1);
      sh[0] = v0.x, sh[1] = v0.y, sh[2] = v0.z, sh[3] = v0.w, sh[4] = v1.x, sh[5] = v1.y, sh[6] = v1.z, sh[7] = v1.w;
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (a.out_f32) a.out_f32[o_i + k] = r[k];
      if (a.partials) {
        if (a.shared_f32) a.shared_f32[o_i + k] = sh[k];
        continue;
      }
      float o = round_bf16(r[k]);
      if (a.use_shared) o += round_bf16(sh[k]);
      a.out[o_i + k] = __float2bfloat16_rn(o);
    }
  }
}

// Peer-memory exchange, consumer side: per element, wait (bounded by
// limit_ns) until every rank's routed and shared entries of this call have
// arrived in the local buffer, then h_out = bf16(h + bf16(bf16(sum_q
// routed_q) + bf16(sum_q shared_q))), ranks summed in order from 0 (identical
// on every rank), and the entries are emptied again; the last CTA advances
// the local call counter. A wait that runs out poisons the buffer instead:
// the counter stays, so entries a late peer stores afterwards sit in a slot
// no later call reads, and every later call reports HS_DEV_TIMEOUT at once.
__global__ void __launch_bounds__(256) ep_combine_kernel(uint8_t* buf, int world, int T, int D, int use_shared,
                                                         const __nv_bfloat16* h, __nv_bfloat16* h_out,
                                                         int32_t* status, uint64_t limit_ns) {
  pdl_trigger();
  HS_TRACE_T(hs_t0);
  pdl_wait();
  HS_TRACE_SLOT(hs_tslot);
  if (threadIdx.x == 0) {
    HS_STAMP_AT(hs_tslot, ::hs::trace::kCombine, blockIdx.x, 0, hs_t0);
    HS_STAMP(hs_tslot, ::hs::trace::kCombine, blockIdx.x, 1);
  }
  uint64_t* hdr = reinterpret_cast<uint64_t*>(buf);
  volatile uint64_t* poison = reinterpret_cast<volatile uint64_t*>(hdr + epx::kPoison);
  if (*poison != 0u) {  // an earlier call gave up: nothing here can be trusted
    if (threadIdx.x == 0) report(status, HS_DEV_TIMEOUT);
    return;
  }
  const uint64_t k = *reinterpret_cast<volatile const uint64_t*>(hdr);
  const int slot = static_cast<int>(k & 1u);
  const int64_t n = static_cast<int64_t>(T) * D;
  bool timed_out = false;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t o = i;  // token-major [8][D] rows: entry (t, d) of this call's T x D output
    // every rank's two entries are read at once (one round trip when they have
    // all arrived); only missing ones are polled again
    uint32_t vr[HS_EP_MAX_RANKS], vs[HS_EP_MAX_RANKS];
#pragma unroll
    for (int q = 0; q < HS_EP_MAX_RANKS; ++q)
      if (q < world) {
        vr[q] = *reinterpret_cast<volatile uint32_t*>(epx::rows(buf, slot, world, q, 0, D) + o);
        vs[q] = *reinterpret_cast<volatile uint32_t*>(epx::rows(buf, slot, world, q, 1, D) + o);
      }
#pragma unroll
    for (int q = 0; q < HS_EP_MAX_RANKS; ++q) {
      if (q >= world || timed_out) continue;
      if (vr[q] == epx::kEmpty || vs[q] == epx::kEmpty) {
        volatile uint32_t* pr = reinterpret_cast<volatile uint32_t*>(epx::rows(buf, slot, world, q, 0, D) + o);
        volatile uint32_t* ps = reinterpret_cast<volatile uint32_t*>(epx::rows(buf, slot, world, q, 1, D) + o);
        const uint64_t t0 = globaltimer_ns();
        for (uint32_t it = 1; vr[q] == epx::kEmpty || vs[q] == epx::kEmpty; ++it) {
          vr[q] = *pr;
          vs[q] = *ps;
          if ((it & 63u) == 0 && (globaltimer_ns() - t0 > limit_ns || *poison != 0u)) {
            report(status, HS_DEV_TIMEOUT);
            *poison = 1u;
            __threadfence();
            timed_out = true;
            break;
          }
        }
      }
    }
    if (timed_out) break;
    float r = 0.f, sh = 0.f;
#pragma unroll
    for (int q = 0; q < HS_EP_MAX_RANKS; ++q)
      if (q < world) {  // ranks summed in order from 0: identical bits on every rank
        r += __uint_as_float(vr[q]);
        sh += __uint_as_float(vs[q]);
        *reinterpret_cast<volatile uint32_t*>(epx::rows(buf, slot, world, q, 0, D) + o) = epx::kEmpty;
        *reinterpret_cast<volatile uint32_t*>(epx::rows(buf, slot, world, q, 1, D) + o) = epx::kEmpty;
      }
    float y = round_bf16(r);
    if (use_shared) y += round_bf16(sh);
    const float yb = __bfloat162float(__float2bfloat16_rn(y));
    h_out[i] = __float2bfloat16_rn(__fadd_rn(__bfloat162float(h[i]), yb));
  }
  if (threadIdx.x == 0) HS_STAMP(hs_tslot, ::hs::trace::kCombine, blockIdx.x, 2);
  // The last CTA advances the call counter unless a wait ran out. Only the
  // poison word needs ordering here: a CTA that poisoned fences before its
  // ticket, the last CTA fences after its own (acquire) before it reads the
  // word. Everything else this call wrote is seen by the next call through
  // grid completion (its kernels wait for this one).
  const bool poisoned_here = __syncthreads_or(timed_out) != 0;
  if (threadIdx.x == 0) {
    if (poisoned_here) __threadfence();
    if (atomicAdd(reinterpret_cast<unsigned int*>(hdr + 1), 1u) == gridDim.x - 1) {
      *reinterpret_cast<volatile unsigned int*>(hdr + 1) = 0u;
      __threadfence();
      if (*poison == 0u) *reinterpret_cast<volatile uint64_t*>(hdr) = k + 1;
    }
    HS_STAMP(hs_tslot, ::hs::trace::kCombine, blockIdx.x, 3);
  }
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// One element of the MoE output from its routed and shared f32 sums:
// bf16(bf16(routed) + bf16(shared)) (engine.py:1530-1536), and the residual
// add when the call carries one.
// res: the residual element a.resid[o_i] when the caller loaded it early.
__device__ __forceinline__ void store_out(const UnitArgs& a, int64_t o_i, float r, float h, float res) {
  if (a.out_f32) a.out_f32[o_i] = r;
  if (a.partials) {
    if (a.shared_f32) a.shared_f32[o_i] = h;
    return;
  }
  float o = round_bf16(r);
  if (a.use_shared) o += round_bf16(h);
  const __nv_bfloat16 y = __float2bfloat16_rn(o);
  if (a.out) a.out[o_i] = y;
  if (a.resid_out) a.resid_out[o_i] = __float2bfloat16_rn(__fadd_rn(res, __bfloat162float(y)));
}
__device__ __forceinline__ void store_out(const UnitArgs& a, int64_t o_i, float r, float h) {
  store_out(a, o_i, r, h, a.resid_out ? __bfloat162float(a.resid[o_i]) : 0.f);
}

// Gate/up epilogue of one 128-row unit from the summed accumulators.
template <int NT, bool kFP8>
__device__ __forceinline__ void gateup_finish(const Desc& d, const UnitArgs& a, const UnitInfo& ui, int row,
                                              const float (&g)[8 * NT], const float (&u)[8 * NT]) {
  const int64_t I_act = max(d.I, d.has_shared ? d.I_sh : 0);
  uint8_t* hi_plane = a.P.act8;
  uint8_t* lo_plane = a.P.act8 + a.act_rows * I_act;
  const int col = ui.tile * kM + row;
#pragma unroll
  for (int r = 0; r < 8 * NT; ++r) {
    if (r < ui.np) {
      const int p = ui.pair0 + r;
      // reference: gate/up rounded to bf16, SwiGLU with clamp 10 in f32,
      // rounded to bf16, times the bf16 routing weight, rounded to bf16
      const float gf = round_bf16(g[r]);
      const float uf = round_bf16(u[r]);
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
}

// The unit's finishing CTA: sum the partial slots of CTAs cf..cl (one row, NV
// values each) in CTA order. Slots are read four CTAs at a time so their
// loads overlap; empty CTAs are skipped; a CTA's slot is 2c when the unit is
// its first segment, else 2c+1.
template <int NV, typename SchedT>
__device__ __forceinline__ void sum_slots(const SchedT& sc, int cf, int cl, int64_t us, const float* part, int slot_floats,
                                          int row, float (&acc)[NV]) {
  constexpr int NB = NV <= 16 ? 4 : (NV <= 32 ? 2 : 1);  // slots in flight (register budget)
#pragma unroll
  for (int t = 0; t < NV; ++t) acc[t] = 0.f;
  int64_t lc = sc.lo(cf);
  for (int c0 = cf; c0 <= cl; c0 += NB) {
    const float* sl[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      const int cc = c0 + b;
      sl[b] = nullptr;
      if (cc <= cl) {
        const int64_t ln = sc.lo(cc + 1);
        if (lc < ln) sl[b] = part + (2 * static_cast<int64_t>(cc) + (lc >= us ? 0 : 1)) * slot_floats;
        lc = ln;
      }
    }
    float v[NB][NV];
#pragma unroll
    for (int b = 0; b < NB; ++b)
#pragma unroll
      for (int t = 0; t < NV; ++t) v[b][t] = sl[b] ? __ldcg(sl[b] + t * kM + row) : 0.f;
#pragma unroll
    for (int b = 0; b < NB; ++b)
      if (sl[b])
#pragma unroll
        for (int t = 0; t < NV; ++t) acc[t] += v[b][t];
  }
}

// A split unit's finishing CTA: the sum, in CTA order, of the partial rows
// the other CTAs c0..cl published in their slots (slot 2c; CTAs without steps
// skipped), NV values of one row. Up to NB peers' rows are loaded at once
// (one L2 round trip per NB peers), then added in CTA order.
template <int NV, typename SchedT>
__device__ __forceinline__ void peer_sum(const SchedT& sc, int c0, int cl, const float* part, int slot_floats,
                                         int row, float (&acc)[NV]) {
  constexpr int NB = NV <= 16 ? 4 : (NV <= 32 ? 2 : 1);  // peers in flight (register budget)
#pragma unroll
  for (int t = 0; t < NV; ++t) acc[t] = 0.f;
  int64_t lc = sc.lo(c0);
  for (int cb = c0; cb <= cl; cb += NB) {
    const float* sl[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      const int cc = cb + b;
      sl[b] = nullptr;
      if (cc <= cl) {
        const int64_t ln = sc.lo(cc + 1);
        if (lc < ln) sl[b] = part + 2 * static_cast<int64_t>(cc) * slot_floats;
        lc = ln;
      }
    }
    float v[NB][NV];
#pragma unroll
    for (int b = 0; b < NB; ++b)
#pragma unroll
      for (int t = 0; t < NV; ++t) v[b][t] = sl[b] ? __ldcg(sl[b] + t * kM + row) : 0.f;
#pragma unroll
    for (int b = 0; b < NB; ++b)
      if (sl[b])
#pragma unroll
        for (int t = 0; t < NV; ++t) acc[t] += v[b][t];
  }
}

// The 128 epilogue threads wait (bounded) until a unit's ticket reaches
// target: thread 0 polls with acquire loads, the named barrier releases the rest.
__device__ __forceinline__ void wait_ticket(const uint32_t* ctr, uint32_t target, int etid, int32_t* status) {
  if (etid == 0) {
    // acquire polls: no fence, which would also wait for this thread's own
    // partial rows just stored for another unit
    if (ld_acquire_gpu(ctr) < target) {
      const uint64_t t0 = globaltimer_ns();
      for (uint32_t i = 1;; ++i) {
        if (ld_acquire_gpu(ctr) >= target) break;
        if ((i & 63u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) {
          report(status, HS_DEV_TIMEOUT);
          break;
        }
      }
    }
  }
  epi_bar();
}

// The chunk's per-token routing weights (bf16 values), loaded before the
// unit's accumulator is ready.
__device__ __forceinline__ void tok_weights(const UnitArgs& a, const UnitInfo& ui, float (&wbv)[8]) {
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    wbv[r] = 0.f;
    if (r < a.T) wbv[r] = ui.shared ? 1.f : __ldcg(a.P.ctab_wb + ui.chunk * 8 + r);
  }
}

// Token-mode gate/up epilogue: the accumulator columns are the (up to 8)
// tokens; every (chunk, token < T) activation row is written, as zeros where
// the token is not routed to the chunk's expert, so the down phase can run
// each unit over all experts with the same 8 token columns. Rows t >= T are
// left as they are: they only feed the down MMA's columns t >= T, which no
// epilogue stores (their values, even non-finite ones, stay in their own
// columns). Each warp
// holds 32 consecutive values of every row (one 32-column block of the down
// MMA's K): the block is scaled by 2^q so its largest magnitude lies in
// [128, 256), which makes the hi/lo e4m3 split of every bf16 value exact down
// to 2^-10 of the block maximum, and 127 - q is written as the row's UE8M0 B
// scale of that block (the scale-atom image the down phase copies).
template <bool kFP8>
__device__ __forceinline__ void gateup_finish_tok(const Desc& d, const UnitArgs& a, const UnitInfo& ui, int row,
                                                  const float (&g)[8], const float (&u)[8], const float (&wbv)[8]) {
  const int64_t I_act = max(d.I, d.has_shared ? d.I_sh : 0);
  uint8_t* hi_plane = a.P.act8;
  uint8_t* lo_plane = a.P.act8 + a.act_rows * I_act;
  const int col = ui.tile * kM + row;
  const int64_t slot = kFP8 ? 0 : 1 + ui.chunk;
  const int lane = row & 31, blk = row >> 5;
  uint8_t* img = a.P.act_img + (slot * (I_act / kM) + ui.tile) * 256;
  float av[8];
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    av[r] = 0.f;
    if (wbv[r] != 0.f) {
      // reference roundings as in gateup_finish
      const float gf = round_bf16(g[r]);
      const float uf = round_bf16(u[r]);
      const float gc = gf > 10.f ? 10.f : gf;
      const float uc = uf > 10.f ? 10.f : (uf < -10.f ? -10.f : uf);
      const float sig = 1.f / (1.f + expf(-gc));
      av[r] = round_bf16((gc * sig) * uc);
      if (!kFP8) av[r] = round_bf16(av[r] * wbv[r]);
    }
  }
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    if (r >= a.T) break;  // uniform over the warp
    // the block's largest magnitude (non-negative float bits order as values)
    const uint32_t mb = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(av[r])));
    const int q = row_prescale(__uint_as_float(mb));
    const float v = av[r] * exp2i(q);
    const __nv_fp8_storage_t hb = __nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
    const __half_raw hr = __nv_cvt_fp8_to_halfraw(hb, __NV_E4M3);
    const float hf = __half2float(*reinterpret_cast<const __half*>(&hr));
    const __nv_fp8_storage_t lb = __nv_cvt_float_to_fp8(v - hf, __NV_SATFINITE, __NV_E4M3);
    hi_plane[(slot * 8 + r) * I_act + col] = hb;
    lo_plane[(slot * 8 + r) * I_act + col] = lb;
    if (lane == r) {
      const uint8_t sf = static_cast<uint8_t>(127 - q);
      img[r * 16 + blk] = sf;        // hi row r
      img[(8 + r) * 16 + blk] = sf;  // lo row r
    }
  }
}

struct F8 {
  float v[8];
};

// The same for T <= 4, not inlined, so that every call runs the same
// instructions: the epilogue warps run it once with dry set (no stores) while
// the CTA waits for the routing, and the first real call then finds its code
// in the instruction cache instead of fetching it line by line from L2 on the
// phase's tail. (At T = 8 the call costs more than the fetch it saves.)
__device__ __noinline__ void gateup_finish_tok_nl(uint8_t* act8, int64_t act_rows, uint8_t* act_img, int64_t I_act,
                                                  int T, int fp8, int tile, int chunk, int row, F8 g, F8 u, F8 wbv,
                                                  int dry) {
  uint8_t* hi_plane = act8;
  uint8_t* lo_plane = act8 + act_rows * I_act;
  const int col = tile * kM + row;
  const int64_t slot = fp8 ? 0 : 1 + chunk;
  const int lane = row & 31, blk = row >> 5;
  uint8_t* img = act_img + (slot * (I_act / kM) + tile) * 256;
  float av[8];
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    av[r] = 0.f;
    if (wbv.v[r] != 0.f) {
      // reference roundings as in gateup_finish
      const float gf = round_bf16(g.v[r]);
      const float uf = round_bf16(u.v[r]);
      const float gc = gf > 10.f ? 10.f : gf;
      const float uc = uf > 10.f ? 10.f : (uf < -10.f ? -10.f : uf);
      const float sig = 1.f / (1.f + expf(-gc));
      av[r] = round_bf16((gc * sig) * uc);
      if (!fp8) av[r] = round_bf16(av[r] * wbv.v[r]);
    }
  }
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    if (r >= T) break;  // uniform over the warp
    // the block's largest magnitude (non-negative float bits order as values)
    const uint32_t mb = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(av[r])));
    const int q = row_prescale(__uint_as_float(mb));
    const float v = av[r] * exp2i(q);
    const __nv_fp8_storage_t hb = __nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
    const __half_raw hr = __nv_cvt_fp8_to_halfraw(hb, __NV_E4M3);
    const float hf = __half2float(*reinterpret_cast<const __half*>(&hr));
    const __nv_fp8_storage_t lb = __nv_cvt_float_to_fp8(v - hf, __NV_SATFINITE, __NV_E4M3);
    if (dry) continue;
    hi_plane[(slot * 8 + r) * I_act + col] = hb;
    lo_plane[(slot * 8 + r) * I_act + col] = lb;
    if (lane == r) {
      const uint8_t sf = static_cast<uint8_t>(127 - q);
      img[r * 16 + blk] = sf;        // hi row r
      img[(8 + r) * 16 + blk] = sf;  // lo row r
    }
  }
}

// Persistent stream-K kernel for one phase. kDown = false: gate/up (A boxes =
// w1 and w3 tiles of one 128-column k-step); kDown = true: down (A boxes = two
// k-boxes of w2). One CTA per SM: warp 4 streams TMA, warp 5 issues tcgen05
// copies and MMAs, warps 0-3 drain the TMEM accumulators (double-buffered, so
// the next unit's MMAs overlap this unit's epilogue). A unit split between
// CTAs writes f32 partials; the last of them (atomic ticket, no waiting) sums
// the partials in CTA order and finishes the unit.
template <bool kDown, int NT, bool kTok = false>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) sk_kernel(const __grid_constant__ Desc d,
                                                         const __grid_constant__ CallMaps cm, UnitArgs a) {
  constexpr int BOXES = kDown ? 2 : 1;
  using L = SmemLayout<NT, BOXES>;
  constexpr int S_ = L::kNumStages;
  constexpr int N = 16 * NT;
  static_assert(S_ >= 2 && S_ <= 4, "stage count");
  static_assert(sizeof(Bars) <= L::kBarBytes, "barrier block");
  // TMEM (256 columns per CTA, two CTAs per SM): accumulator buffers at 0 and
  // 96 (gate at +0, up at +48), A scales at 192 + 8*stage, B scales at 224 + 4*buffer
  constexpr uint32_t kAcc = 96;
  constexpr uint32_t kSfa = 192;
  constexpr uint32_t kSfb = 224;
  constexpr int NP = 8 * NT;                        // pairs per unit (hi and lo columns summed)
  constexpr int kSlot = (kDown ? 1 : 2) * kM * NP;  // floats per partial slot
  extern __shared__ uint8_t smem_raw[];  // 1024-aligned at offset 0 (checked below)
  // the 128B-swizzled stages need a 1024-aligned base; no slack is reserved
  // for realignment (two CTAs per SM leave none), so check it
  if (smem_u32(smem_raw) & 1023u) {
    pdl_wait();
    if (threadIdx.x == 0) report(a.status, HS_DEV_SMEM_ALIGN);
    return;
  }
  uint8_t* base = smem_raw;
  Bars* bars = reinterpret_cast<Bars*>(base + S_ * L::kStage);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D = d.D;
  const int c = blockIdx.x;
  HS_TRACE_T(hs_t0);

  if (threadIdx.x == 0) {
    for (int i = 0; i < S_; ++i) {
      mbar_init(&bars->full[i], 1);
      mbar_init(&bars->empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->acc_full[i], 1);
      mbar_init(&bars->acc_empty[i], 4);
    }
    mbar_init(&bars->mma_done, 1);
    mbar_init(&bars->pub, 128);
    bars->issued = 0;
    bars->consumed = 0;
    fence_mbar_init();
  }
  if (warp == 0) tc5::tmem_alloc(&bars->tmem, 256);
  if (warp == 4 && lane == 0) {
    prefetch_tensormap(kDown ? &d.tm_w2 : &d.tm_w13);
    prefetch_tensormap(kDown ? &d.tm_sw2 : &d.tm_sw13);
    prefetch_tensormap(kDown ? &cm.tm_act8 : &cm.tm_x8);
    // token mode: the shared expert's gate/up and down weights do not depend on
    // the routing; while the routing runs, the CTAs that are resident early
    // (all but the last 40, which wait for the routing cluster's SMs) bring
    // them into L2 in 64 KB pieces, about 90 KB per CTA
    if (kTok && !kDown && a.use_shared && c < a.G - 40) {
      constexpr int64_t kPiece = 65536;
      const int64_t Dl = D, Ish = d.I_sh;
      const uint8_t* base_r[4] = {d.sh_w13, d.sh_w2, d.sh_s13a, d.sh_s2a};
      const int64_t len_r[4] = {2 * Ish * Dl, Dl * Ish, (Ish / kM) * (Dl / kM) * 1024, (Dl / kM) * (Ish / kM) * 512};
      const int64_t nct = a.G - 40;
      int64_t first = 0;  // index of the region's first piece
      for (int r = 0; r < 4; ++r) {
        const int64_t np = (len_r[r] + kPiece - 1) / kPiece;
        for (int64_t i = (c - first % nct + nct) % nct; i < np; i += nct) {
          const int64_t off = i * kPiece, left = len_r[r] - off;
          prefetch_l2_bulk(base_r[r] + off, static_cast<uint32_t>(left < kPiece ? left : kPiece));
        }
        first += np;
      }
    }
  }
  if (kTok && !kDown && warp < 4 && a.T <= kFinishNlMaxT) {  // the activation epilogue's code into the instruction cache
    F8 z, one;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      z.v[r] = 0.f;
      one.v[r] = 1.f;
    }
    gateup_finish_tok_nl(a.P.act8, a.act_rows, a.P.act_img, d.I, a.T, 0, 0, 0, threadIdx.x, z, z, one, 1);
  }
  // everything above overlaps the previous kernel; from here on the plan (and,
  // for the down phase, the gate/up phase) is complete and visible
  pdl_wait();
  pdl_trigger();
  tc5::fence_before_sync();
  __syncthreads();
  tc5::fence_after_sync();
  const uint32_t tmem = bars->tmem;
  HS_TRACE_SLOT(hs_tslot);
  if (kTok && !kDown && threadIdx.x == 0) {
    HS_STAMP_AT(hs_tslot, ::hs::trace::kGateUp, c, 0, hs_t0);
    HS_STAMP(hs_tslot, ::hs::trace::kGateUp, c, 1);
  }
  // token mode: the producer's chunk experts (lane j: chunks j, j+32, j+64,
  // j+96) and token B scales (lane t), loaded together with the schedule's
  // header so the plan costs one round trip (entries past the chunk count are
  // never used; the 512 bytes read lie inside the workspace, whose token-row
  // planes follow the chunk table)
  int px0 = 0, px1 = 0, px2 = 0, px3 = 0;
  uint32_t psb = 127u;
  if (kTok && warp == 4) {
    const int32_t* ce = a.P.chunk_expert;
    px0 = __ldcg(ce + lane);
    px1 = __ldcg(ce + lane + 32);
    px2 = __ldcg(ce + lane + 64);
    px3 = __ldcg(ce + lane + 96);
    if (lane < a.T) psb = __ldcg(a.P.sb1 + lane);
  }
  const Sched sc = make_sched(d, a, kDown);
  const int64_t s_begin = sc.lo(c), s_end = sc.lo(c + 1);

  if (warp == 4) {
    // ---------------- TMA producer (whole warp; lane 0 issues) ----------------
    const uint64_t pol = l2_evict_first_policy();
    int64_t step = 0;
    bool ok = true;
    for (int64_t s = s_begin; s < s_end && ok;) {
      const int64_t u = sc.unit_of(s);
      UnitInfo ui;
      if constexpr (kTok) {
        // unit_info with the chunk's expert from the registers above
        const int tiles_sh = d.has_shared ? d.I_sh / kM : 1, tiles_rt = d.I / kM;
        if (u < sc.n_sh_units) {
          ui.shared = 1;
          ui.chunk = static_cast<int>(u / tiles_sh);
          ui.tile = static_cast<int>(u - static_cast<int64_t>(ui.chunk) * tiles_sh);
          ui.e = 0;
        } else {
          const int64_t uu = u - sc.n_sh_units;
          ui.shared = 0;
          ui.chunk = static_cast<int>(uu / tiles_rt);
          ui.tile = static_cast<int>(uu - static_cast<int64_t>(ui.chunk) * tiles_rt);
          const int grp = ui.chunk >> 5;
          const int sel = grp == 0 ? px0 : grp == 1 ? px1 : grp == 2 ? px2 : px3;
          ui.e = __shfl_sync(0xffffffffu, sel, ui.chunk & 31);
        }
        ui.pair0 = 0;
        ui.np = 0;
      } else {
        ui = unit_info(d, a, sc, u, kDown);
      }
      const int64_t us = sc.ustart(u);
      const int k0 = static_cast<int>(s - us);
      const int k1 = static_cast<int>(min64(static_cast<int64_t>(sc.unk(u)), s_end - us));
      const bool fp8 = ui.shared != 0;
      const CUtensorMap* wm = kDown ? (fp8 ? &d.tm_sw2 : &d.tm_w2) : (fp8 ? &d.tm_sw13 : &d.tm_w13);
      const CUtensorMap* bm = kDown ? &cm.tm_act8 : &cm.tm_x8;
      // first weight row of the unit's step 0 and the rows per step (two tiles
      // of 128 rows per stage in both phases)
      int64_t y0;
      if (!kDown) {
        y0 = fp8 ? static_cast<int64_t>(ui.tile) * (D / kM) * 256
                 : (static_cast<int64_t>(ui.e) * (d.I / kM) + ui.tile) * (D / kM) * 256;
      } else {
        y0 = fp8 ? static_cast<int64_t>(ui.tile) * (d.I_sh / kM) * kM
                 : (static_cast<int64_t>(ui.e) * (D / kM) + ui.tile) * (d.I / kM) * kM;
      }
      const uint8_t* sf0;
      if (!kDown) {
        sf0 = fp8 ? d.sh_s13a + static_cast<int64_t>(ui.tile) * (D / kM) * 1024
                  : d.s13a + (static_cast<int64_t>(ui.e) * (d.I / kM) + ui.tile) * (D / kM) * 1024;
      } else {
        sf0 = fp8 ? d.sh_s2a + static_cast<int64_t>(ui.tile) * (d.I_sh / kM) * 512
                  : d.s2a + (static_cast<int64_t>(ui.e) * (D / kM) + ui.tile) * (d.I / kM) * 512;
      }
      const uint32_t tx = 2 * (fp8 ? kBoxBytes : kBoxBytes / 2) + L::kB + 2 * 512;
      const uint8_t* sbv = kDown ? a.P.sb2 : a.P.sb1;
      for (int k = k0; k < k1; ++k, ++step) {
        const int st = static_cast<int>(step % S_);
        if (step >= S_) {
          bool w = true;
          if (lane == 0) w = mbar_wait(&bars->empty[st], static_cast<uint32_t>(((step / S_) - 1) & 1));
          w = __shfl_sync(0xffffffffu, w ? 1 : 0, 0) != 0;
          if (!w) {
            if (lane == 0) report(a.status, HS_DEV_TIMEOUT);
            ok = false;
            break;
          }
        }
        uint8_t* S = base + st * L::kStage;
        uint8_t* Bs = S + L::kA;
        uint8_t* SF = Bs + L::kB;
        // copies first (their latency overlaps the scale-atom work below): on a
        // segment's first step the barrier gets its bytes now and its arrival
        // once the warp has written the unit's B scale atom
        if (lane == 0) {
          if (k == k0)
            mbar_expect_tx(&bars->full[st], tx);
          else
            mbar_arrive_expect_tx(&bars->full[st], tx);
          const int xa = kDown ? k * 256 : k * 128;
          if (kTok && !kDown && step == 0) HS_STAMP(hs_tslot, ::hs::trace::kGateUp, c, 2);
          tma_load_2d_hint(S, wm, &bars->full[st], 0, static_cast<int>(y0 + static_cast<int64_t>(k) * 256), pol);
          for (int b = 0; b < BOXES; ++b)
            tma_load_3d(Bs + b * 2 * NT * 1024, bm, &bars->full[st], xa + b * 128, kTok ? 0 : ui.pair0, 0);
          bulk_load_hint(SF, sf0 + static_cast<int64_t>(k) * 1024, 1024, &bars->full[st], pol);
        }
        if (k == k0) {
          // the unit's B scale atom: word (m0, m1) = scale of B row n = m0 + 32*m1
          for (int wi = lane; wi < 128; wi += 32) {
            const int m0 = wi >> 2, m1 = wi & 3;
            const int n = m0 + 32 * m1;
            const int r = n % (8 * NT);
            // token rows: lane r holds sb1[r] (every lane takes part in the shuffle)
            const uint32_t tb = kTok ? __shfl_sync(0xffffffffu, psb, r & 31) : 127u;
            uint32_t b = 127u;
            if (n < N) {
              if (kTok) {
                if (r < a.T) b = tb;
              } else if (r < ui.np) {
                b = sbv[ui.pair0 + r];
              }
            }
            *reinterpret_cast<uint32_t*>(SF + 1024 + m0 * 16 + m1 * 4) = b * 0x01010101u;
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars->full[st]);
        }
        __syncwarp();
      }
      s = us + k1;
    }
    if (lane == 0) bars->issued = static_cast<int32_t>(step);
    if (kTok && !kDown && lane == 0) HS_STAMP(hs_tslot, ::hs::trace::kGateUpTail, c, 4);
    // Only this CTA's first segment can be a non-finishing part of a split
    // unit (every later segment starts a unit here). Its partial rows are
    // stored by the epilogue threads, which arrive on `pub` and go on; this
    // warp adds the step count to the unit's ticket after a gpu-scope fence,
    // cumulative over their stores through the barrier.
    if (lane == 0 && s_begin < s_end) {
      const int64_t u0 = sc.unit_of(s_begin), us0 = sc.ustart(u0);
      if (sc.cta_of(us0) != c) {
        const int64_t k1 = min64(static_cast<int64_t>(sc.unk(u0)), s_end - us0);
        if (mbar_wait(&bars->pub, 0)) {
          __threadfence();
          atomicAdd(&a.ucount[u0], static_cast<uint32_t>(k1 - (s_begin - us0)));
          if (kTok && !kDown) HS_STAMP(hs_tslot, ::hs::trace::kCombine, c, 6);
        } else {
          report(a.status, HS_DEV_TIMEOUT);
        }
      }
    }
  } else if (warp == 5) {
    // ---------------- MMA issuer (lane 0) ----------------
    if (lane == 0) {
      int64_t step = 0;
      int seg = 0;
      bool ok = true;
      for (int64_t s = s_begin; s < s_end && ok; ++seg) {
        const int64_t u = sc.unit_of(s);
        const int64_t us = sc.ustart(u);
        const int k0 = static_cast<int>(s - us);
        const int k1 = static_cast<int>(min64(static_cast<int64_t>(sc.unk(u)), s_end - us));
        const uint32_t afmt = u < sc.n_sh_units ? 0u : 5u;
        const int buf = seg & 1;
        if (seg >= 2 && !mbar_wait(&bars->acc_empty[buf], static_cast<uint32_t>(((seg >> 1) - 1) & 1))) {
          report(a.status, HS_DEV_TIMEOUT);
          break;
        }
        tc5::fence_after_sync();
        const uint32_t acc = tmem + buf * kAcc;
        const uint32_t sfb = tmem + kSfb + buf * 4;
        for (int k = k0; k < k1; ++k, ++step) {
          const int st = static_cast<int>(step % S_);
          if (!mbar_wait(&bars->full[st], static_cast<uint32_t>((step / S_) & 1))) {
            report(a.status, HS_DEV_TIMEOUT);
            ok = false;
            break;
          }
          tc5::fence_after_sync();
          uint8_t* S = base + st * L::kStage;
          const uint32_t sA = smem_u32(S), sB = smem_u32(S + L::kA), sSF = smem_u32(S + L::kA + L::kB);
          if (kTok && !kDown && step == 0) HS_STAMP(hs_tslot, ::hs::trace::kGateUp, c, 3);
          if (k == k0) tc5::cp_sf_32x128b(sfb, tc5::sdesc_sf(sSF + 1024));
          const uint32_t sfa0 = tmem + kSfa + st * 8;
          tc5::cp_sf_32x128b(sfa0, tc5::sdesc_sf(sSF));
          tc5::cp_sf_32x128b(sfa0 + 4, tc5::sdesc_sf(sSF + 512));
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const uint64_t ad = tc5::sdesc_sw128(sA + i * kBoxBytes);
            const uint64_t bd = tc5::sdesc_sw128(sB + (kDown ? i * 2 * NT * 1024 : 0));
            const uint32_t dcol = acc + (kDown ? 0u : (i ? static_cast<uint32_t>(kAccUp) : 0u));
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint32_t id = tc5::idesc_mxf8f6f4(afmt, N, j, j);
              const uint32_t accum = (k > k0 || j > 0 || (kDown && i > 0)) ? 1u : 0u;
              tc5::mma_mxf8f6f4(dcol, ad + 2 * j, bd + 2 * j, id, accum,
                                (sfa0 + 4 * i) | (static_cast<uint32_t>(j) << 30),
                                sfb | (static_cast<uint32_t>(j) << 30));
            }
          }
          tc5::commit(&bars->empty[st]);
        }
        tc5::commit(&bars->acc_full[buf]);
        s = us + k1;
      }
      // every tcgen05 operation of this thread done before TMEM is freed
      if (kTok && !kDown) HS_STAMP(hs_tslot, ::hs::trace::kGateUp, c, 4);
      bars->consumed = static_cast<int32_t>(step);
      tc5::commit(&bars->mma_done);
      if (!mbar_wait(&bars->mma_done, 0)) report(a.status, HS_DEV_TIMEOUT);
      if (kTok && !kDown) HS_STAMP(hs_tslot, ::hs::trace::kGateUpTail, c, 3);
    }
  } else {
    // ---------------- epilogue (warps 0-3, TMEM lanes 32w..32w+31) ----------------
    // A unit split between CTAs cf..cl is finished by cf, the CTA holding its
    // first steps (its last segment, so the latest in time); the others publish
    // their partial rows in slot 2c (their first segment) and add their step
    // counts to the unit's ticket. The finisher sums the published rows while
    // its own MMAs still run, so its tail is its accumulator plus the epilogue.
    const int row = 32 * warp + lane;
    const int etid = threadIdx.x;  // 0..127
    const uint32_t lane_off = static_cast<uint32_t>(32 * warp) << 16;
    constexpr int NV = kDown ? NP : 2 * NP;
    // A segment's unit parameters and routing weights come from L2 (a round
    // trip of a microsecond or more while the phase streams): token mode
    // loads them one segment ahead, while the epilogue waits for the previous
    // accumulator.
    struct SegP {
      int64_t u, us;
      int nk, k0, k1, cf, cl;
      UnitInfo ui;
      float wbv[8];
    };
    auto seg_params = [&](int64_t s0, SegP& p) {
      p.u = sc.unit_of(s0);
      p.us = sc.ustart(p.u);
      p.nk = sc.unk(p.u);
      p.k0 = static_cast<int>(s0 - p.us);
      p.k1 = static_cast<int>(min64(static_cast<int64_t>(p.nk), s_end - p.us));
      p.ui = unit_info(d, a, sc, p.u, kDown);
      p.cf = sc.cta_of(p.us);
      p.cl = sc.cta_of(p.us + p.nk - 1);
      if (kTok && (p.cf == p.cl || c == p.cf)) tok_weights(a, p.ui, p.wbv);
    };
    SegP nxt;
    if (kTok && s_begin < s_end) seg_params(s_begin, nxt);
    int seg = 0;
    for (int64_t s = s_begin; s < s_end; ++seg) {
      SegP cur;
      if constexpr (kTok)
        cur = nxt;
      else
        seg_params(s, cur);
      const int64_t s_next = cur.us + cur.k1;
      if (kTok && s_next < s_end) seg_params(s_next, nxt);
      const int64_t u = cur.u;
      const int nk = cur.nk, k0 = cur.k0, k1 = cur.k1;
      const UnitInfo& ui = cur.ui;
      const int buf = seg & 1;
      const int cf = cur.cf, cl = cur.cl;
      const bool split = cf != cl;
      const bool finish = !split || c == cf;
      float pre[NV];
      const float(&wbv)[8] = cur.wbv;
      if (split && finish) {
        if (kTok && !kDown && threadIdx.x == 0) HS_STAMP(hs_tslot, ::hs::trace::kGateUpTail, c, 7);
        wait_ticket(&a.ucount[u], static_cast<uint32_t>(nk - (k1 - k0)), etid, a.status);
        if (kTok && !kDown && threadIdx.x == 0) HS_STAMP(hs_tslot, ::hs::trace::kGateUpTail, c, 0);
        peer_sum<NV>(sc, cf + 1, cl, a.part, kSlot, row, pre);
        if (kTok && !kDown && threadIdx.x == 0) HS_STAMP(hs_tslot, ::hs::trace::kGateUp, c, 7);
      }
      if (!mbar_wait(&bars->acc_full[buf], static_cast<uint32_t>((seg >> 1) & 1))) {
        if (etid == 0) report(a.status, HS_DEV_TIMEOUT);
        break;
      }
      if (kTok && !kDown && seg == 0 && threadIdx.x == 0) HS_STAMP(hs_tslot, ::hs::trace::kGateUp, c, 6);
      if (kTok && !kDown && threadIdx.x == 0) HS_STAMP(hs_tslot, ::hs::trace::kGateUpTail, c, 1);
      tc5::fence_after_sync();
      float c0[N], c1[N];
      const uint32_t acc = tmem + lane_off + buf * kAcc;
#pragma unroll
      for (int q = 0; q < NT; ++q) {
        float v[16];
        tc5::ld_32x32b_x16(acc + q * 16, v);
#pragma unroll
        for (int i = 0; i < 16; ++i) c0[q * 16 + i] = v[i];
        if (!kDown) {
          tc5::ld_32x32b_x16(acc + kAccUp + q * 16, v);
#pragma unroll
          for (int i = 0; i < 16; ++i) c1[q * 16 + i] = v[i];
        }
      }
      tc5::wait_ld();
      tc5::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->acc_empty[buf]);
      // hi + lo columns of each pair: the full dot product of this segment
      float g[NP], v[NP];
#pragma unroll
      for (int r = 0; r < NP; ++r) {
        g[r] = c0[r] + c0[NP + r];
        v[r] = kDown ? 0.f : c1[r] + c1[NP + r];
      }
      if (split && finish) {
#pragma unroll
        for (int n = 0; n < NP; ++n) {
          g[n] += pre[n];
          if (!kDown) v[n] += pre[NP + n];
        }
      } else if (split) {
        // publish: slot 2c; the producer warp adds the ticket (above), so the
        // epilogue goes straight on to its next segment
        float* slot = a.part + 2 * static_cast<int64_t>(c) * kSlot;
#pragma unroll
        for (int n = 0; n < NP; ++n) {
          __stcg(slot + n * kM + row, g[n]);
          if (!kDown) __stcg(slot + (NP + n) * kM + row, v[n]);
        }
        mbar_arrive(&bars->pub);
        if (kTok && !kDown && threadIdx.x == 0) HS_STAMP(hs_tslot, ::hs::trace::kGateUpTail, c, 6);
      }
      if (finish) {
        if constexpr (kTok) {
          if (a.T <= kFinishNlMaxT) {
            F8 gg, vv, ww;
#pragma unroll
            for (int r = 0; r < 8; ++r) {
              gg.v[r] = g[r];
              vv.v[r] = v[r];
              ww.v[r] = wbv[r];
            }
            gateup_finish_tok_nl(a.P.act8, a.act_rows, a.P.act_img, max(d.I, d.has_shared ? d.I_sh : 0), a.T,
                                 ui.shared, ui.tile, ui.chunk, row, gg, vv, ww, 0);
          } else if (ui.shared) {
            gateup_finish_tok<true>(d, a, ui, row, g, v, wbv);
          } else {
            gateup_finish_tok<false>(d, a, ui, row, g, v, wbv);
          }
        } else if (!kDown) {
          if (ui.shared)
            gateup_finish<NT, true>(d, a, ui, row, g, v);
          else
            gateup_finish<NT, false>(d, a, ui, row, g, v);
        } else {
#pragma unroll
          for (int r = 0; r < NP; ++r)
            if (r < ui.np) a.P.out_part[static_cast<int64_t>(ui.pair0 + r) * D + ui.tile * kM + row] = g[r];
          // finalize the 128-row slice of D once every unit on it is done
          if (!a.ext_combine) {
            __threadfence();
            epi_bar();
            if (etid == 0) {
              const uint32_t total = static_cast<uint32_t>(a.n_sh_chunks + a.P.hdr[0]);
              bars->flag = atomicAdd(&a.P.dcount[ui.tile], 1u) == total - 1u;
            }
            epi_bar();
            const bool fin = bars->flag != 0;
            epi_bar();
            if (fin) {
              __threadfence();
              finalize_tile(a, D, ui.tile, etid, 128);
            }
          }
        }
      }
      s = s_next;
    }
    if (kTok && !kDown && threadIdx.x == 0) {
      HS_STAMP(hs_tslot, ::hs::trace::kGateUpTail, c, 2);
      HS_STAMP_AT(hs_tslot, ::hs::trace::kGateUpTail, c, 5, static_cast<unsigned long long>(seg));
    }
    // no unit at all (every pair skipped, no shared expert): write zeros
    if (kDown && sc.U == 0 && !a.ext_combine)
      for (int tile = c; tile < D / kM; tile += a.G) finalize_tile(a, D, tile, etid, 128);
  }

  tc5::fence_before_sync();
  __syncthreads();
  // copies issued but never consumed (only after a timed-out wait): let them
  // land before the CTA's shared memory is released
  if (threadIdx.x == 128) {
    for (int64_t k = bars->consumed; k < bars->issued; ++k)
      if (!mbar_wait(&bars->full[k % S_], static_cast<uint32_t>((k / S_) & 1))) {
        report(a.status, HS_DEV_TIMEOUT);
        break;
      }
  }
  __syncthreads();
  if (warp == 0) {
  if (kTok && !kDown && threadIdx.x == 0) HS_STAMP(hs_tslot, ::hs::trace::kGateUp, c, 5);
    tc5::fence_after_sync();
    tc5::tmem_dealloc(tmem, 256);
  }
}

// ---------------------------------------------------------------------------
// Token-mode down phase (T <= 8)
// ---------------------------------------------------------------------------
// A unit is one 128-row tile of D. Its k-steps are the shared expert's I_sh/256
// steps (FP8, twice the bytes, weight 2) followed by I/256 steps of every
// routed chunk (one expert each) in ascending expert order. B is the chunk's 8
// token rows of act8, so the accumulator columns are tokens and TMEM sums every
// expert's contribution: routed experts into columns [0, 16) of a buffer, the
// shared expert into [48, 64), kept apart so the two sums round to bf16
// separately as the reference's routed + shared add does. The CTA that
// completes a unit writes the output rows; no per-pair rows, no finalize pass.
struct TokSched {
  int U, nsh, nrt, C, Su, G, wsh;
  int64_t Wu, W;

  __device__ __forceinline__ static int64_t udiv(int64_t a, int64_t b) {
    if (((a | b) >> 32) == 0) return static_cast<uint32_t>(a) / static_cast<uint32_t>(b);
    return a / b;
  }
  __device__ __forceinline__ int64_t unit_of(int64_t s) const { return udiv(s, Su); }
  __device__ __forceinline__ int64_t ustart(int64_t u) const { return u * Su; }
  // weight position where step s starts
  __device__ __forceinline__ int64_t wpos(int64_t s) const {
    const int64_t u = unit_of(s);
    const int64_t k = s - u * Su;
    return u * Wu + (k < nsh ? wsh * k : wsh * nsh + (k - nsh));
  }
  // first step at or after weight position w
  __device__ __forceinline__ int64_t step_at(int64_t w) const {
    const int64_t u = udiv(w, Wu);
    const int64_t r = w - u * Wu;
    return u * Su + (r <= wsh * nsh ? (r + wsh - 1) / wsh : nsh + (r - wsh * nsh));
  }
  __device__ __forceinline__ int64_t lo(int c) const {
    if (c >= G) return static_cast<int64_t>(U) * Su;
    return step_at(udiv(W * c, G));
  }
  // largest c with lo(c) <= s (lo(c) <= s <=> floor(W c / G) <= wpos(s))
  __device__ __forceinline__ int cta_of(int64_t s) const {
    const int64_t c = udiv(static_cast<int64_t>(G) * (wpos(s) + 1) - 1, W);
    return c < G - 1 ? static_cast<int>(c) : G - 1;
  }
};

__device__ __forceinline__ TokSched make_tok_sched(const Desc& d, const UnitArgs& a) {
  TokSched s;
  s.U = d.D / kM;
  s.nsh = a.use_shared ? d.I_sh / 256 : 0;
  s.nrt = d.I / 256;
  s.C = __ldcg(a.P.hdr);
  s.Su = s.nsh + s.C * s.nrt;
  s.wsh = a.w_sh;
  s.Wu = s.wsh * s.nsh + static_cast<int64_t>(s.C) * s.nrt;
  s.W = s.Wu * s.U;
  s.G = a.G;
  return s;
}

// kCl = false: stream-K over all tiles (one CTA per SM slot). kCl = true: one
// 8-CTA thread-block cluster per 128-row tile of D; the tile's k-steps are cut
// into 8 equal-weight slices and the 8 partial accumulators are summed through
// distributed shared memory (no partial slots in global memory, no tickets).
template <bool kCl>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) tok_down_kernel(const __grid_constant__ Desc d,
                                                                        const __grid_constant__ CallMaps cm,
                                                                        UnitArgs a) {
  using L = SmemLayout<1, 2>;
  constexpr int S_ = L::kNumStages;
  static_assert(S_ >= 2 && S_ <= 4, "stage count");
  static_assert(sizeof(Bars) <= L::kBarBytes, "barrier block");
  constexpr int N = 16;
  // TMEM (256 columns): accumulator buffers at 0 and 96 (routed at +0, shared
  // at +48), A scales at 192 + 8*stage, B scales at 224 + 8*stage (one atom
  // per 128-column k-tile of the stage, at +0 and +4)
  constexpr uint32_t kAcc = 96;
  constexpr uint32_t kAccSh = 48;
  constexpr uint32_t kSfa = 192;
  constexpr uint32_t kSfb = 224;
  static_assert(kSfb + 8 * S_ <= 256, "TMEM columns");
  // The stage's scale area holds the two A atoms and the two B images (256
  // bytes each, at +1024 and +1280); the copy of image 1 reads a whole atom
  // (512 bytes, its lines 16-31 unused), so 256 bytes of padding follow the
  // last stage before the barrier block.
  static_assert(L::kSF == 1536, "scale area");
  constexpr int kSlot = 2 * kM * 8;  // routed and shared sums of 8 tokens
  extern __shared__ uint8_t smem_raw[];  // 1024-aligned at offset 0 (checked below)
  if (smem_u32(smem_raw) & 1023u) {
    pdl_wait();
    if (threadIdx.x == 0) report(a.status, HS_DEV_SMEM_ALIGN);
    return;
  }
  uint8_t* base = smem_raw;
  Bars* bars = reinterpret_cast<Bars*>(base + S_ * L::kStage + kTokDownPad);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D = d.D;
  const int c = blockIdx.x;
  HS_TRACE_T(hs_t0);
  HS_TRACE_VAR(hs_t2);

  if (threadIdx.x == 0) {
    for (int i = 0; i < S_; ++i) {
      mbar_init(&bars->full[i], 1);
      mbar_init(&bars->empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->acc_full[i], 1);
      mbar_init(&bars->acc_empty[i], 4);
    }
    mbar_init(&bars->mma_done, 1);
    bars->issued = 0;
    bars->consumed = 0;
    fence_mbar_init();
  }
  if (warp == 0) tc5::tmem_alloc(&bars->tmem, 256);
  if (warp == 4 && lane == 0) {
    prefetch_tensormap(&d.tm_w2);
    prefetch_tensormap(&d.tm_sw2);
    prefetch_tensormap(&cm.tm_act8);
  }

  tc5::fence_before_sync();
  __syncthreads();
  tc5::fence_after_sync();
  const uint32_t tmem = bars->tmem;
  // The plan is complete before this grid starts (every gate/up CTA waited for
  // it before letting this grid launch), so the schedule and the chunk table
  // are read now, through L2, and the first stages' weights start streaming
  // while the gate/up phase finishes; only the activation loads wait.
  const TokSched sc = make_tok_sched(d, a);
  const bool any = sc.W > 0;
  int64_t s_begin = 0, s_end = 0;
  if (any) {
    if constexpr (kCl) {
      // cluster u = tile u; rank j takes the weight slice [Wu j/n, Wu (j+1)/n)
      const int64_t u = c / a.ncl, j = c % a.ncl;
      auto kb = [&](int64_t jj) {
        const int64_t w = TokSched::udiv(sc.Wu * jj, a.ncl);
        return w <= sc.wsh * sc.nsh ? (w + sc.wsh - 1) / sc.wsh : sc.nsh + (w - sc.wsh * sc.nsh);
      };
      s_begin = u * sc.Su + kb(j);
      s_end = u * sc.Su + kb(j + 1);
    } else {
      s_begin = sc.lo(c);
      s_end = sc.lo(c + 1);
    }
  }
  const int64_t npre = min64(static_cast<int64_t>(S_), s_end - s_begin);

  // producer state (warp 4): chunk table in registers, lane j keeps the
  // expert ids of chunks j, j+32, j+64, j+96
  static_assert(kTokChunks <= 4 * 32, "token-mode chunk table");
  uint64_t pol = 0;
  // (scalars, not arrays: the lambdas below capture them by reference)
  int ex0 = 0, ex1 = 0, ex2 = 0, ex3 = 0;
  if (warp == 4) {
    pol = l2_evict_first_policy();
    auto load = [&](int cc, int& e) {
      if (cc < sc.C) e = __ldcg(a.P.chunk_expert + cc);
    };
    load(lane, ex0);
    load(lane + 32, ex1);
    load(lane + 64, ex2);
    load(lane + 96, ex3);
  }
  const int64_t I_act = max(d.I, d.has_shared ? d.I_sh : 0);
  // step s -> (tile, shared?, chunk, k within the expert, expert)
  struct Step {
    int tile, ch, kk, e;
    bool shared;
  };
  auto decode = [&](int64_t s) {
    Step r;
    const int64_t u = sc.unit_of(s);
    const int k = static_cast<int>(s - u * sc.Su);
    r.tile = static_cast<int>(u);
    r.shared = k < sc.nsh;
    const int kr = k - sc.nsh;
    r.ch = r.shared ? 0 : kr / sc.nrt;
    r.kk = r.shared ? k : kr - r.ch * sc.nrt;
    const int grp = r.ch >> 5;
    const int e_sel = grp == 0 ? ex0 : grp == 1 ? ex1 : grp == 2 ? ex2 : ex3;
    r.e = __shfl_sync(0xffffffffu, e_sel, r.ch & 31);
    return r;
  };
  // lane 0: weights and their scale atoms (independent of the gate/up phase)
  auto issue_weights = [&](int st, const Step& q) {
    uint8_t* S = base + st * L::kStage;
    uint8_t* SF = S + L::kA + L::kB;
    int64_t ya;
    const uint8_t* sfp;
    if (q.shared) {
      ya = (static_cast<int64_t>(q.tile) * (d.I_sh / kM) + 2 * q.kk) * kM;
      sfp = d.sh_s2a + (static_cast<int64_t>(q.tile) * (d.I_sh / kM) + 2 * q.kk) * 512;
    } else {
      ya = ((static_cast<int64_t>(q.e) * (D / kM) + q.tile) * (d.I / kM) + 2 * q.kk) * kM;
      sfp = d.s2a + ((static_cast<int64_t>(q.e) * (D / kM) + q.tile) * (d.I / kM) + 2 * q.kk) * 512;
    }
    tma_load_2d_hint(S, q.shared ? &d.tm_sw2 : &d.tm_w2, &bars->full[st], 0, static_cast<int>(ya), pol);
    bulk_load_hint(SF, sfp, 1024, &bars->full[st], pol);
  };
  // lane 0: the activation rows and their block scales, lines 0-15 of the
  // stage's B scale atom (both written by the gate/up phase)
  auto issue_act = [&](int st, const Step& q) {
    uint8_t* Bs = base + st * L::kStage + L::kA;
    const int slot = q.shared ? 0 : 1 + q.ch;
    for (int b = 0; b < 2; ++b)
      tma_load_3d(Bs + b * 2048, &cm.tm_act8, &bars->full[st], q.kk * 256 + b * 128, slot * 8, 0);
    const uint8_t* img = a.P.act_img + (static_cast<int64_t>(slot) * (I_act / kM) + 2 * q.kk) * 256;
    bulk_load(Bs + L::kB + 1024, img, 512, &bars->full[st]);  // both k-tiles' images (adjacent)
  };
  auto tx_of = [&](const Step& q) {
    return static_cast<uint32_t>((q.shared ? 2 * kBoxBytes : kBoxBytes) + L::kB + 1024 + 512);
  };

  float res_pre = 0.f;  // cluster epilogue: the preloaded residual element
  int ep_slot = 0;      // peer-memory exchange: this call's slot
  if (warp == 4) {
    for (int64_t step = 0; step < npre; ++step) {  // stages are free: no empty waits yet
      const Step q = decode(s_begin + step);
      const int st = static_cast<int>(step);
      if (lane == 0) {
        mbar_expect_tx(&bars->full[st], tx_of(q));  // bytes now, the arrival after the activations
        if (step == 0) HS_TRACE_SET(hs_t2);
        issue_weights(st, q);
      }
    }
  }
  pdl_wait();  // the gate/up phase's activations are complete
  pdl_trigger();
  HS_TRACE_SLOT(hs_tslot);
  if (kCl && threadIdx.x == 0) {
    HS_STAMP_AT(hs_tslot, ::hs::trace::kDown, c, 0, hs_t0);
    HS_STAMP(hs_tslot, ::hs::trace::kDown, c, 1);
  }
  if (kCl && threadIdx.x == 128) HS_STAMP_AT(hs_tslot, ::hs::trace::kDown, c, 2, hs_t2);

  if (warp == 4) {
    // ---------------- TMA producer (whole warp; lane 0 issues) ----------------
    int64_t step = 0;
    for (; step < npre; ++step) {
      const Step q = decode(s_begin + step);
      if (lane == 0) {
        issue_act(static_cast<int>(step), q);
        mbar_arrive(&bars->full[step]);
      }
      __syncwarp();
    }
    for (int64_t s = s_begin + npre; s < s_end; ++s, ++step) {
      const Step q = decode(s);
      const int st = static_cast<int>(step % S_);
      if (step >= S_) {
        bool w = true;
        if (lane == 0) w = mbar_wait(&bars->empty[st], static_cast<uint32_t>(((step / S_) - 1) & 1));
        w = __shfl_sync(0xffffffffu, w ? 1 : 0, 0) != 0;
        if (!w) {
          if (lane == 0) report(a.status, HS_DEV_TIMEOUT);
          break;
        }
      }
      if (lane == 0) {
        mbar_arrive_expect_tx(&bars->full[st], tx_of(q));
        issue_weights(st, q);
        issue_act(st, q);
      }
      __syncwarp();
    }
    if (lane == 0) bars->issued = static_cast<int32_t>(step);
  } else if (warp == 5) {
    // ---------------- MMA issuer (lane 0) ----------------
    if (lane == 0) {
      int64_t step = 0;
      int seg = 0;
      bool ok = true;
      for (int64_t s = s_begin; s < s_end && ok; ++seg) {
        const int64_t u = sc.unit_of(s);
        const int64_t us = sc.ustart(u);
        const int k0 = static_cast<int>(s - us);
        const int k1 = static_cast<int>(min64(static_cast<int64_t>(sc.Su), s_end - us));
        const int buf = seg & 1;
        if (seg >= 2 && !mbar_wait(&bars->acc_empty[buf], static_cast<uint32_t>(((seg >> 1) - 1) & 1))) {
          report(a.status, HS_DEV_TIMEOUT);
          break;
        }
        tc5::fence_after_sync();
        const uint32_t acc = tmem + buf * kAcc;
        const int first_rt = k0 > sc.nsh ? k0 : sc.nsh;  // first routed step of the segment
        for (int k = k0; k < k1; ++k, ++step) {
          const int st = static_cast<int>(step % S_);
          if (!mbar_wait(&bars->full[st], static_cast<uint32_t>((step / S_) & 1))) {
            report(a.status, HS_DEV_TIMEOUT);
            ok = false;
            break;
          }
          tc5::fence_after_sync();
          uint8_t* S = base + st * L::kStage;
          const uint32_t sA = smem_u32(S), sB = smem_u32(S + L::kA), sSF = smem_u32(S + L::kA + L::kB);
          const uint32_t sfa0 = tmem + kSfa + st * 8;
          const uint32_t sfb = tmem + kSfb + st * 8;
          if (kCl && step == 0) HS_STAMP(hs_tslot, ::hs::trace::kDown, c, 3);
          tc5::cp_sf_32x128b(sfb, tc5::sdesc_sf(sSF + 1024));
          tc5::cp_sf_32x128b(sfb + 4, tc5::sdesc_sf(sSF + 1280));
          tc5::cp_sf_32x128b(sfa0, tc5::sdesc_sf(sSF));
          tc5::cp_sf_32x128b(sfa0 + 4, tc5::sdesc_sf(sSF + 512));
          const bool shared = k < sc.nsh;
          const uint32_t afmt = shared ? 0u : 5u;
          const uint32_t dcol = acc + (shared ? kAccSh : 0u);
          const bool first = shared ? (k == k0) : (k == first_rt);
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const uint64_t ad = tc5::sdesc_sw128(sA + i * kBoxBytes);
            const uint64_t bd = tc5::sdesc_sw128(sB + i * 2048);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint32_t id = tc5::idesc_mxf8f6f4(afmt, N, j, j);
              const uint32_t accum = (first && i == 0 && j == 0) ? 0u : 1u;
              tc5::mma_mxf8f6f4(dcol, ad + 2 * j, bd + 2 * j, id, accum,
                                (sfa0 + 4 * i) | (static_cast<uint32_t>(j) << 30),
                                (sfb + 4 * i) | (static_cast<uint32_t>(j) << 30));
            }
          }
          tc5::commit(&bars->empty[st]);
        }
        tc5::commit(&bars->acc_full[buf]);
        s = us + k1;
      }
      if (kCl) HS_STAMP(hs_tslot, ::hs::trace::kDown, c, 4);
      bars->consumed = static_cast<int32_t>(step);
      tc5::commit(&bars->mma_done);
      if (!mbar_wait(&bars->mma_done, 0)) report(a.status, HS_DEV_TIMEOUT);
    }
  } else if constexpr (kCl) {
    // ---------------- epilogue, cluster mode (one segment) ----------------
    const int row = 32 * warp + lane;
    const uint32_t lane_off = static_cast<uint32_t>(32 * warp) << 16;
    // the residual element this thread adds in the reduction below, loaded now
    // (row rpr * rank + tid % 16 of the tile, token tid / 16)
    {
      const int rpr = (kM + a.ncl - 1) / a.ncl;
      const int rl = threadIdx.x & 15, rowc = static_cast<int>(cg::this_cluster().block_rank()) * rpr + rl;
      if (a.resid_out && (threadIdx.x >> 4) < a.T && rl < rpr && rowc < kM)
        res_pre = __bfloat162float(a.resid[(threadIdx.x >> 4) * static_cast<int64_t>(D) + (c / a.ncl) * kM + rowc]);
    }
    float r[8], h[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) r[t] = h[t] = 0.f;
    if (s_begin < s_end) {
      const int64_t us = sc.ustart(sc.unit_of(s_begin));
      const int k0 = static_cast<int>(s_begin - us), k1 = static_cast<int>(s_end - us);
      if (mbar_wait(&bars->acc_full[0], 0)) {
        if (threadIdx.x == 0) HS_STAMP(hs_tslot, ::hs::trace::kDown, c, 6);
        tc5::fence_after_sync();
        float c0[16], c1[16];
        tc5::ld_32x32b_x16(tmem + lane_off, c0);
        tc5::ld_32x32b_x16(tmem + lane_off + kAccSh, c1);
        tc5::wait_ld();
        tc5::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->acc_empty[0]);
        const bool had_sh = k0 < sc.nsh, had_rt = k1 > sc.nsh;
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          r[t] = had_rt ? c0[t] + c0[8 + t] : 0.f;
          h[t] = had_sh ? c1[t] + c1[8 + t] : 0.f;
        }
      } else if (threadIdx.x == 0) {
        report(a.status, HS_DEV_TIMEOUT);
      }
    }
    // park this CTA's partial rows in stage 0 (every stage is consumed once
    // the accumulator is complete): [token t][row] pairs (routed, shared)
    float2* red = reinterpret_cast<float2*>(base);
#pragma unroll
    for (int t = 0; t < 8; ++t) red[t * kM + row] = make_float2(r[t], h[t]);
  } else {
    // ---------------- epilogue (warps 0-3, TMEM lanes 32w..32w+31) ----------------
    const int row = 32 * warp + lane;
    const int etid = threadIdx.x;
    const uint32_t lane_off = static_cast<uint32_t>(32 * warp) << 16;
    int seg = 0;
    for (int64_t s = s_begin; s < s_end; ++seg) {
      const int64_t u = sc.unit_of(s);
      const int64_t us = sc.ustart(u);
      const int nk = sc.Su;
      const int k0 = static_cast<int>(s - us);
      const int k1 = static_cast<int>(min64(static_cast<int64_t>(nk), s_end - us));
      const int buf = seg & 1;
      if (!mbar_wait(&bars->acc_full[buf], static_cast<uint32_t>((seg >> 1) & 1))) {
        if (etid == 0) report(a.status, HS_DEV_TIMEOUT);
        break;
      }
      tc5::fence_after_sync();
      float c0[16], c1[16];
      const uint32_t acc = tmem + lane_off + buf * kAcc;
      tc5::ld_32x32b_x16(acc, c0);
      tc5::ld_32x32b_x16(acc + kAccSh, c1);
      tc5::wait_ld();
      tc5::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->acc_empty[buf]);
      const bool had_sh = k0 < sc.nsh, had_rt = k1 > sc.nsh;
      float r[8], h[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        r[t] = had_rt ? c0[t] + c0[8 + t] : 0.f;
        h[t] = had_sh ? c1[t] + c1[8 + t] : 0.f;
      }
      const int cf = sc.cta_of(us);
      const int cl = sc.cta_of(us + nk - 1);
      bool finish = (cf == cl);
      if (!finish) {
        float* slot = a.part + (2 * static_cast<int64_t>(c) + (u == sc.unit_of(s_begin) ? 0 : 1)) * kSlot;
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          __stcg(slot + t * kM + row, r[t]);
          __stcg(slot + (8 + t) * kM + row, h[t]);
        }
        __threadfence();
        epi_bar();
        if (etid == 0) {
          const uint32_t mine = static_cast<uint32_t>(k1 - k0);
          bars->flag = atomicAdd(&a.ucount[u], mine) + mine == static_cast<uint32_t>(nk);
        }
        epi_bar();
        finish = bars->flag != 0;
        epi_bar();
        if (finish) {
          __threadfence();
          float rh[16];
          sum_slots<16>(sc, cf, cl, us, a.part, kSlot, row, rh);
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            r[t] = rh[t];
            h[t] = rh[8 + t];
          }
        }
      }
      if (finish) {
        const int64_t dd = u * kM + row;
#pragma unroll
        for (int t = 0; t < 8; ++t)
          if (t < a.T) store_out(a, t * static_cast<int64_t>(D) + dd, r[t], h[t]);
      }
      s = us + k1;
    }
    // nothing to compute (every pair skipped, no shared expert): zeros
    if (!any)
      for (int tile = c; tile < D / kM; tile += sc.G)
        for (int t = 0; t < a.T; ++t) store_out(a, t * static_cast<int64_t>(D) + tile * kM + etid, 0.f, 0.f);
  }

  if constexpr (kCl) {
    // the tile's n partial accumulators, summed in rank order: rank j reduces
    // rows rpr j .. rpr (j + 1) - 1 (rpr = ceil(128 / n) <= 16), thread (row,
    // token) reads its two values from all n and adds the residual element it
    // loaded before the accumulator was ready
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    if (threadIdx.x == 0) HS_STAMP(hs_tslot, ::hs::trace::kDown, c, 7);
    bool ep_poisoned = false;
    if (a.ep_world > 0) {  // this call's slot (the local call counter, advanced by the previous combine)
      const volatile uint64_t* hdr = reinterpret_cast<volatile const uint64_t*>(a.ep_recv[a.ep_rank]);
      ep_slot = static_cast<int>(hdr[0] & 1u);
      ep_poisoned = hdr[epx::kPoison] != 0u;  // an earlier combine gave up: store nothing
    }
    const int rpr = (kM + a.ncl - 1) / a.ncl;
    // thread (token tid / 16, row tid % 16): a warp covers 16 consecutive rows
    // of two tokens, so its output (and peer) stores are contiguous runs
    const int rl = threadIdx.x & 15, t = threadIdx.x >> 4;
    const int rowc = static_cast<int>(cluster.block_rank()) * rpr + rl;
    const bool mine = warp < 4 && rl < rpr && rowc < kM;
    float rs = 0.f, hs = 0.f;
    if (mine) {
      // all remote loads issued before the sum (eight at a time)
      const float2* red = reinterpret_cast<const float2*>(base);
      for (int q0 = 0; q0 < a.ncl; q0 += 8) {
        float2 v[8];
#pragma unroll
        for (int q = 0; q < 8; ++q)
          v[q] = q0 + q < a.ncl ? ld_dsmem_f2(dsmem_addr(red + t * kM + rowc, static_cast<uint32_t>(q0 + q)))
                                : make_float2(0.f, 0.f);
#pragma unroll
        for (int q = 0; q < 8; ++q)
          if (q0 + q < a.ncl) {
            rs += v[q].x;
            hs += v[q].y;
          }
      }
    }
    // this CTA has read its peers: let them leave (the arrival orders the
    // reads before it), store meanwhile, and wait for them before leaving
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    if (mine && t < a.T) {
      if (a.ep_world > 0) {
        // this rank's routed and shared sums into every rank's slot (each
        // entry is its own arrival flag)
        const int64_t o_i = t * static_cast<int64_t>(D) + (c / a.ncl) * kM + rowc;
        for (int q = 0; q < a.ep_world && !ep_poisoned; ++q) {
          epx::rows(a.ep_recv[q], ep_slot, a.ep_world, a.ep_rank, 0, D)[o_i] = rs;
          epx::rows(a.ep_recv[q], ep_slot, a.ep_world, a.ep_rank, 1, D)[o_i] = hs;
        }
      } else {
        store_out(a, t * static_cast<int64_t>(D) + (c / a.ncl) * kM + rowc, rs, hs, res_pre);
      }
    }
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
  }

  tc5::fence_before_sync();
  __syncthreads();

  if (threadIdx.x == 128) {
    for (int64_t k = bars->consumed; k < bars->issued; ++k)
      if (!mbar_wait(&bars->full[k % S_], static_cast<uint32_t>((k / S_) & 1))) {
        report(a.status, HS_DEV_TIMEOUT);
        break;
      }
  }
  __syncthreads();
  if (warp == 0) {
  if (kCl && threadIdx.x == 0) HS_STAMP(hs_tslot, ::hs::trace::kDown, c, 5);
    tc5::fence_after_sync();
    tc5::tmem_dealloc(tmem, 256);
  }
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

// 3D map [planes][rows][cols] with planes plane_rows rows apart (rows <=
// plane_rows visible; rows beyond read as zero): box cols x box_rows x planes,
// 128B swizzle.
static int make_map_3d(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows, uint64_t planes,
                       uint64_t pitch, uint32_t box_rows, uint64_t plane_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return HS_ERR_UNSUPPORTED;
  cuuint64_t dims[3] = {cols, rows, planes};
  cuuint64_t strides[2] = {pitch, pitch * plane_rows};
  cuuint32_t box[3] = {128, box_rows, static_cast<cuuint32_t>(planes)};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_cuda_error(static_cast<int>(r));
    return HS_ERR_CUDA;
  }
  return HS_OK;
}

static bool dim_ok(int64_t v, int64_t mult, int64_t lo, int64_t hi) { return v % mult == 0 && v >= lo && v <= hi; }
static bool aligned32(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 31u) == 0; }

// Number of SMs of the current device, cached.
static int sm_count() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int v = cache[dev].load();
  if (v <= 0) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    cache[dev].store(v);
  }
  return v;
}

template <bool kDown, int NT, bool kTok = false>
static int launch_sk(const Desc& d, const CallMaps& cm, const UnitArgs& a, cudaStream_t st) {
  constexpr int bytes = SmemLayout<NT, kDown ? 2 : 1>::kBytes;
  static std::atomic<uint64_t> done{0};
  int dev = 0;
  HS_CUDA_CHECK(cudaGetDevice(&dev));
  const uint64_t bit = 1ull << (dev & 63);
  if (!(done.load() & bit)) {
    HS_CUDA_CHECK(
        cudaFuncSetAttribute(sk_kernel<kDown, NT, kTok>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    done.fetch_or(bit);
  }
  HS_CUDA_CHECK(launch_pdl(sk_kernel<kDown, NT, kTok>, dim3(static_cast<unsigned>(a.G)), dim3(kThreads), bytes, st,
                           d, cm, a));
  return check_launch();
}

// An empty kernel with the token-mode down kernel's launch shape (threads,
// shared memory, two CTAs per SM): the occupancy calculator's answer for it is
// how many clusters of a given size the GPCs can hold at once. (For the
// tcgen05 kernels themselves it reports one CTA per SM, while two run.)
__global__ void __launch_bounds__(kThreads, kCtasPerSm) cluster_fit_probe() {}

// Cluster size for the token-mode down phase with `tiles` tiles of D: the
// largest n in [8, 16] whose n * tiles CTAs fit the two-per-SM budget and whose
// `tiles` clusters can all be resident at once; 0 when none (stream-K then).
// More CTAs per tile leave fewer SMs running a single CTA, which streams at
// twice the rate of a paired one and would idle at the end.
static int tok_down_cluster(int tiles, int bytes) {
  static std::mutex mu;
  static int cached[64][65];
  static bool have[64][65];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64 || tiles > 64) return 0;
  std::lock_guard<std::mutex> lk(mu);
  if (have[dev][tiles]) return cached[dev][tiles];
  int best = 0;
  if (cudaFuncSetAttribute(cluster_fit_probe, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) == cudaSuccess &&
      cudaFuncSetAttribute(cluster_fit_probe, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess) {
    for (int n = 16; n >= 8 && !best; --n) {
      if (n * tiles > kCtasPerSm * sm_count()) continue;
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(static_cast<unsigned>(n * tiles));
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = static_cast<size_t>(bytes);
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = static_cast<unsigned>(n);
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int m = 0;
      if (cudaOccupancyMaxActiveClusters(&m, cluster_fit_probe, &cfg) == cudaSuccess && m >= tiles) best = n;
    }
  }
  (void)cudaGetLastError();
  cached[dev][tiles] = best;
  have[dev][tiles] = true;
  return best;
}

static int launch_tok_down(const Desc& d, const CallMaps& cm, UnitArgs a, cudaStream_t st, int* grid_out = nullptr) {
  constexpr int bytes = SmemLayout<1, 2>::kBytes + kTokDownPad;
  static_assert(bytes <= kSmemPerCta, "down kernel shared memory");
  static std::atomic<uint64_t> done{0};
  int dev = 0;
  HS_CUDA_CHECK(cudaGetDevice(&dev));
  const uint64_t bit = 1ull << (dev & 63);
  if (!(done.load() & bit)) {
    HS_CUDA_CHECK(cudaFuncSetAttribute(tok_down_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    HS_CUDA_CHECK(cudaFuncSetAttribute(tok_down_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    HS_CUDA_CHECK(cudaFuncSetAttribute(tok_down_kernel<true>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    done.fetch_or(bit);
  }
  const int tiles = d.D / kM;
  // One cluster of n CTAs per tile (D = 4096 on a B200: 32 clusters)
  const int n = tok_down_cluster(tiles, bytes);
  if (n > 0) {
    a.ncl = n;
    a.G = n * tiles;
    if (grid_out) *grid_out = a.G;
    HS_CUDA_CHECK(launch_pdl_cluster(tok_down_kernel<true>, dim3(static_cast<unsigned>(a.G)), dim3(kThreads), bytes,
                                     st, static_cast<unsigned>(n), d, cm, a));
    return check_launch();
  }
  if (a.ep_world > 0) return HS_ERR_UNSUPPORTED;  // the peer exchange runs on the cluster epilogue
  HS_CUDA_CHECK(
      launch_pdl(tok_down_kernel<false>, dim3(static_cast<unsigned>(a.G)), dim3(kThreads), bytes, st, d, cm, a));
  return check_launch();
}

template <bool kDown>
static int launch_nt(int NT, const Desc& d, const CallMaps& cm, const UnitArgs& a, cudaStream_t st) {
  switch (NT) {
    case 1:
      return launch_sk<kDown, 1>(d, cm, a, st);
    case 2:
      return launch_sk<kDown, 2>(d, cm, a, st);
    default:
      return launch_sk<kDown, 3>(d, cm, a, st);
  }
}

// ---------------------------------------------------------------------------
// Token-major grouped GEMM for large calls (many pairs per expert)
// ---------------------------------------------------------------------------
// The kernels above put 128 weight rows on the MMA's M side and at most 24
// pairs (48 hi/lo columns) on N, so each weight tile feeds few MACs and a
// large call is bound by MMA issue. Here the roles swap: A = 128 consecutive
// pair rows of one expert's chunk, as the hi and lo e4m3 planes (two MMAs into
// one accumulator), and B = two 128-row weight tiles, one N = 128 accumulator
// each (gate/up: the w1 and w3 tiles; down: the w2 tiles of two consecutive
// 128-row slices of D, so each A tile feeds twice the MACs). A's scale factors are all 1;
// each pair row's power-of-two prescale (2^e of the token row for gate/up,
// 2^q of the activation for down) is undone in the epilogue, which is exact.
// One CTA per SM: warp 8 streams TMA, warp 9 issues tcgen05 copies and MMAs,
// warps 0-7 drain TMEM (two warps per pair row quadrant, half the columns
// each: the gate/up accumulator is single-buffered, so its epilogue is on the
// MMA's critical path). Units (chunk x weight tile,
// chunk-major so the CTAs on one chunk share its A rows through L2) go to the
// CTAs round-robin and are never split. The down phase writes per-pair f32
// rows and combine_rows_kernel sums them per token.
constexpr int kTmCh = 128;                    // pairs per chunk (the MMA's M)
constexpr int kTmThreads = 320;               // warps 0-7 epilogue, warp 8 TMA, warp 9 MMA
constexpr int64_t kTmMinPairsPerExpert = 32;  // token-major once T*K >= this * E

template <bool kDown>
struct TmLayout {
  static constexpr int kA = 2 * kBoxBytes;  // hi and lo planes of 128 pair rows
  static constexpr int kB = 2 * kBoxBytes;  // the w1 and w3 tiles, or two w2 tiles (256 rows of D)
  static constexpr int kSF = 2 * 512;       // their scale-factor atoms
  static constexpr int kStage = (kA + kB + kSF + 1023) / 1024 * 1024;
  static constexpr int kStages = 3;
  static constexpr int kSfaOff = kStages * kStage;  // the all-ones A scale atom (512 B)
  static constexpr int kBarOff = kSfaOff + 512;
  static constexpr int kBytes = kBarOff + 256 + 1024;  // + slack to realign the base to 1024
};

struct TmBars {
  uint64_t full[4];
  uint64_t empty[4];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t mma_done;
  uint32_t tmem;
  int32_t issued, consumed;
};

// Down-phase weight maps with one 128-row tile (one k-step) per box.
struct TmMaps {
  CUtensorMap w2;
  CUtensorMap sw2;
};

struct TmUnit {
  int shared, e, pair0, np, tile;
};

__device__ __forceinline__ TmUnit tm_unit(const UnitArgs& a, int64_t u, int tiles_sh, int tiles_rt,
                                          int64_t n_sh_units) {
  TmUnit r;
  if (u < n_sh_units) {
    const int c = static_cast<int>(u / tiles_sh);
    r.shared = 1;
    r.tile = static_cast<int>(u - static_cast<int64_t>(c) * tiles_sh);
    r.e = 0;
    r.pair0 = c * kTmCh;  // the shared expert's rows are the token rows 0..T-1
    r.np = min(kTmCh, a.T - r.pair0);
  } else {
    const int64_t uu = u - n_sh_units;
    const int c = static_cast<int>(uu / tiles_rt);
    r.shared = 0;
    r.tile = static_cast<int>(uu - static_cast<int64_t>(c) * tiles_rt);
    r.e = __ldcg(a.P.chunk_expert + c);
    r.pair0 = __ldcg(a.P.chunk_pair0 + c);
    r.np = __ldcg(a.P.chunk_np + c);
  }
  return r;
}

template <bool kDown>
__global__ void __launch_bounds__(kTmThreads, 1) tm_kernel(const __grid_constant__ Desc d,
                                                         const __grid_constant__ CallMaps cm,
                                                         const __grid_constant__ TmMaps tmm, UnitArgs a) {
  using L = TmLayout<kDown>;
  constexpr int S_ = L::kStages;
  constexpr int NB = 1;                // accumulator buffers (256 columns each)
  constexpr uint32_t kAccCols = 256u;  // gate at +0, up at +128; down: D-tiles 2j at +0, 2j+1 at +128
  constexpr uint32_t kSfa = 256;                      // the all-ones A scale atom
  constexpr uint32_t kSfb = 264;                      // B scale atoms, 8 columns per stage
  static_assert(kSfb + 8 * S_ <= 512, "TMEM columns");
  static_assert(sizeof(TmBars) <= 256, "barrier block");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  TmBars* bars = reinterpret_cast<TmBars*>(base + L::kBarOff);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D = d.D;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S_; ++i) {
      mbar_init(&bars->full[i], 1);
      mbar_init(&bars->empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->acc_full[i], 1);
      mbar_init(&bars->acc_empty[i], 8);
    }
    mbar_init(&bars->mma_done, 1);
    bars->issued = 0;
    bars->consumed = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    for (int i = lane; i < 128; i += 32) reinterpret_cast<uint32_t*>(base + L::kSfaOff)[i] = 0x7f7f7f7fu;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 0) tc5::tmem_alloc(&bars->tmem, 512);
  if (warp == 8 && lane == 0) {
    prefetch_tensormap(kDown ? &tmm.w2 : &d.tm_w13);
    prefetch_tensormap(kDown ? &tmm.sw2 : &d.tm_sw13);
    prefetch_tensormap(kDown ? &cm.tm_act8 : &cm.tm_x8);
  }
  pdl_wait();
  pdl_trigger();
  tc5::fence_before_sync();
  __syncthreads();
  tc5::fence_after_sync();
  const uint32_t tmem = bars->tmem;
  const int tiles_sh = kDown ? D / (2 * kM) : (d.has_shared ? d.I_sh / kM : 1);
  const int tiles_rt = kDown ? D / (2 * kM) : d.I / kM;
  const int64_t n_sh_units = static_cast<int64_t>(a.n_sh_chunks) * tiles_sh;
  const int64_t U = n_sh_units + static_cast<int64_t>(__ldcg(a.P.hdr)) * tiles_rt;
  const int nk_sh = kDown ? d.I_sh / kM : D / kM;
  const int nk_rt = kDown ? d.I / kM : D / kM;
  const int64_t G = gridDim.x;

  if (warp == 8) {
    // ---------------- TMA producer (whole warp; lane 0 issues) ----------------
    int64_t step = 0;
    bool ok = true;
    for (int64_t u = blockIdx.x; u < U && ok; u += G) {
      const TmUnit ui = tm_unit(a, u, tiles_sh, tiles_rt, n_sh_units);
      const bool fp8 = ui.shared != 0;
      const int nk = fp8 ? nk_sh : nk_rt;
      const CUtensorMap* wm = kDown ? (fp8 ? &tmm.sw2 : &tmm.w2) : (fp8 ? &d.tm_sw13 : &d.tm_w13);
      const CUtensorMap* am = kDown ? &cm.tm_act8 : &cm.tm_x8;
      // the unit's first weight tile. gate/up: a (w1, w3) tile pair per k-step,
      // adjacent; down: tiles 2j and 2j+1 of D, nk tiles apart
      int64_t t0;
      const uint8_t* sf0;
      if (!kDown) {
        t0 = fp8 ? static_cast<int64_t>(ui.tile) * (D / kM)
                 : (static_cast<int64_t>(ui.e) * (d.I / kM) + ui.tile) * (D / kM);
        sf0 = (fp8 ? d.sh_s13a : d.s13a) + t0 * 1024;
      } else {
        t0 = fp8 ? static_cast<int64_t>(2 * ui.tile) * nk_sh
                 : (static_cast<int64_t>(ui.e) * (D / kM) + 2 * ui.tile) * nk_rt;
        sf0 = (fp8 ? d.sh_s2a : d.s2a) + t0 * 512;
      }
      const int64_t y0 = t0 * (kDown ? kM : 2 * kM);
      // transaction bytes: both A planes, the weight tiles as stored in global
      // memory (packed e2m1 is half the shared-memory footprint), the atoms
      const uint32_t wbytes = fp8 ? kBoxBytes : kBoxBytes / 2;
      const uint32_t tx = 2 * kBoxBytes + 2u * wbytes + L::kSF;
      for (int k = 0; k < nk; ++k, ++step) {
        const int st = static_cast<int>(step % S_);
        if (step >= S_) {
          bool w = true;
          if (lane == 0) w = mbar_wait(&bars->empty[st], static_cast<uint32_t>(((step / S_) - 1) & 1));
          w = __shfl_sync(0xffffffffu, w ? 1 : 0, 0) != 0;
          if (!w) {
            if (lane == 0) report(a.status, HS_DEV_TIMEOUT);
            ok = false;
            break;
          }
        }
        if (lane == 0) {
          uint8_t* S = base + st * L::kStage;
          mbar_arrive_expect_tx(&bars->full[st], tx);
          tma_load_3d(S, am, &bars->full[st], k * 128, ui.pair0, 0);
          if (!kDown) {
            tma_load_2d(S + L::kA, wm, &bars->full[st], 0, static_cast<int>(y0 + static_cast<int64_t>(k) * 2 * kM));
            bulk_load(S + L::kA + L::kB, sf0 + static_cast<int64_t>(k) * 1024, 1024, &bars->full[st]);
          } else {
#pragma unroll
            for (int i = 0; i < 2; ++i) {
              const int64_t tk = static_cast<int64_t>(i) * nk + k;  // tile 2j + i, k-step k
              tma_load_2d(S + L::kA + i * kBoxBytes, wm, &bars->full[st], 0, static_cast<int>(y0 + tk * kM));
              bulk_load(S + L::kA + L::kB + i * 512, sf0 + tk * 512, 512, &bars->full[st]);
            }
          }
        }
        __syncwarp();
      }
    }
    if (lane == 0) bars->issued = static_cast<int32_t>(step);
  } else if (warp == 9) {
    // ---------------- MMA issuer (lane 0) ----------------
    if (lane == 0) {
      tc5::cp_sf_32x128b(tmem + kSfa, tc5::sdesc_sf(smem_u32(base + L::kSfaOff)));
      int64_t step = 0;
      int seg = 0;
      bool ok = true;
      for (int64_t u = blockIdx.x; u < U && ok; u += G, ++seg) {
        const bool fp8 = u < n_sh_units;
        const int nk = fp8 ? nk_sh : nk_rt;
        const uint32_t bfmt = fp8 ? 0u : 5u;
        const int buf = seg % NB;
        if (seg >= NB && !mbar_wait(&bars->acc_empty[buf], static_cast<uint32_t>(((seg / NB) - 1) & 1))) {
          report(a.status, HS_DEV_TIMEOUT);
          break;
        }
        tc5::fence_after_sync();
        const uint32_t acc = tmem + buf * kAccCols;
        for (int k = 0; k < nk; ++k, ++step) {
          const int st = static_cast<int>(step % S_);
          if (!mbar_wait(&bars->full[st], static_cast<uint32_t>((step / S_) & 1))) {
            report(a.status, HS_DEV_TIMEOUT);
            ok = false;
            break;
          }
          tc5::fence_after_sync();
          uint8_t* S = base + st * L::kStage;
          const uint32_t sA = smem_u32(S), sB = smem_u32(S + L::kA), sSF = smem_u32(S + L::kA + L::kB);
          const uint32_t sfb = tmem + kSfb + st * 8;
          tc5::cp_sf_32x128b(sfb, tc5::sdesc_sf(sSF));
          tc5::cp_sf_32x128b(sfb + 4, tc5::sdesc_sf(sSF + 512));
          // one N = 256 MMA per plane and 32-column k-block: B is the two tiles
          // as 256 consecutive K-major rows (gate then up, or D-tile 2j then
          // 2j+1), its scale atoms in columns sfb (rows 0-127) and sfb + 4
          // (rows 128-255); the accumulator's columns follow B's rows
          const uint64_t bd = tc5::sdesc_sw128(sB);
#pragma unroll
          for (int h = 0; h < 2; ++h) {  // hi, lo planes
            const uint64_t ad = tc5::sdesc_sw128(sA + h * kBoxBytes);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint32_t id = tc5::idesc_mxf8f6f4_ab(0u, bfmt, 256, j, j);
              const uint32_t accum = (k > 0 || h > 0 || j > 0) ? 1u : 0u;
              tc5::mma_mxf8f6f4(acc, ad + 2 * j, bd + 2 * j, id, accum, (tmem + kSfa) | (static_cast<uint32_t>(j) << 30),
                                sfb | (static_cast<uint32_t>(j) << 30));
            }
          }
          tc5::commit(&bars->empty[st]);
        }
        tc5::commit(&bars->acc_full[buf]);
      }
      // every tcgen05 operation of this thread done before TMEM is freed
      bars->consumed = static_cast<int32_t>(step);
      tc5::commit(&bars->mma_done);
      if (!mbar_wait(&bars->mma_done, 0)) report(a.status, HS_DEV_TIMEOUT);
    }
  } else {
    // ---------------- epilogue (warps 0-7) ----------------
    // warp w reads TMEM lanes 32 (w % 4) .. +31 (its pair rows) and columns
    // [64 (w / 4), +64) of each accumulator
    const int row = 32 * (warp & 3) + lane;
    const uint32_t lane_off = static_cast<uint32_t>(32 * (warp & 3)) << 16;
    const int c0 = 64 * (warp >> 2);
    const int64_t I_act = max(d.I, d.has_shared ? d.I_sh : 0);
    int seg = 0;
    for (int64_t u = blockIdx.x; u < U; u += G, ++seg) {
      const TmUnit ui = tm_unit(a, u, tiles_sh, tiles_rt, n_sh_units);
      const int buf = seg % NB;
      const bool valid = row < ui.np;
      const int64_t p = static_cast<int64_t>(ui.pair0) + row;
      float rs = 0.f, wb = 0.f, qs = 0.f;
      if (valid) {
        if (kDown) {
          rs = exp2i(static_cast<int>(__ldcg(a.P.sb2 + p)) - 127);
        } else {
          rs = exp2i(static_cast<int>(__ldcg(a.P.sb1 + p)) - 127);
          wb = __ldcg(a.P.pair_wb + p);
          qs = exp2i(__ldcg(a.P.pair_q + p));
        }
      }
      if (!mbar_wait(&bars->acc_full[buf], static_cast<uint32_t>((seg / NB) & 1))) {
        if (threadIdx.x == 0) report(a.status, HS_DEV_TIMEOUT);
        break;
      }
      tc5::fence_after_sync();
      if constexpr (kDown) {
        // warp half h: columns [128 h, 128 h + 128) = D-tile 2j + h. All 128
        // values come into registers first and the accumulator is released
        // before the stores, which then overlap the next unit's MMAs
        const uint32_t accd = tmem + lane_off + buf * kAccCols + 128 * (warp >> 2);
        float* dst = a.P.out_part + p * D + ui.tile * (2 * kM) + 128 * (warp >> 2);
        float v[128];
#pragma unroll
        for (int g = 0; g < 8; ++g) tc5::ld_32x32b_x16(accd + g * 16, *reinterpret_cast<float(*)[16]>(v + 16 * g));
        tc5::wait_ld();
        tc5::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->acc_empty[buf]);
        if (valid) {
          float4* o = reinterpret_cast<float4*>(dst);
#pragma unroll
          for (int i = 0; i < 32; ++i)
            o[i] = make_float4(v[4 * i] * rs, v[4 * i + 1] * rs, v[4 * i + 2] * rs, v[4 * i + 3] * rs);
        }
      } else {
        const uint32_t acc = tmem + lane_off + buf * kAccCols + c0;
        const bool fp8 = ui.shared != 0;
        uint8_t* hi = a.P.act8 + p * I_act + ui.tile * kM + c0;
        uint8_t* lo = hi + a.act_rows * I_act;
        // the warp's 64 gate and 64 up values into registers, the accumulator
        // released, then the epilogue math overlaps the next unit's MMAs
        float gall[64], uall[64];
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          tc5::ld_32x32b_x16(acc + g * 16, *reinterpret_cast<float(*)[16]>(gall + 16 * g));
          tc5::ld_32x32b_x16(acc + 128 + g * 16, *reinterpret_cast<float(*)[16]>(uall + 16 * g));
        }
        tc5::wait_ld();
        tc5::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->acc_empty[buf]);
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          const float* gv = gall + 32 * g;
          const float* uv = uall + 32 * g;
          if (valid) {
            uint32_t hw[8] = {0, 0, 0, 0, 0, 0, 0, 0}, lw[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              // reference roundings as in gateup_finish
              const float gf = round_bf16(gv[i] * rs);
              const float uf = round_bf16(uv[i] * rs);
              const float gc = gf > 10.f ? 10.f : gf;
              const float uc = uf > 10.f ? 10.f : (uf < -10.f ? -10.f : uf);
              const float sig = 1.f / (1.f + expf(-gc));
              float av = round_bf16((gc * sig) * uc);
              if (!fp8) av = round_bf16(av * wb);
              const float v = av * qs;
              const __nv_fp8_storage_t hb = __nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
              const __half_raw hr = __nv_cvt_fp8_to_halfraw(hb, __NV_E4M3);
              const float hf = __half2float(*reinterpret_cast<const __half*>(&hr));
              const __nv_fp8_storage_t lb = __nv_cvt_float_to_fp8(v - hf, __NV_SATFINITE, __NV_E4M3);
              hw[i >> 2] |= static_cast<uint32_t>(hb) << (8 * (i & 3));
              lw[i >> 2] |= static_cast<uint32_t>(lb) << (8 * (i & 3));
            }
            uint4* ho = reinterpret_cast<uint4*>(hi + g * 32);
            uint4* lo4 = reinterpret_cast<uint4*>(lo + g * 32);
            ho[0] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            ho[1] = make_uint4(hw[4], hw[5], hw[6], hw[7]);
            lo4[0] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
            lo4[1] = make_uint4(lw[4], lw[5], lw[6], lw[7]);
          }
        }
      }
    }
  }

  tc5::fence_before_sync();
  __syncthreads();
  // copies issued but never consumed (only after a timed-out wait): let them
  // land before the CTA's shared memory is released
  if (threadIdx.x == 256) {  // the producer's lane 0
    for (int64_t k = bars->consumed; k < bars->issued; ++k)
      if (!mbar_wait(&bars->full[k % S_], static_cast<uint32_t>((k / S_) & 1))) {
        report(a.status, HS_DEV_TIMEOUT);
        break;
      }
  }
  __syncthreads();
  if (warp == 0) {
    tc5::fence_after_sync();
    tc5::tmem_dealloc(tmem, 512);
  }
}

template <bool kDown>
static int launch_tm(const Desc& d, const CallMaps& cm, const TmMaps& tmm, const UnitArgs& a, cudaStream_t st) {
  constexpr int bytes = TmLayout<kDown>::kBytes;
  static std::atomic<uint64_t> done{0};
  int dev = 0;
  HS_CUDA_CHECK(cudaGetDevice(&dev));
  const uint64_t bit = 1ull << (dev & 63);
  if (!(done.load() & bit)) {
    HS_CUDA_CHECK(cudaFuncSetAttribute(tm_kernel<kDown>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    done.fetch_or(bit);
  }
  HS_CUDA_CHECK(launch_pdl(tm_kernel<kDown>, dim3(static_cast<unsigned>(sm_count())), dim3(kTmThreads), bytes, st, d,
                           cm, tmm, a));
  return check_launch();
}


static int plan_smem(int E, int npairs) {
  const int cached = npairs <= kLocalPairs ? 2 * npairs : 0;  // ids and post-duplicate experts
  const int general = 4 * E + 2 + (kPlanThreads / 32) * E;
  const int fast = npairs <= kFastPlanPairs ? 4 * npairs : 0;
  return static_cast<int>((cached + std::max(general, fast)) * sizeof(int32_t));
}

static int launch_seg(const PlanArgs& pa, const Plan& P, int nseg, int32_t* seg_ws, cudaStream_t st) {
  const int64_t npairs = static_cast<int64_t>(pa.T) * pa.K;
  HS_CUDA_CHECK(launch_pdl(plan_seg_kernel, dim3(static_cast<unsigned>(nseg)), dim3(kSegPairs), 0, st, pa, P, seg_ws,
                           seg_ws + npairs, seg_ws + npairs + static_cast<int64_t>(nseg) * kSegMaxE));
  return check_launch();
}

static int launch_plan(const PlanArgs& pa, const Plan& P, int grid, cudaStream_t st) {
  const int smem = pa.seg_lrank ? 0 : plan_smem(pa.E, pa.T * pa.K);
  if (smem > 200 * 1024) return HS_ERR_BAD_SHAPE;
  static std::atomic<uint64_t> done{0};
  int dev = 0;
  HS_CUDA_CHECK(cudaGetDevice(&dev));
  const uint64_t bit = 1ull << (dev & 63);
  if (!(done.load() & bit)) {
    HS_CUDA_CHECK(cudaFuncSetAttribute(plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    done.fetch_or(bit);
  }
  // segmented plan: block 0 only clears counters, so the token CTAs get the
  // threads their row needs (16 values each) and twice as many fit per SM
  const int threads = pa.seg_lrank ? std::max(256, (pa.D / 16 + 31) / 32 * 32) : kPlanThreads;
  HS_CUDA_CHECK(launch_pdl(plan_kernel, dim3(grid), dim3(threads), smem, st, pa, P));
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
  // tiled weights: rows of 128 values (64 packed bytes), two tiles (256 rows) per box
  if ((st = make_map(&d.tm_w13, w->w13, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 128, E * 2 * I * (D / 128), 64, 128,
                     256)))
    return st;
  if ((st = make_map(&d.tm_w2, w->w2, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 128, E * D * (I / 128), 64, 128, 256)))
    return st;
  d.s13a = static_cast<const uint8_t*>(w->s13);
  d.s2a = static_cast<const uint8_t*>(w->s2);
  d.w13 = static_cast<const uint8_t*>(w->w13);
  d.w2 = static_cast<const uint8_t*>(w->w2);
  if (d.has_shared) {
    if (!dim_ok(w->I_sh, 256, 256, 8192)) return HS_ERR_BAD_SHAPE;
    if (!w->sh_s13 || !w->sh_w2 || !w->sh_s2) return HS_ERR_BAD_ARGUMENT;
    if (!aligned16(w->sh_w13) || !aligned16(w->sh_w2) || !aligned16(w->sh_s13) || !aligned16(w->sh_s2))
      return HS_ERR_ALIGN;
    d.I_sh = static_cast<int32_t>(w->I_sh);
    const uint64_t Ish = w->I_sh;
    if ((st = make_map(&d.tm_sw13, w->sh_w13, CU_TENSOR_MAP_DATA_TYPE_UINT8, 128, 2 * Ish * (D / 128), 128, 128,
                       256)))
      return st;
    if ((st = make_map(&d.tm_sw2, w->sh_w2, CU_TENSOR_MAP_DATA_TYPE_UINT8, 128, D * (Ish / 128), 128, 128, 256)))
      return st;
    d.sh_s13a = static_cast<const uint8_t*>(w->sh_s13);
    d.sh_s2a = static_cast<const uint8_t*>(w->sh_s2);
    d.sh_w13 = static_cast<const uint8_t*>(w->sh_w13);
    d.sh_w2 = static_cast<const uint8_t*>(w->sh_w2);
  }
  d.magic = kDescMagic;
  memset(desc_out, 0, desc_bytes);
  memcpy(desc_out, &d, sizeof(d));
  return HS_OK;
}

// The dimensions a descriptor was built for (E = the experts its store holds).
int hs::moe_desc_dims(const void* desc, int64_t* E, int64_t* D, int64_t* I, int64_t* I_sh) {
  if (!desc) return HS_ERR_BAD_ARGUMENT;
  Desc d;
  memcpy(&d, desc, sizeof(d));
  if (d.magic != kDescMagic) return HS_ERR_BAD_ARGUMENT;
  *E = d.E;
  *D = d.D;
  *I = d.I;
  *I_sh = d.has_shared ? d.I_sh : 0;
  return HS_OK;
}

extern "C" size_t hs_moe_workspace_size(int64_t T, int64_t top_k, int64_t D, int64_t I, int64_t I_sh) {
  if (T < 0 || top_k < 1) return 0;
  return geometry(T, top_k, D, I, I_sh, kCtasPerSm * sm_count()).total;
}

// Both MoE entry points: `partials` = 0 writes the bf16 output (and optionally
// the routed f32 sum); 1 writes the un-rounded f32 routed and shared sums only.
// Routing folded into the MoE call (token mode): the router's inputs and outputs.
struct RouteIn {
  const void* gate;
  const void* bias;
  int64_t num_experts, expert_offset;
  float scaling;
  int64_t* idx_out;
  float* w_out;
  // the layer form: rows are the residual stream, normed in the route kernel,
  // and the down phase adds the MoE output back (norm_w == nullptr: normed rows)
  const void* norm_w = nullptr;
  float eps = 0.f;
  void* x_out = nullptr;
  void* h_out = nullptr;
  const int64_t* ids = nullptr;      // hash routing when tid2eid is set
  const int64_t* tid2eid = nullptr;
  int64_t vocab = 0;
  const hs_ep_peers* ep = nullptr;   // peer-memory expert parallelism (layer form)
  // chained expert parallelism: the route kernel first completes the previous
  // call's exchange into the rows (in place), and this call's exchange is left
  // pending for the next call (or hs_ep_combine_pending)
  int chain_prev = 0, chain_prev_shared = 0;
  bool defer = false;
};

static uint64_t ep_wait_limit(const hs_ep_peers* pe) {
  return pe->wait_limit_ns > 0 ? static_cast<uint64_t>(pe->wait_limit_ns) : kWaitLimitNs;
}

static int launch_route(const RouteArgs& ra, const Plan& P, const Desc& d, cudaStream_t st) {
  const int ncta = ra.E / 16;
  const size_t bytes = RouteSmem::bytes(ra.D);
  static std::atomic<uint64_t> done{0};
  int dev = 0;
  HS_CUDA_CHECK(cudaGetDevice(&dev));
  const uint64_t bit = 1ull << (dev & 63);
  if (!(done.load() & bit)) {
    HS_CUDA_CHECK(cudaFuncSetAttribute(route_plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(RouteSmem::bytes(kRouteMaxD))));
    HS_CUDA_CHECK(cudaFuncSetAttribute(route_plan_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    done.fetch_or(bit);
  }
  HS_CUDA_CHECK(launch_pdl_cluster(route_plan_kernel, dim3(static_cast<unsigned>(ncta)), dim3(kRouteThreads), bytes,
                                   st, static_cast<unsigned>(ncta), ra, P, d));
  return check_launch();
}

static int launch_ep_combine(uint8_t* buf, int world, int64_t T, int D, int use_shared, const __nv_bfloat16* h,
                             __nv_bfloat16* h_out, int32_t* status, uint64_t limit, cudaStream_t st) {
  const int64_t n = T * D;
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, 64));
  HS_CUDA_CHECK(launch_pdl(ep_combine_kernel, dim3(grid), dim3(256), 0, st, buf, world, static_cast<int>(T), D,
                           use_shared, h, h_out, status, limit));
  return check_launch();
}

static int moe_ffn_impl(const void* desc, const void* hidden, const int64_t* topk_idx, const float* topk_w,
                        int64_t T, int64_t top_k, int use_shared, int dup_mode, void* out, float* out_f32,
                        float* shared_f32, int partials, void* workspace, size_t workspace_bytes,
                        int32_t* dev_status, void* stream, const RouteIn* route = nullptr) {
  if (!desc) return HS_ERR_BAD_ARGUMENT;
  Desc d;
  memcpy(&d, desc, sizeof(d));
  if (d.magic != kDescMagic) return HS_ERR_BAD_ARGUMENT;
  if (T < 0 || top_k < 1 || top_k > 16) return HS_ERR_BAD_SHAPE;
  if (T == 0) return HS_OK;
  if (T > (1 << 20)) return HS_ERR_BAD_SHAPE;
  if (!hidden || !workspace) return HS_ERR_BAD_ARGUMENT;
  if (!route && (!topk_idx || !topk_w)) return HS_ERR_BAD_ARGUMENT;
  const bool layer = route && route->norm_w;
  if (route) {
    const int64_t Er = route->num_experts;
    const bool hash = route->tid2eid != nullptr;
    if (T > kTokMax || Er < 16 || Er > 256 || Er % 16 || d.D > kRouteMaxD || d.D % (Er / 16 * 16) ||
        (!hash && d.D % router::kKSplitCols) || top_k > Er || route->expert_offset < 0 ||
        route->expert_offset + d.E > Er)
      return HS_ERR_UNSUPPORTED;
    if ((!hash && !route->gate) || (hash && (!route->ids || route->vocab < 1)) || !route->idx_out || !route->w_out)
      return HS_ERR_BAD_ARGUMENT;
    if ((route->gate && !aligned16(route->gate)) || (route->norm_w && !aligned16(route->norm_w)) ||
        (route->x_out && !aligned16(route->x_out)))
      return HS_ERR_ALIGN;
    if (layer && !partials && !route->h_out) return HS_ERR_BAD_ARGUMENT;
    if (route->ep) {
      const hs_ep_peers* pe = route->ep;
      if (!layer || partials || pe->world < 1 || pe->world > HS_EP_MAX_RANKS || pe->rank < 0 ||
          pe->rank >= pe->world)
        return HS_ERR_BAD_ARGUMENT;
      for (int q = 0; q < pe->world; ++q)
        if (!pe->recv[q] || !aligned16(pe->recv[q])) return HS_ERR_BAD_ARGUMENT;
    }
  }
  if (partials ? !out_f32 : (!out && !(layer && route->h_out))) return HS_ERR_BAD_ARGUMENT;
  if (dup_mode != HS_DUP_LAST && dup_mode != HS_DUP_SUM) return HS_ERR_BAD_ARGUMENT;
  if (!aligned16(hidden) || (out && !aligned16(out)) || !aligned16(workspace) || (out_f32 && !aligned16(out_f32)) ||
      (shared_f32 && !aligned16(shared_f32)))
    return HS_ERR_ALIGN;
  use_shared = (use_shared && d.has_shared) ? 1 : 0;
  if (partials && use_shared && !shared_f32) return HS_ERR_BAD_ARGUMENT;
  if (!d.has_shared) d.I_sh = 0;
  const Geometry g = geometry(T, top_k, d.D, d.I, d.has_shared ? d.I_sh : 0, kCtasPerSm * sm_count());
  if (workspace_bytes < g.total) return HS_ERR_WORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const Plan P = plan_views(g, workspace);
  const int NT = static_cast<int>(ntiles(T));
  const int64_t npairs = T * top_k;
  // many pairs per expert: the token-major kernels, chunks of 128 pairs
  const bool tmaj = T > kTokMax && !route && npairs >= kTmMinPairsPerExpert * d.E;
  const int CH = tmaj ? kTmCh : 8 * NT;
  const bool local_rows = npairs <= kLocalPairs;

  CallMaps cm;
  int rc;
  const bool tok = T <= kTokMax;
  // token mode reads the T token rows (rows T..7 of the box read as zero)
  const uint32_t box_rows = tmaj ? kTmCh : 8 * NT;
  if ((rc = make_map_3d(&cm.tm_x8, P.x8, d.D, tok ? T : g.P_max, 2, d.D, box_rows, g.P_max))) return rc;
  if ((rc = make_map_3d(&cm.tm_act8, P.act8, g.I_act, g.act_rows, 2, g.I_act, box_rows, g.act_rows)))
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
  // many pairs: the segmented plan (plan_seg_kernel + token CTAs placing their pairs and rows)
  const bool seg = !tok && !route && npairs > kFastPlanPairs && d.E <= kSegMaxE;
  pa.local_rows = local_rows && !seg ? 1 : 0;
  pa.tok_mode = tok ? 1 : 0;
  pa.n_ctab = tok ? g.C_max * 8 : 0;
  pa.po = PermuteOut{nullptr, nullptr, nullptr};
  pa.status = dev_status;
  pa.ucount = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(workspace) + g.off_ucount);
  pa.n_ucount = g.U_gu + g.U_dn;
  pa.seg_lrank = pa.seg_off = pa.seg_base = nullptr;
  int32_t* seg_ws = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(workspace) + g.off_seg);
  const int nseg = static_cast<int>((npairs + kSegPairs - 1) / kSegPairs);
  if (seg) {
    pa.seg_lrank = seg_ws;
    pa.seg_off = seg_ws + npairs;
    pa.seg_base = seg_ws + npairs + static_cast<int64_t>(nseg) * kSegMaxE;
  }
  if (route) {
    RouteArgs ra;
    const bool hash = route->tid2eid != nullptr;
    ra.x = static_cast<const __nv_bfloat16*>(hidden);
    ra.norm_w = static_cast<const __nv_bfloat16*>(route->norm_w);
    ra.eps = route->eps;
    ra.x_out = static_cast<__nv_bfloat16*>(route->x_out);
    ra.gate = hash ? nullptr : static_cast<const __nv_bfloat16*>(route->gate);
    ra.bias = hash ? nullptr : static_cast<const __nv_bfloat16*>(route->bias);
    ra.ids = route->ids;
    ra.tid2eid = route->tid2eid;
    ra.V = route->vocab;
    ra.T = static_cast<int>(T);
    ra.D = d.D;
    ra.E = static_cast<int>(route->num_experts);
    ra.K = static_cast<int>(top_k);
    // hash weights: torch.full(..., 1.0 / k) with a float32 default dtype
    ra.scaling = hash ? static_cast<float>(1.0 / static_cast<double>(top_k)) : route->scaling;
    ra.status = dev_status;
    ra.dup_mode = dup_mode;
    ra.offset = static_cast<int>(route->expert_offset);
    ra.held = d.E;
    ra.idx_out = route->idx_out;
    ra.w_out = route->w_out;
    ra.ucount = pa.ucount;
    ra.n_ucount = pa.n_ucount;
    ra.n_ctab = g.C_max * 8;
    ra.P_max = g.P_max;
    ra.ep_buf = nullptr;
    ra.h_chain = nullptr;
    ra.ep_world = 0;
    ra.chain_shared = 0;
    ra.wait_ns = 0;
    if (route->ep && route->chain_prev) {
      ra.ep_buf = static_cast<uint8_t*>(route->ep->recv[route->ep->rank]);
      ra.h_chain = static_cast<__nv_bfloat16*>(route->h_out);  // the rows themselves
      ra.ep_world = route->ep->world;
      ra.chain_shared = route->chain_prev_shared;
      ra.wait_ns = ep_wait_limit(route->ep);
    }
    if ((rc = launch_route(ra, P, d, st))) return rc;
  } else if (seg && (rc = launch_seg(pa, P, nseg, seg_ws, st))) {
    return rc;
  } else if ((rc = launch_plan(pa, P, 1 + static_cast<int>(T), st))) {
    return rc;
  }
  if (!route && !local_rows && !tok && !seg) {
    HS_CUDA_CHECK(launch_pdl(gather_kernel, dim3(static_cast<unsigned>(npairs)), dim3(256), 0, st, P,
                             static_cast<int>(T), g.P_max, d.D));
    if ((rc = check_launch())) return rc;
  }

  UnitArgs a;
  a.ncl = 0;
  a.w_sh = tok && use_shared ? 1 : 2;  // token mode prefetches the shared expert into L2
  a.ext_combine = T > kInlineCombineMax ? 1 : 0;
  a.ep_rank = 0;
  a.ep_world = 0;
  for (int q = 0; q < HS_EP_MAX_RANKS; ++q) a.ep_recv[q] = nullptr;
  if (route && route->ep) {
    a.ep_rank = route->ep->rank;
    a.ep_world = route->ep->world;
    for (int q = 0; q < a.ep_world; ++q) a.ep_recv[q] = static_cast<uint8_t*>(route->ep->recv[q]);
  }
  a.P = P;
  a.T = static_cast<int>(T);
  a.K = static_cast<int>(top_k);
  a.CH = CH;
  a.P_max = g.P_max;
  a.n_sh_chunks = use_shared ? static_cast<int>((T + CH - 1) / CH) : 0;
  a.use_shared = use_shared;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.out_f32 = out_f32;
  a.shared_f32 = partials && use_shared ? shared_f32 : nullptr;
  a.partials = partials;
  // (expert parallelism: the residual add happens in the exchange's combine)
  a.resid = layer && !partials && a.ep_world == 0 ? static_cast<const __nv_bfloat16*>(hidden) : nullptr;
  a.resid_out = layer && !partials && a.ep_world == 0 ? static_cast<__nv_bfloat16*>(route->h_out) : nullptr;
  a.status = dev_status;
  a.G = g.G;
  a.aligned = g.aligned;
  a.part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + g.off_part);
  a.act_rows = g.act_rows;
  a.ucount = pa.ucount;
  if (tok) {
    if ((rc = launch_sk<false, 1, true>(d, cm, a, st))) return rc;
    a.ucount = pa.ucount + g.U_gu;
    if (a.ep_world == 0) return launch_tok_down(d, cm, a, st);
    int gdown = 0;
    if ((rc = launch_tok_down(d, cm, a, st, &gdown))) return rc;
    (void)gdown;
    if (route->defer) return HS_OK;  // the next chained call (or hs_ep_combine_pending) completes it
    return launch_ep_combine(a.ep_recv[a.ep_rank], a.ep_world, T, d.D, use_shared,
                             static_cast<const __nv_bfloat16*>(hidden), static_cast<__nv_bfloat16*>(route->h_out),
                             dev_status, ep_wait_limit(route->ep), st);
  }
  if (tmaj) {
    TmMaps tmm;
    const uint64_t E = d.E, D = d.D, I = d.I, Ish = d.I_sh;
    if ((rc = make_map(&tmm.w2, d.w2, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 128, E * D * (I / 128), 64, 128, 128)))
      return rc;
    tmm.sw2 = tmm.w2;
    if (use_shared &&
        (rc = make_map(&tmm.sw2, d.sh_w2, CU_TENSOR_MAP_DATA_TYPE_UINT8, 128, D * (Ish / 128), 128, 128, 128)))
      return rc;
    a.ext_combine = 1;
    if ((rc = launch_tm<false>(d, cm, tmm, a, st))) return rc;
    if ((rc = launch_tm<true>(d, cm, tmm, a, st))) return rc;
  } else {
    if ((rc = launch_nt<false>(NT, d, cm, a, st))) return rc;
    a.ucount = pa.ucount + g.U_gu;
    if ((rc = launch_nt<true>(NT, d, cm, a, st))) return rc;
  }
  if (!a.ext_combine) return HS_OK;
  const int64_t nv = T * (d.D / 8);
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>((nv + 255) / 256, 8 * sm_count()));
  HS_CUDA_CHECK(launch_pdl(combine_rows_kernel, dim3(grid), dim3(256), 0, st, a, d.D));
  return check_launch();
}

extern "C" int hs_moe_ffn_fp4(const void* desc, const void* hidden, const int64_t* topk_idx, const float* topk_w,
                              int64_t T, int64_t top_k, int use_shared, int dup_mode, void* out, float* out_f32,
                              void* workspace, size_t workspace_bytes, int32_t* dev_status, void* stream) {
  return moe_ffn_impl(desc, hidden, topk_idx, topk_w, T, top_k, use_shared, dup_mode, out, out_f32, nullptr, 0,
                      workspace, workspace_bytes, dev_status, stream);
}

extern "C" int hs_moe_route_ffn_fp4(const void* desc, const void* hidden, const void* gate, const void* bias,
                                    int64_t num_experts, int64_t expert_offset, int64_t T, int64_t top_k,
                                    float routed_scaling, int use_shared, int dup_mode, int64_t* topk_idx,
                                    float* topk_w, void* out, float* out_f32, void* workspace,
                                    size_t workspace_bytes, int32_t* dev_status, void* stream) {
  const RouteIn r{gate, bias, num_experts, expert_offset, routed_scaling, topk_idx, topk_w};
  return moe_ffn_impl(desc, hidden, nullptr, nullptr, T, top_k, use_shared, dup_mode, out, out_f32, nullptr, 0,
                      workspace, workspace_bytes, dev_status, stream, &r);
}

extern "C" int hs_moe_route_ffn_fp4_partials(const void* desc, const void* hidden, const void* gate,
                                             const void* bias, int64_t num_experts, int64_t expert_offset, int64_t T,
                                             int64_t top_k, float routed_scaling, int use_shared, int dup_mode,
                                             int64_t* topk_idx, float* topk_w, float* routed_f32,
                                             float* shared_f32, void* workspace, size_t workspace_bytes,
                                             int32_t* dev_status, void* stream) {
  const RouteIn r{gate, bias, num_experts, expert_offset, routed_scaling, topk_idx, topk_w};
  return moe_ffn_impl(desc, hidden, nullptr, nullptr, T, top_k, use_shared, dup_mode, nullptr, routed_f32,
                      shared_f32, 1, workspace, workspace_bytes, dev_status, stream, &r);
}

extern "C" int hs_moe_layer_fp4(const void* desc, const void* h, const void* norm_w, float eps, const void* gate,
                                const void* bias, const int64_t* input_ids, const int64_t* tid2eid, int64_t vocab,
                                int64_t num_experts, int64_t expert_offset, int64_t T, int64_t top_k,
                                float routed_scaling, int use_shared, int dup_mode, int64_t* topk_idx, float* topk_w,
                                void* x_out, void* h_out, void* workspace, size_t workspace_bytes,
                                int32_t* dev_status, void* stream) {
  if (!norm_w || !h_out) return HS_ERR_BAD_ARGUMENT;
  RouteIn r{gate, bias, num_experts, expert_offset, routed_scaling, topk_idx, topk_w};
  r.norm_w = norm_w;
  r.eps = eps;
  r.x_out = x_out;
  r.h_out = h_out;
  r.ids = input_ids;
  r.tid2eid = tid2eid;
  r.vocab = vocab;
  return moe_ffn_impl(desc, h, nullptr, nullptr, T, top_k, use_shared, dup_mode, nullptr, nullptr, nullptr, 0,
                      workspace, workspace_bytes, dev_status, stream, &r);
}

extern "C" int hs_moe_layer_fp4_partials(const void* desc, const void* h, const void* norm_w, float eps,
                                         const void* gate, const void* bias, const int64_t* input_ids,
                                         const int64_t* tid2eid, int64_t vocab, int64_t num_experts,
                                         int64_t expert_offset, int64_t T, int64_t top_k, float routed_scaling,
                                         int use_shared, int dup_mode, int64_t* topk_idx, float* topk_w,
                                         void* x_out, float* routed_f32, float* shared_f32, void* workspace,
                                         size_t workspace_bytes, int32_t* dev_status, void* stream) {
  if (!norm_w) return HS_ERR_BAD_ARGUMENT;
  RouteIn r{gate, bias, num_experts, expert_offset, routed_scaling, topk_idx, topk_w};
  r.norm_w = norm_w;
  r.eps = eps;
  r.x_out = x_out;
  r.ids = input_ids;
  r.tid2eid = tid2eid;
  r.vocab = vocab;
  return moe_ffn_impl(desc, h, nullptr, nullptr, T, top_k, use_shared, dup_mode, nullptr, routed_f32, shared_f32, 1,
                      workspace, workspace_bytes, dev_status, stream, &r);
}

extern "C" int hs_moe_layer_fp4_ep(const void* desc, const void* h, const void* norm_w, float eps, const void* gate,
                                   const void* bias, const int64_t* input_ids, const int64_t* tid2eid, int64_t vocab,
                                   int64_t num_experts, int64_t expert_offset, int64_t T, int64_t top_k,
                                   float routed_scaling, int use_shared, int dup_mode, int64_t* topk_idx,
                                   float* topk_w, void* x_out, const hs_ep_peers* peers, void* h_out,
                                   void* workspace, size_t workspace_bytes, int32_t* dev_status, void* stream) {
  if (!norm_w || !h_out || !peers) return HS_ERR_BAD_ARGUMENT;
  Desc dd;
  if (!desc) return HS_ERR_BAD_ARGUMENT;
  memcpy(&dd, desc, sizeof(dd));
  if (T > epx::kRows || dd.D > 8192) return HS_ERR_UNSUPPORTED;
  RouteIn r{gate, bias, num_experts, expert_offset, routed_scaling, topk_idx, topk_w};
  r.norm_w = norm_w;
  r.eps = eps;
  r.x_out = x_out;
  r.h_out = h_out;
  r.ids = input_ids;
  r.tid2eid = tid2eid;
  r.vocab = vocab;
  r.ep = peers;
  return moe_ffn_impl(desc, h, nullptr, nullptr, T, top_k, use_shared, dup_mode, nullptr, nullptr, nullptr, 0,
                      workspace, workspace_bytes, dev_status, stream, &r);
}

extern "C" int hs_moe_layer_fp4_ep_chained(const void* desc, void* h, const void* norm_w, float eps, const void* gate,
                                           const void* bias, const int64_t* input_ids, const int64_t* tid2eid,
                                           int64_t vocab, int64_t num_experts, int64_t expert_offset, int64_t T,
                                           int64_t top_k, float routed_scaling, int use_shared, int dup_mode,
                                           int64_t* topk_idx, float* topk_w, void* x_out, const hs_ep_peers* peers,
                                           int prev_pending, int prev_use_shared, void* workspace,
                                           size_t workspace_bytes, int32_t* dev_status, void* stream) {
  if (!norm_w || !h || !peers) return HS_ERR_BAD_ARGUMENT;
  Desc dd;
  if (!desc) return HS_ERR_BAD_ARGUMENT;
  memcpy(&dd, desc, sizeof(dd));
  if (T > epx::kRows || dd.D > 8192) return HS_ERR_UNSUPPORTED;
  RouteIn r{gate, bias, num_experts, expert_offset, routed_scaling, topk_idx, topk_w};
  r.norm_w = norm_w;
  r.eps = eps;
  r.x_out = x_out;
  r.h_out = h;
  r.ids = input_ids;
  r.tid2eid = tid2eid;
  r.vocab = vocab;
  r.ep = peers;
  r.chain_prev = prev_pending ? 1 : 0;
  r.chain_prev_shared = prev_use_shared ? 1 : 0;
  r.defer = true;
  return moe_ffn_impl(desc, h, nullptr, nullptr, T, top_k, use_shared, dup_mode, nullptr, nullptr, nullptr, 0,
                      workspace, workspace_bytes, dev_status, stream, &r);
}

extern "C" int hs_ep_combine_pending(const hs_ep_peers* peers, void* h, int64_t T, int64_t D, int use_shared,
                                     int32_t* dev_status, void* stream) {
  if (!peers || !h || peers->world < 1 || peers->world > HS_EP_MAX_RANKS || peers->rank < 0 ||
      peers->rank >= peers->world || !peers->recv[peers->rank])
    return HS_ERR_BAD_ARGUMENT;
  if (T < 0 || T > epx::kRows || D < 8 || D > 8192 || D % 8) return HS_ERR_BAD_SHAPE;
  if (T == 0) return HS_OK;
  return launch_ep_combine(static_cast<uint8_t*>(peers->recv[peers->rank]), peers->world, T, static_cast<int>(D),
                           use_shared, static_cast<const __nv_bfloat16*>(h), static_cast<__nv_bfloat16*>(h),
                           dev_status, ep_wait_limit(peers), static_cast<cudaStream_t>(stream));
}

extern "C" size_t hs_ep_buffer_bytes(int64_t world, int64_t D) {
  if (world < 1 || world > HS_EP_MAX_RANKS || D < 8 || D > 8192) return 0;
  return epx::bytes(world, D);
}

extern "C" int hs_ep_buffer_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return HS_ERR_BAD_ARGUMENT;
  *ptr = nullptr;
  HS_CUDA_CHECK(cudaMalloc(ptr, bytes));
  HS_CUDA_CHECK(cudaMemset(*ptr, 0, static_cast<size_t>(epx::kHdr)));              // counters
  if (bytes > static_cast<size_t>(epx::kHdr))                                        // every entry empty
    HS_CUDA_CHECK(cudaMemset(static_cast<uint8_t*>(*ptr) + epx::kHdr, 0xff, bytes - epx::kHdr));
  HS_CUDA_CHECK(cudaDeviceSynchronize());
  return HS_OK;
}

extern "C" int hs_ep_buffer_free(void* ptr) {
  if (!ptr) return HS_OK;
  HS_CUDA_CHECK(cudaFree(ptr));
  return HS_OK;
}

extern "C" int hs_ipc_get_handle(const void* ptr, void* handle, size_t handle_bytes) {
  if (!ptr || !handle || handle_bytes < sizeof(cudaIpcMemHandle_t)) return HS_ERR_BAD_ARGUMENT;
  cudaIpcMemHandle_t hnd;
  HS_CUDA_CHECK(cudaIpcGetMemHandle(&hnd, const_cast<void*>(ptr)));
  memcpy(handle, &hnd, sizeof(hnd));
  return HS_OK;
}

extern "C" int hs_ipc_open_handle(const void* handle, void** ptr) {
  if (!handle || !ptr) return HS_ERR_BAD_ARGUMENT;
  cudaIpcMemHandle_t hnd;
  memcpy(&hnd, handle, sizeof(hnd));
  *ptr = nullptr;
  HS_CUDA_CHECK(cudaIpcOpenMemHandle(ptr, hnd, cudaIpcMemLazyEnablePeerAccess));
  return HS_OK;
}

extern "C" int hs_ipc_close_handle(void* ptr) {
  if (!ptr) return HS_OK;
  HS_CUDA_CHECK(cudaIpcCloseMemHandle(ptr));
  return HS_OK;
}

extern "C" int hs_moe_ffn_fp4_partials(const void* desc, const void* hidden, const int64_t* topk_idx,
                                       const float* topk_w, int64_t T, int64_t top_k, int use_shared, int dup_mode,
                                       float* routed_f32, float* shared_f32, void* workspace, size_t workspace_bytes,
                                       int32_t* dev_status, void* stream) {
  return moe_ffn_impl(desc, hidden, topk_idx, topk_w, T, top_k, use_shared, dup_mode, nullptr, routed_f32,
                      shared_f32, 1, workspace, workspace_bytes, dev_status, stream);
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
  pa.tok_mode = 0;
  pa.n_ctab = 0;
  pa.po = PermuteOut{pos_to_expert, expert_count, num_pos};
  pa.status = dev_status;
  pa.ucount = nullptr;
  pa.n_ucount = 0;
  pa.seg_lrank = pa.seg_off = pa.seg_base = nullptr;
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
// The cache lives as long as the process: a cudaDeviceReset (a new primary
// context, the module loaded again) makes the kept address stale, which the
// header tells callers.
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

// The tracing build's stamp array ([slot][kernel][CTA][event] u64, which = 0)
// and layer-call counter (u32, which = 1), or NULL in the normal build.
extern "C" void* hs_trace_buffer(int which) {
#ifdef HS_TRACE
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, which == 0 ? static_cast<const void*>(&hs::trace::g_stamp)
                                          : static_cast<const void*>(&hs::trace::g_calls)) != cudaSuccess)
    return nullptr;
  return p;
#else
  (void)which;
  return nullptr;
#endif
}
