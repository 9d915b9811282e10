// Routed FP4 expert FFN + fused FP8 shared expert for the decode / verify
// regime (T <= a few dozen tokens), sm_100a.
//
// Reference being replaced: FusedMoEFFN._forward_legacy
// (home_seek/fused_moe.py:458-551), which dequantises every touched expert to
// BF16 (fused_moe.py:672-735), concatenates the weights (fused_moe.py:515-517)
// and runs three cuBLAS GEMMs; SharedExpertFFN.forward + fused_expert_ffn_pt
// (fused_moe.py:383-392, 573-598) for the shared expert; and the bf16 add of
// the two at inference_engine/engine.py:1530-1536.
//
// Design (B200-first, HBM-bound):
//   plan     one CTA builds the expert-major pair list (deterministic counting
//            sort), T more CTAs convert each token's hidden row to f16 with a
//            per-token power-of-two prescale (exact for bf16 inputs).
//   gateup   one CTA per (chunk of <= 24 pairs of one expert, 64 rows of I).
//            A producer warp streams the packed e2m1 rows of w1 and w3 with TMA
//            (128B-swizzled boxes) plus the token rows with bulk copies through
//            a 4-stage mbarrier ring; 4 consumer warps convert e2m1 -> f16 in
//            registers (cvt.rn.f16x2.e2m1x2, exact) and run m16n8k16 MMAs with
//            f32 accumulation, applying each 32-column E8M0 scale to the group's
//            partial sum (an exact power-of-two multiply). The epilogue rounds
//            gate/up to bf16, applies SwiGLU with clamp 10 in f32, rounds to
//            bf16, multiplies by the bf16 routing weight and stores the result.
//   down     one CTA per (chunk, 64 rows of D) streams w2 the same way and
//            writes an f32 partial row per (token, expert) pair.
//   finalize sums each token's pairs in ascending expert order (deterministic),
//            rounds once to bf16, adds the bf16 shared-expert output.
// The shared expert is one more chunk list with e4m3 weights and 128x128
// block scales (cvt.rn.f16x2.e4m3x2, exact).
#include <algorithm>
#include <atomic>
#include <mutex>

#include "hs_common.cuh"

namespace hs {
namespace moe {

constexpr int kRows = 64;          // weight rows per unit
constexpr int kConsumerWarps = 4;  // 16 rows each
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kStages = 4;
constexpr int kBoxBytes = kRows * 128;     // one TMA box: 64 rows x 128 B
constexpr int kStageA = 2 * kBoxBytes;     // two boxes per stage
constexpr int kMaxNT = 3;                  // n-tiles of 8 pairs per chunk
constexpr uint32_t kDescMagic = 0x48534d31u;  // "HSM1"
constexpr int kPlanThreads = 512;

struct __align__(64) Desc {
  CUtensorMap tm_w13;  // [E*2*I rows][D/2 B], box 128 B x 64, swizzle 128B
  CUtensorMap tm_s13;  // [E*2*I rows][D/32 B], box D/32 x 64
  CUtensorMap tm_w2;   // [E*D rows][I/2 B],  box 128 B x 64, swizzle 128B
  CUtensorMap tm_s2;   // [E*D rows][I/32 B], box I/32 x 64
  CUtensorMap tm_sw13; // [2*I_sh rows][D B] e4m3, box 128 B x 64, swizzle 128B
  CUtensorMap tm_sw2;  // [D rows][I_sh B] e4m3, box 128 B x 64, swizzle 128B
  const uint8_t* sh_s13;
  const uint8_t* sh_s2;
  int32_t E, D, I, I_sh;
  int32_t has_shared;
  uint32_t magic;
};
static_assert(sizeof(Desc) <= HS_MOE_DESC_BYTES, "descriptor blob too small");

// Device views into the caller's workspace.
struct Plan {
  int32_t* hdr;           // [0] routed chunks, [1] slots, [2] routed pairs
  int32_t* chunk_expert;  // [C_max]
  int32_t* chunk_pair0;   // [C_max] first pair index (global)
  int32_t* chunk_np;      // [C_max]
  int32_t* pair_token;    // [P_max]
  float* pair_wb;         // [P_max] bf16-rounded routing weight
  int32_t* pair_q;        // [P_max] power-of-two prescale of the activation
  int32_t* tok_e;         // [T] power-of-two prescale of the hidden row
  int32_t* tok_pos;       // [T][K] ascending routed pair positions, -1 padded
  __half* hx;             // [T][D]
  __half* act;            // [P_max][I_act]
  float* out_part;        // [P_max][D]
};

struct Geometry {
  int64_t T, K, D, I, I_sh, I_act, P_max, C_max;
  size_t off_hdr, off_chunk, off_pair, off_tok, off_tokpos, off_hx, off_act, off_out, total;
};

static size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

static int64_t chunk_rows(int64_t T) {
  int64_t nt = (T + 7) / 8;
  if (nt > kMaxNT) nt = kMaxNT;
  if (nt < 1) nt = 1;
  return nt;
}

static Geometry geometry(int64_t T, int64_t K, int64_t D, int64_t I, int64_t I_sh) {
  Geometry g{};
  g.T = T;
  g.K = K;
  g.D = D;
  g.I = I;
  g.I_sh = I_sh;
  g.I_act = std::max(I, I_sh);
  const int64_t CH = 8 * chunk_rows(T);
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
  g.off_tok = o;
  o = align_up(o + T * sizeof(int32_t), 256);
  g.off_tokpos = o;
  o = align_up(o + T * K * sizeof(int32_t), 256);
  g.off_hx = o;
  o = align_up(o + T * D * sizeof(__half), 256);
  g.off_act = o;
  o = align_up(o + g.P_max * g.I_act * sizeof(__half), 256);
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
  p.tok_e = reinterpret_cast<int32_t*>(b + g.off_tok);
  p.tok_pos = reinterpret_cast<int32_t*>(b + g.off_tokpos);
  p.hx = reinterpret_cast<__half*>(b + g.off_hx);
  p.act = reinterpret_cast<__half*>(b + g.off_act);
  p.out_part = reinterpret_cast<float*>(b + g.off_out);
  return p;
}

// ---------------------------------------------------------------------------
// plan kernel
// ---------------------------------------------------------------------------
// Power-of-two prescale for an activation rounded from a*wb with |a| <= 100:
// |a*wb| * 2^q < 2^15, so the f16 copy never overflows and stays exact.
__device__ __forceinline__ int act_prescale(float wb) {
  const float m = fabsf(wb);
  if (!(m > 0.f) || !isfinite(m)) return 0;
  int ex;
  frexpf(m, &ex);
  int q = 8 - ex;
  return max(-100, min(100, q));
}

// Internal duplicate mode for the standalone permute: every valid (t, j) gets
// its own position.
constexpr int kDupKeepAll = 2;

// Optional outputs of the standalone permute (hs_moe_permute).
struct PermuteOut {
  int32_t* pos_to_expert;  // [T*K] or nullptr
  int32_t* expert_count;   // [E] or nullptr
  int32_t* num_pos;        // [1] or nullptr
};

// Block 0 builds the routing plan; blocks 1..T (when hidden != nullptr)
// convert one token row each. pos_offset is T for the MoE call (shared-expert
// pairs first) and 0 for the standalone permute; sort_tok sorts each token's
// positions ascending (the MoE finalize order) instead of keeping k order.
__global__ void __launch_bounds__(kPlanThreads) plan_kernel(const int64_t* __restrict__ topk_idx,
                                                            const float* __restrict__ topk_w, int T, int K, int E,
                                                            int CH, int dup_mode, const __nv_bfloat16* __restrict__ hidden,
                                                            int D, Plan P, int pos_offset, int sort_tok,
                                                            PermuteOut po, int32_t* status) {
  const int tid = threadIdx.x;
  if (blockIdx.x > 0) {
    // ---- token row conversion: hx[t] = f16(h[t] * 2^e), e from max|h[t]| ----
    const int t = blockIdx.x - 1;
    const __nv_bfloat16* h = hidden + static_cast<int64_t>(t) * D;
    float mx = 0.f;
    for (int k = tid; k < D; k += blockDim.x) mx = fmaxf(mx, fabsf(__bfloat162float(h[k])));
    __shared__ float red[kPlanThreads / 32];
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((tid & 31) == 0) red[tid >> 5] = mx;
    __syncthreads();
    if (tid < 32) {
      float v = tid < (int)(blockDim.x / 32) ? red[tid] : 0.f;
      for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
      if (tid == 0) red[0] = v;
    }
    __syncthreads();
    const float m = red[0];
    int e = 0;
    if (m > 0.f && isfinite(m)) {
      int ex;
      frexpf(m, &ex);
      e = max(-100, min(100, 15 - ex));
    }
    const float sc = exp2i(e);
    __half* dst = P.hx + static_cast<int64_t>(t) * D;
    for (int k = tid; k < D; k += blockDim.x) dst[k] = __float2half_rn(__bfloat162float(h[k]) * sc);
    if (tid == 0) P.tok_e[t] = e;
    return;
  }

  // ---- routing plan (block 0) ----
  extern __shared__ int32_t sm[];
  int32_t* hist = sm;                // [E]
  int32_t* base = hist + E;          // [E+1]
  int32_t* cursor = base + E + 1;    // [E]
  int32_t* cbase = cursor + E;       // [E+1]
  int32_t* wcnt = cbase + E + 1;     // [nwarps][E]
  const int nwarps = blockDim.x / 32;
  const int warp = tid >> 5, lane = tid & 31;
  const int npairs = T * K;

  for (int e = tid; e < E; e += blockDim.x) {
    hist[e] = 0;
    cursor[e] = 0;
  }
  __syncthreads();

  // validity of pair l = t*K + j: expert in range and (dedupe) the occurrence
  // that carries the token's weight for that expert.
  auto pair_expert = [&](int l, float* wsum) -> int {
    const int t = l / K, j = l - t * K;
    const int64_t e64 = topk_idx[l];
    if (e64 < 0) return -1;
    if (e64 >= E) {
      report(status, HS_DEV_BAD_EXPERT);
      return -1;
    }
    const int e = static_cast<int>(e64);
    const int64_t* row = topk_idx + static_cast<int64_t>(t) * K;
    const float* wrow = topk_w ? topk_w + static_cast<int64_t>(t) * K : nullptr;
    if (dup_mode == kDupKeepAll) {
      if (wsum) *wsum = wrow ? wrow[j] : 1.f;
    } else if (dup_mode == HS_DUP_SUM) {
      for (int jj = 0; jj < j; ++jj)
        if (row[jj] == e64) return -1;
      float s = 0.f;
      for (int jj = j; jj < K; ++jj)
        if (row[jj] == e64) s += wrow ? wrow[jj] : 1.f;
      if (wsum) *wsum = s;
    } else {
      for (int jj = j + 1; jj < K; ++jj)
        if (row[jj] == e64) return -1;
      if (wsum) *wsum = wrow ? wrow[j] : 1.f;
    }
    return e;
  };

  // pass 1: histogram
  for (int l = tid; l < npairs; l += blockDim.x) {
    const int e = pair_expert(l, nullptr);
    if (e >= 0) atomicAdd(&hist[e], 1);
  }
  __syncthreads();
  // exclusive scans (pairs and chunks) by warp 0
  if (warp == 0) {
    int run = 0, crun = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int e = e0 + lane;
      const int h = e < E ? hist[e] : 0;
      const int c = (h + CH - 1) / CH;
      int x = h, y = c;
      for (int o = 1; o < 32; o <<= 1) {
        const int xv = __shfl_up_sync(0xffffffffu, x, o);
        const int yv = __shfl_up_sync(0xffffffffu, y, o);
        if (lane >= o) {
          x += xv;
          y += yv;
        }
      }
      if (e < E) {
        base[e] = run + x - h;
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
  // chunk list and header
  for (int e = tid; e < E; e += blockDim.x) {
    const int h = hist[e];
    int cb = cbase[e];
    for (int c = 0; c * CH < h; ++c, ++cb) {
      P.chunk_expert[cb] = e;
      P.chunk_pair0[cb] = pos_offset + base[e] + c * CH;
      P.chunk_np[cb] = min(CH, h - c * CH);
    }
  }
  if (tid == 0) {
    int slots = 0;
    for (int e = 0; e < E; ++e) slots += hist[e] > 0;
    P.hdr[0] = cbase[E];
    P.hdr[1] = slots;
    P.hdr[2] = base[E];
    if (po.num_pos) *po.num_pos = base[E];
  }
  if (po.expert_count)
    for (int e = tid; e < E; e += blockDim.x) po.expert_count[e] = hist[e];
  if (po.pos_to_expert)
    for (int p = base[E] + tid; p < T * K; p += blockDim.x) po.pos_to_expert[p] = -1;
  // shared-expert pairs occupy positions [0, T)
  for (int t = tid; t < pos_offset; t += blockDim.x) {
    P.pair_token[t] = t;
    P.pair_wb[t] = 1.f;
    P.pair_q[t] = 7;
  }
  // pass 2: stable positions, tile by tile (warp-major = pair order)
  const int tile = blockDim.x;
  for (int l0 = 0; l0 < npairs; l0 += tile) {
    const int l = l0 + tid;
    float wsum = 0.f;
    const int e = l < npairs ? pair_expert(l, &wsum) : -1;
    const unsigned m = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(m & ((1u << lane) - 1u));
    for (int x = lane; x < E; x += 32) wcnt[warp * E + x] = 0;
    __syncwarp();
    if (e >= 0 && rank == 0) wcnt[warp * E + e] = __popc(m);
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
        pos = pos_offset + base[e] + wcnt[warp * E + e] + rank;
        const float wb = round_bf16(wsum);
        P.pair_token[pos] = t;
        P.pair_wb[pos] = wb;
        P.pair_q[pos] = act_prescale(wb);
        if (po.pos_to_expert) po.pos_to_expert[pos] = e;
      }
      P.tok_pos[l] = pos;
    }
    __syncthreads();
  }
  __syncthreads();
  // sort each token's positions ascending (= ascending expert id), -1 last
  if (!sort_tok) return;
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


// ---------------------------------------------------------------------------
// streaming units (gate/up and down)
// ---------------------------------------------------------------------------
struct UnitArgs {
  Plan P;
  int T, CH;
  int n_sh_chunks;  // shared-expert chunks (0 when the shared expert is off)
  int32_t* status;
};

struct Smem {
  uint8_t* a;       // kStages x kStageA, 1024-aligned (128B swizzle)
  uint8_t* b;       // kStages x b_stage
  uint8_t* sc;      // per-unit scale rows
  uint64_t* full;   // [kStages] producer -> consumers (TMA transaction bytes)
  uint64_t* empty;  // [kStages] consumers -> producer (one arrive per warp)
  uint64_t* sbar;   // scale rows landed
  int b_stage;
};

constexpr int kPitchGU = 576;     // gate/up B row pitch: 512 B + 64 B pad
constexpr int kPitchDN = 1088;    // down B row pitch: 1024 B + 64 B pad

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~static_cast<uintptr_t>(1023));
}

__device__ __forceinline__ Smem carve(uint8_t* raw, int b_stage, int sc_bytes) {
  Smem s;
  uint8_t* base = align1024(raw);
  s.a = base;
  s.b = base + kStages * kStageA;
  s.sc = s.b + kStages * b_stage;
  uint8_t* bars = s.sc + ((sc_bytes + 127) & ~127);
  s.full = reinterpret_cast<uint64_t*>(bars);
  s.empty = s.full + kStages;
  s.sbar = s.empty + kStages;
  s.b_stage = b_stage;
  return s;
}

__device__ __forceinline__ void init_barriers(const Smem& s) {
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], kConsumerWarps);
    }
    mbar_init(s.sbar, 1);
    fence_mbar_init();
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  __syncthreads();
}

// One group of 32 k columns for 16 weight rows (lo = g, hi = g + 8) and up to
// kMaxNT tiles of 8 pairs. wlo/whi: this thread's 4 (FP4) or 8 (FP8) bytes of
// each row; K order inside the group is permuted identically on both operands
// (thread c owns logical columns 8c..8c+7), so the dot products are exact sums
// of the same terms. Accumulates (scale_lo, scale_hi) * partial into acc.
template <bool kFP8>
__device__ __forceinline__ void group_mma(uint32_t wlo0, uint32_t wlo1, uint32_t whi0, uint32_t whi1, uint32_t bbase,
                                          int pitch, int nt_used, float slo, float shi, float (&acc)[kMaxNT][4]) {
  uint32_t x0, x1, x2, x3, y0, y1, y2, y3;
  if (kFP8) {
    e4m3x4_to_f16x2x2(wlo0, x0, x1);
    e4m3x4_to_f16x2x2(wlo1, x2, x3);
    e4m3x4_to_f16x2x2(whi0, y0, y1);
    e4m3x4_to_f16x2x2(whi1, y2, y3);
  } else {
    e2m1x8_to_f16x2x4(wlo0, x0, x1, x2, x3);
    e2m1x8_to_f16x2x4(whi0, y0, y1, y2, y3);
  }
#pragma unroll
  for (int nt = 0; nt < kMaxNT; ++nt) {
    if (nt < nt_used) {
      const uint4 bv = lds128(bbase + nt * 8 * pitch);
      float t[4] = {0.f, 0.f, 0.f, 0.f};
      mma_f16(t, x0, y0, x1, y1, bv.x, bv.y);
      mma_f16(t, x2, y2, x3, y3, bv.z, bv.w);
      acc[nt][0] = fmaf(t[0], slo, acc[nt][0]);
      acc[nt][1] = fmaf(t[1], slo, acc[nt][1]);
      acc[nt][2] = fmaf(t[2], shi, acc[nt][2]);
      acc[nt][3] = fmaf(t[3], shi, acc[nt][3]);
    }
  }
}

// Producer: lane 0 of the last warp. Streams nk stages; each stage is two TMA
// boxes (x0a/x0b at rows ya/yb) plus np bulk-copied B rows.
struct StageSrc {
  const CUtensorMap* map;
  int ya, yb;          // box rows
  int xa_mul, xb_add;  // box a x = kc*xa_mul, box b x = kc*xa_mul + xb_add
  const __half* bsrc;  // B base for pair row 0 (row r: + r_off(r))
  int brow_elems;      // B elements per row per stage
};

// Consumer wait-or-abort helper: returns false (and reports) on timeout.
__device__ __forceinline__ bool wait_full(const Smem& s, int kc, int32_t* status) {
  if (mbar_wait(&s.full[kc % kStages], (kc / kStages) & 1)) return true;
  report(status, HS_DEV_TIMEOUT);
  return false;
}

__device__ __forceinline__ void release(const Smem& s, int kc) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&s.empty[kc % kStages]);
}

template <bool kFP8>
__device__ __forceinline__ void gateup_unit(const Desc& d, const UnitArgs& a, const Smem& s, int e, int pair0, int np,
                                            int rt) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D = d.D;
  constexpr int KS = kFP8 ? 128 : 256;  // k columns per stage (one 128-byte box)
  const int nk = D / KS;
  constexpr int rowb = KS * 2;          // B bytes per pair row per stage
  const int SB = D / 32;                // FP4 scale bytes per weight row
  const int y1 = kFP8 ? rt * kRows : (2 * e) * d.I + rt * kRows;
  const int y3 = kFP8 ? d.I_sh + rt * kRows : (2 * e + 1) * d.I + rt * kRows;
  const CUtensorMap* tw = kFP8 ? &d.tm_sw13 : &d.tm_w13;

  if (warp == kConsumerWarps) {
    if (lane == 0) {
      if (!kFP8) {
        mbar_arrive_expect_tx(s.sbar, 2 * kRows * SB);
        tma_load_2d(s.sc, &d.tm_s13, s.sbar, 0, y1);
        tma_load_2d(s.sc + kRows * SB, &d.tm_s13, s.sbar, 0, y3);
      }
      for (int kc = 0; kc < nk; ++kc) {
        const int st = kc % kStages;
        if (kc >= kStages && !mbar_wait(&s.empty[st], ((kc / kStages) - 1) & 1)) {
          report(a.status, HS_DEV_TIMEOUT);
          break;
        }
        uint8_t* A = s.a + st * kStageA;
        uint8_t* B = s.b + st * s.b_stage;
        mbar_arrive_expect_tx(&s.full[st], kStageA + np * rowb);
        tma_load_2d(A, tw, &s.full[st], kc * 128, y1);
        tma_load_2d(A + kBoxBytes, tw, &s.full[st], kc * 128, y3);
        for (int r = 0; r < np; ++r) {
          const int t = a.P.pair_token[pair0 + r];
          bulk_load(B + r * kPitchGU, a.P.hx + static_cast<int64_t>(t) * D + kc * KS, rowb, &s.full[st]);
        }
      }
    }
    return;
  }

  const int g = lane >> 2, c = lane & 3;
  const int rlo = 16 * warp + g, rhi = rlo + 8;
  const int nt_used = (np + 7) >> 3;
  float gate[kMaxNT][4], up[kMaxNT][4];
#pragma unroll
  for (int i = 0; i < kMaxNT; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) gate[i][j] = up[i][j] = 0.f;

  if (!kFP8 && !mbar_wait(s.sbar, 0)) {
    report(a.status, HS_DEV_TIMEOUT);
    return;
  }
  const uint32_t a0 = smem_u32(s.a), b0 = smem_u32(s.b), sc0 = smem_u32(s.sc);
  for (int kc = 0; kc < nk; ++kc) {
    if (!wait_full(s, kc, a.status)) return;
    const int st = kc % kStages;
    const uint32_t A = a0 + st * kStageA;
    const uint32_t B = b0 + st * s.b_stage + g * kPitchGU + c * 16;
    if (!kFP8) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const uint32_t sw = ((q ^ g) << 4) + 4 * c;
        const uint32_t w1l = lds32(A + rlo * 128 + sw), w1h = lds32(A + rhi * 128 + sw);
        const uint32_t w3l = lds32(A + kBoxBytes + rlo * 128 + sw), w3h = lds32(A + kBoxBytes + rhi * 128 + sw);
        const int G = kc * 8 + q;
        const float s1l = e8m0_to_f32_torch(lds8(sc0 + rlo * SB + G));
        const float s1h = e8m0_to_f32_torch(lds8(sc0 + rhi * SB + G));
        const float s3l = e8m0_to_f32_torch(lds8(sc0 + (kRows + rlo) * SB + G));
        const float s3h = e8m0_to_f32_torch(lds8(sc0 + (kRows + rhi) * SB + G));
        group_mma<false>(w1l, 0u, w1h, 0u, B + q * 64, kPitchGU, nt_used, s1l, s1h, gate);
        group_mma<false>(w3l, 0u, w3h, 0u, B + q * 64, kPitchGU, nt_used, s3l, s3h, up);
      }
    } else {
      const int nbc = D / 128;  // scale blocks along k
      const int br = (rt * kRows) / 128;
      const float s1 = e8m0_to_f32_shift(d.sh_s13[(br)*nbc + kc]);
      const float s3 = e8m0_to_f32_shift(d.sh_s13[((d.I_sh / 128) + br) * nbc + kc]);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t ch = 2 * q + (c >> 1);
        const uint32_t sw = ((ch ^ g) << 4) + (c & 1) * 8;
        const uint2 w1l = lds64(A + rlo * 128 + sw), w1h = lds64(A + rhi * 128 + sw);
        const uint2 w3l = lds64(A + kBoxBytes + rlo * 128 + sw), w3h = lds64(A + kBoxBytes + rhi * 128 + sw);
        group_mma<true>(w1l.x, w1l.y, w1h.x, w1h.y, B + q * 64, kPitchGU, nt_used, s1, s1, gate);
        group_mma<true>(w3l.x, w3l.y, w3h.x, w3h.y, B + q * 64, kPitchGU, nt_used, s3, s3, up);
      }
    }
    release(s, kc);
  }

  // epilogue: bf16(gate), bf16(up) -> SwiGLU(clamp 10) -> bf16 -> * bf16(w) -> bf16
  const int Iu = kFP8 ? d.I_sh : d.I;
  (void)Iu;
  const int64_t I_act = max(d.I, d.has_shared ? d.I_sh : 0);
#pragma unroll
  for (int nt = 0; nt < kMaxNT; ++nt) {
    if (nt >= nt_used) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = nt * 8 + 2 * c + (j & 1);
      if (n >= np) continue;
      const int r = (j < 2) ? rlo : rhi;
      const int p = pair0 + n;
      const int t = a.P.pair_token[p];
      const float inv = exp2i(-a.P.tok_e[t]);
      const float gf = round_bf16(gate[nt][j] * inv);
      const float uf = round_bf16(up[nt][j] * inv);
      const float gc = gf > 10.f ? 10.f : gf;
      const float uc = uf > 10.f ? 10.f : (uf < -10.f ? -10.f : uf);
      const float sig = 1.f / (1.f + expf(-gc));
      float av = round_bf16((gc * sig) * uc);
      if (!kFP8) av = round_bf16(av * a.P.pair_wb[p]);
      a.P.act[static_cast<int64_t>(p) * I_act + rt * kRows + r] = __float2half_rn(av * exp2i(a.P.pair_q[p]));
    }
  }
}

template <bool kFP8>
__device__ __forceinline__ void down_unit(const Desc& d, const UnitArgs& a, const Smem& s, int e, int pair0, int np,
                                          int dt) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D = d.D;
  const int Iu = kFP8 ? d.I_sh : d.I;
  constexpr int KS = kFP8 ? 256 : 512;  // k columns per stage (two 128-byte boxes)
  const int nk = Iu / KS;
  constexpr int rowb = KS * 2;
  const int SB = d.I / 32;  // FP4 scale bytes per row
  const int y = kFP8 ? dt * kRows : e * D + dt * kRows;
  const CUtensorMap* tw = kFP8 ? &d.tm_sw2 : &d.tm_w2;
  const int64_t I_act = max(d.I, d.has_shared ? d.I_sh : 0);

  if (warp == kConsumerWarps) {
    if (lane == 0) {
      if (!kFP8) {
        mbar_arrive_expect_tx(s.sbar, kRows * SB);
        tma_load_2d(s.sc, &d.tm_s2, s.sbar, 0, y);
      }
      for (int kc = 0; kc < nk; ++kc) {
        const int st = kc % kStages;
        if (kc >= kStages && !mbar_wait(&s.empty[st], ((kc / kStages) - 1) & 1)) {
          report(a.status, HS_DEV_TIMEOUT);
          break;
        }
        uint8_t* A = s.a + st * kStageA;
        uint8_t* B = s.b + st * s.b_stage;
        mbar_arrive_expect_tx(&s.full[st], kStageA + np * rowb);
        tma_load_2d(A, tw, &s.full[st], kc * 256, y);
        tma_load_2d(A + kBoxBytes, tw, &s.full[st], kc * 256 + 128, y);
        for (int r = 0; r < np; ++r)
          bulk_load(B + r * kPitchDN, a.P.act + static_cast<int64_t>(pair0 + r) * I_act + kc * KS, rowb, &s.full[st]);
      }
    }
    return;
  }

  const int g = lane >> 2, c = lane & 3;
  const int rlo = 16 * warp + g, rhi = rlo + 8;
  const int nt_used = (np + 7) >> 3;
  float acc[kMaxNT][4];
#pragma unroll
  for (int i = 0; i < kMaxNT; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

  if (!kFP8 && !mbar_wait(s.sbar, 0)) {
    report(a.status, HS_DEV_TIMEOUT);
    return;
  }
  const uint32_t a0 = smem_u32(s.a), b0 = smem_u32(s.b), sc0 = smem_u32(s.sc);
  for (int kc = 0; kc < nk; ++kc) {
    if (!wait_full(s, kc, a.status)) return;
    const int st = kc % kStages;
    const uint32_t A = a0 + st * kStageA;
    const uint32_t B = b0 + st * s.b_stage + g * kPitchDN + c * 16;
    if (!kFP8) {
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        const uint32_t box = (q >> 3) * kBoxBytes;
        const uint32_t sw = box + (((q & 7) ^ g) << 4) + 4 * c;
        const uint32_t wl = lds32(A + rlo * 128 + sw), wh = lds32(A + rhi * 128 + sw);
        const int G = kc * 16 + q;
        const float sl = e8m0_to_f32_torch(lds8(sc0 + rlo * SB + G));
        const float sh = e8m0_to_f32_torch(lds8(sc0 + rhi * SB + G));
        group_mma<false>(wl, 0u, wh, 0u, B + q * 64, kPitchDN, nt_used, sl, sh, acc);
      }
    } else {
      const int nbc = d.I_sh / 128;
      const int br = (dt * kRows) / 128;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const uint32_t box = (q >> 2) * kBoxBytes;
        const uint32_t ch = 2 * (q & 3) + (c >> 1);
        const uint32_t sw = box + ((ch ^ g) << 4) + (c & 1) * 8;
        const uint2 wl = lds64(A + rlo * 128 + sw), wh = lds64(A + rhi * 128 + sw);
        const float sv = e8m0_to_f32_shift(d.sh_s2[br * nbc + kc * 2 + (q >> 2)]);
        group_mma<true>(wl.x, wl.y, wh.x, wh.y, B + q * 64, kPitchDN, nt_used, sv, sv, acc);
      }
    }
    release(s, kc);
  }

#pragma unroll
  for (int nt = 0; nt < kMaxNT; ++nt) {
    if (nt >= nt_used) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = nt * 8 + 2 * c + (j & 1);
      if (n >= np) continue;
      const int r = (j < 2) ? rlo : rhi;
      const int p = pair0 + n;
      a.P.out_part[static_cast<int64_t>(p) * D + dt * kRows + r] = acc[nt][j] * exp2i(-a.P.pair_q[p]);
    }
  }
}

__global__ void __launch_bounds__(kThreads) gateup_kernel(const __grid_constant__ Desc d, UnitArgs a) {
  extern __shared__ uint8_t smem_raw[];
  int u = blockIdx.x;
  const int sh_tiles = d.has_shared ? d.I_sh / kRows : 0;
  const int n_sh_units = a.n_sh_chunks * sh_tiles;
  bool shared;
  int e = 0, pair0, np, rt;
  if (u < n_sh_units) {
    shared = true;
    const int c = u / sh_tiles;
    rt = u - c * sh_tiles;
    pair0 = c * a.CH;
    np = min(a.CH, a.T - pair0);
  } else {
    shared = false;
    u -= n_sh_units;
    const int tiles = d.I / kRows;
    const int c = u / tiles;
    rt = u - c * tiles;
    if (c >= a.P.hdr[0]) return;
    e = a.P.chunk_expert[c];
    pair0 = a.P.chunk_pair0[c];
    np = a.P.chunk_np[c];
  }
  const int nt_max = (a.CH + 7) >> 3;
  const Smem s = carve(smem_raw, nt_max * 8 * kPitchGU, 2 * kRows * (d.D / 32));
  init_barriers(s);
  if (threadIdx.x == kConsumerWarps * 32) {
    prefetch_tensormap(shared ? &d.tm_sw13 : &d.tm_w13);
    if (!shared) prefetch_tensormap(&d.tm_s13);
  }
  if (shared)
    gateup_unit<true>(d, a, s, e, pair0, np, rt);
  else
    gateup_unit<false>(d, a, s, e, pair0, np, rt);
}

__global__ void __launch_bounds__(kThreads) down_kernel(const __grid_constant__ Desc d, UnitArgs a) {
  extern __shared__ uint8_t smem_raw[];
  int u = blockIdx.x;
  const int tiles = d.D / kRows;
  const int n_sh_units = a.n_sh_chunks * tiles;
  bool shared;
  int e = 0, pair0, np, dt;
  if (u < n_sh_units) {
    shared = true;
    const int c = u / tiles;
    dt = u - c * tiles;
    pair0 = c * a.CH;
    np = min(a.CH, a.T - pair0);
  } else {
    shared = false;
    u -= n_sh_units;
    const int c = u / tiles;
    dt = u - c * tiles;
    if (c >= a.P.hdr[0]) return;
    e = a.P.chunk_expert[c];
    pair0 = a.P.chunk_pair0[c];
    np = a.P.chunk_np[c];
  }
  const int nt_max = (a.CH + 7) >> 3;
  const Smem s = carve(smem_raw, nt_max * 8 * kPitchDN, kRows * (d.I / 32));
  init_barriers(s);
  if (threadIdx.x == kConsumerWarps * 32) {
    prefetch_tensormap(shared ? &d.tm_sw2 : &d.tm_w2);
    if (!shared) prefetch_tensormap(&d.tm_s2);
  }
  if (shared)
    down_unit<true>(d, a, s, e, pair0, np, dt);
  else
    down_unit<false>(d, a, s, e, pair0, np, dt);
}

// out[t] = bf16( bf16(sum of routed partials, ascending expert) + bf16(shared) )
__global__ void __launch_bounds__(256) finalize_kernel(Plan P, int T, int K, int D, int use_shared,
                                                       __nv_bfloat16* __restrict__ out, float* __restrict__ out_f32) {
  const int t = blockIdx.y;
  const int d = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (d >= D) return;
  float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
  const int32_t* pos = P.tok_pos + static_cast<int64_t>(t) * K;
  for (int j = 0; j < K; ++j) {
    const int p = pos[j];
    if (p < 0) break;
    const float4 v = *reinterpret_cast<const float4*>(P.out_part + static_cast<int64_t>(p) * D + d);
    r.x += v.x;
    r.y += v.y;
    r.z += v.z;
    r.w += v.w;
  }
  if (out_f32) *reinterpret_cast<float4*>(out_f32 + static_cast<int64_t>(t) * D + d) = r;
  float o[4] = {round_bf16(r.x), round_bf16(r.y), round_bf16(r.z), round_bf16(r.w)};
  if (use_shared) {
    const float4 sv = *reinterpret_cast<const float4*>(P.out_part + static_cast<int64_t>(t) * D + d);
    o[0] += round_bf16(sv.x);
    o[1] += round_bf16(sv.y);
    o[2] += round_bf16(sv.z);
    o[3] += round_bf16(sv.w);
  }
  __nv_bfloat16* dst = out + static_cast<int64_t>(t) * D + d;
  dst[0] = __float2bfloat16_rn(o[0]);
  dst[1] = __float2bfloat16_rn(o[1]);
  dst[2] = __float2bfloat16_rn(o[2]);
  dst[3] = __float2bfloat16_rn(o[3]);
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

// 2D uint8 tensor map: rows x inner bytes, row pitch = inner bytes.
static int make_map(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows, uint32_t box_inner,
                    uint32_t box_rows, bool swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return HS_ERR_UNSUPPORTED;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {inner};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_cuda_error(static_cast<int>(r));
    return HS_ERR_CUDA;
  }
  return HS_OK;
}

static bool dim_ok(int64_t v, int64_t mult, int64_t lo, int64_t hi) { return v % mult == 0 && v >= lo && v <= hi; }

// The largest dynamic shared memory any launch can ask for (NT = 3, D = I = 8192).
constexpr int kMaxDynSmem = 200 * 1024;

// Raise the kernels' dynamic shared-memory limit once per device (a host-side
// function attribute; safe to call before or during stream capture).
static int opt_in_smem() {
  static std::atomic<uint64_t> done{0};
  int dev = 0;
  HS_CUDA_CHECK(cudaGetDevice(&dev));
  const uint64_t bit = 1ull << (dev & 63);
  if (done.load() & bit) return HS_OK;
  HS_CUDA_CHECK(cudaFuncSetAttribute(gateup_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmem));
  HS_CUDA_CHECK(cudaFuncSetAttribute(down_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmem));
  HS_CUDA_CHECK(cudaFuncSetAttribute(plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024));
  done.fetch_or(bit);
  return HS_OK;
}

static int smem_gateup(int NT, int D) { return 1024 + kStages * kStageA + kStages * NT * 8 * kPitchGU + 2 * kRows * (D / 32) + 256; }
static int smem_down(int NT, int I) { return 1024 + kStages * kStageA + kStages * NT * 8 * kPitchDN + kRows * (I / 32) + 256; }

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
  if (!aligned16(w->w13) || !aligned16(w->s13) || !aligned16(w->w2) || !aligned16(w->s2)) return HS_ERR_ALIGN;
  Desc d;
  memset(&d, 0, sizeof(d));
  d.E = static_cast<int32_t>(w->E);
  d.D = static_cast<int32_t>(w->D);
  d.I = static_cast<int32_t>(w->I);
  d.has_shared = w->sh_w13 != nullptr;
  int st;
  const uint64_t E = w->E, D = w->D, I = w->I;
  if ((st = make_map(&d.tm_w13, w->w13, D / 2, E * 2 * I, 128, kRows, true))) return st;
  if ((st = make_map(&d.tm_s13, w->s13, D / 32, E * 2 * I, static_cast<uint32_t>(D / 32), kRows, false))) return st;
  if ((st = make_map(&d.tm_w2, w->w2, I / 2, E * D, 128, kRows, true))) return st;
  if ((st = make_map(&d.tm_s2, w->s2, I / 32, E * D, static_cast<uint32_t>(I / 32), kRows, false))) return st;
  if (d.has_shared) {
    if (!dim_ok(w->I_sh, 256, 256, 8192)) return HS_ERR_BAD_SHAPE;
    if (!w->sh_s13 || !w->sh_w2 || !w->sh_s2) return HS_ERR_BAD_ARGUMENT;
    if (!aligned16(w->sh_w13) || !aligned16(w->sh_w2)) return HS_ERR_ALIGN;
    d.I_sh = static_cast<int32_t>(w->I_sh);
    const uint64_t Ish = w->I_sh;
    if ((st = make_map(&d.tm_sw13, w->sh_w13, D, 2 * Ish, 128, kRows, true))) return st;
    if ((st = make_map(&d.tm_sw2, w->sh_w2, Ish, D, 128, kRows, true))) return st;
    d.sh_s13 = static_cast<const uint8_t*>(w->sh_s13);
    d.sh_s2 = static_cast<const uint8_t*>(w->sh_s2);
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

static int launch_plan(const int64_t* topk_idx, const float* topk_w, int64_t T, int64_t K, int E, int CH, int dup,
                       const void* hidden, int D, const Plan& P, int pos_offset, int sort_tok, PermuteOut po,
                       int32_t* dev_status, cudaStream_t st) {
  const int nwarps = kPlanThreads / 32;
  const size_t smem = static_cast<size_t>(4 * E + 2 + nwarps * E) * sizeof(int32_t);
  int rc0 = opt_in_smem();
  if (rc0) return rc0;
  const int grid = 1 + (hidden ? static_cast<int>(T) : 0);
  plan_kernel<<<grid, kPlanThreads, smem, st>>>(topk_idx, topk_w, static_cast<int>(T), static_cast<int>(K), E, CH,
                                                dup, static_cast<const __nv_bfloat16*>(hidden), D, P, pos_offset,
                                                sort_tok, po, dev_status);
  return check_launch();
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
  const int NT = static_cast<int>(chunk_rows(T));
  const int CH = 8 * NT;

  int rc = launch_plan(topk_idx, topk_w, T, top_k, d.E, CH, dup_mode, hidden, d.D, P, static_cast<int>(T), 1,
                       PermuteOut{nullptr, nullptr, nullptr}, dev_status, st);
  if (rc) return rc;

  UnitArgs a;
  a.P = P;
  a.T = static_cast<int>(T);
  a.CH = CH;
  a.n_sh_chunks = use_shared ? static_cast<int>((T + CH - 1) / CH) : 0;
  a.status = dev_status;
  // grids cover the largest possible chunk list; CTAs past the device count exit
  const int64_t gu_units = static_cast<int64_t>(a.n_sh_chunks) * (use_shared ? d.I_sh / kRows : 0) +
                           g.C_max * (d.I / kRows);
  const int64_t dn_units = (static_cast<int64_t>(a.n_sh_chunks) + g.C_max) * (d.D / kRows);
  if (gu_units > 0x7fffffff || dn_units > 0x7fffffff) return HS_ERR_BAD_SHAPE;

  const int sm_gu = smem_gateup(NT, d.D), sm_dn = smem_down(NT, d.I);
  if ((rc = opt_in_smem())) return rc;
  gateup_kernel<<<static_cast<unsigned>(gu_units), kThreads, sm_gu, st>>>(d, a);
  if ((rc = check_launch())) return rc;
  down_kernel<<<static_cast<unsigned>(dn_units), kThreads, sm_dn, st>>>(d, a);
  if ((rc = check_launch())) return rc;
  dim3 fg(static_cast<unsigned>((d.D / 4 + 255) / 256), static_cast<unsigned>(T));
  finalize_kernel<<<fg, 256, 0, st>>>(P, static_cast<int>(T), static_cast<int>(top_k), d.D, use_shared,
                                      static_cast<__nv_bfloat16*>(out), out_f32);
  return check_launch();
}

extern "C" size_t hs_moe_permute_workspace_size(int64_t T, int64_t top_k, int64_t E) {
  (void)E;
  if (T < 0 || top_k < 1) return 0;
  // plan views with D = I = I_sh = 0: header, chunk and pair arrays only
  return geometry(T, top_k, 0, 0, 0).total;
}

extern "C" int hs_moe_permute(const int64_t* topk_idx, int64_t T, int64_t top_k, int64_t E, const void* x, int64_t D,
                              int32_t* token_topk_to_pos, int32_t* pos_to_expert, int32_t* expert_count,
                              int32_t* num_pos, void* x_expanded, void* workspace, size_t workspace_bytes,
                              int32_t* dev_status, void* stream) {
  if (T < 0 || top_k < 1 || top_k > 64 || E < 1 || E > 1024) return HS_ERR_BAD_SHAPE;
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
  int rc = launch_plan(topk_idx, nullptr, T, top_k, static_cast<int>(E), 1 << 30, kDupKeepAll, nullptr, 0, P, 0, 0,
                       PermuteOut{pos_to_expert, expert_count, num_pos}, dev_status, st);
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
