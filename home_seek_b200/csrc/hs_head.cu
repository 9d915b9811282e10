// lm_head GEMV with the greedy decision fused in, sm_100a.
//
// Reference being replaced: the logits GEMV + argmax of every decode step of
// home-seek's MTP loop, i.e. `logits = h_3d @ lm_head.t()` followed by
// `logits[:, -1].argmax(-1)` in the draft (inference_engine/engine.py:
// 2327-2333), the fused verify (engine.py:2482-2497, the greedy comparison
// loop) and the main step (engine.py:2846-2853). The reference writes the
// [T, 129280] bf16 logits and then reads them back for each argmax; here the
// logits stay on chip.
//
// Design: the head W [V][D] bf16 (1.06 GB at the model's shape) is streamed
// once. One CTA per SM, persistent, owns a contiguous range of 128-row vocab
// tiles. Warp 4 streams each tile as k-boxes of 128 rows x 64 columns (16 KB,
// 128B-swizzled TMA, L2 evict-first) together with the matching 16 x 64 box
// of the token rows x (rows >= T read as zero) into an 8-stage ring; warp 5
// issues tcgen05.mma.kind::f16 (A = W box, B = x box, M = 128, N = 16, f32
// accumulators in TMEM, double-buffered per tile); warps 0-3 read a finished
// accumulator (thread = vocab row, column = token), round each logit to bf16
// exactly as the reference's bf16 GEMM output is rounded, and keep for every
// token the best (value, first index) key, NaN maximal as torch.argmax. The
// per-CTA keys are reduced by the last CTA to finish (a ticket), which also
// runs the greedy acceptance: n_accept = leading positions whose argmax equals
// the draft id, next token = argmax of row n_accept.
#include "hs_common.cuh"
#include "hs_tcgen05.cuh"

#include <atomic>
#include <mutex>

namespace hs {
namespace head {

constexpr int kM = 128;                     // vocab rows per tile (UMMA M)
constexpr int kKBox = 64;                   // bf16 columns per k-box (one 128-byte swizzle row)
constexpr int kN = 16;                      // UMMA N: token columns (T <= 16)
constexpr int kStages = 8;
constexpr int kWBytes = kM * kKBox * 2;     // 16 KB
constexpr int kXBytes = kN * kKBox * 2;     // 2 KB
constexpr int kStageBytes = kWBytes + kXBytes;
constexpr int kThreads = 192;               // warps 0-3 epilogue, warp 4 TMA, warp 5 MMA
constexpr int kBarBytes = 256;
constexpr int kSmemBytes = kStages * kStageBytes + kBarBytes + 1024;  // + realignment slack
constexpr uint32_t kTmemCols = 32;          // two accumulators of 16 columns
constexpr int kPartStride = 16;             // u64 keys per CTA in the workspace

struct Bars {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t mma_done;
  uint32_t tmem;
  int32_t issued, consumed;
};
static_assert(sizeof(Bars) <= kBarBytes, "barrier block");

struct Args {
  int T, D, V, ntiles;
  int row0, rows;                  // the head rows streamed: [row0, row0 + rows) of the V (keys carry the global index)
  const int64_t* draft_ids;        // [T - 1] or nullptr
  int64_t* argmax_out;             // [T] or nullptr
  int32_t* n_accept;               // [1] or nullptr
  int64_t* next_token;             // [1] or nullptr
  __nv_bfloat16* logits;           // [T][V] bf16 or nullptr
  unsigned long long* part;        // [gridDim.x][kPartStride] per-CTA best keys
  uint32_t* ticket;                // left at zero by every call
  int32_t* status;
  // vocab split over an expert-parallel group (ep_world 0: one GPU): every
  // rank's exchange buffer as mapped here, this rank, the hidden size that
  // places the key region, the bound of the wait for the peers' keys
  uint8_t* ep_buf[HS_EP_MAX_RANKS];
  int ep_rank, ep_world, ep_D;
  uint64_t wait_ns;
};

// Ordered key of a bf16 logit at vocab index v: larger key = larger value,
// then lower index; every NaN above every number (torch.argmax takes the
// first NaN); -0 equal to +0. 0 is below every real key (no candidate).
__device__ __forceinline__ unsigned long long logit_key(uint32_t b16, int v) {
  uint32_t ord;
  if ((b16 & 0x7fffu) > 0x7f80u) {
    ord = 0x10000u;                       // NaN
  } else {
    if (b16 == 0x8000u) b16 = 0u;         // -0 -> +0
    ord = (b16 & 0x8000u) ? (0x7fffu - (b16 & 0x7fffu)) : (0x8000u + b16);
  }
  return (static_cast<unsigned long long>(ord) << 32) | static_cast<uint32_t>(~static_cast<uint32_t>(v));
}
__device__ __forceinline__ int key_index(unsigned long long k) {
  return static_cast<int>(~static_cast<uint32_t>(k & 0xffffffffull));
}

// Warp max of a 64-bit key (all lanes get it).
__device__ __forceinline__ unsigned long long warp_max_key(unsigned long long k) {
  const uint32_t hi = __reduce_max_sync(0xffffffffu, static_cast<uint32_t>(k >> 32));
  const uint32_t lo = __reduce_max_sync(0xffffffffu, static_cast<uint32_t>(k >> 32) == hi
                                                         ? static_cast<uint32_t>(k & 0xffffffffull) : 0u);
  return (static_cast<unsigned long long>(hi) << 32) | lo;
}

// Instruction descriptor of tcgen05.mma.kind::f16: bf16 A and B, both K-major,
// f32 accumulate, M = 128, N = n.
__device__ __forceinline__ uint32_t idesc_bf16(uint32_t n) {
  uint32_t d = 0;
  d |= 1u << 4;                         // D format f32
  d |= 1u << 7;                         // A format bf16
  d |= 1u << 10;                        // B format bf16
  d |= ((n >> 3) & 0x3Fu) << 17;
  d |= ((128u >> 4) & 0x1Fu) << 24;
  return d;
}

__device__ __forceinline__ void mma_bf16_ss(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Vocab split over an expert-parallel group, in the last CTA's 128 epilogue
// threads: thread t < T stores this rank's best key of token t into slot
// (calls & 1) of every rank's exchange buffer, waits (bounded) until every
// rank's key of token t has arrived in its own buffer, keeps the best (the
// same on every rank: the key order is total) and empties the entries; then
// thread 0 advances the call counter. A wait that runs out poisons the local
// buffer (every later exchange on it reports HS_DEV_TIMEOUT at once and stores
// nothing) and leaves the counter, so late keys land in a slot no later call
// reads.
__device__ __forceinline__ void exchange_keys(const Args& a, unsigned long long* key, int T) {
  uint8_t* mine = a.ep_buf[a.ep_rank];
  volatile unsigned long long* hdr = reinterpret_cast<volatile unsigned long long*>(mine);
  const unsigned long long calls = hdr[epx::kHeadCalls];
  const int slot = static_cast<int>(calls & 1ull);
  const bool poisoned = hdr[epx::kHeadPoison] != 0ull;
  const int t = threadIdx.x;
  bool ok = !poisoned;
  unsigned long long best = 0ull;
  if (t < T && ok) {
    const unsigned long long k = key[t];
    for (int q = 0; q < a.ep_world; ++q)
      reinterpret_cast<volatile unsigned long long*>(epx::head_keys(a.ep_buf[q], slot, a.ep_world, a.ep_rank,
                                                                    a.ep_D))[t] = k;
    for (int q = 0; q < a.ep_world && ok; ++q) {
      volatile unsigned long long* e = epx::head_keys(mine, slot, a.ep_world, q, a.ep_D) + t;
      unsigned long long v = *e;
      if (v == epx::kEmptyKey) {
        const uint64_t t0 = globaltimer_ns();
        for (uint32_t it = 1; v == epx::kEmptyKey; ++it) {
          v = *e;
          if ((it & 63u) == 0 && (globaltimer_ns() - t0 > a.wait_ns || hdr[epx::kHeadPoison] != 0ull)) {
            ok = false;
            break;
          }
        }
      }
      if (ok) {
        best = v > best ? v : best;
        *e = epx::kEmptyKey;
      }
    }
  }
  if (t < T) {
    key[t] = ok ? best : 0ull;
    if (!ok) {
      report(a.status, HS_DEV_TIMEOUT);
      hdr[epx::kHeadPoison] = 1ull;
    }
  }
  __threadfence();
  epi_bar();
  if (t == 0 && hdr[epx::kHeadPoison] == 0ull) hdr[epx::kHeadCalls] = calls + 1ull;
  epi_bar();
}

__global__ void __launch_bounds__(kThreads, 1) head_argmax_kernel(const __grid_constant__ CUtensorMap tm_w,
                                                                  const __grid_constant__ CUtensorMap tm_x, Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(base + kStages * kStageBytes);
  __shared__ unsigned long long wbest[4][kN];
  __shared__ int s_last;
  __shared__ int s_am[kN];
  __shared__ unsigned long long s_key[kN];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x, G = gridDim.x;
  const int nk = a.D / kKBox;
  const int t0 = static_cast<int>(static_cast<int64_t>(a.ntiles) * c / G);
  const int t1 = static_cast<int>(static_cast<int64_t>(a.ntiles) * (c + 1) / G);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
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
  if (warp == 0) tc5::tmem_alloc(&bars->tmem, kTmemCols);
  tc5::fence_before_sync();
  __syncthreads();
  tc5::fence_after_sync();
  const uint32_t tmem = bars->tmem;

  if (warp == 4) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      const uint64_t pol = l2_evict_first_policy();
      prefetch_tensormap(&tm_w);
      prefetch_tensormap(&tm_x);
      const int64_t nsteps = static_cast<int64_t>(t1 - t0) * nk;
      // the head does not depend on the previous kernel: the first stages'
      // weight boxes are issued before the wait, their token boxes after it
      const int64_t pre = nsteps < kStages ? nsteps : kStages;
      for (int64_t s = 0; s < pre; ++s) {
        const int tile = t0 + static_cast<int>(s / nk), kb = static_cast<int>(s % nk);
        uint8_t* S = base + s * kStageBytes;
        mbar_arrive_expect_tx(&bars->full[s], kStageBytes);
        tma_load_2d_hint(S, &tm_w, &bars->full[s], kb * kKBox, tile * kM, pol);
      }
      pdl_wait();
      pdl_trigger();
      for (int64_t s = 0; s < pre; ++s) {
        const int kb = static_cast<int>(s % nk);
        tma_load_2d(base + s * kStageBytes + kWBytes, &tm_x, &bars->full[s], kb * kKBox, 0);
      }
      int64_t s = pre;
      for (; s < nsteps; ++s) {
        const int st = static_cast<int>(s % kStages);
        if (!mbar_wait(&bars->empty[st], static_cast<uint32_t>(((s / kStages) - 1) & 1))) {
          report(a.status, HS_DEV_TIMEOUT);
          break;
        }
        const int tile = t0 + static_cast<int>(s / nk), kb = static_cast<int>(s % nk);
        uint8_t* S = base + st * kStageBytes;
        mbar_arrive_expect_tx(&bars->full[st], kStageBytes);
        tma_load_2d_hint(S, &tm_w, &bars->full[st], kb * kKBox, tile * kM, pol);
        tma_load_2d(S + kWBytes, &tm_x, &bars->full[st], kb * kKBox, 0);
      }
      bars->issued = static_cast<int32_t>(s);
    }
  } else if (warp == 5) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      pdl_wait();
      const uint32_t idesc = idesc_bf16(kN);
      int64_t step = 0;
      bool ok = true;
      for (int tile = t0; tile < t1 && ok; ++tile) {
        const int j = tile - t0, buf = j & 1;
        if (j >= 2 && !mbar_wait(&bars->acc_empty[buf], static_cast<uint32_t>(((j >> 1) - 1) & 1))) {
          report(a.status, HS_DEV_TIMEOUT);
          break;
        }
        tc5::fence_after_sync();
        const uint32_t acc = tmem + buf * kN;
        for (int kb = 0; kb < nk; ++kb, ++step) {
          const int st = static_cast<int>(step % kStages);
          if (!mbar_wait(&bars->full[st], static_cast<uint32_t>((step / kStages) & 1))) {
            report(a.status, HS_DEV_TIMEOUT);
            ok = false;
            break;
          }
          tc5::fence_after_sync();
          const uint32_t sA = smem_u32(base + st * kStageBytes);
          const uint64_t ad = tc5::sdesc_sw128(sA), bd = tc5::sdesc_sw128(sA + kWBytes);
#pragma unroll
          for (int k = 0; k < kKBox / 16; ++k)
            mma_bf16_ss(acc, ad + 2 * k, bd + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          tc5::commit(&bars->empty[st]);
        }
        if (ok) tc5::commit(&bars->acc_full[buf]);
      }
      bars->consumed = static_cast<int32_t>(step);
      tc5::commit(&bars->mma_done);
      if (!mbar_wait(&bars->mma_done, 0)) report(a.status, HS_DEV_TIMEOUT);
    }
  } else {
    // ---------------- epilogue (warps 0-3; thread = vocab row of the tile) ----------------
    pdl_wait();
    const int T = a.T;
    unsigned long long best[kN];
#pragma unroll
    for (int t = 0; t < kN; ++t) best[t] = 0ull;
    const uint32_t lane_off = static_cast<uint32_t>(32 * warp) << 16;
    for (int tile = t0; tile < t1; ++tile) {
      const int j = tile - t0, buf = j & 1;
      if (!mbar_wait(&bars->acc_full[buf], static_cast<uint32_t>((j >> 1) & 1))) {
        if (lane == 0) report(a.status, HS_DEV_TIMEOUT);
        break;
      }
      tc5::fence_after_sync();
      float v[16];
      tc5::ld_32x32b_x16(tmem + lane_off + buf * kN, v);
      tc5::wait_ld();
      tc5::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->acc_empty[buf]);
      const int row = tile * kM + 32 * warp + lane;
      const bool inside = row < a.rows;
#pragma unroll
      for (int t = 0; t < kN; ++t) {
        if (t < T) {
          const __nv_bfloat16 lb = __float2bfloat16_rn(v[t]);
          const uint32_t b16 = __bfloat16_as_ushort(lb);
          if (inside && a.logits) a.logits[static_cast<int64_t>(t) * a.V + row] = lb;
          const unsigned long long k = inside ? logit_key(b16, a.row0 + row) : 0ull;
          const unsigned long long wk = warp_max_key(k);
          best[t] = wk > best[t] ? wk : best[t];
        }
      }
    }
    if (lane == 0)
#pragma unroll
      for (int t = 0; t < kN; ++t) wbest[warp][t] = best[t];
    epi_bar();
    // this CTA's best key per token, published for the reduction
    if (threadIdx.x < T) {
      unsigned long long k = wbest[0][threadIdx.x];
      for (int w = 1; w < 4; ++w) k = wbest[w][threadIdx.x] > k ? wbest[w][threadIdx.x] : k;
      __stcg(a.part + static_cast<int64_t>(c) * kPartStride + threadIdx.x, k);
    }
    __threadfence();
    epi_bar();
    if (threadIdx.x == 0) s_last = atomicAdd(a.ticket, 1u) == static_cast<uint32_t>(G - 1);
    epi_bar();
    if (s_last) {
      __threadfence();
      // warp w reduces tokens w, w + 4, ...: lanes stride over the CTAs
      for (int t = warp; t < T; t += 4) {
        unsigned long long k = 0ull;
        for (int g = lane; g < G; g += 32) {
          const unsigned long long q = __ldcg(a.part + static_cast<int64_t>(g) * kPartStride + t);
          k = q > k ? q : k;
        }
        k = warp_max_key(k);
        if (lane == 0) s_key[t] = k;
      }
      epi_bar();
      if (a.ep_world > 0) exchange_keys(a, s_key, T);  // every rank's best of its rows
      if (threadIdx.x < T) {
        const unsigned long long k = s_key[threadIdx.x];
        const int am = k ? key_index(k) : 0;
        s_am[threadIdx.x] = am;
        if (a.argmax_out) a.argmax_out[threadIdx.x] = am;
      }
      epi_bar();
      if (threadIdx.x == 0) {
        int n = 0;
        if (a.draft_ids) {
          while (n < T - 1) {
            const int64_t d = a.draft_ids[n];
            if (d < 0 || d >= a.V) {
              report(a.status, HS_DEV_BAD_DRAFT);
              break;
            }
            if (d != s_am[n]) break;
            ++n;
          }
        }
        if (a.n_accept) *a.n_accept = n;
        if (a.next_token) *a.next_token = s_am[n];
        *a.ticket = 0u;  // ready for the next call (stream order)
      }
    }
  }

  tc5::fence_before_sync();
  __syncthreads();
  // copies issued but never consumed (only after a wait that gave up): let
  // them land before the CTA's shared memory is released
  if (threadIdx.x == 128) {
    for (int64_t k = bars->consumed; k < bars->issued; ++k)
      if (!mbar_wait(&bars->full[k % kStages], static_cast<uint32_t>((k / kStages) & 1))) {
        report(a.status, HS_DEV_TIMEOUT);
        break;
      }
  }
  __syncthreads();
  if (warp == 0) {
    tc5::fence_after_sync();
    tc5::tmem_dealloc(tmem, kTmemCols);
  }
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

// bf16 matrix [rows][cols] (row pitch cols * 2 bytes), box 64 x box_rows, 128B swizzle.
static int bf16_map(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return HS_ERR_UNSUPPORTED;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kKBox), box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_cuda_error(static_cast<int>(r));
    return HS_ERR_CUDA;
  }
  return HS_OK;
}

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

}  // namespace head
}  // namespace hs

using namespace hs;
using namespace hs::head;

extern "C" size_t hs_lm_head_workspace_size(int64_t T) {
  (void)T;
  return static_cast<size_t>(256 + static_cast<int64_t>(sm_count()) * kPartStride * 8);
}

static int head_impl(const void* x, const void* head, int64_t T, int64_t D, int64_t V, int64_t row0, int64_t rows,
                     const int64_t* draft_ids, int64_t* argmax_out, int32_t* n_accept, int64_t* next_token,
                     void* logits_out, const hs_ep_peers* peers, void* workspace, size_t workspace_bytes,
                     int32_t* dev_status, void* stream) {
  if (!x || !head || !workspace) return HS_ERR_BAD_ARGUMENT;
  if (T < 1 || T > kN || D < kKBox || D % kKBox || D > 65536 || V < 1 || V > (int64_t{1} << 30))
    return HS_ERR_BAD_SHAPE;
  if (row0 < 0 || rows < 1 || row0 + rows > V) return HS_ERR_BAD_SHAPE;
  if (!argmax_out && !n_accept && !next_token && !logits_out) return HS_ERR_BAD_ARGUMENT;
  if (!aligned16(x) || !aligned16(head) || !aligned16(workspace) || (logits_out && (V % 8 || !aligned16(logits_out))))
    return HS_ERR_ALIGN;
  if (workspace_bytes < hs_lm_head_workspace_size(T)) return HS_ERR_WORKSPACE;
  if (peers) {
    if (logits_out || peers->world < 1 || peers->world > HS_EP_MAX_RANKS || peers->rank < 0 ||
        peers->rank >= peers->world || D > 8192)
      return HS_ERR_BAD_ARGUMENT;
    for (int q = 0; q < peers->world; ++q)
      if (!peers->recv[q] || !aligned16(peers->recv[q])) return HS_ERR_BAD_ARGUMENT;
  }
  CUtensorMap tm_w, tm_x;
  int rc;
  if ((rc = bf16_map(&tm_w, head, static_cast<uint64_t>(D), static_cast<uint64_t>(rows), kM))) return rc;
  if ((rc = bf16_map(&tm_x, x, static_cast<uint64_t>(D), static_cast<uint64_t>(T), kN))) return rc;
  static std::atomic<uint64_t> done{0};
  int dev = 0;
  HS_CUDA_CHECK(cudaGetDevice(&dev));
  const uint64_t bit = 1ull << (dev & 63);
  if (!(done.load() & bit)) {
    HS_CUDA_CHECK(cudaFuncSetAttribute(head_argmax_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
    done.fetch_or(bit);
  }
  Args a;
  a.T = static_cast<int>(T);
  a.D = static_cast<int>(D);
  a.V = static_cast<int>(V);
  a.row0 = static_cast<int>(row0);
  a.rows = static_cast<int>(rows);
  a.ntiles = static_cast<int>((rows + kM - 1) / kM);
  a.draft_ids = T > 1 ? draft_ids : nullptr;
  a.argmax_out = argmax_out;
  a.n_accept = n_accept;
  a.next_token = next_token;
  a.logits = static_cast<__nv_bfloat16*>(logits_out);
  a.ticket = static_cast<uint32_t*>(workspace);
  a.part = reinterpret_cast<unsigned long long*>(static_cast<uint8_t*>(workspace) + 256);
  a.status = dev_status;
  a.ep_rank = peers ? peers->rank : 0;
  a.ep_world = peers ? peers->world : 0;
  a.ep_D = static_cast<int>(D);
  a.wait_ns = peers && peers->wait_limit_ns > 0 ? static_cast<uint64_t>(peers->wait_limit_ns) : kWaitLimitNs;
  for (int q = 0; q < HS_EP_MAX_RANKS; ++q)
    a.ep_buf[q] = peers && q < peers->world ? static_cast<uint8_t*>(peers->recv[q]) : nullptr;
  const int G = std::min(sm_count(), a.ntiles);
  HS_CUDA_CHECK(launch_pdl(head_argmax_kernel, dim3(static_cast<unsigned>(G)), dim3(kThreads), kSmemBytes,
                           static_cast<cudaStream_t>(stream), tm_w, tm_x, a));
  return check_launch();
}

extern "C" int hs_lm_head_argmax(const void* x, const void* head, int64_t T, int64_t D, int64_t V,
                                 const int64_t* draft_ids, int64_t* argmax_out, int32_t* n_accept,
                                 int64_t* next_token, void* logits_out, void* workspace, size_t workspace_bytes,
                                 int32_t* dev_status, void* stream) {
  return head_impl(x, head, T, D, V, 0, V, draft_ids, argmax_out, n_accept, next_token, logits_out, nullptr,
                   workspace, workspace_bytes, dev_status, stream);
}

extern "C" int hs_lm_head_argmax_ep(const void* x, const void* head_rows, int64_t T, int64_t D, int64_t V,
                                    int64_t row0, int64_t rows, const int64_t* draft_ids, int64_t* argmax_out,
                                    int32_t* n_accept, int64_t* next_token, const hs_ep_peers* peers,
                                    void* workspace, size_t workspace_bytes, int32_t* dev_status, void* stream) {
  if (!peers) return HS_ERR_BAD_ARGUMENT;
  return head_impl(x, head_rows, T, D, V, row0, rows, draft_ids, argmax_out, n_accept, next_token, nullptr, peers,
                   workspace, workspace_bytes, dev_status, stream);
}
