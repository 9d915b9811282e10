// Shared device helpers for the sm_100a kernels: bounded mbarrier waits,
// TMA / bulk-copy issue, FP4/FP8 -> f16 conversion, legacy-layout MMA, and
// bf16 rounding helpers. Everything here is hand-written inline PTX or plain
// CUDA; no library kernels.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "../../include/hs_ext.h"

#define HS_DI __device__ __forceinline__

namespace hs {

// ---------------------------------------------------------------------------
// Host-side error plumbing
// ---------------------------------------------------------------------------
void set_last_cuda_error(int e);

#define HS_CUDA_CHECK(expr)                         \
  do {                                              \
    cudaError_t _e = (expr);                        \
    if (_e != cudaSuccess) {                        \
      ::hs::set_last_cuda_error(static_cast<int>(_e)); \
      return HS_ERR_CUDA;                           \
    }                                               \
  } while (0)

// Returns HS_ERR_CUDA if the most recent launch on this thread failed.
int check_launch();

// The dimensions an hs_moe_make_desc descriptor was built for (hs_moe.cu).
int moe_desc_dims(const void* desc, int64_t* E, int64_t* D, int64_t* I, int64_t* I_sh);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------------------
// Device: time / status
// ---------------------------------------------------------------------------
HS_DI uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

HS_DI void report(int32_t* status, int32_t bits) {
  if (status != nullptr) atomicOr(status, bits);
}

HS_DI uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

HS_DI uint32_t ld_relaxed_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// 16-byte volatile load / store (each 4-byte word is single-copy atomic; a
// reader that sees a torn vector polls again for the words still missing)
HS_DI uint4 ld_volatile_u4(const void* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

HS_DI void st_volatile_u4(void* p, uint4 v) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// Bounded waits give up after this many nanoseconds (about two seconds), after
// which the kernel reports HS_DEV_TIMEOUT and returns.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// Receive buffer of the peer-memory expert-parallel exchange (one per rank,
// every rank's mapped in every process): a 256-byte header of u64 words ([0]
// MoE calls made, [1] MoE combine ticket, [2] MoE exchange poisoned, [3]
// lm_head calls made, [4] lm_head exchange poisoned), then two slots (calls
// alternate) of [world][routed, shared][8 tokens][D] f32 MoE rows, then two
// slots of [HS_EP_MAX_RANKS][16 tokens] u64 lm_head keys. A rank's call k
// writes slot k % 2 of every rank; rank q's call k+2 can only start after
// every rank finished call k+1 and so consumed slot k % 2. An empty entry
// holds all ones (for the rows a NaN bit pattern the sums never produce: their
// NaNs are the canonical 0x7fffffff; no key is all ones), so an entry is its
// own arrival flag: the producer only stores, the consumer waits for every
// entry it reads to be filled and sets it back to empty.
namespace epx {
constexpr int64_t kHdr = 256;
constexpr int kPoison = 2;      // header word set once a MoE combine's wait ran out
constexpr int kHeadCalls = 3;   // header word: lm_head exchanges made
constexpr int kHeadPoison = 4;  // header word set once an lm_head exchange's wait ran out
constexpr uint32_t kEmpty = 0xffffffffu;
constexpr unsigned long long kEmptyKey = 0xffffffffffffffffull;
constexpr int kRows = 8;
constexpr int kHeadTokens = 16;
__host__ __device__ inline float* rows(uint8_t* buf, int slot, int world, int src, int which, int D) {
  return reinterpret_cast<float*>(buf + kHdr) +
         ((static_cast<int64_t>(slot) * world + src) * 2 + which) * kRows * static_cast<int64_t>(D);
}
__host__ __device__ inline int64_t rows_bytes(int64_t world, int64_t D) {
  return 2 * world * 2 * kRows * D * static_cast<int64_t>(sizeof(float));
}
__host__ __device__ inline unsigned long long* head_keys(uint8_t* buf, int slot, int world, int src, int D) {
  return reinterpret_cast<unsigned long long*>(buf + kHdr + rows_bytes(world, D)) +
         (static_cast<int64_t>(slot) * HS_EP_MAX_RANKS + src) * kHeadTokens;
}
inline size_t bytes(int64_t world, int64_t D) {
  return static_cast<size_t>(kHdr + rows_bytes(world, D) +
                             2 * HS_EP_MAX_RANKS * kHeadTokens * static_cast<int64_t>(sizeof(unsigned long long)));
}
}  // namespace epx

// ---------------------------------------------------------------------------
// Device: mbarrier
// ---------------------------------------------------------------------------
HS_DI uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

HS_DI void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

HS_DI void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

HS_DI void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// Add tx bytes to the current phase without arriving (the arrive follows later).
HS_DI void mbar_expect_tx(uint64_t* bar, uint32_t tx) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(tx) : "memory");
}

HS_DI void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

HS_DI bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete; false after the limit.
HS_DI bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) return false;
  }
}

// ---------------------------------------------------------------------------
// Device: TMA (tensor) and bulk (1D) copies global -> shared, completing on an
// mbarrier with transaction bytes. Every copy here targets the issuing CTA only.
// ---------------------------------------------------------------------------
HS_DI void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// L2 policy for data streamed exactly once (expert weights): evict it first so
// data that is read again (activations, partial sums) stays in L2.
HS_DI uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

HS_DI void tma_load_2d_hint(void* dst, const CUtensorMap* map, uint64_t* bar, int32_t x, int32_t y, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, "
      "{%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(pol)
      : "memory");
}

HS_DI void bulk_load_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}

HS_DI void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int32_t x, int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

HS_DI void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// Bring [src, src + bytes) into L2 without waiting (bytes a multiple of 16,
// src 16-byte aligned): data a later phase reads, fetched while HBM is idle.
HS_DI void prefetch_l2_bulk(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(src)), "r"(bytes)
               : "memory");
}

// Distributed shared memory: the address of this CTA's shared variable at
// `local` in cluster rank `rank`, and an 8-byte load from it.
HS_DI uint32_t dsmem_addr(const void* local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(local)), "r"(rank));
  return r;
}
HS_DI float2 ld_dsmem_f2(uint32_t addr) {
  float2 v;
  asm volatile("ld.shared::cluster.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr) : "memory");
  return v;
}

// Programmatic dependent launch. A kernel launched with launch_pdl() may start
// while its predecessor in the stream is still running: it must call
// pdl_wait() before it reads or writes any global memory the predecessor (or
// anything earlier) touches. pdl_trigger() lets the successor launch early.
HS_DI void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
HS_DI void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

HS_DI void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------------------
// Device: shared-memory loads
// ---------------------------------------------------------------------------
HS_DI uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
HS_DI uint2 lds64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}
HS_DI uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}
HS_DI uint32_t lds8(uint32_t addr) {
  uint16_t v;
  asm volatile("ld.shared.u8 %0, [%1];" : "=h"(v) : "r"(addr));
  return v;
}

// ---------------------------------------------------------------------------
// Device: FP4 (e2m1) and FP8 (e4m3) -> f16x2. Both conversions are exact.
// e2m1x2: one byte holds two values; the low nibble lands in the low half.
// e4m3x2: two bytes; the low byte lands in the low half.
// ---------------------------------------------------------------------------
HS_DI void e2m1x8_to_f16x2x4(uint32_t w, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm("{\n .reg .b8 b0, b1, b2, b3;\n mov.b32 {b0, b1, b2, b3}, %4;\n"
      " cvt.rn.f16x2.e2m1x2 %0, b0;\n cvt.rn.f16x2.e2m1x2 %1, b1;\n"
      " cvt.rn.f16x2.e2m1x2 %2, b2;\n cvt.rn.f16x2.e2m1x2 %3, b3;\n}\n"
      : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
      : "r"(w));
}

HS_DI void e4m3x4_to_f16x2x2(uint32_t w, uint32_t& r0, uint32_t& r1) {
  asm("{\n .reg .b16 lo, hi;\n mov.b32 {lo, hi}, %2;\n"
      " cvt.rn.f16x2.e4m3x2 %0, lo;\n cvt.rn.f16x2.e4m3x2 %1, hi;\n}\n"
      : "=r"(r0), "=r"(r1)
      : "r"(w));
}

// ue8m0 -> f32 as torch converts float8_e8m0fnu: 0 -> 2^-127, 255 -> NaN.
HS_DI float e8m0_to_f32_torch(uint32_t s) {
  if (s == 0u) return __uint_as_float(0x00400000u);
  if (s == 255u) return __uint_as_float(0x7fc00000u);
  return __uint_as_float(s << 23);
}
// ue8m0 -> f32 by the bit shift of weight_loader.py:14-19 (0 -> 0, 255 -> inf).
HS_DI float e8m0_to_f32_shift(uint32_t s) { return __uint_as_float(s << 23); }

// ---------------------------------------------------------------------------
// Device: legacy warp MMA m16n8k16, f16 inputs, f32 accumulate.
// ---------------------------------------------------------------------------
HS_DI void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
HS_DI void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---------------------------------------------------------------------------
// Device: rounding helpers (round-to-nearest-even, like torch's .to(bf16)).
// ---------------------------------------------------------------------------
HS_DI float round_bf16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// 2^e as f32 for e in [-126, 127].
HS_DI float exp2i(int e) { return __uint_as_float(static_cast<uint32_t>(e + 127) << 23); }

// Eight bf16 (one 16-byte vector) <-> f32, element i of the vector at f[i].
HS_DI void bf16x8_unpack(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

HS_DI uint4 bf16x8_pack(const float (&f)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t lo = __bfloat16_as_ushort(__float2bfloat16_rn(f[2 * i]));
    const uint32_t hi = __bfloat16_as_ushort(__float2bfloat16_rn(f[2 * i + 1]));
    w[i] = lo | (hi << 16);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// RMSNorm constants shared by every kernel that normalises rows, so all of
// them sum in the same order: a row of D bf16 values is read as D/8 vectors;
// thread j of kNormThreads takes vectors j, j + kNormThreads, ... and sums the
// squares in element order, the warp sums with a fixed xor tree, and the warp
// sums are added in warp order.
constexpr int kNormThreads = 256;
constexpr int kNormMaxVec = 4;  // D <= kNormThreads * 8 * kNormMaxVec = 8192

}  // namespace hs

// Host: launch `kernel` with programmatic stream serialization allowed (the
// kernel must call pdl_wait() before touching global memory).
template <typename... KArgs, typename... Args>
static inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                     Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Host: launch_pdl with thread-block clusters of cluster_x CTAs along x.
template <typename... KArgs, typename... Args>
static inline cudaError_t launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                             cudaStream_t st, unsigned cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster_x;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}
