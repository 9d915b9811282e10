// Verify-state snapshot and restore on the device, sm_100a.
//
// Reference being replaced: the per-step state handling of
// HomeSeekInferenceEngine._mtp_verify_batched (inference_engine/engine.py:
// 2443-2459 snapshot, 2500-2538 trim / restore). Before the fused verify
// forward the reference clones every layer's KV latent cache, compressed KV
// data and index, and compressor state (O(context) bytes per step, plus a
// fresh allocation per tensor); afterwards, unless every position was
// accepted, it trims each KV cache to its old length + n_accept, puts the
// compressed data and compressor states back, and sets the position to
// old + n_accept.
//
// Here the states are registered once as regions of a device-resident table:
//   * append regions (KV caches, the position): a device entry count; the
//     snapshot records it, the commit sets it to saved + n_accept (regions
//     that keep accepted entries) or back to saved; no bytes move;
//   * copy regions (states the forward overwrites in place: compressor
//     states, compressed KV that is rewritten): the snapshot copies them into
//     a caller-owned shadow, the commit copies them back.
// Each call is one launch over all regions, and the commit reads n_accept
// from device memory (written by the acceptance kernel), so a decode
// iteration needs no host synchronisation and can be captured in one graph.
#include <algorithm>

#include "hs_common.cuh"

namespace hs {
namespace state {

constexpr int kThreads = 256;
constexpr int64_t kChunk = 64 * 1024;  // bytes per CTA per copy region

__global__ void __launch_bounds__(kThreads) snapshot_kernel(hs_state_region* regions, int64_t n) {
  const int64_t r = blockIdx.y;
  if (r >= n) return;
  hs_state_region* g = regions + r;
  if (g->length) {
    if (blockIdx.x == 0 && threadIdx.x == 0) g->saved_length = *g->length;
    return;
  }
  const int64_t off = static_cast<int64_t>(blockIdx.x) * kChunk;
  if (!g->shadow || off >= g->bytes) return;
  const int64_t end = min(g->bytes, off + kChunk);
  const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(g->live) + off);
  uint4* dst = reinterpret_cast<uint4*>(static_cast<uint8_t*>(g->shadow) + off);
  for (int64_t i = threadIdx.x; i < (end - off) / 16; i += kThreads) dst[i] = __ldcs(src + i);
}

__global__ void __launch_bounds__(kThreads) commit_kernel(hs_state_region* regions, int64_t n,
                                                          const int32_t* n_accept, int32_t t_total) {
  const int64_t r = blockIdx.y;
  if (r >= n) return;
  const int32_t acc = *n_accept;
  if (acc >= t_total) return;  // every position accepted: keep the verify's state
  hs_state_region* g = regions + r;
  if (g->length) {
    if (blockIdx.x == 0 && threadIdx.x == 0) *g->length = g->saved_length + (g->keep_accepted ? acc : 0);
    return;
  }
  const int64_t off = static_cast<int64_t>(blockIdx.x) * kChunk;
  if (!g->shadow || off >= g->bytes) return;
  const int64_t end = min(g->bytes, off + kChunk);
  const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(g->shadow) + off);
  uint4* dst = reinterpret_cast<uint4*>(static_cast<uint8_t*>(g->live) + off);
  for (int64_t i = threadIdx.x; i < (end - off) / 16; i += kThreads) dst[i] = __ldcs(src + i);
}

static int grid_of(int64_t n, int64_t max_bytes, dim3* grid) {
  if (n < 1 || n > 65535 || max_bytes < 0) return HS_ERR_BAD_SHAPE;
  const int64_t gx = std::max<int64_t>(1, (max_bytes + kChunk - 1) / kChunk);
  if (gx > 0x7fffffff) return HS_ERR_BAD_SHAPE;
  *grid = dim3(static_cast<unsigned>(gx), static_cast<unsigned>(n));
  return HS_OK;
}

}  // namespace state
}  // namespace hs

using namespace hs;
using namespace hs::state;

extern "C" int hs_verify_state_snapshot(hs_state_region* regions, int64_t n, int64_t max_bytes, void* stream) {
  if (!regions) return HS_ERR_BAD_ARGUMENT;
  dim3 grid;
  int rc;
  if ((rc = grid_of(n, max_bytes, &grid))) return rc;
  snapshot_kernel<<<grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(regions, n);
  return check_launch();
}

extern "C" int hs_verify_state_commit(hs_state_region* regions, int64_t n, int64_t max_bytes,
                                      const int32_t* n_accept, int32_t t_total, void* stream) {
  if (!regions || !n_accept || t_total < 1) return HS_ERR_BAD_ARGUMENT;
  dim3 grid;
  int rc;
  if ((rc = grid_of(n, max_bytes, &grid))) return rc;
  commit_kernel<<<grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(regions, n, n_accept, t_total);
  return check_launch();
}
