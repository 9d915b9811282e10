// Library-level helpers: status strings, per-thread last CUDA error, and the
// synthetic byte fill used to build full-size random-init expert stores.
#include "hs_common.cuh"

namespace hs {

static thread_local int g_last_cuda_error = 0;

void set_last_cuda_error(int e) { g_last_cuda_error = e; }

int check_launch() {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_cuda_error(static_cast<int>(e));
    return HS_ERR_CUDA;
  }
  return HS_OK;
}

// splitmix64 finaliser: a counter-based hash, so any byte range can be
// regenerated independently of the launch shape.
__device__ __forceinline__ uint64_t mix64(uint64_t x) {
  x += 0x9e3779b97f4a7c15ull;
  x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
  x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
  return x ^ (x >> 31);
}

__global__ void fill_bytes_kernel(uint8_t* __restrict__ dst, int64_t n, uint64_t seed, uint32_t lo, uint32_t span) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t nwords = n / 8;
  uint64_t* d64 = reinterpret_cast<uint64_t*>(dst);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < nwords; i += stride) {
    uint64_t h = mix64(seed ^ mix64(static_cast<uint64_t>(i)));
    uint64_t out = 0;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      const uint32_t byte = static_cast<uint32_t>((h >> (8 * b)) & 0xffu);
      const uint32_t v = span == 256u ? byte : lo + (byte * span >> 8);
      out |= static_cast<uint64_t>(v & 0xffu) << (8 * b);
    }
    d64[i] = out;
  }
  // tail bytes
  const int64_t t0 = nwords * 8;
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i < n - t0) {
    const uint64_t h = mix64(seed ^ mix64(static_cast<uint64_t>(nwords + i)));
    const uint32_t byte = static_cast<uint32_t>(h & 0xffu);
    dst[t0 + i] = static_cast<uint8_t>(span == 256u ? byte : lo + (byte * span >> 8));
  }
}

}  // namespace hs

extern "C" int hs_abi_version(void) { return HS_ABI_VERSION; }

extern "C" const char* hs_status_string(int status) {
  switch (status) {
    case HS_OK:
      return "ok";
    case HS_ERR_BAD_SHAPE:
      return "unsupported shape";
    case HS_ERR_BAD_ARGUMENT:
      return "bad argument";
    case HS_ERR_WORKSPACE:
      return "workspace too small";
    case HS_ERR_ALIGN:
      return "pointer or stride not 16-byte aligned";
    case HS_ERR_CUDA:
      return "CUDA error";
    case HS_ERR_UNSUPPORTED:
      return "unsupported device or driver";
    case HS_ERR_NCCL:
      return "NCCL error";
    default:
      return "unknown status";
  }
}

extern "C" int hs_last_cuda_error(void) { return hs::g_last_cuda_error; }

extern "C" int hs_fill_bytes(void* dst, int64_t n, uint64_t seed, int32_t lo, int32_t hi, void* stream) {
  if (n < 0 || lo < 0 || hi > 255 || lo > hi) return HS_ERR_BAD_ARGUMENT;
  if (n == 0) return HS_OK;
  if (!dst || (reinterpret_cast<uintptr_t>(dst) & 7u)) return HS_ERR_ALIGN;
  const uint32_t span = static_cast<uint32_t>(hi - lo + 1);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t words = (n + 7) / 8;
  int64_t blocks = (words + 255) / 256;
  if (blocks > static_cast<int64_t>(sms) * 16) blocks = static_cast<int64_t>(sms) * 16;
  if (blocks < 1) blocks = 1;
  hs::fill_bytes_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint8_t*>(dst), n, seed, static_cast<uint32_t>(lo), span);
  return hs::check_launch();
}
