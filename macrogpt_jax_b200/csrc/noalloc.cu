// ufp8_amax_quant_noalloc: per-tensor current-scaling quantization (amax -> scale -> fp8) whose
// scratch lives in this file's static device arrays, so the call needs no amax buffer from the
// caller and allocates nothing.
//
// Scratch (per device, in the module's global memory):
//   g_na_partials[kNaMaxParts]  one partial max|x| per 65 536-element block of x (16 KiB);
//   g_na_amax[0]                the tensor's amax, read by the quantize kernel.
// Every partial the reduction reads is written earlier in the same call, and the reduction
// overwrites g_na_amax[0], so no scratch word has to start at zero and nothing is memset.
//
// Launches, in stream order: na_partial_kernel (one CTA per block of x) -> na_reduce_kernel
// (one CTA) -> the library's quantize kernel with amax = &g_na_amax[0] (the launch
// ufp8_quantize uses).  The result is bit-identical to ufp8_amax_quant.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "internal.h"

namespace ufp8 {
namespace {

constexpr int kNaThreads = 256;
constexpr int64_t kNaBlockElems = 65536;  // elements of x per partial
constexpr int kNaMaxParts = 4096;         // => at most 268 435 456 elements per call
constexpr int kNaMaxDevices = 64;

__device__ __align__(256) uint32_t g_na_partials[kNaMaxParts];
__device__ __align__(256) float g_na_amax[64];  // [0] used; padded to its own 256 bytes

// max|x| over elements [blockIdx.x * kNaBlockElems, ...) as an unsigned max of the sign-cleared
// bf16 bit patterns (NaN above inf above every finite value), stored as f32 bits.
__global__ void __launch_bounds__(kNaThreads) na_partial_kernel(const uint16_t* __restrict__ x, int64_t n,
                                                                bool vec) {
  const int64_t begin = static_cast<int64_t>(blockIdx.x) * kNaBlockElems;
  const int64_t end = min(n, begin + kNaBlockElems);
  uint32_t m2 = 0;  // packed 2 x 16-bit maxima
  if (vec) {
    // begin is a multiple of 8 elements and x is 16-byte aligned: 8 bf16 per load.
    const int64_t nv = (end - begin) / 8;
    const uint4* xv = reinterpret_cast<const uint4*>(x + begin);
    for (int64_t i = threadIdx.x; i < nv; i += kNaThreads) {
      const uint4 w = xv[i];
      m2 = __vmaxu2(m2, w.x & 0x7FFF7FFFu);
      m2 = __vmaxu2(m2, w.y & 0x7FFF7FFFu);
      m2 = __vmaxu2(m2, w.z & 0x7FFF7FFFu);
      m2 = __vmaxu2(m2, w.w & 0x7FFF7FFFu);
    }
    for (int64_t i = begin + nv * 8 + threadIdx.x; i < end; i += kNaThreads)
      m2 = __vmaxu2(m2, static_cast<uint32_t>(x[i]) & 0x7FFFu);
  } else {
    for (int64_t i = begin + threadIdx.x; i < end; i += kNaThreads)
      m2 = __vmaxu2(m2, static_cast<uint32_t>(x[i]) & 0x7FFFu);
  }
  uint32_t m = max(m2 & 0xFFFFu, m2 >> 16);
  m = __reduce_max_sync(0xFFFFFFFFu, m);
  __shared__ uint32_t warp_max[kNaThreads / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) warp_max[warp] = m;
  __syncthreads();
  if (warp == 0) {
    uint32_t v = lane < kNaThreads / 32 ? warp_max[lane] : 0u;
    v = __reduce_max_sync(0xFFFFFFFFu, v);
    if (lane == 0) g_na_partials[blockIdx.x] = v << 16;
  }
}

// g_na_amax[0] = max of the first `parts` partials (0 when parts == 0, i.e. an empty tensor).
__global__ void __launch_bounds__(kNaThreads) na_reduce_kernel(int parts) {
  uint32_t m = 0;
  for (int i = threadIdx.x; i < parts; i += kNaThreads) m = max(m, g_na_partials[i]);
  m = __reduce_max_sync(0xFFFFFFFFu, m);
  __shared__ uint32_t warp_max[kNaThreads / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) warp_max[warp] = m;
  __syncthreads();
  if (warp == 0) {
    uint32_t v = lane < kNaThreads / 32 ? warp_max[lane] : 0u;
    v = __reduce_max_sync(0xFFFFFFFFu, v);
    if (lane == 0) g_na_amax[0] = __uint_as_float(v);
  }
}

// Device address of g_na_amax for the current device.  The lookup (cudaGetSymbolAddress, with
// the device current) runs on the first call in each CUDA context and again whenever the
// device's current context changes (after cudaDeviceReset the module is loaded anew and may sit
// at another address).  A mutex serialises the cache, so first calls from several host threads
// do not race.
using CtxGetCurrentFn = CUresult (*)(CUcontext*);

CtxGetCurrentFn ctx_get_current_fn() {
  static CtxGetCurrentFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<CtxGetCurrentFn>(nullptr);
    return reinterpret_cast<CtxGetCurrentFn>(p);
  }();
  return fn;
}

int na_amax_address(int device, float** out) {
  struct Entry {
    CUcontext ctx;
    float* addr;
  };
  static Entry cache[kNaMaxDevices] = {};
  static std::mutex mu;
  if (device < 0 || device >= kNaMaxDevices)
    return set_error(UFP8_ERR_UNSUPPORTED, "ufp8_amax_quant_noalloc: device %d >= %d", device, kNaMaxDevices);
  CtxGetCurrentFn get_ctx = ctx_get_current_fn();
  CUcontext ctx = nullptr;
  if (!get_ctx || get_ctx(&ctx) != CUDA_SUCCESS || !ctx)
    return set_error(UFP8_ERR_CUDA, "ufp8_amax_quant_noalloc: no current CUDA context");
  std::lock_guard<std::mutex> lock(mu);
  Entry& e = cache[device];
  if (!e.addr || e.ctx != ctx) {
    void* p = nullptr;
    cudaError_t err = cudaGetSymbolAddress(&p, g_na_amax);
    if (err != cudaSuccess) return cuda_error(err, "cudaGetSymbolAddress(no-alloc amax scratch)");
    e.addr = static_cast<float*>(p);
    e.ctx = ctx;
  }
  *out = e.addr;
  return UFP8_OK;
}

}  // namespace
}  // namespace ufp8

using namespace ufp8;

extern "C" int ufp8_amax_quant_noalloc(const void* x_bf16, int64_t n, int fmt, void* q, float* inv_scale,
                                       ufp8_stream_t stream) {
  if (n < 0) return set_error(UFP8_ERR_INVALID, "ufp8_amax_quant_noalloc: n < 0");
  if (fmt != UFP8_E4M3 && fmt != UFP8_E5M2)
    return set_error(UFP8_ERR_INVALID, "ufp8_amax_quant_noalloc: fmt %d is not UFP8_E4M3/UFP8_E5M2", fmt);
  if (!inv_scale || (n > 0 && (!x_bf16 || !q)))
    return set_error(UFP8_ERR_INVALID, "ufp8_amax_quant_noalloc: null pointer");
  if (reinterpret_cast<uintptr_t>(x_bf16) & 1u)
    return set_error(UFP8_ERR_ALIGN, "ufp8_amax_quant_noalloc: x not 2-byte aligned");
  const int64_t parts = (n + kNaBlockElems - 1) / kNaBlockElems;
  if (parts > kNaMaxParts)
    return set_error(UFP8_ERR_UNSUPPORTED,
                     "ufp8_amax_quant_noalloc: %lld elements exceed the static scratch (at most %lld)",
                     static_cast<long long>(n), static_cast<long long>(kNaMaxParts * kNaBlockElems));
  DeviceInfo* dev;
  if (int rc = device_info(&dev)) return rc;
  float* amax = nullptr;
  if (int rc = na_amax_address(dev->device, &amax)) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (parts > 0) {
    const bool vec = (reinterpret_cast<uintptr_t>(x_bf16) & 15u) == 0;
    na_partial_kernel<<<static_cast<int>(parts), kNaThreads, 0, s>>>(static_cast<const uint16_t*>(x_bf16), n, vec);
  }
  na_reduce_kernel<<<1, kNaThreads, 0, s>>>(static_cast<int>(parts));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, "no-alloc amax kernel launch");
  return launch_quantize(x_bf16, n, fmt, amax, q, inv_scale, s, *dev);
}
