// Per-tensor amax and fp8 quantisation (bf16 -> float8_e4m3fn / float8_e5m2).
//
// Semantics (the per-tensor current-scaling recipe around the reference's casts,
// ueaj/utils/gradutils.py:15-54):
//   amax      = max |x|, taken as an unsigned max over the sign-cleared bf16 bit patterns,
//               so it is exact and NaN-propagating (a NaN pattern is above +inf);
//   s         = min(FMAX / amax, FLT_MAX) in IEEE fp32 (FMAX = 448 for e4m3fn, 57344 for
//               e5m2), s = 1 when amax == 0, NaN when amax is NaN;
//   q         = cast(f32(x) * s) with round-to-nearest-even and the ml_dtypes 0.5.4
//               overflow rules (e4m3fn: |p| > 464 or inf -> NaN 0x7F|sign;
//               e5m2: |p| >= 61440 or inf -> inf 0x7C|sign); a NaN product becomes the
//               positive NaN pattern (0x7F e4m3fn, 0x7E e5m2);
//   inv_scale = 1 / s in IEEE fp32.
// The hardware conversion (cvt.rn.satfinite) rounds to nearest even like the cast; it
// only saturates where the cast overflows, so those products (and NaN) are re-encoded.
// With s derived from the tensor's own amax, |x*s| <= 448.0001 (resp. 57344.004) and the
// re-encoding is reached only by non-finite products; a caller-supplied amax below the
// true maximum reaches the overflow rules.
//
// Both kernels are HBM-bound streaming passes: 16-byte vector loads, a grid of a few
// CTAs per SM with grid-stride loops, and (amax) a packed 2x16-bit unsigned max
// followed by a warp shuffle reduction and one atomicMax per CTA.
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include "fp8cast.cuh"
#include "internal.h"

namespace ufp8 {
namespace {

constexpr int kThreads = 256;
constexpr int kCtasPerSm = 8;

__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint32_t absmax2(uint32_t acc, uint32_t w) {
  return __vmaxu2(acc, w & 0x7FFF7FFFu);
}

__device__ __forceinline__ void block_amax_commit(uint32_t m2, unsigned int* amax_bits) {
  uint32_t m = max(m2 & 0xFFFFu, m2 >> 16);
  m = __reduce_max_sync(0xFFFFFFFFu, m);
  __shared__ uint32_t warp_max[kThreads / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) warp_max[warp] = m;
  __syncthreads();
  if (warp == 0) {
    uint32_t v = lane < (kThreads / 32) ? warp_max[lane] : 0u;
    v = __reduce_max_sync(0xFFFFFFFFu, v);
    if (lane == 0 && v != 0u) atomicMax(amax_bits, v << 16);
  }
}

// Vector body: x is 16-byte aligned; n_vec groups of 8 bf16, then n_tail (< 8) scalars.
__global__ void __launch_bounds__(kThreads) amax_vec_kernel(const uint4* __restrict__ x, int64_t n_vec,
                                                            const uint16_t* __restrict__ tail, int n_tail,
                                                            unsigned int* amax_bits) {
  uint32_t m2 = 0;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  // Four independent 16-byte loads in flight per thread per iteration.
  for (; i + 3 * stride < n_vec; i += 4 * stride) {
    const uint4 a = ld_stream(x + i);
    const uint4 b = ld_stream(x + i + stride);
    const uint4 c = ld_stream(x + i + 2 * stride);
    const uint4 d = ld_stream(x + i + 3 * stride);
    m2 = absmax2(m2, a.x); m2 = absmax2(m2, a.y); m2 = absmax2(m2, a.z); m2 = absmax2(m2, a.w);
    m2 = absmax2(m2, b.x); m2 = absmax2(m2, b.y); m2 = absmax2(m2, b.z); m2 = absmax2(m2, b.w);
    m2 = absmax2(m2, c.x); m2 = absmax2(m2, c.y); m2 = absmax2(m2, c.z); m2 = absmax2(m2, c.w);
    m2 = absmax2(m2, d.x); m2 = absmax2(m2, d.y); m2 = absmax2(m2, d.z); m2 = absmax2(m2, d.w);
  }
  for (; i < n_vec; i += stride) {
    const uint4 a = ld_stream(x + i);
    m2 = absmax2(m2, a.x); m2 = absmax2(m2, a.y); m2 = absmax2(m2, a.z); m2 = absmax2(m2, a.w);
  }
  if (blockIdx.x == 0 && threadIdx.x < n_tail) m2 = __vmaxu2(m2, static_cast<uint32_t>(tail[threadIdx.x] & 0x7FFFu));
  block_amax_commit(m2, amax_bits);
}

// Any alignment: one element per thread per step.
__global__ void __launch_bounds__(kThreads) amax_scalar_kernel(const uint16_t* __restrict__ x, int64_t n,
                                                               unsigned int* amax_bits) {
  uint32_t m2 = 0;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * kThreads)
    m2 = max(m2, static_cast<uint32_t>(x[i] & 0x7FFFu));
  block_amax_commit(m2, amax_bits);
}

// Converts two products that are known not to be special (plain satfinite RNE).
__device__ __forceinline__ uint32_t cvt2_plain(float p0, float p1, int fmt) {
  const __nv_fp8_interpretation_t kind = fmt == UFP8_E4M3 ? __NV_E4M3 : __NV_E5M2;
  return static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(make_float2(p0, p1), __NV_SATFINITE, kind));
}

__device__ __forceinline__ uint32_t quant_word_plain(uint32_t w, float s, int fmt) {
  return cvt2_plain(__fmul_rn(bf16lo(w), s), __fmul_rn(bf16hi(w), s), fmt);
}

// Largest sign-cleared bf16 pattern b with fl(bf16(b) * s) not special, or -1 if none.
// fl(x * s) is monotonic in |x| for s >= 0, so a group whose largest |x| is at or below this
// bound contains no special product.  s that is NaN, inf or negative makes every group take
// the exact per-element path.
__device__ __forceinline__ int special_free_bound(float s, int fmt) {
  if (!(s >= 0.0f) || isinf(s)) return -1;
  int lo = 0, hi = 0x7F80;  // 0x7F80 = +inf
  if (is_special(__fmul_rn(__uint_as_float(0u), s), fmt)) return -1;
  while (hi - lo > 1) {  // invariant: lo not special, hi special (inf * s >= inf for s > 0)
    const int mid = (lo + hi) >> 1;
    if (is_special(__fmul_rn(__uint_as_float(static_cast<uint32_t>(mid) << 16), s), fmt))
      hi = mid;
    else
      lo = mid;
  }
  return s == 0.0f ? 0x7F7F : lo;  // s == 0: every finite x gives 0
}

__device__ __forceinline__ uint32_t absmax16(uint32_t m, const uint4& v) {
  m = __vmaxu2(m, v.x & 0x7FFF7FFFu);
  m = __vmaxu2(m, v.y & 0x7FFF7FFFu);
  m = __vmaxu2(m, v.z & 0x7FFF7FFFu);
  return __vmaxu2(m, v.w & 0x7FFF7FFFu);
}

// Vector body: 32 bf16 (four 16-byte loads, all in flight before any use) -> 32 fp8 (two
// 16-byte stores) per step; a last odd group of 16 and the < 16-element tail follow.
// A null `amax` means a unit scale (plain cast); a null `inv_scale` is not written.
__device__ __forceinline__ uint4 quant16(const uint4& a, const uint4& b, float s, int fmt) {
  uint4 o;
  o.x = quant_4bytes(a.x, a.y, s, fmt);
  o.y = quant_4bytes(a.z, a.w, s, fmt);
  o.z = quant_4bytes(b.x, b.y, s, fmt);
  o.w = quant_4bytes(b.z, b.w, s, fmt);
  return o;
}

__device__ __forceinline__ uint4 quant16_plain(const uint4& a, const uint4& b, float s, int fmt) {
  uint4 o;
  o.x = quant_word_plain(a.x, s, fmt) | (quant_word_plain(a.y, s, fmt) << 16);
  o.y = quant_word_plain(a.z, s, fmt) | (quant_word_plain(a.w, s, fmt) << 16);
  o.z = quant_word_plain(b.x, s, fmt) | (quant_word_plain(b.y, s, fmt) << 16);
  o.w = quant_word_plain(b.z, s, fmt) | (quant_word_plain(b.w, s, fmt) << 16);
  return o;
}

__global__ void __launch_bounds__(kThreads) quant_vec_kernel(const uint4* __restrict__ x, int64_t n_vec16,
                                                             const uint16_t* __restrict__ x_tail,
                                                             uint8_t* __restrict__ q_tail, int n_tail,
                                                             int fmt, const float* __restrict__ amax,
                                                             uint4* __restrict__ q, float* __restrict__ inv_scale) {
  const float s = amax ? scale_from_amax(*amax, fmt) : 1.0f;
  if (inv_scale && blockIdx.x == 0 && threadIdx.x == 0) *inv_scale = __fdiv_rn(1.0f, s);
  // The bound depends only on s: one thread searches it, the CTA shares it.
  __shared__ int bound_s;
  if (threadIdx.x == 0) bound_s = special_free_bound(s, fmt);
  __syncthreads();
  const int bound = bound_s;
  const uint32_t bound2 = bound < 0 ? 0u : (static_cast<uint32_t>(bound) * 0x00010001u);
  const int64_t n_vec32 = n_vec16 / 2;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  // Software-pipelined: the next step's four 16-byte loads leave before this step's 32 values
  // are converted and stored, so each thread keeps loads in flight through its compute.
  int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  uint4 a0, b0, a1, b1;
  if (i < n_vec32) {
    a0 = ld_stream(x + 4 * i);
    b0 = ld_stream(x + 4 * i + 1);
    a1 = ld_stream(x + 4 * i + 2);
    b1 = ld_stream(x + 4 * i + 3);
  }
  for (; i < n_vec32; i += stride) {
    const int64_t nx = i + stride;
    uint4 c0 = make_uint4(0u, 0u, 0u, 0u), d0 = c0, c1 = c0, d1 = c0;
    if (nx < n_vec32) {
      c0 = ld_stream(x + 4 * nx);
      d0 = ld_stream(x + 4 * nx + 1);
      c1 = ld_stream(x + 4 * nx + 2);
      d1 = ld_stream(x + 4 * nx + 3);
    }
    const uint32_t m = absmax16(absmax16(absmax16(absmax16(0u, a0), b0), a1), b1);
    // both 16-bit lanes of m at or below the bound: no special product in these 32
    if (bound >= 0 && __vcmpleu2(m, bound2) == 0xFFFFFFFFu) {
      q[2 * i] = quant16_plain(a0, b0, s, fmt);
      q[2 * i + 1] = quant16_plain(a1, b1, s, fmt);
    } else {
      q[2 * i] = quant16(a0, b0, s, fmt);
      q[2 * i + 1] = quant16(a1, b1, s, fmt);
    }
    a0 = c0;
    b0 = d0;
    a1 = c1;
    b1 = d1;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0 && (n_vec16 & 1)) {
    const int64_t j = n_vec16 - 1;
    q[j] = quant16(ld_stream(x + 2 * j), ld_stream(x + 2 * j + 1), s, fmt);
  }
  if (blockIdx.x == 0 && threadIdx.x < n_tail) {
    const float p = __fmul_rn(__uint_as_float(static_cast<uint32_t>(x_tail[threadIdx.x]) << 16), s);
    q_tail[threadIdx.x] = static_cast<uint8_t>(cvt2(p, 0.0f, fmt) & 0xFFu);
  }
}

__global__ void __launch_bounds__(kThreads) quant_scalar_kernel(const uint16_t* __restrict__ x, int64_t n, int fmt,
                                                                const float* __restrict__ amax,
                                                                uint8_t* __restrict__ q,
                                                                float* __restrict__ inv_scale) {
  const float s = amax ? scale_from_amax(*amax, fmt) : 1.0f;
  if (inv_scale && blockIdx.x == 0 && threadIdx.x == 0) *inv_scale = __fdiv_rn(1.0f, s);
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const float p = __fmul_rn(__uint_as_float(static_cast<uint32_t>(x[i]) << 16), s);
    q[i] = static_cast<uint8_t>(cvt2(p, 0.0f, fmt) & 0xFFu);
  }
}

int grid_for(int64_t work_items, const DeviceInfo& dev) {
  const int64_t want = (work_items + kThreads - 1) / kThreads;
  const int64_t cap = static_cast<int64_t>(dev.sm_count) * kCtasPerSm;
  return static_cast<int>(want < 1 ? 1 : (want < cap ? want : cap));
}

}  // namespace

int launch_amax(const void* x, int64_t n, float* amax, cudaStream_t s, const DeviceInfo& dev) {
  cudaError_t e = cudaMemsetAsync(amax, 0, sizeof(float), s);
  if (e != cudaSuccess) return cuda_error(e, "cudaMemsetAsync(amax)");
  if (n == 0) return UFP8_OK;
  unsigned int* bits = reinterpret_cast<unsigned int*>(amax);
  if ((reinterpret_cast<uintptr_t>(x) & 15u) == 0) {
    const int64_t n_vec = n / 8;
    const int n_tail = static_cast<int>(n - n_vec * 8);
    const uint16_t* tail = static_cast<const uint16_t*>(x) + n_vec * 8;
    amax_vec_kernel<<<grid_for((n_vec + 3) / 4, dev), kThreads, 0, s>>>(static_cast<const uint4*>(x), n_vec, tail,
                                                                       n_tail, bits);
  } else {
    amax_scalar_kernel<<<grid_for(n, dev), kThreads, 0, s>>>(static_cast<const uint16_t*>(x), n, bits);
  }
  e = cudaGetLastError();
  return e == cudaSuccess ? UFP8_OK : cuda_error(e, "amax kernel launch");
}

int launch_quantize(const void* x, int64_t n, int fmt, const float* amax, void* q, float* inv_scale,
                    cudaStream_t s, const DeviceInfo& dev) {
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(q)) & 15u) == 0;
  if (aligned) {
    const int64_t n_vec16 = n / 16;
    const int n_tail = static_cast<int>(n - n_vec16 * 16);
    quant_vec_kernel<<<grid_for((n_vec16 + 1) / 2, dev), kThreads, 0, s>>>(
        static_cast<const uint4*>(x), n_vec16, static_cast<const uint16_t*>(x) + n_vec16 * 16,
        static_cast<uint8_t*>(q) + n_vec16 * 16, n_tail, fmt, amax, static_cast<uint4*>(q), inv_scale);
  } else {
    quant_scalar_kernel<<<grid_for(n, dev), kThreads, 0, s>>>(static_cast<const uint16_t*>(x), n, fmt, amax,
                                                              static_cast<uint8_t*>(q), inv_scale);
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? UFP8_OK : cuda_error(e, "quantize kernel launch");
}

}  // namespace ufp8
