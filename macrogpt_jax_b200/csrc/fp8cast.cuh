// Device helpers shared by the quantising kernels (quant.cu, norm.cu): the per-tensor scale
// and the fp8 encoding with the ml_dtypes 0.5.4 cast semantics (see quant.cu's header).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include <cstdint>

#include "../../include/ufp8.h"

namespace ufp8 {
namespace {

__device__ __forceinline__ float fp8_fmax(int fmt) { return fmt == UFP8_E4M3 ? 448.0f : 57344.0f; }

// s = FMAX / amax, capped at the largest finite f32: for amax below FMAX / FLT_MAX (about
// 1.3e-36 for e4m3fn, 1.7e-34 for e5m2; still normal bf16 values) the quotient would be +inf,
// and inf * x would turn every element into a non-finite code (0 * inf into NaN).  With the cap,
// x * s stays finite and below FMAX, and inv_scale = 1 / FLT_MAX = 2^-128 (an f32 subnormal).
// NaN amax keeps s = NaN (NaN propagates into every code, as the unscaled cast would).
__device__ __forceinline__ float scale_from_amax(float amax, int fmt) {
  if (amax == 0.0f) return 1.0f;
  const float s = __fdiv_rn(fp8_fmax(fmt), amax);
  return s > 3.402823466e38f ? 3.402823466e38f : s;  // a NaN s fails the compare and stays NaN
}

// True where the satfinite hardware conversion differs from the non-saturating cast:
// NaN, and magnitudes that round past the largest finite value (e4m3fn: above 464,
// e5m2: 61440 and above, infinities included).
__device__ __forceinline__ bool is_special(float p, int fmt) {
  const float a = fabsf(p);
  return fmt == UFP8_E4M3 ? !(a <= 464.0f) : !(a < 61440.0f);
}

// ml_dtypes encoding of a special product: NaN -> positive NaN pattern, overflow ->
// NaN (e4m3fn, which has no infinity) or inf (e5m2), keeping the sign.
__device__ __forceinline__ uint32_t special_code(float p, int fmt) {
  const uint32_t sign = (__float_as_uint(p) >> 24) & 0x80u;
  if (isnan(p)) return fmt == UFP8_E4M3 ? 0x7Fu : 0x7Eu;
  return (fmt == UFP8_E4M3 ? 0x7Fu : 0x7Cu) | sign;
}

// Converts two products to packed fp8 (first -> low byte).
__device__ __forceinline__ uint32_t cvt2(float p0, float p1, int fmt) {
  const __nv_fp8_interpretation_t kind = fmt == UFP8_E4M3 ? __NV_E4M3 : __NV_E5M2;
  uint32_t v = static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(make_float2(p0, p1), __NV_SATFINITE, kind));
  if (is_special(p0, fmt)) v = (v & 0xFF00u) | special_code(p0, fmt);
  if (is_special(p1, fmt)) v = (v & 0x00FFu) | (special_code(p1, fmt) << 8);
  return v;
}

__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// 2 bf16 (one 32-bit word) -> 2 fp8 bytes.
__device__ __forceinline__ uint32_t quant_word(uint32_t w, float s, int fmt) {
  return cvt2(__fmul_rn(bf16lo(w), s), __fmul_rn(bf16hi(w), s), fmt);
}

__device__ __forceinline__ uint32_t quant_4bytes(uint32_t w0, uint32_t w1, float s, int fmt) {
  return quant_word(w0, s, fmt) | (quant_word(w1, s, fmt) << 16);
}

}  // namespace
}  // namespace ufp8
