// Next-token cross-entropy on the lm_head's bf16 logits: the loss of the reference's
// chunked_softmax_cross_entropy (ueaj/opt/next_token_loss.py:99-174), which applies
// optax.softmax_cross_entropy_with_integer_labels to each chunk's logits and multiplies the
// result by the loss mask, and the derivative JAX takes of it.
//
//   xent_rows_kernel     one CTA per row streams the row's V logits once (16-byte loads, four in
//                        flight per thread) with a running (max, sum exp) per thread; the CTA
//                        merges the 256 partials in a fixed order.  HBM-bound: 2 B per element.
//   xent_combine_kernel  one warp per row merges the 128-column partials that a GEMM with the
//                        UFP8_EPI_XENT epilogue wrote, so the forward never re-reads the logits.
//   xent_amax_kernel     the backward's per-tensor fp8 scale, from the per-row results alone:
//                        max |dl| over a row is |g| * (1 - softmax[label]) (the label column).
//   xent_grad_kernel     one streaming pass logits -> dlogits (bf16 read, fp8 or bf16 written) by a
//                        resident grid walking (row, 8192-column) units.
//
// All arithmetic is f32.  Partials merge as (m, s) + (m', s') = (M, s e^(m-M) + s' e^(m'-M)),
// M = max(m, m'); every merge order is fixed, so results do not depend on scheduling.  exp is the
// MUFU approximation (__expf, a few ulp) in the sums.  A softmax value is
// p = 2^fma(c, log2 e, -lse * log2 e) (one FMA and the MUFU ex2.approx), and the same expression
// gives softmax[label] in the forward (qrow) and in the backward, so the fp8 amax is exactly the
// largest |dl|.
#include <cuda_bf16.h>

#include <cmath>

#include "fp8cast.cuh"
#include "internal.h"

namespace ufp8 {
namespace {

constexpr int kXThreads = 256;
constexpr int kXWarps = kXThreads / 32;
constexpr int kXUnits = 4;                       // 8-column units per thread in the backward
constexpr int kXCols = kXThreads * kXUnits * 8;  // columns per backward CTA
constexpr int kXAmaxThreads = 1024;

struct XentArgs {
  const uint16_t* logits;
  int64_t ldl, rows, V;
  const int32_t* labels;
  const uint8_t* mask;
  // forward outputs
  float* lse;
  float* loss;
  float* qrow;
  // combine input
  const float* stats;
  int64_t ld_stats, groups;
  // backward
  const float* lse_in;
  const float* qrow_in;
  const float* dloss;
  int cap_on;
  float inv_cap;
  int fmt;
  void* out;
  int64_t ldo;
  float* amax;
  float* inv_scale;
  int64_t ctas_per_row;
  int vec;
};

__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ float bf(uint32_t bits16) { return __uint_as_float(bits16 << 16); }
__device__ __forceinline__ float wlo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float whi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// softmax value of logit c in a row with -lse * log2 e = nl2
__device__ __forceinline__ float softmax_p(float c, float nl2) { return ex2_approx(__fmaf_rn(c, kLog2e, nl2)); }

// Column of a label: negative labels count from the end; outside [-V, V): none (-1).
__device__ __forceinline__ int64_t label_col(int32_t lab, int64_t V) {
  int64_t l = lab;
  if (l < 0) l += V;
  return (l >= 0 && l < V) ? l : -1;
}

// (m, s) <- (m, s) + (m2, s2).  m is never NaN (fmaxf skips NaN values); a NaN logit reaches s.
__device__ __forceinline__ void merge(float& m, float& s, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  if (mn == -INFINITY) return;  // both empty
  s = s * __expf(m - mn) + s2 * __expf(m2 - mn);
  m = mn;
}

__device__ __forceinline__ void fold1(float x, float& m, float& s) {
  if (x > m) {
    s *= __expf(m - x);
    m = x;
  }
  s += __expf(x - m);
}

// Eight bf16 logits (one 16-byte word) into the running partials.
__device__ __forceinline__ void fold8(const uint4 w, float& m, float& s) {
  const float v[8] = {wlo(w.x), whi(w.x), wlo(w.y), whi(w.y), wlo(w.z), whi(w.z), wlo(w.w), whi(w.w)};
  const float cm = fmaxf(fmaxf(fmaxf(v[0], v[1]), fmaxf(v[2], v[3])), fmaxf(fmaxf(v[4], v[5]), fmaxf(v[6], v[7])));
  if (cm > m) {
    s *= __expf(m - cm);
    m = cm;
  }
  float acc = 0.0f;
#pragma unroll
  for (int j = 0; j < 8; ++j) acc += __expf(v[j] - m);
  s += acc;
}

__device__ __forceinline__ void warp_merge(float& m, float& s) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float m2 = __shfl_xor_sync(0xFFFFFFFFu, m, off);
    const float s2 = __shfl_xor_sync(0xFFFFFFFFu, s, off);
    merge(m, s, m2, s2);  // commutative bit for bit, so every lane ends with the same pair
  }
}

// Per-row results from the row's merged partials (M, S): lse, masked loss and qrow.
__device__ __forceinline__ void finish_row(const XentArgs& a, int64_t row, float M, float S) {
  const float lse = __fadd_rn(M, logf(S));
  const int64_t col = label_col(a.labels[row], a.V);
  const float cl = col >= 0 ? bf(a.logits[row * a.ldl + col]) : __int_as_float(0x7FC00000);
  const float mk = a.mask ? static_cast<float>(a.mask[row]) : 1.0f;
  a.lse[row] = lse;
  a.loss[row] = __fmul_rn(__fsub_rn(lse, cl), mk);
  a.qrow[row] = col >= 0 ? __fsub_rn(1.0f, softmax_p(cl, __fmul_rn(lse, -kLog2e))) : 1.0f;
}

__global__ void __launch_bounds__(kXThreads) xent_rows_kernel(const XentArgs a) {
  const int64_t row = blockIdx.x;
  const uint16_t* lr = a.logits + row * a.ldl;
  float m = -INFINITY, s = 0.0f;
  int64_t tail0 = 0;
  if (a.vec) {
    const int64_t nv = a.V >> 3;
    const uint4* p = reinterpret_cast<const uint4*>(lr);
    int64_t i = threadIdx.x;
    for (; i + 3 * kXThreads < nv; i += 4 * kXThreads) {
      const uint4 w0 = ld_stream16(p + i);
      const uint4 w1 = ld_stream16(p + i + kXThreads);
      const uint4 w2 = ld_stream16(p + i + 2 * kXThreads);
      const uint4 w3 = ld_stream16(p + i + 3 * kXThreads);
      fold8(w0, m, s);
      fold8(w1, m, s);
      fold8(w2, m, s);
      fold8(w3, m, s);
    }
    for (; i < nv; i += kXThreads) fold8(ld_stream16(p + i), m, s);
    tail0 = nv << 3;
  }
  for (int64_t j = tail0 + threadIdx.x; j < a.V; j += kXThreads) fold1(bf(lr[j]), m, s);
  warp_merge(m, s);
  __shared__ float sm[kXWarps], ss[kXWarps];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sm[warp] = m;
    ss[warp] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = sm[0], S = ss[0];
    for (int w = 1; w < kXWarps; ++w) merge(M, S, sm[w], ss[w]);
    finish_row(a, row, M, S);
  }
}

__global__ void __launch_bounds__(kXThreads) xent_combine_kernel(const XentArgs a) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kXWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= a.rows) return;
  const float2* st = reinterpret_cast<const float2*>(a.stats) + row * a.ld_stats;
  float m = -INFINITY, s = 0.0f;
  for (int64_t g = lane; g < a.groups; g += 32) {
    const float2 v = st[g];
    merge(m, s, v.x, v.y);
  }
  warp_merge(m, s);
  if (lane == 0) finish_row(a, row, m, s);
}

// amax = max_r |dloss_r * mask_r| * qrow_r as an unsigned max over the f32 bit patterns (all
// values are >= 0; a NaN is above +inf), then s and inv_scale as the quantize kernel derives them.
__global__ void __launch_bounds__(kXAmaxThreads) xent_amax_kernel(const XentArgs a) {
  uint32_t mb = 0;
  for (int64_t r = threadIdx.x; r < a.rows; r += kXAmaxThreads) {
    const float g = a.dloss ? a.dloss[r] : 1.0f;
    const float mk = a.mask ? static_cast<float>(a.mask[r]) : 1.0f;
    const float v = __fmul_rn(fabsf(__fmul_rn(g, mk)), a.qrow_in[r]);
    mb = max(mb, __float_as_uint(v) & 0x7FFFFFFFu);
  }
  mb = __reduce_max_sync(0xFFFFFFFFu, mb);
  __shared__ uint32_t wm[kXAmaxThreads / 32];
  if ((threadIdx.x & 31) == 0) wm[threadIdx.x >> 5] = mb;
  __syncthreads();
  if (threadIdx.x < 32) {
    uint32_t v = wm[threadIdx.x];
    v = __reduce_max_sync(0xFFFFFFFFu, v);
    if (threadIdx.x == 0) {
      const float amax = __uint_as_float(v);
      *a.amax = amax;
      *a.inv_scale = __fdiv_rn(1.0f, scale_from_amax(amax, a.fmt));
    }
  }
}

// dl of one logit c, times the row's output factor wr (g for a bf16 gradient, g * s for fp8):
// v = (p - [label]) * wr, then v * (1 - (c / cap)^2) with the soft cap.
__device__ __forceinline__ float xent_dl(float c, bool is_label, float nl2, float wr, int cap_on, float inv_cap) {
  const float p = softmax_p(c, nl2);
  float v = __fmul_rn(is_label ? __fsub_rn(p, 1.0f) : p, wr);
  if (cap_on) {
    const float t = __fmul_rn(c, inv_cap);
    v = __fmul_rn(v, __fsub_rn(1.0f, __fmul_rn(t, t)));
  }
  return v;
}

// Eight scaled gradient values -> eight fp8 bytes.  The hardware conversion rounds like the
// cast except for NaN, infinities and magnitudes past the overflow threshold (fp8cast.cuh), and
// no finite value here gets there: every |dl| of a row is at most |g| * qrow (the label column
// holds the row's largest |softmax - onehot|), so |dl * s| <= FMAX up to rounding, far below the
// threshold (61440 for e5m2, 464 for e4m3).  So one finiteness test of the eight values' sum (a
// NaN or an infinity makes it non-finite) decides whether the re-encoding of cvt2 is needed.
__device__ __forceinline__ uint2 cvt8(const float (&p)[8], int fmt) {
  const float sum = ((p[0] + p[1]) + (p[2] + p[3])) + ((p[4] + p[5]) + (p[6] + p[7]));
  uint32_t w[4];
  if (isfinite(sum)) {
    const __nv_fp8_interpretation_t kind = fmt == UFP8_E4M3 ? __NV_E4M3 : __NV_E5M2;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      w[i] = static_cast<uint32_t>(
          __nv_cvt_float2_to_fp8x2(make_float2(p[2 * i], p[2 * i + 1]), __NV_SATFINITE, kind));
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = cvt2(p[2 * i], p[2 * i + 1], fmt);
  }
  return make_uint2(w[0] | (w[1] << 16), w[2] | (w[3] << 16));
}

// Work unit = kXCols columns of one row; a resident grid walks the units in row-major order,
// advancing (row, chunk) by gridDim.x units without a division, and issues the 16-byte loads of
// its next unit before computing the current one.  Vector units of 8 columns (a 16-byte load, an
// 8-byte fp8 or 16-byte bf16 store) where the unit lies inside the row, element by element
// otherwise.  Per element: p = softmax_p(c), minus 1 in the one unit of the row that holds the
// label, times the row factor, times the soft cap's derivative.
template <bool kFp8>
__device__ __forceinline__ void xent_grad_unit(const XentArgs& a, int64_t row, int ch, float sc,
                                               const uint4 (&w)[kXUnits]) {
  const int c0 = ch * kXCols;
  const int V = static_cast<int>(a.V);
  const uint16_t* lr = a.logits + row * a.ldl;
  uint8_t* q8 = static_cast<uint8_t*>(a.out) + row * a.ldo;     // kFp8
  uint16_t* q16 = static_cast<uint16_t*>(a.out) + row * a.ldo;  // !kFp8
  const float nl2 = __fmul_rn(a.lse_in[row], -kLog2e);
  const float g = a.dloss ? a.dloss[row] : 1.0f;
  const float mk = a.mask ? static_cast<float>(a.mask[row]) : 1.0f;
  const float ge = __fmul_rn(g, mk);
  const float wr = kFp8 ? __fmul_rn(ge, sc) : ge;
  const int lab = static_cast<int>(label_col(a.labels[row], a.V));  // -1: no column
  auto put1 = [&](int cc, float v) {
    if (kFp8)
      q8[cc] = static_cast<uint8_t>(cvt2(v, 0.0f, a.fmt) & 0xFFu);
    else
      q16[cc] = __bfloat16_as_ushort(__float2bfloat16_rn(v));
  };
  if (!a.vec) {
    for (int i = 0; i < kXCols / kXThreads; ++i) {
      const int cc = c0 + i * kXThreads + static_cast<int>(threadIdx.x);
      if (cc < V) put1(cc, xent_dl(bf(lr[cc]), cc == lab, nl2, wr, a.cap_on, a.inv_cap));
    }
    return;
  }
#pragma unroll
  for (int k = 0; k < kXUnits; ++k) {
    const int col = c0 + (k * kXThreads + static_cast<int>(threadIdx.x)) * 8;
    if (col + 8 <= V) {
      const float c[8] = {wlo(w[k].x), whi(w[k].x), wlo(w[k].y), whi(w[k].y),
                          wlo(w[k].z), whi(w[k].z), wlo(w[k].w), whi(w[k].w)};
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = softmax_p(c[j], nl2);
      const unsigned rel = static_cast<unsigned>(lab - col);
      if (rel < 8u) {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (static_cast<unsigned>(j) == rel) v[j] = __fsub_rn(v[j], 1.0f);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = __fmul_rn(v[j], wr);
      if (a.cap_on) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float t = __fmul_rn(c[j], a.inv_cap);
          v[j] = __fmul_rn(v[j], __fsub_rn(1.0f, __fmul_rn(t, t)));
        }
      }
      if (kFp8) {
        *reinterpret_cast<uint2*>(q8 + col) = cvt8(v, a.fmt);
      } else {
        uint4 o;
        uint32_t* ow = &o.x;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const __nv_bfloat162 b = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
          ow[j] = *reinterpret_cast<const uint32_t*>(&b);
        }
        *reinterpret_cast<uint4*>(q16 + col) = o;
      }
    } else {
      for (int cc = col; cc < V && cc < col + 8; ++cc)
        put1(cc, xent_dl(bf(lr[cc]), cc == lab, nl2, wr, a.cap_on, a.inv_cap));
    }
  }
}

__device__ __forceinline__ void xent_grad_load(const XentArgs& a, int64_t row, int ch, uint4 (&w)[kXUnits]) {
  const int V = static_cast<int>(a.V);
  const uint16_t* lr = a.logits + row * a.ldl;
#pragma unroll
  for (int k = 0; k < kXUnits; ++k) {
    const int col = ch * kXCols + (k * kXThreads + static_cast<int>(threadIdx.x)) * 8;
    w[k] = col + 8 <= V ? ld_stream16(lr + col) : make_uint4(0, 0, 0, 0);
  }
}

template <bool kFp8>
__global__ void __launch_bounds__(kXThreads) xent_grad_kernel(const XentArgs a) {
  const float sc = kFp8 ? scale_from_amax(*a.amax, a.fmt) : 1.0f;
  const int cpr = static_cast<int>(a.ctas_per_row);
  if (static_cast<int64_t>(blockIdx.x) >= a.rows * cpr) return;
  int64_t row = blockIdx.x / cpr;
  int ch = static_cast<int>(blockIdx.x - row * cpr);
  const int64_t step_r = gridDim.x / cpr;
  const int step_c = static_cast<int>(gridDim.x % cpr);
  uint4 w[kXUnits], wn[kXUnits];
  if (a.vec) xent_grad_load(a, row, ch, w);
  while (true) {
    int64_t rn = row + step_r;
    int chn = ch + step_c;
    if (chn >= cpr) {
      chn -= cpr;
      ++rn;
    }
    const bool more = rn < a.rows;
    if (a.vec && more) xent_grad_load(a, rn, chn, wn);
    xent_grad_unit<kFp8>(a, row, ch, sc, w);
    if (!more) break;
    row = rn;
    ch = chn;
#pragma unroll
    for (int k = 0; k < kXUnits; ++k) w[k] = wn[k];
  }
}

// Resident CTAs of a kernel on this device (cached per device and kernel).
int resident_ctas(const void* fn, const DeviceInfo& dev, int slot, int64_t* out) {
  static thread_local int dev_of[2] = {-1, -1}, per_sm[2] = {0, 0};
  if (dev_of[slot] != dev.device) {
    int n = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, kXThreads, 0);
    if (e != cudaSuccess) return cuda_error(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor(xent)");
    per_sm[slot] = n < 1 ? 1 : n;
    dev_of[slot] = dev.device;
  }
  *out = static_cast<int64_t>(dev.sm_count) * per_sm[slot];
  return UFP8_OK;
}

bool al(const void* p, uintptr_t n) { return (reinterpret_cast<uintptr_t>(p) & (n - 1)) == 0; }

int xent_check(const void* logits, int64_t rows, int64_t V, int64_t ldl, const int32_t* labels, const char* who) {
  if (rows < 0 || V < 1) return set_error(UFP8_ERR_INVALID, "%s: rows must be >= 0 and V >= 1", who);
  if (ldl < V) return set_error(UFP8_ERR_INVALID, "%s: ldl < V", who);
  if (rows >= (int64_t(1) << 31)) return set_error(UFP8_ERR_INVALID, "%s: rows exceed 2^31", who);
  if (rows > 0 && (!logits || !labels)) return set_error(UFP8_ERR_INVALID, "%s: null logits or labels", who);
  if (!al(logits, 2)) return set_error(UFP8_ERR_ALIGN, "%s: logits not 2-byte aligned", who);
  return UFP8_OK;
}

}  // namespace
}  // namespace ufp8

using namespace ufp8;

extern "C" int ufp8_xent_forward(const void* logits_bf16, int64_t rows, int64_t V, int64_t ldl,
                                 const int32_t* labels, const uint8_t* mask, float* lse, float* loss, float* qrow,
                                 ufp8_stream_t stream) {
  if (int rc = xent_check(logits_bf16, rows, V, ldl, labels, "ufp8_xent_forward")) return rc;
  if (rows > 0 && (!lse || !loss || !qrow)) return set_error(UFP8_ERR_INVALID, "ufp8_xent_forward: null output");
  if (rows == 0) return UFP8_OK;
  DeviceInfo* dev;
  if (int rc = device_info(&dev)) return rc;
  XentArgs a{};
  a.logits = static_cast<const uint16_t*>(logits_bf16);
  a.ldl = ldl;
  a.rows = rows;
  a.V = V;
  a.labels = labels;
  a.mask = mask;
  a.lse = lse;
  a.loss = loss;
  a.qrow = qrow;
  a.vec = al(logits_bf16, 16) && ldl % 8 == 0;
  xent_rows_kernel<<<static_cast<unsigned>(rows), kXThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? UFP8_OK : cuda_error(e, "xent forward launch");
}

extern "C" int ufp8_xent_combine(const float* stats, int64_t ld_stats, const void* logits_bf16, int64_t rows,
                                 int64_t V, int64_t ldl, const int32_t* labels, const uint8_t* mask, float* lse,
                                 float* loss, float* qrow, ufp8_stream_t stream) {
  if (int rc = xent_check(logits_bf16, rows, V, ldl, labels, "ufp8_xent_combine")) return rc;
  const int64_t groups = (V + 127) / 128;
  if (ld_stats < groups) return set_error(UFP8_ERR_INVALID, "ufp8_xent_combine: ld_stats < ceil(V / 128)");
  if (rows > 0 && (!stats || !lse || !loss || !qrow))
    return set_error(UFP8_ERR_INVALID, "ufp8_xent_combine: null stats or output");
  if (!al(stats, 8)) return set_error(UFP8_ERR_ALIGN, "ufp8_xent_combine: stats not 8-byte aligned");
  if (rows == 0) return UFP8_OK;
  DeviceInfo* dev;
  if (int rc = device_info(&dev)) return rc;
  XentArgs a{};
  a.logits = static_cast<const uint16_t*>(logits_bf16);
  a.ldl = ldl;
  a.rows = rows;
  a.V = V;
  a.labels = labels;
  a.mask = mask;
  a.lse = lse;
  a.loss = loss;
  a.qrow = qrow;
  a.stats = stats;
  a.ld_stats = ld_stats;
  a.groups = groups;
  const unsigned grid = static_cast<unsigned>((rows + kXWarps - 1) / kXWarps);
  xent_combine_kernel<<<grid, kXThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? UFP8_OK : cuda_error(e, "xent combine launch");
}

extern "C" int ufp8_xent_backward(const void* logits_bf16, int64_t rows, int64_t V, int64_t ldl,
                                  const int32_t* labels, const uint8_t* mask, const float* lse, const float* qrow,
                                  const float* dloss, float cap, int fmt, void* dlogits, int64_t ldo, float* amax,
                                  float* inv_scale, ufp8_stream_t stream) {
  if (int rc = xent_check(logits_bf16, rows, V, ldl, labels, "ufp8_xent_backward")) return rc;
  const bool fp8 = fmt == UFP8_E4M3 || fmt == UFP8_E5M2;
  if (!fp8 && fmt != UFP8_BF16)
    return set_error(UFP8_ERR_INVALID, "ufp8_xent_backward: fmt %d is not UFP8_E4M3/UFP8_E5M2/UFP8_BF16", fmt);
  if (!(cap >= 0.0f) || std::isinf(cap))
    return set_error(UFP8_ERR_INVALID, "ufp8_xent_backward: cap must be 0 or a finite positive value");
  if (ldo < V) return set_error(UFP8_ERR_INVALID, "ufp8_xent_backward: ldo < V");
  if (rows > 0 && (!lse || !dlogits || (fp8 && !qrow)))
    return set_error(UFP8_ERR_INVALID, "ufp8_xent_backward: null lse, qrow or dlogits");
  if (fp8 && (!amax || !inv_scale)) return set_error(UFP8_ERR_INVALID, "ufp8_xent_backward: null amax or inv_scale");
  if (!fp8 && !al(dlogits, 2)) return set_error(UFP8_ERR_ALIGN, "ufp8_xent_backward: dlogits not 2-byte aligned");
  if (V >= (int64_t(1) << 31) - kXCols) return set_error(UFP8_ERR_INVALID, "ufp8_xent_backward: V exceeds 2^31");
  const int64_t cpr = (V + kXCols - 1) / kXCols;
  DeviceInfo* dev;
  if (int rc = device_info(&dev)) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  XentArgs a{};
  a.logits = static_cast<const uint16_t*>(logits_bf16);
  a.ldl = ldl;
  a.rows = rows;
  a.V = V;
  a.labels = labels;
  a.mask = mask;
  a.lse_in = lse;
  a.qrow_in = qrow;
  a.dloss = dloss;
  a.cap_on = cap > 0.0f;
  a.inv_cap = cap > 0.0f ? 1.0f / cap : 0.0f;
  a.fmt = fmt;
  a.out = dlogits;
  a.ldo = ldo;
  a.amax = amax;
  a.inv_scale = inv_scale;
  a.ctas_per_row = cpr;
  a.vec = al(logits_bf16, 16) && ldl % 8 == 0 && ldo % 8 == 0 && al(dlogits, fp8 ? 8 : 16);
  if (fp8) xent_amax_kernel<<<1, kXAmaxThreads, 0, s>>>(a);
  if (rows > 0) {
    const void* fn = fp8 ? reinterpret_cast<const void*>(xent_grad_kernel<true>)
                         : reinterpret_cast<const void*>(xent_grad_kernel<false>);
    int64_t cap_ctas = 0;
    if (int rc = resident_ctas(fn, *dev, fp8 ? 0 : 1, &cap_ctas)) return rc;
    const unsigned grid = static_cast<unsigned>(rows * cpr < cap_ctas ? rows * cpr : cap_ctas);
    if (fp8)
      xent_grad_kernel<true><<<grid, kXThreads, 0, s>>>(a);
    else
      xent_grad_kernel<false><<<grid, kXThreads, 0, s>>>(a);
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? UFP8_OK : cuda_error(e, "xent backward launch");
}
