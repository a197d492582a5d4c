// RMSNorm (ueaj/model/rmsnorm.py:68-84) fused with the per-tensor fp8 quantisation of its
// output (the FP8 Einsum that follows it quantises exactly that tensor), and its backward.
//
// Forward, per row of d elements (bit-exact with oracle/norm.py):
//   ss  = sum of x_e * x_e in f32, in the fixed order below;
//   r   = 1 / sqrt(ss / d + eps)            (IEEE division, square root and division);
//   y_e = bf16((x_e * r) * w_e)             w = scale ("uncentered"), 1 + scale ("centered"),
//                                           1 (no scale); a one-element scale broadcasts;
// then the per-tensor recipe on y: amax = max |y| (bf16 bit patterns), s = FMAX / amax (capped
// at FLT_MAX), q = fp8(f32(y) * s), inv_scale = 1 / s.
// Fixed summation order: lane l of the row's warp accumulates, in increasing index order, the
// elements of the 8-element chunks c with c % 32 == l (each product and each sum rounded on its
// own, no fused multiply-add); the 32 lane sums are then combined by an xor butterfly over the
// offsets 16, 8, 4, 2, 1, which leaves the same value in every lane.
//
// Launches: norm_stats_kernel (a warp per row: r, amax over y, y itself when asked for) ->
// norm_quant_kernel (a warp per row: y again from x and r, quantised).  HBM traffic is 5 B per
// element (x read twice, fp8 written once) against 9 B for the three passes norm -> amax ->
// quantize.
//
// Backward (the derivative JAX takes of the forward above, in f32):
//   a     = sum_e g_e * w_e * x_e                 (per row, fixed block order)
//   dx_e  = bf16((r * w_e) * g_e - x_e * (r^3 * a / d))
//   dw_e  = sum over rows of (g_e * x_e) * r      (vector scale; a one-element scale sums all e)
// norm_backward_kernel: persistent CTAs, one row at a time per CTA (thread t owns the chunks
// c == t mod 256), per-CTA dw partials in shared memory (vector scale) or a register (one-element
// scale), written to the caller's workspace and summed over CTAs in CTA order by
// norm_dscale_kernel: deterministic.
#include <cuda_bf16.h>

#include <cstdint>

#include "fp8cast.cuh"
#include "internal.h"

namespace ufp8 {
namespace {

constexpr int kNormRowsPerCta = 8;     // forward: one warp per row
constexpr int kNormBwdThreads = 256;   // backward: one CTA per row
constexpr int kNormMaxChunks = 4;      // backward: at most 4 chunks per thread, so d <= 8 * 256 * 4
constexpr int kNormMaxD = 8 * kNormBwdThreads * kNormMaxChunks;

struct NormArgs {
  const uint16_t* x;
  int64_t ldx;
  int64_t rows;
  int d;
  const uint16_t* scale;  // null: no scale
  int scale_len;          // 1 or d
  int centered;
  float eps;
  int vec;                // rows (x, y, dy, dx) 16-byte aligned and d % 8 == 0
  int vec_scale;          // a vector scale that is 16-byte aligned, d % 8 == 0
  float* rstd;
  unsigned int* amax_bits;
  uint16_t* y;            // optional bf16 output
  int64_t ldy;
  uint8_t* q;             // fp8 output [rows][d]
  int fmt;
  const float* amax;
  float* inv_scale;
  // backward
  const uint16_t* dy;
  int64_t lddy;
  uint16_t* dx;
  int64_t lddx;
  float* ws;              // [gridDim.x][scale_len] (vector) or [gridDim.x][256] (scalar) partials
};

__device__ __forceinline__ float bf(uint32_t bits16) { return __uint_as_float(bits16 << 16); }

// 8 bf16 values of chunk c of a row (zeros past d).
__device__ __forceinline__ void load_chunk(const uint16_t* row, int c, int d, bool vec, float (&v)[8]) {
  const int e0 = c * 8;
  // Read-only loads (__ldg): the compiler may move them ahead of this thread's stores.
  if (vec && e0 + 8 <= d) {
    const uint4 w = __ldg(reinterpret_cast<const uint4*>(row + e0));
    v[0] = bf(w.x & 0xFFFFu); v[1] = bf(w.x >> 16); v[2] = bf(w.y & 0xFFFFu); v[3] = bf(w.y >> 16);
    v[4] = bf(w.z & 0xFFFFu); v[5] = bf(w.z >> 16); v[6] = bf(w.w & 0xFFFFu); v[7] = bf(w.w >> 16);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = e0 + j < d ? bf(__ldg(row + e0 + j)) : 0.0f;
  }
}

// The 8 multipliers of chunk c: scale, 1 + scale, or 1.
__device__ __forceinline__ void load_weight(const NormArgs& a, int c, float (&w)[8]) {
  if (a.scale == nullptr) {
#pragma unroll
    for (int j = 0; j < 8; ++j) w[j] = 1.0f;
    return;
  }
  if (a.scale_len == 1) {
    const float s = bf(a.scale[0]);
    const float m = a.centered ? __fadd_rn(1.0f, s) : s;
#pragma unroll
    for (int j = 0; j < 8; ++j) w[j] = m;
    return;
  }
  load_chunk(a.scale, c, a.d, a.vec_scale != 0, w);
  if (a.centered) {
#pragma unroll
    for (int j = 0; j < 8; ++j) w[j] = __fadd_rn(1.0f, w[j]);
  }
}

__device__ __forceinline__ uint32_t bf16_bits_rn(float v) {
  return static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(v)));
}

__device__ __forceinline__ float finish_rstd(float acc, int d, float eps) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xFFFFFFFFu, acc, o));
  const float var = __fdiv_rn(acc, static_cast<float>(d));
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
}

__device__ __forceinline__ float row_rstd(const NormArgs& a, const uint16_t* xr, int lane) {
  const int nch = (a.d + 7) / 8;
  float acc = 0.0f;
#pragma unroll 4
  for (int c = lane; c < nch; c += 32) {
    float v[8];
    load_chunk(xr, c, a.d, a.vec, v);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc = __fadd_rn(acc, __fmul_rn(v[j], v[j]));
  }
  return finish_rstd(acc, a.d, a.eps);
}

__device__ __forceinline__ void store_y8(const NormArgs& a, int64_t row, int c, const uint32_t (&yb)[8]) {
  uint16_t* yr = a.y + row * a.ldy;
  if (a.vec && c * 8 + 8 <= a.d) {
    *reinterpret_cast<uint4*>(yr + c * 8) = make_uint4(yb[0] | (yb[1] << 16), yb[2] | (yb[3] << 16),
                                                      yb[4] | (yb[5] << 16), yb[6] | (yb[7] << 16));
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (c * 8 + j < a.d) yr[c * 8 + j] = static_cast<uint16_t>(yb[j]);
  }
}

// y bits of chunk c from its x values: bf16((x * r) * w); m = running max |y| (bits).
__device__ __forceinline__ void y_chunk(const NormArgs& a, int c, const float (&v)[8], float r, uint32_t (&yb)[8],
                                        uint32_t& m) {
  float w[8];
  load_weight(a, c, w);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    yb[j] = bf16_bits_rn(__fmul_rn(__fmul_rn(v[j], r), w[j]));
    if (c * 8 + j < a.d) m = max(m, yb[j] & 0x7FFFu);
  }
}

__global__ void __launch_bounds__(32 * kNormRowsPerCta) norm_stats_kernel(const NormArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kNormRowsPerCta + warp;
  uint32_t m = 0;
  if (row < a.rows) {
    const uint16_t* xr = a.x + row * a.ldx;
    const float r = row_rstd(a, xr, lane);
    if (lane == 0) a.rstd[row] = r;
    const int nch = (a.d + 7) / 8;
#pragma unroll 4
    for (int c = lane; c < nch; c += 32) {
      float v[8];
      load_chunk(xr, c, a.d, a.vec, v);
      uint32_t yb[8];
      y_chunk(a, c, v, r, yb, m);
      if (a.y != nullptr) store_y8(a, row, c, yb);
    }
  }
  if (a.amax_bits != nullptr) {
    m = __reduce_max_sync(0xFFFFFFFFu, m);
    __shared__ uint32_t warp_max[kNormRowsPerCta];
    if (lane == 0) warp_max[warp] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t v = 0;
      for (int i = 0; i < kNormRowsPerCta; ++i) v = max(v, warp_max[i]);
      if (v != 0u) atomicMax(a.amax_bits, v << 16);
    }
  }
}

__device__ __forceinline__ void quant_chunk_store(const NormArgs& a, uint8_t* qr, int c, const float (&v)[8], float r,
                                                  float s) {
  float w[8];
  load_weight(a, c, w);
  float p[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) p[j] = __fmul_rn(bf(bf16_bits_rn(__fmul_rn(__fmul_rn(v[j], r), w[j]))), s);
  const uint32_t lo = cvt2(p[0], p[1], a.fmt) | (cvt2(p[2], p[3], a.fmt) << 16);
  const uint32_t hi = cvt2(p[4], p[5], a.fmt) | (cvt2(p[6], p[7], a.fmt) << 16);
  if (a.vec && c * 8 + 8 <= a.d) {
    *reinterpret_cast<uint2*>(qr + c * 8) = make_uint2(lo, hi);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (c * 8 + j < a.d) qr[c * 8 + j] = static_cast<uint8_t>(((j < 4 ? lo : hi) >> (8 * (j & 3))) & 0xFFu);
  }
}

__global__ void __launch_bounds__(32 * kNormRowsPerCta) norm_quant_kernel(const NormArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float s = scale_from_amax(*a.amax, a.fmt);
  if (a.inv_scale && blockIdx.x == 0 && threadIdx.x == 0) *a.inv_scale = __fdiv_rn(1.0f, s);
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kNormRowsPerCta + warp;
  if (row >= a.rows) return;
  const uint16_t* xr = a.x + row * a.ldx;
  uint8_t* qr = a.q + row * static_cast<int64_t>(a.d);
  const float r = a.rstd[row];
  const int nch = (a.d + 7) / 8;
#pragma unroll 4
  for (int c = lane; c < nch; c += 32) {
    float v[8];
    load_chunk(xr, c, a.d, a.vec, v);
    quant_chunk_store(a, qr, c, v, r, s);
  }
}

// Sum over the CTA of one value per thread, in a fixed order (warp butterflies, then the eight
// warp sums in warp order); every thread receives the result.
__device__ __forceinline__ float block_sum_fixed(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < kNormBwdThreads / 32; ++i) s = __fadd_rn(s, red[i]);
  __syncthreads();  // red is reused by the next row
  return s;
}

// Two rows' values per CTA-wide sum, in the fixed order of block_sum_fixed for each.
__device__ __forceinline__ float2 block_sum2_fixed(float2 v, float2* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    v.x = __fadd_rn(v.x, __shfl_xor_sync(0xFFFFFFFFu, v.x, o));
    v.y = __fadd_rn(v.y, __shfl_xor_sync(0xFFFFFFFFu, v.y, o));
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float2 s = make_float2(0.0f, 0.0f);
#pragma unroll
  for (int i = 0; i < kNormBwdThreads / 32; ++i) {
    s.x = __fadd_rn(s.x, red[i].x);
    s.y = __fadd_rn(s.y, red[i].y);
  }
  __syncthreads();
  return s;
}

// Raw 8 bf16 of chunk c (zeros past d), kept packed until used.
__device__ __forceinline__ uint4 load_raw8(const uint16_t* row, int c, int d, bool vec) {
  const int e0 = c * 8;
  if (vec && e0 + 8 <= d) return __ldg(reinterpret_cast<const uint4*>(row + e0));
  uint32_t h[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) h[j] = e0 + j < d ? static_cast<uint32_t>(__ldg(row + e0 + j)) : 0u;
  return make_uint4(h[0] | (h[1] << 16), h[2] | (h[3] << 16), h[4] | (h[5] << 16), h[6] | (h[7] << 16));
}

__device__ __forceinline__ float raw_at(const uint4& w, int j) {
  const uint32_t word = j < 2 ? w.x : (j < 4 ? w.y : (j < 6 ? w.z : w.w));
  return (j & 1) ? bf(word >> 16) : bf(word & 0xFFFFu);
}

// CH = chunks per thread (d <= 8 * 256 * CH).  Each iteration takes two rows (row, row + grid),
// all their loads issued before either row's sum.  A vector scale lives in shared memory next
// to the CTA's dw partials (2 d floats of dynamic shared memory); each thread only touches the
// columns of its own chunks there, so no synchronisation guards them.  The dw partials add the
// rows in increasing row order.
template <int CH>
__global__ void __launch_bounds__(kNormBwdThreads) norm_backward_kernel(const NormArgs a) {
  extern __shared__ float norm_smem[];
  __shared__ float2 red[kNormBwdThreads / 32];
  const int t = threadIdx.x;
  const int nch = (a.d + 7) / 8;
  const bool vscale = a.scale != nullptr && a.scale_len != 1;
  float* ws_w = norm_smem;           // [d] multipliers (vector scale)
  float* ws_dw = norm_smem + a.d;    // [d] dw partials (vector scale)
  float wsc = 1.0f;                  // multiplier (scalar or no scale)
  float dsum = 0.0f;                 // dw partial (scalar scale)
  if (a.scale != nullptr && a.scale_len == 1) {
    const float s = bf(a.scale[0]);
    wsc = a.centered ? __fadd_rn(1.0f, s) : s;
  }
  if (vscale) {
#pragma unroll
    for (int i = 0; i < CH; ++i) {
      const int c = t + i * kNormBwdThreads;
      if (c < nch) {
        float w[8];
        load_weight(a, c, w);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (c * 8 + j < a.d) {
            ws_w[c * 8 + j] = w[j];
            ws_dw[c * 8 + j] = 0.0f;
          }
      }
    }
  }
  const float fd = static_cast<float>(a.d);
  const int64_t step = 2 * static_cast<int64_t>(gridDim.x);
  for (int64_t row0 = blockIdx.x; row0 < a.rows; row0 += step) {
    const int64_t rowv[2] = {row0, row0 + gridDim.x};
    const bool has1 = rowv[1] < a.rows;
    uint4 xr[2][CH], gr[2][CH];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int64_t row = has1 || k == 0 ? rowv[k] : rowv[0];
#pragma unroll
      for (int i = 0; i < CH; ++i) {
        const int c = t + i * kNormBwdThreads;
        xr[k][i] = c < nch ? load_raw8(a.x + row * a.ldx, c, a.d, a.vec) : make_uint4(0u, 0u, 0u, 0u);
        gr[k][i] = c < nch ? load_raw8(a.dy + row * a.lddy, c, a.d, a.vec) : make_uint4(0u, 0u, 0u, 0u);
      }
    }
    float2 part = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int i = 0; i < CH; ++i) {
      const int c = t + i * kNormBwdThreads;
      if (c < nch) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float w = vscale ? ws_w[min(c * 8 + j, a.d - 1)] : wsc;
          part.x = __fadd_rn(part.x, __fmul_rn(__fmul_rn(raw_at(gr[0][i], j), w), raw_at(xr[0][i], j)));
          part.y = __fadd_rn(part.y, __fmul_rn(__fmul_rn(raw_at(gr[1][i], j), w), raw_at(xr[1][i], j)));
        }
      }
    }
    const float2 asum = block_sum2_fixed(part, red);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      if (k == 1 && !has1) break;
      const int64_t row = rowv[k];
      const float r = a.rstd[row];
      const float c1 = __fdiv_rn(__fmul_rn(__fmul_rn(__fmul_rn(r, r), r), k == 0 ? asum.x : asum.y), fd);
      uint16_t* dxr = a.dx + row * a.lddx;
#pragma unroll
      for (int i = 0; i < CH; ++i) {
        const int c = t + i * kNormBwdThreads;
        if (c < nch) {
          uint32_t ob[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int e = min(c * 8 + j, a.d - 1);
            const float w = vscale ? ws_w[e] : wsc;
            const float xv = raw_at(xr[k][i], j), gv = raw_at(gr[k][i], j);
            ob[j] = bf16_bits_rn(__fsub_rn(__fmul_rn(__fmul_rn(r, w), gv), __fmul_rn(xv, c1)));
            const float contrib = __fmul_rn(__fmul_rn(gv, xv), r);
            if (vscale) {
              if (c * 8 + j < a.d) ws_dw[e] = __fadd_rn(ws_dw[e], contrib);
            } else {
              dsum = __fadd_rn(dsum, contrib);  // zeros past d add nothing
            }
          }
          if (a.vec && c * 8 + 8 <= a.d) {
            *reinterpret_cast<uint4*>(dxr + c * 8) = make_uint4(ob[0] | (ob[1] << 16), ob[2] | (ob[3] << 16),
                                                               ob[4] | (ob[5] << 16), ob[6] | (ob[7] << 16));
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j)
              if (c * 8 + j < a.d) dxr[c * 8 + j] = static_cast<uint16_t>(ob[j]);
          }
        }
      }
    }
  }
  if (a.ws == nullptr || a.scale == nullptr) return;
  if (!vscale) {
    a.ws[static_cast<int64_t>(blockIdx.x) * kNormBwdThreads + t] = dsum;
  } else {
    float* wr = a.ws + static_cast<int64_t>(blockIdx.x) * a.d;
#pragma unroll
    for (int i = 0; i < CH; ++i) {
      const int c = t + i * kNormBwdThreads;
      if (c < nch)
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (c * 8 + j < a.d) wr[c * 8 + j] = ws_dw[c * 8 + j];
    }
  }
}

// dscale = sum over the CTAs of their partials, in a fixed order.  Vector scale: a CTA per 32
// columns; thread (g, c) of its 8 x 32 threads sums, in CTA order, the partials of the CTAs
// p == g (mod 8) for column c (coalesced 128-byte rows, 8 independent chains), then the eight
// group sums are added in group order.  One-element scale: one CTA; thread t sums entries t,
// t + 256, ... in order, then the CTA's fixed-order sum.
constexpr int kDsCols = 32;
constexpr int kDsGroups = kNormBwdThreads / kDsCols;

__global__ void __launch_bounds__(kNormBwdThreads) norm_dscale_kernel(const float* __restrict__ ws, int parts,
                                                                       int len, float* __restrict__ dscale) {
  if (len == 1) {
    __shared__ float red[kNormBwdThreads / 32];
    float s = 0.0f;
    for (int i = threadIdx.x; i < parts * kNormBwdThreads; i += kNormBwdThreads) s = __fadd_rn(s, ws[i]);
    s = block_sum_fixed(s, red);
    if (threadIdx.x == 0) dscale[0] = s;
    return;
  }
  __shared__ float grp[kDsGroups][kDsCols];
  const int c = threadIdx.x % kDsCols, gi = threadIdx.x / kDsCols;
  const int e = blockIdx.x * kDsCols + c;
  float s = 0.0f;
  if (e < len) {
#pragma unroll 4
    for (int p = gi; p < parts; p += kDsGroups) s = __fadd_rn(s, __ldg(ws + static_cast<int64_t>(p) * len + e));
  }
  grp[gi][c] = s;
  __syncthreads();
  if (gi == 0 && e < len) {
    float tot = 0.0f;
#pragma unroll
    for (int g = 0; g < kDsGroups; ++g) tot = __fadd_rn(tot, grp[g][c]);
    dscale[e] = tot;
  }
}

int norm_check(const void* x, int64_t rows, int64_t d, int64_t ldx, const void* scale, int64_t scale_len,
               const char* who) {
  if (rows < 0 || d <= 0) return set_error(UFP8_ERR_INVALID, "%s: rows must be >= 0 and d > 0", who);
  if (d >= (int64_t(1) << 31)) return set_error(UFP8_ERR_INVALID, "%s: d exceeds 2^31", who);
  if (rows > 0 && !x) return set_error(UFP8_ERR_INVALID, "%s: null x", who);
  if (ldx < d) return set_error(UFP8_ERR_INVALID, "%s: ldx < d", who);
  if (scale && scale_len != 1 && scale_len != d)
    return set_error(UFP8_ERR_INVALID, "%s: scale_len must be 1 or d", who);
  if (reinterpret_cast<uintptr_t>(x) & 1u) return set_error(UFP8_ERR_ALIGN, "%s: x not 2-byte aligned", who);
  return UFP8_OK;
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Persistent grid of the backward: no more CTAs than fit on the device at once (a CTA that
// started late would run its rows after all the others), and no more than rows; at most 8 per SM.
int norm_bwd_grid(int64_t rows, int64_t d, bool vscale, const DeviceInfo& dev, int64_t* grid) {
  const int ch = static_cast<int>((d + 8 * kNormBwdThreads - 1) / (8 * kNormBwdThreads));
  const void* fn = ch <= 1 ? reinterpret_cast<const void*>(norm_backward_kernel<1>)
                 : ch <= 2 ? reinterpret_cast<const void*>(norm_backward_kernel<2>)
                           : reinterpret_cast<const void*>(norm_backward_kernel<4>);
  int per_sm = 0;
  const size_t smem = vscale ? 2 * static_cast<size_t>(d) * sizeof(float) : 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kNormBwdThreads, smem);
  if (e != cudaSuccess) return cuda_error(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor(rmsnorm backward)");
  per_sm = per_sm < 1 ? 1 : (per_sm > 8 ? 8 : per_sm);
  const int64_t cap = static_cast<int64_t>(dev.sm_count) * per_sm;
  *grid = rows < cap ? (rows > 0 ? rows : 1) : cap;
  return UFP8_OK;
}

}  // namespace
}  // namespace ufp8

using namespace ufp8;

extern "C" int ufp8_rmsnorm_quant(const void* x_bf16, int64_t rows, int64_t d, int64_t ldx, const void* scale_bf16,
                                  int64_t scale_len, int centered, float eps, int fmt, void* q, float* amax,
                                  float* inv_scale, float* rstd, void* y_bf16, int64_t ldy, ufp8_stream_t stream) {
  if (int rc = norm_check(x_bf16, rows, d, ldx, scale_bf16, scale_len, "ufp8_rmsnorm_quant")) return rc;
  if (!rstd && rows > 0) return set_error(UFP8_ERR_INVALID, "ufp8_rmsnorm_quant: null rstd");
  // The fp8 output is requested by inv_scale (q may be NULL only for an empty tensor).
  const bool want_q = inv_scale != nullptr;
  if (want_q && (!amax || (rows > 0 && !q)))
    return set_error(UFP8_ERR_INVALID, "ufp8_rmsnorm_quant: the fp8 output needs q and amax");
  if (want_q && fmt != UFP8_E4M3 && fmt != UFP8_E5M2)
    return set_error(UFP8_ERR_INVALID, "ufp8_rmsnorm_quant: fmt %d is not UFP8_E4M3/UFP8_E5M2", fmt);
  if (y_bf16 && ldy < d) return set_error(UFP8_ERR_INVALID, "ufp8_rmsnorm_quant: ldy < d");
  if (!want_q && !y_bf16 && !amax) return set_error(UFP8_ERR_INVALID, "ufp8_rmsnorm_quant: no output requested");
  DeviceInfo* dev;
  if (int rc = device_info(&dev)) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  NormArgs a{};
  a.x = static_cast<const uint16_t*>(x_bf16);
  a.ldx = ldx;
  a.rows = rows;
  a.d = static_cast<int>(d);
  a.scale = static_cast<const uint16_t*>(scale_bf16);
  a.scale_len = scale_bf16 ? static_cast<int>(scale_len) : 0;
  a.centered = centered;
  a.eps = eps;
  a.vec = d % 8 == 0 && al16(x_bf16) && (ldx * 2) % 16 == 0 && (!y_bf16 || (al16(y_bf16) && (ldy * 2) % 16 == 0)) &&
          (!q || (reinterpret_cast<uintptr_t>(q) & 7u) == 0);
  a.vec_scale = scale_bf16 && scale_len == d && d % 8 == 0 && al16(scale_bf16);
  a.rstd = rstd;
  a.amax_bits = reinterpret_cast<unsigned int*>(amax);
  a.y = static_cast<uint16_t*>(y_bf16);
  a.ldy = ldy;
  a.q = static_cast<uint8_t*>(q);
  a.fmt = fmt;
  a.amax = amax;
  a.inv_scale = inv_scale;
  if (amax) {
    cudaError_t e = cudaMemsetAsync(amax, 0, sizeof(float), s);
    if (e != cudaSuccess) return cuda_error(e, "cudaMemsetAsync(amax)");
  }
  if (rows > 0) {
    const int64_t grid = (rows + kNormRowsPerCta - 1) / kNormRowsPerCta;
    if (grid >= (int64_t(1) << 31)) return set_error(UFP8_ERR_INVALID, "ufp8_rmsnorm_quant: too many rows");
    norm_stats_kernel<<<static_cast<unsigned>(grid), 32 * kNormRowsPerCta, 0, s>>>(a);
    if (want_q) norm_quant_kernel<<<static_cast<unsigned>(grid), 32 * kNormRowsPerCta, 0, s>>>(a);
  } else if (want_q) {
    // empty tensor: amax 0 -> s = 1
    norm_quant_kernel<<<1, 32 * kNormRowsPerCta, 0, s>>>(a);
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? UFP8_OK : cuda_error(e, "rmsnorm kernel launch");
}

extern "C" int ufp8_rmsnorm_backward_workspace(int64_t rows, int64_t d, int64_t* bytes) {
  if (!bytes) return set_error(UFP8_ERR_INVALID, "ufp8_rmsnorm_backward_workspace: null pointer");
  if (rows < 0 || d <= 0) return set_error(UFP8_ERR_INVALID, "ufp8_rmsnorm_backward_workspace: bad shape");
  DeviceInfo* dev;
  if (int rc = device_info(&dev)) return rc;
  // the largest grid norm_bwd_grid can return: every SM full of CTAs
  const int64_t grid = rows < int64_t(dev->sm_count) * 8 ? (rows > 0 ? rows : 1) : int64_t(dev->sm_count) * 8;
  const int64_t per = d > kNormBwdThreads ? d : kNormBwdThreads;
  *bytes = grid * per * static_cast<int64_t>(sizeof(float));
  return UFP8_OK;
}

extern "C" int ufp8_rmsnorm_backward(const void* x_bf16, int64_t rows, int64_t d, int64_t ldx, const void* scale_bf16,
                                     int64_t scale_len, int centered, const float* rstd, const void* dy_bf16,
                                     int64_t lddy, void* dx_bf16, int64_t lddx, float* dscale, float* workspace,
                                     int64_t workspace_bytes, ufp8_stream_t stream) {
  if (int rc = norm_check(x_bf16, rows, d, ldx, scale_bf16, scale_len, "ufp8_rmsnorm_backward")) return rc;
  if (d > kNormMaxD) return set_error(UFP8_ERR_UNSUPPORTED, "ufp8_rmsnorm_backward: d %lld > %d",
                                      static_cast<long long>(d), kNormMaxD);
  if (rows > 0 && (!rstd || !dy_bf16 || !dx_bf16)) return set_error(UFP8_ERR_INVALID, "ufp8_rmsnorm_backward: null pointer");
  if (lddy < d || lddx < d) return set_error(UFP8_ERR_INVALID, "ufp8_rmsnorm_backward: lddy / lddx < d");
  if ((reinterpret_cast<uintptr_t>(dy_bf16) | reinterpret_cast<uintptr_t>(dx_bf16)) & 1u)
    return set_error(UFP8_ERR_ALIGN, "ufp8_rmsnorm_backward: dy / dx not 2-byte aligned");
  if (dscale && !scale_bf16) return set_error(UFP8_ERR_INVALID, "ufp8_rmsnorm_backward: dscale without a scale");
  int64_t need = 0;
  if (int rc = ufp8_rmsnorm_backward_workspace(rows, d, &need)) return rc;
  if (dscale && (!workspace || workspace_bytes < need))
    return set_error(UFP8_ERR_INVALID, "ufp8_rmsnorm_backward: workspace of %lld bytes needed",
                     static_cast<long long>(need));
  DeviceInfo* dev;
  if (int rc = device_info(&dev)) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  NormArgs a{};
  a.x = static_cast<const uint16_t*>(x_bf16);
  a.ldx = ldx;
  a.rows = rows;
  a.d = static_cast<int>(d);
  a.scale = static_cast<const uint16_t*>(scale_bf16);
  a.scale_len = scale_bf16 ? static_cast<int>(scale_len) : 0;
  a.centered = centered;
  a.vec = d % 8 == 0 && al16(x_bf16) && al16(dy_bf16) && al16(dx_bf16) && (ldx * 2) % 16 == 0 &&
          (lddy * 2) % 16 == 0 && (lddx * 2) % 16 == 0;
  a.vec_scale = scale_bf16 && scale_len == d && d % 8 == 0 && al16(scale_bf16);
  a.rstd = const_cast<float*>(rstd);
  a.dy = static_cast<const uint16_t*>(dy_bf16);
  a.lddy = lddy;
  a.dx = static_cast<uint16_t*>(dx_bf16);
  a.lddx = lddx;
  a.ws = dscale ? workspace : nullptr;
  const bool vscale = scale_bf16 && scale_len != 1;
  const size_t smem = vscale ? 2 * static_cast<size_t>(d) * sizeof(float) : 0;
  const int ch = static_cast<int>((d + 8 * kNormBwdThreads - 1) / (8 * kNormBwdThreads));
  static thread_local int attr_device = -1;
  if (attr_device != dev->device) {
    // vector scales up to d = 8192 need 64 KiB of dynamic shared memory
    cudaError_t e = cudaFuncSetAttribute(norm_backward_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         2 * kNormMaxD * static_cast<int>(sizeof(float)));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(norm_backward_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               2 * kNormMaxD * static_cast<int>(sizeof(float)));
    if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(rmsnorm backward smem)");
    attr_device = dev->device;
  }
  int64_t grid = 0;
  if (int rc = norm_bwd_grid(rows, d, vscale, *dev, &grid)) return rc;
  if (rows > 0 || dscale) {
    const unsigned g = static_cast<unsigned>(grid);
    if (ch <= 1)
      norm_backward_kernel<1><<<g, kNormBwdThreads, smem, s>>>(a);
    else if (ch <= 2)
      norm_backward_kernel<2><<<g, kNormBwdThreads, smem, s>>>(a);
    else
      norm_backward_kernel<4><<<g, kNormBwdThreads, smem, s>>>(a);
  }
  if (dscale) {
    const int len = static_cast<int>(a.scale_len);
    const unsigned blocks = len == 1 ? 1u : static_cast<unsigned>((len + kDsCols - 1) / kDsCols);
    norm_dscale_kernel<<<blocks, kNormBwdThreads, 0, s>>>(workspace, static_cast<int>(grid), len, dscale);
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? UFP8_OK : cuda_error(e, "rmsnorm backward launch");
}
