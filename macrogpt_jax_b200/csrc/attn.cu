// Softmax attention of the reference's SoftmaxAttention (ueaj/model/soft_attn.py:142-202) and its
// RoPE (ueaj/model/rope.py:10-104).
//
// The reference calls kvax 0.1.2's flash_attention (requirements.txt:35, not installable here):
// out = softmax(scale * Q K^T + mask) V per query head, the mask allowing query position p to see
// key position p' of the same sequence iff p' <= p and both carry the same segment id, padding
// (a negative segment id) seeing and seen by nothing; a row that sees nothing gives 0.  Grouped
// query attention: query head (h, i) uses key/value head h.
//
// B200 layout of the computation: the products are the bf16 CTA-pair GEMM (tcgen05 kind::f16, fp32
// accumulation), one launch per batch element and product over all query heads g = h * I + i; the
// key/value operand repeats each head for its group (batch_group I: product g reads head g / I),
// and dK, dV concatenate the contraction over the group (k_batches).  The scores S (f32) and probabilities P (bf16) of one batch element are
// materialised in HBM (HI x n x n per batch element; P is kept for the backward), and the masked
// softmax and its backward are row kernels between the GEMMs:
//   forward:  S_g = Q_g K_h^T            softmax rows -> P_g (bf16), lse     O_g = P_g V_h
//   backward: dP_g = dO_g V_h^T          dS_g = scale * P_g (dP_g - rowsum(dO_g O_g))
//             dQ_g = dS_g K_h            dK_h = sum_i dS_g^T Q_g             dV_h = sum_i P_g^T dO_g
// With the default positions (0..n-1) the masked upper triangle is skipped: the score products
// compute only the 256 x 256 tiles on or below the diagonal, P V and dS K contract each query tile
// only up to its diagonal, dS^T Q and P^T dO each key tile only from its diagonal (UFP8_TILES_*);
// and S and dP never reach memory: the score product runs once for per-row softmax partials
// (UFP8_EPI_ATTN_STATS, combined into the lse by a row kernel) and once more writing P from its
// accumulators (UFP8_EPI_ATTN_P), and the dP product writes dS = scale P (dP - rowsum(dO O))
// (UFP8_EPI_ATTN_DS).  Explicit positions take the materialised path above.
// No transposed copy is made (MN-major operands).  RoPE: one kernel builds the bf16 sin/cos table
// from positions (f32 angle = position * inv_freq, sinf/cosf, then bf16, as the reference's
// compute_rope_embedding), one applies the rotation (bf16 rounding after each product and sum, as
// the reference's bf16 expression does) or its transpose for the backward.
#include <cuda_bf16.h>

#include <algorithm>
#include <cmath>

#include "internal.h"

namespace ufp8 {
namespace {

constexpr int kAThreads = 256;

__device__ __forceinline__ float bfr(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

__global__ void __launch_bounds__(kAThreads) rope_table_kernel(const float* __restrict__ pos, int64_t count, int half,
                                                               const float* __restrict__ inv_freq,
                                                               __nv_bfloat16* __restrict__ sin_t,
                                                               __nv_bfloat16* __restrict__ cos_t) {
  const int64_t n = count * half;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kAThreads + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * kAThreads) {
    const int64_t p = i / half;
    const int j = static_cast<int>(i - p * half);
    const float a = __fmul_rn(pos[p], inv_freq[j]);
    sin_t[i] = __float2bfloat16_rn(sinf(a));
    cos_t[i] = __float2bfloat16_rn(cosf(a));
  }
}

// x [tokens][heads][d] bf16; token t uses table row t % period.  Forward: (x1 c - x2 s, x2 c + x1 s);
// inverse (the transpose, for the backward): (y1 c + y2 s, y2 c - y1 s).
__global__ void __launch_bounds__(kAThreads) rope_apply_kernel(const __nv_bfloat16* __restrict__ x, int64_t tokens,
                                                               int heads, int half, int64_t period,
                                                               const __nv_bfloat16* __restrict__ sin_t,
                                                               const __nv_bfloat16* __restrict__ cos_t, int inverse,
                                                               __nv_bfloat16* __restrict__ out) {
  const int64_t n = tokens * heads * half;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kAThreads + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * kAThreads) {
    const int64_t row = i / half;  // (token, head)
    const int j = static_cast<int>(i - row * half);
    const int64_t t = row / heads;
    const int64_t tr = (t % period) * half + j;
    const float s = __bfloat162float(sin_t[tr]), c = __bfloat162float(cos_t[tr]);
    const int64_t b = row * 2 * half;
    const float x1 = __bfloat162float(x[b + j]), x2 = __bfloat162float(x[b + half + j]);
    float o1, o2;
    if (!inverse) {
      o1 = __fsub_rn(bfr(__fmul_rn(x1, c)), bfr(__fmul_rn(x2, s)));
      o2 = __fadd_rn(bfr(__fmul_rn(x2, c)), bfr(__fmul_rn(x1, s)));
    } else {
      o1 = __fadd_rn(bfr(__fmul_rn(x1, c)), bfr(__fmul_rn(x2, s)));
      o2 = __fsub_rn(bfr(__fmul_rn(x2, c)), bfr(__fmul_rn(x1, s)));
    }
    out[b + j] = __float2bfloat16_rn(o1);
    out[b + half + j] = __float2bfloat16_rn(o2);
  }
}

struct SoftArgs {
  const float* S;    // [rows][n] scores of one batch element (rows = HI * n, row = g * n + q)
  int64_t rows, n;
  const int32_t* qseg;  // [n] of this batch element (NULL: 0)
  const int32_t* kseg;
  const int32_t* qpos;  // NULL: arange
  const int32_t* kpos;
  float scale;
  __nv_bfloat16* P;  // [rows][n]
  float* lse;        // [rows]
  // backward
  const float* dP;
  const __nv_bfloat16* O;   // [n][HI][d] of this batch element
  const __nv_bfloat16* dO;
  int64_t hi, d;
  __nv_bfloat16* dS;
};

__device__ __forceinline__ bool visible(int32_t sq, int32_t pq, int32_t sk, int32_t pk) {
  return sq >= 0 && sk == sq && pk <= pq;
}

__device__ __forceinline__ void block_max_sum(float& m, float& s, float* sm, float* ss) {
  // merge (m, s) pairs over the CTA in a fixed order
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float m2 = __shfl_xor_sync(0xFFFFFFFFu, m, off), s2 = __shfl_xor_sync(0xFFFFFFFFu, s, off);
    const float mn = fmaxf(m, m2);
    if (mn != -INFINITY) {
      s = s * __expf(m - mn) + s2 * __expf(m2 - mn);
      m = mn;
    }
  }
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sm[w] = m;
    ss[w] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = sm[0], S = ss[0];
    for (int i = 1; i < kAThreads / 32; ++i) {
      const float mn = fmaxf(M, sm[i]);
      if (mn != -INFINITY) {
        S = S * __expf(M - mn) + ss[i] * __expf(sm[i] - mn);
        M = mn;
      }
    }
    sm[0] = M;
    ss[0] = S;
  }
  __syncthreads();
  m = sm[0];
  s = ss[0];
}

// Visibility of the 4 keys k4 * 4 .. k4 * 4 + 3 for a query (segment sq, position pq).
__device__ __forceinline__ void vis4(const SoftArgs& a, int64_t k4, int32_t sq, int32_t pq, bool (&v)[4]) {
  const int4 ks = a.kseg ? reinterpret_cast<const int4*>(a.kseg)[k4] : make_int4(0, 0, 0, 0);
  const int64_t k0 = k4 * 4;
  const int4 kp = a.kpos ? reinterpret_cast<const int4*>(a.kpos)[k4]
                         : make_int4(static_cast<int>(k0), static_cast<int>(k0 + 1), static_cast<int>(k0 + 2),
                                     static_cast<int>(k0 + 3));
  v[0] = visible(sq, pq, ks.x, kp.x);
  v[1] = visible(sq, pq, ks.y, kp.y);
  v[2] = visible(sq, pq, ks.z, kp.z);
  v[3] = visible(sq, pq, ks.w, kp.w);
}

// Keys past `lim` (in groups of 4) cannot be visible: with the default key positions 0..n-1 a key
// is visible only at position <= the query's.
__device__ __forceinline__ int64_t row_limit4(const SoftArgs& a, int32_t sq, int32_t pq) {
  if (sq < 0) return 0;
  if (a.kpos) return a.n / 4;
  const int64_t last = pq < 0 ? -1 : (pq >= a.n ? a.n - 1 : pq);
  return (last + 4) / 4;
}

// One CTA per score row: masked online (max, sum exp) of scale * s, then P = exp(scale s - M) / S.
// 16-byte score loads, 8-byte probability stores (n is a multiple of 8).
__global__ void __launch_bounds__(kAThreads) attn_softmax_kernel(const SoftArgs a) {
  const int64_t row = blockIdx.x;
  const int64_t q = row % a.n;
  const float4* sr = reinterpret_cast<const float4*>(a.S + row * a.n);
  const int32_t sq = a.qseg ? a.qseg[q] : 0;
  const int32_t pq = a.qpos ? a.qpos[q] : static_cast<int32_t>(q);
  const int64_t lim = row_limit4(a, sq, pq);
  float m = -INFINITY, s = 0.0f;
  for (int64_t k4 = threadIdx.x; k4 < lim; k4 += kAThreads) {
    bool v[4];
    vis4(a, k4, sq, pq, v);
    const float4 x = sr[k4];
    const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (!v[j]) continue;
      const float t = __fmul_rn(xs[j], a.scale);
      if (t > m) {
        s *= __expf(m - t);
        m = t;
      }
      s += __expf(t - m);
    }
  }
  __shared__ float sm[kAThreads / 32], ss[kAThreads / 32];
  block_max_sum(m, s, sm, ss);
  const float inv = s > 0.0f ? __fdiv_rn(1.0f, s) : 0.0f;
  uint2* pr = reinterpret_cast<uint2*>(a.P + row * a.n);
  for (int64_t k4 = threadIdx.x; k4 < a.n / 4; k4 += kAThreads) {
    float p[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (k4 < lim) {
      bool v[4];
      vis4(a, k4, sq, pq, v);
      const float4 x = sr[k4];
      const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (v[j]) p[j] = __fmul_rn(__expf(__fsub_rn(__fmul_rn(xs[j], a.scale), m)), inv);
    }
    const __nv_bfloat162 lo = __floats2bfloat162_rn(p[0], p[1]), hi = __floats2bfloat162_rn(p[2], p[3]);
    pr[k4] = make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
  }
  if (threadIdx.x == 0) a.lse[row] = s > 0.0f ? __fadd_rn(m, logf(s)) : -INFINITY;
}

// One CTA per row: D = sum_d dO O (f32, fixed order), dS = bf16(scale * P (dP - D)); past the row's
// key limit P is 0 and dS is written as 0 without reading P or dP.
__global__ void __launch_bounds__(kAThreads) attn_softmax_bwd_kernel(const SoftArgs a) {
  const int64_t row = blockIdx.x;
  const int64_t g = row / a.n, q = row - g * a.n;
  const __nv_bfloat16* o = a.O + (q * a.hi + g) * a.d;
  const __nv_bfloat16* go = a.dO + (q * a.hi + g) * a.d;
  float part = 0.0f;
  for (int64_t j = threadIdx.x; j < a.d; j += kAThreads)
    part = __fadd_rn(part, __fmul_rn(__bfloat162float(o[j]), __bfloat162float(go[j])));
  __shared__ float red[kAThreads];
  red[threadIdx.x] = part;
  __syncthreads();
  for (int off = kAThreads / 2; off > 0; off >>= 1) {
    if (threadIdx.x < off) red[threadIdx.x] = __fadd_rn(red[threadIdx.x], red[threadIdx.x + off]);
    __syncthreads();
  }
  const float D = red[0];
  const int32_t sq = a.qseg ? a.qseg[q] : 0;
  const int32_t pq = a.qpos ? a.qpos[q] : static_cast<int32_t>(q);
  const int64_t lim = row_limit4(a, sq, pq);
  const uint2* pr = reinterpret_cast<const uint2*>(a.P + row * a.n);
  const float4* dpr = reinterpret_cast<const float4*>(a.dP + row * a.n);
  uint2* dsr = reinterpret_cast<uint2*>(a.dS + row * a.n);
  for (int64_t k4 = threadIdx.x; k4 < a.n / 4; k4 += kAThreads) {
    uint2 o2 = make_uint2(0u, 0u);
    if (k4 < lim) {
      const uint2 pw = pr[k4];
      const float4 dp = dpr[k4];
      const float p[4] = {__uint_as_float(pw.x << 16), __uint_as_float(pw.x & 0xFFFF0000u),
                          __uint_as_float(pw.y << 16), __uint_as_float(pw.y & 0xFFFF0000u)};
      const float dpv[4] = {dp.x, dp.y, dp.z, dp.w};
      float r[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) r[j] = __fmul_rn(__fmul_rn(p[j], __fsub_rn(dpv[j], D)), a.scale);
      const __nv_bfloat162 lo = __floats2bfloat162_rn(r[0], r[1]), hi = __floats2bfloat162_rn(r[2], r[3]);
      o2 = make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
    }
    dsr[k4] = o2;
  }
}

// Default positions: the lse of each score row (natural log) from the UFP8_EPI_ATTN_STATS partials
// (one base-2 (max, sum 2^(y - max)) per 128 columns), over the groups up to the end of the row's
// 256-wide diagonal tile (the products skip the tiles past it).  One warp per row (row = g * n + q):
// lane j merges groups j, j + 32, ... (coalesced reads) online, then a fixed xor butterfly merges
// the lanes' (max, sum) pairs.
__global__ void __launch_bounds__(kAThreads) attn_lse_kernel(const float2* __restrict__ stats, int64_t rows,
                                                             int64_t n, int64_t ld, float* __restrict__ lse) {
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * kAThreads + threadIdx.x) / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;  // whole warps
  const int64_t q = row % n;
  const int64_t diag = (q / 256 + 1) * 2;
  const int64_t groups = diag < ld ? diag : ld;
  const float2* st = stats + row * ld;
  float M = -INFINITY, S = 0.0f;  // this lane's (max, sum 2^(y - max)), merged online
  for (int64_t j = lane; j < groups; j += 32) {
    const float2 v = st[j];
    if (v.y > 0.0f) {
      if (v.x > M) {
        S = S * exp2f(M - v.x);  // M = -inf at first: 0 * 0
        M = v.x;
      }
      S += v.y * exp2f(v.x - M);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {  // fixed butterfly over (M, S) pairs
    const float Mo = __shfl_xor_sync(0xFFFFFFFFu, M, o), So = __shfl_xor_sync(0xFFFFFFFFu, S, o);
    const float Mn = fmaxf(M, Mo);
    S = (S > 0.0f ? S * exp2f(M - Mn) : 0.0f) + (So > 0.0f ? So * exp2f(Mo - Mn) : 0.0f);
    M = Mn;
  }
  if (!(S > 0.0f)) {
    if (lane == 0) lse[row] = -INFINITY;
    return;
  }
  if (lane == 0) lse[row] = (M + log2f(S)) * 0.6931471805599453f;  // partials in base 2 -> natural log
}

// rowsum(dO * O) of every (query head g, query q) row of one batch element (O, dO [n][hi][d]):
// one warp per row, f32 products summed lane-strided then by a fixed shuffle tree.
__global__ void __launch_bounds__(kAThreads) attn_rowdot_kernel(const __nv_bfloat16* __restrict__ O,
                                                                const __nv_bfloat16* __restrict__ dO, int64_t n,
                                                                int64_t hi, int64_t d, float* __restrict__ out) {
  const int64_t w = (static_cast<int64_t>(blockIdx.x) * kAThreads + threadIdx.x) / 32;
  const int lane = threadIdx.x & 31;
  if (w >= hi * n) return;
  const int64_t g = w / n, q = w - g * n;
  const __nv_bfloat16* o = O + (q * hi + g) * d;
  const __nv_bfloat16* go = dO + (q * hi + g) * d;
  float part = 0.0f;
  for (int64_t j = lane; j < d; j += 32)
    part = __fadd_rn(part, __fmul_rn(__bfloat162float(o[j]), __bfloat162float(go[j])));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) part = __fadd_rn(part, __shfl_xor_sync(0xFFFFFFFFu, part, off));
  if (lane == 0) out[w] = part;
}

ufp8_operand bop(const void* p, int major, int64_t ld, int64_t bstride, int32_t count, int32_t group = 0) {
  ufp8_operand o{};
  o.batch_group = group;
  o.ptr = p;
  o.fmt = UFP8_BF16;
  o.major = major;
  o.ld = ld;
  o.batch_stride = bstride;
  o.batch_count = count;
  return o;
}

int gemm_bf16(const ufp8_operand& A, const ufp8_operand& B, int64_t M, int64_t N, int64_t K, int32_t batch,
              int32_t kb, void* D, int d_f32, int64_t ldd, int64_t dbs, cudaStream_t s, const DeviceInfo& dev,
              int tile_mask = UFP8_TILES_ALL) {
  ufp8_gemm_desc d{};
  d.tile_mask = tile_mask;
  d.M = M;
  d.N = N;
  d.K = K;
  d.batch = batch;
  d.k_batches = kb;
  d.a = A;
  d.b = B;
  d.d = D;
  d.d_dtype = d_f32 ? UFP8_OUT_F32 : UFP8_OUT_BF16;
  d.epilogue = UFP8_EPI_STORE;
  d.ldd = ldd;
  d.d_batch_stride = dbs;
  return launch_gemm(d, s, dev, 0, UFP8_GEMM_AUTO, 0);
}

// One score-shaped product (M = N = n, batch = query heads) with an attention epilogue.
int gemm_attn(int mode, const ufp8_operand& A, const ufp8_operand& B, int64_t n, int64_t K, int32_t batch, void* D,
              const int32_t* qseg, const int32_t* kseg, float* stats, int64_t ld_stats, const float* row,
              const void* P, float scale, cudaStream_t s, const DeviceInfo& dev) {
  ufp8_gemm_desc d{};
  d.M = n;
  d.N = n;
  d.K = K;
  d.batch = batch;
  d.k_batches = 1;
  d.a = A;
  d.b = B;
  d.d = D;
  d.d_dtype = UFP8_OUT_BF16;
  d.epilogue = mode;
  d.ldd = n;
  d.d_batch_stride = n * n;
  d.tile_mask = UFP8_TILES_LOWER;
  d.attn_q_segment_ids = qseg;
  d.attn_kv_segment_ids = kseg;
  d.attn_stats = stats;
  d.attn_ld_stats = ld_stats;
  d.attn_row = row;
  d.c = P;
  d.ldc = n;
  d.c_batch_stride = n * n;
  d.attn_scale = scale;
  return launch_gemm(d, s, dev, 0, UFP8_GEMM_AUTO, 0);
}

int attn_check(const ufp8_attn_desc* d, const char* who) {
  if (!d) return set_error(UFP8_ERR_INVALID, "%s: null descriptor", who);
  if (d->batch < 0 || d->seq < 1 || d->kv_heads < 1 || d->group < 1 || d->head_dim < 2 || d->head_dim % 8)
    return set_error(UFP8_ERR_INVALID, "%s: bad shape (seq, heads >= 1; head_dim even and a multiple of 8)", who);
  if (d->seq % 8) return set_error(UFP8_ERR_UNSUPPORTED, "%s: seq must be a multiple of 8 (16-byte rows of P)", who);
  if (d->seq >= (int64_t(1) << 31)) return set_error(UFP8_ERR_INVALID, "%s: seq exceeds 2^31", who);
  const uintptr_t ids = reinterpret_cast<uintptr_t>(d->q_segment_ids) | reinterpret_cast<uintptr_t>(d->kv_segment_ids) |
                        reinterpret_cast<uintptr_t>(d->q_positions) | reinterpret_cast<uintptr_t>(d->kv_positions);
  if (ids & 15u) return set_error(UFP8_ERR_ALIGN, "%s: segment id / position arrays not 16-byte aligned", who);
  return UFP8_OK;
}

// Workspaces per batch element.  Default positions (fused): forward = ATTN_STATS partials
// [HI * n][ceil(n / 128)] float2, backward = rowsum(dO O) [HI * n] f32 + dS.  Explicit positions:
// forward = S f32, backward = dP f32 + dS.
struct AttnLayout {
  int64_t S, total_fwd;       // forward workspace: S f32 or the partials, at offset 0
  int64_t P, lse, saved;      // saved: P bf16 and lse of every batch element
  int64_t dP, dS, total_bwd;  // backward workspace: dP f32 or rowsum(dO O) at offset 0, dS bf16
  int64_t ld_stats;           // float2 partials per row (fused path)
};

int64_t al256(int64_t b) { return (b + 255) / 256 * 256; }

bool attn_fused(const ufp8_attn_desc& d) { return d.q_positions == nullptr && d.kv_positions == nullptr; }

AttnLayout attn_layout(const ufp8_attn_desc& d) {
  const int64_t hi = d.kv_heads * d.group, nn = d.seq * d.seq;
  const bool fused = attn_fused(d);
  AttnLayout L{};
  L.ld_stats = (d.seq + 127) / 128;
  L.S = 0;
  L.total_fwd = fused ? al256(hi * d.seq * L.ld_stats * 8) : al256(hi * nn * 4);
  L.P = 0;
  L.lse = al256(d.batch * hi * nn * 2);
  L.saved = L.lse + al256(d.batch * hi * d.seq * 4);
  L.dP = 0;
  L.dS = fused ? al256(hi * d.seq * 4) : al256(hi * nn * 4);
  L.total_bwd = L.dS + al256(hi * nn * 2);
  return L;
}

}  // namespace
}  // namespace ufp8

using namespace ufp8;

extern "C" int ufp8_rope_table(const float* positions, int64_t count, int64_t half, const float* inv_freq,
                               void* sin_bf16, void* cos_bf16, ufp8_stream_t stream) {
  if (count < 0 || half < 1 || half > (1 << 20)) return set_error(UFP8_ERR_INVALID, "ufp8_rope_table: bad shape");
  if (count > 0 && (!positions || !inv_freq || !sin_bf16 || !cos_bf16))
    return set_error(UFP8_ERR_INVALID, "ufp8_rope_table: null pointer");
  if (count == 0) return UFP8_OK;
  DeviceInfo* dev;
  if (int rc = device_info(&dev)) return rc;
  const int64_t n = count * half;
  const int64_t grid = std::min<int64_t>((n + kAThreads - 1) / kAThreads, int64_t(dev->sm_count) * 16);
  rope_table_kernel<<<static_cast<unsigned>(grid), kAThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      positions, count, static_cast<int>(half), inv_freq, static_cast<__nv_bfloat16*>(sin_bf16),
      static_cast<__nv_bfloat16*>(cos_bf16));
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? UFP8_OK : cuda_error(e, "rope table launch");
}

extern "C" int ufp8_rope(const void* x_bf16, int64_t tokens, int64_t heads, int64_t d, const void* sin_bf16,
                         const void* cos_bf16, int64_t period, int inverse, void* out_bf16, ufp8_stream_t stream) {
  if (tokens < 0 || heads < 1 || d < 2 || d % 2 || period < 1)
    return set_error(UFP8_ERR_INVALID, "ufp8_rope: bad shape (d even, heads and period >= 1)");
  if (tokens > 0 && (!x_bf16 || !sin_bf16 || !cos_bf16 || !out_bf16))
    return set_error(UFP8_ERR_INVALID, "ufp8_rope: null pointer");
  if (tokens == 0) return UFP8_OK;
  DeviceInfo* dev;
  if (int rc = device_info(&dev)) return rc;
  const int64_t n = tokens * heads * (d / 2);
  const int64_t grid = std::min<int64_t>((n + kAThreads - 1) / kAThreads, int64_t(dev->sm_count) * 16);
  rope_apply_kernel<<<static_cast<unsigned>(grid), kAThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x_bf16), tokens, static_cast<int>(heads), static_cast<int>(d / 2), period,
      static_cast<const __nv_bfloat16*>(sin_bf16), static_cast<const __nv_bfloat16*>(cos_bf16), inverse ? 1 : 0,
      static_cast<__nv_bfloat16*>(out_bf16));
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? UFP8_OK : cuda_error(e, "rope launch");
}

extern "C" int ufp8_attention_workspace(const ufp8_attn_desc* d, int64_t* fwd_bytes, int64_t* saved_bytes,
                                        int64_t* bwd_bytes) {
  if (int rc = attn_check(d, "ufp8_attention_workspace")) return rc;
  if (!fwd_bytes || !saved_bytes || !bwd_bytes) return set_error(UFP8_ERR_INVALID, "ufp8_attention_workspace: null");
  const AttnLayout L = attn_layout(*d);
  *fwd_bytes = L.total_fwd;
  *saved_bytes = L.saved;
  *bwd_bytes = L.total_bwd;
  return UFP8_OK;
}

extern "C" int ufp8_attention_forward(const ufp8_attn_desc* d, const void* q, const void* k, const void* v, void* out,
                                      void* saved, void* workspace, ufp8_stream_t stream) {
  const char* who = "ufp8_attention_forward";
  if (int rc = attn_check(d, who)) return rc;
  if (d->batch > 0 && (!q || !k || !v || !out || !saved || !workspace))
    return set_error(UFP8_ERR_INVALID, "%s: null pointer", who);
  if ((reinterpret_cast<uintptr_t>(saved) | reinterpret_cast<uintptr_t>(workspace)) & 255u)
    return set_error(UFP8_ERR_ALIGN, "%s: saved / workspace not 256-byte aligned", who);
  if (d->batch == 0) return UFP8_OK;
  DeviceInfo* dev;
  if (int rc = device_info(&dev)) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const AttnLayout L = attn_layout(*d);
  const int64_t n = d->seq, H = d->kv_heads, I = d->group, Dh = d->head_dim, hi = H * I, nn = n * n;
  // Default positions (0..n-1 for queries and keys): a key tile past the query tile is fully
  // masked, so the products skip it (the softmax kernels write the zeros of P / dS there).
  const bool causal = d->q_positions == nullptr && d->kv_positions == nullptr;
  const auto* qb = static_cast<const __nv_bfloat16*>(q);
  const auto* kb = static_cast<const __nv_bfloat16*>(k);
  const auto* vb = static_cast<const __nv_bfloat16*>(v);
  auto* ob = static_cast<__nv_bfloat16*>(out);
  float* S = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + L.S);
  auto* P0 = reinterpret_cast<__nv_bfloat16*>(static_cast<uint8_t*>(saved) + L.P);
  float* lse0 = reinterpret_cast<float*>(static_cast<uint8_t*>(saved) + L.lse);
  for (int64_t b = 0; b < d->batch; ++b) {
    const __nv_bfloat16* qB = qb + b * n * hi * Dh;
    const __nv_bfloat16* kB = kb + b * n * H * Dh;
    const __nv_bfloat16* vB = vb + b * n * H * Dh;
    __nv_bfloat16* P = P0 + b * hi * nn;
    const int32_t* qsegB = d->q_segment_ids ? d->q_segment_ids + b * n : nullptr;
    const int32_t* ksegB = d->kv_segment_ids ? d->kv_segment_ids + b * n : nullptr;
    const ufp8_operand qop = bop(qB, UFP8_K_MAJOR, hi * Dh, Dh, static_cast<int32_t>(hi));
    const ufp8_operand kop = bop(kB, UFP8_K_MAJOR, H * Dh, Dh, static_cast<int32_t>(H), static_cast<int32_t>(I));
    if (causal) {
      // Fused: the score product runs twice without storing S, first for the per-row softmax
      // partials (-> lse), then writing P = exp(scale s - lse) straight from the accumulators.
      auto* stats = reinterpret_cast<float*>(S);
      int rc = gemm_attn(UFP8_EPI_ATTN_STATS, qop, kop, n, Dh, static_cast<int32_t>(hi), nullptr, qsegB, ksegB, stats,
                         L.ld_stats, nullptr, nullptr, d->scale, s, *dev);
      if (rc) return rc;
      const int64_t rows = hi * n;
      attn_lse_kernel<<<static_cast<unsigned>((rows * 32 + kAThreads - 1) / kAThreads), kAThreads, 0, s>>>(
          reinterpret_cast<const float2*>(stats), rows, n, L.ld_stats, lse0 + b * hi * n);
      cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) return cuda_error(e, "attention lse launch");
      rc = gemm_attn(UFP8_EPI_ATTN_P, qop, kop, n, Dh, static_cast<int32_t>(hi), P, qsegB, ksegB, nullptr, 0,
                     lse0 + b * hi * n, nullptr, d->scale, s, *dev);
      if (rc) return rc;
      rc = gemm_bf16(bop(P, UFP8_K_MAJOR, n, nn, static_cast<int32_t>(hi)),
                     bop(vB, UFP8_MN_MAJOR, H * Dh, Dh, static_cast<int32_t>(H), static_cast<int32_t>(I)), n, Dh, n,
                     static_cast<int32_t>(hi), 1, ob + b * n * hi * Dh, 0, hi * Dh, Dh, s, *dev,
                     UFP8_TILES_K_TO_DIAG);
      if (rc) return rc;
      continue;
    }
    // S_g = Q_g K_h^T for every query head g = h * I + i in one launch (key head g / I).
    int rc = gemm_bf16(bop(qB, UFP8_K_MAJOR, hi * Dh, Dh, static_cast<int32_t>(hi)),
                       bop(kB, UFP8_K_MAJOR, H * Dh, Dh, static_cast<int32_t>(H), static_cast<int32_t>(I)), n, n,
                       Dh, static_cast<int32_t>(hi), 1, S, 1, n, nn, s, *dev,
                       UFP8_TILES_ALL);
    if (rc) return rc;
    SoftArgs a{};
    a.S = S;
    a.rows = hi * n;
    a.n = n;
    a.qseg = d->q_segment_ids ? d->q_segment_ids + b * n : nullptr;
    a.kseg = d->kv_segment_ids ? d->kv_segment_ids + b * n : nullptr;
    a.qpos = d->q_positions ? d->q_positions + b * n : nullptr;
    a.kpos = d->kv_positions ? d->kv_positions + b * n : nullptr;
    a.scale = d->scale;
    a.P = P;
    a.lse = lse0 + b * hi * n;
    attn_softmax_kernel<<<static_cast<unsigned>(hi * n), kAThreads, 0, s>>>(a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_error(e, "attention softmax launch");
    // O_g = P_g V_{g / I}
    rc = gemm_bf16(bop(P, UFP8_K_MAJOR, n, nn, static_cast<int32_t>(hi)),
                   bop(vB, UFP8_MN_MAJOR, H * Dh, Dh, static_cast<int32_t>(H), static_cast<int32_t>(I)), n, Dh, n,
                   static_cast<int32_t>(hi), 1, ob + b * n * hi * Dh, 0, hi * Dh, Dh, s, *dev,
                   UFP8_TILES_ALL);
    if (rc) return rc;
  }
  return UFP8_OK;
}

extern "C" int ufp8_attention_backward(const ufp8_attn_desc* d, const void* q, const void* k, const void* v,
                                       const void* out, const void* dout, const void* saved, void* dq, void* dk,
                                       void* dv, void* workspace, ufp8_stream_t stream) {
  const char* who = "ufp8_attention_backward";
  if (int rc = attn_check(d, who)) return rc;
  if (d->batch > 0 && (!q || !k || !v || !out || !dout || !saved || !dq || !dk || !dv || !workspace))
    return set_error(UFP8_ERR_INVALID, "%s: null pointer", who);
  if ((reinterpret_cast<uintptr_t>(saved) | reinterpret_cast<uintptr_t>(workspace)) & 255u)
    return set_error(UFP8_ERR_ALIGN, "%s: saved / workspace not 256-byte aligned", who);
  if (d->batch == 0) return UFP8_OK;
  DeviceInfo* dev;
  if (int rc = device_info(&dev)) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const AttnLayout L = attn_layout(*d);
  const int64_t n = d->seq, H = d->kv_heads, I = d->group, Dh = d->head_dim, hi = H * I, nn = n * n;
  // Default positions (0..n-1 for queries and keys): a key tile past the query tile is fully
  // masked, so the products skip it (the softmax kernels write the zeros of P / dS there).
  const bool causal = d->q_positions == nullptr && d->kv_positions == nullptr;
  const auto* qb = static_cast<const __nv_bfloat16*>(q);
  const auto* kb = static_cast<const __nv_bfloat16*>(k);
  const auto* vb = static_cast<const __nv_bfloat16*>(v);
  const auto* ob = static_cast<const __nv_bfloat16*>(out);
  const auto* gob = static_cast<const __nv_bfloat16*>(dout);
  auto* dqb = static_cast<__nv_bfloat16*>(dq);
  auto* dkb = static_cast<__nv_bfloat16*>(dk);
  auto* dvb = static_cast<__nv_bfloat16*>(dv);
  const auto* P0 = reinterpret_cast<const __nv_bfloat16*>(static_cast<const uint8_t*>(saved) + L.P);
  float* dP = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + L.dP);
  auto* dS = reinterpret_cast<__nv_bfloat16*>(static_cast<uint8_t*>(workspace) + L.dS);
  for (int64_t b = 0; b < d->batch; ++b) {
    const __nv_bfloat16* qB = qb + b * n * hi * Dh;
    const __nv_bfloat16* kB = kb + b * n * H * Dh;
    const __nv_bfloat16* vB = vb + b * n * H * Dh;
    const __nv_bfloat16* oB = ob + b * n * hi * Dh;
    const __nv_bfloat16* goB = gob + b * n * hi * Dh;
    const __nv_bfloat16* P = P0 + b * hi * nn;
    int rc;
    if (causal) {
      // Fused: D = rowsum(dO O), then the dP product writes dS = scale P (dP - D) from its
      // accumulators and the saved P (no dP in memory).
      float* Drow = dP;
      const int64_t warps = hi * n;
      attn_rowdot_kernel<<<static_cast<unsigned>((warps * 32 + kAThreads - 1) / kAThreads), kAThreads, 0, s>>>(
          oB, goB, n, hi, Dh, Drow);
      cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) return cuda_error(e, "attention rowdot launch");
      rc = gemm_attn(UFP8_EPI_ATTN_DS, bop(goB, UFP8_K_MAJOR, hi * Dh, Dh, static_cast<int32_t>(hi)),
                         bop(vB, UFP8_K_MAJOR, H * Dh, Dh, static_cast<int32_t>(H), static_cast<int32_t>(I)), n, Dh,
                         static_cast<int32_t>(hi), dS, d->q_segment_ids ? d->q_segment_ids + b * n : nullptr,
                         d->kv_segment_ids ? d->kv_segment_ids + b * n : nullptr, nullptr, 0, Drow, P, d->scale, s,
                         *dev);
      if (rc) return rc;
    } else {
      // dP_g = dO_g V_{g / I}^T, then the softmax backward rows
      rc = gemm_bf16(bop(goB, UFP8_K_MAJOR, hi * Dh, Dh, static_cast<int32_t>(hi)),
                     bop(vB, UFP8_K_MAJOR, H * Dh, Dh, static_cast<int32_t>(H), static_cast<int32_t>(I)), n, n, Dh,
                     static_cast<int32_t>(hi), 1, dP, 1, n, nn, s, *dev, UFP8_TILES_ALL);
      if (rc) return rc;
      SoftArgs a{};
      a.rows = hi * n;
      a.n = n;
      a.scale = d->scale;
      a.P = const_cast<__nv_bfloat16*>(P);
      a.dP = dP;
      a.O = oB;
      a.dO = goB;
      a.hi = hi;
      a.d = Dh;
      a.dS = dS;
      a.qseg = d->q_segment_ids ? d->q_segment_ids + b * n : nullptr;
      a.kseg = d->kv_segment_ids ? d->kv_segment_ids + b * n : nullptr;
      a.qpos = d->q_positions ? d->q_positions + b * n : nullptr;
      a.kpos = d->kv_positions ? d->kv_positions + b * n : nullptr;
      attn_softmax_bwd_kernel<<<static_cast<unsigned>(hi * n), kAThreads, 0, s>>>(a);
      cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) return cuda_error(e, "attention softmax backward launch");
    }
    // dQ_g = dS_g K_{g / I}
    rc = gemm_bf16(bop(dS, UFP8_K_MAJOR, n, nn, static_cast<int32_t>(hi)),
                   bop(kB, UFP8_MN_MAJOR, H * Dh, Dh, static_cast<int32_t>(H), static_cast<int32_t>(I)), n, Dh, n,
                   static_cast<int32_t>(hi), 1, dqb + b * n * hi * Dh, 0, hi * Dh, Dh, s, *dev,
                   causal ? UFP8_TILES_K_TO_DIAG : UFP8_TILES_ALL);
    if (rc) return rc;
    // dK_h = sum_i dS_g^T Q_g, dV_h = sum_i P_g^T dO_g: one launch over the kv heads (batch H), the
    // contraction running over the group's query rows (k_batches I, slice h * I + i = g).
    rc = gemm_bf16(bop(dS, UFP8_MN_MAJOR, n, nn, static_cast<int32_t>(hi)),
                       bop(qB, UFP8_MN_MAJOR, hi * Dh, Dh, static_cast<int32_t>(hi)), n, Dh, n,
                       static_cast<int32_t>(H), static_cast<int32_t>(I), dkb + b * n * H * Dh, 0, H * Dh, Dh, s, *dev,
                       causal ? UFP8_TILES_K_FROM_DIAG : UFP8_TILES_ALL);
    if (rc) return rc;
    rc = gemm_bf16(bop(P, UFP8_MN_MAJOR, n, nn, static_cast<int32_t>(hi)),
                   bop(goB, UFP8_MN_MAJOR, hi * Dh, Dh, static_cast<int32_t>(hi)), n, Dh, n,
                   static_cast<int32_t>(H), static_cast<int32_t>(I), dvb + b * n * H * Dh, 0, H * Dh, Dh, s, *dev,
                   causal ? UFP8_TILES_K_FROM_DIAG : UFP8_TILES_ALL);
    if (rc) return rc;
  }
  return UFP8_OK;
}
