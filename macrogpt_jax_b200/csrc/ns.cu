// Newton-Schulz orthogonalisation of Muon (ueaj/opt/multiscale.py:110-141, which vmaps
// optax.contrib orthogonalize_via_newton_schulz (optax 0.2.6, requirements.txt:45) over the leading
// axes of a canonical weight): per slice X [m, n], work on the short side (X^T when m > n),
// X <- X / (||X||_F + eps), then per step with coefficients (a, b, c):
//     A = X X^T,  B = b A + c A A,  X <- a X + B X.
//
// B200 layout of the computation: every product is one launch of the bf16 CTA-pair GEMM
// (tcgen05.mma kind::f16, fp32 accumulation) batched over the slices, and the two updates are its
// AXPBY epilogue (D = alpha acc + beta C), so a step is three GEMMs with no other pass:
//     m <= n:  A = X X^T (both operands K-major);  B = c (A A) + b A;  X' = (B X) + a X (X as an
//              MN-major operand);
//     m >  n:  A = X^T X (both MN-major);          B as above;         X' = (X B) + a X (B taken
//              as B^T: it is symmetric).
// A and B are symmetric, and bitwise so (element (i, j) sums the same products in the same order
// as (j, i)): their GEMMs compute only the 256 x 256 tiles on or below the diagonal
// (UFP8_TILES_LOWER) and a transpose-copy kernel fills the rest, a quarter fewer FLOPs per step
// (3 s^2 l + s^3 instead of 4 s^2 l + 2 s^3 for the short side s and long side l) with the same
// bits.  No transposed copy of X is made.  X, A and B are kept in bf16 between the GEMMs; the last step
// writes the result straight in the output's type (f32 or bf16).  The normalisation is two
// passes: per-slice partial sums of squares (fixed order), then x / (sqrt(sum) + eps) rounded to
// bf16.
#include <cuda_bf16.h>

#include <cmath>
#include <cstring>

#include "internal.h"

namespace ufp8 {
namespace {

constexpr int kNsThreads = 256;
constexpr int kNsParts = 64;  // partial sums per slice

struct NsNormArgs {
  const void* g;
  int g_f32;
  int64_t per_slice;  // m * n
  float* parts;       // [batch][kNsParts]
  float eps;
  __nv_bfloat16* x;
};

__device__ __forceinline__ float g_at(const NsNormArgs& a, int64_t i) {
  return a.g_f32 ? static_cast<const float*>(a.g)[i]
                 : __bfloat162float(static_cast<const __nv_bfloat16*>(a.g)[i]);
}

// grid (kNsParts, batch): CTA p of slice b sums the squares of elements p*256 + t + k*256*kNsParts
// in order, then the CTA sum in a fixed tree.
__global__ void __launch_bounds__(kNsThreads) ns_sumsq_kernel(const NsNormArgs a) {
  const int64_t base = static_cast<int64_t>(blockIdx.y) * a.per_slice;
  float acc = 0.0f;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kNsThreads + threadIdx.x; i < a.per_slice;
       i += static_cast<int64_t>(kNsThreads) * kNsParts) {
    const float v = g_at(a, base + i);
    acc = __fadd_rn(acc, __fmul_rn(v, v));
  }
  __shared__ float red[kNsThreads];
  red[threadIdx.x] = acc;
  __syncthreads();
  for (int o = kNsThreads / 2; o > 0; o >>= 1) {
    if (threadIdx.x < o) red[threadIdx.x] = __fadd_rn(red[threadIdx.x], red[threadIdx.x + o]);
    __syncthreads();
  }
  if (threadIdx.x == 0) a.parts[blockIdx.y * kNsParts + blockIdx.x] = red[0];
}

// x = bf16(g / (||g||_F + eps)); every CTA adds its slice's partials in index order.
__global__ void __launch_bounds__(kNsThreads) ns_scale_kernel(const NsNormArgs a) {
  const int64_t base = static_cast<int64_t>(blockIdx.y) * a.per_slice;
  __shared__ float denom;
  if (threadIdx.x == 0) {
    float ss = 0.0f;
    for (int p = 0; p < kNsParts; ++p) ss = __fadd_rn(ss, a.parts[blockIdx.y * kNsParts + p]);
    denom = __fadd_rn(__fsqrt_rn(ss), a.eps);
  }
  __syncthreads();
  const float dn = denom;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kNsThreads + threadIdx.x; i < a.per_slice;
       i += static_cast<int64_t>(gridDim.x) * kNsThreads)
    a.x[base + i] = __float2bfloat16_rn(__fdiv_rn(g_at(a, base + i), dn));
}

int64_t align256(int64_t b) { return (b + 255) / 256 * 256; }

// Fills the tiles UFP8_TILES_LOWER skipped in each [s, s] slice: element (i, j) with
// j / 256 > i / 256 becomes (j, i).  One CTA per 32 x 32 block of the upper part, through shared
// memory (coalesced reads of the source rows, coalesced writes of the destination rows).
__global__ void __launch_bounds__(kNsThreads) ns_mirror_kernel(__nv_bfloat16* m, int64_t s, int64_t ss) {
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * 32, c0 = static_cast<int64_t>(blockIdx.x) * 32;
  if ((c0 >> 8) <= (r0 >> 8)) return;  // computed by the GEMM (also the whole diagonal tile)
  __shared__ __nv_bfloat16 t[32][33];
  __nv_bfloat16* base = m + static_cast<int64_t>(blockIdx.z) * ss;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
  for (int k = ty; k < 32; k += 8) {  // source rows c0 + k, columns r0 + tx
    const int64_t i = c0 + k, j = r0 + tx;
    if (i < s && j < s) t[k][tx] = base[i * s + j];
  }
  __syncthreads();
  for (int k = ty; k < 32; k += 8) {  // destination rows r0 + k, columns c0 + tx
    const int64_t i = r0 + k, j = c0 + tx;
    if (i < s && j < s) base[i * s + j] = t[tx][k];
  }
}

struct NsLayout {
  int64_t x0, x1, A, B, parts, total;
};

NsLayout ns_layout(int64_t batch, int64_t m, int64_t n) {
  const int64_t s = m <= n ? m : n;
  NsLayout L{};
  const int64_t xb = align256(batch * m * n * 2), sb = align256(batch * s * s * 2);
  L.x0 = 0;
  L.x1 = L.x0 + xb;
  L.A = L.x1 + xb;
  L.B = L.A + sb;
  L.parts = L.B + sb;
  L.total = L.parts + align256(batch * kNsParts * 4);
  return L;
}

ufp8_operand bf16_operand(const void* p, int major, int64_t ld, int64_t bstride, int64_t batch) {
  ufp8_operand o{};
  o.ptr = p;
  o.fmt = UFP8_BF16;
  o.major = major;
  o.ld = ld;
  o.batch_stride = bstride;
  o.batch_count = static_cast<int32_t>(batch);
  o.inv_scale = nullptr;
  return o;
}

}  // namespace
}  // namespace ufp8

using namespace ufp8;

extern "C" int ufp8_newton_schulz_workspace(int64_t batch, int64_t m, int64_t n, int64_t* bytes) {
  if (!bytes) return set_error(UFP8_ERR_INVALID, "ufp8_newton_schulz_workspace: null pointer");
  if (batch < 0 || m < 1 || n < 1) return set_error(UFP8_ERR_INVALID, "ufp8_newton_schulz_workspace: bad shape");
  *bytes = ns_layout(batch, m, n).total;
  return UFP8_OK;
}

extern "C" int ufp8_newton_schulz(const void* g, int g_dtype, int64_t batch, int64_t m, int64_t n, int steps,
                                  const float* coeffs, float eps, void* out, int out_dtype, void* workspace,
                                  int64_t workspace_bytes, ufp8_stream_t stream) {
  const char* who = "ufp8_newton_schulz";
  if (batch < 0 || m < 1 || n < 1) return set_error(UFP8_ERR_INVALID, "%s: batch must be >= 0, m and n >= 1", who);
  if (g_dtype != UFP8_OUT_F32 && g_dtype != UFP8_OUT_BF16)
    return set_error(UFP8_ERR_INVALID, "%s: g_dtype must be UFP8_OUT_F32 or UFP8_OUT_BF16", who);
  if (out_dtype != UFP8_OUT_F32 && out_dtype != UFP8_OUT_BF16)
    return set_error(UFP8_ERR_INVALID, "%s: out_dtype must be UFP8_OUT_F32 or UFP8_OUT_BF16", who);
  if (steps < 1 || steps > 64 || !coeffs) return set_error(UFP8_ERR_INVALID, "%s: steps must be 1..64 with coeffs", who);
  if (m % 8 || n % 8)
    return set_error(UFP8_ERR_UNSUPPORTED, "%s: m and n must be multiples of 8 (16-byte rows of bf16)", who);
  if (batch > 65535 || m * n >= (int64_t(1) << 40))
    return set_error(UFP8_ERR_INVALID, "%s: too large", who);
  const NsLayout L = ns_layout(batch, m, n);
  if (!workspace || workspace_bytes < L.total)
    return set_error(UFP8_ERR_INVALID, "%s: workspace of %lld bytes needed", who, static_cast<long long>(L.total));
  if (batch > 0 && (!g || !out)) return set_error(UFP8_ERR_INVALID, "%s: null g or out", who);
  if (reinterpret_cast<uintptr_t>(workspace) & 255u)
    return set_error(UFP8_ERR_ALIGN, "%s: workspace not 256-byte aligned", who);
  if (reinterpret_cast<uintptr_t>(out) & 15u) return set_error(UFP8_ERR_ALIGN, "%s: out not 16-byte aligned", who);
  if (reinterpret_cast<uintptr_t>(g) & (g_dtype == UFP8_OUT_F32 ? 3u : 1u))
    return set_error(UFP8_ERR_ALIGN, "%s: g misaligned", who);
  for (int i = 0; i < 3 * steps; ++i)
    if (!std::isfinite(coeffs[i])) return set_error(UFP8_ERR_INVALID, "%s: non-finite coefficient", who);
  if (batch == 0) return UFP8_OK;
  DeviceInfo* dev;
  if (int rc = device_info(&dev)) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  __nv_bfloat16* X[2] = {reinterpret_cast<__nv_bfloat16*>(ws + L.x0), reinterpret_cast<__nv_bfloat16*>(ws + L.x1)};
  __nv_bfloat16* A = reinterpret_cast<__nv_bfloat16*>(ws + L.A);
  __nv_bfloat16* B = reinterpret_cast<__nv_bfloat16*>(ws + L.B);

  NsNormArgs na{};
  na.g = g;
  na.g_f32 = g_dtype == UFP8_OUT_F32;
  na.per_slice = m * n;
  na.parts = reinterpret_cast<float*>(ws + L.parts);
  na.eps = eps;
  na.x = X[0];
  ns_sumsq_kernel<<<dim3(kNsParts, static_cast<unsigned>(batch)), kNsThreads, 0, s>>>(na);
  const int64_t blocks = (m * n + kNsThreads - 1) / kNsThreads;
  ns_scale_kernel<<<dim3(static_cast<unsigned>(blocks < 1024 ? blocks : 1024), static_cast<unsigned>(batch)),
                    kNsThreads, 0, s>>>(na);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, "newton-schulz normalisation launch");

  const bool tr = m > n;            // work on X^T
  const int64_t sd = tr ? n : m;    // short side
  const int64_t mn = m * n, ss = sd * sd;
  const dim3 mgrid(static_cast<unsigned>((sd + 31) / 32), static_cast<unsigned>((sd + 31) / 32),
                   static_cast<unsigned>(batch));
  auto mirror = [&](__nv_bfloat16* mat) -> int {
    if (sd <= 256) return UFP8_OK;  // one diagonal tile: nothing skipped
    ns_mirror_kernel<<<mgrid, kNsThreads, 0, s>>>(mat, sd, ss);
    const cudaError_t me = cudaGetLastError();
    return me == cudaSuccess ? UFP8_OK : cuda_error(me, "newton-schulz mirror launch");
  };
  for (int it = 0; it < steps; ++it) {
    const float ca = coeffs[3 * it], cb = coeffs[3 * it + 1], cc = coeffs[3 * it + 2];
    const __nv_bfloat16* Xc = X[it & 1];
    const bool last = it == steps - 1;
    void* Xn = last ? out : X[(it + 1) & 1];
    // A = X X^T (m <= n) or X^T X (m > n): [sd, sd], contraction over the long side.
    ufp8_gemm_desc d{};
    d.M = sd;
    d.N = sd;
    d.K = tr ? m : n;
    d.batch = static_cast<int32_t>(batch);
    d.k_batches = 1;
    d.a = bf16_operand(Xc, tr ? UFP8_MN_MAJOR : UFP8_K_MAJOR, n, mn, batch);
    d.b = d.a;
    d.d = A;
    d.d_dtype = UFP8_OUT_BF16;
    d.epilogue = UFP8_EPI_STORE;
    d.ldd = sd;
    d.d_batch_stride = ss;
    d.tile_mask = UFP8_TILES_LOWER;
    if (int rc = launch_gemm(d, s, *dev, 0, UFP8_GEMM_AUTO, 0)) return rc;
    if (int rc = mirror(A)) return rc;
    // B = c (A A) + b A   (A symmetric: its transpose is itself, a K-major B operand)
    d = ufp8_gemm_desc{};
    d.M = sd;
    d.N = sd;
    d.K = sd;
    d.batch = static_cast<int32_t>(batch);
    d.k_batches = 1;
    d.a = bf16_operand(A, UFP8_K_MAJOR, sd, ss, batch);
    d.b = d.a;
    d.d = B;
    d.d_dtype = UFP8_OUT_BF16;
    d.epilogue = UFP8_EPI_AXPBY;
    d.ldd = sd;
    d.d_batch_stride = ss;
    d.c = A;
    d.ldc = sd;
    d.c_batch_stride = ss;
    d.alpha = cc;
    d.beta = cb;
    d.tile_mask = UFP8_TILES_LOWER;
    if (int rc = launch_gemm(d, s, *dev, 0, UFP8_GEMM_AUTO, 0)) return rc;
    if (int rc = mirror(B)) return rc;
    // X' = (B X) + a X  (m <= n)   or   X' = (X B) + a X  (m > n)
    d = ufp8_gemm_desc{};
    d.M = m;
    d.N = n;
    d.K = sd;
    d.batch = static_cast<int32_t>(batch);
    d.k_batches = 1;
    if (!tr) {
      d.a = bf16_operand(B, UFP8_K_MAJOR, sd, ss, batch);
      d.b = bf16_operand(Xc, UFP8_MN_MAJOR, n, mn, batch);
    } else {
      d.a = bf16_operand(Xc, UFP8_K_MAJOR, n, mn, batch);
      d.b = bf16_operand(B, UFP8_K_MAJOR, sd, ss, batch);
    }
    d.d = Xn;
    d.d_dtype = last ? out_dtype : UFP8_OUT_BF16;
    d.epilogue = UFP8_EPI_AXPBY;
    d.ldd = n;
    d.d_batch_stride = mn;
    d.c = Xc;
    d.ldc = n;
    d.c_batch_stride = mn;
    d.alpha = 1.0f;
    d.beta = ca;
    if (int rc = launch_gemm(d, s, *dev, 0, UFP8_GEMM_AUTO, 0)) return rc;
  }
  return UFP8_OK;
}
