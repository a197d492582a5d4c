// Persistent, warp-specialised FP8 GEMMs for sm_100a (tcgen05 + TMEM + TMA).
//
//   D[g][m][n] = alpha * sum_k A[m][k] * B[n][k],  alpha = inv_scale_a * inv_scale_b
//
// Two kernels: gemm_fp8_pair_kernel (the default; further down) computes 256x256 tiles on a
// cluster of two CTAs with tcgen05.mma.cta_group::2, in three instantiations that differ only
// in how the epilogue moves data (direct stores; U/G of the dSwiGLU epilogue staged by TMA;
// reduce-scatter rows pushed to peer GPUs by bulk stores).  gemm_fp8_kernel, described next,
// is the one-CTA variant (UFP8_GEMM_SINGLE_CTA), kept for comparison and for the tests.
//
// One-CTA kernel: one CTA per SM (192 threads, ~193 KB shared memory, all 512 TMEM columns):
//   warp 0      TMA producer: 4-stage ring of {A 128x128, B 256x128} fp8 tiles in
//               128-byte-swizzled shared memory (plain per-CTA tiled loads);
//   warp 1      MMA issuer: one elected thread issues tcgen05.mma.cta_group::1.kind::f8f6f4
//               (M=128, N=256, K=32) into a double-buffered fp32 TMEM accumulator
//               (2 x 256 columns) and frees ring slots with tcgen05.commit;
//   warps 2..5  epilogue: tcgen05.ld (32 lanes x 32 columns), scale, bf16/f32 cast and the
//               fused GMLP math, 16-byte global stores; overlaps the next tile's MMAs.
// Operands may be K-major or MN-major (both legal for e4m3/e5m2 on tcgen05), so the
// backward contractions over tokens read the row-major activations directly and no
// transposed copy is ever made.  Every mbarrier wait is bounded (see ptx.cuh).
#include <cuda_bf16.h>

#include <algorithm>
#include <cmath>
#include <cstring>

#include "internal.h"
#include "ptx.cuh"

namespace ufp8 {
namespace {

// 3-D tiled bulk tensor store from this CTA's shared memory (bulk-group completion).
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* smem_src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(x), "r"(y), "r"(z)
               : "memory");
}

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 128;  // bytes of K per stage = one 128-byte swizzle atom row
constexpr int kStages = 4;
constexpr int kTileBytesA = kBM * kBK;                      // 16 KiB
constexpr int kHalfBytesB = 128 * kBK;                      // 16 KiB: 128 rows of B
constexpr int kStageBytes = kTileBytesA + 2 * kHalfBytesB;  // 48 KiB
constexpr int kThreads = 192;
constexpr int kTmemCols = 512;
constexpr int kBarrierBytes = 256;
constexpr int kSmemBytes = kStages * kStageBytes + kBarrierBytes + 1024;  // + alignment slack

struct GemmArgs {
  int M, N, K;
  int batch, k_batches, mode;
  int a_major, b_major, a_bcast, b_bcast;
  int a_group, b_group;  // GEMM batch g reads operand slice g / group (k_batches == 1)
  int tiles_m, tiles_n, ksteps;
  uint32_t idesc;
  const float* inv_a;
  const float* inv_b;
  void* d;
  int d_f32;
  int vec_ok;
  long long ldd, d_bstride;
  __nv_bfloat16* h;
  long long ldh;
  const __nv_bfloat16* ug;
  long long ldug, ug_bstride;
  unsigned int* amax_bits;
  int* status;
  int group_m;  // tile raster: M tiles per group swept before moving along N
  int m_shift;  // rotation of the M tile index (RS_PUSH: start at this rank's own rows)
  void* const* rs_slots;  // RS_PUSH: owners' staging slots
  int rs_rank;
  long long rs_rows;
  const uint32_t* ag_flags;  // all-gathered A: arrival flags per source rank (null = none)
  uint32_t ag_epoch;
  int ag_rank;
  long long ag_rows;
  float* xent_stats;  // XENT: per-row (max, sum exp) of each 128-column group
  long long xent_ld;
  float xent_cap;     // XENT: soft cap (0 = none)
  const __nv_bfloat16* c;  // AXPBY (bf16 operands): D = alpha * acc * sa * sb + beta * C
  long long ldc, c_bstride;
  float alpha_mul, beta;
  int c_vec;  // AXPBY: C rows 16-byte aligned
  int tile_mask;  // UFP8_TILES_* (bf16 operands only)
  // UFP8_EPI_ATTN_* (bf16 operands): segment ids of rows / columns, STATS partials, the per-row
  // value (lse for P, rowsum(dO O) for DS), P for DS (pitch ldc, slice pitch c_bstride), scale.
  const int32_t* attn_qseg;
  const int32_t* attn_kseg;
  float* attn_stats;
  long long attn_ld;
  const float* attn_row;
  const __nv_bfloat16* attn_p;
  float attn_scale;
  int attn_kseg_vec;  // column ids readable as int4
};

// The tiles of a masked bf16 GEMM (UFP8_TILES_*): whether M tile mb / N tile nb runs, and its k-step
// range [lo, hi) within each K slice (k-steps of `step` elements; tiles are 256 x 256).
__device__ __forceinline__ bool masked_tile(const GemmArgs& a, int mb, int nb, int step, int& lo, int& hi) {
  lo = 0;
  hi = a.ksteps;
  if (a.tile_mask == UFP8_TILES_LOWER) return nb <= mb;
  if (a.tile_mask == UFP8_TILES_K_TO_DIAG) {
    const int e = (mb + 1) * 2 * kBM;
    hi = min(hi, (e + step - 1) / step);
  } else if (a.tile_mask == UFP8_TILES_K_FROM_DIAG) {
    lo = (mb * 2 * kBM) / step;
  }
  return hi > lo;
}

// Waits until the all-gather block of rank s has arrived (flag == epoch), bounded like the
// pipeline waits; on expiry raises abort_flag and the peer-timeout status bit.  After the
// acquire, a proxy fence orders the TMA (async-proxy) reads of the block after it.
__device__ __forceinline__ bool ag_wait(const GemmArgs& a, int s, volatile int* abort_flag) {
  const uint32_t* f = a.ag_flags + s;
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
  if (v != a.ag_epoch) {
    const uint64_t t0 = globaltimer_ns();
    while (true) {
      asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
      if (v == a.ag_epoch) break;
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
        *abort_flag = 1;
        atomicOr(a.status, UFP8_STATUS_PEER_TIMEOUT);
        return false;
      }
    }
  }
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  asm volatile("fence.proxy.async.global;" ::: "memory");
  return true;
}

__device__ __forceinline__ void map_tile(int tile, const GemmArgs& a, int& g, int& mb, int& nb) {
  const int tpb = a.tiles_m * a.tiles_n;
  g = tile / tpb;
  const int r = tile - g * tpb;
  const int span = a.group_m * a.tiles_n;
  const int grp = r / span;
  const int first_m = grp * a.group_m;
  const int gm = min(a.tiles_m - first_m, a.group_m);
  const int rr = r - grp * span;
  mb = first_m + rr % gm;
  nb = rr / gm;
  mb += a.m_shift;
  if (mb >= a.tiles_m) mb -= a.tiles_m;
}

__device__ __forceinline__ uint32_t bf16_bits(float v) {
  return static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(v)));
}
__device__ __forceinline__ float bf16_round(float v) { return __uint_as_float(bf16_bits(v) << 16); }
__device__ __forceinline__ float bf16_to_f(uint32_t bits16) { return __uint_as_float(bits16 << 16); }

// Logistic function for the gating epilogues: MUFU exp2 and approximate reciprocal (a few
// ulp, far below bf16 resolution).  g << 0 gives 1 + inf -> 0, g >> 0 gives 1.
__device__ __forceinline__ float sigmoidf_(float g) { return __fdividef(1.0f, 1.0f + __expf(-g)); }

// Stores 32 consecutive bf16 values (bit patterns in the low halves of v[]) at p;
// columns at or past `valid` are skipped.  Vector path when the whole run is in range.
__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* p, const uint32_t (&v)[32], int valid, bool vec) {
  if (vec && valid >= 32) {
    uint4* q = reinterpret_cast<uint4*>(p);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint4 o;
      o.x = v[8 * i + 0] | (v[8 * i + 1] << 16);
      o.y = v[8 * i + 2] | (v[8 * i + 3] << 16);
      o.z = v[8 * i + 4] | (v[8 * i + 5] << 16);
      o.w = v[8 * i + 6] | (v[8 * i + 7] << 16);
      q[i] = o;
    }
  } else {
    uint16_t* q = reinterpret_cast<uint16_t*>(p);
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < valid) q[j] = static_cast<uint16_t>(v[j]);
  }
}

__device__ __forceinline__ void load_bf16x32(const __nv_bfloat16* p, uint32_t (&v)[32], int valid, bool vec) {
  if (vec && valid >= 32) {
    const uint4* q = reinterpret_cast<const uint4*>(p);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 w = q[i];
      v[8 * i + 0] = w.x & 0xFFFFu; v[8 * i + 1] = w.x >> 16;
      v[8 * i + 2] = w.y & 0xFFFFu; v[8 * i + 3] = w.y >> 16;
      v[8 * i + 4] = w.z & 0xFFFFu; v[8 * i + 5] = w.z >> 16;
      v[8 * i + 6] = w.w & 0xFFFFu; v[8 * i + 7] = w.w >> 16;
    }
  } else {
    const uint16_t* q = reinterpret_cast<const uint16_t*>(p);
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = j < valid ? q[j] : 0u;
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    gemm_fp8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_tiles = args.tiles_m * args.tiles_n * args.batch;
  const int total_k = args.ksteps * args.k_batches;
  const bool swiglu = args.mode == UFP8_EPI_SWIGLU;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0, armed_parity = 0;  // per-stage bookkeeping for the abort drain
      for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
        int g, mb, nb;
        map_tile(tile, args, g, mb, nb);
        for (int ks = 0; ks < total_k; ++ks) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) break;
          const int kb = ks / args.ksteps;
          const int k0 = (ks - kb * args.ksteps) * kBK;
          uint8_t* sa = smem + stage * kStageBytes;
          uint8_t* sb = sa + kTileBytesA;
          mbar_arrive_expect_tx(&full[stage], kStageBytes);
          armed |= 1u << stage;
          armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
          const int az = args.a_bcast ? 0 : (args.k_batches > 1 ? g * args.k_batches + kb : g / args.a_group);
          if (args.a_major == UFP8_K_MAJOR)
            tma_load_3d(sa, &tmA, &full[stage], k0, mb * kBM, az);
          else
            tma_load_3d(sa, &tmA, &full[stage], mb * kBM, k0, az);
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            int n0, bz;
            if (swiglu) {
              n0 = nb * 128;
              bz = half;
            } else {
              n0 = nb * kBN + half * 128;
              bz = args.b_bcast ? 0 : (args.k_batches > 1 ? g * args.k_batches + kb : g / args.b_group);
            }
            if (args.b_major == UFP8_K_MAJOR)
              tma_load_3d(sb + half * kHalfBytesB, &tmB, &full[stage], k0, n0, bz);
            else
              tma_load_3d(sb + half * kHalfBytesB, &tmB, &full[stage], n0, k0, bz);
          }
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (*abort_flag) {
        // Let every load this thread issued land before the CTA can exit.
        volatile int never = 0;
        for (int s = 0; s < kStages; ++s)
          if (armed & (1u << s)) mbar_wait(&full[s], (armed_parity >> s) & 1u, &never);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x, ++local) {
        const int buf = local & 1;
        const uint32_t tphase = (local >> 1) & 1;
        if (!mbar_wait(&tempty[buf], tphase ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * kBN);
        bool ok = true;
        for (int ks = 0; ks < total_k; ++ks) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * kStageBytes);
          const uint32_t sb = sa + kTileBytesA;
#pragma unroll
          for (int kk = 0; kk < kBK / 32; ++kk) {
            const uint64_t adesc = args.a_major == UFP8_K_MAJOR
                                       ? make_sdesc_sw128(sa + kk * 32, 16, 1024)
                                       : make_sdesc_sw128(sa + kk * 32 * 128, kHalfBytesB, 1024);
            const uint64_t bdesc = args.b_major == UFP8_K_MAJOR
                                       ? make_sdesc_sw128(sb + kk * 32, 16, 1024)
                                       : make_sdesc_sw128(sb + kk * 32 * 128, kHalfBytesB, 1024);
            umma_f8f6f4(d_tmem, adesc, bdesc, args.idesc, (ks | kk) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[buf]);
      }
      // All MMAs this thread issued must finish before TMEM is released.
      umma_commit(drain);
      volatile int never = 0;
      mbar_wait(drain, 0, &never);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ epilogue
    const int quad = warp & 3;  // TMEM lanes this warp may read: [32*quad, 32*quad+32)
    const int row_in_tile = quad * 32 + lane;
    const float alpha = __fmul_rn(*args.inv_a, *args.inv_b);
    const int vec = args.vec_ok;
    uint32_t amax = 0;  // max |value| over bf16 bit patterns written by this thread
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int buf = local & 1;
      const uint32_t tphase = (local >> 1) & 1;
      bool ok = mbar_wait(&tfull[buf], tphase, abort_flag);
      ok = __all_sync(0xFFFFFFFFu, ok);
      if (!ok) break;
      tc_fence_after();
      int g, mb, nb;
      map_tile(tile, args, g, mb, nb);
      const int row = mb * kBM + row_in_tile;
      const bool row_ok = row < args.M;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(buf * kBN);

      if (args.mode == UFP8_EPI_STORE) {
#pragma unroll 1
        for (int c = 0; c < kBN; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tbase + c, r);
          tmem_ld_wait();
          const int col0 = nb * kBN + c;
          if (row_ok && col0 < args.N) {
            const int valid = args.N - col0;
            if (args.d_f32) {
              float* p = static_cast<float*>(args.d) + g * args.d_bstride + row * args.ldd + col0;
              if (vec && valid >= 32) {
#pragma unroll
                for (int i = 0; i < 8; ++i)
                  reinterpret_cast<float4*>(p)[i] =
                      make_float4(__uint_as_float(r[4 * i]) * alpha, __uint_as_float(r[4 * i + 1]) * alpha,
                                  __uint_as_float(r[4 * i + 2]) * alpha, __uint_as_float(r[4 * i + 3]) * alpha);
              } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (j < valid) p[j] = __uint_as_float(r[j]) * alpha;
              }
            } else {
              uint32_t o[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) o[j] = bf16_bits(__uint_as_float(r[j]) * alpha);
              __nv_bfloat16* p = static_cast<__nv_bfloat16*>(args.d) + g * args.d_bstride + row * args.ldd + col0;
              store_bf16x32(p, o, valid, vec);
            }
          }
        }
      } else if (args.mode == UFP8_EPI_SWIGLU) {
        // TMEM columns [0,128) hold up, [128,256) hold gate for hidden units nb*128 + c.
#pragma unroll 1
        for (int c = 0; c < 128; c += 32) {
          uint32_t ru[32], rg[32];
          tmem_ld_32x32b_x32(tbase + c, ru);
          tmem_ld_32x32b_x32(tbase + 128 + c, rg);
          tmem_ld_wait();
          const int col0 = nb * 128 + c;
          if (row_ok && col0 < args.N) {
            const int valid = args.N - col0;
            uint32_t oh[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const uint32_t ub = bf16_bits(__uint_as_float(ru[j]) * alpha);
              const uint32_t gb = bf16_bits(__uint_as_float(rg[j]) * alpha);
              const float u = bf16_to_f(ub), gt = bf16_to_f(gb);
              const float hv = u * (gt * sigmoidf_(gt));
              const uint32_t hb = bf16_bits(hv);
              ru[j] = ub;
              rg[j] = gb;
              oh[j] = hb;
              if (j < valid) amax = max(amax, hb & 0x7FFFu);
            }
            __nv_bfloat16* pu = static_cast<__nv_bfloat16*>(args.d) + row * args.ldd + col0;
            store_bf16x32(pu, ru, valid, vec);
            store_bf16x32(pu + args.d_bstride, rg, valid, vec);
            store_bf16x32(args.h + row * args.ldh + col0, oh, valid, vec);
          }
        }
      } else {  // UFP8_EPI_DSWIGLU
#pragma unroll 1
        for (int c = 0; c < kBN; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tbase + c, r);
          tmem_ld_wait();
          const int col0 = nb * kBN + c;
          if (row_ok && col0 < args.N) {
            const int valid = args.N - col0;
            uint32_t u16[32], g16[32];
            const __nv_bfloat16* pu = args.ug + row * args.ldug + col0;
            load_bf16x32(pu, u16, valid, vec);
            load_bf16x32(pu + args.ug_bstride, g16, valid, vec);
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float dh = bf16_round(__uint_as_float(r[j]) * alpha);
              const float u = bf16_to_f(u16[j]), gt = bf16_to_f(g16[j]);
              const float sg = sigmoidf_(gt);
              const float du = dh * (gt * sg);
              const float dg = (dh * u) * (sg * (1.0f + gt * (1.0f - sg)));
              u16[j] = bf16_bits(du);
              g16[j] = bf16_bits(dg);
              if (j < valid) amax = max(amax, max(u16[j] & 0x7FFFu, g16[j] & 0x7FFFu));
            }
            __nv_bfloat16* pd = static_cast<__nv_bfloat16*>(args.d) + row * args.ldd + col0;
            store_bf16x32(pd, u16, valid, vec);
            store_bf16x32(pd + args.d_bstride, g16, valid, vec);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[buf]);
    }
    if (args.amax_bits != nullptr) {
      amax = __reduce_max_sync(0xFFFFFFFFu, amax);
      if (lane == 0 && amax != 0u) atomicMax(args.amax_bits, amax << 16);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicOr(args.status, UFP8_STATUS_WAIT_TIMEOUT);
}

// ============================================================================= CTA-pair kernel
// Same contraction with 2-CTA MMAs: a cluster of two CTAs computes a 256 x 256 tile, each CTA
// holding 128 rows of A and 128 rows (N) of B per stage, so a CTA streams 32 KiB per 128-deep
// k-step instead of 48 KiB and six stages fit in shared memory.  The even CTA's MMA thread
// issues tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 32) and signals its commits to
// both CTAs' barriers; both CTAs' loads complete on the even CTA's "full" barrier.  Eight
// epilogue warps per CTA (two per TMEM lane quadrant, splitting the columns).
//
// The RS_PUSH instantiation (STAGED) trades two ring stages for a per-warp staging area:
// each epilogue warp converts 64 columns of its 32 rows into shared memory (rows padded to
// 144 B, so the 16-byte writes of a warp spread over all banks) and every lane then sends
// its own 128-byte row segment with one cp.async.bulk store.  Stores into a peer GPU's
// memory then leave as bulk transfers issued by the copy engine of the SM, not as 16-byte
// writes that stall the epilogue warp (plain remote stores reach ~170 GB/s; bulk ones run
// at link rate), and the warp moves on as soon as the row has been read out of shared memory.
constexpr int kPStages = 7;
constexpr int kPStagesStaged = 5;
constexpr int kPStagesWide = 3;                   // ring depth with two 128-byte K chunks per stage
constexpr int kPHalfBytes = 128 * kBK;            // 16 KiB: 128 rows x 128 B
constexpr int kPStageBytes = 2 * kPHalfBytes;     // A half + B half (one 128-byte K chunk)
constexpr int kPEpiWarps = 8;
constexpr int kPThreads = 64 + 32 * kPEpiWarps;   // 320
constexpr int kPStgCols = 64;                     // columns per staged row segment
constexpr int kPStgStride = kPStgCols * 2 + 16;   // 144 B: padded row pitch
constexpr int kPStgWarpBytes = 32 * kPStgStride;  // 4.5 KiB per epilogue warp
constexpr int kPStgBytes = kPEpiWarps * kPStgWarpBytes;
//
// The DSWIGLU instantiation (kVarUgStaged) likewise gives up two ring stages so that the saved
// U / G the gating backward reads arrive by TMA instead of by per-thread global loads: each
// epilogue warp streams 32-row x 32-column bf16 boxes of U and G (64-byte swizzle, so the
// lanes' 16-byte reads of their own rows are bank-conflict free) into a double buffer two
// chunks ahead of its TMEM reads, including across tiles, so the loads of the next tile run
// while this tile's MMAs are still in flight.  dU / dG overwrite the U / G granules they were
// computed from and leave by TMA stores of the same boxes (a tensor map over D [2][M][N]), so
// the epilogue warps issue no global stores either.
constexpr int kVarDirect = 0;     // every epilogue, plain stores from registers
constexpr int kVarRsStaged = 1;   // RS_PUSH rows through shared memory, bulk stores
constexpr int kVarUgStaged = 2;   // DSWIGLU with U / G staged by TMA
constexpr int kPUgCols = 32;                        // columns per U / G chunk
constexpr int kPUgBoxBytes = 32 * kPUgCols * 2;     // 2 KiB: 32 rows x 32 bf16
constexpr int kPUgBufBytes = 2 * kPUgBoxBytes;      // U box + G box
constexpr int kPUgWarpBytes = 2 * kPUgBufBytes;     // double buffer: 8 KiB per warp
constexpr int kPUgBytes = kPEpiWarps * kPUgWarpBytes + 256;  // + the warps' mbarriers
__host__ __device__ constexpr int pair_extra_bytes(int var) {
  return var == kVarRsStaged ? kPStgBytes : (var == kVarUgStaged ? kPUgBytes : 0);
}
__host__ __device__ constexpr int pair_smem_bytes(int stages, int var, int kch = 1) {
  return stages * kch * kPStageBytes + pair_extra_bytes(var) + kBarrierBytes + 1024;
}
constexpr int kPSmemBytes = pair_smem_bytes(kPStages, kVarDirect);
constexpr int kPSmemBytesWide = pair_smem_bytes(kPStagesWide, kVarDirect, 2);
constexpr int kPStagesWideStaged = 2;  // beside the RS rows (36 KiB) or U/G boxes (64 KiB)
constexpr int kPSmemBytesWideStaged = pair_smem_bytes(kPStagesWideStaged, kVarRsStaged, 2);
constexpr int kPSmemBytesWideUg = pair_smem_bytes(kPStagesWideStaged, kVarUgStaged, 2);
constexpr int kPSmemBytesStaged = pair_smem_bytes(kPStagesStaged, kVarRsStaged);
constexpr int kPSmemBytesUg = pair_smem_bytes(kPStagesStaged, kVarUgStaged);
static_assert(kPSmemBytesStaged <= 232448, "staged CTA-pair kernel exceeds shared memory");
static_assert(kPSmemBytesUg <= 232448, "U/G-staged CTA-pair kernel exceeds shared memory");
static_assert(kPSmemBytes <= 232448, "CTA-pair kernel exceeds shared memory");
static_assert(kPSmemBytesWide <= 232448, "wide-stage CTA-pair kernel exceeds shared memory");
static_assert(kPSmemBytesWideStaged <= 232448, "wide-stage RS kernel exceeds shared memory");
static_assert(kPSmemBytesWideUg <= 232448, "wide-stage U/G kernel exceeds shared memory");

// Stores 32 consecutive bf16 values packed two per word (element 2j in the low half of w[j]).
__device__ __forceinline__ void store_bf16x32_packed(__nv_bfloat16* p, const uint32_t (&w)[16], int valid,
                                                     bool vec) {
  if (vec && valid >= 32) {
    uint4* q = reinterpret_cast<uint4*>(p);
#pragma unroll
    for (int i = 0; i < 4; ++i) q[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
  } else {
    uint16_t* q = reinterpret_cast<uint16_t*>(p);
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < valid) q[j] = static_cast<uint16_t>((j & 1) ? (w[j >> 1] >> 16) : (w[j >> 1] & 0xFFFFu));
  }
}

// Stores 16 consecutive bf16 values packed two per word.
__device__ __forceinline__ void store_bf16x16_packed(__nv_bfloat16* p, const uint32_t (&w)[8], int valid,
                                                     bool vec) {
  if (vec && valid >= 16) {
    uint4* q = reinterpret_cast<uint4*>(p);
    q[0] = make_uint4(w[0], w[1], w[2], w[3]);
    q[1] = make_uint4(w[4], w[5], w[6], w[7]);
  } else {
    uint16_t* q = reinterpret_cast<uint16_t*>(p);
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (j < valid) q[j] = static_cast<uint16_t>((j & 1) ? (w[j >> 1] >> 16) : (w[j >> 1] & 0xFFFFu));
  }
}

// vec: 0 = element stores, 1 = 16-byte stores (16-byte aligned rows), 2 = 32-byte stores
// (32-byte aligned rows).
__device__ __forceinline__ void store_bf16x16_packed_h(__nv_bfloat16* p, const uint32_t (&w)[8], int valid,
                                                       int vec, uint64_t pol) {
  if (vec >= 2 && valid >= 16) {
    st_global_v8_hint(p, make_uint4(w[0], w[1], w[2], w[3]), make_uint4(w[4], w[5], w[6], w[7]), pol);
  } else if (vec && valid >= 16) {
    st_global_v4_hint(p, make_uint4(w[0], w[1], w[2], w[3]), pol);
    st_global_v4_hint(p + 8, make_uint4(w[4], w[5], w[6], w[7]), pol);
  } else {
    store_bf16x16_packed(p, w, valid, vec);
  }
}

__device__ __forceinline__ void store_bf16x32_packed_h(__nv_bfloat16* p, const uint32_t (&w)[16], int valid,
                                                       int vec, uint64_t pol) {
  if (vec >= 2 && valid >= 32) {
    st_global_v8_hint(p, make_uint4(w[0], w[1], w[2], w[3]), make_uint4(w[4], w[5], w[6], w[7]), pol);
    st_global_v8_hint(p + 16, make_uint4(w[8], w[9], w[10], w[11]), make_uint4(w[12], w[13], w[14], w[15]), pol);
  } else if (vec && valid >= 32) {
#pragma unroll
    for (int i = 0; i < 4; ++i) st_global_v4_hint(p + 8 * i, make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]), pol);
  } else {
    store_bf16x32_packed(p, w, valid, vec);
  }
}

// Two floats -> packed bf16x2 (lo in the low half) with one cvt.rn.bf16x2.f32.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}
__device__ __forceinline__ float lo_f(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi_f(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// XENT epilogue, one 32-column chunk of a row (bf16 logits packed in o[]): applies the soft cap
// c = bf16(cap * bf16(tanh(bf16(l / cap)))) when cap > 0 (bf16 rounding after each operation, as
// the reference's bf16 expression 15 * jnp.tanh(logits / 15) computes it), then folds the chunk's
// columns below `valid` into the running softmax partials (m = max c, s = sum exp(c - m)),
// rescaling s when the maximum grows.  exp is the MUFU approximation (a few ulp).  A NaN logit
// leaves m alone and makes s NaN, so the row's loss becomes NaN.
__device__ __forceinline__ void xent_chunk(uint32_t (&o)[16], int valid, float cap, float& m, float& s) {
  if (cap > 0.0f) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float t0 = bf16_round(tanhf(bf16_round(__fdiv_rn(lo_f(o[j]), cap))));
      const float t1 = bf16_round(tanhf(bf16_round(__fdiv_rn(hi_f(o[j]), cap))));
      o[j] = pack_bf16x2(cap * t0, cap * t1);
    }
  }
  float cm = -INFINITY;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    if (2 * j < valid) cm = fmaxf(cm, lo_f(o[j]));
    if (2 * j + 1 < valid) cm = fmaxf(cm, hi_f(o[j]));
  }
  if (cm > m) {
    s = s * __expf(m - cm);  // m = -inf on the first chunk: s = 0 * 0
    m = cm;
  }
  float acc = 0.0f;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    if (2 * j < valid) acc += __expf(lo_f(o[j]) - m);
    if (2 * j + 1 < valid) acc += __expf(hi_f(o[j]) - m);
  }
  s += acc;
}

// Loads 16 consecutive bf16 values packed two per word; elements at or past `valid` read 0.
__device__ __forceinline__ void load_bf16x16_packed(const __nv_bfloat16* p, uint32_t (&w)[8], int valid,
                                                    bool vec) {
  if (vec && valid >= 16) {
    const uint4* q = reinterpret_cast<const uint4*>(p);
    const uint4 t0 = q[0], t1 = q[1];
    w[0] = t0.x; w[1] = t0.y; w[2] = t0.z; w[3] = t0.w;
    w[4] = t1.x; w[5] = t1.y; w[6] = t1.z; w[7] = t1.w;
  } else {
    const uint16_t* q = reinterpret_cast<const uint16_t*>(p);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t lo = (2 * j < valid) ? q[2 * j] : 0u;
      const uint32_t hi = (2 * j + 1 < valid) ? q[2 * j + 1] : 0u;
      w[j] = lo | (hi << 16);
    }
  }
}


// One 32-column chunk of an attention epilogue (UFP8_EPI_ATTN_*): accumulators r of row `row`
// (query), columns col0 .. col0 + 31 (keys; `valid` of them below N), batch entry g; sq = the
// row's segment id, rv = its attn_row value.  Column c is visible iff c <= row and its segment id
// equals sq >= 0.  STATS folds the visible x = scale * acc into the running (m, s) of this
// thread's 128 columns; P and DS store 32 bf16 values at d.
__device__ __forceinline__ float attn_ex2(float x) {  // 2^x, the MUFU instruction
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
constexpr float kAttnLog2e = 1.4426950408889634f;

__device__ __forceinline__ uint32_t attn_vis(const GemmArgs& a, int row, int col0, int valid, int sq, bool uni,
                                             uint32_t segmask) {
  uint32_t vis = 0;
  const int lim = min(min(valid, 32), row - col0 + 1);  // causal: columns <= row
  if (sq >= 0 && lim > 0) {
    const uint32_t upto = lim >= 32 ? 0xFFFFFFFFu : ((1u << lim) - 1u);
    if (uni) {  // the warp's rows share sq: segmask = the columns carrying it (one ballot)
      vis = segmask & upto;
    } else if (a.attn_kseg == nullptr) {
      vis = sq == 0 ? upto : 0u;
    } else if (a.attn_kseg_vec && valid >= 32) {
      const int4* kp = reinterpret_cast<const int4*>(a.attn_kseg + col0);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int4 k4 = kp[i];
        vis |= (static_cast<uint32_t>(k4.x == sq) | (static_cast<uint32_t>(k4.y == sq) << 1) |
                (static_cast<uint32_t>(k4.z == sq) << 2) | (static_cast<uint32_t>(k4.w == sq) << 3))
               << (4 * i);
      }
      vis &= upto;
    } else {
#pragma unroll 4
      for (int j = 0; j < 32; ++j)
        if (j < lim && a.attn_kseg[col0 + j] == sq) vis |= 1u << j;
    }
  }
  return vis;
}

// STATS over 64 columns (two 32-column chunks r0, r1 from col0), base 2: the visible
// y = acc * scale * log2(e) fold into the running (m, s) = (max y, sum 2^(y - m)) of this
// thread's 128 columns with one rescale.
__device__ __forceinline__ void attn_stats64(const GemmArgs& a, uint32_t (&r0)[32], uint32_t (&r1)[32], int row,
                                             int col0, int valid, int sq, bool uni, uint32_t sm0, uint32_t sm1,
                                             float& m, float& s) {
  const uint32_t v0 = attn_vis(a, row, col0, valid, sq, uni, sm0);
  const uint32_t v1 = valid > 32 ? attn_vis(a, row, col0 + 32, valid - 32, sq, uni, sm1) : 0u;
  if ((v0 | v1) == 0u) return;
  const float c = a.attn_scale * kAttnLog2e;
  float cm2[2] = {-INFINITY, -INFINITY};  // independent partial maxima / sums (short chains)
  if ((v0 & v1) == 0xFFFFFFFFu) {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float y0 = __uint_as_float(r0[j]) * c, y1 = __uint_as_float(r1[j]) * c;
      r0[j] = __float_as_uint(y0);
      r1[j] = __float_as_uint(y1);
      cm2[j & 1] = fmaxf(cm2[j & 1], fmaxf(y0, y1));
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float y0 = ((v0 >> j) & 1u) ? __uint_as_float(r0[j]) * c : -INFINITY;
      const float y1 = ((v1 >> j) & 1u) ? __uint_as_float(r1[j]) * c : -INFINITY;
      r0[j] = __float_as_uint(y0);
      r1[j] = __float_as_uint(y1);
      cm2[j & 1] = fmaxf(cm2[j & 1], fmaxf(y0, y1));
    }
  }
  const float cm = fmaxf(cm2[0], cm2[1]);
  if (cm > m) {
    s = s * attn_ex2(m - cm);  // m = -inf on the first visible chunk: s = 0 * 0
    m = cm;
  }
  float acc2[2] = {0.0f, 0.0f};
#pragma unroll
  for (int j = 0; j < 32; ++j)  // masked: 2^-inf = 0
    acc2[j & 1] += attn_ex2(__uint_as_float(r0[j]) - m) + attn_ex2(__uint_as_float(r1[j]) - m);
  s += acc2[0] + acc2[1];
}

// P / DS for one 32-column chunk (see attn_vis for the mask), stored as 32 bf16 at d.
__device__ __forceinline__ void attn_chunk(const GemmArgs& a, const uint32_t (&r)[32], int row, int col0, int valid,
                                           int g, int sq, float rv, __nv_bfloat16* d, int vec, uint64_t pol,
                                           bool uni, uint32_t segmask) {
  const uint32_t vis = a.mode == UFP8_EPI_ATTN_P ? attn_vis(a, row, col0, valid, sq, uni, segmask) : 0u;
  uint32_t o[16];
  if (a.mode == UFP8_EPI_ATTN_P) {  // P = 2^(acc * scale * log2(e) - lse * log2(e)); rv = -lse * log2(e)
    const float c = a.attn_scale * kAttnLog2e;
    if (vis == 0xFFFFFFFFu) {
#pragma unroll
      for (int j = 0; j < 16; ++j)
        o[j] = pack_bf16x2(attn_ex2(__fmaf_rn(__uint_as_float(r[2 * j]), c, rv)),
                           attn_ex2(__fmaf_rn(__uint_as_float(r[2 * j + 1]), c, rv)));
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float p0 = ((vis >> (2 * j)) & 1u) ? attn_ex2(__fmaf_rn(__uint_as_float(r[2 * j]), c, rv)) : 0.0f;
        const float p1 = ((vis >> (2 * j + 1)) & 1u) ? attn_ex2(__fmaf_rn(__uint_as_float(r[2 * j + 1]), c, rv)) : 0.0f;
        o[j] = pack_bf16x2(p0, p1);
      }
    }
  } else {  // DS
    const __nv_bfloat16* pp = a.attn_p + g * a.c_bstride + static_cast<long long>(row) * a.ldc + col0;
    uint32_t pw[2][8];
    load_bf16x16_packed(pp, pw[0], valid, a.c_vec);
    load_bf16x16_packed(pp + 16, pw[1], valid - 16, a.c_vec);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint32_t w2 = pw[j >> 3][j & 7];
      const float d0 = __fmul_rn(__fmul_rn(lo_f(w2), __fsub_rn(__uint_as_float(r[2 * j]), rv)), a.attn_scale);
      const float d1 = __fmul_rn(__fmul_rn(hi_f(w2), __fsub_rn(__uint_as_float(r[2 * j + 1]), rv)), a.attn_scale);
      o[j] = pack_bf16x2(d0, d1);
    }
  }
  store_bf16x32_packed_h(d, o, valid, vec, pol);
}

// KCH = 128-byte K chunks per ring stage (1 or 2): a stage holds KCH A sub-tiles followed by KCH
// B sub-tiles of 16 KiB each, and the MMA thread issues 4 * KCH MMAs per stage, so the per-stage
// barrier hand-offs (full -> MMA issue -> commit -> empty -> next load) occur half as often.
// kBf16: bf16 operands (tcgen05.mma kind::f16).  The ring stages hold the same bytes: a 128-byte K
// chunk is 64 elements, a K-major sub-tile 128 rows x 128 B as for fp8, and an MN-major sub-tile
// two 64-element (128-byte) MN atoms of 64 K rows each, 8 KiB apart (the descriptor's leading
// byte offset).  Each MMA consumes K = 16 (32 bytes), four per chunk as with fp8.  Only the STORE,
// AXPBY and ATTN epilogues are compiled in.
template <int NSTAGES, int kVar, int KCH = 1, bool kBf16 = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPThreads, 1)
    gemm_fp8_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                         const __grid_constant__ CUtensorMap tmUG, const __grid_constant__ CUtensorMap tmD,
                         const GemmArgs args) {
  constexpr bool kStaged = kVar == kVarRsStaged;
  constexpr bool kUgStaged = kVar == kVarUgStaged;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int kStageBytes = KCH * kPStageBytes;
  uint8_t* staging = smem + NSTAGES * kStageBytes;  // staged variants only
  uint64_t* ugbar_all = reinterpret_cast<uint64_t*>(staging + kPEpiWarps * kPUgWarpBytes);  // kUgStaged only
  uint64_t* full = reinterpret_cast<uint64_t*>(staging + pair_extra_bytes(kVar));
  uint64_t* empty = full + NSTAGES;
  uint64_t* tfull = empty + NSTAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NSTAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 2 * kPEpiWarps);
    }
    mbar_init(drain, 1);
    if (kUgStaged)
      for (int i = 0; i < 2 * kPEpiWarps; ++i) mbar_init(&ugbar_all[i], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (kUgStaged) tma_prefetch_desc(&tmUG);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int cluster_id = blockIdx.x >> 1;
  const int num_clusters = gridDim.x >> 1;
  const int num_tiles = args.tiles_m * args.tiles_n * args.batch;
  const int total_k = args.ksteps * args.k_batches;
  const bool swiglu = args.mode == UFP8_EPI_SWIGLU;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0, armed_parity = 0;
      uint32_t arrived = 0;  // all-gather blocks seen complete (bit per source rank)
      for (int tile = cluster_id; tile < num_tiles && !*abort_flag; tile += num_clusters) {
        int g, mb, nb;
        map_tile(tile, args, g, mb, nb);
        constexpr int kKc = kBf16 ? kBK / 2 : kBK;  // K elements per 128-byte chunk
        int lo = 0, hi = args.ksteps;
        if constexpr (kBf16) {
          if (!masked_tile(args, mb, nb, KCH * kKc, lo, hi)) continue;
        }
        const int span = hi - lo;
        const int row0 = mb * 2 * kBM + static_cast<int>(rank) * kBM;
        if (args.ag_flags != nullptr && row0 < args.M) {
          const int src = static_cast<int>(row0 / args.ag_rows);
          if (src != args.ag_rank && !((arrived >> src) & 1u)) {
            if (!ag_wait(args, src, abort_flag)) break;
            arrived |= 1u << src;
          }
        }
        for (int ks = 0; ks < args.k_batches * span; ++ks) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) break;
          const int kb = ks / span;
          const int k0 = (lo + ks - kb * span) * (KCH * kKc);
          uint8_t* sa = smem + stage * kStageBytes;
          uint8_t* sb = sa + KCH * kPHalfBytes;
          if (leader) {
            mbar_arrive_expect_tx(&full[stage], 2 * kStageBytes);
            armed |= 1u << stage;
            armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
          }
          const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);
          const int az = args.a_bcast ? 0 : (args.k_batches > 1 ? g * args.k_batches + kb : g / args.a_group);
          int n0, bz;
          if (swiglu) {
            n0 = nb * 128;
            bz = static_cast<int>(rank);
          } else {
            n0 = nb * kBN + static_cast<int>(rank) * 128;
            bz = args.b_bcast ? 0 : (args.k_batches > 1 ? g * args.k_batches + kb : g / args.b_group);
          }
#pragma unroll
          for (int j = 0; j < KCH; ++j) {
            // K chunks past K (or past this slice's K for k_batches) read as zeros.  The tensor
            // maps address bytes along their contiguous dimension.
            const int kj = k0 + j * kKc;
            if constexpr (kBf16) {
              if (args.a_major == UFP8_K_MAJOR) {
                tma_load_3d_pair(sa + j * kPHalfBytes, &tmA, bar, 2 * kj, row0, az);
              } else {
                tma_load_3d_pair(sa + j * kPHalfBytes, &tmA, bar, 2 * row0, kj, az);
                tma_load_3d_pair(sa + j * kPHalfBytes + kPHalfBytes / 2, &tmA, bar, 2 * row0 + 128, kj, az);
              }
              if (args.b_major == UFP8_K_MAJOR) {
                tma_load_3d_pair(sb + j * kPHalfBytes, &tmB, bar, 2 * kj, n0, bz);
              } else {
                tma_load_3d_pair(sb + j * kPHalfBytes, &tmB, bar, 2 * n0, kj, bz);
                tma_load_3d_pair(sb + j * kPHalfBytes + kPHalfBytes / 2, &tmB, bar, 2 * n0 + 128, kj, bz);
              }
            } else {
              if (args.a_major == UFP8_K_MAJOR)
                tma_load_3d_pair(sa + j * kPHalfBytes, &tmA, bar, kj, row0, az);
              else
                tma_load_3d_pair(sa + j * kPHalfBytes, &tmA, bar, row0, kj, az);
              if (args.b_major == UFP8_K_MAJOR)
                tma_load_3d_pair(sb + j * kPHalfBytes, &tmB, bar, kj, n0, bz);
              else
                tma_load_3d_pair(sb + j * kPHalfBytes, &tmB, bar, n0, kj, bz);
            }
          }
          if (++stage == NSTAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (*abort_flag && leader) {
        // Both CTAs' loads for a stage complete on the leader's barrier: wait for every
        // armed stage so that no load is still in flight when the cluster exits.
        volatile int never = 0;
        for (int s = 0; s < NSTAGES; ++s)
          if (armed & (1u << s)) mbar_wait(&full[s], (armed_parity >> s) & 1u, &never);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (even CTA)
    if (lane == 0 && leader) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int tile = cluster_id; tile < num_tiles && !*abort_flag; tile += num_clusters, ++local) {
        int tile_k = total_k;
        if constexpr (kBf16) {
          int g, mb, nb, lo, hi;
          map_tile(tile, args, g, mb, nb);
          if (!masked_tile(args, mb, nb, KCH * (kBK / 2), lo, hi)) {
            --local;  // a skipped tile takes no TMEM buffer
            continue;
          }
          tile_k = args.k_batches * (hi - lo);
        }
        const int buf = local & 1;
        const uint32_t tphase = (local >> 1) & 1;
        if (!mbar_wait(&tempty[buf], tphase ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * kBN);
        bool ok = true;
        for (int ks = 0; ks < tile_k; ++ks) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa0 = smem_u32(smem + stage * kStageBytes);
#pragma unroll
          for (int j = 0; j < KCH; ++j) {
            const uint32_t sa = sa0 + j * kPHalfBytes;
            const uint32_t sb = sa0 + (KCH + j) * kPHalfBytes;
#pragma unroll
            for (int kk = 0; kk < kBK / 32; ++kk) {
              // MN-major: an MMA's K rows are 128 bytes apart (32 rows for fp8, 16 for bf16); the
              // bf16 sub-tile's second MN atom sits half a sub-tile further (leading byte offset).
              constexpr uint32_t kMnStep = kBf16 ? 16 * 128 : 32 * 128;
              constexpr uint32_t kMnLbo = kBf16 ? kPHalfBytes / 2 : kPHalfBytes;
              const uint64_t adesc = args.a_major == UFP8_K_MAJOR ? make_sdesc_sw128(sa + kk * 32, 16, 1024)
                                                                  : make_sdesc_sw128(sa + kk * kMnStep, kMnLbo, 1024);
              const uint64_t bdesc = args.b_major == UFP8_K_MAJOR ? make_sdesc_sw128(sb + kk * 32, 16, 1024)
                                                                  : make_sdesc_sw128(sb + kk * kMnStep, kMnLbo, 1024);
              if constexpr (kBf16)
                umma_f16_pair(d_tmem, adesc, bdesc, args.idesc, (ks | j | kk) != 0 ? 1u : 0u);
              else
                umma_f8f6f4_pair(d_tmem, adesc, bdesc, args.idesc, (ks | j | kk) != 0 ? 1u : 0u);
            }
          }
          umma_commit_pair(&empty[stage], 0x3);
          if (++stage == NSTAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair(&tfull[buf], 0x3);
      }
      umma_commit_pair(drain, 0x1);
      volatile int never = 0;
      mbar_wait(drain, 0, &never);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ epilogue (both CTAs)
    const int e = warp - 2;
    const int quad = warp & 3;   // TMEM lanes this warp may read: [32*quad, 32*quad+32)
    const int chalf = e >> 2;    // which half of the tile's columns this warp handles
    const int row_in_tile = static_cast<int>(rank) * kBM + quad * 32 + lane;
    // fp8: alpha = sa * sb; bf16 operands: scales optional (1), times the AXPBY / STORE multiplier.
    const float alpha = kBf16 ? __fmul_rn(__fmul_rn(args.inv_a ? *args.inv_a : 1.0f, args.inv_b ? *args.inv_b : 1.0f),
                                          args.alpha_mul)
                              : __fmul_rn(*args.inv_a, *args.inv_b);
    const int vec = args.vec_ok;
    const uint32_t tempty_leader0 = mapa_shared(smem_u32(&tempty[0]), 0);
    const uint64_t stream = l2_policy_evict_first();  // outputs are not re-read by this kernel
    uint32_t amax = 0;
    // kUgStaged: this warp's U / G chunk stream.  Chunk j (4 per tile: 32 of this warp's 128
    // columns each) lands in buffer j & 1 on mbarrier ugbar[j & 1], phase (j >> 1) & 1.
    uint8_t* ugw = staging + e * kPUgWarpBytes;
    uint64_t* ugbar = ugbar_all + 2 * e;
    int ug_issued = 0;  // chunks issued (lane 0)
    int ug_used = 0;    // chunks consumed
    auto ug_issue = [&](int j) -> bool {
      const int t = cluster_id + (j >> 2) * num_clusters;
      if (t >= num_tiles) return false;
      int g_, mb_, nb_;
      map_tile(t, args, g_, mb_, nb_);
      const int b = j & 1;
      uint8_t* dst = ugw + b * kPUgBufBytes;
      const int x = nb_ * kBN + chalf * 128 + (j & 3) * kPUgCols;
      const int y = mb_ * 2 * kBM + static_cast<int>(rank) * kBM + quad * 32;
      mbar_arrive_expect_tx(&ugbar[b], kPUgBufBytes);
      tma_load_3d(dst, &tmUG, &ugbar[b], x, y, 0);
      tma_load_3d(dst + kPUgBoxBytes, &tmUG, &ugbar[b], x, y, 1);
      return true;
    };
    if (kUgStaged && lane == 0) {
      if (ug_issue(0)) ug_issued = 1;
      if (ug_issued == 1 && ug_issue(1)) ug_issued = 2;
    }
    int local = 0;
    for (int tile = cluster_id; tile < num_tiles; tile += num_clusters, ++local) {
      int pf_sq = 0;      // ATTN: this row's segment id and attn_row value, loaded before the wait
      float pf_rv = 0.0f;
      if constexpr (kBf16) {
        int g_, mb_, nb_, lo_, hi_;
        map_tile(tile, args, g_, mb_, nb_);
        if (!masked_tile(args, mb_, nb_, KCH * (kBK / 2), lo_, hi_)) {
          --local;
          continue;
        }
        const int row_ = mb_ * 2 * kBM + row_in_tile;
        if (args.mode >= UFP8_EPI_ATTN_STATS && row_ < args.M) {
          pf_sq = args.attn_qseg ? args.attn_qseg[row_] : 0;
          if (args.attn_row) pf_rv = args.attn_row[static_cast<long long>(g_) * args.M + row_];
          if (args.mode == UFP8_EPI_ATTN_P) pf_rv = -pf_rv * kAttnLog2e;  // the exponent's offset, base 2
          const int c0 = nb_ * kBN + chalf * 128;
          if (args.attn_p != nullptr && c0 < args.N) {  // DS: this row's 128 P values into L2
            const __nv_bfloat16* pp = args.attn_p + g_ * args.c_bstride + static_cast<long long>(row_) * args.ldc + c0;
            asm volatile("prefetch.global.L2 [%0];" ::"l"(pp));
            if (c0 + 64 < args.N) asm volatile("prefetch.global.L2 [%0];" ::"l"(pp + 64));
          }
        }
      }
      const int buf = local & 1;
      const uint32_t tphase = (local >> 1) & 1;
      bool ok = mbar_wait(&tfull[buf], tphase, abort_flag);
      ok = __all_sync(0xFFFFFFFFu, ok);
      if (!ok) break;
      tc_fence_after();
      int g, mb, nb;
      map_tile(tile, args, g, mb, nb);
      const int row = mb * 2 * kBM + row_in_tile;
      const bool row_ok = row < args.M;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(buf * kBN);

      if (kUgStaged) {
        // DSWIGLU with U / G from shared memory (TMA-staged two chunks ahead); dU / dG written
        // back into the same boxes and stored by TMA.
        bool ug_ok = true;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          const int j = local * 4 + c;
          const int b = j & 1;
          uint32_t r[32];
          tmem_ld_32x32b_x32(tbase + chalf * 128 + c * kPUgCols, r);
          bool okc = mbar_wait(&ugbar[b], (j >> 1) & 1, abort_flag);
          okc = __all_sync(0xFFFFFFFFu, okc);
          tmem_ld_wait();
          if (!okc) {
            ug_ok = false;
            break;
          }
          ug_used = j + 1;
          const int col0 = nb * kBN + chalf * 128 + c * kPUgCols;
          const int valid = row_ok ? args.N - col0 : 0;
          uint8_t* box = ugw + b * kPUgBufBytes;
          uint8_t* su = box + lane * (kPUgCols * 2);
          uint8_t* sg = su + kPUgBoxBytes;
          const int sw = (lane >> 1) & 3;  // 64-byte swizzle of this row's 16-byte granules
          uint32_t m2 = 0;                 // packed 2 x 16-bit max of |dU|, |dG|
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4* pu = reinterpret_cast<uint4*>(su + ((q ^ sw) << 4));
            uint4* pg = reinterpret_cast<uint4*>(sg + ((q ^ sw) << 4));
            const uint4 uq = *pu, gq = *pg;
            const uint32_t cu[4] = {uq.x, uq.y, uq.z, uq.w};
            const uint32_t cg[4] = {gq.x, gq.y, gq.z, gq.w};
            uint32_t du[4], dg[4];
#pragma unroll
            for (int w = 0; w < 4; ++w) {
              const int jj = q * 4 + w;  // output word: columns 2jj, 2jj + 1
              const uint32_t dhw =
                  pack_bf16x2(__uint_as_float(r[2 * jj]) * alpha, __uint_as_float(r[2 * jj + 1]) * alpha);
              const float dh0 = lo_f(dhw), dh1 = hi_f(dhw);
              const float u0 = lo_f(cu[w]), u1 = hi_f(cu[w]);
              const float g0 = lo_f(cg[w]), g1 = hi_f(cg[w]);
              const float s0 = sigmoidf_(g0), s1 = sigmoidf_(g1);
              du[w] = pack_bf16x2(dh0 * (g0 * s0), dh1 * (g1 * s1));
              dg[w] = pack_bf16x2((dh0 * u0) * (s0 * (1.0f + g0 * (1.0f - s0))),
                                  (dh1 * u1) * (s1 * (1.0f + g1 * (1.0f - s1))));
              const uint32_t keep = (2 * jj + 1 < valid) ? 0x7FFF7FFFu : (2 * jj < valid ? 0x00007FFFu : 0u);
              m2 = __vmaxu2(m2, __vmaxu2(du[w] & keep, dg[w] & keep));
            }
            // dU, dG overwrite the U, G granules they came from (same lane, same row).
            *pu = make_uint4(du[0], du[1], du[2], du[3]);
            *pg = make_uint4(dg[0], dg[1], dg[2], dg[3]);
          }
          amax = max(amax, max(m2 & 0xFFFFu, m2 >> 16));
          fence_proxy_async_smem();  // this lane's shared-memory writes -> the TMA store
          __syncwarp();
          if (lane == 0) {
            // Rows >= M and columns >= N of the box lie outside the tensor map: not stored.
            const int y = mb * 2 * kBM + static_cast<int>(rank) * kBM + quad * 32;
            if (col0 < args.N && y < args.M) {
              tma_store_3d(&tmD, box, col0, y, 0);
              tma_store_3d(&tmD, box + kPUgBoxBytes, col0, y, 1);
              bulk_commit();
              bulk_wait_read_all();  // the stores have read the box: it may be refilled
            }
            if (ug_issued == j + 2 && ug_issue(j + 2)) ug_issued = j + 3;
          }
          __syncwarp();
        }
        if (!ug_ok) break;
      } else if (kStaged) {
        // RS_PUSH through shared memory: 64-column row segments leave as bulk stores into
        // the row owner's staging slot.
        __nv_bfloat16* rs_row = nullptr;
        if (row_ok) {
          const long long owner = row / args.rs_rows;
          rs_row = static_cast<__nv_bfloat16*>(args.rs_slots[owner]) +
                   (args.rs_rank * args.rs_rows + (row - owner * args.rs_rows)) * args.ldd;
        }
        uint8_t* stg_row = staging + e * kPStgWarpBytes + lane * kPStgStride;
#pragma unroll 1
        for (int c = chalf * 128; c < chalf * 128 + 128; c += kPStgCols) {
          uint32_t r0[32], r1[32];
          tmem_ld_32x32b_x32(tbase + c, r0);
          tmem_ld_32x32b_x32(tbase + c + 32, r1);
          tmem_ld_wait();
          const int col0 = nb * kBN + c;
          if (row_ok && col0 < args.N) {
            const int valid = args.N - col0;
            uint32_t o0[16], o1[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              o0[j] = pack_bf16x2(__uint_as_float(r0[2 * j]) * alpha, __uint_as_float(r0[2 * j + 1]) * alpha);
              o1[j] = pack_bf16x2(__uint_as_float(r1[2 * j]) * alpha, __uint_as_float(r1[2 * j + 1]) * alpha);
            }
            if (valid >= kPStgCols) {
              bulk_wait_read_all();  // the previous segment has left this row's staging
              uint4* srow = reinterpret_cast<uint4*>(stg_row);
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                srow[i] = make_uint4(o0[4 * i], o0[4 * i + 1], o0[4 * i + 2], o0[4 * i + 3]);
                srow[4 + i] = make_uint4(o1[4 * i], o1[4 * i + 1], o1[4 * i + 2], o1[4 * i + 3]);
              }
              fence_proxy_async_smem();
              bulk_store_s2g(rs_row + col0, smem_u32(stg_row), kPStgCols * 2);
              bulk_commit();
            } else {
              store_bf16x32_packed(rs_row + col0, o0, valid, true);
              if (valid > 32) store_bf16x32_packed(rs_row + col0 + 32, o1, valid - 32, true);
            }
          }
        }
      } else if (args.mode == UFP8_EPI_STORE || args.mode == UFP8_EPI_RS_PUSH || args.mode == UFP8_EPI_XENT ||
                 args.mode == UFP8_EPI_AXPBY || args.mode >= UFP8_EPI_ATTN_STATS) {
        // RS_PUSH: this row goes to its owner's staging slot for this rank (peer memory).
        // XENT: bf16 logits (soft-capped if asked) and the softmax partials of this warp's 128 columns.
        const bool xent = args.mode == UFP8_EPI_XENT;
        float xm = -INFINITY, xs = 0.0f;
        __nv_bfloat16* rs_row = nullptr;
        if (args.mode == UFP8_EPI_RS_PUSH && row_ok) {
          const long long owner = row / args.rs_rows;
          rs_row = static_cast<__nv_bfloat16*>(args.rs_slots[owner]) +
                   (args.rs_rank * args.rs_rows + (row - owner * args.rs_rows)) * args.ldd;
        }
        const bool attn = kBf16 && args.mode >= UFP8_EPI_ATTN_STATS;
        int attn_sq = 0;
        float attn_rv = 0.0f;
        if (attn && row_ok) {
          attn_sq = pf_sq;
          attn_rv = pf_rv;
        }
        // All rows of this warp in range and of one segment: one ballot per chunk gives the
        // columns of that segment (row_ok differs only in a partial last tile).
        const int attn_sq0 = __shfl_sync(0xFFFFFFFFu, attn_sq, 0);
        const bool attn_uni = attn && __all_sync(0xFFFFFFFFu, row_ok && attn_sq == attn_sq0);
        if (attn) {
          // 64 columns per step: two TMEM loads under one wait, the key segment ballots issued
          // before it (warp-uniform conditions: every lane takes part).
#pragma unroll 1
          for (int c = chalf * 128; c < chalf * 128 + 128; c += 64) {
            uint32_t r0[32], r1[32];
            tmem_ld_32x32b_x32(tbase + c, r0);
            tmem_ld_32x32b_x32(tbase + c + 32, r1);
            const int col0 = nb * kBN + c;
            uint32_t sm0 = 0xFFFFFFFFu, sm1 = 0xFFFFFFFFu;
            if (attn_uni && col0 < args.N && args.mode != UFP8_EPI_ATTN_DS) {
              if (args.attn_kseg != nullptr) {
                const int k0 = col0 + lane, k1 = col0 + 32 + lane;
                const int kv0 = k0 < args.N ? args.attn_kseg[k0] : -1;
                const int kv1 = k1 < args.N ? args.attn_kseg[k1] : -1;
                sm0 = __ballot_sync(0xFFFFFFFFu, kv0 == attn_sq0);
                sm1 = __ballot_sync(0xFFFFFFFFu, kv1 == attn_sq0);
              } else {
                sm0 = sm1 = attn_sq0 == 0 ? 0xFFFFFFFFu : 0u;
              }
            }
            tmem_ld_wait();
            if (row_ok && col0 < args.N) {
              const int valid = args.N - col0;
              if (args.mode == UFP8_EPI_ATTN_STATS) {
                attn_stats64(args, r0, r1, row, col0, valid, attn_sq, attn_uni, sm0, sm1, xm, xs);
              } else {
                __nv_bfloat16* dp = static_cast<__nv_bfloat16*>(args.d) + g * args.d_bstride +
                                    static_cast<long long>(row) * args.ldd + col0;
                attn_chunk(args, r0, row, col0, valid, g, attn_sq, attn_rv, dp, vec, stream, attn_uni, sm0);
                if (valid > 32)
                  attn_chunk(args, r1, row, col0 + 32, valid - 32, g, attn_sq, attn_rv, dp + 32, vec, stream, attn_uni,
                             sm1);
              }
            }
          }
        }
#pragma unroll 1
        for (int c = chalf * 128; !attn && c < chalf * 128 + 128; c += 32) {  // the other modes
          uint32_t r[32];
          tmem_ld_32x32b_x32(tbase + c, r);
          tmem_ld_wait();
          const int col0 = nb * kBN + c;
          if (row_ok && col0 < args.N) {
            const int valid = args.N - col0;
            float am = alpha;  // the accumulator multiplier of the stores below
            if constexpr (kBf16) {
              if (args.c != nullptr) {
                // AXPBY: v = acc * alpha + beta * C, each product and the sum rounded once.
                const __nv_bfloat16* cp = args.c + g * args.c_bstride + static_cast<long long>(row) * args.ldc + col0;
                uint32_t cw[2][8];
                load_bf16x16_packed(cp, cw[0], valid, args.c_vec);
                load_bf16x16_packed(cp + 16, cw[1], valid - 16, args.c_vec);
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                  const uint32_t w2 = cw[j >> 4][(j & 15) >> 1];
                  const float cv = (j & 1) ? hi_f(w2) : lo_f(w2);
                  r[j] = __float_as_uint(__fadd_rn(__fmul_rn(__uint_as_float(r[j]), alpha), __fmul_rn(cv, args.beta)));
                }
                am = 1.0f;
              }
            }
            if (args.d_f32) {
              float* p = static_cast<float*>(args.d) + g * args.d_bstride + row * args.ldd + col0;
              if (vec && valid >= 32) {
#pragma unroll
                for (int i = 0; i < 8; ++i)
                  reinterpret_cast<float4*>(p)[i] =
                      make_float4(__uint_as_float(r[4 * i]) * am, __uint_as_float(r[4 * i + 1]) * am,
                                  __uint_as_float(r[4 * i + 2]) * am, __uint_as_float(r[4 * i + 3]) * am);
              } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (j < valid) p[j] = __uint_as_float(r[j]) * am;
              }
            } else {
              uint32_t o[16];
#pragma unroll
              for (int j = 0; j < 16; ++j)
                o[j] = pack_bf16x2(__uint_as_float(r[2 * j]) * am, __uint_as_float(r[2 * j + 1]) * am);
              if (xent) xent_chunk(o, valid, args.xent_cap, xm, xs);
              __nv_bfloat16* p = rs_row ? rs_row + col0
                                        : static_cast<__nv_bfloat16*>(args.d) + g * args.d_bstride + row * args.ldd + col0;
              store_bf16x32_packed_h(p, o, valid, vec, stream);
            }
          }
        }
        if (xent && row_ok && nb * kBN + chalf * 128 < args.N)
          *reinterpret_cast<float2*>(args.xent_stats + 2 * (static_cast<long long>(row) * args.xent_ld + nb * 2 + chalf)) =
              make_float2(xm, xs);
        if (attn && args.mode == UFP8_EPI_ATTN_STATS && row_ok && nb * kBN + chalf * 128 < args.N)
          *reinterpret_cast<float2*>(args.attn_stats +
                                     2 * ((static_cast<long long>(g) * args.M + row) * args.attn_ld + nb * 2 + chalf)) =
              make_float2(xm, xs);
      } else if (args.mode == UFP8_EPI_SWIGLU) {
        // TMEM columns [0,128) hold up, [128,256) hold gate for hidden units nb*128 + c.
#pragma unroll 1
        for (int c = chalf * 64; c < chalf * 64 + 64; c += 16) {
          uint32_t ru[16], rg[16];
          tmem_ld_32x32b_x16(tbase + c, ru);
          tmem_ld_32x32b_x16(tbase + 128 + c, rg);
          tmem_ld_wait();
          const int col0 = nb * 128 + c;
          if (row_ok && col0 < args.N) {
            const int valid = args.N - col0;
            uint32_t ou[8], og[8], oh[8];
            uint32_t m2 = 0;  // packed 2 x 16-bit max of |H|
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const uint32_t uw = pack_bf16x2(__uint_as_float(ru[2 * j]) * alpha, __uint_as_float(ru[2 * j + 1]) * alpha);
              const uint32_t gw = pack_bf16x2(__uint_as_float(rg[2 * j]) * alpha, __uint_as_float(rg[2 * j + 1]) * alpha);
              const float g0 = lo_f(gw), g1 = hi_f(gw);
              const uint32_t hw = pack_bf16x2(lo_f(uw) * (g0 * sigmoidf_(g0)), hi_f(uw) * (g1 * sigmoidf_(g1)));
              ou[j] = uw;
              og[j] = gw;
              oh[j] = hw;
              const uint32_t keep = (2 * j + 1 < valid) ? 0x7FFF7FFFu : (2 * j < valid ? 0x00007FFFu : 0u);
              m2 = __vmaxu2(m2, hw & keep);
            }
            amax = max(amax, max(m2 & 0xFFFFu, m2 >> 16));
            __nv_bfloat16* pu = static_cast<__nv_bfloat16*>(args.d) + row * args.ldd + col0;
            store_bf16x16_packed_h(pu, ou, valid, vec, stream);
            store_bf16x16_packed_h(pu + args.d_bstride, og, valid, vec, stream);
            store_bf16x16_packed_h(args.h + row * args.ldh + col0, oh, valid, vec, stream);
          }
        }
      } else {  // UFP8_EPI_DSWIGLU: 16-column chunks; U / G loads run two chunks ahead
        const int c_begin = chalf * 128;
        const __nv_bfloat16* ug_row = args.ug + row * args.ldug;
        uint32_t bu[3][8], bg[3][8];
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          const int col0 = nb * kBN + c_begin + 16 * p;
          const int valid = row_ok ? args.N - col0 : 0;
          if (valid > 0) {
            load_bf16x16_packed(ug_row + col0, bu[p], valid, vec);
            load_bf16x16_packed(ug_row + args.ug_bstride + col0, bg[p], valid, vec);
          }
        }
#pragma unroll
        for (int ci = 0; ci < 8; ++ci) {
          const int c = c_begin + 16 * ci;
          uint32_t r[16];
          tmem_ld_32x32b_x16(tbase + c, r);
          if (ci + 2 < 8) {
            const int ncol0 = nb * kBN + c + 32;
            const int nvalid = row_ok ? args.N - ncol0 : 0;
            if (nvalid > 0) {
              load_bf16x16_packed(ug_row + ncol0, bu[(ci + 2) % 3], nvalid, vec);
              load_bf16x16_packed(ug_row + args.ug_bstride + ncol0, bg[(ci + 2) % 3], nvalid, vec);
            }
          }
          tmem_ld_wait();
          const int col0 = nb * kBN + c;
          if (row_ok && col0 < args.N) {
            const int valid = args.N - col0;
            const uint32_t(&cu)[8] = bu[ci % 3];
            const uint32_t(&cg)[8] = bg[ci % 3];
            uint32_t odu[8], odg[8];
            uint32_t m2 = 0;  // packed 2 x 16-bit max of |dU|, |dG|
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const uint32_t dhw = pack_bf16x2(__uint_as_float(r[2 * j]) * alpha, __uint_as_float(r[2 * j + 1]) * alpha);
              const float dh0 = lo_f(dhw), dh1 = hi_f(dhw);
              const float u0 = lo_f(cu[j]), u1 = hi_f(cu[j]);
              const float g0 = lo_f(cg[j]), g1 = hi_f(cg[j]);
              const float s0 = sigmoidf_(g0), s1 = sigmoidf_(g1);
              odu[j] = pack_bf16x2(dh0 * (g0 * s0), dh1 * (g1 * s1));
              odg[j] = pack_bf16x2((dh0 * u0) * (s0 * (1.0f + g0 * (1.0f - s0))),
                                   (dh1 * u1) * (s1 * (1.0f + g1 * (1.0f - s1))));
              const uint32_t keep = (2 * j + 1 < valid) ? 0x7FFF7FFFu : (2 * j < valid ? 0x00007FFFu : 0u);
              m2 = __vmaxu2(m2, __vmaxu2(odu[j] & keep, odg[j] & keep));
            }
            amax = max(amax, max(m2 & 0xFFFFu, m2 >> 16));
            __nv_bfloat16* pd = static_cast<__nv_bfloat16*>(args.d) + row * args.ldd + col0;
            store_bf16x16_packed_h(pd, odu, valid, vec, stream);
            store_bf16x16_packed_h(pd + args.d_bstride, odg, valid, vec, stream);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader0 + static_cast<uint32_t>(buf * sizeof(uint64_t)));
    }
    if (args.amax_bits != nullptr) {
      amax = __reduce_max_sync(0xFFFFFFFFu, amax);
      if (lane == 0 && amax != 0u) atomicMax(args.amax_bits, amax << 16);
    }
    // kUgStaged after an abort: wait (bounded) for this warp's U / G loads still in flight, so
    // that no TMA write lands in shared memory after the CTA has exited.
    if (kUgStaged && lane == 0) {
      volatile int never = 0;
      for (int j = ug_used; j < ug_issued; ++j) mbar_wait(&ugbar[j & 1], (j >> 1) & 1, &never);
      bulk_wait_all();  // dU / dG stores complete before the CTA exits
    }
    // Peer stores must be complete and visible system-wide before the finish kernel's flag write.
    if (kStaged) bulk_wait_all();
    if (args.mode == UFP8_EPI_RS_PUSH) __threadfence_system();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicOr(args.status, UFP8_STATUS_WAIT_TIMEOUT);
}

// ============================================================================= 256 x 512 pair tiles
// The same contraction on a cluster of two CTAs computing 256 x 512 tiles.  Every 128-byte K
// step issues two tcgen05.mma.cta_group::2 (M = 256, N = 256) with the same A sub-tiles, into
// TMEM columns [0, 256) ("half 0") and [256, 512) ("half 1"), so a CTA streams 48 KiB (A: 128
// rows; B: two sub-tiles of 128 rows) for twice the MMAs of a 256 x 256 tile: 25 % fewer operand
// bytes per FLOP cross from L2 into shared memory, which is what limits the 256 x 256 kernel on
// long-K contractions (no TMA multicast is used).
//
// The accumulator fills all 512 TMEM columns, so it is handed over per half.  When a tile's
// MMAs complete, the epilogue warps copy half 0 into registers (packed bf16, 64 registers a
// thread), release it (tempty[0]), store it, then do the same with half 1 (tempty[1]).  The MMA
// thread starts the next tile with the half-0 MMAs of its first kWStages K steps as soon as
// tempty[0] completes, then issues their half-1 MMAs once tempty[1] completes (only then are
// those ring stages released), and continues with both halves per K step.
//
// Epilogues: STORE (bf16; half j = tile columns [256 j, 256 j + 256)) and SWIGLU (half j holds
// 128 hidden units: up in its first 128 columns, gate in the next 128, loaded by the even and
// the odd CTA respectively; U and G are rounded to bf16 before H = U * swish(G), as in the other
// kernels, so the results are the same bits).
constexpr int kWStages = 4;
constexpr int kWStageBytes = 3 * kPHalfBytes;  // A + two B sub-tiles: 48 KiB
constexpr int kWSmemBytes = kWStages * kWStageBytes + kBarrierBytes + 1024;
static_assert(kWSmemBytes <= 232448, "256 x 512 CTA-pair kernel exceeds shared memory");

// The three shared-memory descriptors (A, B half 0, B half 1) of MMA K step kk of the ring
// stage at shared address sa.
__device__ __forceinline__ void n512_descs(uint32_t sa, int kk, bool a_k, bool b_k, uint64_t& ad, uint64_t& b0,
                                           uint64_t& b1) {
  const uint32_t sb0 = sa + kPHalfBytes, sb1 = sa + 2 * kPHalfBytes;
  ad = a_k ? make_sdesc_sw128(sa + kk * 32, 16, 1024) : make_sdesc_sw128(sa + kk * 32 * 128, kPHalfBytes, 1024);
  b0 = b_k ? make_sdesc_sw128(sb0 + kk * 32, 16, 1024) : make_sdesc_sw128(sb0 + kk * 32 * 128, kPHalfBytes, 1024);
  b1 = b_k ? make_sdesc_sw128(sb1 + kk * 32, 16, 1024) : make_sdesc_sw128(sb1 + kk * 32 * 128, kPHalfBytes, 1024);
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPThreads, 1)
    gemm_fp8_n512_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                         const GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kWStages * kWStageBytes);
  uint64_t* empty = full + kWStages;
  uint64_t* tfull = empty + kWStages;
  uint64_t* tempty = tfull + 1;  // [2]: one per accumulator half
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kWStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(&tempty[0], 2 * kPEpiWarps);
    mbar_init(&tempty[1], 2 * kPEpiWarps);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int cluster_id = blockIdx.x >> 1;
  const int num_clusters = gridDim.x >> 1;
  const int num_tiles = args.tiles_m * args.tiles_n * args.batch;
  const int total_k = args.ksteps * args.k_batches;
  const bool swiglu = args.mode == UFP8_EPI_SWIGLU;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0, armed_parity = 0;
      uint32_t arrived = 0;  // all-gather blocks seen complete (bit per source rank)
      for (int tile = cluster_id; tile < num_tiles && !*abort_flag; tile += num_clusters) {
        int g, mb, nb;
        map_tile(tile, args, g, mb, nb);
        const int row0 = mb * 2 * kBM + static_cast<int>(rank) * kBM;
        if (args.ag_flags != nullptr && row0 < args.M) {
          const int src = static_cast<int>(row0 / args.ag_rows);
          if (src != args.ag_rank && !((arrived >> src) & 1u)) {
            if (!ag_wait(args, src, abort_flag)) break;
            arrived |= 1u << src;
          }
        }
        for (int ks = 0; ks < total_k; ++ks) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) break;
          const int kb = ks / args.ksteps;
          const int k0 = (ks - kb * args.ksteps) * kBK;
          uint8_t* sa = smem + stage * kWStageBytes;
          if (leader) {
            mbar_arrive_expect_tx(&full[stage], 2 * kWStageBytes);
            armed |= 1u << stage;
            armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
          }
          const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);
          const int az = args.a_bcast ? 0 : (args.k_batches > 1 ? g * args.k_batches + kb : g / args.a_group);
          if (args.a_major == UFP8_K_MAJOR)
            tma_load_3d_pair(sa, &tmA, bar, k0, row0, az);
          else
            tma_load_3d_pair(sa, &tmA, bar, row0, k0, az);
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            int n0, bz;
            if (swiglu) {  // half j: hidden units nb*256 + 128 j; even CTA up, odd CTA gate
              n0 = nb * kBN + j * 128;
              bz = static_cast<int>(rank);
            } else {
              n0 = nb * 2 * kBN + j * kBN + static_cast<int>(rank) * 128;
              bz = args.b_bcast ? 0 : (args.k_batches > 1 ? g * args.k_batches + kb : g / args.b_group);
            }
            uint8_t* sb = sa + (1 + j) * kPHalfBytes;
            if (args.b_major == UFP8_K_MAJOR)
              tma_load_3d_pair(sb, &tmB, bar, k0, n0, bz);
            else
              tma_load_3d_pair(sb, &tmB, bar, n0, k0, bz);
          }
          if (++stage == kWStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (*abort_flag && leader) {
        volatile int never = 0;
        for (int s = 0; s < kWStages; ++s)
          if (armed & (1u << s)) mbar_wait(&full[s], (armed_parity >> s) & 1u, &never);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (even CTA)
    if (lane == 0 && leader) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      const int pre = total_k < kWStages ? total_k : kWStages;  // K steps issued half 0 first
      const bool a_k = args.a_major == UFP8_K_MAJOR, b_k = args.b_major == UFP8_K_MAJOR;
      bool ok = true;
      for (int tile = cluster_id; tile < num_tiles && ok && !*abort_flag; tile += num_clusters, ++local) {
        const uint32_t tpar = (local & 1) ^ 1u;  // tile `local` needs the epilogue of local - 1
        // Half 0 of the first `pre` K steps, as soon as the epilogue has released half 0.
        if (!mbar_wait(&tempty[0], tpar, abort_flag)) break;
        tc_fence_after();
        int st = stage;
        uint32_t ph = phase;
        for (int ks = 0; ks < pre; ++ks) {
          if (!mbar_wait(&full[st], ph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + st * kWStageBytes);
#pragma unroll
          for (int kk = 0; kk < kBK / 32; ++kk) {
            uint64_t ad, b0, b1;
            n512_descs(sa, kk, a_k, b_k, ad, b0, b1);
            umma_f8f6f4_pair(tmem_base, ad, b0, args.idesc, (ks | kk) != 0 ? 1u : 0u);
          }
          if (++st == kWStages) {
            st = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        // Half 1 of the same K steps once half 1 is free; their ring stages are released here.
        if (!mbar_wait(&tempty[1], tpar, abort_flag)) break;
        tc_fence_after();
        for (int ks = 0; ks < pre; ++ks) {
          const uint32_t sa = smem_u32(smem + stage * kWStageBytes);
#pragma unroll
          for (int kk = 0; kk < kBK / 32; ++kk) {
            uint64_t ad, b0, b1;
            n512_descs(sa, kk, a_k, b_k, ad, b0, b1);
            umma_f8f6f4_pair(tmem_base + kBN, ad, b1, args.idesc, (ks | kk) != 0 ? 1u : 0u);
          }
          umma_commit_pair(&empty[stage], 0x3);
          if (++stage == kWStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        // The remaining K steps: both halves per stage.
        for (int ks = pre; ks < total_k; ++ks) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * kWStageBytes);
#pragma unroll
          for (int kk = 0; kk < kBK / 32; ++kk) {
            uint64_t ad, b0, b1;
            n512_descs(sa, kk, a_k, b_k, ad, b0, b1);
            umma_f8f6f4_pair(tmem_base, ad, b0, args.idesc, 1u);
            umma_f8f6f4_pair(tmem_base + kBN, ad, b1, args.idesc, 1u);
          }
          umma_commit_pair(&empty[stage], 0x3);
          if (++stage == kWStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair(tfull, 0x3);
      }
      umma_commit_pair(drain, 0x1);
      volatile int never = 0;
      mbar_wait(drain, 0, &never);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ epilogue (both CTAs)
    const int e = warp - 2;
    const int quad = warp & 3;  // TMEM lanes this warp may read: [32*quad, 32*quad+32)
    const int chalf = e >> 2;   // which half of each accumulator half this warp drains
    const int row_in_tile = static_cast<int>(rank) * kBM + quad * 32 + lane;
    const float alpha = __fmul_rn(*args.inv_a, *args.inv_b);
    const int vec = args.vec_ok;
    const uint32_t tempty_leader = mapa_shared(smem_u32(tempty), 0);
    const uint64_t stream = l2_policy_evict_first();
    uint32_t amax = 0;
    int local = 0;
    for (int tile = cluster_id; tile < num_tiles; tile += num_clusters, ++local) {
      bool ok = mbar_wait(tfull, local & 1, abort_flag);
      ok = __all_sync(0xFFFFFFFFu, ok);
      if (!ok) break;
      tc_fence_after();
      int g, mb, nb;
      map_tile(tile, args, g, mb, nb);
      const int row = mb * 2 * kBM + row_in_tile;
      const bool row_ok = row < args.M;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        const uint32_t hbase = tbase + static_cast<uint32_t>(half * kBN);
        uint32_t pk[64];  // 128 accumulator columns of this row, packed bf16
        // Four 32-column chunks: STORE columns [128 chalf, +128); SWIGLU 64 hidden units, up in
        // columns [64 chalf, +64) -> pk[0, 32), gate in [128 + 64 chalf, +64) -> pk[32, 64).
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t col = swiglu ? static_cast<uint32_t>((c >> 1) * 128 + chalf * 64 + (c & 1) * 32)
                                      : static_cast<uint32_t>(chalf * 128 + c * 32);
          uint32_t r[32];
          tmem_ld_32x32b_x32(hbase + col, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j)
            pk[16 * c + j] = pack_bf16x2(__uint_as_float(r[2 * j]) * alpha, __uint_as_float(r[2 * j + 1]) * alpha);
        }
        // This half is in registers: hand it back to the MMA thread before storing.
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(tempty_leader + static_cast<uint32_t>(half * sizeof(uint64_t)));
        if (row_ok) {
          if (swiglu) {
            const int unit0 = nb * kBN + half * 128 + chalf * 64;
            __nv_bfloat16* pu = static_cast<__nv_bfloat16*>(args.d) + row * args.ldd;
            __nv_bfloat16* ph = args.h + row * args.ldh;
#pragma unroll
            for (int q = 0; q < 2; ++q) {
              const int col0 = unit0 + 32 * q;
              if (col0 < args.N) {
                const int valid = args.N - col0;
                uint32_t uw[16], gw[16], hw[16];
                uint32_t m2 = 0;
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                  uw[j] = pk[16 * q + j];
                  gw[j] = pk[32 + 16 * q + j];
                  const float g0 = lo_f(gw[j]), g1 = hi_f(gw[j]);
                  hw[j] = pack_bf16x2(lo_f(uw[j]) * (g0 * sigmoidf_(g0)), hi_f(uw[j]) * (g1 * sigmoidf_(g1)));
                  const uint32_t keep = (2 * j + 1 < valid) ? 0x7FFF7FFFu : (2 * j < valid ? 0x00007FFFu : 0u);
                  m2 = __vmaxu2(m2, hw[j] & keep);
                }
                amax = max(amax, max(m2 & 0xFFFFu, m2 >> 16));
                store_bf16x32_packed_h(pu + col0, uw, valid, vec, stream);
                store_bf16x32_packed_h(pu + args.d_bstride + col0, gw, valid, vec, stream);
                store_bf16x32_packed_h(ph + col0, hw, valid, vec, stream);
              }
            }
          } else {
            const int colbase = nb * 2 * kBN + half * kBN + chalf * 128;
            __nv_bfloat16* pd = static_cast<__nv_bfloat16*>(args.d) + g * args.d_bstride + row * args.ldd;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int col0 = colbase + 32 * q;
              if (col0 < args.N) {
                uint32_t w[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) w[j] = pk[16 * q + j];
                store_bf16x32_packed_h(pd + col0, w, args.N - col0, vec, stream);
              }
            }
          }
        }
      }
    }
    if (args.amax_bits != nullptr) {
      amax = __reduce_max_sync(0xFFFFFFFFu, amax);
      if (lane == 0 && amax != 0u) atomicMax(args.amax_bits, amax << 16);
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicOr(args.status, UFP8_STATUS_WAIT_TIMEOUT);
}

// Writes zeros to every output of an empty-K contraction (K == 0).
__global__ void zero_outputs_kernel(GemmArgs a) {
  const long long total = static_cast<long long>(a.batch) * a.M * a.N;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long g = i / (static_cast<long long>(a.M) * a.N);
    const long long r = i - g * a.M * a.N;
    const long long m = r / a.N, n = r - m * a.N;
    const int slices = a.mode == UFP8_EPI_STORE ? 1 : 2;
    for (int s = 0; s < slices; ++s) {
      const long long off = (g + s) * a.d_bstride + m * a.ldd + n;
      if (a.d_f32)
        static_cast<float*>(a.d)[off] = 0.0f;
      else
        static_cast<__nv_bfloat16*>(a.d)[off] = __float2bfloat16_rn(0.0f);
    }
    if (a.mode == UFP8_EPI_SWIGLU) a.h[m * a.ldh + n] = __float2bfloat16_rn(0.0f);
  }
}

// ----------------------------------------------------------------------------- host side
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<EncodeTiledFn>(nullptr);
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

// 3-D map over one operand in bytes: x = contiguous index (bytes), y = the other matrix index,
// z = batch slice.  Box = 128 bytes x 128 rows (x 64 rows for an MN-major bf16 operand, whose
// sub-tile is two such boxes) x 1, 128-byte swizzle.
int encode_operand(CUtensorMap* map, const ufp8_operand& op, int64_t rows, int64_t K, const char* name) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return set_error(UFP8_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  const int64_t esz = op.fmt == UFP8_BF16 ? 2 : 1;
  const int64_t inner = op.major == UFP8_K_MAJOR ? K : rows;
  const int64_t outer = op.major == UFP8_K_MAJOR ? rows : K;
  const int64_t slices = op.batch_count < 1 ? 1 : op.batch_count;
  const int64_t bstride = slices > 1 ? op.batch_stride : op.ld * outer;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(inner * esz), static_cast<cuuint64_t>(outer),
                        static_cast<cuuint64_t>(slices)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(op.ld * esz), static_cast<cuuint64_t>(bstride * esz)};
  cuuint32_t box[3] = {128, (esz == 2 && op.major == UFP8_MN_MAJOR) ? 64u : 128u, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(op.ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(UFP8_ERR_INVALID, "cuTensorMapEncodeTiled failed for operand %s (CUresult %d)", name,
                     static_cast<int>(r));
  return UFP8_OK;
}

// 3-D map over the saved bf16 U / G of a DSWIGLU GEMM: x = column (N), y = row (M), z = slice
// (0 = U, 1 = G).  Box = 32 x 32 x 1 elements (64-byte rows) with 64-byte swizzle.
int encode_ug(CUtensorMap* map, const ufp8_gemm_desc& d) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return set_error(UFP8_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(d.N), static_cast<cuuint64_t>(d.M), 2};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(d.ldug) * 2, static_cast<cuuint64_t>(d.ug_batch_stride) * 2};
  cuuint32_t box[3] = {32, 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(d.ug), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(UFP8_ERR_INVALID, "cuTensorMapEncodeTiled failed for U/G (CUresult %d)", static_cast<int>(r));
  return UFP8_OK;
}

// 3-D map over a bf16 [2][rows][cols] tensor in 32 x 32 boxes with 64-byte swizzle (the layout
// of the U/G staging boxes), for TMA stores of dU / dG.
int encode_bf16_boxes(CUtensorMap* map, void* base, int64_t cols, int64_t rows, int64_t ld, int64_t bstride,
                      const char* name) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return set_error(UFP8_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows), 2};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld) * 2, static_cast<cuuint64_t>(bstride) * 2};
  cuuint32_t box[3] = {32, 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(UFP8_ERR_INVALID, "cuTensorMapEncodeTiled failed for %s (CUresult %d)", name, static_cast<int>(r));
  return UFP8_OK;
}

int check_operand(const ufp8_operand& op, int64_t rows, int64_t K, int need_slices, const char* name) {
  if (!op.ptr) return set_error(UFP8_ERR_INVALID, "operand %s: null pointer", name);
  if (op.fmt != UFP8_E4M3 && op.fmt != UFP8_E5M2 && op.fmt != UFP8_BF16)
    return set_error(UFP8_ERR_INVALID, "operand %s: fmt %d is not UFP8_E4M3/UFP8_E5M2/UFP8_BF16", name, op.fmt);
  if (!op.inv_scale && op.fmt != UFP8_BF16) return set_error(UFP8_ERR_INVALID, "operand %s: null inv_scale", name);
  const int64_t esz = op.fmt == UFP8_BF16 ? 2 : 1;
  if (op.major != UFP8_K_MAJOR && op.major != UFP8_MN_MAJOR)
    return set_error(UFP8_ERR_INVALID, "operand %s: major %d is not K/MN", name, op.major);
  const int64_t inner = op.major == UFP8_K_MAJOR ? K : rows;
  if (op.ld < inner) return set_error(UFP8_ERR_INVALID, "operand %s: ld %lld < contiguous extent %lld", name,
                                      static_cast<long long>(op.ld), static_cast<long long>(inner));
  if (reinterpret_cast<uintptr_t>(op.ptr) & 15u)
    return set_error(UFP8_ERR_ALIGN, "operand %s: base pointer is not 16-byte aligned", name);
  if ((op.ld * esz) % 16 != 0)
    return set_error(UFP8_ERR_ALIGN, "operand %s: ld %lld is not a multiple of 16 bytes", name,
                     static_cast<long long>(op.ld));
  if (op.batch_count > 1 && (op.batch_stride * esz) % 16 != 0)
    return set_error(UFP8_ERR_ALIGN, "operand %s: batch_stride is not a multiple of 16 bytes", name);
  if (need_slices > 1 && op.batch_count < need_slices)
    return set_error(UFP8_ERR_INVALID, "operand %s: needs %d batch slices, has %d", name, need_slices,
                     op.batch_count);
  if (inner * esz >= (int64_t(1) << 31) || (op.major == UFP8_K_MAJOR ? rows : K) >= (int64_t(1) << 31))
    return set_error(UFP8_ERR_INVALID, "operand %s: extent exceeds 2^31", name);
  return UFP8_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

int launch_gemm(const ufp8_gemm_desc& d, cudaStream_t stream, const DeviceInfo& dev, int ctas_override,
                int variant, int group_m) {
  if (d.M < 0 || d.N < 0 || d.K < 0) return set_error(UFP8_ERR_INVALID, "negative GEMM extent");
  if (d.batch < 1 || d.k_batches < 1) return set_error(UFP8_ERR_INVALID, "batch and k_batches must be >= 1");
  if (d.epilogue < UFP8_EPI_STORE || d.epilogue > UFP8_EPI_ATTN_DS)
    return set_error(UFP8_ERR_INVALID, "unknown epilogue %d", d.epilogue);
  const bool attn = d.epilogue >= UFP8_EPI_ATTN_STATS;
  const bool bf16 = d.a.fmt == UFP8_BF16;
  if (bf16 != (d.b.fmt == UFP8_BF16))
    return set_error(UFP8_ERR_INVALID, "A and B must both be fp8 or both be bf16 (one MMA kind)");
  if (bf16 && d.epilogue != UFP8_EPI_STORE && d.epilogue != UFP8_EPI_AXPBY && !attn)
    return set_error(UFP8_ERR_UNSUPPORTED, "bf16 operands take the STORE, AXPBY and ATTN epilogues only");
  if (attn) {
    if (!bf16) return set_error(UFP8_ERR_UNSUPPORTED, "the ATTN epilogues take bf16 operands");
    if (d.K == 0) return set_error(UFP8_ERR_UNSUPPORTED, "ATTN epilogues with K == 0");
    if (d.epilogue != UFP8_EPI_ATTN_STATS && d.d_dtype != UFP8_OUT_BF16)
      return set_error(UFP8_ERR_INVALID, "ATTN_P / ATTN_DS write bf16");
    const uintptr_t ids = reinterpret_cast<uintptr_t>(d.attn_q_segment_ids) |
                          reinterpret_cast<uintptr_t>(d.attn_kv_segment_ids);
    if (ids & 3u) return set_error(UFP8_ERR_ALIGN, "ATTN: segment ids not 4-byte aligned");
    if (d.epilogue == UFP8_EPI_ATTN_STATS) {
      if (!d.attn_stats || d.attn_ld_stats < (d.N + 127) / 128)
        return set_error(UFP8_ERR_INVALID, "ATTN_STATS needs attn_stats with attn_ld_stats >= ceil(N / 128)");
      if (reinterpret_cast<uintptr_t>(d.attn_stats) & 7u)
        return set_error(UFP8_ERR_ALIGN, "ATTN_STATS: attn_stats not 8-byte aligned");
    } else if (!d.attn_row) {
      return set_error(UFP8_ERR_INVALID, "ATTN_P / ATTN_DS need attn_row");
    }
    if (d.epilogue == UFP8_EPI_ATTN_DS) {
      if (!d.c || d.ldc < d.N) return set_error(UFP8_ERR_INVALID, "ATTN_DS needs P in c with ldc >= N");
      if (reinterpret_cast<uintptr_t>(d.c) & 1u) return set_error(UFP8_ERR_ALIGN, "ATTN_DS: c not 2-byte aligned");
    }
  }
  if (d.epilogue == UFP8_EPI_AXPBY) {
    if (!bf16) return set_error(UFP8_ERR_UNSUPPORTED, "AXPBY takes bf16 operands");
    if (!d.c || d.ldc < d.N) return set_error(UFP8_ERR_INVALID, "AXPBY needs c with ldc >= N");
    if (reinterpret_cast<uintptr_t>(d.c) & 1u) return set_error(UFP8_ERR_ALIGN, "AXPBY: c not 2-byte aligned");
    if (d.K == 0 && d.M > 0 && d.N > 0) return set_error(UFP8_ERR_UNSUPPORTED, "AXPBY with K == 0");
  }
  if (d.tile_mask < UFP8_TILES_ALL || d.tile_mask > UFP8_TILES_K_FROM_DIAG)
    return set_error(UFP8_ERR_INVALID, "unknown tile_mask %d", d.tile_mask);
  if (d.tile_mask != UFP8_TILES_ALL && !bf16)
    return set_error(UFP8_ERR_UNSUPPORTED, "tile masks take bf16 operands");
  if (bf16 && (variant == UFP8_GEMM_SINGLE_CTA || d.ag_flags != nullptr))
    return set_error(UFP8_ERR_UNSUPPORTED, "bf16 operands run on the CTA-pair kernel without all-gather");
  if (d.epilogue == UFP8_EPI_XENT) {
    if (d.d_dtype != UFP8_OUT_BF16 || d.batch != 1)
      return set_error(UFP8_ERR_INVALID, "XENT needs bf16 output and batch 1");
    if (!d.xent_stats || d.xent_ld_stats < (d.N + 127) / 128)
      return set_error(UFP8_ERR_INVALID, "XENT needs xent_stats with xent_ld_stats >= ceil(N / 128)");
    if (reinterpret_cast<uintptr_t>(d.xent_stats) & 7u)
      return set_error(UFP8_ERR_ALIGN, "XENT: xent_stats is not 8-byte aligned");
    if (!(d.xent_cap >= 0.0f) || std::isinf(d.xent_cap))
      return set_error(UFP8_ERR_INVALID, "XENT: xent_cap must be 0 or a finite positive value");
    if (variant == UFP8_GEMM_SINGLE_CTA)
      return set_error(UFP8_ERR_UNSUPPORTED, "XENT runs on the CTA-pair kernel only");
    if (d.K == 0 && d.M > 0 && d.N > 0) return set_error(UFP8_ERR_UNSUPPORTED, "XENT with K == 0");
  }
  const bool rs = d.epilogue == UFP8_EPI_RS_PUSH;
  if (rs && (!d.rs_slots || d.rs_rows_per_rank <= 0 || d.rs_rank < 0 || d.d_dtype != UFP8_OUT_BF16 ||
             d.batch != 1 || d.M % d.rs_rows_per_rank != 0 || d.rs_rank >= d.M / d.rs_rows_per_rank))
    return set_error(UFP8_ERR_INVALID, "RS_PUSH needs rs_slots, bf16 output, batch 1, and M a multiple of "
                                       "rs_rows_per_rank with rs_rank < M / rs_rows_per_rank");
  const bool ag = d.ag_flags != nullptr;
  if (ag && (rs || variant == UFP8_GEMM_SINGLE_CTA || d.batch != 1 || d.k_batches != 1 || d.ag_rows_per_rank <= 0 ||
             d.ag_rows_per_rank % (2 * kBM) != 0 || d.M % d.ag_rows_per_rank != 0 || d.ag_rank < 0 ||
             d.ag_rank >= d.M / d.ag_rows_per_rank || d.M / d.ag_rows_per_rank > 32))
    return set_error(UFP8_ERR_INVALID, "all-gathered A needs the CTA-pair kernel, no RS_PUSH, batch 1, k_batches 1, "
                                       "ag_rows_per_rank a multiple of 256 dividing M into at most 32 blocks, and "
                                       "ag_rank < M / ag_rows_per_rank");
  if (rs && variant == UFP8_GEMM_SINGLE_CTA)
    return set_error(UFP8_ERR_UNSUPPORTED, "RS_PUSH runs on the CTA-pair kernel only");
  if (d.d_dtype != UFP8_OUT_BF16 && d.d_dtype != UFP8_OUT_F32)
    return set_error(UFP8_ERR_INVALID, "unknown output dtype %d", d.d_dtype);
  if ((d.epilogue == UFP8_EPI_SWIGLU || d.epilogue == UFP8_EPI_DSWIGLU) &&
      (d.d_dtype != UFP8_OUT_BF16 || d.batch != 1 || d.k_batches != 1))
    return set_error(UFP8_ERR_INVALID, "SWIGLU/DSWIGLU epilogues need bf16 output, batch 1, k_batches 1");
  if (!d.d && !rs && d.epilogue != UFP8_EPI_ATTN_STATS) return set_error(UFP8_ERR_INVALID, "null output pointer");
  if (d.ldd < d.N) return set_error(UFP8_ERR_INVALID, "ldd < N");
  if (d.epilogue == UFP8_EPI_SWIGLU && (!d.h || d.ldh < d.N))
    return set_error(UFP8_ERR_INVALID, "SWIGLU needs h with ldh >= N");
  if (d.epilogue == UFP8_EPI_DSWIGLU && (!d.ug || d.ldug < d.N))
    return set_error(UFP8_ERR_INVALID, "DSWIGLU needs ug with ldug >= N");
  if ((d.epilogue == UFP8_EPI_SWIGLU || d.epilogue == UFP8_EPI_DSWIGLU) && !d.amax_out)
    return set_error(UFP8_ERR_INVALID, "SWIGLU/DSWIGLU need amax_out");
  if (d.M >= (int64_t(1) << 31) || d.N >= (int64_t(1) << 31) || d.K >= (int64_t(1) << 31))
    return set_error(UFP8_ERR_INVALID, "extent exceeds 2^31");

  cudaError_t e;
  if (d.amax_out) {
    e = cudaMemsetAsync(d.amax_out, 0, sizeof(float), stream);
    if (e != cudaSuccess) return cuda_error(e, "cudaMemsetAsync(amax_out)");
  }
  if (d.M == 0 || d.N == 0) return UFP8_OK;

  GemmArgs a{};
  a.M = static_cast<int>(d.M);
  a.N = static_cast<int>(d.N);
  a.K = static_cast<int>(d.K);
  a.batch = d.batch;
  a.k_batches = d.k_batches;
  a.mode = d.epilogue;
  a.d = d.d;
  a.d_f32 = d.d_dtype == UFP8_OUT_F32;
  a.ldd = d.ldd;
  a.d_bstride = d.d_batch_stride;
  a.h = static_cast<__nv_bfloat16*>(d.h);
  a.ldh = d.ldh;
  a.ug = static_cast<const __nv_bfloat16*>(d.ug);
  a.ldug = d.ldug;
  a.ug_bstride = d.ug_batch_stride;
  a.amax_bits = reinterpret_cast<unsigned int*>(d.amax_out);
  a.status = dev.status_word;
  a.group_m = group_m > 0 ? group_m : 16;
  a.rs_slots = d.rs_slots;
  a.rs_rank = d.rs_rank;
  a.rs_rows = d.rs_rows_per_rank;
  a.ag_flags = d.ag_flags;
  a.ag_epoch = d.ag_epoch;
  a.ag_rank = d.ag_rank;
  a.ag_rows = d.ag_rows_per_rank;
  a.xent_stats = d.epilogue == UFP8_EPI_XENT ? d.xent_stats : nullptr;
  a.xent_ld = d.xent_ld_stats;
  a.xent_cap = d.xent_cap;
  a.c = d.epilogue == UFP8_EPI_AXPBY ? static_cast<const __nv_bfloat16*>(d.c) : nullptr;
  a.ldc = d.ldc;
  a.c_bstride = d.c_batch_stride;
  a.alpha_mul = d.epilogue == UFP8_EPI_AXPBY ? d.alpha : 1.0f;
  a.beta = d.beta;
  a.c_vec = a.c != nullptr && aligned16(d.c) && (d.ldc * 2) % 16 == 0 && (d.c_batch_stride * 2) % 16 == 0;
  a.tile_mask = d.tile_mask;
  a.attn_qseg = attn ? d.attn_q_segment_ids : nullptr;
  a.attn_kseg = attn ? d.attn_kv_segment_ids : nullptr;
  a.attn_stats = d.epilogue == UFP8_EPI_ATTN_STATS ? d.attn_stats : nullptr;
  a.attn_ld = d.attn_ld_stats;
  a.attn_row = attn ? d.attn_row : nullptr;
  a.attn_p = d.epilogue == UFP8_EPI_ATTN_DS ? static_cast<const __nv_bfloat16*>(d.c) : nullptr;
  a.attn_scale = d.attn_scale;
  a.attn_kseg_vec = (reinterpret_cast<uintptr_t>(d.attn_kv_segment_ids) & 15u) == 0;
  if (d.epilogue == UFP8_EPI_ATTN_DS) {
    a.ldc = d.ldc;
    a.c_bstride = d.c_batch_stride;
    a.c_vec = aligned16(d.c) && (d.ldc * 2) % 16 == 0 && (d.c_batch_stride * 2) % 16 == 0;
  }

  if (d.K == 0) {
    if (rs) return set_error(UFP8_ERR_UNSUPPORTED, "RS_PUSH with K == 0");
    zero_outputs_kernel<<<dev.sm_count * 4, 256, 0, stream>>>(a);
    e = cudaGetLastError();
    return e == cudaSuccess ? UFP8_OK : cuda_error(e, "zero-fill launch");
  }

  const bool swiglu = d.epilogue == UFP8_EPI_SWIGLU;
  // k_batches > 1: operand slice g * k_batches + kb holds batch g's K block kb.
  const int64_t kslices = static_cast<int64_t>(d.batch) * d.k_batches;
  if (kslices >= (int64_t(1) << 31)) return set_error(UFP8_ERR_INVALID, "batch * k_batches exceeds 2^31");
  const int a_group = d.a.batch_group > 1 ? d.a.batch_group : 1;
  const int b_group = d.b.batch_group > 1 ? d.b.batch_group : 1;
  if (d.a.batch_group < 0 || d.b.batch_group < 0) return set_error(UFP8_ERR_INVALID, "negative batch_group");
  if ((a_group > 1 || b_group > 1) && (d.k_batches > 1 || swiglu))
    return set_error(UFP8_ERR_UNSUPPORTED, "batch_group > 1 with k_batches > 1 or SWIGLU");
  const int a_need = (d.batch + a_group - 1) / a_group, b_need = (d.batch + b_group - 1) / b_group;
  int rc = check_operand(d.a, d.M, d.K, d.k_batches > 1 ? static_cast<int>(kslices) : (d.a.batch_count > 1 ? a_need : 1), "A");
  if (rc) return rc;
  rc = check_operand(d.b, d.N, d.K, swiglu ? 2 : (d.k_batches > 1 ? static_cast<int>(kslices) : (d.b.batch_count > 1 ? b_need : 1)),
                     "B");
  if (rc) return rc;
  a.a_group = a_group;
  a.b_group = b_group;

  a.a_major = d.a.major;
  a.b_major = d.b.major;
  a.a_bcast = d.a.batch_count <= 1 && d.k_batches == 1;
  a.b_bcast = !swiglu && d.b.batch_count <= 1 && d.k_batches == 1;
  a.inv_a = d.a.inv_scale;
  a.inv_b = d.b.inv_scale;
  const bool pair = variant != UFP8_GEMM_SINGLE_CTA;
  const int bm = pair ? 2 * kBM : kBM;
  a.tiles_m = static_cast<int>((d.M + bm - 1) / bm);
  const int bn = swiglu ? 128 : kBN;
  a.tiles_n = static_cast<int>((d.N + bn - 1) / bn);
  a.ksteps = static_cast<int>((d.K + kBK - 1) / kBK);
  // RS_PUSH: every rank computes the same tile sequence, so without a rotation all ranks
  // would push into the same owner at the same time and share its inbound links.  Rank r
  // starts at its own rows instead; at any moment the ranks then write to different owners.
  a.m_shift = rs ? static_cast<int>((static_cast<int64_t>(d.rs_rank) * d.rs_rows_per_rank / bm) % a.tiles_m) : 0;
  if (ag) {
    // All-gathered A: start at this rank's own rows (no wait), then the blocks in the order
    // ufp8_tp_ag_push delivers them (rank + 1, rank + 2, ...), one block per raster group.
    a.m_shift = static_cast<int>((static_cast<int64_t>(d.ag_rank) * d.ag_rows_per_rank / bm) % a.tiles_m);
    a.group_m = static_cast<int>(std::min<int64_t>(a.group_m, d.ag_rows_per_rank / bm));
  }
  a.idesc = (1u << 4)                                       // f32 accumulator
            | (static_cast<uint32_t>(bf16 ? 1 : d.a.fmt) << 7)   // A format (kind::f16: 1 = bf16)
            | (static_cast<uint32_t>(bf16 ? 1 : d.b.fmt) << 10)  // B format
            | (static_cast<uint32_t>(d.a.major) << 15)      // A major
            | (static_cast<uint32_t>(d.b.major) << 16)      // B major
            | (static_cast<uint32_t>(kBN >> 3) << 17)       // N = 256
            | (static_cast<uint32_t>(bm >> 4) << 24);       // M = 128 (one CTA) or 256 (CTA pair)

  const int esz = a.d_f32 ? 4 : 2;
  bool vec = (rs || aligned16(d.d)) && (d.ldd * esz) % 16 == 0 && (d.d_batch_stride * esz) % 16 == 0;
  if (swiglu) vec = vec && aligned16(d.h) && (d.ldh * 2) % 16 == 0;
  if (d.epilogue == UFP8_EPI_DSWIGLU) vec = vec && aligned16(d.ug) && (d.ldug * 2) % 16 == 0 && (d.ug_batch_stride * 2) % 16 == 0;
  // 32-byte stores where every row start is 32-byte aligned (the direct epilogues' bf16 rows).
  auto aligned32 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 31u) == 0; };
  bool vec32 = vec && !a.d_f32 && !rs && aligned32(d.d) && (d.ldd * esz) % 32 == 0 && (d.d_batch_stride * esz) % 32 == 0;
  if (swiglu) vec32 = vec32 && aligned32(d.h) && (d.ldh * 2) % 32 == 0;
  a.vec_ok = vec ? (vec32 ? 2 : 1) : 0;

  CUtensorMap tmA, tmB;
  rc = encode_operand(&tmA, d.a, d.M, d.K, "A");
  if (rc) return rc;
  rc = encode_operand(&tmB, d.b, d.N, d.K, "B");
  if (rc) return rc;

  static thread_local int attr_device = -1;
  if (attr_device != dev.device) {
    e = cudaFuncSetAttribute(gemm_fp8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gemm_fp8_pair_kernel<kPStages, kVarDirect>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, kPSmemBytes);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gemm_fp8_pair_kernel<kPStagesStaged, kVarRsStaged>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, kPSmemBytesStaged);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gemm_fp8_pair_kernel<kPStagesStaged, kVarUgStaged>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, kPSmemBytesUg);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gemm_fp8_pair_kernel<kPStagesWide, kVarDirect, 2>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, kPSmemBytesWide);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gemm_fp8_pair_kernel<kPStagesWideStaged, kVarRsStaged, 2>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, kPSmemBytesWideStaged);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gemm_fp8_pair_kernel<kPStagesWideStaged, kVarUgStaged, 2>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, kPSmemBytesWideUg);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gemm_fp8_n512_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kWSmemBytes);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gemm_fp8_pair_kernel<kPStagesWide, kVarDirect, 2, true>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, kPSmemBytesWide);
    if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(gemm smem)");
    attr_device = dev.device;
  }
  // Staged variants of the CTA-pair kernel, whenever the rows they touch are 16-byte aligned:
  // RS_PUSH rows leave through shared memory as bulk stores; DSWIGLU reads U / G through TMA.
  // (Plain local outputs keep the direct stores and the deeper ring: at these tile sizes their
  // stores never limit the epilogue, while two more ring stages help the long-K contractions.)
  int var = kVarDirect;
  if (pair && variant != UFP8_GEMM_CTA_PAIR_DIRECT && vec) {
    if (rs) var = kVarRsStaged;
    if (d.epilogue == UFP8_EPI_DSWIGLU) var = kVarUgStaged;
  }
  // Direct epilogues on the pair kernel (the default, UFP8_GEMM_AUTO, and UFP8_GEMM_CTA_PAIR_WIDE):
  // ring stages of two 128-byte K chunks, 3 deep.  Half as many full/empty hand-offs per FLOP as
  // the 7-deep ring of single chunks (UFP8_GEMM_CTA_PAIR), which measured 8-9 % slower on the
  // long-K GMLP contractions (F2 754 vs 694 us, B4 1484 vs 1355 us at 16384 x 4096 x 14336 / 28672).
  // The staged epilogues keep the single-chunk ring unless UFP8_GEMM_CTA_PAIR_WIDE asks for two
  // chunks there too (2 stages beside the RS rows or the U/G boxes).
  // 256 x 512 tiles (gemm_fp8_n512_kernel) for bf16 STORE / SWIGLU outputs: always with
  // UFP8_GEMM_CTA_PAIR_N512; by default (UFP8_GEMM_AUTO) for bf16 STORE outputs when the tile
  // rounds favour it.  A 256 x 512 tile runs in ~0.92x the time of two 256 x 256 tiles on the
  // long-K GMLP contractions (F2 650 vs 680 us, B4 1250 vs 1311 us, B3 1305 vs 1333 us), but
  // half as many tiles quantise worse onto the persistent grid and a ragged N wastes more.
  bool n512 = pair && var == kVarDirect && !a.d_f32 && (d.epilogue == UFP8_EPI_STORE || swiglu) &&
              variant == UFP8_GEMM_CTA_PAIR_N512 && !bf16;
  if (pair && var == kVarDirect && !a.d_f32 && d.epilogue == UFP8_EPI_STORE && variant == UFP8_GEMM_AUTO && !bf16) {
    const int64_t nc = dev.sm_count / 2;
    const int64_t t256 = static_cast<int64_t>(a.tiles_m) * ((d.N + 255) / 256) * d.batch;
    const int64_t t512 = static_cast<int64_t>(a.tiles_m) * ((d.N + 511) / 512) * d.batch;
    n512 = 1.84 * static_cast<double>((t512 + nc - 1) / nc) <= static_cast<double>((t256 + nc - 1) / nc);
  }
  const bool wide = bf16 || (!n512 && pair &&
                    ((var == kVarDirect && (variant == UFP8_GEMM_AUTO || variant == UFP8_GEMM_CTA_PAIR_WIDE)) ||
                     (var != kVarDirect && variant == UFP8_GEMM_CTA_PAIR_WIDE)));
  if (n512) a.tiles_n = static_cast<int>((d.N + 2 * bn - 1) / (2 * bn));
  const int kch = wide ? 2 : 1;
  const int kelems = bf16 ? kBK / 2 : kBK;  // K elements per 128-byte chunk
  a.ksteps = static_cast<int>((d.K + kch * kelems - 1) / (kch * kelems));
  CUtensorMap tmUG, tmD;
  std::memset(&tmUG, 0, sizeof(tmUG));
  std::memset(&tmD, 0, sizeof(tmD));
  if (var == kVarUgStaged) {
    rc = encode_ug(&tmUG, d);
    if (rc) return rc;
    rc = encode_bf16_boxes(&tmD, d.d, d.N, d.M, d.ldd, d.d_batch_stride, "D");
    if (rc) return rc;
  }
  using PairFn = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap, const GemmArgs);
  PairFn pair_kernel;
  int pair_smem;
  if (var == kVarRsStaged) {
    pair_kernel = wide ? gemm_fp8_pair_kernel<kPStagesWideStaged, kVarRsStaged, 2> : gemm_fp8_pair_kernel<kPStagesStaged, kVarRsStaged>;
    pair_smem = wide ? kPSmemBytesWideStaged : kPSmemBytesStaged;
  } else if (var == kVarUgStaged) {
    pair_kernel = wide ? gemm_fp8_pair_kernel<kPStagesWideStaged, kVarUgStaged, 2> : gemm_fp8_pair_kernel<kPStagesStaged, kVarUgStaged>;
    pair_smem = wide ? kPSmemBytesWideUg : kPSmemBytesUg;
  } else if (bf16) {
    pair_kernel = gemm_fp8_pair_kernel<kPStagesWide, kVarDirect, 2, true>;
    pair_smem = kPSmemBytesWide;
  } else {
    pair_kernel = wide ? gemm_fp8_pair_kernel<kPStagesWide, kVarDirect, 2> : gemm_fp8_pair_kernel<kPStages, kVarDirect>;
    pair_smem = wide ? kPSmemBytesWide : kPSmemBytes;
  }
  if (n512) pair_smem = kWSmemBytes;
  const void* pair_fn = n512 ? reinterpret_cast<const void*>(gemm_fp8_n512_kernel)
                             : reinterpret_cast<const void*>(pair_kernel);
  const int occ_slot = bf16 ? 7 : (n512 ? 6 : var + (wide ? 3 : 0));
  const long long num_tiles = static_cast<long long>(a.tiles_m) * a.tiles_n * a.batch;
  if (num_tiles >= (1ll << 31)) return set_error(UFP8_ERR_INVALID, "too many tiles");
  int ctas = ctas_override > 0 ? ctas_override : dev.sm_count;
  if (pair) {
    static thread_local int occ_device[8] = {-1, -1, -1, -1, -1, -1, -1, -1}, occ_clusters[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (occ_device[occ_slot] != dev.device) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2 * (dev.sm_count / 2), 1, 1);
      cfg.blockDim = dim3(kPThreads, 1, 1);
      cfg.dynamicSmemBytes = pair_smem;
      int n = 0;
      e = cudaOccupancyMaxActiveClusters(&n, pair_fn, &cfg);
      if (e != cudaSuccess) return cuda_error(e, "cudaOccupancyMaxActiveClusters");
      if (n < 1) return set_error(UFP8_ERR_DEVICE, "no CTA pair of the GEMM kernel fits on this device");
      occ_clusters[occ_slot] = n;
      occ_device[occ_slot] = dev.device;
    }
    const int max_clusters = occ_clusters[occ_slot];
    // Persistent grid: no more clusters than can be resident at once.
    if (ctas_override <= 0 || ctas > 2 * max_clusters) ctas = 2 * max_clusters;
    long long clusters = ctas / 2;
    if (clusters < 1) clusters = 1;
    if (num_tiles < clusters) clusters = num_tiles;
    const int grid = static_cast<int>(2 * clusters);
    if (n512)
      gemm_fp8_n512_kernel<<<grid, kPThreads, pair_smem, stream>>>(tmA, tmB, a);
    else
      pair_kernel<<<grid, kPThreads, pair_smem, stream>>>(tmA, tmB, tmUG, tmD, a);
  } else {
    if (num_tiles < ctas) ctas = static_cast<int>(num_tiles);
    gemm_fp8_kernel<<<ctas, kThreads, kSmemBytes, stream>>>(tmA, tmB, a);
  }
  e = cudaGetLastError();
  return e == cudaSuccess ? UFP8_OK : cuda_error(e, "gemm kernel launch");
}

}  // namespace ufp8
