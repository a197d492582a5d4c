// Tensor-parallel reduce-scatter support: peer-mapped staging buffers over NVLink (CUDA IPC,
// no multicast objects) and the owner-side finish kernel.
//
// Protocol for one reduce-scatter of a [T, C] bf16 partial sum over k ranks (rows split in
// k contiguous blocks of R = T / k):
//   1. every rank's GEMM epilogue (UFP8_EPI_RS_PUSH) stores row m of its partial into the
//      owner o = m / R, in o's staging buffer, slot = its own rank:  slot[src][m - o*R][c];
//   2. ufp8_tp_finish on every rank: CTA 0 first publishes "my partials for epoch e are
//      written" by storing e into every peer's flag[src = me] (after a system-scope fence);
//      every CTA then waits until its own flag[src] == e for all src (bounded by a timeout; on
//      expiry it sets UFP8_STATUS_PEER_TIMEOUT in the status word and stops), then sums the k
//      slots in fp32 in rank order and writes the bf16 result.
// Two staging buffers alternate by epoch, so a fast rank that moves on to the next
// reduce-scatter writes into the other buffer while slower owners are still summing.
//
// The all-gather (ufp8_tp_ag_push) uses the same layout the other way round: slot [s] of
// every rank's buffer receives rank s's block, by copy engine, and flag[s] = epoch follows
// each copy; the consuming GEMM waits per row block (ufp8_gemm_desc.ag_*).
#include <cuda_bf16.h>

#include <algorithm>
#include <cstring>
#include <vector>

#include "internal.h"
#include "ptx.cuh"

namespace ufp8 {

constexpr int kMaxRanks = 8;
constexpr size_t kFlagBytes = 256;  // flag[src] (u32) per buffer, padded
// Small-value exchange region after the two staging buffers: [2 buffers][kMaxRanks sources]
// entries of 64 bytes, {u32 epoch, u32 pad, u32 value bits[kMaxExchange]}.
constexpr int kMaxExchange = 8;
constexpr size_t kExEntryBytes = 64;
constexpr size_t kExBytes = 2 * kMaxRanks * kExEntryBytes;

struct TPContext {
  int device = -1;
  int rank = 0;
  int world = 1;
  size_t slot_bytes = 0;     // one source rank's block in one buffer
  size_t buffer_bytes = 0;   // flags + world slots
  char* base = nullptr;      // own allocation: 2 buffers
  char* peer_base[kMaxRanks] = {};
  bool peer_opened[kMaxRanks] = {};
  void** d_slot_ptrs = nullptr;  // device array [2][world]: data region of buffer b on each rank
  uint64_t epoch = 0;
  uint64_t ex_epoch = 0;          // small-value exchanges issued
  int timeout_ms = 5000;
  // Copy lanes: the copy-engine pushes spread their per-peer copies over `lanes` streams
  // (forked from and joined back into the caller's stream), created on first use.
  int lanes = 1;
  cudaStream_t lane_stream[kMaxRanks] = {};
  cudaEvent_t fork_event = nullptr;
  cudaEvent_t lane_event[kMaxRanks] = {};
  char* ex_region(int p) const { return peer_base[p] + 2 * buffer_bytes; }
};

namespace {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_relaxed_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Forks the copy lanes from `s`: every lane stream waits for the work issued on `s` so far.
// With one lane the caller's stream is the lane.  Returns 0 or a UFP8 error code.
int lanes_fork(TPContext* c, cudaStream_t s, int n) {
  if (n <= 1) {
    c->lane_stream[0] = nullptr;
    return UFP8_OK;
  }
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_error(e, "copy lanes: cudaGetDevice");
  if (dev != c->device) return set_error(UFP8_ERR_INVALID, "copy lanes: current device %d, context on %d", dev, c->device);
  if (!c->fork_event && (e = cudaEventCreateWithFlags(&c->fork_event, cudaEventDisableTiming)) != cudaSuccess)
    return cuda_error(e, "copy lanes: event");
  for (int l = 0; l < n; ++l) {
    if (!c->lane_stream[l] && (e = cudaStreamCreateWithFlags(&c->lane_stream[l], cudaStreamNonBlocking)) != cudaSuccess)
      return cuda_error(e, "copy lanes: stream");
    if (!c->lane_event[l] && (e = cudaEventCreateWithFlags(&c->lane_event[l], cudaEventDisableTiming)) != cudaSuccess)
      return cuda_error(e, "copy lanes: event");
  }
  if ((e = cudaEventRecord(c->fork_event, s)) != cudaSuccess) return cuda_error(e, "copy lanes: fork record");
  for (int l = 0; l < n; ++l)
    if ((e = cudaStreamWaitEvent(c->lane_stream[l], c->fork_event, 0)) != cudaSuccess)
      return cuda_error(e, "copy lanes: fork wait");
  return UFP8_OK;
}

cudaStream_t lane_of(const TPContext* c, cudaStream_t s, int n, int i) {
  return n <= 1 ? s : c->lane_stream[i % n];
}

// Joins the lanes back into `s`: work issued on `s` afterwards waits for every lane's copies.
int lanes_join(TPContext* c, cudaStream_t s, int n) {
  if (n <= 1) return UFP8_OK;
  cudaError_t e;
  for (int l = 0; l < n; ++l) {
    if ((e = cudaEventRecord(c->lane_event[l], c->lane_stream[l])) != cudaSuccess)
      return cuda_error(e, "copy lanes: join record");
    if ((e = cudaStreamWaitEvent(s, c->lane_event[l], 0)) != cudaSuccess) return cuda_error(e, "copy lanes: join wait");
  }
  return UFP8_OK;
}

struct FinishArgs {
  uint32_t* flags_local;            // this rank's flags of the buffer in use
  uint32_t* flags_peer[kMaxRanks];  // every rank's flags of the buffer in use
  const __nv_bfloat16* slots;       // this rank's data region of the buffer in use
  long long slot_elems;             // elements per slot (R * ld_slot)
  long long ld_slot;
  int world, rank;
  uint32_t epoch;
  long long rows, cols;
  __nv_bfloat16* out;
  long long ld_out;
  uint64_t timeout_ns;
  int* status;
  int vec8;  // cols, pitches and out allow 16-byte accesses
};

__global__ void __launch_bounds__(256) tp_finish_kernel(const FinishArgs a) {
  __shared__ int ok_shared;
  if (threadIdx.x == 0) {
    // One signal per rank (CTA 0); every CTA then polls the k local flags with relaxed
    // system-scope loads and takes a single acquire fence once all of them carry the epoch.
    // (All CTAs are resident: the grid is capped at 4 CTAs of 256 threads per SM.)
    if (blockIdx.x == 0) {
      __threadfence_system();
      for (int p = 0; p < a.world; ++p) st_release_sys(a.flags_peer[p] + a.rank, a.epoch);
    }
    int ok = 1;
    const uint64_t t0 = globaltimer_ns();
    for (int src = 0; src < a.world && ok; ++src) {
      while (ld_relaxed_sys(a.flags_local + src) != a.epoch) {
        if (globaltimer_ns() - t0 > a.timeout_ns) {
          ok = 0;
          atomicOr(a.status, UFP8_STATUS_PEER_TIMEOUT);
          break;
        }
      }
    }
    fence_acq_rel_sys();
    ok_shared = ok;
  }
  __syncthreads();
  if (!ok_shared) return;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  if (a.vec8) {
    // 8 columns per thread: one 16-byte load per slot, fp32 sums, one 16-byte store.
    const long long cols8 = a.cols / 8;
    const long long total8 = a.rows * cols8;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total8; i += stride) {
      const long long r = i / cols8, c = (i - r * cols8) * 8;
      uint4 v8[kMaxRanks];
#pragma unroll
      for (int src = 0; src < kMaxRanks; ++src)  // all loads in flight before the sums
        if (src < a.world) v8[src] = *reinterpret_cast<const uint4*>(a.slots + src * a.slot_elems + r * a.ld_slot + c);
      float acc[8] = {};
#pragma unroll
      for (int src = 0; src < kMaxRanks; ++src) {
        if (src >= a.world) break;
        const uint32_t w[4] = {v8[src].x, v8[src].y, v8[src].z, v8[src].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc[2 * j] += __uint_as_float(w[j] << 16);
          acc[2 * j + 1] += __uint_as_float(w[j] & 0xFFFF0000u);
        }
      }
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const __nv_bfloat162 b = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
        o[j] = *reinterpret_cast<const uint32_t*>(&b);
      }
      *reinterpret_cast<uint4*>(a.out + r * a.ld_out + c) = make_uint4(o[0], o[1], o[2], o[3]);
    }
    return;
  }
  const long long cols2 = a.cols / 2;  // bf16 pairs (cols is even)
  const long long total = a.rows * cols2;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total; i += stride) {
    const long long r = i / cols2, c = (i - r * cols2) * 2;
    float s0 = 0.0f, s1 = 0.0f;
    for (int src = 0; src < a.world; ++src) {
      const __nv_bfloat162 v =
          *reinterpret_cast<const __nv_bfloat162*>(a.slots + src * a.slot_elems + r * a.ld_slot + c);
      s0 += __bfloat162float(v.x);
      s1 += __bfloat162float(v.y);
    }
    *reinterpret_cast<__nv_bfloat162*>(a.out + r * a.ld_out + c) = __floats2bfloat162_rn(s0, s1);
  }
}

struct ExchangeArgs {
  char* entry_peer[kMaxRanks];  // &peer p's exchange entry [b][rank]
  const char* entry_local;      // &own exchange entry [b][0]
  const uint32_t* in;           // n f32 bit patterns (non-negative values or NaN)
  uint32_t* out;
  int n, world;
  uint32_t epoch;
  uint64_t timeout_ns;
  int* status;
};

// MAX all-reduce of n <= 8 non-negative f32 values (amax values) over the group: one warp.
// Lane p stores the values into peer p's entry [b][rank] and then the epoch with a system-scope
// release; lane s waits (bounded) for entry [b][s] of this rank to carry the epoch and reads
// it.  Unsigned max of the bit patterns = float max for non-negative values, and propagates
// NaN (0x7FC00000 is above every finite value and inf), as the amax kernel does.
__global__ void __launch_bounds__(32) tp_exchange_max_kernel(const ExchangeArgs a) {
  const int lane = threadIdx.x;
  uint32_t v[kMaxExchange];
#pragma unroll
  for (int i = 0; i < kMaxExchange; ++i) v[i] = i < a.n ? a.in[i] : 0u;
  if (lane < a.world) {
    uint32_t* e = reinterpret_cast<uint32_t*>(a.entry_peer[lane]);
#pragma unroll
    for (int i = 0; i < kMaxExchange; ++i)
      if (i < a.n) asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(e + 2 + i), "r"(v[i]) : "memory");
    st_release_sys(e, a.epoch);
  }
  bool ok = true;
  uint32_t m[kMaxExchange];
#pragma unroll
  for (int i = 0; i < kMaxExchange; ++i) m[i] = 0u;
  if (lane < a.world) {
    const uint32_t* e = reinterpret_cast<const uint32_t*>(a.entry_local + lane * kExEntryBytes);
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_sys(e) != a.epoch) {
      if (globaltimer_ns() - t0 > a.timeout_ns) {
        ok = false;
        break;
      }
    }
    if (ok) {
#pragma unroll
      for (int i = 0; i < kMaxExchange; ++i)
        if (i < a.n) {
          uint32_t x;
          asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(x) : "l"(e + 2 + i) : "memory");
          m[i] = x;
        }
    }
  }
  ok = __all_sync(0xFFFFFFFFu, ok);
  if (!ok) {
    if (lane == 0) atomicOr(a.status, UFP8_STATUS_PEER_TIMEOUT);
    return;
  }
#pragma unroll
  for (int i = 0; i < kMaxExchange; ++i) {
    const uint32_t r = __reduce_max_sync(0xFFFFFFFFu, m[i]);
    if (lane == 0 && i < a.n) a.out[i] = r;
  }
}

constexpr int kAgThreads = 256;
constexpr int kAgCtas = 64;
constexpr size_t kAgCounterOffset = 128;  // per-destination counters inside the flags area

struct AgPushArgs {
  const uint4* src;
  uint4* dst[kMaxRanks];        // [i-1]: slot [rank] of peer rank-i
  uint32_t* flag[kMaxRanks];    // [i-1]: flag[rank] of peer rank-i
  unsigned int* counter;        // [i-1]: CTAs done with destination i (own memory, self-resetting)
  long long n16;
  int ndst;
  uint32_t epoch;
};

// Copies this rank's all-gather block to the k-1 peers, one destination after the other so
// that the blocks arrive staggered in the order the consuming GEMMs use them.  Every CTA
// copies its share of the block to destination i (coalesced 16-byte loads and remote stores),
// then thread 0 (after __syncthreads) fences at system scope and counts; the last CTA of a
// destination resets the count and releases that peer's flag.  No shared memory, at most 32
// registers a thread: with the maximum shared-memory carveout its CTAs fit beside a persistent
// GEMM CTA (320 threads x 168 registers, ~225 KiB of shared memory).
__global__ void __launch_bounds__(kAgThreads, 8) tp_ag_push_kernel(const AgPushArgs a) {
  const long long stride = static_cast<long long>(gridDim.x) * kAgThreads;
  for (int di = 0; di < a.ndst; ++di) {
    uint4* dst = a.dst[di];
    long long i = static_cast<long long>(blockIdx.x) * kAgThreads + threadIdx.x;
    for (; i + stride < a.n16; i += 2 * stride) {
      const uint4 v0 = a.src[i], v1 = a.src[i + stride];
      dst[i] = v0;
      dst[i + stride] = v1;
    }
    if (i < a.n16) dst[i] = a.src[i];
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence_system();
      const unsigned int prev = atomicAdd(a.counter + di, 1u);
      if (prev == gridDim.x - 1) {
        a.counter[di] = 0u;
        __threadfence_system();
        st_release_sys(a.flag[di], a.epoch);
      }
    }
  }
}

}  // namespace

}  // namespace ufp8

using namespace ufp8;

extern "C" {

int ufp8_tp_create(int rank, int world, int64_t slot_bytes, ufp8_tp_ctx** out, uint8_t* ipc_handle_out) {
  if (!out || !ipc_handle_out) return set_error(UFP8_ERR_INVALID, "ufp8_tp_create: null pointer");
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world)
    return set_error(UFP8_ERR_INVALID, "ufp8_tp_create: rank %d / world %d (world must be 1..%d)", rank, world,
                     kMaxRanks);
  if (slot_bytes <= 0 || slot_bytes % 256) return set_error(UFP8_ERR_INVALID, "ufp8_tp_create: slot_bytes must be a positive multiple of 256");
  DeviceInfo* dev;
  if (int rc = device_info(&dev)) return rc;
  TPContext* c = new TPContext();
  c->device = dev->device;
  c->rank = rank;
  c->world = world;
  c->slot_bytes = static_cast<size_t>(slot_bytes);
  c->buffer_bytes = kFlagBytes + c->slot_bytes * world;
  cudaError_t e = cudaMalloc(&c->base, 2 * c->buffer_bytes + kExBytes);
  if (e == cudaSuccess) e = cudaMemset(c->base, 0, 2 * c->buffer_bytes + kExBytes);
  if (e == cudaSuccess) e = cudaMalloc(&c->d_slot_ptrs, 2 * kMaxRanks * sizeof(void*));
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, c->base);
  if (e != cudaSuccess) {
    if (c->base) cudaFree(c->base);
    if (c->d_slot_ptrs) cudaFree(c->d_slot_ptrs);
    delete c;
    return cuda_error(e, "ufp8_tp_create");
  }
  std::memcpy(ipc_handle_out, &h, sizeof(h));
  c->peer_base[rank] = c->base;
  *out = reinterpret_cast<ufp8_tp_ctx*>(c);
  return UFP8_OK;
}

int ufp8_tp_connect(ufp8_tp_ctx* ctx, const uint8_t* ipc_handles) {
  TPContext* c = reinterpret_cast<TPContext*>(ctx);
  if (!c || !ipc_handles) return set_error(UFP8_ERR_INVALID, "ufp8_tp_connect: null pointer");
  cudaError_t e;
  for (int p = 0; p < c->world; ++p) {
    if (p == c->rank || c->peer_opened[p]) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, ipc_handles + p * UFP8_IPC_HANDLE_BYTES, sizeof(h));
    void* ptr = nullptr;
    if ((e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess)) != cudaSuccess)
      return cuda_error(e, "ufp8_tp_connect: cudaIpcOpenMemHandle");
    c->peer_base[p] = static_cast<char*>(ptr);
    c->peer_opened[p] = true;
  }
  void* host[2 * kMaxRanks] = {};
  for (int b = 0; b < 2; ++b)
    for (int p = 0; p < c->world; ++p) host[b * kMaxRanks + p] = c->peer_base[p] + b * c->buffer_bytes + kFlagBytes;
  if ((e = cudaMemcpy(c->d_slot_ptrs, host, sizeof(host), cudaMemcpyHostToDevice)) != cudaSuccess)
    return cuda_error(e, "ufp8_tp_connect: peer table");
  return UFP8_OK;
}

int ufp8_tp_connect_local(ufp8_tp_ctx* ctx, ufp8_tp_ctx* const* peers) {
  TPContext* c = reinterpret_cast<TPContext*>(ctx);
  if (!c || !peers) return set_error(UFP8_ERR_INVALID, "ufp8_tp_connect_local: null pointer");
  for (int p = 0; p < c->world; ++p) {
    const TPContext* q = reinterpret_cast<const TPContext*>(peers[p]);
    if (!q || q->world != c->world || q->rank != p || q->slot_bytes != c->slot_bytes)
      return set_error(UFP8_ERR_INVALID, "ufp8_tp_connect_local: peers[%d] is not rank %d of this group", p, p);
    if (p != c->rank) c->peer_base[p] = q->base;
  }
  void* host[2 * kMaxRanks] = {};
  for (int b = 0; b < 2; ++b)
    for (int p = 0; p < c->world; ++p) host[b * kMaxRanks + p] = c->peer_base[p] + b * c->buffer_bytes + kFlagBytes;
  cudaError_t e = cudaMemcpy(c->d_slot_ptrs, host, sizeof(host), cudaMemcpyHostToDevice);
  return e == cudaSuccess ? UFP8_OK : cuda_error(e, "ufp8_tp_connect_local: peer table");
}

int ufp8_tp_destroy(ufp8_tp_ctx* ctx) {
  TPContext* c = reinterpret_cast<TPContext*>(ctx);
  if (!c) return UFP8_OK;
  for (int l = 0; l < kMaxRanks; ++l) {
    if (c->lane_stream[l]) cudaStreamDestroy(c->lane_stream[l]);
    if (c->lane_event[l]) cudaEventDestroy(c->lane_event[l]);
  }
  if (c->fork_event) cudaEventDestroy(c->fork_event);
  for (int p = 0; p < kMaxRanks; ++p)
    if (c->peer_opened[p]) cudaIpcCloseMemHandle(c->peer_base[p]);
  if (c->d_slot_ptrs) cudaFree(c->d_slot_ptrs);
  if (c->base) cudaFree(c->base);
  delete c;
  return UFP8_OK;
}

int ufp8_tp_set_timeout_ms(ufp8_tp_ctx* ctx, int ms) {
  TPContext* c = reinterpret_cast<TPContext*>(ctx);
  if (!c || ms <= 0) return set_error(UFP8_ERR_INVALID, "ufp8_tp_set_timeout_ms: bad argument");
  c->timeout_ms = ms;
  return UFP8_OK;
}

int ufp8_tp_begin(ufp8_tp_ctx* ctx, void* const** slot_table, uint64_t* epoch) {
  TPContext* c = reinterpret_cast<TPContext*>(ctx);
  if (!c || !slot_table || !epoch) return set_error(UFP8_ERR_INVALID, "ufp8_tp_begin: null pointer");
  for (int p = 0; p < c->world; ++p)
    if (!c->peer_base[p]) return set_error(UFP8_ERR_INVALID, "ufp8_tp_begin: rank %d is not connected", p);
  c->epoch += 1;
  *epoch = c->epoch;
  *slot_table = c->d_slot_ptrs + (c->epoch & 1) * kMaxRanks;
  return UFP8_OK;
}

int ufp8_tp_finish(ufp8_tp_ctx* ctx, uint64_t epoch, int64_t rows, int64_t cols, int64_t ld_slot, void* out,
                   int64_t ld_out, ufp8_stream_t stream) {
  TPContext* c = reinterpret_cast<TPContext*>(ctx);
  if (!c || !out) return set_error(UFP8_ERR_INVALID, "ufp8_tp_finish: null pointer");
  if (epoch == 0 || epoch > c->epoch) return set_error(UFP8_ERR_INVALID, "ufp8_tp_finish: epoch not begun");
  if (rows < 0 || cols <= 0 || cols % 2 || ld_slot < cols || ld_out < cols || ld_slot % 2 || ld_out % 2)
    return set_error(UFP8_ERR_INVALID, "ufp8_tp_finish: bad extents (cols and pitches must be even)");
  if (static_cast<size_t>(rows * ld_slot * 2) > c->slot_bytes)
    return set_error(UFP8_ERR_INVALID, "ufp8_tp_finish: %lld x %lld rows exceed the staging slot", (long long)rows,
                     (long long)ld_slot);
  if (reinterpret_cast<uintptr_t>(out) & 3u) return set_error(UFP8_ERR_ALIGN, "ufp8_tp_finish: out not 4-byte aligned");
  for (int p = 0; p < c->world; ++p)
    if (!c->peer_base[p]) return set_error(UFP8_ERR_INVALID, "ufp8_tp_finish: rank %d is not connected", p);
  DeviceInfo* dev;
  if (int rc = device_info(&dev)) return rc;
  const int b = static_cast<int>(epoch & 1);
  FinishArgs a{};
  a.flags_local = reinterpret_cast<uint32_t*>(c->base + b * c->buffer_bytes);
  for (int p = 0; p < c->world; ++p) a.flags_peer[p] = reinterpret_cast<uint32_t*>(c->peer_base[p] + b * c->buffer_bytes);
  a.slots = reinterpret_cast<const __nv_bfloat16*>(c->base + b * c->buffer_bytes + kFlagBytes);
  a.slot_elems = static_cast<long long>(c->slot_bytes / 2);
  a.ld_slot = ld_slot;
  a.world = c->world;
  a.rank = c->rank;
  a.epoch = static_cast<uint32_t>(epoch);
  a.rows = rows;
  a.cols = cols;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.ld_out = ld_out;
  a.timeout_ns = static_cast<uint64_t>(c->timeout_ms) * 1000000ull;
  a.status = dev->status_word;
  a.vec8 = (cols % 8 == 0 && ld_slot % 8 == 0 && ld_out % 8 == 0 && (c->slot_bytes % 16) == 0 &&
            (reinterpret_cast<uintptr_t>(out) & 15u) == 0)
               ? 1
               : 0;
  const long long items = a.vec8 ? rows * (cols / 8) : rows * (cols / 2);
  int grid = static_cast<int>((items + 255) / 256);
  if (grid > 4 * dev->sm_count) grid = 4 * dev->sm_count;  // all resident (256 threads, no shared memory)
  if (grid < 1) grid = 1;
  tp_finish_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? UFP8_OK : cuda_error(e, "tp finish launch");
}

int ufp8_tp_allreduce_max(ufp8_tp_ctx* ctx, const float* in, float* out, int n, ufp8_stream_t stream) {
  TPContext* c = reinterpret_cast<TPContext*>(ctx);
  if (!c || !in || !out) return set_error(UFP8_ERR_INVALID, "ufp8_tp_allreduce_max: null pointer");
  if (n < 1 || n > kMaxExchange)
    return set_error(UFP8_ERR_INVALID, "ufp8_tp_allreduce_max: n = %d (1..%d)", n, kMaxExchange);
  for (int p = 0; p < c->world; ++p)
    if (!c->peer_base[p]) return set_error(UFP8_ERR_INVALID, "ufp8_tp_allreduce_max: rank %d is not connected", p);
  DeviceInfo* dev;
  if (int rc = device_info(&dev)) return rc;
  c->ex_epoch += 1;
  const int b = static_cast<int>(c->ex_epoch & 1);
  ExchangeArgs a{};
  for (int p = 0; p < c->world; ++p)
    a.entry_peer[p] = c->ex_region(p) + (b * kMaxRanks + c->rank) * kExEntryBytes;
  a.entry_local = c->ex_region(c->rank) + b * kMaxRanks * kExEntryBytes;
  a.in = reinterpret_cast<const uint32_t*>(in);
  a.out = reinterpret_cast<uint32_t*>(out);
  a.n = n;
  a.world = c->world;
  a.epoch = static_cast<uint32_t>(c->ex_epoch);
  a.timeout_ns = static_cast<uint64_t>(c->timeout_ms) * 1000000ull;
  a.status = dev->status_word;
  tp_exchange_max_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? UFP8_OK : cuda_error(e, "tp exchange launch");
}

int ufp8_tp_local(ufp8_tp_ctx* ctx, uint64_t epoch, void** data, uint32_t** flags) {
  TPContext* c = reinterpret_cast<TPContext*>(ctx);
  if (!c || !data || !flags) return set_error(UFP8_ERR_INVALID, "ufp8_tp_local: null pointer");
  if (epoch == 0 || epoch > c->epoch) return set_error(UFP8_ERR_INVALID, "ufp8_tp_local: epoch not begun");
  char* buf = c->base + (epoch & 1) * c->buffer_bytes;
  *flags = reinterpret_cast<uint32_t*>(buf);
  *data = buf + kFlagBytes;
  return UFP8_OK;
}

int ufp8_tp_ag_push(ufp8_tp_ctx* ctx, uint64_t epoch, int64_t bytes, int engine, ufp8_stream_t stream) {
  TPContext* c = reinterpret_cast<TPContext*>(ctx);
  if (!c) return set_error(UFP8_ERR_INVALID, "ufp8_tp_ag_push: null context");
  if (engine != UFP8_AG_COPY_ENGINE && engine != UFP8_AG_SM)
    return set_error(UFP8_ERR_INVALID, "ufp8_tp_ag_push: unknown engine %d", engine);
  if (bytes % 16) return set_error(UFP8_ERR_ALIGN, "ufp8_tp_ag_push: bytes must be a multiple of 16");
  if (epoch == 0 || epoch > c->epoch) return set_error(UFP8_ERR_INVALID, "ufp8_tp_ag_push: epoch not begun");
  if (bytes < 0 || static_cast<size_t>(bytes) > c->slot_bytes)
    return set_error(UFP8_ERR_INVALID, "ufp8_tp_ag_push: %lld bytes exceed the slot", static_cast<long long>(bytes));
  for (int p = 0; p < c->world; ++p)
    if (!c->peer_base[p]) return set_error(UFP8_ERR_INVALID, "ufp8_tp_ag_push: rank %d is not connected", p);
  if (engine == UFP8_AG_SM) {
    if (c->world == 1) return UFP8_OK;
    const size_t off = (epoch & 1) * c->buffer_bytes;
    AgPushArgs a{};
    a.src = reinterpret_cast<const uint4*>(c->base + off + kFlagBytes + c->rank * c->slot_bytes);
    for (int i = 1; i < c->world; ++i) {
      const int p = (c->rank - i + c->world) % c->world;
      a.dst[i - 1] = reinterpret_cast<uint4*>(c->peer_base[p] + off + kFlagBytes + c->rank * c->slot_bytes);
      a.flag[i - 1] = reinterpret_cast<uint32_t*>(c->peer_base[p] + off) + c->rank;
    }
    a.counter = reinterpret_cast<unsigned int*>(c->base + off + kAgCounterOffset);
    a.n16 = bytes / 16;
    a.ndst = c->world - 1;
    a.epoch = static_cast<uint32_t>(epoch);
    static thread_local int carveout_device = -1;
    if (carveout_device != c->device) {
      // Without this hint the driver may run the push CTAs with a small shared-memory carveout,
      // and no GEMM CTA (~225 KiB) can join an SM until they leave.
      cudaError_t e = cudaFuncSetAttribute(tp_ag_push_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                           cudaSharedmemCarveoutMaxShared);
      if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(push carveout)");
      carveout_device = c->device;
    }
    tp_ag_push_kernel<<<kAgCtas, kAgThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? UFP8_OK : cuda_error(e, "all-gather push launch");
  }
  using WriteValueFn = CUresult (*)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);
  static WriteValueFn write_value = [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuStreamWriteValue32", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<WriteValueFn>(nullptr);
    return reinterpret_cast<WriteValueFn>(fn);
  }();
  if (!write_value) return set_error(UFP8_ERR_CUDA, "cuStreamWriteValue32 is unavailable from the driver");
  const size_t off = (epoch & 1) * c->buffer_bytes;
  const char* src = c->base + off + kFlagBytes + c->rank * c->slot_bytes;
  cudaStream_t s0 = reinterpret_cast<cudaStream_t>(stream);
  const int nl = c->world > 1 ? std::min(c->lanes, c->world - 1) : 1;
  if (int rc = lanes_fork(c, s0, nl)) return rc;
  for (int i = 1; i < c->world; ++i) {
    const int p = (c->rank - i + c->world) % c->world;
    cudaStream_t s = lane_of(c, s0, nl, i - 1);
    char* dst = c->peer_base[p] + off + kFlagBytes + c->rank * c->slot_bytes;
    if (bytes > 0) {
      cudaError_t e = cudaMemcpyAsync(dst, src, static_cast<size_t>(bytes), cudaMemcpyDeviceToDevice, s);
      if (e != cudaSuccess) return cuda_error(e, "ufp8_tp_ag_push: peer copy");
    }
    const CUdeviceptr flag = reinterpret_cast<CUdeviceptr>(c->peer_base[p] + off) + c->rank * sizeof(uint32_t);
    CUresult r = write_value(reinterpret_cast<CUstream>(s), flag, static_cast<cuuint32_t>(epoch),
                             CU_STREAM_WRITE_VALUE_DEFAULT);
    if (r != CUDA_SUCCESS) return set_error(UFP8_ERR_CUDA, "ufp8_tp_ag_push: cuStreamWriteValue32 (CUresult %d)", r);
  }
  return lanes_join(c, s0, nl);
}

int ufp8_tp_set_copy_lanes(ufp8_tp_ctx* ctx, int lanes) {
  TPContext* c = reinterpret_cast<TPContext*>(ctx);
  if (!c || lanes < 1 || lanes > kMaxRanks) return set_error(UFP8_ERR_INVALID, "ufp8_tp_set_copy_lanes: bad argument");
  c->lanes = lanes;
  return UFP8_OK;
}

int ufp8_tp_rs_push_copy(ufp8_tp_ctx* ctx, uint64_t epoch, const void* src, int64_t ld_src, int64_t rows,
                         int64_t cols, ufp8_stream_t stream) {
  TPContext* c = reinterpret_cast<TPContext*>(ctx);
  if (!c || (!src && rows > 0)) return set_error(UFP8_ERR_INVALID, "ufp8_tp_rs_push_copy: null pointer");
  if (epoch == 0 || epoch > c->epoch) return set_error(UFP8_ERR_INVALID, "ufp8_tp_rs_push_copy: epoch not begun");
  if (rows < 0 || cols <= 0 || ld_src < cols)
    return set_error(UFP8_ERR_INVALID, "ufp8_tp_rs_push_copy: bad extents");
  if (static_cast<size_t>(rows * cols * 2) > c->slot_bytes)
    return set_error(UFP8_ERR_INVALID, "ufp8_tp_rs_push_copy: %lld x %lld rows exceed the staging slot",
                     static_cast<long long>(rows), static_cast<long long>(cols));
  if (reinterpret_cast<uintptr_t>(src) & 1u) return set_error(UFP8_ERR_ALIGN, "ufp8_tp_rs_push_copy: src not 2-byte aligned");
  for (int p = 0; p < c->world; ++p)
    if (!c->peer_base[p]) return set_error(UFP8_ERR_INVALID, "ufp8_tp_rs_push_copy: rank %d is not connected", p);
  if (rows == 0) return UFP8_OK;
  const size_t off = (epoch & 1) * c->buffer_bytes;
  cudaStream_t s0 = reinterpret_cast<cudaStream_t>(stream);
  const int nl = std::min(c->lanes, c->world);
  if (int rc = lanes_fork(c, s0, nl)) return rc;
  const size_t row_bytes = static_cast<size_t>(cols) * 2, pitch = static_cast<size_t>(ld_src) * 2;
  for (int i = 0; i < c->world; ++i) {  // own block first, then rank+1, rank+2, ... (mod k)
    const int p = (c->rank + i) % c->world;
    cudaStream_t s = lane_of(c, s0, nl, i);
    char* dst = c->peer_base[p] + off + kFlagBytes + c->rank * c->slot_bytes;
    const char* blk = static_cast<const char*>(src) + static_cast<size_t>(p) * rows * pitch;
    const cudaError_t e =
        pitch == row_bytes
            ? cudaMemcpyAsync(dst, blk, row_bytes * rows, cudaMemcpyDeviceToDevice, s)
            : cudaMemcpy2DAsync(dst, row_bytes, blk, pitch, row_bytes, static_cast<size_t>(rows),
                                cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) return cuda_error(e, "ufp8_tp_rs_push_copy: peer copy");
  }
  return lanes_join(c, s0, nl);
}

int ufp8_tp_slot_bytes(const ufp8_tp_ctx* ctx, int64_t* out) {
  const TPContext* c = reinterpret_cast<const TPContext*>(ctx);
  if (!c || !out) return set_error(UFP8_ERR_INVALID, "ufp8_tp_slot_bytes: null pointer");
  *out = static_cast<int64_t>(c->slot_bytes);
  return UFP8_OK;
}

}  // extern "C"
