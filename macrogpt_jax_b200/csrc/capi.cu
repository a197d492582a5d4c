// extern "C" entry points of libufp8 (declared in include/ufp8.h): host-side validation,
// per-thread error text, per-device facts and the device status word.
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "internal.h"

namespace ufp8 {

// Status word the kernels raise bits in (UFP8_STATUS_*); one per device.
__device__ int g_status_word;

namespace {
thread_local char g_last_error[512] = "";
std::mutex g_dev_mutex;
DeviceInfo g_devices[64];
}  // namespace

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_error(cudaError_t e, const char* what) {
  return set_error(UFP8_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

int device_info(DeviceInfo** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return set_error(UFP8_ERR_DEVICE, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_dev_mutex);
  DeviceInfo& d = g_devices[dev];
  if (d.device != dev) {
    int sms = 0, major = 0, minor = 0;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess)
      return cuda_error(e, "cudaDeviceGetAttribute");
    if (major != 10 || minor != 0)
      return set_error(UFP8_ERR_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a only", dev, major,
                       minor);
    void* status = nullptr;
    if ((e = cudaGetSymbolAddress(&status, g_status_word)) != cudaSuccess)
      return cuda_error(e, "cudaGetSymbolAddress(status word)");
    d.sm_count = sms;
    d.cc_major = major;
    d.cc_minor = minor;
    d.status_word = static_cast<int*>(status);
    d.device = dev;
  }
  *out = &d;
  return UFP8_OK;
}

namespace {
int g_gemm_ctas = 0;
int g_gemm_variant = UFP8_GEMM_AUTO;
int g_gemm_group_m = 0;

bool is_fmt(int fmt) { return fmt == UFP8_E4M3 || fmt == UFP8_E5M2; }
}  // namespace

}  // namespace ufp8

using namespace ufp8;

extern "C" {

const char* ufp8_last_error(void) { return g_last_error; }

int ufp8_abi_version(void) { return UFP8_ABI_VERSION; }

int ufp8_amax(const void* x_bf16, int64_t n, float* amax, ufp8_stream_t stream) {
  if (n < 0) return set_error(UFP8_ERR_INVALID, "ufp8_amax: n < 0");
  if (!amax || (n > 0 && !x_bf16)) return set_error(UFP8_ERR_INVALID, "ufp8_amax: null pointer");
  if (reinterpret_cast<uintptr_t>(amax) & 3u) return set_error(UFP8_ERR_ALIGN, "ufp8_amax: amax not 4-byte aligned");
  if (reinterpret_cast<uintptr_t>(x_bf16) & 1u) return set_error(UFP8_ERR_ALIGN, "ufp8_amax: x not 2-byte aligned");
  DeviceInfo* dev;
  if (int rc = device_info(&dev)) return rc;
  return launch_amax(x_bf16, n, amax, reinterpret_cast<cudaStream_t>(stream), *dev);
}

int ufp8_quantize(const void* x_bf16, int64_t n, int fmt, const float* amax, void* q, float* inv_scale,
                  ufp8_stream_t stream) {
  if (n < 0) return set_error(UFP8_ERR_INVALID, "ufp8_quantize: n < 0");
  if (!is_fmt(fmt)) return set_error(UFP8_ERR_INVALID, "ufp8_quantize: fmt %d is not UFP8_E4M3/UFP8_E5M2", fmt);
  if (!amax || !inv_scale || (n > 0 && (!x_bf16 || !q)))
    return set_error(UFP8_ERR_INVALID, "ufp8_quantize: null pointer");
  if (reinterpret_cast<uintptr_t>(x_bf16) & 1u) return set_error(UFP8_ERR_ALIGN, "ufp8_quantize: x not 2-byte aligned");
  DeviceInfo* dev;
  if (int rc = device_info(&dev)) return rc;
  return launch_quantize(x_bf16, n, fmt, amax, q, inv_scale, reinterpret_cast<cudaStream_t>(stream), *dev);
}

int ufp8_amax_quant(const void* x_bf16, int64_t n, int fmt, void* q, float* amax, float* inv_scale,
                    ufp8_stream_t stream) {
  if (!is_fmt(fmt)) return set_error(UFP8_ERR_INVALID, "ufp8_amax_quant: fmt %d is not UFP8_E4M3/UFP8_E5M2", fmt);
  if (n > 0 && !q) return set_error(UFP8_ERR_INVALID, "ufp8_amax_quant: null q");
  if (!inv_scale) return set_error(UFP8_ERR_INVALID, "ufp8_amax_quant: null inv_scale");
  int rc = ufp8_amax(x_bf16, n, amax, stream);
  if (rc) return rc;
  return ufp8_quantize(x_bf16, n, fmt, amax, q, inv_scale, stream);
}

int ufp8_cast(const void* x_bf16, int64_t n, int fmt, void* q, ufp8_stream_t stream) {
  if (n < 0) return set_error(UFP8_ERR_INVALID, "ufp8_cast: n < 0");
  if (!is_fmt(fmt)) return set_error(UFP8_ERR_INVALID, "ufp8_cast: fmt %d is not UFP8_E4M3/UFP8_E5M2", fmt);
  if (n > 0 && (!x_bf16 || !q)) return set_error(UFP8_ERR_INVALID, "ufp8_cast: null pointer");
  if (reinterpret_cast<uintptr_t>(x_bf16) & 1u) return set_error(UFP8_ERR_ALIGN, "ufp8_cast: x not 2-byte aligned");
  if (n == 0) return UFP8_OK;
  DeviceInfo* dev;
  if (int rc = device_info(&dev)) return rc;
  return launch_quantize(x_bf16, n, fmt, nullptr, q, nullptr, reinterpret_cast<cudaStream_t>(stream), *dev);
}

int ufp8_gemm(const ufp8_gemm_desc* desc, ufp8_stream_t stream) {
  if (!desc) return set_error(UFP8_ERR_INVALID, "ufp8_gemm: null descriptor");
  DeviceInfo* dev;
  if (int rc = device_info(&dev)) return rc;
  return launch_gemm(*desc, reinterpret_cast<cudaStream_t>(stream), *dev, g_gemm_ctas, g_gemm_variant, g_gemm_group_m);
}

int ufp8_device_status(int* status, int clear) {
  if (!status) return set_error(UFP8_ERR_INVALID, "ufp8_device_status: null pointer");
  DeviceInfo* dev;
  if (int rc = device_info(&dev)) return rc;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_error(e, "cudaDeviceSynchronize");
  if ((e = cudaMemcpy(status, dev->status_word, sizeof(int), cudaMemcpyDeviceToHost)) != cudaSuccess)
    return cuda_error(e, "read status word");
  if (clear && (e = cudaMemset(dev->status_word, 0, sizeof(int))) != cudaSuccess)
    return cuda_error(e, "clear status word");
  return UFP8_OK;
}

int ufp8_set_gemm_variant(int variant) {
  if (variant != UFP8_GEMM_AUTO && variant != UFP8_GEMM_SINGLE_CTA && variant != UFP8_GEMM_CTA_PAIR &&
      variant != UFP8_GEMM_CTA_PAIR_DIRECT && variant != UFP8_GEMM_CTA_PAIR_WIDE &&
      variant != UFP8_GEMM_CTA_PAIR_N512)
    return set_error(UFP8_ERR_INVALID, "ufp8_set_gemm_variant: unknown variant %d", variant);
  g_gemm_variant = variant;
  return UFP8_OK;
}

int ufp8_set_gemm_raster(int group_m) {
  if (group_m < 0 || group_m > 4096) return set_error(UFP8_ERR_INVALID, "ufp8_set_gemm_raster: group_m %d", group_m);
  g_gemm_group_m = group_m;
  return UFP8_OK;
}

int ufp8_set_gemm_ctas(int ctas) {
  if (ctas < 0) return set_error(UFP8_ERR_INVALID, "ufp8_set_gemm_ctas: ctas < 0");
  g_gemm_ctas = ctas;
  return UFP8_OK;
}

}  // extern "C"
