// Host-side declarations shared by the translation units of libufp8.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "../../include/ufp8.h"

namespace ufp8 {

// Records a formatted message as the calling thread's last error and returns `code`.
int set_error(int code, const char* fmt, ...);
// Wraps a failing CUDA runtime status into UFP8_ERR_CUDA with the call site named.
int cuda_error(cudaError_t e, const char* what);

struct DeviceInfo {
  int device = -1;
  int sm_count = 0;
  int cc_major = 0;
  int cc_minor = 0;
  int* status_word = nullptr;  // address of the library's device status word on this device
};
// Per-device facts, looked up once per device (device must be current).
int device_info(DeviceInfo** out);

// quant.cu
int launch_amax(const void* x, int64_t n, float* amax, cudaStream_t s, const DeviceInfo& dev);
int launch_quantize(const void* x, int64_t n, int fmt, const float* amax, void* q, float* inv_scale,
                    cudaStream_t s, const DeviceInfo& dev);

// gemm.cu
int launch_gemm(const ufp8_gemm_desc& d, cudaStream_t s, const DeviceInfo& dev, int ctas_override, int variant,
                int group_m);

}  // namespace ufp8
