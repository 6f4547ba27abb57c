// Host-side helpers shared by the C-ABI translation units: error reporting,
// per-device attribute caching and TMA tensor-map encoding.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>

#include "../../include/focal_b200.h"

namespace focal {

// Record a message for focal_last_error() and return `code`.
int set_error(int code, const char* fmt, ...);
void clear_error();

// Returns FOCAL_OK or FOCAL_ERR_CUDA (with message) for a CUDA runtime result.
int check_cuda(cudaError_t e, const char* what);

struct DeviceInfo {
  int device = -1;
  int sm_count = 0;
  int max_smem_optin = 0;  // bytes per block with opt-in
  int cc_major = 0, cc_minor = 0;
  int* status = nullptr;       // status word, device view (mapped pinned host memory)
  int* status_host = nullptr;  // the same word, host view
};

// Zero the no-allocation GEMV scratch on the current device (w4a16_gemv.cu).
int noalloc_clear();

// Attributes of the current device (cached per device ordinal).
int current_device_info(DeviceInfo* out);

// Ensure `kernel` may use `smem_bytes` of dynamic shared memory on the
// current device (cudaFuncSetAttribute issued at most once per growth).
int ensure_dynamic_smem(const void* kernel, int slot, int smem_bytes);

// 2-D / 3-D tiled tensor maps through the driver entry point (no libcuda link).
int encode_tensor_map(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                      const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                      CUtensorMapSwizzle swizzle);

// Per-device status word written by kernels whose bounded waits gave up.

inline bool aligned(const void* p, uintptr_t a) {
  return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0;
}

}  // namespace focal
