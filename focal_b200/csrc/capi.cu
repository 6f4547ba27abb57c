// Host plumbing of the C ABI plus the two small helper kernels on the W4A16
// path: int4 packing (replaces focal_w4a16/__init__.py:38-54) and fp32
// dequantisation (bit-identical to dequant_ref, focal_w4a16/__init__.py:57-91).
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "host_common.h"

namespace focal {

// One status word per device; kernels whose bounded waits give up write it.

namespace {
thread_local std::string g_last_error;

constexpr int kMaxDevices = 64;
DeviceInfo g_info[kMaxDevices];
std::once_flag g_info_once[kMaxDevices];
int g_info_err[kMaxDevices];

constexpr int kMaxKernelSlots = 64;
std::mutex g_smem_mutex;
int g_smem_set[kMaxDevices][kMaxKernelSlots];

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
}  // namespace

int set_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

void clear_error() { g_last_error.clear(); }

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return FOCAL_OK;
  return set_error(FOCAL_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

int current_device_info(DeviceInfo* out) {
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (rc) return rc;
  if (dev < 0 || dev >= kMaxDevices) return set_error(FOCAL_ERR_CUDA, "device ordinal %d", dev);
  std::call_once(g_info_once[dev], [dev]() {
    DeviceInfo d;
    d.device = dev;
    cudaError_t e = cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess)
      e = cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (e == cudaSuccess && d.cc_major == 10) {
      // the status word: one int of mapped pinned host memory per device, so
      // the host reads it without synchronizing with the device
      void* hp = nullptr;
      e = cudaHostAlloc(&hp, sizeof(int), cudaHostAllocMapped | cudaHostAllocPortable);
      if (e == cudaSuccess) {
        *static_cast<volatile int*>(hp) = 0;
        void* dp = nullptr;
        e = cudaHostGetDevicePointer(&dp, hp, 0);
        d.status = static_cast<int*>(dp);
        d.status_host = static_cast<int*>(hp);
      }
    }
    g_info_err[dev] = static_cast<int>(e);
    g_info[dev] = d;
  });
  if (g_info_err[dev] != 0)
    return check_cuda(static_cast<cudaError_t>(g_info_err[dev]), "cudaDeviceGetAttribute");
  if (g_info[dev].cc_major != 10)
    return set_error(FOCAL_ERR_CUDA,
                     "focal_b200 kernels are built for sm_100a; device %d is sm_%d%d", dev,
                     g_info[dev].cc_major, g_info[dev].cc_minor);
  *out = g_info[dev];
  return FOCAL_OK;
}

int ensure_dynamic_smem(const void* kernel, int slot, int smem_bytes) {
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (rc) return rc;
  if (slot < 0 || slot >= kMaxKernelSlots || dev < 0 || dev >= kMaxDevices)
    return set_error(FOCAL_ERR_INVALID_VALUE, "kernel slot %d / device %d out of range", slot, dev);
  std::lock_guard<std::mutex> lock(g_smem_mutex);
  if (g_smem_set[dev][slot] >= smem_bytes) return FOCAL_OK;
  rc = check_cuda(
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes),
      "cudaFuncSetAttribute(MaxDynamicSharedMemorySize)");
  if (rc) return rc;
  g_smem_set[dev][slot] = smem_bytes;
  return FOCAL_OK;
}

int encode_tensor_map(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                      const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                      CUtensorMapSwizzle swizzle) {
  std::call_once(g_encode_once, []() {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode) return set_error(FOCAL_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint32_t elem_strides[5] = {1, 1, 1, 1, 1};
  CUresult r = g_encode(map, dtype, rank, const_cast<void*>(base),
                        reinterpret_cast<const cuuint64_t*>(dims),
                        reinterpret_cast<const cuuint64_t*>(strides_bytes),
                        reinterpret_cast<const cuuint32_t*>(box), elem_strides,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(FOCAL_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return FOCAL_OK;
}


// ------------------------------------------------------------------ kernels
// One thread per packed word: eight bytes in, one int32 out.
__global__ void pack_int4_kernel(const uint8_t* __restrict__ q, int32_t* __restrict__ wq,
                                 long long words) {
  const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (i >= words) return;
  const uint2 b = reinterpret_cast<const uint2*>(q)[i];
  // byte j of b holds value 8i+j; keep its low nibble at bits 4j..4j+3
  uint32_t lo = b.x & 0x0F0F0F0Fu, hi = b.y & 0x0F0F0F0Fu;
  // spread: bytes (v0,v1,v2,v3) -> nibbles 0..3
  lo = (lo | (lo >> 4)) & 0x00FF00FFu;
  lo = (lo | (lo >> 8)) & 0x0000FFFFu;
  hi = (hi | (hi >> 4)) & 0x00FF00FFu;
  hi = (hi | (hi >> 8)) & 0x0000FFFFu;
  wq[i] = static_cast<int32_t>(lo | (hi << 16));
}

// One thread per packed word: 8 fp32 outputs.  The nibbles go through the
// same bf16 "128 + q" conversion the GEMV kernels feed to the tensor cores,
// so this kernel doubles as the bit-exact check of that unpacking.
__global__ void dequant_kernel(const uint32_t* __restrict__ wq, const __half* __restrict__ scales,
                               const __half* __restrict__ zeros, float* __restrict__ w, int K,
                               long long words) {
  const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (i >= words) return;
  const int kw = K >> 3;
  const long long n = i / kw;
  const int k0 = static_cast<int>(i - n * kw) * 8;
  const long long gi = n * (K >> 7) + (k0 >> 7);
  const float s = __half2float(scales[gi]);
  const float z = __half2float(zeros[gi]);
  const uint32_t word = wq[i];
  float out[8];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t pr = nib_pair_bf16(word, j);   // (128+q_j, 128+q_{j+4})
    const float qa = bf16_lo(pr) - 128.0f;        // exact small integers
    const float qb = bf16_hi(pr) - 128.0f;
    out[j] = (qa - z) * s;
    out[j + 4] = (qb - z) * s;
  }
  float4* dst = reinterpret_cast<float4*>(w + n * K + k0);
  dst[0] = make_float4(out[0], out[1], out[2], out[3]);
  dst[1] = make_float4(out[4], out[5], out[6], out[7]);
}

}  // namespace focal

using namespace focal;

extern "C" {

const char* focal_last_error(void) { return g_last_error.c_str(); }

int focal_abi_version(void) { return 1; }

int focal_pack_int4(const uint8_t* q, int32_t* wq, int N, int K, cudaStream_t stream) {
  clear_error();
  if (N < 0 || K < 0) return set_error(FOCAL_ERR_INVALID_VALUE, "N and K must be non-negative");
  if (K % 8 != 0) return set_error(FOCAL_ERR_UNSUPPORTED, "K must be divisible by 8");
  const long long words = (long long)N * (K / 8);
  if (words == 0) return FOCAL_OK;
  if (!q || !wq) return set_error(FOCAL_ERR_INVALID_VALUE, "null pointer");
  if (!aligned(q, 8) || !aligned(wq, 4))
    return set_error(FOCAL_ERR_INVALID_VALUE, "q must be 8-byte and wq 4-byte aligned");
  const int threads = 256;
  const long long blocks = (words + threads - 1) / threads;
  pack_int4_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(q, wq, words);
  return check_cuda(cudaGetLastError(), "pack_int4_kernel launch");
}

int focal_w4a16_dequant(const int32_t* wq, const void* scales, const void* zeros, float* w,
                        int K, int N, cudaStream_t stream) {
  clear_error();
  if (N < 0 || K <= 0) return set_error(FOCAL_ERR_INVALID_VALUE, "N and K must be positive");
  if (K % 128 != 0) return set_error(FOCAL_ERR_UNSUPPORTED, "K must be divisible by 128");
  const long long words = (long long)N * (K / 8);
  if (words == 0) return FOCAL_OK;
  if (!wq || !scales || !zeros || !w) return set_error(FOCAL_ERR_INVALID_VALUE, "null pointer");
  if (!aligned(wq, 4) || !aligned(scales, 2) || !aligned(zeros, 2) || !aligned(w, 16))
    return set_error(FOCAL_ERR_INVALID_VALUE, "misaligned pointer");
  const int threads = 256;
  const long long blocks = (words + threads - 1) / threads;
  dequant_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
      reinterpret_cast<const uint32_t*>(wq), static_cast<const __half*>(scales),
      static_cast<const __half*>(zeros), w, K, words);
  return check_cuda(cudaGetLastError(), "dequant_kernel launch");
}

int focal_device_status(int* status_out) {
  clear_error();
  if (!status_out) return set_error(FOCAL_ERR_INVALID_VALUE, "null pointer");
  DeviceInfo d;
  int rc = current_device_info(&d);
  if (rc) return rc;
  rc = check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  if (rc) return rc;
  *status_out = *static_cast<volatile int*>(d.status_host);
  return FOCAL_OK;
}

int focal_device_status_peek(int* status_out) {
  clear_error();
  if (!status_out) return set_error(FOCAL_ERR_INVALID_VALUE, "null pointer");
  DeviceInfo d;
  const int rc = current_device_info(&d);
  if (rc) return rc;
  *status_out = *static_cast<volatile int*>(d.status_host);
  return FOCAL_OK;
}

int focal_reset_device_status(void) {
  clear_error();
  DeviceInfo d;
  const int rc = current_device_info(&d);
  if (rc) return rc;
  *static_cast<volatile int*>(d.status_host) = 0;
  return noalloc_clear();
}

}  // extern "C"
