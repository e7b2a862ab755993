// C-ABI utilities: error messages, device error word, pinned/mapped host
// memory helpers.

#include <stdio.h>
#include <string.h>

#include "fd_internal.h"

namespace {
thread_local char g_msg[512] = "";
}

namespace fdh {

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return status;
}

int ensure_smem(const void* kernel, int bytes, unsigned long long* done_mask) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
  const unsigned long long bit = dev < 64 ? (1ull << dev) : 0ull;
  if (bit != 0ull && (__atomic_load_n(done_mask, __ATOMIC_ACQUIRE) & bit)) return FD_OK;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(MaxDynamicSharedMemorySize)");
  if (bit != 0ull) __atomic_fetch_or(done_mask, bit, __ATOMIC_RELEASE);
  return FD_OK;
}

int device_sms(int* dev, int* sms) {
  static int cached[64] = {0};
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
  if (*dev >= 0 && *dev < 64) {
    const int c = __atomic_load_n(&cached[*dev], __ATOMIC_RELAXED);
    if (c > 0) {
      *sms = c;
      return FD_OK;
    }
  }
  e = cudaDeviceGetAttribute(sms, cudaDevAttrMultiProcessorCount, *dev);
  if (e != cudaSuccess) return cuda_status(e, "cudaDeviceGetAttribute(MultiProcessorCount)");
  if (*dev >= 0 && *dev < 64) __atomic_store_n(&cached[*dev], *sms, __ATOMIC_RELAXED);
  return FD_OK;
}

}  // namespace fdh

extern "C" const char* fd_last_error_message(void) { return g_msg; }

extern "C" const char* fd_device_error_string(int32_t code) {
  switch (code) {
    case FD_DEVERR_NONE:
      return "no error";
    case FD_DEVERR_BLOCK_ID:
      return "block id outside both KV tiers";
    case FD_DEVERR_LEN:
      return "sequence length needs more blocks than the block-table row holds";
    case FD_DEVERR_TIMEOUT:
      return "bounded wait on a pipeline barrier timed out";
    case FD_DEVERR_SLOT:
      return "KV-write slot outside both KV tiers";
    case FD_DEVERR_SPLITS:
      return "sequence length exceeds the max_len the launch was sized for";
    case FD_DEVERR_PLAN:
      return "step planner: query offsets not 0-based, decreasing or past the token capacity, or a request "
             "extending prior context by more than one token while part of its KV is in the host tier";
    default:
      return "unknown device error";
  }
}

extern "C" int fd_read_error(int32_t* error, int32_t* value, int32_t clear, void* stream) {
  if (error == nullptr || value == nullptr) return fdh::fail(FD_ERR_INVALID, "fd_read_error: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(value, error, sizeof(int32_t), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return fdh::cuda_status(e, "fd_read_error");
  if (clear && *value != 0) {
    e = cudaMemsetAsync(error, 0, sizeof(int32_t), s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return fdh::cuda_status(e, "fd_read_error clear");
  }
  return FD_OK;
}

extern "C" int fd_host_device_pointer(void* host, void** device_ptr) {
  if (host == nullptr || device_ptr == nullptr)
    return fdh::fail(FD_ERR_INVALID, "fd_host_device_pointer: null pointer");
  cudaPointerAttributes attr;
  cudaError_t e = cudaPointerGetAttributes(&attr, host);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fdh::fail(FD_ERR_INVALID, "pointer %p is not pinned host memory (%s)", host, cudaGetErrorString(e));
  }
  if (attr.type != cudaMemoryTypeHost || attr.devicePointer == nullptr)
    return fdh::fail(FD_ERR_INVALID, "pointer %p is not pinned, device-mapped host memory", host);
  void* d = nullptr;
  e = cudaHostGetDevicePointer(&d, host, 0);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fdh::fail(FD_ERR_INVALID, "cudaHostGetDevicePointer(%p): %s", host, cudaGetErrorString(e));
  }
  *device_ptr = d;
  return FD_OK;
}

extern "C" int fd_host_register(void* host, size_t bytes) {
  if (host == nullptr || bytes == 0) return fdh::fail(FD_ERR_INVALID, "fd_host_register: empty range");
  return fdh::cuda_status(cudaHostRegister(host, bytes, cudaHostRegisterMapped | cudaHostRegisterPortable),
                          "cudaHostRegister");
}

extern "C" int fd_host_unregister(void* host) {
  if (host == nullptr) return fdh::fail(FD_ERR_INVALID, "fd_host_unregister: null pointer");
  return fdh::cuda_status(cudaHostUnregister(host), "cudaHostUnregister");
}

extern "C" int fd_version(void) { return 101; }

extern "C" int fd_abi_sizes(size_t* decode_args_bytes, size_t* kv_tier_bytes) {
  if (decode_args_bytes != nullptr) *decode_args_bytes = sizeof(fd_decode_args);
  if (kv_tier_bytes != nullptr) *kv_tier_bytes = sizeof(fd_kv_tier);
  return FD_OK;
}
