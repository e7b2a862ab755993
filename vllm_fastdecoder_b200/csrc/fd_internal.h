// Host-side helpers shared by the C-ABI translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>

#include "fastdecode_b200.h"

namespace fdh {

// Record a message for fd_last_error_message() and return `status`.
int fail(int status, const char* fmt, ...);

inline int elem_size(int32_t dtype) {
  switch (dtype) {
    case FD_DTYPE_F16:
    case FD_DTYPE_BF16:
      return 2;
    case FD_DTYPE_F32:
      return 4;
    default:
      return 0;
  }
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return FD_OK;
  return fail(FD_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// Raise the dynamic shared-memory limit of `kernel` once per device.
int ensure_smem(const void* kernel, int bytes, unsigned long long* done_mask);

// The current device and its SM count (queried once per device).
int device_sms(int* dev, int* sms);

// Launch `kernel(param)` (a kernel taking one parameter struct by value),
// as a programmatic dependent of the kernel ahead on the stream when `pdl`
// (the kernel then must pass griddepcontrol.wait before touching what that
// kernel writes), else as an ordinary launch.
template <typename P>
int launch_maybe_pdl(const void* kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl, const P& param,
                     const char* what) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = pdl ? attr : nullptr;
  cfg.numAttrs = pdl ? 1 : 0;
  void* args[1] = {const_cast<P*>(&param)};
  return cuda_status(cudaLaunchKernelExC(&cfg, kernel, args), what);
}

}  // namespace fdh
