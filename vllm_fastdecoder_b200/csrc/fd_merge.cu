// Log-sum-exp merge of attention partials (o, lse).
//
// Rule (vLLM merge_attn_states, restated by the reference in
// fastdecode/cpu_ops.py:93-113):  an lse of +inf is an empty partial
// (FlashAttention's convention) and is treated as -inf;  m = max lse;  a row
// empty on every side gets weights 0 and total 1, i.e. zeros;  otherwise
// out = sum_p o_p * exp(lse_p - m) / sum_p exp(lse_p - m),
// lse_out = m + log(sum_p exp(lse_p - m)).
// One CTA per (head, row); threads stride over the head dimension.

#include <math.h>

#include "fd_common.cuh"
#include "fd_internal.h"

namespace fdk {

__device__ __forceinline__ float empty_to_neg_inf(float x) { return x == INFINITY ? -INFINITY : x; }

struct Merge2Params {
  void* out;
  int out_dtype;
  int64_t out_sn;
  const int64_t* out_rows;
  float* out_lse;
  const void* oa;
  const void* ob;
  const float* la;
  const float* lb;
  int in_dtype;
  int n, H, D;
};

__global__ void fd_merge2_kernel(const __grid_constant__ Merge2Params p) {
  const int h = blockIdx.x;
  const int i = blockIdx.y;
  const float a = empty_to_neg_inf(p.la[(int64_t)h * p.n + i]);
  const float b = empty_to_neg_inf(p.lb[(int64_t)h * p.n + i]);
  float m = fmaxf(a, b);
  const bool both_empty = (m == -INFINITY);
  if (both_empty) m = 0.f;
  float wa = expf(a - m);
  float wb = expf(b - m);
  float tot = wa + wb;
  if (both_empty) tot = 1.f;
  wa = wa / tot;
  wb = wb / tot;
  const int64_t orow = p.out_rows ? p.out_rows[i] : i;
  const int64_t ibase = ((int64_t)i * p.H + h) * p.D;
  const int64_t obase = orow * p.out_sn + (int64_t)h * p.D;
  for (int d = threadIdx.x; d < p.D; d += blockDim.x) {
    const float x = load_in(p.oa, ibase + d, p.in_dtype) * wa + load_in(p.ob, ibase + d, p.in_dtype) * wb;
    store_out(p.out, obase + d, p.out_dtype, x);
  }
  if (threadIdx.x == 0 && p.out_lse != nullptr)
    p.out_lse[(int64_t)h * p.n + i] = both_empty ? -INFINITY : m + logf(tot);
}

struct MergePParams {
  const float* o;
  const float* lse;
  int64_t part_stride;
  int P, n, H, D;
  void* out;
  int out_dtype;
  float* out_lse;
};

__global__ void fd_mergeP_kernel(const __grid_constant__ MergePParams p) {
  extern __shared__ float w[];
  const int h = blockIdx.x;
  const int i = blockIdx.y;
  float m = -INFINITY;
  for (int q = 0; q < p.P; ++q) m = fmaxf(m, empty_to_neg_inf(p.lse[q * p.part_stride + (int64_t)h * p.n + i]));
  const bool all_empty = (m == -INFINITY);
  if (all_empty) m = 0.f;
  for (int q = threadIdx.x; q < p.P; q += blockDim.x)
    w[q] = expf(empty_to_neg_inf(p.lse[q * p.part_stride + (int64_t)h * p.n + i]) - m);
  __syncthreads();
  float tot = 0.f;
  for (int q = 0; q < p.P; ++q) tot += w[q];
  if (all_empty) tot = 1.f;
  const float inv = 1.f / tot;
  const int64_t base = ((int64_t)i * p.H + h) * p.D;
  for (int d = threadIdx.x; d < p.D; d += blockDim.x) {
    float x = 0.f;
    for (int q = 0; q < p.P; ++q) x = fmaf(w[q] * inv, p.o[q * p.part_stride + base + d], x);
    store_out(p.out, base + d, p.out_dtype, x);
  }
  if (threadIdx.x == 0 && p.out_lse != nullptr)
    p.out_lse[(int64_t)h * p.n + i] = all_empty ? -INFINITY : m + logf(tot);
}

}  // namespace fdk

extern "C" int fd_merge_attn_states(void* out, int32_t out_dtype, int64_t out_stride_n,
                                    const int64_t* out_rows, float* out_lse, const void* o_a,
                                    const float* lse_a, const void* o_b, const float* lse_b,
                                    int32_t in_dtype, int32_t n, int32_t num_heads,
                                    int32_t head_size, void* stream) {
  if (n < 0 || num_heads <= 0 || head_size <= 0)
    return fdh::fail(FD_ERR_INVALID, "fd_merge_attn_states: bad shape n=%d H=%d D=%d", n, num_heads,
                     head_size);
  if (fdh::elem_size(out_dtype) == 0 || fdh::elem_size(in_dtype) == 0)
    return fdh::fail(FD_ERR_UNSUPPORTED, "fd_merge_attn_states: unsupported dtype");
  if (n == 0) return FD_OK;
  if (out == nullptr || o_a == nullptr || o_b == nullptr || lse_a == nullptr || lse_b == nullptr)
    return fdh::fail(FD_ERR_INVALID, "fd_merge_attn_states: null pointer");
  if (n > 65535) return fdh::fail(FD_ERR_UNSUPPORTED, "fd_merge_attn_states: at most 65535 rows");
  fdk::Merge2Params p{out, out_dtype, out_stride_n, out_rows, out_lse, o_a, o_b, lse_a, lse_b,
                      in_dtype, n, num_heads, head_size};
  const int threads = head_size <= 64 ? 64 : (head_size <= 128 ? 128 : 256);
  fdk::fd_merge2_kernel<<<dim3(num_heads, n), threads, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return fdh::cuda_status(cudaGetLastError(), "fd_merge2_kernel launch");
}

extern "C" int fd_merge_partials(const float* o_parts, const float* lse_parts, int64_t part_stride,
                                 int32_t num_parts, int32_t n, int32_t num_heads, int32_t head_size,
                                 void* out, int32_t out_dtype, float* out_lse, void* stream) {
  if (n < 0 || num_heads <= 0 || head_size <= 0 || num_parts <= 0)
    return fdh::fail(FD_ERR_INVALID, "fd_merge_partials: bad shape");
  if (fdh::elem_size(out_dtype) == 0) return fdh::fail(FD_ERR_UNSUPPORTED, "fd_merge_partials: dtype");
  if (n == 0) return FD_OK;
  if (o_parts == nullptr || lse_parts == nullptr || out == nullptr)
    return fdh::fail(FD_ERR_INVALID, "fd_merge_partials: null pointer");
  if (n > 65535 || num_parts > 8192) return fdh::fail(FD_ERR_UNSUPPORTED, "fd_merge_partials: too large");
  fdk::MergePParams p{o_parts, lse_parts, part_stride, num_parts, n, num_heads, head_size,
                      out, out_dtype, out_lse};
  const int threads = head_size <= 64 ? 64 : (head_size <= 128 ? 128 : 256);
  fdk::fd_mergeP_kernel<<<dim3(num_heads, n), threads, num_parts * sizeof(float),
                          static_cast<cudaStream_t>(stream)>>>(p);
  return fdh::cuda_status(cudaGetLastError(), "fd_mergeP_kernel launch");
}
