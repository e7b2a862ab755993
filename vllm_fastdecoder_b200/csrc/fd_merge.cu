// Log-sum-exp merge of attention partials (o, lse).
//
// Rule (vLLM merge_attn_states, restated by the reference in
// fastdecode/cpu_ops.py:93-113):  an lse of +inf is an empty partial
// (FlashAttention's convention) and is treated as -inf;  m = max lse;  a row
// empty on every side gets weights 0 and total 1, i.e. zeros;  otherwise
// out = sum_p o_p * exp(lse_p - m) / sum_p exp(lse_p - m),
// lse_out = m + log(sum_p exp(lse_p - m)).
//
// Fast path (16-byte aligned rows, the usual case): one thread per 16-byte
// chunk of the inputs (8 dims of fp16 / bf16, 4 of fp32) over a grid-stride
// loop of a few CTAs per SM; each thread reads its row-head's lse values
// (L1 hits for the 16 or 32 threads sharing them), computes the weights and
// merges its chunk, so a launch is one memory round trip for the lse values
// and one for the partials instead of one small CTA per (head, row).  The
// arithmetic per element is the same as the general kernels' (one CTA per
// (head, row), threads striding over the head dimension), which remain for
// unaligned shapes.

#include <math.h>

#include <algorithm>

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
  for (int d = threadIdx.x; orow >= 0 && d < p.D; d += blockDim.x) {
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

// 16 bytes of input -> `kE` floats
template <typename T>
struct Chunk {
  static constexpr int kE = 16 / (int)sizeof(T);
  __device__ static __forceinline__ void load(const void* base, int64_t elem, float (&f)[kE]) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(static_cast<const T*>(base) + elem));
    Dt<T>::widen(v, f);
  }
};

// Store E merged floats at element `idx` of an out_dtype array: one 16-byte
// (or 8-byte) store when `packed` (the caller checked the alignment), else
// element by element.
template <int E>
__device__ __forceinline__ void store_chunk(void* base, int64_t idx, int dtype, const float (&x)[E], bool packed) {
  if (packed) {
    if (dtype == FD_DTYPE_F32) {
#pragma unroll
      for (int e = 0; e < E; e += 4)
        *reinterpret_cast<float4*>(static_cast<float*>(base) + idx + e) = make_float4(x[e], x[e + 1], x[e + 2], x[e + 3]);
      return;
    }
    uint32_t w[E / 2];
#pragma unroll
    for (int e = 0; e < E; e += 2) {
      if (dtype == FD_DTYPE_F16) {
        const __half2 h = __floats2half2_rn(x[e], x[e + 1]);
        w[e / 2] = *reinterpret_cast<const uint32_t*>(&h);
      } else {
        const __nv_bfloat162 h = __floats2bfloat162_rn(x[e], x[e + 1]);
        w[e / 2] = *reinterpret_cast<const uint32_t*>(&h);
      }
    }
    if constexpr (E == 8) {
      *reinterpret_cast<uint4*>(static_cast<__half*>(base) + idx) = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
      *reinterpret_cast<uint2*>(static_cast<__half*>(base) + idx) = make_uint2(w[0], w[1]);
    }
    return;
  }
#pragma unroll
  for (int e = 0; e < E; ++e) store_out(base, idx + e, dtype, x[e]);
}

template <typename TIn>
__global__ void __launch_bounds__(256) fd_merge2v_kernel(const __grid_constant__ Merge2Params p, bool packed) {
  constexpr int E = Chunk<TIn>::kE;
  const int cpr = p.D / E;  // chunks per (row, head)
  const int64_t total = (int64_t)p.n * p.H * cpr;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t rh = idx / cpr;
    const int c = (int)(idx - rh * cpr);
    const int i = (int)(rh / p.H), h = (int)(rh - (int64_t)i * p.H);
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
    float xa[E], xb[E];
    const int64_t ib = rh * p.D + (int64_t)c * E;
    Chunk<TIn>::load(p.oa, ib, xa);
    Chunk<TIn>::load(p.ob, ib, xb);
    const int64_t orow = p.out_rows ? p.out_rows[i] : i;
    const int64_t ob = orow * p.out_sn + (int64_t)h * p.D + (int64_t)c * E;
    float x[E];
#pragma unroll
    for (int e = 0; e < E; ++e) x[e] = xa[e] * wa + xb[e] * wb;
    if (orow >= 0) store_chunk<E>(p.out, ob, p.out_dtype, x, packed);
    if (c == 0 && p.out_lse != nullptr) p.out_lse[(int64_t)h * p.n + i] = both_empty ? -INFINITY : m + logf(tot);
  }
}

// P-way merge of fp32 partials, 4 dims per thread; at most kMaxPV parts
constexpr int kMaxPV = 16;

__global__ void __launch_bounds__(256) fd_mergePv_kernel(const __grid_constant__ MergePParams p, bool packed) {
  const int cpr = p.D / 4;
  const int64_t total = (int64_t)p.n * p.H * cpr;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t rh = idx / cpr;
    const int c = (int)(idx - rh * cpr);
    const int i = (int)(rh / p.H), h = (int)(rh - (int64_t)i * p.H);
    float l[kMaxPV];
    float m = -INFINITY;
#pragma unroll
    for (int q = 0; q < kMaxPV; ++q) {
      l[q] = q < p.P ? empty_to_neg_inf(__ldg(p.lse + q * p.part_stride + (int64_t)h * p.n + i)) : -INFINITY;
      m = fmaxf(m, l[q]);
    }
    const bool all_empty = (m == -INFINITY);
    if (all_empty) m = 0.f;
    float tot = 0.f;
#pragma unroll
    for (int q = 0; q < kMaxPV; ++q) {
      l[q] = q < p.P ? expf(l[q] - m) : 0.f;  // the weight of part q
      if (q < p.P) tot += l[q];
    }
    if (all_empty) tot = 1.f;
    const float inv = 1.f / tot;
    const int64_t base = rh * p.D + (int64_t)c * 4;
    float x[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int q = 0; q < kMaxPV; ++q) {
      if (q < p.P) {
        const float4 o = __ldg(reinterpret_cast<const float4*>(p.o + q * p.part_stride + base));
        const float wq = l[q] * inv;
        x[0] = fmaf(wq, o.x, x[0]);
        x[1] = fmaf(wq, o.y, x[1]);
        x[2] = fmaf(wq, o.z, x[2]);
        x[3] = fmaf(wq, o.w, x[3]);
      }
    }
    store_chunk<4>(p.out, base, p.out_dtype, x, packed);
    if (c == 0 && p.out_lse != nullptr) p.out_lse[(int64_t)h * p.n + i] = all_empty ? -INFINITY : m + logf(tot);
  }
}

// CTAs of the grid-stride kernels: enough for every chunk, at most 8 per SM
inline unsigned merge_grid(int64_t chunks) {
  int dev = 0, sms = 0;
  if (fdh::device_sms(&dev, &sms) != FD_OK || sms <= 0) sms = 148;
  const int64_t want = (chunks + 255) / 256;
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)sms * 8));
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
  const int ies = fdh::elem_size(in_dtype);
  if (((int64_t)head_size * ies) % 16 == 0 && fdh::aligned16(o_a) && fdh::aligned16(o_b)) {
    const int64_t chunks = (int64_t)n * num_heads * head_size * ies / 16;
    const unsigned grid = fdk::merge_grid(chunks);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // packed stores: every chunk's destination 16-byte (8-byte for fp32
    // inputs into a 16-bit output) aligned
    const int oes = fdh::elem_size(out_dtype);
    const int chunk_out = 16 / ies * oes;
    const bool packed = (reinterpret_cast<uintptr_t>(out) % chunk_out == 0) && (out_stride_n * oes) % chunk_out == 0 &&
                        ((int64_t)head_size * oes) % chunk_out == 0;
    if (in_dtype == FD_DTYPE_F16)
      fdk::fd_merge2v_kernel<__half><<<grid, 256, 0, s>>>(p, packed);
    else if (in_dtype == FD_DTYPE_BF16)
      fdk::fd_merge2v_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(p, packed);
    else
      fdk::fd_merge2v_kernel<float><<<grid, 256, 0, s>>>(p, packed);
    return fdh::cuda_status(cudaGetLastError(), "fd_merge2v_kernel launch");
  }
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
  if (num_parts <= fdk::kMaxPV && head_size % 4 == 0 && part_stride % 4 == 0 && fdh::aligned16(o_parts)) {
    const unsigned grid = fdk::merge_grid((int64_t)n * num_heads * head_size / 4);
    const int oes = fdh::elem_size(out_dtype);
    const bool packed = reinterpret_cast<uintptr_t>(out) % (4 * oes) == 0;  // rows of D = 4k elements
    fdk::fd_mergePv_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(p, packed);
    return fdh::cuda_status(cudaGetLastError(), "fd_mergePv_kernel launch");
  }
  const int threads = head_size <= 64 ? 64 : (head_size <= 128 ? 128 : 256);
  fdk::fd_mergeP_kernel<<<dim3(num_heads, n), threads, num_parts * sizeof(float),
                          static_cast<cudaStream_t>(stream)>>>(p);
  return fdh::cuda_status(cudaGetLastError(), "fd_mergeP_kernel launch");
}
