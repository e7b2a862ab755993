// Tier-aware KV write: one kernel puts each new K/V row into its slot in the
// HBM tier or in the mapped host tier.  Bit-exact 16-byte copies.
//
// Addressing follows the reference store_kv (fastdecode/csrc/cpu_attn.cpp
// :413-431): blk = slot / BS, off = slot % BS, destination
// blk*blk_stride + head*head_stride + off*tok_stride.  Range checking follows
// :506-510, except that it runs on the device: every CTA scans all slots
// first and, if any is outside both tiers, nothing is written and the error
// word gets FD_DEVERR_SLOT.  slot < 0 means "not this call's" and is skipped,
// like reshape_and_cache_flash.

#include "fd_common.cuh"
#include "fd_internal.h"

namespace fdk {

struct StoreParams {
  const unsigned char* key;
  const unsigned char* value;
  int64_t k_sn, k_sh, v_sn, v_sh;  // bytes
  const int64_t* slots;
  int m, KVH, nch, BS;
  unsigned char* tk[2];
  unsigned char* tv[2];
  int64_t blk_sb[2], head_sb[2], tok_sb[2];
  int64_t nblk[2];
  int64_t split;
  int32_t* err;
};

__global__ void fd_store_kv_kernel(const __grid_constant__ StoreParams p) {
  __shared__ int bad;
  if (threadIdx.x == 0) bad = 0;
  __syncthreads();
  for (int j = threadIdx.x; j < p.m; j += blockDim.x) {
    const int64_t s = p.slots[j];
    if (s < 0) continue;
    int64_t b = s / p.BS;
    int t = 0;
    if (b >= p.split) {
      t = 1;
      b -= p.split;
    }
    if (b >= p.nblk[t]) bad = 1;
  }
  __syncthreads();
  if (bad) {
    if (blockIdx.x == 0 && threadIdx.x == 0) set_error(p.err, FD_DEVERR_SLOT);
    return;
  }
  const int64_t per_row = (int64_t)p.KVH * p.nch;
  const int64_t total = (int64_t)p.m * per_row;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t j = idx / per_row;
    const int64_t rem = idx - j * per_row;
    const int64_t h = rem / p.nch;
    const int64_t c = rem - h * p.nch;
    const int64_t s = p.slots[j];
    if (s < 0) continue;
    int64_t b = s / p.BS;
    const int64_t off = s - b * p.BS;
    int t = 0;
    if (b >= p.split) {
      t = 1;
      b -= p.split;
    }
    const int64_t dst = b * p.blk_sb[t] + h * p.head_sb[t] + off * p.tok_sb[t] + c * 16;
    const uint4 kv = *reinterpret_cast<const uint4*>(p.key + j * p.k_sn + h * p.k_sh + c * 16);
    const uint4 vv = *reinterpret_cast<const uint4*>(p.value + j * p.v_sn + h * p.v_sh + c * 16);
    *reinterpret_cast<uint4*>(p.tk[t] + dst) = kv;
    *reinterpret_cast<uint4*>(p.tv[t] + dst) = vv;
  }
}

}  // namespace fdk

extern "C" int fd_store_kv(const void* key, int64_t key_stride_n, int64_t key_stride_h,
                           const void* value, int64_t value_stride_n, int64_t value_stride_h,
                           const int64_t* slots, int32_t m, int32_t num_kv_heads, int32_t head_size,
                           int32_t block_size, int32_t dtype, const fd_kv_tier* tiers,
                           int64_t tier_split, int32_t* error, void* stream) {
  const int es = fdh::elem_size(dtype);
  if (es == 0) return fdh::fail(FD_ERR_UNSUPPORTED, "fd_store_kv: unsupported dtype %d", dtype);
  if (m < 0 || num_kv_heads <= 0 || head_size <= 0 || block_size <= 0)
    return fdh::fail(FD_ERR_INVALID, "fd_store_kv: bad shape");
  if (m == 0) return FD_OK;
  if (key == nullptr || value == nullptr || slots == nullptr || tiers == nullptr)
    return fdh::fail(FD_ERR_INVALID, "fd_store_kv: null pointer");
  if (((int64_t)head_size * es) % 16 != 0)
    return fdh::fail(FD_ERR_ALIGN, "fd_store_kv: head_size*elem_size must be a multiple of 16");
  if (!fdh::aligned16(key) || !fdh::aligned16(value) || (key_stride_n * es) % 16 ||
      (key_stride_h * es) % 16 || (value_stride_n * es) % 16 || (value_stride_h * es) % 16)
    return fdh::fail(FD_ERR_ALIGN, "fd_store_kv: key/value pointers and strides must be 16-byte aligned");
  fdk::StoreParams p{};
  p.key = static_cast<const unsigned char*>(key);
  p.value = static_cast<const unsigned char*>(value);
  p.k_sn = key_stride_n * es;
  p.k_sh = key_stride_h * es;
  p.v_sn = value_stride_n * es;
  p.v_sh = value_stride_h * es;
  p.slots = slots;
  p.m = m;
  p.KVH = num_kv_heads;
  p.nch = head_size * es / 16;
  p.BS = block_size;
  p.split = tier_split;
  p.err = error;
  for (int t = 0; t < 2; ++t) {
    p.tk[t] = static_cast<unsigned char*>(tiers[t].k);
    p.tv[t] = static_cast<unsigned char*>(tiers[t].v);
    p.blk_sb[t] = tiers[t].blk_stride * es;
    p.head_sb[t] = tiers[t].head_stride * es;
    p.tok_sb[t] = tiers[t].tok_stride * es;
    p.nblk[t] = tiers[t].num_blocks > 0 ? tiers[t].num_blocks : 0;
    if (p.nblk[t] > 0) {
      if (p.tk[t] == nullptr || p.tv[t] == nullptr)
        return fdh::fail(FD_ERR_INVALID, "fd_store_kv: tier %d has blocks but no K/V pointer", t);
      if (!fdh::aligned16(p.tk[t]) || !fdh::aligned16(p.tv[t]) || p.blk_sb[t] % 16 ||
          p.head_sb[t] % 16 || p.tok_sb[t] % 16)
        return fdh::fail(FD_ERR_ALIGN, "fd_store_kv: tier %d pointers/strides must be 16-byte aligned", t);
    }
  }
  const int64_t total = (int64_t)m * num_kv_heads * p.nch;
  const int threads = 256;
  int64_t blocks = (total + threads - 1) / threads;
  if (blocks > 148 * 8) blocks = 148 * 8;
  fdk::fd_store_kv_kernel<<<(unsigned)blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return fdh::cuda_status(cudaGetLastError(), "fd_store_kv_kernel launch");
}
