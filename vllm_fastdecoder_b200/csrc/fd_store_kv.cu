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
//
// The all-or-nothing check makes every CTA read all m slots, so the grid is
// kept to at most two CTAs of 512 threads per SM (a prefill-sized m = 16k
// reads ~40 MB of slots from L2 in all, not the ~150 MB of one CTA per 256
// chunks), the scan reads two slots per 16-byte load, and the copy keeps two
// 16-byte loads of K and V in flight per thread so the few CTAs still stream
// at HBM rate.

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

constexpr int kStoreThreads = 512;
constexpr int kStoreUnroll = 2;

__global__ void __launch_bounds__(kStoreThreads, 2) fd_store_kv_kernel(const __grid_constant__ StoreParams p) {
  auto out_of_range = [&](int64_t s) -> bool {
    if (s < 0) return false;
    int64_t b = s / p.BS;
    int t = 0;
    if (b >= p.split) {
      t = 1;
      b -= p.split;
    }
    return b >= p.nblk[t];
  };
  // slots are 8-byte aligned; pairs from a 16-byte boundary, the odd one out alone
  const int lead = (reinterpret_cast<uintptr_t>(p.slots) & 15u) ? 1 : 0;
  bool mine = false;
  if (lead && threadIdx.x == 0 && p.m > 0) mine = out_of_range(p.slots[0]);
  const int pairs = (p.m - lead) / 2;
  const longlong2* sp = reinterpret_cast<const longlong2*>(p.slots + lead);
  for (int j = threadIdx.x; j < pairs; j += blockDim.x) {
    const longlong2 v = sp[j];
    mine |= out_of_range(v.x) | out_of_range(v.y);
  }
  if (threadIdx.x == 0 && lead + 2 * pairs < p.m) mine |= out_of_range(p.slots[p.m - 1]);
  if (__syncthreads_or(mine ? 1 : 0)) {
    if (blockIdx.x == 0 && threadIdx.x == 0) set_error(p.err, FD_DEVERR_SLOT);
    return;
  }
  // 32-bit chunk indices (the host refuses calls of 2^31 chunks or more)
  const uint32_t per_row = (uint32_t)p.KVH * (uint32_t)p.nch;
  const uint32_t total = (uint32_t)p.m * per_row;
  const uint32_t stride = gridDim.x * blockDim.x;
  for (uint32_t base = blockIdx.x * blockDim.x + threadIdx.x; base < total; base += stride * kStoreUnroll) {
    uint4 kv[kStoreUnroll], vv[kStoreUnroll];
    int64_t dst[kStoreUnroll];
    int tier[kStoreUnroll];
#pragma unroll
    for (int u = 0; u < kStoreUnroll; ++u) {
      const uint32_t idx = base + u * stride;
      dst[u] = -1;
      tier[u] = 0;
      if (idx >= total) continue;
      const uint32_t j = idx / per_row;
      const uint32_t rem = idx - j * per_row;
      const uint32_t h = rem / (uint32_t)p.nch;
      const uint32_t c = rem - h * (uint32_t)p.nch;
      const int64_t s = p.slots[j];
      if (s < 0) continue;
      int64_t b = s / p.BS;
      const int64_t off = s - b * p.BS;
      const int t = b >= p.split ? 1 : 0;
      if (t) b -= p.split;
      tier[u] = t;
      dst[u] = b * p.blk_sb[t] + (int64_t)h * p.head_sb[t] + off * p.tok_sb[t] + c * 16;
      kv[u] = *reinterpret_cast<const uint4*>(p.key + j * p.k_sn + h * p.k_sh + c * 16);
      vv[u] = *reinterpret_cast<const uint4*>(p.value + j * p.v_sn + h * p.v_sh + c * 16);
    }
#pragma unroll
    for (int u = 0; u < kStoreUnroll; ++u) {
      if (dst[u] < 0) continue;
      *reinterpret_cast<uint4*>(p.tk[tier[u]] + dst[u]) = kv[u];
      *reinterpret_cast<uint4*>(p.tv[tier[u]] + dst[u]) = vv[u];
    }
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
  if (total >= (int64_t)1 << 31)
    return fdh::fail(FD_ERR_UNSUPPORTED, "fd_store_kv: %lld 16-byte chunks in one call (at most 2^31 - 1)",
                     (long long)total);
  const int threads = fdk::kStoreThreads;
  int dev = 0, sms = 0;
  const int st = fdh::device_sms(&dev, &sms);
  if (st != FD_OK) return st;
  int64_t blocks = (total + (int64_t)threads * fdk::kStoreUnroll - 1) / ((int64_t)threads * fdk::kStoreUnroll);
  if (blocks > 2 * (int64_t)sms) blocks = 2 * (int64_t)sms;  // every CTA scans all slots: few, wide CTAs
  fdk::fd_store_kv_kernel<<<(unsigned)blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return fdh::cuda_status(cudaGetLastError(), "fd_store_kv_kernel launch");
}
