// Tier-aware KV write: one kernel puts each new K/V row into its slot in the
// HBM tier or in the mapped host tier.  Bit-exact 16-byte copies.
//
// Addressing follows the reference store_kv (fastdecode/csrc/cpu_attn.cpp
// :413-431): blk = slot / BS, off = slot % BS, destination
// blk*blk_stride + head*head_stride + off*tok_stride.  Range checking follows
// :506-510, except that it runs on the device: all slots are checked before
// any row is written and, if any is outside both tiers, nothing is written
// and the error word gets FD_DEVERR_SLOT.  slot < 0 means "not this call's" and is skipped,
// like reshape_and_cache_flash.
//
// The all-or-nothing check takes one of two forms.  Up to kSmallM rows (a
// decode step's writes) one kernel does it all: every CTA scans all m slots
// (two per 16-byte load) before it copies, on a grid of at most two CTAs of
// 512 threads per SM.  Above kSmallM (prefill-sized writes, where every CTA
// scanning every slot would cost a fifth of the copy) a check kernel scans
// the slots once (1024 per CTA, one load per thread; the last CTA to finish
// folds the CTAs' results into one flag of this call; itself a programmatic
// dependent of the kernel ahead, whose completion it awaits before reading
// the slots) and the copy kernel, launched as its
// programmatic dependent on a grid that covers all chunks, issues its first
// loads, waits for the check (griddepcontrol.wait), and writes only if the
// flag is clear.  A call's flag is a slot of a ring of kFlagRing, chosen on
// the host per call; two calls in flight at once share one only if they are
// kFlagRing calls apart.

#include <atomic>

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
  int flag;  // this call's slot of the flag ring (two-kernel form)
};

constexpr int kStoreThreads = 512;
constexpr int kStoreUnroll = 2;
constexpr int kSmallM = 2048;        // rows up to which one kernel checks and copies
constexpr int kCheckThreads = 512;
constexpr int kCheckSlots = 2 * kCheckThreads;  // slots per check CTA: one 16-byte load per thread
constexpr int kFlagRing = 1024;
__device__ int g_store_bad[kFlagRing];          // per call: 1 = some slot out of range
__device__ int g_store_acc[kFlagRing];          // OR of the check CTAs' results (reset by the last)
__device__ unsigned g_store_done[kFlagRing];    // check CTAs finished (reset by the last)

__device__ __forceinline__ bool slot_out_of_range(const StoreParams& p, int64_t s) {
  if (s < 0) return false;
  int64_t b = s / p.BS;
  int t = 0;
  if (b >= p.split) {
    t = 1;
    b -= p.split;
  }
  return b >= p.nblk[t];
}

// Does any of slots [lo, hi) fall outside both tiers?  (The block's threads
// together; slots are 8-byte aligned: pairs from a 16-byte boundary, the odd
// ones at either end alone.)
__device__ __forceinline__ bool scan_slots(const StoreParams& p, int lo, int hi) {
  bool mine = false;
  if (lo >= hi) return false;
  const int lead = (reinterpret_cast<uintptr_t>(p.slots + lo) & 15u) ? 1 : 0;
  if (lead && threadIdx.x == 0) mine = slot_out_of_range(p, p.slots[lo]);
  const int pairs = (hi - lo - lead) / 2;
  const longlong2* sp = reinterpret_cast<const longlong2*>(p.slots + lo + lead);
  for (int j = threadIdx.x; j < pairs; j += blockDim.x) {
    const longlong2 v = sp[j];
    mine |= slot_out_of_range(p, v.x) | slot_out_of_range(p, v.y);
  }
  if (threadIdx.x == 0 && lo + lead + 2 * pairs < hi) mine |= slot_out_of_range(p, p.slots[hi - 1]);
  return mine;
}

// The check of the two-kernel form.
__global__ void __launch_bounds__(kCheckThreads) fd_store_check_kernel(const __grid_constant__ StoreParams p) {
  griddep_wait();               // the kernel ahead (which may have written the slots) has completed
  griddep_launch_dependents();  // the copy kernel's CTAs may start loading now
  const int lo = blockIdx.x * kCheckSlots;
  const bool bad = __syncthreads_or(scan_slots(p, lo, min(p.m, lo + kCheckSlots)) ? 1 : 0) != 0;
  if (threadIdx.x == 0) {
    if (bad) atomicOr(&g_store_acc[p.flag], 1);
    __threadfence();
    if (atomicAdd(&g_store_done[p.flag], 1u) == gridDim.x - 1) {  // the last check CTA of this call
      __threadfence();
      const int any = atomicExch(&g_store_acc[p.flag], 0);
      g_store_done[p.flag] = 0u;
      g_store_bad[p.flag] = any;
      if (any) set_error(p.err, FD_DEVERR_SLOT);
    }
  }
}

// kChecked = false: the one-kernel form (every CTA scans all slots first);
// true: the copy of the two-kernel form (the check kernel ahead of it).
template <bool kChecked, int kUnroll>
__global__ void __launch_bounds__(kStoreThreads) fd_store_kv_kernel(const __grid_constant__ StoreParams p) {
  if (!kChecked && __syncthreads_or(scan_slots(p, 0, p.m) ? 1 : 0)) {
    if (blockIdx.x == 0 && threadIdx.x == 0) set_error(p.err, FD_DEVERR_SLOT);
    return;
  }
  // 32-bit chunk indices (the host refuses calls of 2^31 chunks or more)
  const uint32_t per_row = (uint32_t)p.KVH * (uint32_t)p.nch;
  const uint32_t total = (uint32_t)p.m * per_row;
  const uint32_t stride = gridDim.x * blockDim.x;
  bool first = true;
  for (uint32_t base = blockIdx.x * blockDim.x + threadIdx.x;; base += stride * kUnroll) {
    if (kChecked && first) {
      // the first loads (below) are issued; then the check's verdict
    } else if (base >= total) {
      break;
    }
    uint4 kv[kUnroll], vv[kUnroll];
    int64_t dst[kUnroll];
    int tier[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
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
      if (b >= p.nblk[t]) continue;  // never written (the check has rejected the call); no address formed
      tier[u] = t;
      dst[u] = b * p.blk_sb[t] + (int64_t)h * p.head_sb[t] + off * p.tok_sb[t] + c * 16;
      kv[u] = *reinterpret_cast<const uint4*>(p.key + j * p.k_sn + h * p.k_sh + c * 16);
      vv[u] = *reinterpret_cast<const uint4*>(p.value + j * p.v_sn + h * p.v_sh + c * 16);
    }
    if (kChecked && first) {
      griddep_wait();  // the check kernel has completed and its flag is visible
      if (*reinterpret_cast<volatile const int*>(&g_store_bad[p.flag]) != 0) return;
    }
    first = false;
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
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
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (m <= fdk::kSmallM) {
    int dev = 0, sms = 0;
    const int st = fdh::device_sms(&dev, &sms);
    if (st != FD_OK) return st;
    int64_t blocks = (total + (int64_t)threads * fdk::kStoreUnroll - 1) / ((int64_t)threads * fdk::kStoreUnroll);
    if (blocks > 2 * (int64_t)sms) blocks = 2 * (int64_t)sms;  // every CTA scans all slots: few, wide CTAs
    fdk::fd_store_kv_kernel<false, fdk::kStoreUnroll><<<(unsigned)blocks, threads, 0, s>>>(p);
    return fdh::cuda_status(cudaGetLastError(), "fd_store_kv_kernel launch");
  }
  static std::atomic<unsigned> next_flag{0};
  p.flag = (int)(next_flag.fetch_add(1u, std::memory_order_relaxed) % (unsigned)fdk::kFlagRing);
  const unsigned checks = (unsigned)((m + fdk::kCheckSlots - 1) / fdk::kCheckSlots);
  int st = fdh::launch_maybe_pdl(reinterpret_cast<const void*>(fdk::fd_store_check_kernel), dim3(checks),
                                  dim3(fdk::kCheckThreads), 0, s, true, p, "fd_store_check_kernel launch");
  if (st != FD_OK) return st;
  // every thread two 16-byte chunks of K and V, one per pass
  const int64_t blocks = (total + (int64_t)threads * 2 - 1) / ((int64_t)threads * 2);
  return fdh::launch_maybe_pdl(reinterpret_cast<const void*>(fdk::fd_store_kv_kernel<true, 1>), dim3((unsigned)blocks),
                               dim3(threads), 0, s, true, p, "fd_store_kv_kernel launch");
}
