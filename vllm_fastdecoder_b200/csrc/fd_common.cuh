// Device helpers shared by the fastdecode_b200 kernels (sm_100a only):
// dtype traits, mbarrier / bulk-copy PTX wrappers with bounded waits, and the
// device error word.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "fastdecode_b200.h"

namespace fdk {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// A bounded wait gives up after this long (the longest legitimate wait on a
// pipeline stage is a few microseconds of HBM or PCIe latency).
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ void set_error(int32_t* err, int32_t code) {
  if (err != nullptr) atomicCAS(err, 0, code);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ------------------------------------------------------------- mbarrier

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

// Make barrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

// Raise the transaction count of the current phase without arriving.
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking test of the phase with the given parity (no suspend window),
// for a thread that polls several barriers in turn.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete; gives up after
// kWaitLimitNs, records FD_DEVERR_TIMEOUT and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int32_t* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) {
      set_error(err, FD_DEVERR_TIMEOUT);
      return false;
    }
  }
}

// 4-byte asynchronous copy global -> shared (LDGSTS), tracked by commit
// groups of the issuing thread; src and dst 4-byte aligned.
__device__ __forceinline__ void cp_async4(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// Wait until at most N of this thread's commit groups are pending.
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Programmatic dependent launch: a kernel launched with programmatic stream
// serialization may start before the kernel ahead of it in the stream ends;
// griddep_wait() blocks until that kernel has completed and its memory
// operations are visible, and griddep_launch_dependents() lets the
// dependent kernel start launching once every CTA has called it or exited.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// Fetch the 128-byte line holding p into L2 (no register result).
__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// Bulk (non-tensor) TMA copy global -> shared, completion counted in bytes on
// `bar`.  dst, src and bytes must be multiples of 16.  No multicast.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes,
                                         uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Tiled TMA load of a 4-D box described by a tensor map (kernel parameter,
// __grid_constant__) into shared memory, completion as bytes on `bar`.
// dst must be 128-byte aligned.  No multicast.
__device__ __forceinline__ void tma_load_4d(void* smem_dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            int c3, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// L2 policy for data read exactly once (K/V streams).
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ void named_barrier_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ uint4 lds128(const void* p) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(smem_u32(p)));
  return v;
}

__device__ __forceinline__ void sts128(void* p, const uint4& v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(smem_u32(p)), "r"(v.x),
               "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// ------------------------------------------------------------- packed fp32x2

// Two fp32 values in one 64-bit register pair, operated on by the packed
// fp32 pipe of sm_100 (fma/mul .f32x2: two lanes per instruction).
typedef unsigned long long f2_t;

__device__ __forceinline__ f2_t f2_pack(float lo, float hi) {
  f2_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}

__device__ __forceinline__ void f2_unpack(f2_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}

__device__ __forceinline__ f2_t f2_fma(f2_t a, f2_t b, f2_t c) {
  f2_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

__device__ __forceinline__ f2_t f2_add(f2_t a, f2_t b) {
  f2_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

__device__ __forceinline__ f2_t f2_mul(f2_t a, f2_t b) {
  f2_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// ------------------------------------------------------------- dtypes

template <typename T>
struct Dt;

template <>
struct Dt<__half> {
  static constexpr int kEPC = 8;  // elements per 16-byte chunk
  __device__ static __forceinline__ void widen(const uint4& v, float* f) {
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 x = __half22float2(h[i]);
      f[2 * i] = x.x;
      f[2 * i + 1] = x.y;
    }
  }
  // 16 bytes -> 4 packed pairs
  __device__ static __forceinline__ void widen2(const uint4& v, f2_t* f) {
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 x = __half22float2(h[i]);
      f[i] = f2_pack(x.x, x.y);
    }
  }
  __device__ static __forceinline__ __half narrow(float x) { return __float2half_rn(x); }
  __device__ static __forceinline__ float to_f32(__half x) { return __half2float(x); }
};

template <>
struct Dt<__nv_bfloat16> {
  static constexpr int kEPC = 8;
  __device__ static __forceinline__ void widen(const uint4& v, float* f) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
  __device__ static __forceinline__ void widen2(const uint4& v, f2_t* f) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) f[i] = f2_pack(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xffff0000u));
  }
  __device__ static __forceinline__ __nv_bfloat16 narrow(float x) { return __float2bfloat16_rn(x); }
  __device__ static __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
};

template <>
struct Dt<float> {
  static constexpr int kEPC = 4;
  __device__ static __forceinline__ void widen(const uint4& v, float* f) {
    f[0] = __uint_as_float(v.x);
    f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z);
    f[3] = __uint_as_float(v.w);
  }
  __device__ static __forceinline__ void widen2(const uint4& v, f2_t* f) {
    f[0] = f2_pack(__uint_as_float(v.x), __uint_as_float(v.y));
    f[1] = f2_pack(__uint_as_float(v.z), __uint_as_float(v.w));
  }
  __device__ static __forceinline__ float narrow(float x) { return x; }
  __device__ static __forceinline__ float to_f32(float x) { return x; }
};

__device__ __forceinline__ void store_out(void* base, int64_t idx, int dtype, float x) {
  if (dtype == FD_DTYPE_F32) {
    static_cast<float*>(base)[idx] = x;
  } else if (dtype == FD_DTYPE_F16) {
    static_cast<__half*>(base)[idx] = __float2half_rn(x);
  } else {
    static_cast<__nv_bfloat16*>(base)[idx] = __float2bfloat16_rn(x);
  }
}

__device__ __forceinline__ float load_in(const void* base, int64_t idx, int dtype) {
  if (dtype == FD_DTYPE_F32) return static_cast<const float*>(base)[idx];
  if (dtype == FD_DTYPE_F16) return __half2float(static_cast<const __half*>(base)[idx]);
  return __bfloat162float(static_cast<const __nv_bfloat16*>(base)[idx]);
}

}  // namespace fdk
