// Exchange + merge of the sharded decode's partials over peer memory: the
// fused replacement of "NCCL all-gather, then the P-way merge kernel" of the
// long-context path (one rank per GPU, KV sharded over the ranks).
//
// Each rank owns one device allocation, mapped into every other rank's
// process with CUDA IPC (plain device memory: no multicast object, no NVLS):
//   [0]   step counter      u64, this rank's completed steps
//   [8]   CTA counter       u64, this rank's finished CTAs
//   [16]  push counter      u64, this rank's CTAs done pushing
//   [64]  arrival flags     u64 [FD_MAX_PEERS]: flag q holds the last step
//                            whose slot rank q has delivered into this
//                            buffer (written only by rank q, st.release.sys)
//   [256] receive buffer    fp32 [2 parities][world][slot], slot = the packed
//                            partial [o (n*H*D) | lse (H*n)] rounded to 4
// One launch per step of at most 64 small CTAs, which the SMs hold at once
// (every wait is bounded in any case):
//   1. every CTA stores its share of the rank's packed partial into slot
//      [parity][rank] of every rank's receive buffer (16-byte stores over
//      NVLink; the own copy is local), fences at system scope and counts
//      itself on the rank's push counter; the last CTA of the rank fences
//      again and writes the step into flag [rank] of every rank's buffer
//      (world remote release stores per rank and step);
//   2. it waits (bounded, %globaltimer) until every flag of its own buffer
//      holds at least the step: each rank's slot of this step has landed.
//      Per-source flags, not one summed counter: a peer that is already a
//      step ahead must not stand in for a rank whose signal of this step is
//      still in flight;
//   3. it merges its (row, head) pairs from the receive buffer with the
//      log-sum-exp rule of fd_merge_partials, same operations in the same
//      order (so the result equals the NCCL path bit for bit);
//   4. the last CTA to finish advances the step counter, so the next launch
//      (or graph replay) uses the other parity and the next step number.
// Double buffering by parity keeps a rank that is one step ahead from
// overwriting a slot another rank is still merging; it cannot get two steps
// ahead, because finishing a step needs every rank's flag of that step, and
// a rank raises its flag of step s + 1 only after its merge of step s ended.
//
// The kernel is launched as a programmatic dependent of the kernel before it
// on the stream (the decode's combine): its launch overlaps that kernel's
// tail, and griddepcontrol.wait holds every CTA until the partial it pushes
// is complete.

#include <math.h>
#include <stdint.h>
#include <string.h>

#include "fd_common.cuh"
#include "fd_internal.h"

namespace fdk {

struct ExchangeParams {
  const float* send;                      // [slot] this rank's packed partial
  float* recv[FD_MAX_PEERS];              // rank q's receive buffer (mapped)
  unsigned long long* flag_at[FD_MAX_PEERS];  // this rank's arrival flag in rank q's buffer (mapped)
  const unsigned long long* flags;        // this rank's arrival flags [world]
  unsigned long long* step;               // this rank's step counter
  unsigned long long* done;               // this rank's finished-CTA counter
  unsigned long long* pushed;             // this rank's CTAs done pushing
  int rank, world, n, H, D;
  int64_t slot;                           // floats per rank slot (multiple of 4)
  void* out;
  int out_dtype;
  float* out_lse;
  int64_t timeout_ns;
  int32_t* err;
};

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ float lse_or_empty(float x) { return x == INFINITY ? -INFINITY : x; }

__global__ void fd_exchange_merge_kernel(const __grid_constant__ ExchangeParams p) {
  __shared__ unsigned long long s_step;
  __shared__ int s_ok;
  griddep_wait();  // the partial in p.send is complete (programmatic dependent launch)
  if (threadIdx.x == 0) {
    s_step = *reinterpret_cast<volatile unsigned long long*>(p.step) + 1;
    s_ok = 1;
  }
  __syncthreads();
  const unsigned long long step = s_step;
  const int par = (int)(step & 1ull);

  // 1. push this rank's slot to every rank
  const float4* src = reinterpret_cast<const float4*>(p.send);
  const int64_t nvec = p.slot / 4;
  const int64_t dst_off = ((int64_t)par * p.world + p.rank) * p.slot;
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < nvec; c += (int64_t)gridDim.x * blockDim.x) {
    const float4 v = src[c];
    for (int q = 0; q < p.world; ++q) reinterpret_cast<float4*>(p.recv[q] + dst_off)[c] = v;
  }
  __syncthreads();  // the CTA's stores happen before thread 0's fence and release

  // 2. the rank's last CTA to finish pushing raises the rank's flag in every
  // rank's buffer; then every CTA waits for every rank's flag of this step
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned long long prev = atomicAdd(p.pushed, 1ull);
    if (prev + 1 == step * gridDim.x) {
      __threadfence_system();  // the other CTAs' fenced stores happen before the flags
      for (int q = 0; q < p.world; ++q) st_release_sys(p.flag_at[q], step);
    }
    const uint64_t t0 = globaltimer_ns();
    uint32_t it = 0;
    for (int q = 0; q < p.world && s_ok; ++q) {
      while (ld_acquire_sys(p.flags + q) < step) {
        if ((++it & 63u) == 0 && globaltimer_ns() - t0 > (uint64_t)p.timeout_ns) {
          set_error(p.err, FD_DEVERR_TIMEOUT);
          s_ok = 0;
          break;
        }
      }
    }
  }
  __syncthreads();

  // 3. merge (one warp per (row, head) pair)
  if (s_ok) {
    const float* base = p.recv[p.rank] + (int64_t)par * p.world * p.slot;
    const int64_t o_floats = (int64_t)p.n * p.H * p.D;
    const int lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const int64_t pairs = (int64_t)p.n * p.H;
    for (int64_t pr = (int64_t)blockIdx.x * nw + (threadIdx.x >> 5); pr < pairs; pr += (int64_t)gridDim.x * nw) {
      const int i = (int)(pr / p.H), h = (int)(pr - (int64_t)i * p.H);
      const int64_t lo = o_floats + (int64_t)h * p.n + i;
      // lane q reads rank q's lse; every lane then holds all of them
      const float mine = lane < p.world ? lse_or_empty(__ldcg(base + lane * p.slot + lo)) : -INFINITY;
      float lse_q[FD_MAX_PEERS];
#pragma unroll
      for (int q = 0; q < FD_MAX_PEERS; ++q) lse_q[q] = __shfl_sync(0xffffffffu, mine, q);
      float m = -INFINITY;
#pragma unroll
      for (int q = 0; q < FD_MAX_PEERS; ++q)
        if (q < p.world) m = fmaxf(m, lse_q[q]);
      const bool all_empty = (m == -INFINITY);
      if (all_empty) m = 0.f;
      float w[FD_MAX_PEERS];
      float tot = 0.f;
#pragma unroll
      for (int q = 0; q < FD_MAX_PEERS; ++q) {
        w[q] = q < p.world ? expf(lse_q[q] - m) : 0.f;
        if (q < p.world) tot += w[q];
      }
      if (all_empty) tot = 1.f;
      const float inv = 1.f / tot;
      const int64_t ob = ((int64_t)i * p.H + h) * p.D;
      for (int d = lane; d < p.D; d += 32) {
        float o_q[FD_MAX_PEERS];
#pragma unroll
        for (int q = 0; q < FD_MAX_PEERS; ++q) o_q[q] = q < p.world ? __ldcg(base + q * p.slot + ob + d) : 0.f;
        float x = 0.f;
#pragma unroll
        for (int q = 0; q < FD_MAX_PEERS; ++q)
          if (q < p.world) x = fmaf(w[q] * inv, o_q[q], x);
        store_out(p.out, ob + d, p.out_dtype, x);
      }
      if (lane == 0 && p.out_lse != nullptr) p.out_lse[(int64_t)h * p.n + i] = all_empty ? -INFINITY : m + logf(tot);
    }
  }

  // 4. the last CTA of the step advances the step counter
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned long long prev = atomicAdd(p.done, 1ull);
    if (prev + 1 == step * gridDim.x) {
      __threadfence();
      *reinterpret_cast<volatile unsigned long long*>(p.step) = step;
    }
  }
}

}  // namespace fdk

namespace {
constexpr size_t kStepOffset = 0;
constexpr size_t kDoneOffset = 8;
constexpr size_t kPushedOffset = 16;
constexpr size_t kFlagsOffset = 64;
constexpr size_t kRecvOffset = 256;
static_assert(kFlagsOffset + 8 * FD_MAX_PEERS <= kRecvOffset, "arrival flags overlap the receive buffer");
}

extern "C" size_t fd_peer_buffer_bytes(int32_t world, int64_t slot_floats) {
  if (world < 1 || world > FD_MAX_PEERS || slot_floats < 0) return 0;
  const int64_t slot = (slot_floats + 3) / 4 * 4;
  return kRecvOffset + (size_t)2 * (size_t)world * (size_t)slot * sizeof(float);
}

extern "C" int fd_peer_alloc(size_t bytes, void** ptr, void* ipc_handle) {
  if (ptr == nullptr || ipc_handle == nullptr || bytes < kRecvOffset)
    return fdh::fail(FD_ERR_INVALID, "fd_peer_alloc: null output or size below %zu bytes", kRecvOffset);
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return fdh::cuda_status(e, "fd_peer_alloc: cudaMalloc");
  e = cudaMemset(p, 0, bytes);  // counters start at 0
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fdh::cuda_status(e, "fd_peer_alloc: cudaMemset / cudaIpcGetMemHandle");
  }
  static_assert(sizeof(cudaIpcMemHandle_t) <= FD_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return FD_OK;
}

extern "C" int fd_peer_open(const void* ipc_handle, void** ptr) {
  if (ptr == nullptr || ipc_handle == nullptr) return fdh::fail(FD_ERR_INVALID, "fd_peer_open: null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  return fdh::cuda_status(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
}

extern "C" int fd_peer_close(void* ptr) {
  if (ptr == nullptr) return fdh::fail(FD_ERR_INVALID, "fd_peer_close: null pointer");
  return fdh::cuda_status(cudaIpcCloseMemHandle(ptr), "cudaIpcCloseMemHandle");
}

extern "C" int fd_peer_free(void* ptr) {
  if (ptr == nullptr) return fdh::fail(FD_ERR_INVALID, "fd_peer_free: null pointer");
  return fdh::cuda_status(cudaFree(ptr), "fd_peer_free: cudaFree");
}

extern "C" int fd_exchange_merge(const fd_peer_exchange* x, const float* send, int32_t n, int32_t num_heads,
                                 int32_t head_size, void* out, int32_t out_dtype, float* out_lse, int32_t num_ctas,
                                 int64_t timeout_ns, int32_t* error, void* stream) {
  if (x == nullptr || send == nullptr || out == nullptr)
    return fdh::fail(FD_ERR_INVALID, "fd_exchange_merge: null argument");
  if (x->world < 1 || x->world > FD_MAX_PEERS || x->rank < 0 || x->rank >= x->world)
    return fdh::fail(FD_ERR_INVALID, "fd_exchange_merge: rank %d of world %d (at most %d)", x->rank, x->world,
                     FD_MAX_PEERS);
  if (n < 0 || num_heads < 1 || head_size < 1) return fdh::fail(FD_ERR_INVALID, "fd_exchange_merge: bad shape");
  const int64_t need = (int64_t)n * num_heads * head_size + (int64_t)num_heads * n;
  if (x->slot_floats < need || x->slot_floats % 4 != 0)
    return fdh::fail(FD_ERR_INVALID, "fd_exchange_merge: slot of %lld floats, need >= %lld and a multiple of 4",
                     (long long)x->slot_floats, (long long)need);
  if (fdh::elem_size(out_dtype) == 0) return fdh::fail(FD_ERR_UNSUPPORTED, "fd_exchange_merge: out dtype");
  if ((reinterpret_cast<uintptr_t>(send) & 15u) != 0)
    return fdh::fail(FD_ERR_ALIGN, "fd_exchange_merge: send buffer not 16-byte aligned");
  for (int q = 0; q < x->world; ++q)
    if (x->base[q] == nullptr) return fdh::fail(FD_ERR_INVALID, "fd_exchange_merge: rank %d buffer unmapped", q);
  constexpr int kThreads = 256;
  const int ctas = num_ctas > 0 ? num_ctas : 32;
  if (ctas > 64) return fdh::fail(FD_ERR_INVALID, "fd_exchange_merge: at most 64 CTAs (%d)", ctas);
  fdk::ExchangeParams p{};
  p.send = send;
  unsigned char* own = static_cast<unsigned char*>(x->base[x->rank]);
  for (int q = 0; q < x->world; ++q) {
    unsigned char* b = static_cast<unsigned char*>(x->base[q]);
    p.recv[q] = reinterpret_cast<float*>(b + kRecvOffset);
    p.flag_at[q] = reinterpret_cast<unsigned long long*>(b + kFlagsOffset) + x->rank;
  }
  p.flags = reinterpret_cast<const unsigned long long*>(own + kFlagsOffset);
  p.step = reinterpret_cast<unsigned long long*>(own + kStepOffset);
  p.done = reinterpret_cast<unsigned long long*>(own + kDoneOffset);
  p.pushed = reinterpret_cast<unsigned long long*>(own + kPushedOffset);
  p.rank = x->rank;
  p.world = x->world;
  p.n = n;
  p.H = num_heads;
  p.D = head_size;
  p.slot = x->slot_floats;
  p.out = out;
  p.out_dtype = out_dtype;
  p.out_lse = out_lse;
  p.timeout_ns = timeout_ns > 0 ? timeout_ns : (int64_t)fdk::kWaitLimitNs;
  p.err = error;
  // Every CTA waits for every other.  A cooperative launch would guarantee
  // co-residency but cost ~55 us per step on B200 (measured); at most 64
  // CTAs of 256 threads and no shared memory are resident together on an
  // otherwise idle stream, and the bounded wait turns any exception into
  // FD_DEVERR_TIMEOUT rather than a hang.  Programmatic dependent launch:
  // the CTAs may start while the kernel ahead on the stream finishes and
  // wait for it in griddepcontrol.wait.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ctas);
  cfg.blockDim = dim3((unsigned)kThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, fdk::fd_exchange_merge_kernel, p);
  if (e != cudaSuccess) return fdh::cuda_status(e, "fd_exchange_merge_kernel launch");
  return fdh::cuda_status(cudaGetLastError(), "fd_exchange_merge_kernel launch");
}
