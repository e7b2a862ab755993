// Exchange + merge of the sharded decode's partials over peer memory: the
// fused replacement of "combine kernel, NCCL all-gather, then the P-way merge
// kernel" of the long-context path (one rank per GPU, KV sharded over the
// ranks).
//
// Each rank owns one device allocation, mapped into every other rank's
// process with CUDA IPC (plain device memory: no multicast object, no NVLS):
//   [0]    step counters    u64 [kMaxCtas]: CTA b's completed steps (its own)
//   [8192] receive slots    [2 parities][world][slot] tagged words: float i of
//                            a slot is the 8-byte word {value bits, step}
// One launch per step of at most 64 CTAs of 128 threads, which the SMs hold
// at once (every wait is bounded in any case):
//   1. every CTA stores its share of the rank's packed partial into slot
//      [parity][rank] of every rank's buffer over NVLink, each float with the
//      step number in the same 8-byte word (16-byte volatile stores of two
//      tagged words; the own copy is local).  Given the decode launch's
//      geometry (fd_decode_exchange_merge) the share is a set of (row,
//      kv-head chunk) segments: a segment one decode CTA finished is copied
//      from the decode's output, a segment that decode CTA ranges cut is
//      merged from the decode's partial slots on the way (the rule and order
//      of the decode's own combine), so no combine launch runs before the
//      exchange;
//   2. each warp merges (row, head) pairs: it reads every rank's words for
//      its pair from its own buffer, re-reading each until it carries this
//      step (bounded, %globaltimer), and applies the log-sum-exp rule of
//      fd_merge_partials with the same operations in the same order (so the
//      result equals the NCCL path bit for bit);
//   3. the CTA advances its own step counter (every CTA keeps its own step,
//      and all CTAs of a launch agree on it).
// A value and its step land together (an aligned 8-byte word is written and
// read as a whole), so no fence and no separate arrival flag is needed: a
// reader that sees the step sees the value.  A word of another step (an
// older one in the slot, or a rank that is ahead) never matches, since a
// reader waits for equality.  Double buffering by parity keeps a rank that
// is one step ahead from overwriting a slot another rank is still merging;
// it cannot get two steps ahead, because finishing a step needs every rank's
// words of that step, and a rank writes step s + 1 only after its launch of
// step s has completed.
//
// The kernel is launched as a programmatic dependent of the kernel before it
// on the stream (the decode): its launch overlaps that kernel's tail, and
// griddepcontrol.wait holds every CTA until the decode's output is complete.

#include <math.h>
#include <stdint.h>
#include <string.h>

#include "fd_common.cuh"
#include "fd_decode.cuh"
#include "fd_internal.h"

namespace fdk {

// threads per exchange CTA: small CTAs (128 threads x ~145 registers) fit on
// an SM beside a tensor-core decode CTA, so the next step's decode, launched
// as a programmatic dependent of this kernel, can be resident on every SM
// while the exchange runs
constexpr int kXThreads = 128;
constexpr int kXMaxCtas = 64;   // CTAs per launch, at most (per-CTA step counters)

struct ExchangeParams {
  const float* send;                      // [slot] this rank's packed partial [o | lse]
  uint32_t* recv[FD_MAX_PEERS];           // rank q's receive slots (mapped): word i = u32 [2 i, 2 i + 1]
  unsigned long long* steps;              // this rank's per-CTA step counters [kXMaxCtas]
  ShardGeom geom;                         // the decode launch's segments (prefix null: send is complete)
  int rank, world, n, H, D;
  int64_t slot;                           // floats per rank slot (multiple of 4)
  void* out;
  int out_dtype;
  float* out_lse;
  int64_t timeout_ns;
  int32_t* err;
};

__device__ __forceinline__ float lse_or_empty(float x) { return x == INFINITY ? -INFINITY : x; }

// Tagged words: float i of a slot is the 8-byte word {value, step} at u32
// index 2 i.  Volatile accesses (not cached in L1, not merged or split by
// the compiler); an aligned 8-byte word is written and read whole.
__device__ __forceinline__ void st_tagged2(uint32_t* w, float a, float b, uint32_t tag) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(w), "r"(__float_as_uint(a)), "r"(tag),
               "r"(__float_as_uint(b)), "r"(tag)
               : "memory");
}
__device__ __forceinline__ void st_tagged1(uint32_t* w, float a, uint32_t tag) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(w), "r"(__float_as_uint(a)), "r"(tag) : "memory");
}
__device__ __forceinline__ uint2 ld_tagged1(const uint32_t* w) {
  uint2 v;
  asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(w) : "memory");
  return v;
}

// Read tagged word w until it carries `tag`; false once the wait, measured
// from t0, exceeds timeout_ns.
__device__ __forceinline__ bool get_tagged(const uint32_t* w, uint32_t tag, uint64_t t0, int64_t timeout_ns, float& v) {
  uint2 x = ld_tagged1(w);
  for (uint32_t it = 1; x.y != tag; ++it) {
    if ((it & 63u) == 0 && globaltimer_ns() - t0 > (uint64_t)timeout_ns) return false;
    x = ld_tagged1(w);
  }
  v = __uint_as_float(x.x);
  return true;
}

// Store at float offset `off` (a multiple of 4 for put4) of this rank's slot
// in every rank's buffer, tagged with the step.
__device__ __forceinline__ void put4(const ExchangeParams& p, int64_t off, const float4& v, uint32_t tag) {
  for (int q = 0; q < p.world; ++q) {
    uint32_t* w = p.recv[q] + 2 * off;
    st_tagged2(w, v.x, v.y, tag);
    st_tagged2(w + 4, v.z, v.w, tag);
  }
}
__device__ __forceinline__ void put1(const ExchangeParams& p, int64_t off, float v, uint32_t tag) {
  for (int q = 0; q < p.world; ++q) st_tagged1(p.recv[q] + 2 * off, v, tag);
}

// Up to this many CTAs share a cut segment on the fast path (their partials
// are loaded at once, two memory round trips); more fall back to a loop.
constexpr int kSpanFast = 4;

// Push this rank's partial segment by segment (1.): items are 4 consecutive
// dims of one head of one (row, kv-head chunk) segment, spread over the grid.
// A segment one decode CTA finished is copied from `send`, where the decode
// wrote it (empty rows included); a cut segment is merged from the decode's
// fp32 partial slots with the decode combine's rule and order: M = max lse,
// w = 2^((lse - M) log2 e), o = sum(w o) / sum(w), lse = M + ln sum(w).
__device__ void push_segments(const ExchangeParams& p, int64_t dst_off, uint32_t tag) {
  const ShardGeom& g = p.geom;
  const int Y = g.KVH * g.gcs;
  const int* P = g.prefix;
  const int64_t T = (int64_t)P[p.n] * Y;
  const int64_t N = g.ncta;
  const int c4 = p.D / 4;
  const int64_t per_seg = (int64_t)g.GQ * c4;
  const int64_t items = (int64_t)p.n * Y * per_seg;
  const int64_t o_floats = (int64_t)p.n * p.H * p.D;
  for (int64_t it = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; it < items;
       it += (int64_t)gridDim.x * blockDim.x) {
    const int64_t sgi = it / per_seg;
    const int e = (int)(it - sgi * per_seg);
    const int gq = e / c4, d = (e - gq * c4) * 4;
    const int i = (int)(sgi / Y), y = (int)(sgi - (int64_t)i * Y);
    const int kh = y / g.gcs, gc = y - kh * g.gcs;
    const int h = kh * g.G + gc * g.GQ + gq;
    const int64_t oi = ((int64_t)i * p.H + h) * p.D + d;
    const int64_t li = o_floats + (int64_t)h * p.n + i;
    SegSpan sp{0, 0, 0};
    if (P[i + 1] > P[i]) sp = seg_span(P, Y, g.vtiles, N, T, i, y);  // else an empty row, written to send
    if (sp.c0 == sp.c1) {
      put4(p, dst_off + oi, __ldcg(reinterpret_cast<const float4*>(p.send + oi)), tag);
      if (d == 0) put1(p, dst_off + li, __ldcg(p.send + li), tag);
      continue;
    }
    float M = -INFINITY, L = 0.f;
    float O[4] = {0.f, 0.f, 0.f, 0.f};
    if (sp.c1 - sp.c0 < kSpanFast) {
      float l[kSpanFast];
      float4 o[kSpanFast];
      bool on[kSpanFast];
#pragma unroll
      for (int k = 0; k < kSpanFast; ++k) {
        const int64_t cc = sp.c0 + k;
        on[k] = cc <= sp.c1 && seg_nonempty(cc, N, T);
        const int64_t sl = (cc * 2 + (k == 0 ? sp.first_slot : 0)) * g.GQ + gq;
        l[k] = on[k] ? __ldcg(g.part_lse + sl) : -INFINITY;
        o[k] = on[k] ? __ldcg(reinterpret_cast<const float4*>(g.part_o + sl * p.D + d)) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int k = 0; k < kSpanFast; ++k)
        if (on[k]) M = fmaxf(M, l[k]);
#pragma unroll
      for (int k = 0; k < kSpanFast; ++k) {
        if (!on[k]) continue;
        const float w = exp2f((l[k] - M) * kLog2e);
        L += w;
        O[0] = fmaf(w, o[k].x, O[0]);
        O[1] = fmaf(w, o[k].y, O[1]);
        O[2] = fmaf(w, o[k].z, O[2]);
        O[3] = fmaf(w, o[k].w, O[3]);
      }
    } else {
      for (int64_t cc = sp.c0; cc <= sp.c1; ++cc) {
        if (!seg_nonempty(cc, N, T)) continue;
        M = fmaxf(M, __ldcg(g.part_lse + (cc * 2 + (cc == sp.c0 ? sp.first_slot : 0)) * g.GQ + gq));
      }
      for (int64_t cc = sp.c0; cc <= sp.c1; ++cc) {
        if (!seg_nonempty(cc, N, T)) continue;
        const int64_t sl = (cc * 2 + (cc == sp.c0 ? sp.first_slot : 0)) * g.GQ + gq;
        const float w = exp2f((__ldcg(g.part_lse + sl) - M) * kLog2e);
        const float4 ov = __ldcg(reinterpret_cast<const float4*>(g.part_o + sl * p.D + d));
        L += w;
        O[0] = fmaf(w, ov.x, O[0]);
        O[1] = fmaf(w, ov.y, O[1]);
        O[2] = fmaf(w, ov.z, O[2]);
        O[3] = fmaf(w, ov.w, O[3]);
      }
    }
    put4(p, dst_off + oi, make_float4(O[0] / L, O[1] / L, O[2] / L, O[3] / L), tag);
    if (d == 0) put1(p, dst_off + li, M + logf(L), tag);
  }
}

__global__ void __launch_bounds__(kXThreads) fd_exchange_merge_kernel(const __grid_constant__ ExchangeParams p) {
  const int cta = blockIdx.x;
  // this CTA's own step counter (written only by this CTA of the previous
  // launch, which has completed): read before waiting for the decode
  const unsigned long long step = *reinterpret_cast<volatile const unsigned long long*>(p.steps + cta) + 1;
  const uint32_t tag = (uint32_t)step;
  const int par = (int)(step & 1ull);
  griddep_wait();  // the decode's output is complete (programmatic dependent launch)
  // the next step's decode, when launched as a programmatic dependent of this
  // kernel (FD_DECODE_PDL), may start its set-up now; it waits for this grid
  // to complete before writing the partial this kernel pushes
  griddep_launch_dependents();

  // 1. push this rank's share to every rank, each value tagged with the step
  const int64_t dst_off = ((int64_t)par * p.world + p.rank) * p.slot;
  if (p.geom.prefix != nullptr) {
    push_segments(p, dst_off, tag);
  } else {
    const float4* src = reinterpret_cast<const float4*>(p.send);
    const int64_t nvec = p.slot / 4;
    for (int64_t c = (int64_t)cta * blockDim.x + threadIdx.x; c < nvec; c += (int64_t)gridDim.x * blockDim.x)
      put4(p, dst_off + c * 4, __ldcg(src + c), tag);
  }

  // 2. merge (one warp per (row, head) pair): every word the pair needs is
  // requested at once, then the ones not yet carrying this step re-read
  // until they do (bounded)
  const uint32_t* base = p.recv[p.rank] + 2 * (int64_t)par * p.world * p.slot;
  const int64_t o_floats = (int64_t)p.n * p.H * p.D;
  const int lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int64_t pairs = (int64_t)p.n * p.H;
  const uint64_t t0 = globaltimer_ns();
  constexpr int kJ = 4;  // dims per lane per pass: 128 dims a pass
  bool ok = true;
  for (int64_t pr = (int64_t)cta * nw + (threadIdx.x >> 5); ok && pr < pairs; pr += (int64_t)gridDim.x * nw) {
    const int i = (int)(pr / p.H), h = (int)(pr - (int64_t)i * p.H);
    const int64_t lo = o_floats + (int64_t)h * p.n + i;
    const int64_t ob = ((int64_t)i * p.H + h) * p.D;
    // lane q < world: rank q's lse word
    const uint32_t* lw = base + 2 * ((int64_t)(lane < p.world ? lane : 0) * p.slot + lo);
    uint2 l = lane < p.world ? ld_tagged1(lw) : make_uint2(__float_as_uint(-INFINITY), tag);
    float w[FD_MAX_PEERS];
    float inv = 1.f, m = 0.f, tot = 1.f;
    bool all_empty = true;
    for (int d0 = 0; ok && d0 < p.D; d0 += 32 * kJ) {
      uint2 v[FD_MAX_PEERS][kJ];
#pragma unroll
      for (int q = 0; q < FD_MAX_PEERS; ++q)
#pragma unroll
        for (int j = 0; j < kJ; ++j) {
          const int d = d0 + lane + 32 * j;
          v[q][j] = (q < p.world && d < p.D) ? ld_tagged1(base + 2 * ((int64_t)q * p.slot + ob + d)) : make_uint2(0u, tag);
        }
      for (uint32_t it = 1;; ++it) {
        bool mine = l.y == tag;
#pragma unroll
        for (int q = 0; q < FD_MAX_PEERS; ++q)
#pragma unroll
          for (int j = 0; j < kJ; ++j) mine = mine && v[q][j].y == tag;
        if (__all_sync(0xffffffffu, mine)) break;
        // the lanes agree on giving up (a warp-wide vote), so the warp stays converged
        if ((it & 15u) == 0 && __any_sync(0xffffffffu, globaltimer_ns() - t0 > (uint64_t)p.timeout_ns)) {
          ok = false;
          break;
        }
        if (l.y != tag) l = ld_tagged1(lw);
#pragma unroll
        for (int q = 0; q < FD_MAX_PEERS; ++q)
#pragma unroll
          for (int j = 0; j < kJ; ++j)
            if (v[q][j].y != tag) v[q][j] = ld_tagged1(base + 2 * ((int64_t)q * p.slot + ob + d0 + lane + 32 * j));
      }
      if (!ok) break;
      if (d0 == 0) {
        // every lane holds every rank's lse after the shuffles
        const float mine = lse_or_empty(__uint_as_float(l.x));
        float lse_q[FD_MAX_PEERS];
#pragma unroll
        for (int q = 0; q < FD_MAX_PEERS; ++q) lse_q[q] = __shfl_sync(0xffffffffu, mine, q);
        m = -INFINITY;
#pragma unroll
        for (int q = 0; q < FD_MAX_PEERS; ++q)
          if (q < p.world) m = fmaxf(m, lse_q[q]);
        all_empty = (m == -INFINITY);
        if (all_empty) m = 0.f;
        tot = 0.f;
#pragma unroll
        for (int q = 0; q < FD_MAX_PEERS; ++q) {
          w[q] = q < p.world ? expf(lse_q[q] - m) : 0.f;
          if (q < p.world) tot += w[q];
        }
        if (all_empty) tot = 1.f;
        inv = 1.f / tot;
      }
#pragma unroll
      for (int j = 0; j < kJ; ++j) {
        const int d = d0 + lane + 32 * j;
        if (d >= p.D) continue;
        float x = 0.f;
#pragma unroll
        for (int q = 0; q < FD_MAX_PEERS; ++q)
          if (q < p.world) x = fmaf(w[q] * inv, __uint_as_float(v[q][j].x), x);
        store_out(p.out, ob + d, p.out_dtype, x);
      }
    }
    if (!ok) {
      if (lane == 0) set_error(p.err, FD_DEVERR_TIMEOUT);
      break;
    }
    if (lane == 0 && p.out_lse != nullptr) p.out_lse[(int64_t)h * p.n + i] = all_empty ? -INFINITY : m + logf(tot);
  }

  // 3. this CTA's step is done
  __syncthreads();
  if (threadIdx.x == 0) *reinterpret_cast<volatile unsigned long long*>(p.steps + cta) = step;
}

}  // namespace fdk

namespace {
constexpr size_t kStepsOffset = 0;

constexpr size_t kRecvOffset = FD_PEER_RECV_OFFSET;
static_assert(kStepsOffset + 8 * fdk::kXMaxCtas <= kRecvOffset, "step counters overlap the receive slots");
}

extern "C" size_t fd_peer_buffer_bytes(int32_t world, int64_t slot_floats) {
  if (world < 1 || world > FD_MAX_PEERS || slot_floats < 0) return 0;
  const int64_t slot = (slot_floats + 3) / 4 * 4;
  return kRecvOffset + (size_t)2 * (size_t)world * (size_t)slot * 8;  // one 8-byte tagged word per float
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

namespace {

// Validate the exchange arguments and fill the kernel parameters (all but
// the decode geometry).
int exchange_params(const fd_peer_exchange* x, const float* send, int32_t n, int32_t num_heads, int32_t head_size,
                    void* out, int32_t out_dtype, float* out_lse, int32_t num_ctas, int64_t timeout_ns,
                    int32_t* error, const char* what, fdk::ExchangeParams* p, int* ctas) {
  if (x == nullptr || send == nullptr || out == nullptr) return fdh::fail(FD_ERR_INVALID, "%s: null argument", what);
  if (x->world < 1 || x->world > FD_MAX_PEERS || x->rank < 0 || x->rank >= x->world)
    return fdh::fail(FD_ERR_INVALID, "%s: rank %d of world %d (at most %d)", what, x->rank, x->world, FD_MAX_PEERS);
  if (n < 0 || num_heads < 1 || head_size < 1) return fdh::fail(FD_ERR_INVALID, "%s: bad shape", what);
  const int64_t need = (int64_t)n * num_heads * head_size + (int64_t)num_heads * n;
  if (x->slot_floats < need || x->slot_floats % 4 != 0)
    return fdh::fail(FD_ERR_INVALID, "%s: slot of %lld floats, need >= %lld and a multiple of 4", what,
                     (long long)x->slot_floats, (long long)need);
  if (fdh::elem_size(out_dtype) == 0) return fdh::fail(FD_ERR_UNSUPPORTED, "%s: out dtype", what);
  if ((reinterpret_cast<uintptr_t>(send) & 15u) != 0)
    return fdh::fail(FD_ERR_ALIGN, "%s: send buffer not 16-byte aligned", what);
  for (int q = 0; q < x->world; ++q)
    if (x->base[q] == nullptr) return fdh::fail(FD_ERR_INVALID, "%s: rank %d buffer unmapped", what, q);
  *ctas = num_ctas > 0 ? num_ctas : 64;
  if (*ctas > fdk::kXMaxCtas) return fdh::fail(FD_ERR_INVALID, "%s: at most %d CTAs (%d)", what, fdk::kXMaxCtas, *ctas);
  *p = fdk::ExchangeParams{};
  p->send = send;
  unsigned char* own = static_cast<unsigned char*>(x->base[x->rank]);
  for (int q = 0; q < x->world; ++q)
    p->recv[q] = reinterpret_cast<uint32_t*>(static_cast<unsigned char*>(x->base[q]) + kRecvOffset);
  p->steps = reinterpret_cast<unsigned long long*>(own + kStepsOffset);
  p->geom.prefix = nullptr;
  p->rank = x->rank;
  p->world = x->world;
  p->n = n;
  p->H = num_heads;
  p->D = head_size;
  p->slot = x->slot_floats;
  p->out = out;
  p->out_dtype = out_dtype;
  p->out_lse = out_lse;
  p->timeout_ns = timeout_ns > 0 ? timeout_ns : (int64_t)fdk::kWaitLimitNs;
  p->err = error;
  return FD_OK;
}

// Every CTA waits for every other.  A cooperative launch would guarantee
// co-residency but cost ~55 us per step on B200 (measured); at most 64 CTAs
// of 128 threads and no shared memory are resident together (beside decode
// CTAs too), and the bounded wait turns any exception into
// FD_DEVERR_TIMEOUT rather than a hang.  Programmatic dependent launch: the
// CTAs may start while the kernel ahead on the stream finishes and wait for
// it in griddepcontrol.wait.
int launch_exchange(const fdk::ExchangeParams& p, int ctas, void* stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ctas);
  cfg.blockDim = dim3((unsigned)fdk::kXThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return fdh::cuda_status(cudaLaunchKernelEx(&cfg, fdk::fd_exchange_merge_kernel, p), "fd_exchange_merge_kernel launch");
}

}  // namespace

extern "C" int fd_exchange_merge(const fd_peer_exchange* x, const float* send, int32_t n, int32_t num_heads,
                                 int32_t head_size, void* out, int32_t out_dtype, float* out_lse, int32_t num_ctas,
                                 int64_t timeout_ns, int32_t* error, void* stream) {
  fdk::ExchangeParams p;
  int ctas = 0;
  const int st = exchange_params(x, send, n, num_heads, head_size, out, out_dtype, out_lse, num_ctas, timeout_ns,
                                 error, "fd_exchange_merge", &p, &ctas);
  if (st != FD_OK) return st;
  return launch_exchange(p, ctas, stream);
}

namespace {
int decode_exchange(const fd_decode_args* a, const fd_peer_exchange* x, void* out, int32_t out_dtype, float* out_lse,
                    int32_t num_ctas, int64_t timeout_ns, void* stream, bool decode, const char* what) {
  if (a == nullptr) return fdh::fail(FD_ERR_INVALID, "%s: null args", what);
  const int64_t n = a->n, H = a->num_heads, D = a->head_size;
  const float* send = static_cast<const float*>(a->out);
  // the decode's output must be this rank's packed partial: fp32 o [n, H, D]
  // contiguous, then lse [H, n]
  if (a->out_dtype != FD_DTYPE_F32 || a->out_rows != nullptr || a->out_stride_h != D || a->out_stride_n != H * D ||
      a->lse != send + n * H * D || a->lse_stride_h != n || a->lse_stride_n != 1)
    return fdh::fail(FD_ERR_INVALID,
                     "%s: the decode must write fp32 o [n, H, D] and lse [H, n] packed back to back (the "
                     "exchange's send buffer), without out_rows", what);
  if (D % 4 != 0) return fdh::fail(FD_ERR_UNSUPPORTED, "%s: head_size must be a multiple of 4", what);
  fdk::ExchangeParams p;
  int ctas = 0;
  int st = exchange_params(x, send, a->n, a->num_heads, a->head_size, out, out_dtype, out_lse, num_ctas, timeout_ns,
                           a->error, what, &p, &ctas);
  if (st != FD_OK) return st;
  st = fdk::launch_decode_for_exchange(a, stream, &p.geom, decode);
  if (st != FD_OK) return st;
  return launch_exchange(p, ctas, stream);
}
}  // namespace

extern "C" int fd_decode_exchange_merge(const fd_decode_args* a, const fd_peer_exchange* x, void* out,
                                        int32_t out_dtype, float* out_lse, int32_t num_ctas, int64_t timeout_ns,
                                        void* stream) {
  return decode_exchange(a, x, out, out_dtype, out_lse, num_ctas, timeout_ns, stream, true, "fd_decode_exchange_merge");
}

extern "C" int fd_exchange_merge_decoded(const fd_decode_args* a, const fd_peer_exchange* x, void* out,
                                         int32_t out_dtype, float* out_lse, int32_t num_ctas, int64_t timeout_ns,
                                         void* stream) {
  return decode_exchange(a, x, out, out_dtype, out_lse, num_ctas, timeout_ns, stream, false,
                         "fd_exchange_merge_decoded");
}
