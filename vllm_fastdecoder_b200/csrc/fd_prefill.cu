// Causal prefill attention on the 5th-generation tensor cores (tcgen05),
// sm_100a: the P (prefill with cached context) and F (fresh prefill) request
// classes of the split path, which the reference hands to FlashAttention
// (fastdecode/backend.py:317-340, flash_attn_varlen_func with causal=True).
//
// A CTA computes two query tiles A and B of one request for one kv head
// (two consecutive tiles, the longer B last; a tile is 128 rows: 128 / G
// query tokens times the G query heads that share the kv head, row = token
// * G + head), so each K/V tile is loaded once for 256 rows:
//   S [128 q x 128 keys] = Q [128 x D] . K^T        (tcgen05, K-major A and B)
//   O [128 q x D]       = P [128 x 128 keys] . V   (tcgen05, P from TMEM, V as MN-major B)
// over the key tiles the causal mask leaves (query i of a request with q_len
// queries and k_len keys sees keys 0 .. k_len - q_len + i: the bottom-right
// alignment of FlashAttention's causal mask).  Eleven warps:
//   warps 8, 10  TMA producers: warp 8 loads both query tiles once (box
//            {64, G, 128 / G, 1}) and the K tiles of 128 keys into a 3-slot
//            ring, warp 10 the V tiles into a 2-slot ring (a slot is free
//            once the products of its tile completed), one 16-key box per
//            lane and 64-dim half (128-byte swizzle, the layout the MMA
//            reads); keys come from the paged HBM cache through the block
//            table, or from the batch's own new K/V rows (fresh prefills)
//   warp 9   MMA issuer (one thread), in an order that lets one tile's
//            softmax overlap the other tile's products:
//            P.V(A, j), q.K^T(A, j + 1), P.V(B, j), q.K^T(B, j + 1);
//            tcgen05.commit to mbarriers
//   warps 0-7  softmax, warpgroup x for query tile x: one thread per row
//            loads the row's 128 scores of a key tile from TMEM, masks them
//            (tiles below the causal diagonal skip the mask) and writes
//            P = 2^(s - m) as 16-bit values packed two per TMEM column over
//            the first 64 columns of the same S buffer, the A operand of
//            P.V; O accumulates in TMEM over the tiles, rescaled only when
//            the row's maximum moves past its reference m by more than 2^8;
//            at the end o = O / l.
//   TMEM: S/P of A [0,128), S/P of B [128,256), O of A [256,384), O of B [384,512).
// Numerics: scores fp32 from the exact 16-bit q and K, P rounded to the
// input type for P.V and its row sum over the fp32 values (as FlashAttention
// does), accumulation fp32.  Every
// mbarrier wait is bounded (FD_DEVERR_TIMEOUT); TMEM is released on every
// path.

#include <math.h>

#include <algorithm>
#include <type_traits>

#include "fd_common.cuh"
#include "fd_decode.cuh"
#include "fd_internal.h"
#include "fd_tcgen05.cuh"

namespace fdk {
namespace pf {

constexpr int kD = 128;                 // head size
constexpr int kM = 128;                 // rows per query tile (MMA M)
constexpr int kKT = 128;                // keys per tile (MMA N of S, K of P.V)
constexpr int kSub = 16;                // keys per TMA box
constexpr int kSubs = kKT / kSub;       // boxes per 64-dim half of a tile
constexpr int kPanel = 128 * 128;       // 128 rows x 128 B (64 dims)
constexpr int kTile = 2 * kPanel;       // K or V of one tile / one query tile (32 KB)
constexpr int kSoftWarps = 8;           // two warpgroups: query tile A (warps 0-3) and B (warps 4-7)
constexpr int kWarpK = 8, kWarpMma = 9, kWarpV = 10;  // K producer, MMA issuer, V producer
constexpr int kThreads = 11 * 32;
constexpr int kTmemCols = 512;          // S/P A [0,128) S/P B [128,256) O A [256,384) O B [384,512)
constexpr int kRingK = 3;               // slots of the K ring
constexpr int kRingV = 2;               // slots of the V ring (V of a tile is read after its softmax)

// shared memory: Q A | Q B | K ring | V ring | barriers | TMEM slot | misc
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + 2 * kTile;
constexpr int kOffV = kOffK + kRingK * kTile;
constexpr int kOffBar = kOffV + kRingV * kTile;
// q_full, k full/empty, v full/empty, s_full[2], p_full[2], o_full[2], drain
constexpr int kNumBars = 1 + 2 * kRingK + 2 * kRingV + 3 * 2 + 1;
constexpr int kOffTmem = kOffBar + kNumBars * 8;
constexpr int kOffMisc = (kOffTmem + 16 + 15) / 16 * 16;  // [0] abort, [1] request, [2] its first pair
constexpr int kSmem = kOffMisc + 64 + 1024;                // + 1024 to align the base
static_assert(kSmem <= 227 * 1024, "smem budget");

struct PrefillParams {
  CUtensorMap tmap_q;   // {D, H, T, 1}, box {64, 1, 128, 1}, swizzled
  CUtensorMap tmap_k;   // paged: {D, KVH, BS, blocks}; contiguous: {D, KVH, T, 1}; box {64, 1, 16, 1}
  CUtensorMap tmap_v;
  CUtensorMap tmap_o;   // out as tmap_q: {D, H, T, 1}, box {64, G, 128 / G, 1}, swizzled
  void* out;
  int64_t out_st, out_sh;  // elements
  const int32_t* bt;       // null: keys are the batch's own rows (q_start + j)
  int64_t bt_stride;
  int bt_width;
  int64_t nblk;            // blocks of the paged cache (range check)
  const int32_t* q_start;
  const int32_t* q_len;
  const int32_t* k_len;
  const int32_t* bt_row;
  int n, H, G, BS;
  int tq;     // query tokens per tile: 128 / G (the G heads of a kv head share the tile's 128 rows)
  float sl2;  // scale * log2(e)
  int dtype;
  int32_t* err;
};

// One producer warp's share of a key tile: lane l < 8 loads keys
// [128 j + 16 l, +16) of K or V (both 64-dim halves) into `dst`, completion
// as bytes on `bar` (lane 0 arms it with the bytes of the lanes that load).
// With zero_missing, boxes past k_len are written as zeros instead (the warp
// together, before the arrival): P is 0 there, and 0 x V must stay 0.  K
// needs no fill: the causal mask replaces every score past k_len.
__device__ __forceinline__ void load_kv_tile(const PrefillParams& p, const CUtensorMap* map, unsigned char* dst,
                                             uint64_t* bar, int j, int klen, int qst, int trow, int kh, int lane,
                                             uint64_t pol, bool zero_missing) {
  const int t = j * kKT + lane * kSub;
  bool valid = lane < kSubs && t < klen;
  int blk = 0, r0 = 0;
  if (valid) {
    if (p.bt != nullptr) {
      const int64_t id = p.bt[(int64_t)trow * p.bt_stride + t / p.BS];
      r0 = t % p.BS;
      if (id >= 0 && id < p.nblk) {
        blk = (int)id;
      } else {
        set_error(p.err, FD_DEVERR_BLOCK_ID);
        valid = false;
      }
    } else {
      r0 = qst + t;
    }
  }
  const unsigned vmask = __ballot_sync(0xffffffffu, valid);
  if (lane == 0) mbar_expect_tx(bar, (uint32_t)__popc(vmask) * 2u * (kSub * 128u));
  __syncwarp();
  if (valid) {
    tma_load_4d(dst + lane * kSub * 128, map, 0, kh, r0, blk, bar, pol);
    tma_load_4d(dst + kPanel + lane * kSub * 128, map, 64, kh, r0, blk, bar, pol);
  }
  unsigned missing = ~vmask & ((1u << kSubs) - 1u);
  if (zero_missing && missing != 0u) {
    while (missing != 0u) {  // each missing box: 2 x 2 KB, 128 bytes per lane
      const int s = __ffs(missing) - 1;
      missing &= missing - 1u;
      unsigned char* box = dst + s * kSub * 128 + lane * 64;
      sts128(box, make_uint4(0u, 0u, 0u, 0u));
      sts128(box + 16, make_uint4(0u, 0u, 0u, 0u));
      sts128(box + 32, make_uint4(0u, 0u, 0u, 0u));
      sts128(box + 48, make_uint4(0u, 0u, 0u, 0u));
      sts128(box + kPanel, make_uint4(0u, 0u, 0u, 0u));
      sts128(box + kPanel + 16, make_uint4(0u, 0u, 0u, 0u));
      sts128(box + kPanel + 32, make_uint4(0u, 0u, 0u, 0u));
      sts128(box + kPanel + 48, make_uint4(0u, 0u, 0u, 0u));
    }
    fence_proxy_async_smem();  // the zeros before the tensor cores read the slot
  }
  __syncwarp();
  if (lane == 0) mbar_arrive(bar);
}

// Wait for the phase of `bar` with the given parity, giving up when another
// role raised the abort flag or after kWaitLimitNs (FD_DEVERR_TIMEOUT).
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                              int32_t* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        set_error(err, FD_DEVERR_TIMEOUT);
        return false;
      }
    }
  }
}

// The same, polling without suspending (the MMA issuer: a waiting thread
// resumes within a few cycles of the phase completing).
__device__ __forceinline__ bool poll_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                              int32_t* err) {
  if (mbar_test_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_test_wait(bar, parity)) return true;
    if ((it & 255u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        set_error(err, FD_DEVERR_TIMEOUT);
        return false;
      }
    }
  }
}

// Tensor store of a box from shared memory (bulk async group of this thread).
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int c0, int c1, int c2, int c3) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(map),
               "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}

// Named barrier over `count` threads that also ANDs a predicate across them.
__device__ __forceinline__ bool bar_sync_and(int id, int count, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %2, 0;\n\t"
      "bar.red.and.pred p, %1, %3, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(id), "r"((uint32_t)v), "r"(count)
      : "memory");
  return r != 0;
}

// 2^x by the SFU's ex2 instruction (relative error a few ulp of fp32;
// 2^-inf = +0).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// max(a, b, c) in one instruction (the three-input form of sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Two floats rounded to T and packed (lo, hi) in one conversion.
template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  const __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) fd_prefill_kernel(const __grid_constant__ PrefillParams p) {
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kIdQK = instr_desc(kBF16, false, kM, kKT);
  constexpr uint32_t kIdPV = instr_desc(kBF16, false, kM, kD, true);  // V: MN-major B (dims contiguous)
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  unsigned char* smem = smem_raw + ((((raw + 1023u) & ~1023u)) - raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars;               // producer lane 0 + the TMA bytes of the query tiles
  uint64_t* k_full = bars + 1;           // [kRingK] K tile landed
  uint64_t* k_empty = k_full + kRingK;   // [kRingK] MMA commit after the q.K^T products that read it
  uint64_t* v_full = k_empty + kRingK;   // [kRingV] V tile landed
  uint64_t* v_empty = v_full + kRingV;   // [kRingV] MMA commit after the P.V products that read it
  uint64_t* s_full = v_empty + kRingV;   // [2] MMA commit: S of query tile A / B ready
  uint64_t* p_full = s_full + 2;         // [2] the four softmax warps of the tile wrote P
  uint64_t* o_full = p_full + 2;         // [2] MMA commit after the tile's last P.V
  uint64_t* drain = o_full + 2;          // MMA commit before TMEM release
  static_assert(1 + 2 * kRingK + 2 * kRingV + 6 + 1 == kNumBars, "barrier count");
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmem);
  volatile int* misc = reinterpret_cast<volatile int*>(smem + kOffMisc);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int kh = blockIdx.y;    // kv head; rows of a tile are (query token, head of its group) pairs
  const int h0 = kh * p.G;      // first query head of the group
  const int tq = p.tq;          // query tokens per tile (128 / G)
  const int b = blockIdx.x;

  // ---------------------------------------------------------------- setup
  // this CTA's request: the one whose tile pairs (ceil(ceil(q_len / tq) / 2)
  // each, in request order) contain pair b; a running scan over the requests
  if (warp == 0) {
    int carry = 0, found = -1, first = 0;
    for (int base = 0; base < p.n && found < 0; base += 32) {
      const int i = base + lane;
      const int ql = i < p.n ? p.q_len[i] : 0;
      const int c = ql > 0 ? ((ql + tq - 1) / tq + 1) / 2 : 0;
      int v = c;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, v, off);
        if (lane >= off) v += u;
      }
      const int lo = carry + v - c;  // first pair of request i
      const unsigned hit = __ballot_sync(0xffffffffu, i < p.n && c > 0 && lo <= b && b < lo + c);
      if (hit != 0u) {
        const int w = __ffs(hit) - 1;
        found = base + w;
        first = __shfl_sync(0xffffffffu, lo, w);
      }
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
    if (lane == 0) {
      misc[1] = found;
      misc[2] = first;
    }
  }
  if (threadIdx.x == 32) {
    misc[0] = 0;
    mbar_init(q_full, 1);
    for (int s = 0; s < kRingK; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < kRingV; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&p_full[s], kSoftWarps / 2);  // one arrival per warp of the tile's warpgroup
      mbar_init(&o_full[s], 1);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  __syncthreads();
  const int r = misc[1];
  if (r < 0) return;  // spare CTA of the grid's upper bound (before any TMEM is held)
  const int qlen = p.q_len[r];
  const int klen = p.k_len[r];
  const int qst = p.q_start[r];
  const int trow = p.bt_row != nullptr ? p.bt_row[r] : r;
  if (klen < qlen || (p.bt != nullptr && (klen + p.BS - 1) / p.BS > p.bt_width)) {
    if (threadIdx.x == 0) set_error(p.err, FD_DEVERR_LEN);
    return;
  }
  // pair kk of the request holds tiles tB and tA = tB - 1, the last two
  // tiles first (the longest causal rows start first); tA = -1: the
  // request's first tile alone (odd tile count)
  const int kk = b - misc[2];
  const int tB = (qlen + tq - 1) / tq - 1 - 2 * kk;
  const int tA = tB - 1;
  const int q0B = tB * tq, q0A = tA * tq;
  const int nkvB = (klen - qlen + min(q0B + tq, qlen) - 1) / kKT + 1;  // key tiles the causal mask leaves
  const int nkvA = tA >= 0 ? (klen - qlen + q0A + tq - 1) / kKT + 1 : 0;  // <= nkvB (tile A is never last)

  if (warp == kWarpMma) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kWarpK || warp == kWarpV) {
    // ------------------------------------------------------------ producers
    // warp 8: both query tiles, then the K tiles (a K slot is free once the
    // q.K^T products of its tile completed); warp 10: the V tiles (a V slot
    // is free once the P.V products of its tile completed)
    const bool is_k = warp == kWarpK;
    if (is_k && lane == 0) {
      mbar_expect_tx(q_full, (uint32_t)((tA >= 0 ? 2 : 1) * kTile));
      // box {64 dims, G heads, 128 / G tokens}: row r = token (r / G), head h0 + r % G
      if (tA >= 0) {
        tma_load_4d(smem + kOffQ, &p.tmap_q, 0, h0, qst + q0A, 0, q_full, 0ull);
        tma_load_4d(smem + kOffQ + kPanel, &p.tmap_q, 64, h0, qst + q0A, 0, q_full, 0ull);
      }
      tma_load_4d(smem + kOffQ + kTile, &p.tmap_q, 0, h0, qst + q0B, 0, q_full, 0ull);
      tma_load_4d(smem + kOffQ + kTile + kPanel, &p.tmap_q, 64, h0, qst + q0B, 0, q_full, 0ull);
      mbar_arrive(q_full);
    }
    const uint64_t pol = l2_evict_first_policy();
    const int ring_n = is_k ? kRingK : kRingV;
    uint64_t* fullb = is_k ? k_full : v_full;
    uint64_t* emptyb = is_k ? k_empty : v_empty;
    unsigned char* ring = smem + (is_k ? kOffK : kOffV);
    int issued = 0;
    for (int j = 0; j < nkvB; ++j) {
      const int st = j % ring_n;
      const bool free_slot = j < ring_n || wait_or_abort(&emptyb[st], (uint32_t)((j / ring_n) - 1) & 1u, misc, p.err);
      if (!__all_sync(0xffffffffu, free_slot)) {
        misc[0] = 1;
        break;
      }
      if (__any_sync(0xffffffffu, misc[0] != 0)) break;
      load_kv_tile(p, is_k ? &p.tmap_k : &p.tmap_v, ring + st * kTile, &fullb[st], j, klen, qst, trow, kh, lane,
                   pol, !is_k);
      issued = j + 1;
    }
    // no copy of this warp is in flight when the CTA ends: wait (bounded)
    // for the last tile issued into each slot (at once on the normal path,
    // where the MMA issuer waited for every tile)
    for (int st = 0; st < ring_n && st < issued; ++st) {
      const int jl = st + ring_n * ((issued - 1 - st) / ring_n);
      mbar_wait(&fullb[st], (uint32_t)(jl / ring_n) & 1u, p.err);
    }
  } else if (warp == kWarpMma) {
    // ------------------------------------------------------------ MMA issuer
    // One thread, in a fixed order that lets one tile's softmax run while the
    // tensor cores work for the other tile:
    //   q.K^T of tile 0 for A and B; then for each key tile j:
    //   P.V(A, j), q.K^T(A, j + 1), P.V(B, j), q.K^T(B, j + 1).
    // P of a query tile lives in the first 64 columns of its S buffer: the
    // next q.K^T into that buffer is issued after the P.V that reads it
    // (tcgen05.mma operations of one thread execute in order), and the
    // commit of an S also tells its softmax that O holds every earlier tile.
    if (lane == 0) {
      const uint32_t sq0 = smem_u32(smem + kOffQ);
      auto qk = [&](int x, int j) {  // S_x = Q_x . K(j)^T, K-major A and B
        const uint32_t sq = sq0 + x * kTile;
        const uint32_t sk = smem_u32(smem + kOffK + (j % kRingK) * kTile);
#pragma unroll
        for (int ks = 0; ks < kD / 16; ++ks) {
          const uint32_t off = (ks >> 2) * kPanel + (ks & 3) * 32;
          umma_f16(tmem + x * kKT, sw128_desc(sq + off, 16, 1024), sw128_desc(sk + off, 16, 1024), kIdQK,
                   ks > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[x]);
      };
      auto pv = [&](int x, int j) {  // O_x += P_x . V(j), P from TMEM: 16 keys = 8 packed columns per step
        const uint32_t sv = smem_u32(smem + kOffV + (j % kRingV) * kTile);
#pragma unroll
        for (int ks = 0; ks < kKT / 16; ++ks)
          umma_f16_ts(tmem + 2 * kKT + x * kD, tmem + x * kKT + 8 * ks, sw128_desc(sv + ks * 2048, kPanel, 1024),
                      kIdPV, (j > 0 || ks > 0) ? 1u : 0u);
      };
      bool ok = poll_or_abort(q_full, 0u, misc, p.err) && poll_or_abort(&k_full[0], 0u, misc, p.err);
      if (ok) {
        tc_fence_after();
        if (nkvA > 0) qk(0, 0);
        qk(1, 0);
        umma_commit(&k_empty[0]);
      }
      for (int j = 0; ok && j < nkvB; ++j) {
        for (int x = 0; x < 2; ++x) {
          const int nk = x ? nkvB : nkvA;
          if (j >= nk) continue;
          // the first of the tile's users waits for V(j) (A, when it still runs)
          if (!poll_or_abort(&p_full[x], (uint32_t)j & 1u, misc, p.err) ||
              ((x == 0 || j >= nkvA) &&
               !poll_or_abort(&v_full[j % kRingV], (uint32_t)(j / kRingV) & 1u, misc, p.err))) {
            ok = false;
            break;
          }
          tc_fence_after();
          pv(x, j);
          if (j == nk - 1) umma_commit(&o_full[x]);
          if (j + 1 < nk) {
            const int t = j + 1;
            if ((x == 0 || t >= nkvA) &&
                !poll_or_abort(&k_full[t % kRingK], (uint32_t)(t / kRingK) & 1u, misc, p.err)) {
              ok = false;
              break;
            }
            tc_fence_after();
            qk(x, t);
            if (x == 1) umma_commit(&k_empty[t % kRingK]);  // B reads every K tile last
          }
        }
        if (ok) umma_commit(&v_empty[j % kRingV]);
      }
      if (!ok) misc[0] = 1;
      // all MMAs issued by this thread complete before TMEM is released
      umma_commit(drain);
      mbar_wait(drain, 0u, p.err);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax warps 0-7
    // Warpgroup x (warps 4x .. 4x + 3) owns query tile x (0: A, 1: B); warp
    // w of it owns rows 32 (w % 4) .. + 31 (TMEM lanes), one row per thread
    // with all 128 keys of each key tile, so no row statistics cross warps.
    // O accumulates in TMEM across the tiles (P.V with accumulate); P of a
    // tile is 2^(s - m) for the row's running reference m, which moves only
    // when the tile's maximum exceeds it by more than 2^8 (then the row's O
    // in TMEM and the sum l are rescaled once), so values of P stay <= 256.
    const int x = warp >> 2;
    const int nkv = x ? nkvB : nkvA;
    const int q0 = x ? q0B : q0A;
    const int row = (warp & 3) * 32 + lane;                  // row of the tile = TMEM lane
    const int qi = q0 + row / p.G;                            // its query index within the request
    const bool row_ok = qi < qlen;
    const int lim = row_ok ? klen - qlen + qi : -1;          // last key this query sees
    const int lim_all = klen - qlen + q0;                     // keys every query of the tile sees
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t t_s = tmem + lane_base + x * kKT;          // S of the tile, then P in columns 0 .. 63
    const uint32_t t_o = tmem + lane_base + 2 * kKT + x * kD; // O of the tile
    float m = -INFINITY, l = 0.f;  // m: log2-domain reference of the row; l: its sum
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      if (!__all_sync(0xffffffffu, wait_or_abort(&s_full[x], (uint32_t)j & 1u, misc, p.err))) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sr[4][32];  // the S row: four loads, one wait
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32_nowait(t_s + 32 * c, sr[c]);
      tmem_wait_ld();
      // the causal mask (skipped below the diagonal of every row), then the
      // row maximum
      float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      if (j * kKT + kKT - 1 > lim_all) {
        const int nv = lim - j * kKT + 1;  // keys of the tile this row sees (may be <= 0 or >= 128)
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (32 * c + e >= nv) sr[c][e] = __float_as_uint(-INFINITY);
      }
      // four independent chains of three-input maxima (two scores each)
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int e = 0; e < 32; e += 2)
          m4[(e >> 1) & 3] = fmax3(m4[(e >> 1) & 3], __uint_as_float(sr[c][e]), __uint_as_float(sr[c][e + 1]));
      const float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      const float mxs = mx * p.sl2;  // log2 domain (scale > 0)
      const bool grow = m != -INFINITY && mxs > m + 8.f;
      if (__any_sync(0xffffffffu, grow)) {
        // O holds tiles 0 .. j - 1: their P.V were issued before this S's commit
        const float alpha = grow ? exp2f(m - mxs) : 1.f;
#pragma unroll 1
        for (int c = 0; c < kD / 16; ++c) {
          uint32_t o[16];
          tmem_ld16_nowait(t_o + 16 * c, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st16(t_o + 16 * c, o);
        }
        l *= alpha;
      }
      if (grow || m == -INFINITY) m = mxs;  // the first keys of the row set the reference
      const float neg_m = m == -INFINITY ? 0.f : -m;
      // P as 64 packed columns (column c: keys 2c, 2c + 1 in the low and high
      // halves) over columns 0 .. 63 of the S buffer: the A operand of P.V
      // the row sum l adds the fp32 values of P, as FlashAttention's does;
      // P.V multiplies them rounded to T
      const f2_t sl2x2 = f2_pack(p.sl2, p.sl2), nm2 = f2_pack(neg_m, neg_m);
      f2_t ls[2] = {f2_pack(0.f, 0.f), f2_pack(0.f, 0.f)};  // packed partial sums
#pragma unroll
      for (int q = 0; q < 4; ++q) {  // keys 32 q .. 32 q + 31: packed columns 16 q .. 16 q + 15
        uint32_t pk[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          // 2^(s * scale * log2 e - m) by the hardware ex2 (2^-inf = 0 for masked keys)
          float a0, a1;
          f2_unpack(f2_fma(f2_pack(__uint_as_float(sr[q][2 * c]), __uint_as_float(sr[q][2 * c + 1])), sl2x2, nm2), a0,
                    a1);
          const float p0 = ex2_approx(a0), p1 = ex2_approx(a1);
          pk[c] = pack2<T>(p0, p1);
          ls[c & 1] = f2_add(ls[c & 1], f2_pack(p0, p1));
        }
        tmem_st16(t_s + 16 * q, pk);
      }
      tmem_wait_st();
      {
        float a0, a1, b0, b1;
        f2_unpack(ls[0], a0, a1);
        f2_unpack(ls[1], b0, b1);
        l += (a0 + a1) + (b0 + b1);
      }
      tc_fence_before();  // TMEM stores of P (and of a rescaled O) before the MMA reads them
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[x]);
    }
    if (ok && nkv > 0) {
      ok = __all_sync(0xffffffffu, wait_or_abort(&o_full[x], 0u, misc, p.err));
      tc_fence_after();
    }
    // o = O / l, staged in the tile's Q buffer (its last q.K^T completed
    // before this tile's last S) in the layout of the Q box: two 64-dim
    // panels of 128-byte rows, 128-byte swizzle; then one tensor store of
    // the tile, or (the request's last tile, whose box would reach into the
    // next request) plain stores of the rows that belong to the request.
    // All four warps of the warpgroup reach the barrier on every path.
    unsigned char* stage = smem + kOffQ + x * kTile;
    const bool fine = ok && nkv > 0;
    if (fine) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
      for (int c = 0; c < kD / 32; ++c) {
        uint32_t o[32];
        tmem_ld32_nowait(t_o + 32 * c, o);
        tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t w[4];
#pragma unroll
          for (int k = 0; k < 4; ++k)
            w[k] = pack2<T>(__uint_as_float(o[8 * q + 2 * k]) * inv, __uint_as_float(o[8 * q + 2 * k + 1]) * inv);
          sts128(stage + (c >> 1) * kPanel + swz(row, (c & 1) * 4 + q), make_uint4(w[0], w[1], w[2], w[3]));
        }
      }
      fence_proxy_async_smem();  // the staged rows before the tensor store reads them
    }
    if (!ok) misc[0] = 1;
    if (bar_sync_and(1 + x, kSoftWarps / 2 * 32, fine)) {
      if (q0 + tq <= qlen) {
        if ((warp & 3) == 0 && lane == 0) {
          tma_store_4d(&p.tmap_o, stage, 0, h0, qst + q0, 0);
          tma_store_4d(&p.tmap_o, stage + kPanel, 64, h0, qst + q0, 0);
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");
          asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");  // smem read before the CTA ends
        }
      } else {
        const int ch = lane & 15;
#pragma unroll 4
        for (int i = 0; i < 16; ++i) {  // this warp's rows, two per instruction
          const int rr = (warp & 3) * 32 + 2 * i + (lane >> 4);
          const int qr = q0 + rr / p.G;
          const uint4 v = lds128(stage + (ch >> 3) * kPanel + swz(rr, ch & 7));
          if (qr < qlen)
            *reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.out) + (int64_t)(qst + qr) * p.out_st +
                                      (int64_t)(h0 + rr % p.G) * p.out_sh + 8 * ch) = v;
        }
      }
    }
  }

  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kWarpMma)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

}  // namespace pf
}  // namespace fdk

extern "C" int fd_prefill_attn(const fd_prefill_args* a, void* stream) {
  using fdk::pf::PrefillParams;
  if (a == nullptr) return fdh::fail(FD_ERR_INVALID, "fd_prefill_attn: null args");
  if (a->n < 0 || a->n > 65535)
    return fdh::fail(FD_ERR_UNSUPPORTED, "fd_prefill_attn: %d requests (at most 65535)", a->n);
  if (a->n == 0 || a->total_q <= 0) return FD_OK;
  if (a->dtype != FD_DTYPE_F16 && a->dtype != FD_DTYPE_BF16)
    return fdh::fail(FD_ERR_UNSUPPORTED, "fd_prefill_attn: q/K/V must be fp16 or bf16");
  if (a->head_size != fdk::pf::kD) return fdh::fail(FD_ERR_UNSUPPORTED, "fd_prefill_attn: head_size must be 128");
  if (a->num_kv_heads <= 0 || a->num_heads <= 0 || a->num_heads % a->num_kv_heads != 0)
    return fdh::fail(FD_ERR_INVALID, "fd_prefill_attn: num_heads must be a multiple of num_kv_heads");
  if (a->num_heads > 65535) return fdh::fail(FD_ERR_UNSUPPORTED, "fd_prefill_attn: too many heads");
  if (a->q == nullptr || a->out == nullptr || a->kv.k == nullptr || a->kv.v == nullptr || a->q_start == nullptr ||
      a->q_len == nullptr || a->k_len == nullptr)
    return fdh::fail(FD_ERR_INVALID, "fd_prefill_attn: q, out, K/V and the per-request arrays are required");
  if (a->kv.host_mapped) return fdh::fail(FD_ERR_UNSUPPORTED, "fd_prefill_attn: K/V must be device memory");
  if (a->num_tokens <= 0) return fdh::fail(FD_ERR_INVALID, "fd_prefill_attn: num_tokens must be positive");
  const int es = 2;
  const int64_t D = a->head_size;
  if (!fdh::aligned16(a->q) || !fdh::aligned16(a->out) || (a->q_stride_t * es) % 16 != 0 ||
      (a->q_stride_h * es) % 16 != 0 || (a->out_stride_t * es) % 16 != 0 || (a->out_stride_h * es) % 16 != 0)
    return fdh::fail(FD_ERR_ALIGN, "fd_prefill_attn: q / out pointers and strides must be 16-byte aligned");
  const fd_kv_tier& kv = a->kv;
  if (!fdh::aligned16(kv.k) || !fdh::aligned16(kv.v) || (kv.head_stride * es) % 16 != 0 ||
      (kv.tok_stride * es) % 16 != 0 || (kv.blk_stride * es) % 16 != 0)
    return fdh::fail(FD_ERR_ALIGN, "fd_prefill_attn: K/V pointers and strides must be 16-byte aligned");
  const bool paged = a->block_table != nullptr;
  if (paged && (a->block_size <= 0 || a->block_size % fdk::pf::kSub != 0 || a->bt_width <= 0 || kv.num_blocks <= 0))
    return fdh::fail(FD_ERR_UNSUPPORTED, "fd_prefill_attn: paged K/V needs a block size that is a multiple of 16");
  if (!paged && kv.num_blocks <= 0)
    return fdh::fail(FD_ERR_INVALID, "fd_prefill_attn: contiguous K/V needs num_blocks = rows of k / v");

  PrefillParams p{};
  const int H = a->num_heads, KVH = a->num_kv_heads;
  const int G = H / KVH;
  if (G > 16 || fdk::pf::kM % G != 0)
    return fdh::fail(FD_ERR_UNSUPPORTED, "fd_prefill_attn: query group %d must divide 128 (at most 16)", G);
  const int tq = fdk::pf::kM / G;
  // q as {D, H, tokens, 1} with a box of the G heads of a kv head x 128 / G queries
  bool ok = fdk::encode_kv_map(&p.tmap_q, a->q, a->dtype, (int)D, H, a->num_tokens, 1, a->q_stride_h * es,
                               a->q_stride_t * es, a->q_stride_t * es * a->num_tokens, tq, true, G);
  if (paged) {
    ok = ok && fdk::encode_kv_map(&p.tmap_k, kv.k, a->dtype, (int)D, KVH, a->block_size, kv.num_blocks,
                                  kv.head_stride * es, kv.tok_stride * es, kv.blk_stride * es, fdk::pf::kSub, true);
    ok = ok && fdk::encode_kv_map(&p.tmap_v, kv.v, a->dtype, (int)D, KVH, a->block_size, kv.num_blocks,
                                  kv.head_stride * es, kv.tok_stride * es, kv.blk_stride * es, fdk::pf::kSub, true);
  } else {
    // the batch's own K/V rows [tokens, KVH, D] as one block of num_blocks tokens
    const int64_t T = kv.num_blocks;
    ok = ok && fdk::encode_kv_map(&p.tmap_k, kv.k, a->dtype, (int)D, KVH, (int)T, 1, kv.head_stride * es,
                                  kv.tok_stride * es, kv.tok_stride * es * T, fdk::pf::kSub, true);
    ok = ok && fdk::encode_kv_map(&p.tmap_v, kv.v, a->dtype, (int)D, KVH, (int)T, 1, kv.head_stride * es,
                                  kv.tok_stride * es, kv.tok_stride * es * T, fdk::pf::kSub, true);
  }
  // out as q: tile stores of full query tiles
  ok = ok && fdk::encode_kv_map(&p.tmap_o, a->out, a->dtype, (int)D, H, a->num_tokens, 1, a->out_stride_h * es,
                                a->out_stride_t * es, a->out_stride_t * es * a->num_tokens, tq, true, G);
  if (!ok)
    return fdh::fail(FD_ERR_UNSUPPORTED, "fd_prefill_attn: tensor map encoding rejected the q / K / V / out views");
  p.out = a->out;
  p.out_st = a->out_stride_t;
  p.out_sh = a->out_stride_h;
  p.bt = a->block_table;
  p.bt_stride = a->bt_stride;
  p.bt_width = a->bt_width;
  p.nblk = kv.num_blocks;
  p.q_start = a->q_start;
  p.q_len = a->q_len;
  p.k_len = a->k_len;
  p.bt_row = a->bt_row;
  p.n = a->n;
  p.H = H;
  p.G = G;
  p.tq = tq;
  p.BS = paged ? a->block_size : 1;
  p.sl2 = a->scale * fdk::kLog2e;
  p.dtype = a->dtype;
  p.err = a->error;

  // grid: an upper bound of the tile pairs (a request's ceil(ceil(q_len /
  // tq) / 2) <= q_len / (2 tq) + 1, summed) by kv heads; spare CTAs return
  // at once
  const int64_t tiles = ((int64_t)a->total_q + 2 * tq - 1) / (2 * tq) + a->n;
  if (tiles > 0x7fffffff) return fdh::fail(FD_ERR_UNSUPPORTED, "fd_prefill_attn: too many query tiles");
  const void* kern = a->dtype == FD_DTYPE_BF16 ? reinterpret_cast<const void*>(fdk::pf::fd_prefill_kernel<__nv_bfloat16>)
                                               : reinterpret_cast<const void*>(fdk::pf::fd_prefill_kernel<__half>);
  static unsigned long long done_h = 0, done_b = 0;
  int st = fdh::ensure_smem(kern, fdk::pf::kSmem, a->dtype == FD_DTYPE_BF16 ? &done_b : &done_h);
  if (st != FD_OK) return st;
  return fdh::launch_maybe_pdl(kern, dim3((unsigned)tiles, (unsigned)KVH), dim3(fdk::pf::kThreads), fdk::pf::kSmem,
                               static_cast<cudaStream_t>(stream), false, p, "fd_prefill_kernel launch");
}

extern "C" size_t fd_prefill_args_bytes(void) { return sizeof(fd_prefill_args); }
