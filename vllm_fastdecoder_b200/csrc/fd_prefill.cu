// Causal prefill attention on the 5th-generation tensor cores (tcgen05),
// sm_100a: the P (prefill with cached context) and F (fresh prefill) request
// classes of the split path, which the reference hands to FlashAttention
// (fastdecode/backend.py:317-340, flash_attn_varlen_func with causal=True).
//
// A CTA computes 128 rows of one request for one kv head: 128 / G query
// tokens times the G query heads that share the kv head (row = token * G +
// head), so each K/V tile is loaded once for the whole group:
//   S [128 q x 128 keys] = Q [128 x D] . K^T        (tcgen05, K-major A and B)
//   O [128 q x D]       = P [128 x 128 keys] . V   (tcgen05, P from TMEM, V as MN-major B)
// over the key tiles the causal mask leaves (query i of a request with q_len
// queries and k_len keys sees keys 0 .. k_len - q_len + i: the bottom-right
// alignment of FlashAttention's causal mask).  Six warps:
//   warps 8, 10  TMA producers: warp 8 loads Q once (box {64, 1, 128, 1})
//            and the K tiles of 128 keys into a 3-slot ring, warp 10 the V
//            tiles into their own 3-slot ring (a K slot is free once its
//            q.K^T completed, a V slot once its P.V did), one 16-key box per
//            lane and 64-dim half (128-byte swizzle, the layout the MMA
//            reads); keys come from the paged HBM cache through the block
//            table, or from the batch's own new K/V rows (fresh prefills)
//   warp 9   MMA issuer (one thread): polls both products and issues q.K^T
//            of a tile into one of two TMEM S buffers once its keys landed,
//            P.V of a tile once its P (double-buffered in TMEM) and V are
//            in place; tcgen05.commit to mbarriers
//   warps 0-7  softmax, two warpgroups: warp w owns query rows 32 (w % 4) ..
//            + 31 (TMEM lanes) and keys 64 (w / 4) .. + 63 of each tile; it
//            loads its half of the S row into registers, masks it (tiles
//            below the causal diagonal skip the mask), exchanges the half-
//            row maximum with its partner warp through shared memory, and
//            writes P = 2^(s - m) as 16-bit values packed two per TMEM
//            column, the A operand of P.V (no shared-memory round trip and
//            no proxy fence); O accumulates in TMEM over the
//            tiles, rescaled (each warpgroup its 64 dims) only when the
//            row's maximum moves past its reference m by more than 2^8; at
//            the end o = O / l.
// Numerics: scores fp32 from the exact 16-bit q and K, P rounded to the
// input type for P.V (as FlashAttention does), accumulation fp32.  Every
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
constexpr int kM = 128;                 // query rows per CTA (MMA M)
constexpr int kKT = 128;                // keys per tile (MMA N of S, K of P.V)
constexpr int kSub = 16;                // keys per TMA box
constexpr int kSubs = kKT / kSub;       // boxes per 64-dim half of a tile
constexpr int kPanel = 128 * 128;       // 128 rows x 128 B (64 dims)
constexpr int kTile = 2 * kPanel;       // K or V of one tile / Q (32 KB)
constexpr int kSoftWarps = 8;           // two warpgroups: keys 0-63 and 64-127 of each tile
constexpr int kWarpK = 8, kWarpMma = 9, kWarpV = 10;  // K producer, MMA issuer, V producer
constexpr int kThreads = 11 * 32;
constexpr int kTmemCols = 512;          // S0 [0,128) S1 [128,256) O [256,384) P0, P1 [384,512)

// shared memory: Q | K ring [3] | V ring [3] | barriers | TMEM slot | misc | row reductions
constexpr int kOffQ = 0;
constexpr int kRing = 3;                // slots of the K ring and of the V ring
constexpr int kOffK = kOffQ + kTile;
constexpr int kOffV = kOffK + kRing * kTile;
constexpr int kOffBar = kOffV + kRing * kTile;
constexpr int kNumBars = 1 + 4 * kRing + 2 * 2 + 2 * 2 + 1;  // q_full, k/v full/empty, s_full/empty, p_full/free, drain
constexpr int kTmemP = 3 * kKT;         // P0 [384, 448), P1 [448, 512): 16-bit P packed two per column
constexpr int kOffTmem = kOffBar + kNumBars * 8;
constexpr int kOffMisc = (kOffTmem + 16 + 15) / 16 * 16;  // [0] abort, [1] request, [2] its first tile
constexpr int kOffRed = kOffMisc + 64;                     // [2 halves][128 rows] floats: row maxima, then sums
constexpr int kSmem = kOffRed + 2 * 128 * 4 + 1024;        // + 1024 to align the base
static_assert(kSmem <= 227 * 1024, "smem budget");

struct PrefillParams {
  CUtensorMap tmap_q;   // {D, H, T, 1}, box {64, 1, 128, 1}, swizzled
  CUtensorMap tmap_k;   // paged: {D, KVH, BS, blocks}; contiguous: {D, KVH, T, 1}; box {64, 1, 16, 1}
  CUtensorMap tmap_v;
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
__device__ __forceinline__ void load_kv_tile(const PrefillParams& p, const CUtensorMap* map, unsigned char* dst,
                                             uint64_t* bar, int j, int klen, int qst, int trow, int kh, int lane,
                                             uint64_t pol) {
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
  __syncwarp();
  if (lane == 0) mbar_arrive(bar);
}

// 2^x by the SFU's ex2 instruction (relative error a few ulp of fp32;
// 2^-inf = +0).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Two floats rounded to T and packed (lo, hi) in one conversion; r0, r1 the
// rounded values as floats.
template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b, float& r0, float& r1);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b, float& r0, float& r1) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  const uint32_t u = *reinterpret_cast<const uint32_t*>(&v);
  r0 = __uint_as_float(u << 16);
  r1 = __uint_as_float(u & 0xffff0000u);
  return u;
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b, float& r0, float& r1) {
  const __half2 v = __floats2half2_rn(a, b);
  const float2 f = __half22float2(v);
  r0 = f.x;
  r1 = f.y;
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
  unsigned char* qs = smem + kOffQ;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars;                    // producer lane 0 + the TMA bytes of Q
  uint64_t* k_full = bars + 1;                // [kRing] K tile landed
  uint64_t* k_empty = k_full + kRing;         // [kRing] MMA commit after q.K^T
  uint64_t* v_full = k_empty + kRing;         // [kRing] V tile landed
  uint64_t* v_empty = v_full + kRing;         // [kRing] MMA commit after P.V
  uint64_t* s_full = v_empty + kRing;         // [2] MMA commit: S ready
  uint64_t* s_empty = s_full + 2;             // [2] softmax warps read S
  uint64_t* p_full = s_empty + 2;             // [2] softmax warps wrote P (TMEM)
  uint64_t* p_free = p_full + 2;              // [2] MMA commit after P.V: P buffer free, O up to date
  uint64_t* drain = p_free + 2;               // MMA commit before TMEM release
  static_assert(1 + 4 * kRing + 8 + 1 == kNumBars, "barrier count");
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmem);
  volatile int* misc = reinterpret_cast<volatile int*>(smem + kOffMisc);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int kh = blockIdx.y;    // kv head; rows of the tile are (query token, head of its group) pairs
  const int h0 = kh * p.G;      // first query head of the group
  const int tq = p.tq;          // query tokens per tile (128 / G)
  const int b = blockIdx.x;

  // ---------------------------------------------------------------- setup
  // this CTA's request: the one whose query tiles (ceil(q_len / 128) each,
  // in request order) contain tile b; a running scan over the requests
  if (warp == 0) {
    int carry = 0, found = -1, first = 0;
    for (int base = 0; base < p.n && found < 0; base += 32) {
      const int i = base + lane;
      const int ql = i < p.n ? p.q_len[i] : 0;
      const int c = ql > 0 ? (ql + tq - 1) / tq : 0;
      int v = c;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, v, off);
        if (lane >= off) v += u;
      }
      const int lo = carry + v - c;  // first tile of request i
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
    for (int s = 0; s < kRing; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_empty[s], kSoftWarps);  // one arrival per softmax warp
      mbar_init(&p_full[s], kSoftWarps);
      mbar_init(&p_free[s], 1);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  __syncthreads();
  const int r = misc[1];
  if (r < 0) return;  // spare CTA of the grid's upper bound (before any TMEM is held)
  const int q0 = (b - misc[2]) * tq;
  const int qlen = p.q_len[r];
  const int klen = p.k_len[r];
  const int qst = p.q_start[r];
  const int trow = p.bt_row != nullptr ? p.bt_row[r] : r;
  if (klen < qlen || (p.bt != nullptr && (klen + p.BS - 1) / p.BS > p.bt_width)) {
    if (threadIdx.x == 0) set_error(p.err, FD_DEVERR_LEN);
    return;
  }
  const int i_last = min(q0 + tq, qlen) - 1;         // last query of this tile
  const int nkv = (klen - qlen + i_last) / kKT + 1;  // key tiles the causal mask leaves

  // K and V rings start as zeros: boxes not loaded (keys past k_len) hold
  // finite values, which P = 0 cancels
  for (int o = threadIdx.x * 16; o < 2 * kRing * kTile; o += kThreads * 16)
    sts128(smem + kOffK + o, make_uint4(0u, 0u, 0u, 0u));
  fence_proxy_async_smem();
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
    // warp 8: Q, then K tiles (a K slot is free once its q.K^T completed);
    // warp 10: V tiles (a V slot is free once its P.V completed)
    const bool is_k = warp == kWarpK;
    if (is_k && lane == 0) {
      mbar_expect_tx(q_full, (uint32_t)kTile);
      // box {64 dims, G heads, 128 / G tokens}: row r = token (r / G), head h0 + r % G
      tma_load_4d(qs, &p.tmap_q, 0, h0, qst + q0, 0, q_full, 0ull);
      tma_load_4d(qs + kPanel, &p.tmap_q, 64, h0, qst + q0, 0, q_full, 0ull);
      mbar_arrive(q_full);
    }
    const uint64_t pol = l2_evict_first_policy();
    uint64_t* fullb = is_k ? k_full : v_full;
    uint64_t* emptyb = is_k ? k_empty : v_empty;
    unsigned char* ring = smem + (is_k ? kOffK : kOffV);
    for (int j = 0; j < nkv; ++j) {
      const int st = j % kRing;
      if (j >= kRing && !mbar_wait(&emptyb[st], (uint32_t)((j / kRing) - 1) & 1u, p.err)) {
        misc[0] = 1;
        break;
      }
      if (misc[0]) break;
      load_kv_tile(p, is_k ? &p.tmap_k : &p.tmap_v, ring + st * kTile, &fullb[st], j, klen, qst, trow, kh, lane,
                   pol);
    }
  } else if (warp == kWarpMma) {
    // ------------------------------------------------------------ MMA issuer
    // One thread polls both products and issues whichever is ready: q.K^T of
    // tile kq once K landed and its S buffer is free (at most two ahead),
    // P.V of tile kp once P and V are in shared memory.
    if (lane == 0) {
      bool ok = mbar_wait(q_full, 0u, p.err);
      const uint32_t sq = smem_u32(qs);
      int kq = 0, kp = 0;
      uint32_t spins = 0;
      uint64_t t_idle = 0;
      while (ok && kp < nkv) {
        bool prog = false;
        if (kq < nkv && kq < kp + 2) {
          const int sb = kq & 1, kslot = kq % kRing;
          if (mbar_test_wait(&k_full[kslot], (uint32_t)(kq / kRing) & 1u) &&
              (kq < 2 || mbar_test_wait(&s_empty[sb], (uint32_t)((kq >> 1) - 1) & 1u))) {
            tc_fence_after();
            const uint32_t sk = smem_u32(smem + kOffK + kslot * kTile);
#pragma unroll
            for (int ks = 0; ks < kD / 16; ++ks) {
              const uint32_t off = (ks >> 2) * kPanel + (ks & 3) * 32;
              umma_f16(tmem + sb * kKT, sw128_desc(sq + off, 16, 1024), sw128_desc(sk + off, 16, 1024), kIdQK,
                       ks > 0 ? 1u : 0u);
            }
            umma_commit(&s_full[sb]);
            umma_commit(&k_empty[kslot]);
            ++kq;
            prog = true;
          }
        }
        if (kp < kq) {
          const int pb = kp & 1, vslot = kp % kRing;
          if (mbar_test_wait(&p_full[pb], (uint32_t)(kp >> 1) & 1u) &&
              mbar_test_wait(&v_full[vslot], (uint32_t)(kp / kRing) & 1u)) {
            tc_fence_after();
            const uint32_t sv = smem_u32(smem + kOffV + vslot * kTile);
#pragma unroll
            for (int ks = 0; ks < kKT / 16; ++ks)  // A = P from TMEM: 16 keys = 8 packed columns per step
              umma_f16_ts(tmem + 2 * kKT, tmem + kTmemP + 64 * pb + 8 * ks, sw128_desc(sv + ks * 2048, kPanel, 1024),
                          kIdPV, (kp > 0 || ks > 0) ? 1u : 0u);  // O accumulates over the tiles
            umma_commit(&p_free[pb]);
            umma_commit(&v_empty[vslot]);
            ++kp;
            prog = true;
          }
        }
        if (prog) {
          spins = 0;
          t_idle = 0;
        } else if ((++spins & 255u) == 0u) {
          if (misc[0]) ok = false;
          const uint64_t now = globaltimer_ns();
          if (t_idle == 0) {
            t_idle = now;
          } else if (now - t_idle > kWaitLimitNs) {
            set_error(p.err, FD_DEVERR_TIMEOUT);
            ok = false;
          }
        }
      }
      if (!ok) misc[0] = 1;
      // all MMAs issued by this thread complete before TMEM is released
      umma_commit(drain);
      mbar_wait(drain, 0u, p.err);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax warps 0-7
    // Warp w owns query rows 32 (w % 4) .. + 31 (TMEM lanes) and keys
    // 64 (w / 4) .. + 63 of every tile (its half); the two warps of a row
    // exchange their half-row maxima through shared memory once per tile.
    // O accumulates in TMEM across the tiles (P.V with accumulate); P of a
    // tile is 2^(s - m) for the row's running reference m, which moves only
    // when the tile's maximum exceeds it by more than 2^8 (then the row's O
    // in TMEM, each half its 64 dims, and the sums l are rescaled once), so
    // values of P stay <= 256.
    const int half = warp >> 2;
    const int row = (warp & 3) * 32 + lane;                  // row of the tile = TMEM lane
    const int qi = q0 + row / p.G;                            // its query index within the request
    const int h = h0 + row % p.G;                             // and its query head
    const bool row_ok = qi < qlen;
    const int lim = row_ok ? klen - qlen + qi : -1;          // last key this query sees
    const int lim_all = klen - qlen + q0;                     // keys every query of the tile sees
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t t_o = tmem + lane_base + 2 * kKT + 64 * half;  // this half's 64 dims of O
    float* red = reinterpret_cast<float*>(smem + kOffRed);   // [2 halves][128 rows]
    float m = -INFINITY, l = 0.f;  // m: log2-domain reference of the row; l: this half's sum
    // Every softmax warp runs all nkv iterations and passes both named
    // barriers of each (a warp that failed a wait, or saw another role
    // abort, only skips its work and its waits), so no barrier is ever left
    // waiting for a warp that has gone.
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      if (ok && __any_sync(0xffffffffu, misc[0] != 0)) ok = false;  // warp-uniform (TMEM access is warp-wide)
      const int sb = j & 1;
      if (ok && !__all_sync(0xffffffffu, mbar_wait(&s_full[sb], (uint32_t)(j >> 1) & 1u, p.err))) ok = false;
      uint32_t sr[2][32];  // this half of the S row: two loads, one wait
      float mx = -INFINITY;  // raw score maximum (scale > 0)
      const int kbase = j * kKT + 64 * half;
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 2; ++c) tmem_ld32_nowait(tmem + lane_base + sb * kKT + 64 * half + 32 * c, sr[c]);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_empty[sb]);  // S buffer free for the tile after next
      }
      const bool full_tile = j * kKT + kKT - 1 <= lim_all;  // below the diagonal for every row: no mask
      if (ok) {
        // eight independent partial maxima (short dependency chains)
        float m8[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) m8[k] = -INFINITY;
        if (full_tile) {
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int e = 0; e < 32; ++e) m8[e & 7] = fmaxf(m8[e & 7], __uint_as_float(sr[c][e]));
        } else {
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              const float x = (kbase + 32 * c + e <= lim) ? __uint_as_float(sr[c][e]) : -INFINITY;
              sr[c][e] = __float_as_uint(x);
              m8[e & 7] = fmaxf(m8[e & 7], x);
            }
        }
        mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])), fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
      }
      // the row's maximum over both halves (two barriers: values written,
      // then read, before the next tile overwrites them)
      red[half * 128 + row] = mx;
      named_barrier_sync(1, kSoftWarps * 32);
      mx = fmaxf(mx, red[(1 - half) * 128 + row]);
      named_barrier_sync(1, kSoftWarps * 32);
      if (!ok) continue;
      const float mxs = mx * p.sl2;  // log2 domain
      // P buffer sb is free once the P.V of tile j - 2 completed
      if (j >= 2 && !__all_sync(0xffffffffu, mbar_wait(&p_free[sb], (uint32_t)((j >> 1) - 1) & 1u, p.err))) {
        ok = false;
        continue;
      }
      const bool grow = m != -INFINITY && mxs > m + 8.f;
      if (__any_sync(0xffffffffu, grow)) {
        // O must hold every tile up to j - 1: wait for the P.V of tile j - 1
        // (P.V products complete in order)
        if (!__all_sync(0xffffffffu, mbar_wait(&p_free[(j - 1) & 1], (uint32_t)((j - 1) >> 1) & 1u, p.err))) {
          ok = false;
          continue;
        }
        tc_fence_after();
        const float alpha = grow ? exp2f(m - mxs) : 1.f;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t o[32];
          tmem_ld32_nowait(t_o + 32 * c, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st32(t_o + 32 * c, o);
        }
        tmem_wait_st();
        l *= alpha;
      }
      if (grow || m == -INFINITY) m = mxs;  // the first keys of the row set the reference
      const float neg_m = m == -INFINITY ? 0.f : -m;
      // this half's 64 keys as 32 packed columns of P[sb] in TMEM (column c:
      // keys 2c, 2c + 1 in the low and high halves), the A operand of P.V
      float ls[4] = {0.f, 0.f, 0.f, 0.f};  // four partial sums
      uint32_t pk[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        // 2^(s * scale * log2 e - m) by the hardware ex2 (2^-inf = 0 for masked keys)
        const float p0 = ex2_approx(fmaf(__uint_as_float(sr[c >> 4][(2 * c) & 31]), p.sl2, neg_m));
        const float p1 = ex2_approx(fmaf(__uint_as_float(sr[c >> 4][(2 * c + 1) & 31]), p.sl2, neg_m));
        float r0, r1;
        pk[c] = pack2<T>(p0, p1, r0, r1);  // rounded to T; r0, r1: the values P.V multiplies
        ls[c & 3] += r0 + r1;
      }
      tmem_st32(tmem + lane_base + kTmemP + 64 * sb + 32 * half, pk);
      tmem_wait_st();
      l += (ls[0] + ls[1]) + (ls[2] + ls[3]);
      tc_fence_before();  // TMEM stores of P (and of a rescaled O) before the MMA reads them
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[sb]);
    }
    if (ok && nkv > 0) {
      ok = __all_sync(0xffffffffu, mbar_wait(&p_free[(nkv - 1) & 1], (uint32_t)((nkv - 1) >> 1) & 1u, p.err));
      tc_fence_after();
    }
    // the row's sum over both halves (every softmax warp reaches this barrier)
    red[half * 128 + row] = l;
    named_barrier_sync(1, kSoftWarps * 32);
    l += red[(1 - half) * 128 + row];
    if (!ok) {
      misc[0] = 1;
    } else {
      uint32_t o[2][32];
#pragma unroll
      for (int c = 0; c < 2; ++c) tmem_ld32_nowait(t_o + 32 * c, o[c]);
      tmem_wait_ld();
      if (row_ok) {
        const float inv = l > 0.f ? 1.f / l : 0.f;
        T* orow = reinterpret_cast<T*>(p.out) + (int64_t)(qst + qi) * p.out_st + (int64_t)h * p.out_sh + 64 * half;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint32_t w[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float a0 = __uint_as_float(o[c >> 2][(c & 3) * 8 + 2 * k]) * inv;
            const float a1 = __uint_as_float(o[c >> 2][(c & 3) * 8 + 2 * k + 1]) * inv;
            w[k] = bits16(Dt<T>::narrow(a0)) | (bits16(Dt<T>::narrow(a1)) << 16);
          }
          *reinterpret_cast<uint4*>(orow + 8 * c) = make_uint4(w[0], w[1], w[2], w[3]);
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
  if (!ok) return fdh::fail(FD_ERR_UNSUPPORTED, "fd_prefill_attn: tensor map encoding rejected the q / K / V views");
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

  // grid: an upper bound of the query tiles (sum of ceil(q_len / tq) <=
  // ceil(total_q / tq) + n) by kv heads; spare CTAs return at once
  const int64_t tiles = ((int64_t)a->total_q + tq - 1) / tq + a->n;
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
