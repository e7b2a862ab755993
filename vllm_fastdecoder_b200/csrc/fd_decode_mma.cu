// Paged GQA decode on the 5th-generation tensor cores (tcgen05), sm_100a.
//
// For a kv head with a query group of G <= 8 heads the two products of
// decode attention are small matrix products per 128-token stage:
//   S^T [128 tokens x 8] = K [128 x 128] . q^T [128 x 8]       (q.K^T)
//   O^T [128 dims  x 8] = V^T [128 x 128] . P^T [128 x 8]      (P.V)
// (the group padded to the MMA's N = 16).  One CTA per SM, nine warps:
//   warps 4, 6-8  TMA producers: K and V tiles (16 tokens, one kv head) into
//            a 3-stage ring in the 128-byte-swizzled layout the MMA reads
//            (tiled TMA, box {64 dims, 1, 16, 1}), two tiles of a stage
//            each (a warp issues its TMA boxes one after another, ~45 ns
//            apiece, so the 32 boxes of a 64 KB stage are spread over four
//            warps); host-tier tiles by 16-byte loads stored with the same
//            swizzle; warp 4 also stages q of each piece.  Block ids are
//            fetched six stages ahead (cp.async ring).
//   warp 5   MMA issuer: one thread polls the barriers and issues
//            tcgen05.mma into TMEM (S and O double-buffered, 64 columns) for
//            whichever product is ready, q.K^T up to two stages ahead of
//            P.V; tcgen05.commit to mbarriers
//   warps 0-3  softmax: thread r owns token row r of S (TMEM lane r): scale,
//            mask, block max (per stage, butterfly over the group), exp2, P
//            written as 16-bit pairs into the swizzled B operand; then thread
//            d owns dim d of O (TMEM lane d) and folds the PREVIOUS stage's O
//            into an fp32 accumulator with the online-softmax rescale, so a
//            stage's P.V round trip overlaps the next stage's softmax.
//            Per-thread partial sums of p give the denominator.
// The schedule is the persistent one of fd_decode.cu (equal tile ranges per
// CTA, pieces, two partial slots per CTA, fd_persistent_combine_kernel).
// Numerics: scores and softmax in fp32 from the exact 16-bit q and K; P
// enters the P.V product as a sum of two 16-bit values (hi in rows 0..G-1,
// lo in rows G..2G-1 of the N = 16 operand), so P.V keeps nearly fp32
// precision;
// all accumulation fp32.

#include <math.h>

#include <algorithm>
#include <type_traits>

#include "fd_common.cuh"
#include "fd_decode.cuh"
#include "fd_internal.h"
#include "fd_tcgen05.cuh"

#ifndef FD_MMA_PRODUCERS
#define FD_MMA_PRODUCERS 4  // producer warps of the tcgen05 kernel
#endif

namespace fdk {
namespace mma {

constexpr int kD = 128;             // head size handled here
constexpr int kN = 16;              // query heads of a kv head, padded (MMA N; M=128 takes N%16)
constexpr int kTok = 128;           // tokens per stage (MMA M of q.K^T)
constexpr int kTT = 16;             // tokens per tile
constexpr int kTilesPerStage = kTok / kTT;
constexpr int kNST = 3;             // stages in the ring
constexpr int kPanel = kTok * 128;  // 128 token rows x 128 B (64 dims)
constexpr int kKV = 2 * kPanel;     // K or V of one stage (32 KB)
constexpr int kStage = 2 * kKV;     // K + V (64 KB)
static_assert(kTilesPerStage % FD_MMA_PRODUCERS == 0, "tiles split evenly between the producer warps");
constexpr int kQB = 2 * kN * 128;   // q: two panels of 16 rows x 128 B
constexpr int kPB = 2 * kN * 128;   // P: two panels (tokens 0-63, 64-127) x 16 rows
constexpr int kProd = FD_MMA_PRODUCERS;          // producer warps (4, then 6, 7, ...), kTilesPerProd tiles each
constexpr int kTilesPerProd = kTilesPerStage / kProd;
constexpr int kThreads = (4 + 1 + kProd) * 32;
constexpr int kTmemCols = 4 * kN;  // S0 S1 O0 O1, kN columns each

constexpr int kOffQ = kNST * kStage;
constexpr int kOffP = kOffQ + 2 * kQB;
constexpr int kOffRed = kOffP + 2 * kPB;         // [2][4 warps][kN] floats: per-stage maxima
constexpr int kOffL = kOffRed + 2 * 4 * kN * 4;  // [4 warps][kN] floats: per-piece sums
constexpr int kOffBar = kOffL + 4 * kN * 4;
constexpr int kNumBars = 3 + 3 + 2 * 7 + 1 + 2 + 1;
constexpr int kOffTmem = kOffBar + kNumBars * 8;
constexpr int kOffIds = (kOffTmem + 16 + 127) / 128 * 128;  // producer's block-id ring
constexpr int kOffPrefix = kOffIds + kProd * kIdRingBytes;
constexpr int kSmemFixed = kOffPrefix + 1024;  // + 1024 for aligning the base
// the tile prefix [n + 1], the lengths [n] and the block-table rows [n]
// follow, 16-byte aligned each
constexpr int kRowsBytes = (kMaxPersistentRows + 1 + 3) / 4 * 16;
static_assert(kSmemFixed + 3 * kRowsBytes <= 227 * 1024, "smem budget");


// One stage as the producer sees it, fetched one stage ahead.
struct ProdStage {
  Piece pc;
  int st0, st1, qi;
  bool pf;
};

template <typename T, int GM>
__global__ void __launch_bounds__(kThreads, 1) fd_decode_mma_kernel(const __grid_constant__ DecodeParams p) {
  static_assert(GM >= 2 && 2 * GM <= kN && (GM * 16) % 32 == 0, "query group (hi and lo rows of P) must fit the MMA N");
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kIdQK = instr_desc(kBF16, false, kTok, kN);
  constexpr uint32_t kIdPV = instr_desc(kBF16, true, kD, kN);
  constexpr int G = GM;
  constexpr int kQV = G * 16 / 32;  // 16-byte chunks of a piece's q per producer lane
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  unsigned char* smem = smem_raw + ((((raw + 1023u) & ~1023u)) - raw);
  unsigned char* stages = smem;
  unsigned char* qbuf = smem + kOffQ;
  unsigned char* pbuf = smem + kOffP;
  float* red = reinterpret_cast<float*>(smem + kOffRed);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* full = bars;          // [3] TMA bytes + 32 lanes of each producer warp
  uint64_t* empty = bars + 3;     // [3] MMA commit: stage consumed
  uint64_t* s_full = bars + 6;    // [2] MMA commit: S ready
  uint64_t* s_empty = bars + 8;   // [2] 4 softmax warps read S
  uint64_t* p_full = bars + 10;   // [2] 4 softmax warps wrote P
  uint64_t* o_full = bars + 12;   // [2] MMA commit: O ready
  uint64_t* o_empty = bars + 14;  // [2] 4 softmax warps read O
  uint64_t* q_full = bars + 16;   // [2] 32 producer lanes wrote q
  uint64_t* q_empty = bars + 18;  // [2] MMA commit: q.K^T of the piece done
  uint64_t* drain = bars + 20;    // [1] MMA commit before TMEM release
  uint64_t* red_full = bars + 21; // [2] 4 softmax warps wrote their stage maxima
  uint64_t* l_full = bars + 23;   // [1] 4 softmax warps wrote their piece sums
  float* lsum = reinterpret_cast<float*>(smem + kOffL);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmem);
  int* prefix = reinterpret_cast<int*>(smem + kOffPrefix);  // [n + 1] tile prefix
  int* lens_s = prefix + ((p.n + 4) & ~3);                   // [n] lengths
  int* trow_s = lens_s + ((p.n + 4) & ~3);                   // [n] block-table rows (bt_rows)
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int Y = p.KVH;

  // ---------------------------------------------------------------- setup
  // lengths and table rows into shared memory by every thread (independent
  // loads: one memory round trip), then warp 0 scans them
  warm_block_table(p);
  for (int i = threadIdx.x; i < p.n; i += kThreads) {
    lens_s[i] = p.lens[i];
    trow_s[i] = p.bt_rows != nullptr ? p.bt_rows[i] : i;
  }
  // q and P buffers start zeroed: the padding rows stay zero
  for (int o = threadIdx.x * 16; o < 2 * kQB + 2 * kPB; o += kThreads * 16)
    sts128(qbuf + o, make_uint4(0u, 0u, 0u, 0u));
  fence_proxy_async_smem();
  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < 3; ++s) {
      mbar_init(&full[s], 32 * kProd);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_empty[b], 4);
      mbar_init(&p_full[b], 4);
      mbar_init(&o_full[b], 1);
      mbar_init(&o_empty[b], 4);
      mbar_init(&q_full[b], 32);
      mbar_init(&q_empty[b], 1);
    }
    mbar_init(drain, 1);
    mbar_init(&red_full[0], 4);
    mbar_init(&red_full[1], 4);
    mbar_init(l_full, 4);
    fence_barrier_init();
  }
  if (warp == 5) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  __syncthreads();
  if (warp == 0) {
    int carry = 0;
    for (int base = 0; base < p.n; base += 32) {
      const int i = base + lane;
      int nt = 0;
      if (i < p.n) {
        const int len = lens_s[i];
        if (len > 0 && (len + p.BS - 1) / p.BS <= p.bt_width) nt = (len + kTT - 1) / kTT + p.vtiles;
      }
      int v = nt;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, v, off);
        if (lane >= off) v += u;
      }
      if (i < p.n) prefix[i + 1] = carry + v;
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
    if (lane == 0) prefix[0] = 0;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Programmatic dependent launch (fd_decode_args.flags & FD_DECODE_PDL): the
  // setup above and the producers' block-id and q prefetch below only read
  // inputs the caller guarantees the kernel ahead on the stream does not
  // write; the producers pass griddep_wait() before their first K/V read and
  // the softmax warps before their first global write (a no-op for an
  // ordinary launch; the MMA warp touches no global memory).
  const int64_t total = (int64_t)prefix[p.n] * Y;
  const int64_t g0 = (int64_t)blockIdx.x * total / gridDim.x;
  const int64_t g1 = (int64_t)(blockIdx.x + 1) * total / gridDim.x;
  int row0 = 0;
  if (g0 < g1) {
    int lo = 0, hi = p.n - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if ((int64_t)prefix[mid] * Y <= g0) lo = mid; else hi = mid - 1;
    }
    row0 = lo;
  }

  if (warp == 4 || warp >= 6) {
    // ------------------------------------------------------------ producers
    // Producer pw (warp 4, then warps 6, 7, ...) fills tiles
    // [pw * kTilesPerProd, (pw + 1) * kTilesPerProd) of every stage: one
    // warp issues its TMA boxes one after another (~45 ns each), so the
    // warps share a stage's issue time.  Block ids come kIdAhead stages ahead
    // through a cp.async ring per warp (q of the coming pieces is prefetched
    // into L2 there); warp 4 also loads q into registers one stage ahead of
    // its piece and stores it for the MMA.
    const int pw = warp == 4 ? 0 : warp - 5;
    const bool q_owner = pw == 0;
    const uint64_t pol = l2_evict_first_policy();
    StageIter it;
    it.init(g0, g1, row0, prefix, lens_s, p.n, Y, kTilesPerStage, p.vtiles);
    IdPrefetch ids;
    ids.it.init(g0, g1, row0, prefix, nullptr, p.n, Y, kTilesPerStage, p.vtiles);
    ids.it.trows = trow_s;
    ids.ring = reinterpret_cast<int*>(smem + kOffIds + pw * kIdRingBytes);
    ids.issued = 0;
    const int q_heads = q_owner ? G : 0;
    for (int i = 0; i < kIdAhead; ++i) ids.push(p, lane, q_heads, kD * (int)sizeof(T), pw * kTilesPerProd, kTilesPerProd);
    ProdStage cur, nxt;
    uint4 q_c[kQV], q_n[kQV];
    auto advance = [&](ProdStage& s) -> bool {
      bool pl;
      if (!it.next(s.st0, s.st1, s.pf, pl)) return false;
      s.pc = it.pc;
      s.qi = it.pieces - 1;
      return true;
    };
    auto fetch = [&](const ProdStage& s, uint4 (&qr)[kQV]) {
      if (q_owner && s.pf) {
        const int64_t qrow = p.q_rows ? p.q_rows[s.pc.row] : s.pc.row;
        const unsigned char* qsrc = p.q + qrow * p.q_sn + (int64_t)(s.pc.y * G) * p.q_sh;
#pragma unroll
        for (int u = 0; u < kQV; ++u) {
          const int c = u * 32 + lane;
          qr[u] = __ldg(reinterpret_cast<const uint4*>(qsrc + (c >> 4) * p.q_sh + (c & 15) * 16));
        }
      }
    };
    int k = 0;
    bool aborted = false;
    bool have = advance(cur);
    if (have) fetch(cur, q_c);
    griddep_wait();  // K/V below may be written by the kernel ahead (the KV write)
    while (have) {
      const bool have_n = advance(nxt);
      if (have_n) fetch(nxt, q_n);
      ids.push(p, lane, q_heads, kD * (int)sizeof(T), pw * kTilesPerProd, kTilesPerProd);  // stage k + kIdAhead
      const int64_t id_c = ids.take(k, lane);
      const int kh = cur.pc.y;
      if (q_owner && cur.pf) {
        // q of this piece into q buffer qi % 2
        const int qb = cur.qi & 1;
        if (cur.qi >= 2 && !mbar_wait(&q_empty[qb], ((cur.qi >> 1) - 1) & 1u, p.err)) {
          aborted = true;
          break;
        }
#pragma unroll
        for (int u = 0; u < kQV; ++u) {
          const int c = u * 32 + lane;
          const int g = c >> 4, ch = c & 15;
          sts128(qbuf + qb * kQB + (ch >> 3) * (kN * 128) + swz(g, ch & 7), q_c[u]);
        }
        fence_proxy_async_smem();
        mbar_arrive(&q_full[qb]);
      }
      const int st = k % kNST;
      const uint32_t use = (uint32_t)(k / kNST);
      if (use > 0 && !mbar_wait(&empty[st], (use - 1) & 1u, p.err)) {
        aborted = true;
        break;
      }
      unsigned char* sk = stages + st * kStage;
      unsigned char* sv = sk + kKV;
      const int j = pw * kTilesPerProd + lane;  // lanes 0..3 own tiles j of this stage
      const int tile = cur.st0 + j;
      int tier = 0, blk_id = 0, r0 = 0;
      bool valid = false;
      if (lane < kTilesPerProd && tile < cur.st1) {
        const int b = tile / p.tiles_per_block;
        r0 = (tile - b * p.tiles_per_block) * kTT;
        int64_t id = id_c;
        if (id >= p.split) {
          tier = 1;
          id -= p.split;
        }
        if (id >= 0 && id < p.nblk[tier]) {
          valid = true;
          blk_id = (int)id;
        } else {
          set_error(p.err, FD_DEVERR_BLOCK_ID);
        }
      }
      const bool dev_tile = valid && !p.host[tier];
      const unsigned dev_mask = __ballot_sync(0xffffffffu, dev_tile);
      const unsigned host_mask = __ballot_sync(0xffffffffu, valid && !dev_tile);
      if (lane == 0 && dev_mask != 0u) mbar_expect_tx(&full[st], (uint32_t)__popc(dev_mask) * 4u * 2048u);
      __syncwarp();
      if (dev_tile) {
        // four 2 KB boxes: K dims 0-63 / 64-127, V dims 0-63 / 64-127
        tma_load_4d(sk + j * 2048, &p.tmap_k[tier], 0, kh, r0, blk_id, &full[st], pol);
        tma_load_4d(sk + kPanel + j * 2048, &p.tmap_k[tier], 64, kh, r0, blk_id, &full[st], pol);
        tma_load_4d(sv + j * 2048, &p.tmap_v[tier], 0, kh, r0, blk_id, &full[st], pol);
        tma_load_4d(sv + kPanel + j * 2048, &p.tmap_v[tier], 64, kh, r0, blk_id, &full[st], pol);
      }
      for (unsigned m = host_mask; m != 0u; m &= m - 1u) {
        const int w = __ffs(m) - 1;
        const int tr = __shfl_sync(0xffffffffu, tier, w);
        const int bid = __shfl_sync(0xffffffffu, blk_id, w);
        const int rr0 = __shfl_sync(0xffffffffu, r0, w);
        const int64_t off = (int64_t)bid * p.blk_sb[tr] + (int64_t)kh * p.head_sb[tr] + (int64_t)rr0 * p.tok_sb[tr];
        const unsigned char* kw = p.k[tr] + off;
        const unsigned char* vw = p.v[tr] + off;
        // 16 rows x 16 chunks for K and for V: 8 chunks per lane each
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int c = u * 32 + lane;
          const int row = c >> 4, ch = c & 15;
          const uint4 kv = *reinterpret_cast<const uint4*>(kw + row * p.tok_sb[tr] + ch * 16);
          const uint4 vv = *reinterpret_cast<const uint4*>(vw + row * p.tok_sb[tr] + ch * 16);
          const int r = (pw * kTilesPerProd + w) * kTT + row;
          sts128(sk + (ch >> 3) * kPanel + swz(r, ch & 7), kv);
          sts128(sv + (ch >> 3) * kPanel + swz(r, ch & 7), vv);
        }
      }
      if (host_mask != 0u) fence_proxy_async_smem();  // generic smem writes before the MMA reads them
      mbar_arrive(&full[st]);
      ++k;
      cur = nxt;
#pragma unroll
      for (int u = 0; u < kQV; ++u) q_c[u] = q_n[u];
      have = have_n;
    }
    if (aborted) atomicExch(&abort_flag, 1);
    cp_async_wait<0>();  // no id copy outlives the CTA
    // every issued stage has landed before shared memory goes away (in a
    // normal run the MMA warp already waited on all of them)
    for (int q = std::max(0, k - kNST); q < k; ++q) mbar_wait(&full[q % kNST], (uint32_t)(q / kNST) & 1u, p.err);
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    // One thread polls the barriers of both products and issues whichever is
    // ready: q.K^T of a stage as soon as its tiles landed (at most two ahead,
    // bounded by the two S buffers), P.V as soon as the softmax wrote P.
    if (lane == 0) {
      StageIter it;
      it.init(g0, g1, row0, prefix, lens_s, p.n, Y, kTilesPerStage, p.vtiles);
      int kq = 0, kp = 0;  // next q.K^T stage, next P.V stage
      int st0, st1;
      bool qf, ql;
      bool have_qk = it.next(st0, st1, qf, ql);
      int qi = it.pieces - 1;
      bool ok = true;
      uint32_t spins = 0;
      uint64_t t_idle = 0;
      while (have_qk || kp < kq) {
        bool prog = false;
        if (have_qk) {
          const int st = kq % kNST, b = kq & 1, qb = qi & 1;
          if ((!qf || mbar_test_wait(&q_full[qb], (uint32_t)(qi >> 1) & 1u)) &&
              mbar_test_wait(&full[st], (uint32_t)(kq / kNST) & 1u) &&
              (kq < 2 || mbar_test_wait(&s_empty[b], (uint32_t)((kq >> 1) - 1) & 1u))) {
            tc_fence_after();
            const uint32_t sk = smem_u32(stages + st * kStage);
            const uint32_t sq = smem_u32(qbuf + qb * kQB);
#pragma unroll
            for (int ks = 0; ks < kD / 16; ++ks) {
              const uint32_t koff = (ks >> 2) * kPanel + (ks & 3) * 32;
              const uint32_t qoff = (ks >> 2) * (kN * 128) + (ks & 3) * 32;
              umma_f16(tmem + kN * b, sw128_desc(sk + koff, 16, 1024), sw128_desc(sq + qoff, 16, 1024), kIdQK,
                       ks > 0 ? 1u : 0u);
            }
            umma_commit(&s_full[b]);
            if (ql) umma_commit(&q_empty[qb]);
            ++kq;
            have_qk = it.next(st0, st1, qf, ql);
            qi = it.pieces - 1;
            prog = true;
          }
        }
        if (kp < kq) {
          const int st = kp % kNST, b = kp & 1;
          if (mbar_test_wait(&p_full[b], (uint32_t)(kp >> 1) & 1u) &&
              (kp < 2 || mbar_test_wait(&o_empty[b], (uint32_t)((kp >> 1) - 1) & 1u))) {
            tc_fence_after();
            const uint32_t sv = smem_u32(stages + st * kStage + kKV);
            const uint32_t sp = smem_u32(pbuf + b * kPB);
#pragma unroll
            for (int ks = 0; ks < kTok / 16; ++ks) {
              const uint32_t voff = ks * 2048;  // 16 token rows
              const uint32_t poff = (ks >> 2) * (kN * 128) + (ks & 3) * 32;
              umma_f16(tmem + 2 * kN + kN * b, sw128_desc(sv + voff, kPanel, 1024), sw128_desc(sp + poff, 16, 1024),
                       kIdPV, ks > 0 ? 1u : 0u);
            }
            umma_commit(&o_full[b]);
            umma_commit(&empty[st]);
            ++kp;
            prog = true;
          }
        }
        if (prog) {
          spins = 0;
          t_idle = 0;
        } else if ((++spins & 255u) == 0u) {
          const uint64_t now = globaltimer_ns();
          if (t_idle == 0) {
            t_idle = now;
          } else if (now - t_idle > kWaitLimitNs) {
            set_error(p.err, FD_DEVERR_TIMEOUT);
            ok = false;
            break;
          }
        }
      }
      if (!ok) atomicExch(&abort_flag, 1);
      // all MMAs issued by this thread complete before TMEM is released
      umma_commit(drain);
      mbar_wait(drain, 0u, p.err);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax warps 0-3
    // Per stage: S -> block max -> P (published) -> fold O of the PREVIOUS
    // stage, so the P.V round trip of stage k overlaps the softmax of k + 1.
    // A piece's last stage is folded, and the piece finished (denominators,
    // output or partial slot), after the NEXT piece's first P is published,
    // so that round trip and the epilogue overlap the next piece's products.
    const int r = threadIdx.x;  // token row of S, dim of O (TMEM lane)
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    griddep_wait();  // outputs, partial slots and the prefix are written below
    if (blockIdx.x == 0 && p.ws_prefix != nullptr)
      for (int i = r; i <= p.n; i += 128) p.ws_prefix[i] = prefix[i];
    // rows without tiles: empty -> o = 0, lse = -inf (reference
    // cpu_attn.cpp:324-331); overrun -> error word
    for (int i = blockIdx.x; i < p.n; i += gridDim.x) {
      if (prefix[i + 1] != prefix[i]) continue;
      const int len = lens_s[i];
      if (len > 0) {
        if (r == 0) set_error(p.err, FD_DEVERR_LEN);
        continue;
      }
      const int64_t orow = p.out_rows ? p.out_rows[i] : i;
      for (int o = r; orow >= 0 && o < p.H * kD; o += 128) {
        const int h = o / kD, d = o - h * kD;
        store_out(p.out, orow * p.out_sn + (int64_t)h * p.out_sh + d, p.out_dtype, 0.f);
      }
      if (p.lse != nullptr)
        for (int h = r; h < p.H; h += 128) p.lse[(int64_t)h * p.lse_sh + (int64_t)i * p.lse_sn] = -INFINITY;
    }
    StageIter it;
    it.init(g0, g1, row0, prefix, lens_s, p.n, Y, kTilesPerStage, p.vtiles);
    int k = 0;
    int st0, st1;
    bool pf, pl;
    float m_run[G], l_part[G], acc[G], alpha_prev[G];
    int h0 = 0;
    int64_t orow = 0;
    bool ok = true, pend = false;
    // the finished piece whose last fold and epilogue are still to come
    struct Done {
      float m[G], l[G], acc[G], alpha[G];
      int k_last, h0, row, slot, idx;
      int64_t orow;
      bool whole;
    } dn = {};
    bool pend_done = false;
    // fold O of stage kk (TMEM buffer kk & 1) into a_acc with the rescale a;
    // column g holds the hi part, column G + g the lo part of P.V
    auto fold = [&](int kk, const float (&a)[G], float (&a_acc)[G]) -> bool {
      const int bb = kk & 1;
      if (!mbar_wait(&o_full[bb], (uint32_t)(kk >> 1) & 1u, p.err)) return false;
      tc_fence_after();
      float o[16];
      tmem_ld16(tmem + lane_base + 2 * kN + kN * bb, o);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_empty[bb]);
#pragma unroll
      for (int g = 0; g < G; ++g) a_acc[g] = a_acc[g] * a[g] + (o[g] + o[G + g]);
      return true;
    };
    // last fold + denominators + output row or partial slot of piece dn
    auto finish = [&]() -> bool {
      if (!fold(dn.k_last, dn.alpha, dn.acc)) return false;
      float L[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float v = dn.l[g];
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
        L[g] = v;
      }
      float* lb = lsum;
      if (lane == 0) {
#pragma unroll
        for (int g = 0; g < G; ++g) lb[warp * kN + g] = L[g];
        mbar_arrive(l_full);
      }
      if (!mbar_wait(l_full, (uint32_t)dn.idx & 1u, p.err)) return false;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float Lg = lb[g] + lb[kN + g] + lb[2 * kN + g] + lb[3 * kN + g];
        const float lse_nat = (dn.m[g] + log2f(Lg)) * kLn2;
        const int h = dn.h0 + g;
        const float val = dn.acc[g] / Lg;
        if (dn.whole) {
          if (dn.orow >= 0) store_out(p.out, dn.orow * p.out_sn + (int64_t)h * p.out_sh + r, p.out_dtype, val);
          if (r == 0 && p.lse != nullptr) p.lse[(int64_t)h * p.lse_sh + (int64_t)dn.row * p.lse_sn] = lse_nat;
        } else {
          const int64_t pidx = ((int64_t)blockIdx.x * 2 + dn.slot) * G + g;
          p.part_o[pidx * kD + r] = val;
          if (r == 0) p.part_lse[pidx] = lse_nat;
        }
      }
      return true;
    };
    while (ok && it.next(st0, st1, pf, pl)) {
      const Piece& pc = it.pc;
      if (pf) {
        h0 = pc.y * G;
        if (pc.whole) orow = p.out_rows ? p.out_rows[pc.row] : pc.row;
#pragma unroll
        for (int g = 0; g < G; ++g) {
          m_run[g] = -INFINITY;
          l_part[g] = 0.f;
          acc[g] = 0.f;
        }
        pend = false;
      }
      const int b = k & 1;
      const int st = k % kNST;
      // ---- S of this stage
      if (!mbar_wait(&s_full[b], (uint32_t)(k >> 1) & 1u, p.err)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[8];
      tmem_ld8(tmem + lane_base + kN * b, s);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[b]);
      const int tile = st0 + (r >> 4);
      const int tok = tile * kTT + (r & 15);
      const bool valid = (tile < st1) && (tok < pc.len);
#pragma unroll
      for (int g = 0; g < G; ++g) s[g] = valid ? s[g] * p.qscale : -INFINITY;
      // warp max of each of the G columns by a halving butterfly: after it
      // this lane holds the max of column gm (set by lane bits 4, 3, 2)
      float bm[G];
#pragma unroll
      for (int g = 0; g < G; ++g) bm[g] = s[g];
      int gm = 0;
#pragma unroll
      for (int h = G / 2, m = 16; h >= 1; h >>= 1, m >>= 1) {
        const bool upper = (lane & m) != 0;
#pragma unroll
        for (int i = 0; i < h; ++i) {
          const float send = upper ? bm[i] : bm[h + i];
          const float keep = upper ? bm[h + i] : bm[i];
          bm[i] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, m));
        }
        if (upper) gm += h;
      }
#pragma unroll
      for (int m = 16 / (G / 2) / 2; m >= 1; m >>= 1) bm[0] = fmaxf(bm[0], __shfl_xor_sync(0xffffffffu, bm[0], m));
      float* rb = red + b * 4 * kN;
      if ((lane & (32 / G - 1)) == 0) rb[warp * kN + gm] = bm[0];
      __syncwarp();
      if (lane == 0) mbar_arrive(&red_full[b]);
      if (!mbar_wait(&red_full[b], (uint32_t)(k >> 1) & 1u, p.err)) {
        ok = false;
        break;
      }
      float alpha[G], pv[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float M = fmaxf(fmaxf(rb[g], rb[kN + g]), fmaxf(rb[2 * kN + g], rb[3 * kN + g]));
        const float mn = fmaxf(m_run[g], M);
        alpha[g] = (mn == -INFINITY) ? 1.f : exp2f(m_run[g] - mn);
        pv[g] = (s[g] == -INFINITY) ? 0.f : exp2f(s[g] - mn);
        l_part[g] = l_part[g] * alpha[g] + pv[g];
        m_run[g] = mn;
      }
      // ---- P (16-bit) into the swizzled B operand: p = hi + lo, hi in row g
      // and lo in row G + g, so columns g and G + g of O sum to P.V at nearly
      // fp32 precision.  Lane pairs swap halves: the even lane stores the hi
      // pair of its two tokens as one word, the odd lane the lo pair.
      unsigned char* pb = pbuf + b * kPB + (r >> 6) * (kN * 128);
      const int col = (r & 63) & ~1;
      const bool odd = (lane & 1) != 0;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const T hi = Dt<T>::narrow(pv[g]);
        const T lo = Dt<T>::narrow(pv[g] - Dt<T>::to_f32(hi));
        const uint32_t hb = bits16(hi);
        const uint32_t lb = bits16(lo);
        // even lane r gives lo_r and takes hi_r+1; odd lane gives hi_r and takes lo_r-1
        const uint32_t other = __shfl_xor_sync(0xffffffffu, odd ? hb : lb, 1);
        const uint32_t word = odd ? (other | (lb << 16)) : (hb | (other << 16));
        const int row = odd ? G + g : g;
        *reinterpret_cast<uint32_t*>(pb + swz(row, col >> 3) + (col & 7) * 2) = word;
      }
      if (!valid) {
        unsigned char* sv = stages + st * kStage + kKV;
        const uint4 z = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          sts128(sv + r * 128 + c * 16, z);
          sts128(sv + kPanel + r * 128 + c * 16, z);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[b]);
      // ---- O of the previous stage of this piece, then the previous piece
      if (pend && !fold(k - 1, alpha_prev, acc)) {
        ok = false;
        break;
      }
      if (pend_done) {
        if (!finish()) {
          ok = false;
          break;
        }
        pend_done = false;
      }
      if (!pl) {
#pragma unroll
        for (int g = 0; g < G; ++g) alpha_prev[g] = alpha[g];
        pend = true;
        ++k;
        continue;
      }
      // last stage of the piece: finished after the next piece's first P
#pragma unroll
      for (int g = 0; g < G; ++g) {
        dn.m[g] = m_run[g];
        dn.l[g] = l_part[g];
        dn.acc[g] = acc[g];
        dn.alpha[g] = alpha[g];
      }
      dn.k_last = k;
      dn.h0 = h0;
      dn.row = pc.row;
      dn.slot = pc.slot;
      dn.idx = it.pieces - 1;
      dn.orow = orow;
      dn.whole = pc.whole;
      pend_done = true;
      pend = false;
      ++k;
    }
    if (ok && pend_done && !finish()) ok = false;
    if (!ok) atomicExch(&abort_flag, 1);
  }

  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 5)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  griddep_launch_dependents();  // this CTA's writes are issued: the combine may launch
}

}  // namespace mma

template <int GM>
int launch_mma_g(const DecodeParams& q, int dtype, size_t smem, int n, cudaStream_t s, bool pdl) {
  static unsigned long long done_h = 0, done_b = 0;
  const int budget = mma::kSmemFixed + 3 * mma::kRowsBytes;
  const void* kern = dtype == FD_DTYPE_BF16
                         ? reinterpret_cast<const void*>(mma::fd_decode_mma_kernel<__nv_bfloat16, GM>)
                         : reinterpret_cast<const void*>(mma::fd_decode_mma_kernel<__half, GM>);
  const int st = fdh::ensure_smem(kern, budget, dtype == FD_DTYPE_BF16 ? &done_b : &done_h);
  if (st != FD_OK) return st;
  return fdh::launch_maybe_pdl(kern, dim3((unsigned)n), dim3(mma::kThreads), smem, s, pdl, q,
                               "fd_decode_mma_kernel launch");
}

bool mma_eligible(int dtype, int D, int G, int BS) {
  return (dtype == FD_DTYPE_F16 || dtype == FD_DTYPE_BF16) && D == mma::kD && (G == 2 || G == 4 || G == 8) &&
         BS % mma::kTT == 0;
}

int launch_decode_mma(const DecodeParams& p, int dtype, int D, size_t extra_smem, cudaStream_t s, int* ncta,
                      bool* launched, bool pdl) {
  *launched = false;
  if (!mma_eligible(dtype, D, p.G, p.BS) || p.gcs != 1 || p.TT != mma::kTT || !p.persistent) return FD_OK;
  for (int t = 0; t < 2; ++t)
    if (p.nblk[t] > 0 && !p.host[t] && !p.use_tmap[t]) return FD_OK;
  const size_t smem = (size_t)mma::kSmemFixed + 3 * extra_smem;  // prefix, lengths, table rows
  int dev = 0, sms = 0;
  int st0 = fdh::device_sms(&dev, &sms);
  if (st0 != FD_OK) return st0;
  const int n = std::max(1, std::min(*ncta, std::min(sms, kMaxPersistentCtas)));
  DecodeParams q = p;
  q.ncta = n;
  int st;
  switch (p.G) {
    case 2: st = launch_mma_g<2>(q, dtype, smem, n, s, pdl); break;
    case 4: st = launch_mma_g<4>(q, dtype, smem, n, s, pdl); break;
    default: st = launch_mma_g<8>(q, dtype, smem, n, s, pdl); break;
  }
  if (st == FD_OK) {
    *launched = true;
    *ncta = n;
  }
  return st;
}

}  // namespace fdk
