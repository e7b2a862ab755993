// Paged GQA decode on the 5th-generation tensor cores (tcgen05), sm_100a.
//
// For a kv head with a query group of G <= 8 heads the two products of
// decode attention are small matrix products per 128-token stage:
//   S^T [128 tokens x 8] = K [128 x 128] . q^T [128 x 8]       (q.K^T)
//   O^T [128 dims  x 8] = V^T [128 x 128] . P^T [128 x 8]      (P.V)
// (the group padded to the MMA's N = 16).  One CTA per SM, six warps:
//   warp 4   TMA producer: K and V tiles (16 tokens, one kv head) into a
//            3-stage ring in the 128-byte-swizzled layout the MMA reads
//            (tiled TMA, box {64 dims, 1, 16, 1}); host-tier tiles by
//            16-byte loads stored with the same swizzle; q of each piece
//   warp 5   MMA issuer: one thread issues tcgen05.mma into TMEM (S and O
//            double-buffered, 64 columns) and tcgen05.commit to mbarriers;
//            q.K^T of stage k+1 is issued before P.V of stage k
//   warps 0-3  softmax: thread r owns token row r of S (TMEM lane r): scale,
//            mask, block max (per stage), exp2, P written as 16-bit into the
//            swizzled B operand; then thread d owns dim d of O (TMEM lane d)
//            and folds it into an fp32 accumulator with the online-softmax
//            rescale.  Per-thread partial sums of p give the denominator.
// The schedule is the persistent one of fd_decode.cu (equal tile ranges per
// CTA, pieces, two partial slots per CTA, fd_persistent_combine_kernel).
// Numerics: scores and softmax in fp32 from the exact 16-bit q and K; P
// enters the P.V product as a sum of two 16-bit values (hi + lo, in the
// padding rows of the N = 16 operand), so P.V keeps nearly fp32 precision;
// all accumulation fp32.

#include <math.h>

#include <algorithm>
#include <type_traits>

#include "fd_common.cuh"
#include "fd_decode.cuh"
#include "fd_internal.h"

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
constexpr int kQB = 2 * kN * 128;   // q: two panels of 16 rows x 128 B
constexpr int kPB = 2 * kN * 128;   // P: two panels (tokens 0-63, 64-127) x 16 rows
constexpr int kThreads = 6 * 32;
constexpr int kTmemCols = 4 * kN;  // S0 S1 O0 O1, kN columns each

constexpr int kOffQ = kNST * kStage;
constexpr int kOffP = kOffQ + 2 * kQB;
constexpr int kOffRed = kOffP + 2 * kPB;         // [2][4 warps][kN] floats: per-stage maxima
constexpr int kOffL = kOffRed + 2 * 4 * kN * 4;  // [4 warps][kN] floats: per-piece sums
constexpr int kOffBar = kOffL + 4 * kN * 4;
constexpr int kNumBars = 3 + 3 + 2 * 7 + 1 + 2 + 1;
constexpr int kOffTmem = kOffBar + kNumBars * 8;
constexpr int kOffPrefix = (kOffTmem + 16 + 127) / 128 * 128;
constexpr int kSmemFixed = kOffPrefix + 1024;  // + 1024 for aligning the base
static_assert(kSmemFixed + (kMaxPersistentRows + 1) * 4 <= 227 * 1024, "smem budget");

// UMMA shared-memory descriptor, 128-byte swizzle, sm_100 version bits.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor of kind::f16 with fp32 accumulation.
constexpr uint32_t instr_desc(bool bf16, bool a_mn_major, int M, int N) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((a_mn_major ? 1u : 0u) << 15) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 lanes x 8 consecutive 32-bit columns starting at taddr.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// Byte offset of 16-byte chunk c (0..7) of row r inside 128-byte-swizzled
// rows (the 8-row atom pattern of TMA SWIZZLE_128B / UMMA SWIZZLE_128B).
__device__ __forceinline__ uint32_t swz(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

// Stage enumeration shared by the three roles: a stage is up to 8 tiles of
// one piece.
struct StageIter {
  int64_t g_cur, g_end;
  int row_cur;
  bool first, split_done, have;
  Piece pc;
  int t;       // first tile of the next stage of pc
  int pieces;  // pieces started so far

  __device__ void init(int64_t g0, int64_t g1, int row) {
    g_cur = g0;
    g_end = g1;
    row_cur = row;
    first = true;
    split_done = false;
    have = false;
    t = 0;
    pieces = 0;
  }

  __device__ bool next_piece(const DecodeParams& p, const int* prefix, int Y) {
    if (g_cur >= g_end) return false;
    const int nt = prefix[row_cur + 1] - prefix[row_cur];
    const int64_t local = g_cur - (int64_t)prefix[row_cur] * Y;
    const int y = (int)(local / nt);
    const int t0 = (int)(local - (int64_t)y * nt);
    const int t1 = (int)min((int64_t)nt, (int64_t)t0 + (g_end - g_cur));
    pc.row = row_cur;
    pc.y = y;
    pc.t0 = t0;
    pc.t1 = t1;
    pc.len = p.lens[row_cur];
    pc.whole = (t0 == 0 && t1 == nt);
    pc.slot = first ? 0 : 1;
    first = false;
    g_cur += t1 - t0;
    if (t1 == nt && y == Y - 1) {
      do {
        ++row_cur;
      } while (row_cur < p.n && prefix[row_cur + 1] == prefix[row_cur]);
    }
    return true;
  }

  // Next stage: tiles [st_t0, st_t1) of piece *pc; flags for piece bounds.
  __device__ bool next(const DecodeParams& p, const int* prefix, int Y, int& st_t0, int& st_t1, bool& piece_first,
                       bool& piece_last) {
    if (!have || t >= pc.t1) {
      if (!next_piece(p, prefix, Y)) return false;
      have = true;
      t = pc.t0;
      ++pieces;
      piece_first = true;
    } else {
      piece_first = false;
    }
    st_t0 = t;
    st_t1 = min(pc.t1, t + kTilesPerStage);
    t = st_t1;
    piece_last = (t >= pc.t1);
    return true;
  }
};

template <typename T, int GM>
__global__ void __launch_bounds__(kThreads, 1) fd_decode_mma_kernel(const __grid_constant__ DecodeParams p) {
  static_assert(GM >= 1 && 2 * GM <= kN, "query group (hi and lo rows of P) must fit the MMA N");
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kIdQK = instr_desc(kBF16, false, kTok, kN);
  constexpr uint32_t kIdPV = instr_desc(kBF16, true, kD, kN);
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  unsigned char* smem = smem_raw + ((((raw + 1023u) & ~1023u)) - raw);
  unsigned char* stages = smem;
  unsigned char* qbuf = smem + kOffQ;
  unsigned char* pbuf = smem + kOffP;
  float* red = reinterpret_cast<float*>(smem + kOffRed);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* full = bars;          // [3] TMA bytes + 32 producer lanes
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
  int* prefix = reinterpret_cast<int*>(smem + kOffPrefix);
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  constexpr int G = GM;
  const int Y = p.KVH;

  // ---------------------------------------------------------------- setup
  if (warp == 0) {
    int carry = 0;
    for (int base = 0; base < p.n; base += 32) {
      const int i = base + lane;
      int nt = 0;
      if (i < p.n) {
        const int len = p.lens[i];
        if (len > 0 && (len + p.BS - 1) / p.BS <= p.bt_width) nt = (len + kTT - 1) / kTT;
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
  // q and P buffers start zeroed: the padding rows g >= G stay zero
  for (int o = threadIdx.x * 16; o < 2 * kQB + 2 * kPB; o += kThreads * 16)
    sts128(qbuf + o, make_uint4(0u, 0u, 0u, 0u));
  fence_proxy_async_smem();
  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < 3; ++s) {
      mbar_init(&full[s], 32);
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
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (blockIdx.x == 0 && p.ws_prefix != nullptr)
    for (int i = threadIdx.x; i <= p.n; i += blockDim.x) p.ws_prefix[i] = prefix[i];
  for (int i = blockIdx.x; i < p.n; i += gridDim.x) {
    if (prefix[i + 1] != prefix[i]) continue;
    const int len = p.lens[i];
    if (len > 0) {
      if (threadIdx.x == 0) set_error(p.err, FD_DEVERR_LEN);
      continue;
    }
    const int64_t orow = p.out_rows ? p.out_rows[i] : i;
    for (int o = threadIdx.x; o < p.H * kD; o += blockDim.x) {
      const int h = o / kD, d = o - h * kD;
      store_out(p.out, orow * p.out_sn + (int64_t)h * p.out_sh + d, p.out_dtype, 0.f);
    }
    if (p.lse != nullptr)
      for (int h = threadIdx.x; h < p.H; h += blockDim.x) p.lse[(int64_t)h * p.lse_sh + (int64_t)i * p.lse_sn] = -INFINITY;
  }
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

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    const uint64_t pol = l2_evict_first_policy();
    StageIter it;
    it.init(g0, g1, row0);
    int k = 0, last_piece = 0;
    int st0, st1;
    bool pf, pl;
    bool aborted = false;
    while (!aborted && it.next(p, prefix, Y, st0, st1, pf, pl)) {
      const Piece& pc = it.pc;
      const int kh = pc.y;
      if (pf) {
        // q of this piece into q buffer (pieces-1) % 2
        const int qi = it.pieces - 1;
        const int qb = qi & 1;
        if (qi >= 2 && !mbar_wait(&q_empty[qb], ((qi >> 1) - 1) & 1u, p.err)) {
          aborted = true;
          break;
        }
        const int64_t qrow = p.q_rows ? p.q_rows[pc.row] : pc.row;
        const unsigned char* qsrc = p.q + qrow * p.q_sn + (int64_t)(kh * G) * p.q_sh;
        for (int c = lane; c < G * 16; c += 32) {
          const int g = c >> 4, ch = c & 15;
          const uint4 v = __ldg(reinterpret_cast<const uint4*>(qsrc + g * p.q_sh + ch * 16));
          sts128(qbuf + qb * kQB + (ch >> 3) * (kN * 128) + swz(g, ch & 7), v);
        }
        fence_proxy_async_smem();
        mbar_arrive(&q_full[qb]);
        last_piece = qi;
      }
      const int st = k % kNST;
      const uint32_t use = (uint32_t)(k / kNST);
      if (use > 0 && !mbar_wait(&empty[st], (use - 1) & 1u, p.err)) {
        aborted = true;
        break;
      }
      unsigned char* sk = stages + st * kStage;
      unsigned char* sv = sk + kKV;
      const int32_t* btrow = p.bt + (int64_t)pc.row * p.bt_stride;
      const int j = lane;  // lanes 0..7 own tiles j of this stage
      const int tile = st0 + j;
      int tier = 0, blk_id = 0, r0 = 0;
      bool valid = false;
      if (j < kTilesPerStage && tile < st1) {
        const int b = tile / p.tiles_per_block;
        r0 = (tile - b * p.tiles_per_block) * kTT;
        int64_t id = btrow[b];
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
          const int r = w * kTT + row;
          sts128(sk + (ch >> 3) * kPanel + swz(r, ch & 7), kv);
          sts128(sv + (ch >> 3) * kPanel + swz(r, ch & 7), vv);
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(&full[st]);
      ++k;
    }
    (void)last_piece;
    if (aborted) atomicExch(&abort_flag, 1);
    // every issued stage has landed before shared memory goes away (in a
    // normal run the MMA warp already waited on all of them)
    for (int q = std::max(0, k - kNST); q < k; ++q) mbar_wait(&full[q % kNST], (uint32_t)(q / kNST) & 1u, p.err);
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    StageIter qk_it, pv_it;
    qk_it.init(g0, g1, row0);
    pv_it.init(g0, g1, row0);
    int kq = 0, kp = 0;  // next q.K^T stage, next P.V stage
    int st0, st1;
    bool pf, pl;
    bool have_qk = qk_it.next(p, prefix, Y, st0, st1, pf, pl);
    bool qk_first = pf, qk_last = pl;
    bool ok = true;
    // issue q.K^T for stage kq (its inputs landed, S buffer free, q ready)
    auto issue_qk = [&]() -> bool {
      const int st = kq % kNST, b = kq & 1;
      const int qi = qk_it.pieces - 1, qb = qi & 1;
      if (qk_first && !mbar_wait(&q_full[qb], (qi >> 1) & 1u, p.err)) return false;
      if (!mbar_wait(&full[st], (kq / kNST) & 1u, p.err)) return false;
      if (kq >= 2 && !mbar_wait(&s_empty[b], ((kq >> 1) - 1) & 1u, p.err)) return false;
      tc_fence_after();
      if (lane == 0) {
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
        if (qk_last) umma_commit(&q_empty[qb]);
      }
      __syncwarp();
      return true;
    };
    if (have_qk) ok = issue_qk();
    while (ok && have_qk) {
      // look one stage ahead so q.K^T(k+1) overlaps the softmax of stage k
      const int cur = kq;
      ++kq;
      have_qk = qk_it.next(p, prefix, Y, st0, st1, pf, pl);
      qk_first = pf;
      qk_last = pl;
      if (have_qk && !issue_qk()) {
        ok = false;
        break;
      }
      // P.V for stage cur
      int pst0, pst1;
      bool ppf, ppl;
      pv_it.next(p, prefix, Y, pst0, pst1, ppf, ppl);
      const int st = cur % kNST, b = cur & 1;
      if (!mbar_wait(&p_full[b], (cur >> 1) & 1u, p.err)) {
        ok = false;
        break;
      }
      if (cur >= 2 && !mbar_wait(&o_empty[b], ((cur >> 1) - 1) & 1u, p.err)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t sv = smem_u32(stages + st * kStage + kKV);
        const uint32_t sp = smem_u32(pbuf + b * kPB);
#pragma unroll
        for (int ks = 0; ks < kTok / 16; ++ks) {
          const uint32_t voff = ks * 2048;  // 16 token rows
          const uint32_t poff = (ks >> 2) * (kN * 128) + (ks & 3) * 32;
          umma_f16(tmem + 2 * kN + kN * b, sw128_desc(sv + voff, kPanel, 1024), sw128_desc(sp + poff, 16, 1024), kIdPV,
                   ks > 0 ? 1u : 0u);
        }
        umma_commit(&o_full[b]);
        umma_commit(&empty[st]);
      }
      __syncwarp();
      ++kp;
    }
    if (!ok) atomicExch(&abort_flag, 1);
    // all MMAs issued by this thread complete before TMEM is released
    if (lane == 0) umma_commit(drain);
    __syncwarp();
    mbar_wait(drain, 0u, p.err);
  } else {
    // ------------------------------------------------------------ softmax warps 0-3
    const int r = threadIdx.x;  // token row of S, dim of O (TMEM lane)
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    StageIter it;
    it.init(g0, g1, row0);
    int k = 0;
    int st0, st1;
    bool pf, pl;
    float m_run[G], l_part[G], acc[G];
    int h0 = 0;
    bool ok = true;
    while (ok && it.next(p, prefix, Y, st0, st1, pf, pl)) {
      const Piece& pc = it.pc;
      if (pf) {
        h0 = pc.y * G;
#pragma unroll
        for (int g = 0; g < G; ++g) {
          m_run[g] = -INFINITY;
          l_part[g] = 0.f;
          acc[g] = 0.f;
        }
      }
      const int b = k & 1;
      const int st = k % kNST;
      // ---- S of this stage
      if (!mbar_wait(&s_full[b], (k >> 1) & 1u, p.err)) {
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
      float bm[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        s[g] = valid ? s[g] * p.qscale : -INFINITY;
        bm[g] = s[g];
      }
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1)
#pragma unroll
        for (int g = 0; g < G; ++g) bm[g] = fmaxf(bm[g], __shfl_xor_sync(0xffffffffu, bm[g], off));
      float* rb = red + b * 4 * kN;
      if (lane == 0) {
#pragma unroll
        for (int g = 0; g < G; ++g) rb[warp * kN + g] = bm[g];
        mbar_arrive(&red_full[b]);
      }
      if (!mbar_wait(&red_full[b], (k >> 1) & 1u, p.err)) {
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
      // ---- P (16-bit) into the swizzled B operand; masked tokens zero their V row
      unsigned char* pb = pbuf + b * kPB + (r >> 6) * (kN * 128);
      const int col = r & 63;
      // p = hi + lo in the 16-bit type: rows g and 8 + g of the B operand, so
      // columns g and 8 + g of O sum to P.V at nearly fp32 precision
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const T hi = Dt<T>::narrow(pv[g]);
        const T lo = Dt<T>::narrow(pv[g] - Dt<T>::to_f32(hi));
        *reinterpret_cast<T*>(pb + swz(g, col >> 3) + (col & 7) * 2) = hi;
        *reinterpret_cast<T*>(pb + swz(8 + g, col >> 3) + (col & 7) * 2) = lo;
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
      // ---- O of this stage, folded into the accumulator
      if (!mbar_wait(&o_full[b], (k >> 1) & 1u, p.err)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float o[8], o_lo[8];
      tmem_ld8(tmem + lane_base + 2 * kN + kN * b, o);
      tmem_ld8(tmem + lane_base + 2 * kN + kN * b + 8, o_lo);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_empty[b]);
#pragma unroll
      for (int g = 0; g < G; ++g) acc[g] = acc[g] * alpha[g] + (o[g] + o_lo[g]);
      ++k;

      if (pl) {
        // ---- piece epilogue: denominators, output row or partial slot
        float L[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
          float v = l_part[g];
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
        if (!mbar_wait(l_full, (uint32_t)(it.pieces - 1) & 1u, p.err)) {
          ok = false;
          break;
        }
        const int64_t orow = p.out_rows ? p.out_rows[pc.row] : pc.row;
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float Lg = lb[g] + lb[kN + g] + lb[2 * kN + g] + lb[3 * kN + g];
          const float lse_nat = (m_run[g] + log2f(Lg)) * kLn2;
          const int h = h0 + g;
          const float val = acc[g] / Lg;
          if (pc.whole) {
            store_out(p.out, orow * p.out_sn + (int64_t)h * p.out_sh + r, p.out_dtype, val);
            if (r == 0 && p.lse != nullptr) p.lse[(int64_t)h * p.lse_sh + (int64_t)pc.row * p.lse_sn] = lse_nat;
          } else {
            const int64_t pidx = ((int64_t)blockIdx.x * 2 + pc.slot) * G + g;
            p.part_o[pidx * kD + r] = val;
            if (r == 0) p.part_lse[pidx] = lse_nat;
          }
        }
      }
    }
    if (!ok) atomicExch(&abort_flag, 1);
  }

  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 5)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

}  // namespace mma

template <int GM>
int launch_mma_g(const DecodeParams& q, int dtype, size_t smem, int n, cudaStream_t s) {
  static unsigned long long done_h = 0, done_b = 0;
  const int budget = mma::kSmemFixed + (kMaxPersistentRows + 1) * 4 + 16;
  int st;
  if (dtype == FD_DTYPE_BF16) {
    st = fdh::ensure_smem(reinterpret_cast<const void*>(mma::fd_decode_mma_kernel<__nv_bfloat16, GM>), budget, &done_b);
    if (st != FD_OK) return st;
    mma::fd_decode_mma_kernel<__nv_bfloat16, GM><<<n, mma::kThreads, smem, s>>>(q);
  } else {
    st = fdh::ensure_smem(reinterpret_cast<const void*>(mma::fd_decode_mma_kernel<__half, GM>), budget, &done_h);
    if (st != FD_OK) return st;
    mma::fd_decode_mma_kernel<__half, GM><<<n, mma::kThreads, smem, s>>>(q);
  }
  return fdh::cuda_status(cudaGetLastError(), "fd_decode_mma_kernel launch");
}

bool mma_eligible(int dtype, int D, int G, int BS) {
  return (dtype == FD_DTYPE_F16 || dtype == FD_DTYPE_BF16) && D == mma::kD && (G == 2 || G == 4 || G == 8) &&
         BS % mma::kTT == 0;
}

int launch_decode_mma(const DecodeParams& p, int dtype, int D, size_t extra_smem, cudaStream_t s, int* ncta,
                      bool* launched) {
  *launched = false;
  if (!mma_eligible(dtype, D, p.G, p.BS) || p.gcs != 1 || p.TT != mma::kTT || !p.persistent) return FD_OK;
  for (int t = 0; t < 2; ++t)
    if (p.nblk[t] > 0 && !p.host[t] && !p.use_tmap[t]) return FD_OK;
  const size_t smem = (size_t)mma::kSmemFixed + extra_smem;
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return fdh::cuda_status(e, "device attributes");
  const int n = std::max(1, std::min(*ncta, std::min(sms, kMaxPersistentCtas)));
  DecodeParams q = p;
  q.ncta = n;
  int st;
  switch (p.G) {
    case 2: st = launch_mma_g<2>(q, dtype, smem, n, s); break;
    case 4: st = launch_mma_g<4>(q, dtype, smem, n, s); break;
    default: st = launch_mma_g<8>(q, dtype, smem, n, s); break;
  }
  if (st == FD_OK) {
    *launched = true;
    *ncta = n;
  }
  return st;
}

}  // namespace fdk
