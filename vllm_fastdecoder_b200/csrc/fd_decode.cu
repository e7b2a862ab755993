// Split-KV paged decode attention over a two-tier (HBM + mapped host) block
// table, for sm_100a.
//
// Grid: x = split of the row's token range, y = (kv head, query-head chunk),
// z = row.  Each CTA streams its split's K/V tiles (tile = min(block_size,16)
// tokens of one block and one kv head) through an NST-deep shared-memory ring:
//   * warps 4-5 (producers) fill a stage, two tiles each (a warp issues its
//     copies one after another): device-memory tiles with TMA bulk copies
//     (cp.async.bulk, completion counted in bytes on the stage's mbarrier),
//     host-tier tiles (pinned, mapped) with 16-byte loads;
//   * warps 0-3 (consumers) each own one tile per stage: q.K^T with fp32 FMAs
//     and shuffle reductions, an fp32 online softmax in the exp2 domain, then
//     P.V into per-lane fp32 accumulators, and release the stage.
// The four warp-level states are merged through shared memory at the end.
// A row that fits in one split writes o / lse directly; otherwise the split
// writes an fp32 partial (o normalised, lse) into the workspace and
// fd_split_merge_kernel combines them with the log-sum-exp rule.
//
// Numerics follow the reference CPU kernel (fastdecode/csrc/cpu_attn.cpp
// :298-411): fp16/bf16 widened to fp32, q pre-scaled in fp32 (:338), fp32
// accumulation, output = acc * (1/sum) cast to the output type (:401-405),
// lse = max + log(sum) (:406), empty row -> o = 0, lse = -inf (:324-331).

#include <math.h>

#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <mutex>

#include <cudaTypedefs.h>

#include "fd_common.cuh"
#include "fd_decode.cuh"
#include "fd_internal.h"

namespace fdk {

constexpr int p2div(int x, int p) { return (x % (2 * p) == 0 && 2 * p <= 32) ? p2div(x, 2 * p) : p; }
constexpr int ceil_pow2(int x, int p) { return p >= x ? p : ceil_pow2(x, 2 * p); }
constexpr int cmin(int a, int b) { return a < b ? a : b; }
constexpr int cmax(int a, int b) { return a > b ? a : b; }
constexpr int round128(int x) { return (x + 127) / 128 * 128; }

template <typename T, int D, int GQ>
struct Cfg {
  static constexpr int kE = sizeof(T);
  static constexpr int kRB = D * kE;  // bytes of one token row of one head
  static constexpr int kNCH = kRB / 16;
  static constexpr int kEPC = 16 / kE;
  static constexpr int kNW = 4;  // consumer warps
  // producer warps: a warp issues its copies one after another, so the
  // tiles of a stage are split between two of them
  static constexpr int kNP = 2;
  static constexpr int kTilesPerProd = kNW / kNP;  // tiles of a stage per producer warp
  static constexpr int kThreads = (kNW + kNP) * 32;
  static constexpr int kMaxTT = 16;
  // q.K: kTPT lanes per token, each holding kCPL 16-byte chunks of q per head
  static constexpr int kTPT = cmin(p2div(kNCH, 1), ceil_pow2(cmax(2, GQ * D / 64), 1));
  static constexpr int kCPL = kNCH / kTPT;
  static constexpr int kTPP = 32 / kTPT;  // tokens per pass
  static constexpr int kNPASS = (kMaxTT + kTPP - 1) / kTPP;
  // P.V: lane owns chunk (lane % kNCH) of token rows (lane / kNCH) + k*kRPI
  static constexpr int kRPI = 32 / kNCH;
  static constexpr int kPVL = kRPI * kNCH;
  // the kRPI row groups of a warp are summed with shuffles when they tile
  // the warp exactly, otherwise through shared memory
  static constexpr bool kShflRed = (kPVL == 32);
  static constexpr int kRedRows = kShflRed ? 1 : kRPI;
  static constexpr int kTileBytes = kMaxTT * kRB;
  // smem slot of one K or V tile, 128-byte aligned for tiled TMA
  static constexpr int kTileSlot = round128(kTileBytes);
  static constexpr int kStageBytes = kNW * 2 * kTileSlot;
  static constexpr int kNST = cmax(2, cmin(4, 98304 / kStageBytes));
  static constexpr int kBarBytes = 128;
  static constexpr int kPsBytes = round128(kNW * kMaxTT * GQ * 4);
  static constexpr int kRedBytes = round128((2 * kNW * GQ + kNW * kRedRows * GQ * D) * 4);
  static constexpr int kSmem = kBarBytes + kNP * kIdRingBytes + kPsBytes + kRedBytes + kNST * kStageBytes;
  static constexpr int kPrefixMax = round128((kMaxPersistentRows + 1) * 4);
  static constexpr bool kValid = (kRB % 16 == 0) && kNCH <= 32 && (GQ * kCPL * kEPC <= 64 || GQ == 1) &&
                                 (2 * kNST + 2) * 8 <= kBarBytes && kSmem + kPrefixMax <= 227 * 1024;
};

template <typename T, int D, int GQ>
__global__ void __launch_bounds__(Cfg<T, D, GQ>::kThreads, 2)
    fd_decode_kernel(const __grid_constant__ DecodeParams p) {
  using C = Cfg<T, D, GQ>;
  using DT = Dt<T>;
  constexpr int EPC = C::kEPC;
  constexpr int EP2 = EPC / 2;
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + C::kNST;
  uint64_t* comb_full = empty + C::kNST;  // 4 consumer warps wrote their piece state
  uint64_t* comb_done = comb_full + 1;    // 4 consumer warps finished the piece outputs
  int* id_ring = reinterpret_cast<int*>(smem + C::kBarBytes);  // [kNP] rings
  float* ps_all = reinterpret_cast<float*>(smem + C::kBarBytes + C::kNP * kIdRingBytes);
  float* red_m = reinterpret_cast<float*>(smem + C::kBarBytes + C::kNP * kIdRingBytes + C::kPsBytes);
  float* red_l = red_m + C::kNW * GQ;
  float* red_acc = red_l + C::kNW * GQ;
  unsigned char* stages = smem + C::kBarBytes + C::kNP * kIdRingBytes + C::kPsBytes + C::kRedBytes;
  int* prefix = reinterpret_cast<int*>(stages + C::kNST * C::kStageBytes);
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int Y = p.KVH * p.gcs;

  // ---------------------------------------------------------------- setup
  // prefix[i] = positions of rows < i: tiles + vtiles per row (0 for empty
  // rows and rows whose length overruns their table row).  Every thread
  // loads lengths (independent loads: one memory round trip) and leaves
  // row i's count in prefix[i + 1]; warp 0 then scans in place.
  if (p.persistent) {
    for (int i = threadIdx.x; i < p.n; i += blockDim.x) {
      const int len = p.lens[i];
      prefix[i + 1] = (len > 0 && (len + p.BS - 1) / p.BS <= p.bt_width) ? (len + p.TT - 1) / p.TT + p.vtiles : 0;
    }
  }
  if (threadIdx.x == 0) {
    abort_flag = 0;
#pragma unroll
    for (int s = 0; s < C::kNST; ++s) {
      mbar_init(&full[s], 32 * C::kNP);
      mbar_init(&empty[s], C::kNW);
    }
    mbar_init(comb_full, C::kNW);
    mbar_init(comb_done, C::kNW);
    fence_barrier_init();
  }
  __syncthreads();
  if (p.persistent && warp == 0) {
    int carry = 0;
    for (int base = 0; base < p.n; base += 32) {
      const int i = base + lane;
      int v = i < p.n ? prefix[i + 1] : 0;
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
  if (p.persistent) __syncthreads();

  // Programmatic dependent launch (fd_decode_args.flags & FD_DECODE_PDL):
  // everything up to here, and the producers' block-id and q prefetch below,
  // only reads inputs the caller guarantees the kernel ahead on the stream
  // does not write; every thread passes griddep_wait() before its first
  // K/V read and its first global write (a no-op for an ordinary launch).
  int64_t g_cur = 0, g_end = 0;
  int row_cur = 0;
  if (p.persistent) {
    const int64_t total = (int64_t)prefix[p.n] * Y;
    g_cur = (int64_t)blockIdx.x * total / gridDim.x;
    g_end = (int64_t)(blockIdx.x + 1) * total / gridDim.x;
    if (g_cur < g_end) {
      int lo = 0, hi = p.n - 1;  // last row whose first tile is <= g_cur
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if ((int64_t)prefix[mid] * Y <= g_cur) lo = mid; else hi = mid - 1;
      }
      row_cur = lo;
    }
  } else {
    // split grid: x = split, y = kv-head chunk, z = row
    const int i = blockIdx.z;
    const int len = p.lens[i];
    if (len <= 0) {
      griddep_wait();
      if (blockIdx.x == 0) {
        const int kh = blockIdx.y / p.gcs, gc = blockIdx.y - kh * p.gcs;
        const int h0 = kh * p.G + gc * GQ;
        const int64_t orow = p.out_rows ? p.out_rows[i] : i;
        for (int o = threadIdx.x; orow >= 0 && o < GQ * D; o += blockDim.x) {
          const int g = o / D, d = o - g * D;
          store_out(p.out, orow * p.out_sn + (int64_t)(h0 + g) * p.out_sh + d, p.out_dtype, 0.f);
        }
        if (p.lse != nullptr && threadIdx.x < GQ)
          p.lse[(int64_t)(h0 + threadIdx.x) * p.lse_sh + (int64_t)i * p.lse_sn] = -INFINITY;
      }
      return;
    }
    const int nblk = (len + p.BS - 1) / p.BS;
    const int ntiles = (len + p.TT - 1) / p.TT;
    const int nsplits = (ntiles + p.tiles_per_split - 1) / p.tiles_per_split;
    if (nblk > p.bt_width || nsplits > p.max_splits) {
      if (threadIdx.x == 0 && blockIdx.x == 0) set_error(p.err, nblk > p.bt_width ? FD_DEVERR_LEN : FD_DEVERR_SPLITS);
      return;
    }
    if ((int)blockIdx.x >= nsplits) return;
  }

  // Pieces of this CTA, enumerated identically by the producer and consumers.
  StageIter pieces;
  if (p.persistent) {
    pieces.init(g_cur, g_end, row_cur, prefix, p.lens, p.n, Y, C::kNW, p.vtiles);
    pieces.trows = p.bt_rows;
  } else {
    const int i = blockIdx.z;
    const int len = p.lens[i];
    const int ntiles = (len + p.TT - 1) / p.TT;
    const int nsplits = (ntiles + p.tiles_per_split - 1) / p.tiles_per_split;
    Piece sp;
    sp.row = i;
    sp.y = blockIdx.y;
    sp.t0 = blockIdx.x * p.tiles_per_split;
    sp.t1 = min(ntiles, sp.t0 + p.tiles_per_split);
    sp.len = len;
    sp.trow = p.bt_rows != nullptr ? p.bt_rows[i] : i;
    sp.whole = (nsplits == 1);
    sp.slot = blockIdx.x;
    pieces.init_single(sp, C::kNW);
  }
  auto next_piece = [&](Piece& pc) -> bool {
    if (!pieces.next_piece()) return false;
    pc = pieces.pc;
    return true;
  };

  const uint32_t tile_bytes = (uint32_t)p.TT * C::kRB;

  if (warp >= C::kNW) {
    // ------------------------------------------------------------ producers
    // producer pw fills tiles [pw * kTilesPerProd, (pw + 1) * kTilesPerProd)
    // of every stage;
    // block ids kIdAhead stages ahead (a cp.async ring per producer), q of
    // coming pieces prefetched into L2 for the consumers (producer 0)
    const int pw = warp - C::kNW;
    const int slot0 = pw * C::kTilesPerProd;  // first tile slot of this producer in a stage
    const int q_heads = pw == 0 ? GQ : 0;
    const uint64_t pol = l2_evict_first_policy();
    IdPrefetch ids;
    ids.it = pieces;  // a copy, before any piece was taken: the same sequence
    ids.ring = id_ring + pw * (kIdRingBytes / 4);
    ids.issued = 0;
    for (int i = 0; i < kIdAhead; ++i) ids.push(p, lane, q_heads, C::kRB, slot0, C::kTilesPerProd);
    griddep_wait();  // K/V below may be written by the kernel ahead (the KV write)
    int k = 0;
    Piece pc;
    while (next_piece(pc)) {
      const int kh = pc.y / p.gcs;
      for (int t = pc.t0; t < pc.t1; t += C::kNW, ++k) {
        ids.push(p, lane, q_heads, C::kRB, slot0, C::kTilesPerProd);  // stage k + kIdAhead
        const int64_t id_k = ids.take(k, lane);
        const int st = k % C::kNST;
        const uint32_t use = (uint32_t)(k / C::kNST);
        if (use > 0 && !mbar_wait(&empty[st], (use - 1) & 1u, p.err)) {
          cp_async_wait<0>();
          return;
        }
        unsigned char* sbase = stages + st * C::kStageBytes;
        const int tile = t + slot0 + lane;
        int tier = 0;
        bool valid = false;
        const unsigned char* ks = nullptr;
        const unsigned char* vs = nullptr;
        int blk_id = 0, r0 = 0;
        if (lane < C::kTilesPerProd && tile < pc.t1) {
          const int b = tile / p.tiles_per_block;
          r0 = (tile - b * p.tiles_per_block) * p.TT;
          int64_t id = id_k;
          if (id >= p.split) {
            tier = 1;
            id -= p.split;
          }
          if (id >= 0 && id < p.nblk[tier]) {
            valid = true;
            blk_id = (int)id;
            const int64_t off = id * p.blk_sb[tier] + (int64_t)kh * p.head_sb[tier] + (int64_t)r0 * p.tok_sb[tier];
            ks = p.k[tier] + off;
            vs = p.v[tier] + off;
          } else {
            set_error(p.err, FD_DEVERR_BLOCK_ID);
          }
        }
        const bool bulk = valid && !p.host[tier];
        const unsigned bulk_mask = __ballot_sync(0xffffffffu, bulk);
        const unsigned host_mask = __ballot_sync(0xffffffffu, valid && !bulk);
        if (lane == 0 && bulk_mask != 0u)
          mbar_expect_tx(&full[st], (uint32_t)__popc(bulk_mask) * 2u * tile_bytes);
        __syncwarp();
        // contiguous tiles and tensor-map tiles: each lane issues its own
        // tile's two copies (no cross-lane traffic on the issue path)
        const bool own = bulk && (p.contig[tier] || p.use_tmap[tier]);
        if (own) {
          unsigned char* kd = sbase + (2 * (slot0 + lane)) * C::kTileSlot;
          unsigned char* vd = kd + C::kTileSlot;
          if (p.contig[tier]) {
            bulk_g2s(kd, ks, tile_bytes, &full[st], pol);
            bulk_g2s(vd, vs, tile_bytes, &full[st], pol);
          } else {
            tma_load_4d(kd, &p.tmap_k[tier], 0, kh, r0, blk_id, &full[st], pol);
            tma_load_4d(vd, &p.tmap_v[tier], 0, kh, r0, blk_id, &full[st], pol);
          }
        }
        // other device tiles: one bulk copy per token row, rows spread over lanes
        for (unsigned m = bulk_mask & ~__ballot_sync(0xffffffffu, own); m != 0u; m &= m - 1u) {
          const int w = __ffs(m) - 1;
          const unsigned char* kw = reinterpret_cast<const unsigned char*>(
              __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(ks), w));
          const unsigned char* vw = reinterpret_cast<const unsigned char*>(
              __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(vs), w));
          const int tr = __shfl_sync(0xffffffffu, tier, w);
          unsigned char* kd = sbase + (2 * (slot0 + w)) * C::kTileSlot;
          unsigned char* vd = kd + C::kTileSlot;
          for (int r = lane; r < p.TT; r += 32) {
            bulk_g2s(kd + r * C::kRB, kw + r * p.tok_sb[tr], C::kRB, &full[st], pol);
            bulk_g2s(vd + r * C::kRB, vw + r * p.tok_sb[tr], C::kRB, &full[st], pol);
          }
        }
        for (unsigned m = host_mask; m != 0u; m &= m - 1u) {
          const int w = __ffs(m) - 1;
          const unsigned char* kw = reinterpret_cast<const unsigned char*>(
              __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(ks), w));
          const unsigned char* vw = reinterpret_cast<const unsigned char*>(
              __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(vs), w));
          const int tr = __shfl_sync(0xffffffffu, tier, w);
          const int64_t tsb = p.tok_sb[tr];
          unsigned char* kd = sbase + (2 * (slot0 + w)) * C::kTileSlot;
          unsigned char* vd = kd + C::kTileSlot;
          const int nch = p.TT * C::kNCH;
          constexpr int U = 4;
          for (int c0 = 0; c0 < nch; c0 += 32 * U) {
            uint4 kb[U], vb[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
              const int c = c0 + u * 32 + lane;
              if (c < nch) {
                const int row = c / C::kNCH;
                const int64_t off = row * tsb + (c - row * C::kNCH) * 16;
                kb[u] = *reinterpret_cast<const uint4*>(kw + off);
                vb[u] = *reinterpret_cast<const uint4*>(vw + off);
              }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
              const int c = c0 + u * 32 + lane;
              if (c < nch) {
                sts128(kd + c * 16, kb[u]);
                sts128(vd + c * 16, vb[u]);
              }
            }
          }
        }
        // order this stage's generic smem writes before later TMA writes to it
        if (host_mask != 0u) fence_proxy_async_smem();
        mbar_arrive(&full[st]);
      }
    }
    cp_async_wait<0>();  // no id copy outlives the CTA
    return;
  }

  // -------------------------------------------------------------- consumers
  griddep_wait();  // outputs, partial slots and the prefix are written below
  constexpr int kCT = C::kNW * 32;  // consumer threads
  if (p.persistent) {
    if (blockIdx.x == 0 && p.ws_prefix != nullptr)
      for (int i = threadIdx.x; i <= p.n; i += kCT) p.ws_prefix[i] = prefix[i];
    // rows without tiles: empty -> o = 0, lse = -inf (reference
    // cpu_attn.cpp:324-331); overrun -> error word
    for (int i = blockIdx.x; i < p.n; i += gridDim.x) {
      if (prefix[i + 1] != prefix[i]) continue;
      const int len = p.lens[i];
      if (len > 0) {
        if (threadIdx.x == 0) set_error(p.err, FD_DEVERR_LEN);
        continue;
      }
      const int64_t orow = p.out_rows ? p.out_rows[i] : i;
      for (int o = threadIdx.x; orow >= 0 && o < p.H * D; o += kCT) {
        const int h = o / D, d = o - h * D;
        store_out(p.out, orow * p.out_sn + (int64_t)h * p.out_sh + d, p.out_dtype, 0.f);
      }
      if (p.lse != nullptr)
        for (int h = threadIdx.x; h < p.H; h += kCT) p.lse[(int64_t)h * p.lse_sh + (int64_t)i * p.lse_sn] = -INFINITY;
    }
  }
  const int tp = lane / C::kTPT;
  const int sub = lane - tp * C::kTPT;
  const int rot = tp % C::kCPL;
  const int cpv = lane % C::kNCH;
  const int rg = lane / C::kNCH;
  const bool pv_on = lane < C::kPVL;
  float* psw = ps_all + warp * C::kMaxTT * GQ;
  int k = 0;
  uint32_t npieces = 0;
  Piece pc;
  while (next_piece(pc)) {
    const int kh = pc.y / p.gcs;
    const int gc = pc.y - kh * p.gcs;
    const int h0 = kh * p.G + gc * GQ;

    // q for this lane's chunks, widened and pre-scaled (reference :334-339),
    // in the rotated order the K reads use (bank-conflict free), as packed
    // fp32 pairs
    f2_t qr[GQ][C::kCPL][EP2];
    {
      const int64_t qrow = p.q_rows ? p.q_rows[pc.row] : pc.row;
      const unsigned char* qb = p.q + qrow * p.q_sn + (int64_t)h0 * p.q_sh;
      const f2_t qs2 = f2_pack(p.qscale, p.qscale);
#pragma unroll
      for (int g = 0; g < GQ; ++g) {
#pragma unroll
        for (int jj = 0; jj < C::kCPL; ++jj) {
          const int c = sub + C::kTPT * ((jj + rot) % C::kCPL);
          const uint4 v = __ldg(reinterpret_cast<const uint4*>(qb + g * p.q_sh + c * 16));
          DT::widen2(v, qr[g][jj]);
#pragma unroll
          for (int e = 0; e < EP2; ++e) qr[g][jj][e] = f2_mul(qr[g][jj][e], qs2);
        }
      }
    }

    float m_run[GQ], l_run[GQ];
    f2_t acc[GQ][EP2];
#pragma unroll
    for (int g = 0; g < GQ; ++g) {
      m_run[g] = -INFINITY;
      l_run[g] = 0.f;
#pragma unroll
      for (int e = 0; e < EP2; ++e) acc[g][e] = f2_pack(0.f, 0.f);
    }
    bool ok = true;

    for (int t = pc.t0; t < pc.t1; t += C::kNW, ++k) {
      const int st = k % C::kNST;
      const uint32_t use = (uint32_t)(k / C::kNST);
      if (!mbar_wait(&full[st], use & 1u, p.err)) {
        ok = false;
        break;
      }
      const int tile = t + warp;
      if (tile < pc.t1) {
        const int ntok = min(p.TT, pc.len - tile * p.TT);
        const unsigned char* ks = stages + st * C::kStageBytes + (2 * warp) * C::kTileSlot;
        const unsigned char* vs = ks + C::kTileSlot;

        // ---- scores s = q.k (log2 domain), one token per lane group per pass
        float s[GQ][C::kNPASS];
#pragma unroll
        for (int pp = 0; pp < C::kNPASS; ++pp) {
          const int tk = pp * C::kTPP + tp;
          f2_t dot2[GQ];
#pragma unroll
          for (int g = 0; g < GQ; ++g) dot2[g] = f2_pack(0.f, 0.f);
          if (tk < ntok) {
#pragma unroll
            for (int jj = 0; jj < C::kCPL; ++jj) {
              const int c = sub + C::kTPT * ((jj + rot) % C::kCPL);
              const uint4 kv = lds128(ks + tk * C::kRB + c * 16);
              f2_t kf[EP2];
              DT::widen2(kv, kf);
#pragma unroll
              for (int g = 0; g < GQ; ++g)
#pragma unroll
                for (int e = 0; e < EP2; ++e) dot2[g] = f2_fma(qr[g][jj][e], kf[e], dot2[g]);
            }
          }
          float dot[GQ];
#pragma unroll
          for (int g = 0; g < GQ; ++g) {
            float lo, hi;
            f2_unpack(dot2[g], lo, hi);
            dot[g] = lo + hi;
          }
#pragma unroll
          for (int off = C::kTPT / 2; off >= 1; off >>= 1)
#pragma unroll
            for (int g = 0; g < GQ; ++g) dot[g] += __shfl_xor_sync(0xffffffffu, dot[g], off);
#pragma unroll
          for (int g = 0; g < GQ; ++g) s[g][pp] = (tk < ntok) ? dot[g] : -INFINITY;
        }

        // ---- online softmax update for this tile
        float alpha[GQ];
#pragma unroll
        for (int g = 0; g < GQ; ++g) {
          float bm = s[g][0];
#pragma unroll
          for (int pp = 1; pp < C::kNPASS; ++pp) bm = fmaxf(bm, s[g][pp]);
#pragma unroll
          for (int off = C::kTPT; off < 32; off <<= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, off));
          const float mn = fmaxf(m_run[g], bm);
          alpha[g] = exp2f(m_run[g] - mn);
          float sum = 0.f;
#pragma unroll
          for (int pp = 0; pp < C::kNPASS; ++pp) {
            const float e = exp2f(s[g][pp] - mn);
            s[g][pp] = e;
            sum += e;
          }
#pragma unroll
          for (int off = C::kTPT; off < 32; off <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
          l_run[g] = l_run[g] * alpha[g] + sum;
          m_run[g] = mn;
        }
        if (sub == 0) {
#pragma unroll
          for (int pp = 0; pp < C::kNPASS; ++pp) {
            const int tk = pp * C::kTPP + tp;
            if (tk < C::kMaxTT)
#pragma unroll
              for (int g = 0; g < GQ; ++g) psw[tk * GQ + g] = s[g][pp];
          }
        }
        __syncwarp();

        // ---- acc = acc * alpha + P.V
#pragma unroll
        for (int g = 0; g < GQ; ++g) {
          const f2_t a2 = f2_pack(alpha[g], alpha[g]);
#pragma unroll
          for (int e = 0; e < EP2; ++e) acc[g][e] = f2_mul(acc[g][e], a2);
        }
        if (pv_on) {
#pragma unroll 4
          for (int r = rg; r < ntok; r += C::kRPI) {
            const uint4 vv = lds128(vs + r * C::kRB + cpv * 16);
            f2_t vf[EP2];
            DT::widen2(vv, vf);
#pragma unroll
            for (int g = 0; g < GQ; ++g) {
              const float pg = psw[r * GQ + g];
              const f2_t p2 = f2_pack(pg, pg);
#pragma unroll
              for (int e = 0; e < EP2; ++e) acc[g][e] = f2_fma(p2, vf[e], acc[g][e]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }

    // ------------------------------------------------------------ combine
    if (C::kShflRed) {
#pragma unroll
      for (int off = C::kNCH; off < 32; off <<= 1)
#pragma unroll
        for (int g = 0; g < GQ; ++g)
#pragma unroll
          for (int e = 0; e < EP2; ++e) {
            float lo, hi, lo2, hi2;
            f2_unpack(acc[g][e], lo, hi);
            lo2 = __shfl_xor_sync(0xffffffffu, lo, off);
            hi2 = __shfl_xor_sync(0xffffffffu, hi, off);
            acc[g][e] = f2_pack(lo + lo2, hi + hi2);
          }
    }
    if (lane == 0) {
#pragma unroll
      for (int g = 0; g < GQ; ++g) {
        red_m[warp * GQ + g] = ok ? m_run[g] : -INFINITY;
        red_l[warp * GQ + g] = ok ? l_run[g] : 0.f;
      }
      if (!ok) atomicExch(&abort_flag, 1);
    }
    if (pv_on && (!C::kShflRed || rg == 0)) {
      const int rr = C::kShflRed ? 0 : rg;
#pragma unroll
      for (int g = 0; g < GQ; ++g)
#pragma unroll
        for (int e = 0; e < EP2; ++e) {
          float lo, hi;
          f2_unpack(acc[g][e], lo, hi);
          red_acc[((warp * C::kRedRows + rr) * GQ + g) * D + cpv * EPC + 2 * e] = lo;
          red_acc[((warp * C::kRedRows + rr) * GQ + g) * D + cpv * EPC + 2 * e + 1] = hi;
        }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(comb_full);
    if (!mbar_wait(comb_full, npieces & 1u, p.err)) return;

    const int64_t orow = p.out_rows ? p.out_rows[pc.row] : pc.row;
    for (int o = threadIdx.x; o < GQ * D; o += C::kNW * 32) {
      const int g = o / D;
      const int d = o - g * D;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < C::kNW; ++w) M = fmaxf(M, red_m[w * GQ + g]);
      float L = 0.f, O = 0.f;
#pragma unroll
      for (int w = 0; w < C::kNW; ++w) {
        const float sc = exp2f(red_m[w * GQ + g] - M);
        L += red_l[w * GQ + g] * sc;
        float a = 0.f;
#pragma unroll
        for (int r = 0; r < C::kRedRows; ++r) a += red_acc[((w * C::kRedRows + r) * GQ + g) * D + d];
        O += a * sc;
      }
      const float inv = 1.f / L;
      const float lse_nat = (M + log2f(L)) * kLn2;
      const int h = h0 + g;
      if (pc.whole) {
        if (orow >= 0) store_out(p.out, orow * p.out_sn + (int64_t)h * p.out_sh + d, p.out_dtype, O * inv);
        if (d == 0 && p.lse != nullptr) p.lse[(int64_t)h * p.lse_sh + (int64_t)pc.row * p.lse_sn] = lse_nat;
      } else {
        const int64_t pidx = p.persistent ? ((int64_t)blockIdx.x * 2 + pc.slot) * GQ + g
                                          : ((int64_t)pc.row * p.H + h) * p.max_splits + pc.slot;
        p.part_o[pidx * D + d] = O * inv;
        if (d == 0) p.part_lse[pidx] = lse_nat;
      }
    }
    // red_* is rewritten by the next piece
    __syncwarp();
    if (lane == 0) mbar_arrive(comb_done);
    if (!mbar_wait(comb_done, npieces & 1u, p.err)) return;
    ++npieces;
    if (abort_flag) return;
  }
  griddep_launch_dependents();  // this CTA's writes are issued: the combine may launch
}

// Split-grid schedule: combine the split partials of rows that needed more
// than one split.
__global__ void fd_split_merge_kernel(const __grid_constant__ DecodeParams p, int D) {
  extern __shared__ float wsm[];
  const int h = blockIdx.x;
  const int i = blockIdx.y;
  const int len = p.lens[i];
  if (len <= 0) return;
  const int nblk = (len + p.BS - 1) / p.BS;
  if (nblk > p.bt_width) return;
  const int ntiles = (len + p.TT - 1) / p.TT;
  const int ns = (ntiles + p.tiles_per_split - 1) / p.tiles_per_split;
  if (ns <= 1 || ns > p.max_splits) return;
  const int64_t base = ((int64_t)i * p.H + h) * p.max_splits;
  float M = -INFINITY;
  for (int s = 0; s < ns; ++s) M = fmaxf(M, p.part_lse[base + s]);
  for (int s = threadIdx.x; s < ns; s += blockDim.x) wsm[s] = exp2f((p.part_lse[base + s] - M) * kLog2e);
  __syncthreads();
  float L = 0.f;
  for (int s = 0; s < ns; ++s) L += wsm[s];
  const float inv = 1.f / L;
  const int64_t orow = p.out_rows ? p.out_rows[i] : i;
  for (int d = threadIdx.x; orow >= 0 && d < D; d += blockDim.x) {
    float O = 0.f;
    for (int s = 0; s < ns; ++s) O = fmaf(wsm[s], p.part_o[(base + s) * D + d], O);
    store_out(p.out, orow * p.out_sn + (int64_t)h * p.out_sh + d, p.out_dtype, O * inv);
  }
  if (threadIdx.x == 0 && p.lse != nullptr) p.lse[(int64_t)h * p.lse_sh + (int64_t)i * p.lse_sn] = M + logf(L);
}

// Persistent schedule: merge the segments that CTA ranges cut.  One CTA per
// decode CTA c: it merges the segment containing its range start when that
// segment began in an earlier CTA and its last real tile lies in c's range,
// so every cut segment is merged exactly once (by the CTA holding its last
// tile) and the grid stays at the decode kernel's CTA count instead of one
// CTA per (row, kv-head chunk) segment.  Slot rule: the first contributing
// CTA wrote into slot 0 if the segment was its first real piece, else slot
// 1; every later one into slot 0.
__global__ void fd_persistent_combine_kernel(const __grid_constant__ DecodeParams p, int D) {
  griddep_wait();  // launched early (programmatic dependent launch): the decode's partials first
  griddep_launch_dependents();  // a dependent (the sharded exchange) may launch and wait for this grid
  const int* P = p.ws_prefix;
  const int Y = p.KVH * p.gcs;
  const int64_t N = p.ncta;
  const int64_t T = (int64_t)P[p.n] * Y;
  const int64_t c = blockIdx.x;
  const int64_t ga = c * T / N, gb = (c + 1) * T / N;
  if (ga >= gb) return;
  int lo = 0, hi = p.n - 1;  // last row whose first position is <= ga
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if ((int64_t)P[mid] * Y <= ga) lo = mid; else hi = mid - 1;
  }
  const int i = lo;
  const int nv = P[i + 1] - P[i];
  if (nv == 0) return;
  const int nt = nv - p.vtiles;  // real tiles of the segment; the rest only weigh the split
  const int64_t local = ga - (int64_t)P[i] * Y;
  const int y = (int)(local / nv);
  const int t0 = (int)(local - (int64_t)y * nv);
  if (t0 == 0 || t0 >= nt) return;  // starts here, or only weight positions left
  const int64_t g0 = (int64_t)P[i] * Y + (int64_t)y * nv;
  if (g0 + nt - 1 >= gb) return;  // continues into a later CTA, which merges it
  // CTAs c0 (owning position g0) .. c (this one, owning the last real tile)
  // wrote partials; c0 into slot first_slot (seg_span)
  const SegSpan sp = seg_span(P, Y, p.vtiles, N, T, i, y);
  const int64_t c0 = sp.c0;
  const int64_t c1 = c;
  const int first_slot = sp.first_slot;
  const int GQ = p.gq;
  const int kh = y / p.gcs, gc = y - kh * p.gcs;
  const int h0 = kh * p.G + gc * GQ;
  const int64_t orow = p.out_rows ? p.out_rows[i] : i;
  for (int o = threadIdx.x; o < GQ * D; o += blockDim.x) {
    const int g = o / D, d = o - g * D;
    float M = -INFINITY;
    for (int64_t cc = c0; cc <= c1; ++cc) {
      if ((cc * T) / N == ((cc + 1) * T) / N) continue;
      const int64_t s = (cc * 2 + (cc == c0 ? first_slot : 0)) * GQ + g;
      M = fmaxf(M, p.part_lse[s]);
    }
    float L = 0.f, O = 0.f;
    for (int64_t cc = c0; cc <= c1; ++cc) {
      if ((cc * T) / N == ((cc + 1) * T) / N) continue;
      const int64_t s = (cc * 2 + (cc == c0 ? first_slot : 0)) * GQ + g;
      const float w = exp2f((p.part_lse[s] - M) * kLog2e);
      L += w;
      O = fmaf(w, p.part_o[s * D + d], O);
    }
    const int h = h0 + g;
    if (orow >= 0) store_out(p.out, orow * p.out_sn + (int64_t)h * p.out_sh + d, p.out_dtype, O / L);
    if (d == 0 && p.lse != nullptr) p.lse[(int64_t)h * p.lse_sh + (int64_t)i * p.lse_sn] = M + logf(L);
  }
}

}  // namespace fdk

// ============================================================== host side

namespace {

using fdk::Cfg;
using fdk::DecodeParams;

constexpr int kTargetCtas = 148 * 2 * 8;  // split grid: ~8 waves at 2 CTAs per SM

struct Geometry {
  int TT, tiles_per_block, tiles_per_split, max_splits, G, GQ, gcs;
  bool persistent;
  bool mma;  // tcgen05 GQA kernel (fd_decode_mma.cu)
  int vtiles;  // persistent schedule: weight positions per (row, kv-head chunk) segment
  size_t ws_bytes;
  // persistent workspace layout: partial o | partial lse | row-tile prefix
  size_t off_lse, off_prefix;
};

// launch(p, grid, extra dynamic smem, stream, programmatic dependent launch)
// / resident CTAs per SM
typedef int (*launch_fn)(const DecodeParams&, dim3, size_t, cudaStream_t, bool);
typedef int (*occ_fn)(int*);

template <typename T, int D, int GQ>
int launch_impl(const DecodeParams& p, dim3 grid, size_t extra, cudaStream_t s, bool pdl) {
  using C = Cfg<T, D, GQ>;
  static unsigned long long done = 0;
  auto kern = fdk::fd_decode_kernel<T, D, GQ>;
  int st = fdh::ensure_smem(reinterpret_cast<const void*>(kern), C::kSmem + C::kPrefixMax, &done);
  if (st != FD_OK) return st;
  return fdh::launch_maybe_pdl(reinterpret_cast<const void*>(kern), grid, dim3(C::kThreads), C::kSmem + extra, s,
                               pdl, p, "fd_decode_kernel launch");
}

// resident CTAs per SM of this kernel (queried once per device)
template <typename T, int D, int GQ>
int occupancy_impl(int* per_sm) {
  using C = Cfg<T, D, GQ>;
  static unsigned long long done = 0;
  static int cached[64] = {0};
  auto kern = fdk::fd_decode_kernel<T, D, GQ>;
  int st = fdh::ensure_smem(reinterpret_cast<const void*>(kern), C::kSmem + C::kPrefixMax, &done);
  if (st != FD_OK) return st;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fdh::cuda_status(e, "cudaGetDevice");
  if (dev >= 0 && dev < 64) {
    const int c = __atomic_load_n(&cached[dev], __ATOMIC_RELAXED);
    if (c > 0) {
      *per_sm = c;
      return FD_OK;
    }
  }
  st = fdh::cuda_status(cudaOccupancyMaxActiveBlocksPerMultiprocessor(per_sm, kern, C::kThreads,
                                                                      C::kSmem + C::kPrefixMax),
                        "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
  if (st == FD_OK && *per_sm > 0 && dev >= 0 && dev < 64) __atomic_store_n(&cached[dev], *per_sm, __ATOMIC_RELAXED);
  return st;
}

struct KernelFns {
  launch_fn launch;
  occ_fn occupancy;
};

template <typename T, int D, int GQ>
constexpr KernelFns pick() {
  if constexpr (Cfg<T, D, GQ>::kValid) {
    return KernelFns{&launch_impl<T, D, GQ>, &occupancy_impl<T, D, GQ>};
  } else {
    return KernelFns{nullptr, nullptr};
  }
}

template <typename T, int D>
KernelFns pick_gq(int gq) {
  switch (gq) {
    case 1:
      return pick<T, D, 1>();
    case 2:
      return pick<T, D, 2>();
    case 4:
      return pick<T, D, 4>();
    default:
      return KernelFns{nullptr, nullptr};
  }
}

template <typename T>
KernelFns pick_d(int D, int gq) {
  switch (D) {
    case 64:
      return pick_gq<T, 64>(gq);
    case 72:
      return pick_gq<T, 72>(gq);
    case 96:
      return pick_gq<T, 96>(gq);
    case 128:
      return pick_gq<T, 128>(gq);
    case 256:
      return pick_gq<T, 256>(gq);
    default:
      return KernelFns{nullptr, nullptr};
  }
}

KernelFns pick_kernel(int dtype, int D, int gq) {
  switch (dtype) {
    case FD_DTYPE_F16:
      return pick_d<__half>(D, gq);
    case FD_DTYPE_BF16:
      return pick_d<__nv_bfloat16>(D, gq);
    case FD_DTYPE_F32:
      return pick_d<float>(D, gq);
    default:
      return KernelFns{nullptr, nullptr};
  }
}

// Largest query-head group per CTA (4, 2 or 1) that divides G and is built.
int choose_gq(int dtype, int D, int G) {
  const int opts[3] = {4, 2, 1};
  for (int gq : opts)
    if (G % gq == 0 && pick_kernel(dtype, D, gq).launch != nullptr) return gq;
  return 0;
}

int geometry(const fd_decode_args* a, Geometry* g) {
  const int BS = a->block_size;
  if (BS <= 0) return fdh::fail(FD_ERR_INVALID, "block_size must be positive, got %d", BS);
  if (BS > 16 && BS % 16 != 0)
    return fdh::fail(FD_ERR_UNSUPPORTED, "block_size %d: above 16 it must be a multiple of 16", BS);
  if (a->num_kv_heads <= 0 || a->num_heads <= 0 || a->num_heads % a->num_kv_heads != 0)
    return fdh::fail(FD_ERR_INVALID, "num_heads must be a multiple of num_kv_heads");
  g->TT = BS <= 16 ? BS : 16;
  g->tiles_per_block = BS / g->TT;
  g->G = a->num_heads / a->num_kv_heads;
  g->GQ = choose_gq(a->dtype, a->head_size, g->G);
  if (g->GQ == 0)
    return fdh::fail(FD_ERR_UNSUPPORTED, "no decode kernel for dtype %d head_size %d", a->dtype,
                     a->head_size);
  g->gcs = g->G / g->GQ;
  const int64_t max_len =
      a->max_len > 0 ? (int64_t)a->max_len : (int64_t)a->bt_width * (int64_t)BS;
  const int64_t ntiles_max = std::max<int64_t>(1, (max_len + g->TT - 1) / g->TT);
  g->persistent = (a->tiles_per_split <= 0 && a->n > 0 && a->n <= fdk::kMaxPersistentRows);
  g->off_lse = g->off_prefix = 0;
  const char* mma_env = getenv("FASTDECODE_B200_MMA");
  g->mma = g->persistent && fdk::mma_eligible(a->dtype, a->head_size, g->G, BS) &&
           !(mma_env != nullptr && mma_env[0] == '0');
  if (g->mma) {  // one CTA handles the whole query group of a kv head
    g->GQ = g->G;
    g->gcs = 1;
  }
  // A piece costs its stages plus a fixed overhead (q load, the last stage's
  // round trip, the epilogue, and a last stage that is on average half
  // empty).  Measured on B200 (lognormal lengths for the tensor-core kernel,
  // uniform ones for the CUDA-core kernel), the balance is best at a weight
  // of 16 tiles per segment for the tensor-core kernel (8-tile stages, four
  // producer warps) and 5 for the CUDA-core kernel (4-tile stages);
  // FASTDECODE_B200_VTILES overrides it.
  g->vtiles = 0;
  if (g->persistent) {
    g->vtiles = g->mma ? 16 : 5;
    const char* vt_env = getenv("FASTDECODE_B200_VTILES");
    if (vt_env != nullptr && vt_env[0] >= '0' && vt_env[0] <= '9') g->vtiles = std::min(atoi(vt_env), 64);
  }
  if (g->persistent) {
    // every CTA owns two partial slots of GQ heads
    const size_t slots = (size_t)fdk::kMaxPersistentCtas * 2 * (size_t)g->GQ;
    g->tiles_per_split = 0;
    g->max_splits = 1;
    g->off_lse = (slots * (size_t)a->head_size * 4 + 255) / 256 * 256;
    g->off_prefix = g->off_lse + (slots * 4 + 255) / 256 * 256;
    g->ws_bytes = g->off_prefix + ((size_t)(a->n + 1) * 4 + 255) / 256 * 256;
    return FD_OK;
  }
  int64_t tps = a->tiles_per_split;
  if (tps <= 0) {
    const int64_t ctas_per_row = (int64_t)a->num_kv_heads * g->gcs;
    const int64_t est = (int64_t)std::max(a->n, 1) * ctas_per_row * ntiles_max;
    tps = std::max<int64_t>(8, (est + kTargetCtas - 1) / kTargetCtas);
  }
  tps = (tps + 3) / 4 * 4;  // whole stages of the 4 consumer warps
  g->tiles_per_split = (int)std::min<int64_t>(tps, 1 << 30);
  g->max_splits = (int)((ntiles_max + tps - 1) / tps);
  g->ws_bytes = 0;
  if (g->max_splits > 1) {
    const size_t rows = (size_t)a->n * (size_t)a->num_heads * (size_t)g->max_splits;
    const size_t o_bytes = (rows * (size_t)a->head_size * 4 + 255) / 256 * 256;
    g->ws_bytes = o_bytes + (rows * 4 + 255) / 256 * 256;
  }
  return FD_OK;
}

}  // namespace

extern "C" size_t fd_decode_workspace_size(const fd_decode_args* a) {
  if (a == nullptr || a->n <= 0) return 0;
  Geometry g;
  if (geometry(a, &g) != FD_OK) return 0;
  return g.ws_bytes;
}

namespace {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    else
      cudaGetLastError();
  });
  return fn;
}

// Describe one K or V view of a device tier as a 4-D tensor {D, KVH, BS,
// blocks} with byte strides {head, token, block} and a box of one tile
// {D, 1, TT, 1}.  Returns false when the driver rejects it (the caller then
// copies tile rows one by one).
bool encode_tier_map_uncached(CUtensorMap* m, const void* base, int dtype, int D, int KVH, int BS, int64_t nblk,
                              int64_t head_sb, int64_t tok_sb, int64_t blk_sb, int TT, bool swizzle128, int BH) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (enc == nullptr || nblk <= 0 || nblk > (int64_t)0xffffffff) return false;
  CUtensorMapDataType dt = dtype == FD_DTYPE_F16    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                           : dtype == FD_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                    : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)KVH, (cuuint64_t)BS, (cuuint64_t)nblk};
  const cuuint64_t strides[3] = {(cuuint64_t)head_sb, (cuuint64_t)tok_sb, (cuuint64_t)blk_sb};
  // swizzled: 128-byte box rows (64 16-bit dims), the layout the UMMA reads
  const cuuint32_t box[4] = {swizzle128 ? 64u : (cuuint32_t)D, (cuuint32_t)BH, (cuuint32_t)TT, 1u};
  const cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  const CUresult r = enc(m, dt, 4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Tensor maps of the recently used K/V views (a KV cache lives for the whole
// run, so the same few views come back every call): encoding one is a driver
// call of about a microsecond.  The key is every input of the encoding.
struct TmapKey {
  const void* base;
  int64_t nblk, head_sb, tok_sb, blk_sb;
  int dtype, D, KVH, BS, TT, swizzle, BH;
};

bool encode_tier_map(CUtensorMap* m, const void* base, int dtype, int D, int KVH, int BS, int64_t nblk,
                     int64_t head_sb, int64_t tok_sb, int64_t blk_sb, int TT, bool swizzle128 = false,
                     int BH = 1) {
  constexpr int kSlots = 32;
  struct Entry {
    TmapKey key;
    CUtensorMap map;
    bool used;
  };
  static Entry cache[kSlots];
  static int next = 0;
  static std::mutex mu;
  TmapKey key;
  memset(&key, 0, sizeof(key));  // padding bytes take part in the comparison
  key.base = base;
  key.nblk = nblk;
  key.head_sb = head_sb;
  key.tok_sb = tok_sb;
  key.blk_sb = blk_sb;
  key.dtype = dtype;
  key.D = D;
  key.KVH = KVH;
  key.BS = BS;
  key.TT = TT;
  key.swizzle = swizzle128 ? 1 : 0;
  key.BH = BH;
  {
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < kSlots; ++i)
      if (cache[i].used && memcmp(&cache[i].key, &key, sizeof(key)) == 0) {
        *m = cache[i].map;
        return true;
      }
  }
  if (!encode_tier_map_uncached(m, base, dtype, D, KVH, BS, nblk, head_sb, tok_sb, blk_sb, TT, swizzle128, BH))
    return false;
  std::lock_guard<std::mutex> lock(mu);
  Entry& e = cache[next];
  next = (next + 1) % kSlots;
  e.key = key;
  e.map = *m;
  e.used = true;
  return true;
}

}  // namespace

namespace fdk {
// Cached 4-D tiled tensor map {D, heads, BS, blocks} with box {64 or D,
// box_heads, box_tokens, 1} (the encoder the decode kernels use), for the
// prefill kernel.
bool encode_kv_map(CUtensorMap* m, const void* base, int dtype, int D, int heads, int BS, int64_t nblk,
                   int64_t head_sb, int64_t tok_sb, int64_t blk_sb, int box_tokens, bool swizzle128, int box_heads) {
  return encode_tier_map(m, base, dtype, D, heads, BS, nblk, head_sb, tok_sb, blk_sb, box_tokens, swizzle128,
                         box_heads);
}
}  // namespace fdk

namespace {

// Validate `a` and fill the kernel parameters; launch_main / launch_combine
// select which of the two kernels run.
int decode_impl(const fd_decode_args* a, void* stream, bool launch_main, bool launch_combine,
                void* ws_override = nullptr, size_t ws_override_bytes = 0, fdk::ShardGeom* geom = nullptr) {
  if (geom != nullptr) geom->prefix = nullptr;
  if (a == nullptr) return fdh::fail(FD_ERR_INVALID, "fd_decode_attn: null args");
  if (a->n < 0) return fdh::fail(FD_ERR_INVALID, "n must be >= 0");
  if (a->n == 0) return FD_OK;
  const int es = fdh::elem_size(a->dtype);
  if (es == 0) return fdh::fail(FD_ERR_UNSUPPORTED, "unsupported dtype %d", a->dtype);
  if (a->out_dtype != a->dtype && a->out_dtype != FD_DTYPE_F32)
    return fdh::fail(FD_ERR_UNSUPPORTED, "out_dtype must equal dtype or be FD_DTYPE_F32");
  if (a->q == nullptr || a->out == nullptr || a->block_table == nullptr || a->lens == nullptr)
    return fdh::fail(FD_ERR_INVALID, "q, out, block_table and lens are required");
  if (a->bt_width <= 0) return fdh::fail(FD_ERR_INVALID, "bt_width must be positive");
  if (a->n > 65535) return fdh::fail(FD_ERR_UNSUPPORTED, "at most 65535 rows per call");
  Geometry g;
  int st = geometry(a, &g);
  if (st != FD_OK) return st;
  const int D = a->head_size;
  const int64_t row_bytes = (int64_t)D * es;
  if (row_bytes % 16 != 0) return fdh::fail(FD_ERR_ALIGN, "head_size*elem_size must be a multiple of 16");
  if (!fdh::aligned16(a->q) || (a->q_stride_h * es) % 16 != 0 || (a->q_stride_n * es) % 16 != 0)
    return fdh::fail(FD_ERR_ALIGN, "q pointer and strides must be 16-byte aligned");

  DecodeParams p{};
  p.q = static_cast<const unsigned char*>(a->q);
  p.q_sn = a->q_stride_n * es;
  p.q_sh = a->q_stride_h * es;
  p.q_rows = a->q_rows;
  for (int t = 0; t < 2; ++t) {
    const fd_kv_tier& tr = a->tier[t];
    p.k[t] = static_cast<const unsigned char*>(tr.k);
    p.v[t] = static_cast<const unsigned char*>(tr.v);
    p.blk_sb[t] = tr.blk_stride * es;
    p.head_sb[t] = tr.head_stride * es;
    p.tok_sb[t] = tr.tok_stride * es;
    p.nblk[t] = tr.num_blocks > 0 ? tr.num_blocks : 0;
    p.host[t] = tr.host_mapped ? 1 : 0;
    p.contig[t] = (p.tok_sb[t] == row_bytes) ? 1 : 0;
    p.use_tmap[t] = 0;
    if (p.nblk[t] > 0) {
      if (tr.k == nullptr || tr.v == nullptr)
        return fdh::fail(FD_ERR_INVALID, "tier %d has blocks but no K/V pointer", t);
      if (!fdh::aligned16(tr.k) || !fdh::aligned16(tr.v) || p.blk_sb[t] % 16 != 0 ||
          p.head_sb[t] % 16 != 0 || p.tok_sb[t] % 16 != 0)
        return fdh::fail(FD_ERR_ALIGN, "tier %d K/V pointers and strides must be 16-byte aligned", t);
      if (!p.host[t] && (!p.contig[t] || g.mma)) {
        const bool ok_k = encode_tier_map(&p.tmap_k[t], tr.k, a->dtype, D, a->num_kv_heads, a->block_size,
                                          p.nblk[t], p.head_sb[t], p.tok_sb[t], p.blk_sb[t], g.TT, g.mma);
        const bool ok_v = ok_k && encode_tier_map(&p.tmap_v[t], tr.v, a->dtype, D, a->num_kv_heads,
                                                  a->block_size, p.nblk[t], p.head_sb[t], p.tok_sb[t],
                                                  p.blk_sb[t], g.TT, g.mma);
        p.use_tmap[t] = (ok_k && ok_v) ? 1 : 0;
        if (g.mma && !p.use_tmap[t]) {
          // the tensor-core kernel needs swizzled tiles: use the CUDA-core kernel
          g.mma = false;
          g.GQ = choose_gq(a->dtype, D, g.G);
          g.gcs = g.G / g.GQ;
          t = -1;  // re-encode every tier for the CUDA-core kernel
          continue;
        }
      }
    }
  }
  p.split = a->tier_split;
  p.bt = a->block_table;
  p.bt_stride = a->bt_stride;
  p.bt_width = a->bt_width;
  p.lens = a->lens;
  p.n = a->n;
  p.H = a->num_heads;
  p.KVH = a->num_kv_heads;
  p.BS = a->block_size;
  p.G = g.G;
  p.gcs = g.gcs;
  p.TT = g.TT;
  p.tiles_per_block = g.tiles_per_block;
  p.tiles_per_split = g.tiles_per_split;
  p.max_splits = g.max_splits;
  p.qscale = a->scale * fdk::kLog2e;
  p.out = a->out;
  p.out_dtype = a->out_dtype;
  p.out_sn = a->out_stride_n;
  p.out_sh = a->out_stride_h;
  p.out_rows = a->out_rows;
  p.bt_rows = a->bt_rows;
  p.lse = a->lse;
  p.lse_sh = a->lse_stride_h;
  p.lse_sn = a->lse_stride_n;
  p.err = a->error;
  p.gq = g.GQ;
  if (g.ws_bytes > 0) {
    void* ws = ws_override != nullptr ? ws_override : a->workspace;
    const size_t ws_bytes = ws_override != nullptr ? ws_override_bytes : a->workspace_bytes;
    if (ws == nullptr || ws_bytes < g.ws_bytes)
      return fdh::fail(FD_ERR_WORKSPACE, "workspace of %zu bytes needed, got %zu", g.ws_bytes, ws_bytes);
    if ((reinterpret_cast<uintptr_t>(ws) & 255u) != 0)
      return fdh::fail(FD_ERR_ALIGN, "workspace must be 256-byte aligned");
    unsigned char* wb = static_cast<unsigned char*>(ws);
    if (g.persistent) {
      p.part_o = reinterpret_cast<float*>(wb);
      p.part_lse = reinterpret_cast<float*>(wb + g.off_lse);
      p.ws_prefix = reinterpret_cast<int*>(wb + g.off_prefix);
    } else {
      const size_t rows = (size_t)a->n * (size_t)a->num_heads * (size_t)g.max_splits;
      const size_t o_bytes = (rows * (size_t)D * 4 + 255) / 256 * 256;
      p.part_o = reinterpret_cast<float*>(wb);
      p.part_lse = reinterpret_cast<float*>(wb + o_bytes);
    }
  }
  if ((int64_t)a->num_kv_heads * g.gcs > 65535)
    return fdh::fail(FD_ERR_UNSUPPORTED, "too many heads for the grid");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const KernelFns fns = pick_kernel(a->dtype, D, g.GQ);
  const bool pdl = (a->flags & FD_DECODE_PDL) != 0;
  if (g.persistent) {
    // as many CTAs as fit on the device at once (capped by the partial slots
    // and by the tile count, at least 16 tiles each)
    int dev = 0, sms = 0, per_sm = 0;
    st = fdh::device_sms(&dev, &sms);
    if (st != FD_OK) return st;
    if (g.mma) {
      per_sm = 1;  // the tensor-core kernel takes most of an SM's shared memory
    } else {
      st = fns.occupancy(&per_sm);
      if (st != FD_OK) return st;
    }
    const int64_t max_len =
        a->max_len > 0 ? (int64_t)a->max_len : (int64_t)a->bt_width * (int64_t)a->block_size;
    const int64_t tiles_max = (int64_t)a->n * ((max_len + g.TT - 1) / g.TT) * a->num_kv_heads * g.gcs;
    int64_t ncta = std::min<int64_t>((int64_t)std::max(1, sms * std::max(1, per_sm)), fdk::kMaxPersistentCtas);
    ncta = std::max<int64_t>(1, std::min<int64_t>(ncta, (tiles_max + 15) / 16));
    p.persistent = 1;
    p.ncta = (int)ncta;
    p.vtiles = g.vtiles;
    const size_t extra = ((size_t)(a->n + 1) * 4 + 15) / 16 * 16;
    if (g.mma) {
      // the tensor-core kernel runs one CTA per SM; the combine must see the
      // same CTA count, so it is computed even when only combining
      int n_mma = (int)ncta;
      bool launched = false;
      DecodeParams pm = p;
      pm.ncta = n_mma;
      if (launch_main) {
        st = fdk::launch_decode_mma(pm, a->dtype, D, extra, s, &n_mma, &launched, pdl);
        if (st != FD_OK) return st;
        if (!launched) return fdh::fail(FD_ERR_UNSUPPORTED, "tensor-core decode kernel declined the call");
      } else {
        n_mma = std::max(1, std::min((int)ncta, std::min(sms, fdk::kMaxPersistentCtas)));
      }
      p.ncta = n_mma;
      ncta = n_mma;
    } else if (launch_main) {
      st = fns.launch(p, dim3((unsigned)ncta), extra, s, pdl);
      if (st != FD_OK) return st;
    }
    if (geom != nullptr) {
      // the consumer merges the cut segments itself: no combine launch
      geom->prefix = p.ws_prefix;
      geom->part_o = p.part_o;
      geom->part_lse = p.part_lse;
      geom->ncta = (int)ncta;
      geom->vtiles = p.vtiles;
      geom->KVH = p.KVH;
      geom->gcs = p.gcs;
      geom->G = p.G;
      geom->GQ = g.GQ;
      return st;
    }
    if (launch_combine && ncta > 1) {
      // programmatic dependent launch: the combine's launch overlaps the
      // decode's last CTAs; the kernel waits for the decode grid before
      // reading its partials
      const int threads = g.GQ * D <= 128 ? 128 : 256;
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3((unsigned)ncta);
      cfg.blockDim = dim3((unsigned)threads);
      cfg.dynamicSmemBytes = 0;
      cfg.stream = s;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[0].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      st = fdh::cuda_status(cudaLaunchKernelEx(&cfg, fdk::fd_persistent_combine_kernel, p, D),
                            "fd_persistent_combine_kernel launch");
    }
    return st;
  }
  if (launch_main) {
    dim3 grid(g.max_splits, a->num_kv_heads * g.gcs, a->n);
    st = fns.launch(p, grid, 0, s, pdl);
    if (st != FD_OK) return st;
  }
  if (launch_combine && g.max_splits > 1) {
    const int threads = D <= 128 ? 128 : 256;
    const size_t sm = (size_t)g.max_splits * sizeof(float);
    if (sm > 48 * 1024) return fdh::fail(FD_ERR_UNSUPPORTED, "too many splits (%d)", g.max_splits);
    fdk::fd_split_merge_kernel<<<dim3(a->num_heads, a->n), threads, sm, s>>>(p, D);
    st = fdh::cuda_status(cudaGetLastError(), "fd_split_merge_kernel launch");
  }
  return st;
}

}  // namespace

extern "C" int fd_decode_attn(const fd_decode_args* a, void* stream) {
  return decode_impl(a, stream, true, true);
}

extern "C" int fd_decode_attn_partials(const fd_decode_args* a, void* stream) {
  return decode_impl(a, stream, true, false);
}

extern "C" int fd_decode_attn_combine(const fd_decode_args* a, void* stream) {
  return decode_impl(a, stream, false, true);
}

namespace fdk {
int launch_decode_for_exchange(const fd_decode_args* a, void* stream, ShardGeom* geom, bool decode) {
  return decode_impl(a, stream, decode, true, nullptr, 0, geom);
}
}  // namespace fdk

// ------------------------------------------------------------ no-allocation variant

// Scratch of fd_decode_attn_noalloc: a file-scope device array, so the entry
// point needs no cudaMalloc.  Every GPU that loads this library holds these
// FD_NOALLOC_SCRATCH_BYTES until the process exits.  In host code the name is
// only a handle for cudaGetSymbolAddress, never a device address.
static __device__ __align__(256) unsigned char g_noalloc_scratch[FD_NOALLOC_SCRATCH_BYTES];

namespace {
std::mutex g_noalloc_mu;
// Device address of g_noalloc_scratch per device ordinal, with the CUDA
// context it was looked up in: a context torn down and created again
// (cudaDeviceReset) loads the module afresh, so the address is looked up
// again whenever the current context differs from the cached one.
struct NoallocSlot {
  void* ctx;
  void* addr;
};
NoallocSlot g_noalloc_slot[64] = {};

typedef CUresult (*ctx_get_current_fn)(CUcontext*);

ctx_get_current_fn ctx_get_current() {
  static ctx_get_current_fn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<ctx_get_current_fn>(f);
    else
      cudaGetLastError();
  });
  return fn;
}

// Device address of the scratch on the current device: looked up with the
// device current on the first call in each CUDA context, then cached.
int noalloc_scratch(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fdh::cuda_status(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fdh::fail(FD_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  CUcontext ctx = nullptr;
  ctx_get_current_fn get = ctx_get_current();
  if (get == nullptr || get(&ctx) != CUDA_SUCCESS)
    return fdh::fail(FD_ERR_CUDA, "fd_decode_attn_noalloc: cuCtxGetCurrent unavailable");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  NoallocSlot& slot = g_noalloc_slot[dev];
  if (slot.addr == nullptr || ctx == nullptr || slot.ctx != static_cast<void*>(ctx)) {
    // no context current on this thread yet, or another one than the cached
    // address belongs to: the lookup makes the device's context current
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return fdh::cuda_status(e, "cudaGetSymbolAddress(no-alloc scratch)");
    if (get(&ctx) != CUDA_SUCCESS || ctx == nullptr)
      return fdh::fail(FD_ERR_CUDA, "fd_decode_attn_noalloc: no current CUDA context");
    slot.ctx = static_cast<void*>(ctx);
    slot.addr = p;
  }
  *out = slot.addr;
  return FD_OK;
}
}  // namespace

extern "C" int fd_decode_attn_noalloc(const fd_decode_args* a, void* stream) {
  if (a == nullptr) return fdh::fail(FD_ERR_INVALID, "fd_decode_attn_noalloc: null args");
  if (a->n <= 0) return decode_impl(a, stream, true, true);
  Geometry g;
  const int st = geometry(a, &g);
  if (st != FD_OK) return st;
  if (g.ws_bytes > (size_t)FD_NOALLOC_SCRATCH_BYTES)
    return fdh::fail(FD_ERR_WORKSPACE,
                     "fd_decode_attn_noalloc: these arguments need %zu bytes of split scratch but the "
                     "built-in scratch holds %zu (FD_NOALLOC_SCRATCH_BYTES); use fd_decode_attn with a "
                     "caller workspace, or a larger tiles_per_split",
                     g.ws_bytes, (size_t)FD_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  if (g.ws_bytes > 0) {
    const int rc = noalloc_scratch(&scratch);
    if (rc != FD_OK) return rc;
  }
  return decode_impl(a, stream, true, true, scratch, (size_t)FD_NOALLOC_SCRATCH_BYTES);
}

namespace {
void paged_args(fd_decode_args* a, const void* q, const void* k_cache, const void* v_cache,
                int32_t cache_is_host, const int32_t* block_table, const int32_t* lens, int32_t n,
                int32_t H, int32_t KVH, int32_t D, int32_t BS, int64_t num_blocks, int32_t W,
                float scale, int32_t dtype, void* out, float* lse, void* ws, size_t ws_bytes,
                int32_t* error) {
  *a = fd_decode_args{};
  a->q = q;
  a->q_stride_n = (int64_t)H * D;
  a->q_stride_h = D;
  a->tier[0].k = const_cast<void*>(k_cache);
  a->tier[0].v = const_cast<void*>(v_cache);
  a->tier[0].blk_stride = (int64_t)KVH * BS * D;
  a->tier[0].head_stride = (int64_t)BS * D;
  a->tier[0].tok_stride = D;
  a->tier[0].num_blocks = num_blocks;
  a->tier[0].host_mapped = cache_is_host;
  a->tier_split = INT64_MAX;
  a->block_table = block_table;
  a->bt_stride = W;
  a->bt_width = W;
  a->lens = lens;
  a->n = n;
  a->num_heads = H;
  a->num_kv_heads = KVH;
  a->head_size = D;
  a->block_size = BS;
  a->scale = scale;
  a->dtype = dtype;
  a->out = out;
  a->out_dtype = dtype;
  a->out_stride_n = (int64_t)H * D;
  a->out_stride_h = D;
  a->lse = lse;
  a->lse_stride_h = n;
  a->lse_stride_n = 1;
  a->workspace = ws;
  a->workspace_bytes = ws_bytes;
  a->error = error;
}
}  // namespace

extern "C" size_t fd_decode_attn_paged_workspace_size(int32_t n, int32_t num_heads,
                                                      int32_t num_kv_heads, int32_t head_size,
                                                      int32_t block_size, int32_t bt_width,
                                                      int32_t dtype) {
  fd_decode_args a;
  paged_args(&a, nullptr, nullptr, nullptr, 0, nullptr, nullptr, n, num_heads, num_kv_heads,
             head_size, block_size, 0, bt_width, 1.f, dtype, nullptr, nullptr, nullptr, 0,
             nullptr);
  return fd_decode_workspace_size(&a);
}

extern "C" int fd_decode_attn_paged(const void* q, const void* k_cache, const void* v_cache,
                                    int32_t cache_is_host, const int32_t* block_table,
                                    const int32_t* lens, int32_t n, int32_t num_heads,
                                    int32_t num_kv_heads, int32_t head_size, int32_t block_size,
                                    int64_t num_blocks, int32_t bt_width, float scale,
                                    int32_t dtype, void* out, float* lse, void* workspace,
                                    size_t workspace_bytes, int32_t* error, void* stream) {
  fd_decode_args a;
  paged_args(&a, q, k_cache, v_cache, cache_is_host, block_table, lens, n, num_heads,
             num_kv_heads, head_size, block_size, num_blocks, bt_width, scale, dtype, out, lse,
             workspace, workspace_bytes, error);
  return fd_decode_attn(&a, stream);
}
