// Kernel parameters and schedule constants shared by the decode kernels
// (the CUDA-core kernel in fd_decode.cu and the tcgen05 GQA kernel in
// fd_decode_mma.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "fd_common.cuh"

namespace fdk {

struct alignas(64) DecodeParams {
  // tiled-TMA descriptors of device tiers whose tiles are not contiguous
  // (dims {D, KVH, BS, blocks}, box {D, 1, TT, 1}); used when use_tmap[t]
  CUtensorMap tmap_k[2];
  CUtensorMap tmap_v[2];
  int use_tmap[2];
  const unsigned char* q;
  int64_t q_sn, q_sh;  // bytes
  const int64_t* q_rows;
  const unsigned char* k[2];
  const unsigned char* v[2];
  int64_t blk_sb[2], head_sb[2], tok_sb[2];  // bytes
  int64_t nblk[2];
  int host[2];
  int contig[2];
  int64_t split;
  const int32_t* bt;
  const int32_t* bt_rows;  // optional: work row i reads table row bt_rows[i]
  int64_t bt_stride;
  int bt_width;
  const int32_t* lens;
  int n, H, KVH, BS, G, gcs, gq;
  int TT, tiles_per_block, tiles_per_split, max_splits;
  // persistent schedule: ncta CTAs share the flattened (row, kv-head chunk,
  // tile) space evenly; prefix of per-row tile counts published in ws_prefix
  int persistent, ncta;
  // per-(row, kv-head chunk) cost of a piece in tile units: every segment of
  // nt tiles occupies nt + vtiles positions of the flattened space, so the
  // equal split also balances per-piece overheads (the extra positions carry
  // no work)
  int vtiles;
  int* ws_prefix;
  float qscale;  // scale * log2(e)
  void* out;
  int out_dtype;
  int64_t out_sn, out_sh;  // elements
  const int64_t* out_rows;
  float* lse;
  int64_t lse_sh, lse_sn;
  float* part_o;
  float* part_lse;
  int32_t* err;
};

// Largest row count handled by the persistent schedule (its per-row tile
// prefix sits in shared memory).
constexpr int kMaxPersistentRows = 1024;
// Upper bound on persistent CTAs (2 per SM on 148 SMs, with headroom); sizes
// the partial slots of the workspace.
constexpr int kMaxPersistentCtas = 320;

// One piece of work: tiles [t0, t1) of row `row` for kv-head chunk y.  A piece
// covering its whole (row, chunk) segment writes the final output; otherwise
// it writes an fp32 partial into `slot`.
struct Piece {
  int row, y, t0, t1, len, slot;
  int trow;  // block-table row of `row` (bt_rows indirection)
  bool whole;
};

// Enumerates one CTA's stages (up to `tps` consecutive tiles of one piece):
// the pieces of its persistent range [g0, g1) of the flattened space, or the
// single piece of a split-grid CTA.  In the flattened space each (row, y)
// segment has prefix[row+1] - prefix[row] = nt + vtiles positions: nt real
// tiles, then vtiles positions that only weigh the split; a piece consisting
// of those alone is skipped.  A CTA's first real piece takes partial slot 0,
// later ones slot 1 (only its first and last piece can be partial).  Every
// role of a kernel runs its own copy over the same sequence.  prefix/lens
// may live in shared memory; lens may be null when the caller does not need
// Piece::len.
// Warm L2 with the block-table rows a CTA of a persistent launch is likely
// to start in, while the row lengths load (the first block ids are then an L2
// hit instead of a DRAM round trip): the whole table when it spans at most 64
// lines, else the rows around the CTA's even share of rows.  A hint only:
// the rows actually read come from the prefix.  Every address lies within a
// row's first bt_width entries.  Measured on B200: config 2 (tensor-core
// kernel) 0.2395 -> 0.2377 ms; the CUDA-core kernel on configs 0 and 1 lost
// ~0.5 %, so only the tensor-core kernel calls it.
__device__ __forceinline__ void warm_block_table(const DecodeParams& p) {
  if (p.bt_rows != nullptr || p.n <= 0) return;  // table rows of a device-built list are not known yet
  const int lpr = (p.bt_width * 4 + 127) / 128;  // 128-byte lines per row
  int r0 = 0, r1 = p.n;
  if ((int64_t)p.n * lpr > 64) {
    const int est = (int)(((int64_t)blockIdx.x * p.n) / gridDim.x);
    r0 = est > 0 ? est - 1 : 0;
    r1 = est + 2 < p.n ? est + 2 : p.n;
  }
  const int total = (r1 - r0) * lpr;
  for (int l = threadIdx.x; l < total; l += blockDim.x) {
    const int r = r0 + l / lpr;
    const int e = (l % lpr) * 32 < p.bt_width ? (l % lpr) * 32 : p.bt_width - 1;
    prefetch_l2(p.bt + (int64_t)r * p.bt_stride + e);
  }
}

struct StageIter {
  int64_t g_cur, g_end;
  const int* prefix;
  const int* lens;
  const int32_t* trows;  // block-table row of each work row (null: the row itself)
  int n, Y, tps, vt;
  int row_cur;
  bool first, have, single;
  Piece pc;
  int t;       // first tile of the next stage of pc
  int pieces;  // pieces started so far

  __device__ void init(int64_t g0, int64_t g1, int row, const int* prefix_s, const int* lens_s, int n_rows, int y,
                       int tiles_per_stage, int vtiles) {
    vt = vtiles;
    trows = nullptr;
    g_cur = g0;
    g_end = g1;
    prefix = prefix_s;
    lens = lens_s;
    n = n_rows;
    Y = y;
    tps = tiles_per_stage;
    row_cur = row;
    first = true;
    have = false;
    single = false;
    t = 0;
    pieces = 0;
  }

  __device__ void init_single(const Piece& piece, int tiles_per_stage) {
    pc = piece;
    trows = nullptr;
    g_cur = 0;
    g_end = 1;
    tps = tiles_per_stage;
    first = false;
    have = false;
    single = true;
    t = 0;
    pieces = 0;
  }

  __device__ bool next_piece() {
    if (single) {
      if (g_cur >= g_end) return false;
      g_cur = g_end;
      return true;
    }
    while (g_cur < g_end) {
      const int nv = prefix[row_cur + 1] - prefix[row_cur];
      const int nt = nv - vt;  // nv > 0 for a visited row, so nt >= 1
      const int64_t local = g_cur - (int64_t)prefix[row_cur] * Y;
      const int y = (int)(local / nv);
      const int t0 = (int)(local - (int64_t)y * nv);
      const int t1 = (int)min((int64_t)nv, (int64_t)t0 + (g_end - g_cur));
      const int row = row_cur;
      g_cur += t1 - t0;
      if (t1 == nv && y == Y - 1) {
        do {
          ++row_cur;
        } while (row_cur < n && prefix[row_cur + 1] == prefix[row_cur]);
      }
      if (t0 >= nt) continue;  // weight positions only
      pc.row = row;
      pc.y = y;
      pc.t0 = t0;
      pc.t1 = min(t1, nt);
      pc.len = lens != nullptr ? lens[row] : 0;
      pc.trow = trows != nullptr ? trows[row] : row;
      pc.whole = (t0 == 0 && t1 >= nt);
      pc.slot = first ? 0 : 1;
      first = false;
      return true;
    }
    return false;
  }

  // Next stage: tiles [st_t0, st_t1) of piece pc; flags for piece bounds.
  __device__ bool next(int& st_t0, int& st_t1, bool& piece_first, bool& piece_last) {
    if (!have || t >= pc.t1) {
      if (!next_piece()) return false;
      have = true;
      t = pc.t0;
      ++pieces;
      piece_first = true;
    } else {
      piece_first = false;
    }
    st_t0 = t;
    st_t1 = min(pc.t1, t + tps);
    t = st_t1;
    piece_last = (t >= pc.t1);
    return true;
  }
};

// Producer-side lookahead of block-table entries.  A table entry read at the
// moment its tiles are issued costs a loaded-HBM round trip (1-2 us) per
// stage, which alone caps a CTA's stream; instead lane j fetches the entry of
// tile j of stage k + kIdAhead with cp.async into ring slot
// (k + kIdAhead) % kIdRing, one commit group per stage, and stage k reads its
// slot after cp.async.wait_group(kIdAhead).  At a piece's first stage the
// piece's q rows are prefetched into L2 at the same distance.
constexpr int kIdAhead = 6;
constexpr int kIdRing = 8;   // > kIdAhead: a slot is rewritten only after its stage read it
constexpr int kIdLanes = 8;  // tiles per stage, at most
constexpr int kIdRingBytes = kIdRing * kIdLanes * 4;

struct IdPrefetch {
  StageIter it;  // runs kIdAhead stages ahead of the producer
  int* ring;     // shared memory [kIdRing][kIdLanes]
  int issued;    // stages whose ids were requested

  // Request stage `issued`'s ids and commit one group, possibly empty, so
  // group counting stays uniform.  Lane j < nlanes fetches tile
  // first_tile + j of the stage.  A piece's q is heads_per_piece rows of
  // row_bytes from head y * heads_per_piece on (heads_per_piece 0: no q
  // prefetch).
  __device__ void push(const DecodeParams& p, int lane, int heads_per_piece, int row_bytes, int first_tile = 0,
                       int nlanes = kIdLanes) {
    int a0, a1;
    bool apf, apl;
    if (it.next(a0, a1, apf, apl)) {
      const int tile = a0 + first_tile + lane;
      if (lane < nlanes && tile < a1)
        cp_async4(ring + (issued % kIdRing) * kIdLanes + lane,
                  p.bt + (int64_t)it.pc.trow * p.bt_stride + tile / p.tiles_per_block);
      if (apf && heads_per_piece > 0) {
        if (p.q_rows != nullptr) {
          if (lane == 0) prefetch_l2(p.q_rows + it.pc.row);
        } else {
          const unsigned char* q0 = p.q + (int64_t)it.pc.row * p.q_sn;
          const int lph = (row_bytes + 127) >> 7;  // lines per head row, each starting inside the row
          for (int l = lane; l < heads_per_piece * lph; l += 32) {
            const int h = l / lph;
            prefetch_l2(q0 + (int64_t)(it.pc.y * heads_per_piece + h) * p.q_sh + (l - h * lph) * 128);
          }
        }
      }
      ++issued;
    }
    cp_async_commit();
  }

  // The ids of stage k (this lane's tile) after the prologue pushed
  // kIdAhead stages and stage k pushed its own lookahead.
  __device__ int64_t take(int k, int lane) {
    cp_async_wait<kIdAhead>();
    return (int64_t)ring[(k % kIdRing) * kIdLanes + (lane & (kIdLanes - 1))];
  }
};

// Launch hook of the tcgen05 GQA kernel (fd_decode_mma.cu): returns FD_OK and
// sets *launched when it handled the call, FD_OK with *launched = false when
// the shape is not one it covers.
int launch_decode_mma(const DecodeParams& p, int dtype, int D, size_t extra_smem, cudaStream_t s, int* ncta,
                      bool* launched, bool pdl);

// Tiled tensor map of a 4-D view {D, heads, BS, blocks} (byte strides of
// heads, tokens and blocks), box {64 (swizzled) or D, box_heads, box_tokens,
// 1}, cached per view (fd_decode.cu); false when the driver rejects it.
bool encode_kv_map(CUtensorMap* m, const void* base, int dtype, int D, int heads, int BS, int64_t nblk,
                   int64_t head_sb, int64_t tok_sb, int64_t blk_sb, int box_tokens, bool swizzle128,
                   int box_heads = 1);

// Whether the tcgen05 kernel covers this shape (16-bit KV, head size 128,
// query group 2, 4 or 8, block size a multiple of 16).
bool mma_eligible(int dtype, int D, int G, int BS);

// The CTAs whose ranges hold real tiles of the segment (row, y) of a
// persistent launch of N CTAs over T = prefix[n] * Y positions: c0 (the owner
// of its first position g0) to c1 (the owner of its last real tile); c0 == c1
// means one CTA wrote the segment's output directly.  Otherwise every CTA of
// c0..c1 whose range is not empty wrote an fp32 partial: c0 into slot
// first_slot (0 when the segment is its first real piece, i.e. its range
// starts at most vtiles weight positions before g0), the others into slot 0
// (the segment is their first piece).  The owner of position g is the
// largest c with floor(c * T / N) <= g, i.e. ((g + 1) * N - 1) / T.
struct SegSpan {
  int64_t c0, c1;
  int first_slot;
};

__device__ __forceinline__ SegSpan seg_span(const int* prefix, int Y, int vtiles, int64_t N, int64_t T, int row,
                                            int y) {
  SegSpan sp;
  const int nv = prefix[row + 1] - prefix[row];
  const int nt = nv - vtiles;
  const int64_t g0 = (int64_t)prefix[row] * Y + (int64_t)y * nv;
  sp.c0 = ((g0 + 1) * N - 1) / T;
  sp.c1 = ((g0 + nt) * N - 1) / T;
  sp.first_slot = ((sp.c0 * T) / N >= g0 - vtiles) ? 0 : 1;
  return sp;
}

__device__ __forceinline__ bool seg_nonempty(int64_t cc, int64_t N, int64_t T) {
  return (cc * T) / N != ((cc + 1) * T) / N;
}

// Where a persistent decode launch left each (row, kv-head chunk) segment of
// its output, for a kernel that reads the output right after it (the peer
// exchange of the sharded path) and merges the segments that CTA ranges cut
// on the way, instead of a separate combine launch.  prefix == nullptr: the
// output is complete in the decode's out / lse.
struct ShardGeom {
  const int* prefix;      // positions per row, [n + 1] (written by the decode's CTA 0)
  const float* part_o;    // fp32 partial slots [ncta * 2 * GQ][D]
  const float* part_lse;  // [ncta * 2 * GQ]
  int ncta;               // CTAs of the decode launch
  int vtiles;             // weight positions per segment
  int KVH, gcs, G, GQ;    // segments are (row, kv head * gcs + chunk); a chunk holds GQ of G query heads
};

// Launch the decode of `a` on `stream` for a consumer that merges cut
// segments itself: with the persistent schedule only the decode kernel runs
// and `geom` describes its partials; otherwise (split grid) the decode and its
// combine run and geom->prefix is null.  decode = false: the caller launched
// the decode kernel already (fd_decode_attn_partials with the same arguments);
// only the split grid's combine is launched, and `geom` filled.
int launch_decode_for_exchange(const fd_decode_args* a, void* stream, ShardGeom* geom, bool decode);

}  // namespace fdk
