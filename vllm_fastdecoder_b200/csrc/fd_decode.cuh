// Kernel parameters and schedule constants shared by the decode kernels
// (the CUDA-core kernel in fd_decode.cu and the tcgen05 GQA kernel in
// fd_decode_mma.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

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
  int64_t bt_stride;
  int bt_width;
  const int32_t* lens;
  int n, H, KVH, BS, G, gcs, gq;
  int TT, tiles_per_block, tiles_per_split, max_splits;
  // persistent schedule: ncta CTAs share the flattened (row, kv-head chunk,
  // tile) space evenly; prefix of per-row tile counts published in ws_prefix
  int persistent, ncta;
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
  bool whole;
};

// Launch hook of the tcgen05 GQA kernel (fd_decode_mma.cu): returns FD_OK and
// sets *launched when it handled the call, FD_OK with *launched = false when
// the shape is not one it covers.
int launch_decode_mma(const DecodeParams& p, int dtype, int D, size_t extra_smem, cudaStream_t s, int* ncta,
                      bool* launched);

// Whether the tcgen05 kernel covers this shape (16-bit KV, head size 128,
// query group 2, 4 or 8, block size a multiple of 16).
bool mma_eligible(int dtype, int D, int G, int BS);

}  // namespace fdk
