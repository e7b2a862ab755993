/*
 * fastdecode_b200.h -- C ABI of the B200 paged decode-attention engine.
 *
 * Every entry point takes plain pointers, sizes and strides (no torch types),
 * is asynchronous on the caller's CUDA stream (passed as `void *stream`,
 * i.e. a cudaStream_t; NULL means the legacy default stream) and returns an
 * fd_status code.  The caller owns and allocates every buffer: outputs, the
 * KV tiers and the scratch workspace.  The library never allocates device
 * memory on its own.
 *
 * Block numbering (the G+C convention of the reference plugin,
 * fastdecode/patches.py:1-7 and fastdecode/plan.py:3-4):
 *   block id b <  tier_split  ->  tier[0], block b       (HBM tier)
 *   block id b >= tier_split  ->  tier[1], block b - G   (host tier)
 * A tier whose memory is pinned host memory mapped into the device address
 * space (cudaHostAlloc / cudaHostRegister, flag Mapped) is marked
 * host_mapped = 1 and is read over PCIe with 16-byte loads; device tiers are
 * streamed with TMA bulk copies.
 *
 * Device-side checks (block id range, row length vs. block-table width, slot
 * range, bounded waits) never trap: they write a nonzero code into the
 * optional `error` word (int32 in device memory) and skip the access.  Read
 * it with fd_read_error().
 */
#ifndef FASTDECODE_B200_H
#define FASTDECODE_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define FD_API __attribute__((visibility("default")))
#else
#define FD_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- codes */

enum fd_dtype {
  FD_DTYPE_F16 = 0,
  FD_DTYPE_BF16 = 1,
  FD_DTYPE_F32 = 2
};

enum fd_status {
  FD_OK = 0,
  FD_ERR_INVALID = 1,     /* bad shape / argument (message: fd_last_error_message) */
  FD_ERR_UNSUPPORTED = 2, /* valid but not built (dtype, head size, group size) */
  FD_ERR_ALIGN = 3,       /* pointer or stride not 16-byte aligned */
  FD_ERR_WORKSPACE = 4,   /* workspace missing or too small */
  FD_ERR_CUDA = 5,        /* a CUDA runtime call failed */
  FD_ERR_RANGE = 6        /* host-visible index out of range */
};

/* codes written by kernels into the device error word */
enum fd_device_error {
  FD_DEVERR_NONE = 0,
  FD_DEVERR_BLOCK_ID = 1,  /* block-table entry outside both tiers */
  FD_DEVERR_LEN = 2,       /* lens[i] needs more blocks than the table row holds */
  FD_DEVERR_TIMEOUT = 3,   /* a bounded wait on an mbarrier gave up */
  FD_DEVERR_SLOT = 4,      /* KV-write slot outside both tiers */
  FD_DEVERR_SPLITS = 5,    /* lens[i] exceeds the max_len the grid was sized for */
  FD_DEVERR_PLAN = 6       /* fd_plan_step: bad query offsets, or a request that
                              extends prior context by > 1 token while part of
                              its KV is in the host tier (fastdecode/plan.py:142-149) */
};

/* ---------------------------------------------------------------- types */

/* One KV tier.  Element (block b, kv head h, token t, dim d) of K lives at
 * k + b*blk_stride + h*head_stride + t*tok_stride + d   (in elements).
 * Host-store layout [C, KVH, BS, D] (fastdecode/state.py:66):
 *     blk_stride = KVH*BS*D, head_stride = BS*D, tok_stride = D.
 * vLLM NHD layout [B, BS, KVH, 2D] split into K/V views (backend.py:265):
 *     blk_stride = BS*KVH*2D, head_stride = 2D, tok_stride = KVH*2D. */
typedef struct fd_kv_tier {
  void *k;
  void *v;
  int64_t blk_stride;
  int64_t head_stride;
  int64_t tok_stride;
  int64_t num_blocks;  /* valid ids of this tier are [0, num_blocks) */
  int32_t host_mapped; /* 1: pinned host memory read over PCIe */
  int32_t _pad;
} fd_kv_tier;

/* Arguments of the split-KV decode kernel.  Strides are in elements. */
typedef struct fd_decode_args {
  /* queries: q[row, h, d] = q + row*q_stride_n + h*q_stride_h + d, with
   * row = q_rows ? q_rows[i] : i  (q_rows fuses the index_select of
   * fastdecode/backend.py:287) */
  const void *q;
  int64_t q_stride_n;
  int64_t q_stride_h;
  const int64_t *q_rows;

  fd_kv_tier tier[2];
  int64_t tier_split; /* G */

  /* block_table[i*bt_stride + j], j < ceil(lens[i]/block_size) <= bt_width;
   * entries past a row's last block are never read */
  const int32_t *block_table;
  int64_t bt_stride;
  int32_t bt_width;
  const int32_t *lens; /* [n] tokens of each row (0: empty row) */

  int32_t n;
  int32_t num_heads;
  int32_t num_kv_heads;
  int32_t head_size;
  int32_t block_size;
  float scale;
  int32_t dtype; /* of q, K and V */

  /* output rows: out[orow, h, d], orow = out_rows ? out_rows[i] : i
   * (out_rows fuses output.index_copy_ of backend.py:356); a negative
   * out_rows[i] writes no output for row i (padding of a device-built row
   * list); out_dtype is dtype or FD_DTYPE_F32 (fp32 partials for a later
   * merge) */
  void *out;
  int32_t out_dtype;
  int32_t _pad0;
  int64_t out_stride_n;
  int64_t out_stride_h;
  const int64_t *out_rows;

  /* lse[h*lse_stride_h + i*lse_stride_n] (natural log; -inf for empty
   * rows); NULL to skip.  The reference layout [H, n] is
   * lse_stride_h = n, lse_stride_n = 1. */
  float *lse;
  int64_t lse_stride_h;
  int64_t lse_stride_n;

  int32_t max_len;         /* upper bound on lens[] (0: bt_width*block_size) */
  int32_t tiles_per_split; /* 0: heuristic; a tile is min(block_size,16) tokens */

  void *workspace; /* scratch for split partials, fd_decode_workspace_size() bytes */
  size_t workspace_bytes;
  int32_t *error;  /* optional device error word */

  /* optional: row i reads block-table row bt_rows[i] (else row i), so a
   * device-built list of work rows (fd_plan_step) runs on the batch's own
   * table without gathering it (replaces the index_select of table rows in
   * fastdecode/plan.py:224-245).  Like q_rows and out_rows, its entries must
   * address rows of their tensors: row indices are the caller's contract
   * and are not range-checked (block ids and lengths are). */
  const int32_t *bt_rows;

  /* FD_DECODE_* bits (0: none) */
  int32_t flags;
  int32_t _pad1;
} fd_decode_args;

/* fd_decode_args.flags: launch the decode as a programmatic dependent of the
 * kernel ahead of it on the stream (CUDA programmatic dependent launch), so
 * that its set-up -- reading lens, the block table, bt_rows / q_rows /
 * out_rows and q, and prefetching block ids -- overlaps that kernel's tail.
 * K/V reads and every write of the decode wait until that kernel has
 * completed.  The caller guarantees that the kernel directly ahead does not
 * write lens, the block table, the row maps or q (e.g. it is the layer's KV
 * write, or the previous decode's combine or exchange).  No effect on a
 * stream whose previous operation is not a kernel. */
#define FD_DECODE_PDL 1

/* ---------------------------------------------------------------- decode */

/* Scratch bytes fd_decode_attn needs for these arguments (0 when every row
 * fits in one split).  Pure host arithmetic. */
FD_API size_t fd_decode_workspace_size(const fd_decode_args *a);

/* Paged decode attention over a two-tier block table.
 *   o[i,h]   = softmax(q[i,h] . K[i]^T * scale) @ V[i]
 *   lse[h,i] = logsumexp(q[i,h] . K[i]^T * scale)
 * Replaces, on the GPU, both halves of the reference split path:
 *   - decode_attn, fastdecode/csrc/cpu_attn.cpp:298-411,456-489 (host tier)
 *   - the FlashAttention paged partial, fastdecode/backend.py:293-316 (HBM tier)
 * and the LSE merge of the two (backend.py:354-356), because one pass over
 * the unified table covers both tiers. */
FD_API int fd_decode_attn(const fd_decode_args *a, void *stream);

/* The two launches fd_decode_attn makes, for callers that want to place
 * other work (or timing events) between them:
 *   fd_decode_attn_partials  the split-KV kernel; rows that fit in one split
 *                            are final after it, others leave fp32 partials
 *                            in the workspace
 *   fd_decode_attn_combine   the log-sum-exp combine of those partials
 * Both take the same arguments; calling them in order on one stream equals
 * fd_decode_attn.  fd_decode_attn_combine launches nothing when every row
 * fits in one split. */
FD_API int fd_decode_attn_partials(const fd_decode_args *a, void *stream);
FD_API int fd_decode_attn_combine(const fd_decode_args *a, void *stream);

/* Size of the scratch array built into the library for
 * fd_decode_attn_noalloc (32 MiB of device memory on every GPU that loads
 * the library, held until the process exits). */
#define FD_NOALLOC_SCRATCH_BYTES (32u << 20)

/* fd_decode_attn for callers that cannot allocate device memory.  It has no
 * counterpart in the reference.
 *
 * Some callers of this kernel must not call cudaMalloc: code that runs after
 * vLLM has sized its KV cache to fill the memory its profiler left free (a
 * late allocation can fail), code inside a framework that owns all device
 * memory through its own allocator, and loops where cudaMalloc / cudaFree
 * would synchronise the device.  This entry point takes the same arguments
 * as fd_decode_attn but ignores `workspace` / `workspace_bytes`: the split
 * partials go to a file-scope __device__ array of FD_NOALLOC_SCRATCH_BYTES
 * inside the library, so it calls no cudaMalloc, cudaFree or other allocating
 * routine.  Arguments whose partials would not fit (fd_decode_workspace_size()
 * larger than FD_NOALLOC_SCRATCH_BYTES) are rejected with FD_ERR_WORKSPACE
 * before anything is launched; a larger tiles_per_split needs less scratch.
 *
 * The first call on each device looks up the array's device address
 * (cudaGetSymbolAddress, with that device current) and caches it with the
 * CUDA context it belongs to; make that first call before any stream
 * capture.  A context torn down and created again (cudaDeviceReset) is seen
 * by the next call, which looks the address up again.  All calls share the one array and it
 * keeps the last call's contents; nothing in it needs to start at zero (every
 * partial, and the row-tile prefix, is written by the decode kernel before
 * the combine kernel of the same call reads it).  Calls whose
 * executions overlap on the GPU (other streams of the same device) race on
 * the array: order them, e.g. on one stream. */
FD_API int fd_decode_attn_noalloc(const fd_decode_args *a, void *stream);

/* Drop-in for the reference pybind op
 *   decode_attn(q, k_cache, v_cache, block_table, lens, scale, out, lse)
 * (fastdecode/csrc/cpu_attn.cpp:456-489): contiguous q [n,H,D], caches
 * [C,KVH,BS,D] (device memory, or mapped pinned host memory), block_table
 * [n,W] int32 with cache-relative ids, lens [n] int32, out [n,H,D] (q dtype),
 * lse [H,n] fp32. */
FD_API int fd_decode_attn_paged(const void *q, const void *k_cache, const void *v_cache,
                         int32_t cache_is_host, const int32_t *block_table,
                         const int32_t *lens, int32_t n, int32_t num_heads,
                         int32_t num_kv_heads, int32_t head_size, int32_t block_size,
                         int64_t num_blocks, int32_t bt_width, float scale, int32_t dtype,
                         void *out, float *lse, void *workspace, size_t workspace_bytes,
                         int32_t *error, void *stream);

/* Workspace bytes fd_decode_attn_paged needs. */
FD_API size_t fd_decode_attn_paged_workspace_size(int32_t n, int32_t num_heads,
                                           int32_t num_kv_heads, int32_t head_size,
                                           int32_t block_size, int32_t bt_width,
                                           int32_t dtype);

/* ---------------------------------------------------------------- merge */

/* ---------------------------------------------------------------- plan */

/* Slots of the plan header (int32[FD_PLAN_HEADER_LEN], device memory). */
enum fd_plan_header {
  FD_PLAN_FLAGS = 0,          /* FD_PLAN_* bits below */
  FD_PLAN_N_TOK = 1,          /* tokens of the step (query_start_loc[R]) */
  FD_PLAN_N_CPU_W = 2,        /* tokens whose KV goes to the host tier */
  FD_PLAN_N_P = 3,            /* class P requests (all KV in HBM) */
  FD_PLAN_N_P_TOK = 4,
  FD_PLAN_P_MAX_Q = 5,
  FD_PLAN_P_MAX_K = 6,
  FD_PLAN_N_S = 7,            /* class S: decodes touching the host tier */
  FD_PLAN_S_GPU_WIDTH = 8,    /* width of the compacted HBM table (multiple of 16) */
  FD_PLAN_S_MAX_GPU_LEN = 9,
  FD_PLAN_S_CPU_WIDTH = 10,   /* width of the compacted host table */
  FD_PLAN_N_F = 11,           /* class F: fresh prefills touching the host tier */
  FD_PLAN_N_F_TOK = 12,
  FD_PLAN_F_MAX = 13,
  FD_PLAN_S_MAX_LEN = 14,
  FD_PLAN_N_PD = 15,          /* P requests that are decodes */
  FD_PLAN_PD_MAX_LEN = 16,
  FD_PLAN_N_PP = 17,          /* P requests that are prefills */
  FD_PLAN_N_PP_TOK = 18,
  FD_PLAN_PP_MAX_Q = 19,
  FD_PLAN_PP_MAX_K = 20,
  FD_PLAN_N_DECODE = 21,      /* rows of the decode list (S and P decodes) */
  FD_PLAN_DECODE_MAX_LEN = 22,
  FD_PLAN_HEADER_LEN = 32
};
enum fd_plan_flags {
  FD_PLAN_TOUCHES_HOST = 1, /* some request or new token uses the host tier (the
                               reference planner returns None otherwise) */
  FD_PLAN_BAD_BLOCK_ID = 2, /* a block id >= G + C (reference: RuntimeError) */
  FD_PLAN_HOST_EXTEND = 4,  /* reference: NotImplementedError (FD_DEVERR_PLAN) */
  FD_PLAN_BAD_OFFSETS = 8   /* query_start_loc not 0-based, decreasing, or past
                               max_tokens: nothing else was written */
};

/* The per-step plan computed on the device (fastdecode/plan.py:103-245).
 * Inputs are device tensors of the step; outputs are caller-allocated
 * device buffers of the given capacities (R = num_reqs rows, T =
 * max_tokens tokens); the header says how many entries of each are valid.
 * Each output matches the reference HostPlan / DevicePlan field of the same
 * name bit for bit. */
typedef struct fd_plan_args {
  const int32_t *query_start_loc; /* [R + 1] */
  const int32_t *seq_lens;        /* [R] tokens including this step's */
  const int32_t *block_table;     /* [R, bt_stride], unified ids */
  int64_t bt_stride;
  int32_t bt_width;
  int32_t num_reqs;
  const int64_t *slot_mapping;    /* [>= T] unified slots (-1: padding) */
  int32_t max_tokens;             /* T */
  int32_t block_size;
  int64_t num_gpu_blocks;         /* G */
  int64_t num_cpu_blocks;         /* C */

  int32_t *header;                /* [FD_PLAN_HEADER_LEN] */
  /* KV writes */
  int64_t *gpu_slot_mapping;      /* [T] host slots replaced by -1 */
  int64_t *cpu_w_tok;             /* [T] */
  int64_t *cpu_w_slot;            /* [T] host-relative */
  /* P */
  int64_t *p_tok;                 /* [T] */
  int32_t *p_cu;                  /* [R + 1] */
  int32_t *p_seqlens;             /* [R] */
  int64_t *p_req;                 /* [R] */
  /* S */
  int64_t *s_tok;                 /* [R] */
  int32_t *s_gpu_bt;              /* [R, s_gpu_bt_stride], width in the header */
  int64_t s_gpu_bt_stride;        /* >= bt_width rounded up to 16 */
  int32_t *s_gpu_lens;            /* [R] */
  int32_t *s_cpu_bt;              /* [R, s_cpu_bt_stride] host-relative ids */
  int64_t s_cpu_bt_stride;        /* >= bt_width */
  int32_t *s_cpu_lens;            /* [R] */
  /* F */
  int64_t *f_tok;                 /* [T] */
  int32_t *f_cu;                  /* [R + 1] */
  /* this engine's additions (plan.py of this repository) */
  int64_t *s_req;                 /* [R] */
  int32_t *s_seq_lens;            /* [R] */
  int64_t *pd_req;                /* [R] */
  int64_t *pd_tok;                /* [R] */
  int32_t *pd_seq_lens;           /* [R] */
  int64_t *pp_req;                /* [R] */
  int64_t *pp_tok;                /* [T] */
  int32_t *pp_cu;                 /* [R + 1] */
  int32_t *pp_seqlens;            /* [R] */
  /* decode list for fd_decode_attn: q_rows = out_rows = d_tok, bt_rows =
   * d_row, lens = d_lens, n = R; entries past the header's N_DECODE have
   * d_tok = -1 and d_lens = 0 (no work, no output) */
  int64_t *d_tok;                 /* [R] */
  int32_t *d_row;                 /* [R] */
  int32_t *d_lens;                /* [R] */
  int32_t *error;                 /* optional device error word */
} fd_plan_args;

/* Replaces the reference's host planner build_host_plan + to_device
 * (fastdecode/plan.py:103-245, called per step at fastdecode/backend.py:
 * 140-178): one single-CTA launch on the caller's stream, no host
 * synchronisation, no host copies.  Capacities are checked on the host;
 * query offsets past max_tokens are caught on the device
 * (FD_PLAN_BAD_OFFSETS, FD_DEVERR_PLAN). */
FD_API int fd_plan_step(const fd_plan_args *a, void *stream);

/* sizeof(fd_plan_args) as compiled into the library (binding check). */
FD_API size_t fd_plan_args_bytes(void);

/* ------------------------------------------------------- peer exchange */

/* The sharded long-context path (no reference counterpart: the reference
 * has no multi-GPU path) exchanges each rank's fp32 partial over peer
 * memory instead of an NCCL all-gather: one launch per step pushes the
 * rank's packed [o (n*H*D) | lse (H*n)] into every rank's receive buffer
 * over NVLink, waits (bounded) for every rank's, and merges with the rule
 * of fd_merge_partials.  Buffers are plain device memory shared with CUDA
 * IPC (no multicast object). */
#define FD_MAX_PEERS 8
#define FD_IPC_HANDLE_BYTES 64
/* Layout of one rank's allocation (fd_peer_alloc): u64 step counters of its
 * exchange CTAs [64] at byte 0; the receive slots [2 parities][world][slot]
 * from FD_PEER_RECV_OFFSET, float i of a slot stored as the 8-byte word
 * {u32 value bits, u32 step} (the step travels with each value, so a reader
 * needs no fence and no separate arrival flag). */
#define FD_PEER_RECV_OFFSET 8192

typedef struct fd_peer_exchange {
  void *base[FD_MAX_PEERS]; /* rank q's allocation as mapped in this process:
                               the own one from fd_peer_alloc, the others
                               from fd_peer_open */
  int32_t rank;
  int32_t world;
  int64_t slot_floats;      /* floats per rank slot: >= n*H*D + H*n, multiple of 4 */
} fd_peer_exchange;

/* Bytes of one rank's allocation (counters + 2 x world slots of 8-byte words). */
FD_API size_t fd_peer_buffer_bytes(int32_t world, int64_t slot_floats);
/* cudaMalloc + zero + IPC handle (FD_IPC_HANDLE_BYTES written to ipc_handle). */
FD_API int fd_peer_alloc(size_t bytes, void **ptr, void *ipc_handle);
/* Map another rank's allocation (cudaIpcOpenMemHandle) / unmap it. */
FD_API int fd_peer_open(const void *ipc_handle, void **ptr);
FD_API int fd_peer_close(void *ptr);
FD_API int fd_peer_free(void *ptr);
/* One step: every rank calls it once per step, in the same order, with the
 * same n / heads / head size / num_ctas (0: 64, at most 64; CTAs of 128 threads).  send: this rank's packed
 * partial (16-byte aligned); out [n, H, D] in out_dtype; out_lse [H, n] or
 * NULL.  Each value a rank pushes carries the step number in the same
 * 8-byte word; the merge waits until every word it reads carries this step
 * exactly (so neither an old value nor a rank that is a step ahead can
 * complete another rank's step).  Launched as a
 * programmatic dependent of the kernel ahead of it on the stream (it waits
 * for that kernel before reading send).  A wait longer than timeout_ns (0:
 * 2 s) records FD_DEVERR_TIMEOUT in *error and returns with the outputs
 * unwritten; the caller must read the error word (fd_read_error) after each
 * step it cannot otherwise vouch for, and after a timeout the exchange must
 * be freed and rebuilt on every rank. */
FD_API int fd_exchange_merge(const fd_peer_exchange *x, const float *send, int32_t n, int32_t num_heads,
                             int32_t head_size, void *out, int32_t out_dtype, float *out_lse, int32_t num_ctas,
                             int64_t timeout_ns, int32_t *error, void *stream);

/* The whole sharded step in two launches: the decode of `a` over this rank's
 * shard, then the exchange and merge of fd_exchange_merge, which also does
 * the decode's combine.  `a` must write the rank's packed partial: out_dtype
 * FD_DTYPE_F32, out = o [n, H, D] contiguous, lse = out + n*H*D laid out
 * [H, n], no out_rows (this is the exchange's send buffer, 16-byte aligned).
 * With the persistent schedule the decode's combine launch is skipped: the
 * exchange pushes each (row, kv-head chunk) segment that one decode CTA
 * finished straight from `out`, and merges each segment that decode CTAs cut
 * from their partial slots in the workspace on its way to the other ranks
 * (the combine's rule and order, so the result equals decode + combine +
 * fd_exchange_merge bit for bit).  The error word is a->error.  Same
 * collective rules as fd_exchange_merge. */
FD_API int fd_decode_exchange_merge(const fd_decode_args *a, const fd_peer_exchange *x, void *out,
                                    int32_t out_dtype, float *out_lse, int32_t num_ctas, int64_t timeout_ns,
                                    void *stream);
/* The exchange half of fd_decode_exchange_merge, for callers that launched
 * the decode themselves (fd_decode_attn_partials with the same arguments,
 * earlier on the stream) and want other work or timing events in between. */
FD_API int fd_exchange_merge_decoded(const fd_decode_args *a, const fd_peer_exchange *x, void *out,
                                     int32_t out_dtype, float *out_lse, int32_t num_ctas, int64_t timeout_ns,
                                     void *stream);

/* Two-way log-sum-exp merge, the rule of vLLM merge_attn_states as restated
 * in fastdecode/cpu_ops.py:93-113 and called at fastdecode/backend.py:54-55,
 * 354-356: an lse of +inf (FlashAttention's empty row) counts as -inf, and a
 * row empty on both sides yields zeros.
 *   o_a, o_b: [n, H, D] contiguous, dtype in_dtype (F16/BF16/F32)
 *   lse_a, lse_b: [H, n] fp32
 *   out: rows out_rows[i] (or i) of an [*, H, D] tensor with out_stride_n,
 *        dtype out_dtype (a negative out_rows[i] writes no row);
 *        out_lse [H, n] fp32 or NULL. */
FD_API int fd_merge_attn_states(void *out, int32_t out_dtype, int64_t out_stride_n,
                         const int64_t *out_rows, float *out_lse,
                         const void *o_a, const float *lse_a,
                         const void *o_b, const float *lse_b, int32_t in_dtype,
                         int32_t n, int32_t num_heads, int32_t head_size, void *stream);

/* P-way merge of fp32 partials (the same rule over P parts), used for the
 * KV-sharded long-context path after an all-gather of per-GPU partials.
 *   o of part p:   o_parts  + p*part_stride, layout [n, H, D]
 *   lse of part p: lse_parts + p*part_stride, layout [H, n]
 *   out [n, H, D] contiguous of out_dtype; out_lse [H, n] or NULL. */
FD_API int fd_merge_partials(const float *o_parts, const float *lse_parts, int64_t part_stride,
                      int32_t num_parts, int32_t n, int32_t num_heads, int32_t head_size,
                      void *out, int32_t out_dtype, float *out_lse, void *stream);

/* ---------------------------------------------------------------- prefill */

/* Causal prefill attention for the P (prefill over cached context) and F
 * (fresh prefill) request classes, which the reference runs through vLLM's
 * FlashAttention (fastdecode/backend.py:317-340: flash_attn_varlen_func with
 * causal=True, paged block_table for P, the batch's own k / v for F).
 * Request r has q_len[r] queries at batch rows q_start[r] .. + q_len[r] - 1
 * and k_len[r] >= q_len[r] keys; query i sees keys 0 .. k_len - q_len + i
 * (FlashAttention's bottom-right causal alignment).  Keys and values come
 * from the HBM tier of the paged cache (block_table != NULL: key j of request
 * r lies in block block_table[bt_row[r] * bt_stride + j / block_size], row
 * j % block_size of `kv`, block_size a multiple of 16) or, block_table ==
 * NULL, from the batch's own new K/V rows: kv.k / kv.v are [rows, KVH, D]
 * (kv.tok_stride, kv.head_stride; kv.num_blocks = rows) and key j of request
 * r is row q_start[r] + j.  out [num_tokens, H, D] rows of the requests'
 * queries are written in q's dtype; other rows are untouched.  fp16 / bf16,
 * head size 128, any GQA group.  Replaces FlashAttention on the tcgen05
 * tensor cores; no lse output. */
typedef struct fd_prefill_args {
  const void *q;            /* [num_tokens, H, D] */
  int64_t q_stride_t;
  int64_t q_stride_h;
  void *out;                /* [num_tokens, H, D], q's dtype */
  int64_t out_stride_t;
  int64_t out_stride_h;
  fd_kv_tier kv;            /* device memory only */
  const int32_t *block_table;
  int64_t bt_stride;
  int32_t bt_width;
  int32_t num_tokens;       /* rows of q and out */
  const int32_t *q_start;   /* [n] device, int32 */
  const int32_t *q_len;     /* [n] */
  const int32_t *k_len;     /* [n] */
  const int32_t *bt_row;    /* [n] or NULL (row r) */
  int32_t n;                /* requests, at most 65535 */
  int32_t num_heads;
  int32_t num_kv_heads;
  int32_t head_size;
  int32_t block_size;
  float scale;
  int32_t dtype;
  int32_t total_q;          /* sum of q_len (an upper bound is fine): sizes the grid */
  int32_t *error;           /* optional device error word */
} fd_prefill_args;

FD_API int fd_prefill_attn(const fd_prefill_args *a, void *stream);

/* sizeof(fd_prefill_args) as compiled into the library (binding check). */
FD_API size_t fd_prefill_args_bytes(void);

/* ---------------------------------------------------------------- KV write */

/* Tier-aware KV write: new K/V rows go straight to their slot in whichever
 * tier owns it.  slot s -> block s / block_size, offset s % block_size;
 * block < tier_split -> tier[0], else tier[1] at block - tier_split.
 * slot < 0 is skipped (reshape_and_cache_flash convention).  If any slot is
 * outside both tiers nothing is written and the error word gets
 * FD_DEVERR_SLOT.  Bit-exact copy.  Up to 2048 rows: one launch.  More: two
 * launches (a check, then the copy as its programmatic dependent); the
 * check's verdict lives in one of 1024 device flags, taken per call in turn,
 * so two such calls share a flag only if they are 1024 calls apart (a CUDA
 * graph holding the call reuses its flag on every replay: replay it on one
 * stream at a time).
 * Replaces vLLM reshape_and_cache_flash (fastdecode/backend.py:269-273) plus
 * the D2H staging and store_kv (backend.py:279-285,344-346;
 * fastdecode/csrc/cpu_attn.cpp:413-431,492-517).
 *   key/value: row j, head h at key + j*key_stride_n + h*key_stride_h */
FD_API int fd_store_kv(const void *key, int64_t key_stride_n, int64_t key_stride_h,
                const void *value, int64_t value_stride_n, int64_t value_stride_h,
                const int64_t *slots, int32_t m, int32_t num_kv_heads, int32_t head_size,
                int32_t block_size, int32_t dtype, const fd_kv_tier *tiers,
                int64_t tier_split, int32_t *error, void *stream);

/* ---------------------------------------------------------------- utilities */

/* Message of the last FD_ERR_* returned on this thread. */
FD_API const char *fd_last_error_message(void);

/* Text for an fd_device_error code. */
FD_API const char *fd_device_error_string(int32_t code);

/* Synchronise `stream`, copy the device error word to *value and, if
 * `clear`, reset it to 0. */
FD_API int fd_read_error(int32_t *error, int32_t *value, int32_t clear, void *stream);

/* Device address of pinned host memory (cudaHostGetDevicePointer); fails
 * with FD_ERR_INVALID when `host` is not pinned and mapped. */
FD_API int fd_host_device_pointer(void *host, void **device_ptr);

/* Pin and map an existing host range (cudaHostRegister, Mapped|Portable),
 * and undo it. */
FD_API int fd_host_register(void *host, size_t bytes);
FD_API int fd_host_unregister(void *host);

/* Library version, e.g. 101 for 0.1.1 (101: fd_plan_step, bt_rows). */
FD_API int fd_version(void);

/* sizeof(fd_decode_args) and sizeof(fd_kv_tier) as compiled into the
 * library, so bindings can check their struct mirrors. */
FD_API int fd_abi_sizes(size_t *decode_args_bytes, size_t *kv_tier_bytes);

#ifdef __cplusplus
}
#endif

#endif /* FASTDECODE_B200_H */
