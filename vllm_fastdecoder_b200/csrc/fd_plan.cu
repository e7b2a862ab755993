// Device-side step planner: the reference's per-step plan
// (fastdecode/plan.py:103-245, build_host_plan + to_device) computed on the
// GPU from the step's device tensors, so a step needs neither the block
// table and slots on the host nor the planner's host->device copies.
//
// One CTA of 512 threads, three passes:
//   1. rows (chunks of 512 with carried offsets): class of every request
//      (P all-HBM, S decode touching the host tier, F fresh prefill touching
//      it), per-tier token counts of S rows, and every per-class list
//      (request rows, token spans, cu offsets, lengths), placed by
//      block-wide exclusive scans; maxima by block-wide reductions
//   2. S rows: the compacted HBM table (width padded to 16) and host table
//      (host-relative ids), zero-filled past each row's count
//   3. tokens: KV-write routing (host slots -> -1 in the HBM mapping, their
//      token rows and host-relative slots compacted)
// plus this engine's decode list: every decode row (S or P with one query
// token) in request order, padded with out-row -1 / length 0, which
// fd_decode_attn consumes directly (q_rows = out_rows = token, bt_rows =
// request row).  Integer work throughout; results are bit-exact with the
// reference planner (tests compare every field).

#include <stdint.h>

#include "fd_common.cuh"
#include "fd_internal.h"

namespace fdk {

constexpr int kPlanThreads = 512;
constexpr int kPlanWarps = kPlanThreads / 32;
static_assert(kPlanWarps <= 32, "one warp scans the warp totals");

// Block-wide exclusive scan of K counters per thread; returns the block
// totals in tot[].  All threads of the CTA must call it.
template <int K>
__device__ void block_scan(int64_t (&v)[K], int64_t (&tot)[K], int64_t* sm /* [kPlanWarps * 16] */) {
  static_assert(K <= 16, "scratch holds 16 counters per warp");
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int64_t inc[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    int64_t x = v[k];
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int64_t y = __shfl_up_sync(0xffffffffu, x, off);
      if (lane >= off) x += y;
    }
    inc[k] = x;
  }
  if (lane == 31)
#pragma unroll
    for (int k = 0; k < K; ++k) sm[warp * K + k] = inc[k];
  __syncthreads();
  if (warp == 0) {
#pragma unroll
    for (int k = 0; k < K; ++k) {
      int64_t x = lane < kPlanWarps ? sm[lane * K + k] : 0;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int64_t y = __shfl_up_sync(0xffffffffu, x, off);
        if (lane >= off) x += y;
      }
      if (lane < kPlanWarps) sm[lane * K + k] = x;  // inclusive over warps
    }
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const int64_t before = warp > 0 ? sm[(warp - 1) * K + k] : 0;
    tot[k] = sm[(kPlanWarps - 1) * K + k];
    v[k] = before + inc[k] - v[k];  // exclusive
  }
  __syncthreads();
}

template <int K>
__device__ void block_max(int64_t (&v)[K], int64_t* sm /* [kPlanWarps * 16] */) {
  static_assert(K <= 16, "scratch holds 16 values per warp");
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int k = 0; k < K; ++k) {
    int64_t x = v[k];
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) x = max(x, (int64_t)__shfl_xor_sync(0xffffffffu, x, off));
    v[k] = x;
  }
  if (lane == 0)
#pragma unroll
    for (int k = 0; k < K; ++k) sm[warp * K + k] = v[k];
  __syncthreads();
#pragma unroll
  for (int k = 0; k < K; ++k) {
    int64_t x = sm[k];
    for (int w = 1; w < kPlanWarps; ++w) x = max(x, sm[w * K + k]);
    v[k] = x;
  }
  __syncthreads();
}

struct PlanRow {
  int64_t q0, qlen, seq;
  int nb;  // blocks of the row inside the table width
  int host_blocks, hbm_blocks;
  int64_t host_tok, hbm_tok;
  bool touches_host, bad_id;
};

__device__ PlanRow plan_row(const fd_plan_args& a, int r) {
  PlanRow o;
  const int64_t G = a.num_gpu_blocks, C = a.num_cpu_blocks, bs = a.block_size;
  o.q0 = a.query_start_loc[r];
  o.qlen = (int64_t)a.query_start_loc[r + 1] - o.q0;
  o.seq = a.seq_lens[r];
  const int64_t used = (o.seq + bs - 1) / bs;
  o.nb = (int)min(used, (int64_t)a.bt_width);
  o.host_blocks = o.hbm_blocks = 0;
  o.host_tok = o.hbm_tok = 0;
  o.bad_id = false;
  const int32_t* row = a.block_table + (int64_t)r * a.bt_stride;
  for (int j = 0; j < o.nb; ++j) {
    const int64_t id = row[j];
    const int64_t t = (j == used - 1) ? o.seq - (used - 1) * bs : bs;
    if (id >= G) {
      ++o.host_blocks;
      o.host_tok += t;
      if (id >= G + C) o.bad_id = true;
    } else {
      ++o.hbm_blocks;
      o.hbm_tok += t;
    }
  }
  o.touches_host = o.host_blocks > 0;
  return o;
}

// counters of pass 1 (per row): P rows, P tokens, S rows, F rows, F tokens,
// P-decode rows, P-prefill rows, P-prefill tokens, decode rows
enum { cP, cPT, cS, cF, cFT, cPD, cPP, cPPT, cD, kCnt };
// maxima of pass 1: P q, P seq, S hbm blocks, S host blocks, S hbm tokens,
// S seq, F q, PD seq, PP q, PP seq, decode seq, any host, bad id, bad class
enum { mPQ, mPK, mSGB, mSCB, mSGL, mSL, mFQ, mPDL, mPPQ, mPPK, mDL, mHost, mBadId, mBadCls, kMax };

__global__ void __launch_bounds__(kPlanThreads, 1) fd_plan_kernel(const fd_plan_args a) {
  __shared__ int64_t sm[kPlanWarps * 16];
  const int R = a.num_reqs;
  const int64_t G = a.num_gpu_blocks, bs = a.block_size;
  const int64_t n_tok = (int64_t)a.query_start_loc[R];

  // ---- pass 0: the offsets must start at 0, never decrease and stay within
  // the token capacity, which bounds every token-indexed write below
  {
    int64_t bad[1] = {0};
    for (int r = threadIdx.x; r < R; r += kPlanThreads)
      if (a.query_start_loc[r + 1] < a.query_start_loc[r]) bad[0] = 1;
    if (threadIdx.x == 0 && (a.query_start_loc[0] != 0 || n_tok > a.max_tokens)) bad[0] = 1;
    block_max<1>(bad, sm);
    if (bad[0]) {
      if (threadIdx.x == 0) {
        for (int k = 0; k < FD_PLAN_HEADER_LEN; ++k) a.header[k] = 0;
        a.header[FD_PLAN_FLAGS] = FD_PLAN_BAD_OFFSETS;
        set_error(a.error, FD_DEVERR_PLAN);
      }
      return;
    }
  }

  // ---- pass 1: rows
  int64_t base[kCnt] = {};
  int64_t mx[kMax];
#pragma unroll
  for (int k = 0; k < kMax; ++k) mx[k] = 0;
  for (int c0 = 0; c0 < R; c0 += kPlanThreads) {
    const int r = c0 + threadIdx.x;
    PlanRow o{};
    bool live = false, S = false, F = false, P = false, bad = false;
    if (r < R) {
      o = plan_row(a, r);
      live = o.qlen > 0;
      S = live && o.touches_host && o.qlen == 1;
      F = live && o.touches_host && o.qlen > 1 && o.seq - o.qlen == 0;
      bad = live && o.touches_host && o.qlen > 1 && o.seq - o.qlen > 0;
      P = live && !o.touches_host;
    }
    const bool PD = P && o.qlen == 1, PP = P && o.qlen > 1, DEC = S || PD;
    int64_t v[kCnt] = {P, P ? o.qlen : 0, S, F, F ? o.qlen : 0, PD, PP, PP ? o.qlen : 0, DEC};
    int64_t tot[kCnt];
    block_scan<kCnt>(v, tot, sm);
    if (r < R) {
      if (P) {
        const int64_t i = base[cP] + v[cP], t0 = base[cPT] + v[cPT];
        a.p_req[i] = r;
        a.p_seqlens[i] = (int32_t)o.seq;
        a.p_cu[i + 1] = (int32_t)(t0 + o.qlen);
        for (int64_t t = 0; t < o.qlen; ++t) a.p_tok[t0 + t] = o.q0 + t;
      }
      if (S) {
        const int64_t i = base[cS] + v[cS];
        a.s_req[i] = r;
        a.s_tok[i] = o.q0;
        a.s_gpu_lens[i] = (int32_t)o.hbm_tok;
        a.s_cpu_lens[i] = (int32_t)o.host_tok;
        a.s_seq_lens[i] = (int32_t)o.seq;
      }
      if (F) {
        const int64_t i = base[cF] + v[cF], t0 = base[cFT] + v[cFT];
        a.f_cu[i + 1] = (int32_t)(t0 + o.qlen);
        for (int64_t t = 0; t < o.qlen; ++t) a.f_tok[t0 + t] = o.q0 + t;
      }
      if (PD) {
        const int64_t i = base[cPD] + v[cPD];
        a.pd_req[i] = r;
        a.pd_tok[i] = o.q0;
        a.pd_seq_lens[i] = (int32_t)o.seq;
      }
      if (PP) {
        const int64_t i = base[cPP] + v[cPP], t0 = base[cPPT] + v[cPPT];
        a.pp_req[i] = r;
        a.pp_seqlens[i] = (int32_t)o.seq;
        a.pp_cu[i + 1] = (int32_t)(t0 + o.qlen);
        for (int64_t t = 0; t < o.qlen; ++t) a.pp_tok[t0 + t] = o.q0 + t;
      }
      if (DEC) {
        const int64_t i = base[cD] + v[cD];
        a.d_tok[i] = o.q0;
        a.d_row[i] = r;
        a.d_lens[i] = (int32_t)o.seq;
      }
      if (P) {
        mx[mPQ] = max(mx[mPQ], o.qlen);
        mx[mPK] = max(mx[mPK], o.seq);
      }
      if (S) {
        mx[mSGB] = max(mx[mSGB], (int64_t)o.hbm_blocks);
        mx[mSCB] = max(mx[mSCB], (int64_t)o.host_blocks);
        mx[mSGL] = max(mx[mSGL], o.hbm_tok);
        mx[mSL] = max(mx[mSL], o.seq);
      }
      if (F) mx[mFQ] = max(mx[mFQ], o.qlen);
      if (PD) mx[mPDL] = max(mx[mPDL], o.seq);
      if (PP) {
        mx[mPPQ] = max(mx[mPPQ], o.qlen);
        mx[mPPK] = max(mx[mPPK], o.seq);
      }
      if (DEC) mx[mDL] = max(mx[mDL], o.seq);
      if (o.touches_host) mx[mHost] = 1;
      if (o.bad_id) mx[mBadId] = 1;
      if (bad) mx[mBadCls] = 1;
    }
#pragma unroll
    for (int k = 0; k < kCnt; ++k) base[k] += tot[k];
  }
  block_max<kMax>(mx, sm);
  if (threadIdx.x == 0) {
    a.p_cu[0] = 0;
    a.f_cu[0] = 0;
    a.pp_cu[0] = 0;
  }
  const int64_t nS = base[cS], nD = base[cD];
  const int gw = (int)((max((int64_t)1, mx[mSGB]) + 15) / 16 * 16);  // HBM table width, padded to 16
  const int cw = (int)max((int64_t)1, mx[mSCB]);                      // host table width

  // decode list padding
  for (int64_t i = nD + threadIdx.x; i < R; i += kPlanThreads) {
    a.d_tok[i] = -1;
    a.d_row[i] = 0;
    a.d_lens[i] = 0;
  }
  __syncthreads();  // s_req of pass 1 is read below

  // ---- pass 2: compacted tables of the S rows
  for (int64_t i = threadIdx.x; i < nS; i += kPlanThreads) {
    const int r = (int)a.s_req[i];
    const int64_t seq = a.seq_lens[r];
    const int nb = (int)min((seq + bs - 1) / bs, (int64_t)a.bt_width);
    const int32_t* row = a.block_table + (int64_t)r * a.bt_stride;
    int32_t* g = a.s_gpu_bt + i * a.s_gpu_bt_stride;
    int32_t* h = a.s_cpu_bt + i * a.s_cpu_bt_stride;
    int ng = 0, nh = 0;
    for (int j = 0; j < nb; ++j) {
      const int64_t id = row[j];
      if (id >= G) h[nh++] = (int32_t)(id - G);
      else g[ng++] = (int32_t)id;
    }
    for (int j = ng; j < gw; ++j) g[j] = 0;
    for (int j = nh; j < cw; ++j) h[j] = 0;
  }

  // ---- pass 3: KV-write routing over the step's tokens
  int64_t nw = 0;
  bool host_slot_any = false;
  for (int64_t c0 = 0; c0 < n_tok; c0 += kPlanThreads) {
    const int64_t t = c0 + threadIdx.x;
    int64_t slot = 0;
    bool host = false;
    if (t < n_tok) {
      slot = a.slot_mapping[t];
      host = slot >= G * bs;
      a.gpu_slot_mapping[t] = host ? -1 : slot;
    }
    int64_t v[1] = {host}, tot[1];
    block_scan<1>(v, tot, sm);
    if (host) {
      a.cpu_w_tok[nw + v[0]] = t;
      a.cpu_w_slot[nw + v[0]] = slot - G * bs;
    }
    nw += tot[0];
    host_slot_any = host_slot_any || tot[0] > 0;
  }

  if (threadIdx.x == 0) {
    int32_t* hd = a.header;
    const bool any = mx[mHost] != 0 || host_slot_any;
    hd[FD_PLAN_FLAGS] = (any ? FD_PLAN_TOUCHES_HOST : 0) | (mx[mBadId] ? FD_PLAN_BAD_BLOCK_ID : 0) |
                        (mx[mBadCls] ? FD_PLAN_HOST_EXTEND : 0);
    hd[FD_PLAN_N_TOK] = (int32_t)n_tok;
    hd[FD_PLAN_N_CPU_W] = (int32_t)nw;
    hd[FD_PLAN_N_P] = (int32_t)base[cP];
    hd[FD_PLAN_N_P_TOK] = (int32_t)base[cPT];
    hd[FD_PLAN_P_MAX_Q] = (int32_t)mx[mPQ];
    hd[FD_PLAN_P_MAX_K] = (int32_t)mx[mPK];
    hd[FD_PLAN_N_S] = (int32_t)nS;
    hd[FD_PLAN_S_GPU_WIDTH] = gw;
    hd[FD_PLAN_S_MAX_GPU_LEN] = (int32_t)mx[mSGL];
    hd[FD_PLAN_S_CPU_WIDTH] = cw;
    hd[FD_PLAN_N_F] = (int32_t)base[cF];
    hd[FD_PLAN_N_F_TOK] = (int32_t)base[cFT];
    hd[FD_PLAN_F_MAX] = (int32_t)mx[mFQ];
    hd[FD_PLAN_S_MAX_LEN] = (int32_t)mx[mSL];
    hd[FD_PLAN_N_PD] = (int32_t)base[cPD];
    hd[FD_PLAN_PD_MAX_LEN] = (int32_t)mx[mPDL];
    hd[FD_PLAN_N_PP] = (int32_t)base[cPP];
    hd[FD_PLAN_N_PP_TOK] = (int32_t)base[cPPT];
    hd[FD_PLAN_PP_MAX_Q] = (int32_t)mx[mPPQ];
    hd[FD_PLAN_PP_MAX_K] = (int32_t)mx[mPPK];
    hd[FD_PLAN_N_DECODE] = (int32_t)nD;
    hd[FD_PLAN_DECODE_MAX_LEN] = (int32_t)mx[mDL];
    if (mx[mBadId]) set_error(a.error, FD_DEVERR_BLOCK_ID);
    if (mx[mBadCls]) set_error(a.error, FD_DEVERR_PLAN);
  }
}

}  // namespace fdk

extern "C" size_t fd_plan_args_bytes(void) { return sizeof(fd_plan_args); }

extern "C" int fd_plan_step(const fd_plan_args* a, void* stream) {
  if (a == nullptr) return fdh::fail(FD_ERR_INVALID, "fd_plan_step: null arguments");
  if (a->num_reqs < 0 || a->bt_width < 1 || a->block_size < 1 || a->num_gpu_blocks < 0 || a->num_cpu_blocks < 0)
    return fdh::fail(FD_ERR_INVALID, "fd_plan_step: bad sizes (reqs %d, width %d, block size %d)", a->num_reqs,
                     a->bt_width, a->block_size);
  if (a->bt_stride < a->bt_width)
    return fdh::fail(FD_ERR_INVALID, "fd_plan_step: bt_stride %lld < bt_width %d", (long long)a->bt_stride,
                     a->bt_width);
  if (a->s_gpu_bt_stride < (a->bt_width + 15) / 16 * 16 || a->s_cpu_bt_stride < a->bt_width)
    return fdh::fail(FD_ERR_INVALID,
                     "fd_plan_step: compacted table strides must hold a full row (HBM %lld >= %d, host %lld >= %d)",
                     (long long)a->s_gpu_bt_stride, (a->bt_width + 15) / 16 * 16, (long long)a->s_cpu_bt_stride,
                     a->bt_width);
  const void* need[] = {a->query_start_loc, a->seq_lens, a->block_table, a->header, a->gpu_slot_mapping,
                        a->cpu_w_tok, a->cpu_w_slot, a->p_tok, a->p_cu, a->p_seqlens, a->p_req, a->s_tok,
                        a->s_gpu_bt, a->s_gpu_lens, a->s_cpu_bt, a->s_cpu_lens, a->f_tok, a->f_cu, a->s_req,
                        a->s_seq_lens, a->pd_req, a->pd_tok, a->pd_seq_lens, a->pp_req, a->pp_tok, a->pp_cu,
                        a->pp_seqlens, a->d_tok, a->d_row, a->d_lens};
  for (const void* ptr : need)
    if (ptr == nullptr) return fdh::fail(FD_ERR_INVALID, "fd_plan_step: a required buffer is null");
  if (a->slot_mapping == nullptr && a->max_tokens > 0)
    return fdh::fail(FD_ERR_INVALID, "fd_plan_step: slot_mapping is null");
  fdk::fd_plan_kernel<<<1, fdk::kPlanThreads, 0, static_cast<cudaStream_t>(stream)>>>(*a);
  return fdh::cuda_status(cudaGetLastError(), "fd_plan_kernel launch");
}
