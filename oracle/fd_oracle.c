/*
 * TEST INFRASTRUCTURE ONLY -- not part of the product.  Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg load this file's
 * library, and only as a checker / timing baseline.
 *
 * Plain-C restatement of the reference algorithm of the decode path of
 * Cybercricetus/vllm_fastdecoder (file:line within that project):
 *
 *   fdo_decode_attn   fastdecode/csrc/cpu_attn.cpp:298-411 (decode_attn_impl)
 *                     with the tier lookup of fastdecode/plan.py:3-4 added
 *                     (block id < split -> tier 0, else tier 1 at id - split)
 *   fdo_store_kv      fastdecode/csrc/cpu_attn.cpp:413-431 + range check
 *                     :506-510
 *   fdo_merge2        fastdecode/cpu_ops.py:93-113 (merge_partials_torch)
 *   fdo_merge_parts   the same rule over P parts (cpu_attn.cpp:9-17)
 *
 * Numerics as in the reference: fp16/bf16 widened exactly to fp32, q
 * pre-scaled in fp32 (:338), two passes per (row, kv head): scores, max,
 * exp(s - max) and their sum, then P.V in fp32; out = acc * (1/sum)
 * rounded to nearest-even into the output type (:401-405); lse = max +
 * log(sum) (:406); an empty row gives zeros and lse = -inf (:324-331).
 * The one difference is the exponential: the reference evaluates a Cephes
 * polynomial in AVX2 (:124-154, rel. err ~2e-7); this file calls libm expf.
 *
 * Layout of a tier: element (block b, kv head h, token t, dim d) is at
 * base + b*blk_stride + h*head_stride + t*tok_stride + d (elements).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

enum { FDO_F16 = 0, FDO_BF16 = 1, FDO_F32 = 2 };

static float half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: renormalise */
      exp = 127 - 15 + 1;
      while ((man & 0x400u) == 0) {
        man <<= 1;
        exp--;
      }
      man &= 0x3ffu;
      bits = sign | (exp << 23) | (man << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

static float bf16_to_float(uint16_t b) {
  const uint32_t bits = (uint32_t)b << 16;
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

/* round-to-nearest-even float -> binary16 */
static uint16_t float_to_half(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t absx = x & 0x7fffffffu;
  if (absx >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (absx > 0x7f800000u ? 0x200u : 0));
  if (absx >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* rounds to >= 65520 -> inf */
  if (absx < 0x38800000u) { /* below 2^-14: subnormal (or zero) in binary16 */
    /* result = |f| / 2^-24 rounded half-to-even; exact in double */
    const double r = fabs((double)f) * 16777216.0;
    const double fl = floor(r);
    const double diff = r - fl;
    uint32_t qi = (uint32_t)fl;
    if (diff > 0.5 || (diff == 0.5 && (qi & 1u))) qi++;
    return (uint16_t)(sign | qi); /* qi == 0x400 is the smallest normal */
  }
  const uint32_t e = (absx >> 23) - 127 + 15;
  uint32_t m = absx & 0x7fffffu;
  uint32_t hv = (e << 10) | (m >> 13);
  const uint32_t rem = m & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (hv & 1u))) hv++;
  return (uint16_t)(sign | hv);
}

/* round-to-nearest-even float -> bfloat16 (NaN stays NaN) */
static uint16_t float_to_bf16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u);
  const uint32_t lsb = (x >> 16) & 1u;
  x += 0x7fffu + lsb;
  return (uint16_t)(x >> 16);
}

static float load_elem(const void* base, int64_t idx, int dtype) {
  switch (dtype) {
    case FDO_F16:
      return half_to_float(((const uint16_t*)base)[idx]);
    case FDO_BF16:
      return bf16_to_float(((const uint16_t*)base)[idx]);
    default:
      return ((const float*)base)[idx];
  }
}

static void store_elem(void* base, int64_t idx, int dtype, float v) {
  switch (dtype) {
    case FDO_F16:
      ((uint16_t*)base)[idx] = float_to_half(v);
      break;
    case FDO_BF16:
      ((uint16_t*)base)[idx] = float_to_bf16(v);
      break;
    default:
      ((float*)base)[idx] = v;
  }
}

int fdo_elem_size(int dtype) { return dtype == FDO_F32 ? 4 : 2; }

/* exported for tests of the conversions themselves */
float fdo_half_to_float(uint16_t h) { return half_to_float(h); }
uint16_t fdo_float_to_half(float f) { return float_to_half(f); }
uint16_t fdo_float_to_bf16(float f) { return float_to_bf16(f); }

typedef struct {
  const void* k;
  const void* v;
  int64_t blk_stride, head_stride, tok_stride, num_blocks;
} fdo_tier;

/*
 * q[i,h,d] at q + i*q_sn + h*q_sh + d; out[i,h,d] at out + i*o_sn + h*o_sh + d
 * (out_dtype may be FDO_F32 for partials); lse[h*lse_sh + i*lse_sn].
 * block ids < split -> tier0, else tier1 at id - split.
 * Returns 0, or -1 if a block id is outside its tier, -2 if a row needs
 * more blocks than W.
 */
int fdo_decode_attn(const void* q, int64_t q_sn, int64_t q_sh, const fdo_tier* tier0,
                    const fdo_tier* tier1, int64_t split, const int32_t* bt, int64_t bt_stride,
                    int32_t W, const int32_t* lens, int32_t n, int32_t H, int32_t KVH, int32_t D,
                    int32_t BS, float scale, int32_t dtype, void* out, int32_t out_dtype,
                    int64_t o_sn, int64_t o_sh, float* lse, int64_t lse_sh, int64_t lse_sn) {
  const int G = H / KVH;
  float* qf = (float*)malloc(sizeof(float) * (size_t)G * D);
  float* acc = (float*)malloc(sizeof(float) * (size_t)G * D);
  float* mx = (float*)malloc(sizeof(float) * G);
  float* sm = (float*)malloc(sizeof(float) * G);
  float* scores = NULL;
  size_t cap = 0;
  int rc = 0;
  for (int i = 0; i < n && rc == 0; ++i) {
    const int len = lens[i];
    for (int kh = 0; kh < KVH && rc == 0; ++kh) {
      if (len <= 0) {
        for (int g = 0; g < G; ++g) {
          const int h = kh * G + g;
          for (int d = 0; d < D; ++d) store_elem(out, i * o_sn + h * o_sh + d, out_dtype, 0.f);
          if (lse) lse[h * lse_sh + i * lse_sn] = -INFINITY;
        }
        continue;
      }
      const int nb = (len + BS - 1) / BS;
      if (nb > W) {
        rc = -2;
        break;
      }
      for (int g = 0; g < G; ++g) {
        const int h = kh * G + g;
        for (int d = 0; d < D; ++d) qf[g * D + d] = load_elem(q, i * q_sn + h * q_sh + d, dtype) * scale;
      }
      if (cap < (size_t)G * len) {
        cap = (size_t)G * len;
        scores = (float*)realloc(scores, sizeof(float) * cap);
      }
      /* pass 1: scores */
      for (int t = 0; t < len; ++t) {
        int64_t id = bt[i * bt_stride + t / BS];
        const fdo_tier* tr = tier0;
        if (id >= split) {
          tr = tier1;
          id -= split;
        }
        if (tr == NULL || id < 0 || id >= tr->num_blocks) {
          rc = -1;
          break;
        }
        const int64_t row = id * tr->blk_stride + kh * tr->head_stride + (t % BS) * tr->tok_stride;
        for (int g = 0; g < G; ++g) {
          float s = 0.f;
          for (int d = 0; d < D; ++d) s += qf[g * D + d] * load_elem(tr->k, row + d, dtype);
          scores[(size_t)g * len + t] = s;
        }
      }
      if (rc) break;
      /* softmax numerators */
      for (int g = 0; g < G; ++g) {
        float* sg = scores + (size_t)g * len;
        float m = -INFINITY;
        for (int t = 0; t < len; ++t) m = sg[t] > m ? sg[t] : m;
        float s = 0.f;
        for (int t = 0; t < len; ++t) {
          sg[t] = expf(sg[t] - m);
          s += sg[t];
        }
        mx[g] = m;
        sm[g] = s;
      }
      /* pass 2: P.V */
      memset(acc, 0, sizeof(float) * (size_t)G * D);
      for (int t = 0; t < len; ++t) {
        int64_t id = bt[i * bt_stride + t / BS];
        const fdo_tier* tr = tier0;
        if (id >= split) {
          tr = tier1;
          id -= split;
        }
        const int64_t row = id * tr->blk_stride + kh * tr->head_stride + (t % BS) * tr->tok_stride;
        for (int g = 0; g < G; ++g) {
          const float p = scores[(size_t)g * len + t];
          for (int d = 0; d < D; ++d) acc[g * D + d] += p * load_elem(tr->v, row + d, dtype);
        }
      }
      for (int g = 0; g < G; ++g) {
        const int h = kh * G + g;
        const float inv = 1.f / sm[g];
        for (int d = 0; d < D; ++d) store_elem(out, i * o_sn + h * o_sh + d, out_dtype, acc[g * D + d] * inv);
        if (lse) lse[h * lse_sh + i * lse_sn] = mx[g] + logf(sm[g]);
      }
    }
  }
  free(qf);
  free(acc);
  free(mx);
  free(sm);
  free(scores);
  return rc;
}

/* Reference-shaped call: contiguous q [n,H,D], cache [C,KVH,BS,D], bt [n,W],
 * out [n,H,D] (q dtype), lse [H,n]. */
int fdo_decode_attn_paged(const void* q, const void* kc, const void* vc, const int32_t* bt,
                          const int32_t* lens, int32_t n, int32_t H, int32_t KVH, int32_t D,
                          int32_t BS, int64_t C, int32_t W, float scale, int32_t dtype, void* out,
                          float* lse) {
  fdo_tier t = {kc, vc, (int64_t)KVH * BS * D, (int64_t)BS * D, D, C};
  return fdo_decode_attn(q, (int64_t)H * D, D, &t, NULL, INT64_MAX, bt, W, W, lens, n, H, KVH, D, BS,
                         scale, dtype, out, dtype, (int64_t)H * D, D, lse, n, 1);
}

/* k, v [m, KVH, D] contiguous; slots [m] int64 cache-relative; caches
 * [C, KVH, BS, D].  Returns -1 (and writes nothing) if any slot is outside
 * [0, C*BS), as the reference raises before writing (cpu_attn.cpp:506-510). */
int fdo_store_kv(const void* k, const void* v, const int64_t* slots, int32_t m, int32_t KVH,
                 int32_t D, int32_t BS, int64_t C, int32_t dtype, void* kc, void* vc) {
  const int es = fdo_elem_size(dtype);
  for (int j = 0; j < m; ++j)
    if (slots[j] < 0 || slots[j] >= C * BS) return -1;
  for (int j = 0; j < m; ++j) {
    const int64_t blk = slots[j] / BS, off = slots[j] % BS;
    for (int h = 0; h < KVH; ++h) {
      const int64_t dst = (blk * KVH + h) * BS * D + off * D;
      const int64_t src = ((int64_t)j * KVH + h) * D;
      memcpy((char*)kc + dst * es, (const char*)k + src * es, (size_t)D * es);
      memcpy((char*)vc + dst * es, (const char*)v + src * es, (size_t)D * es);
    }
  }
  return 0;
}

/* merge_partials_torch (cpu_ops.py:93-113): o_a, o_b [n,H,D] of in_dtype,
 * lse [H,n]; out [n,H,D] fp32. */
void fdo_merge2(const void* o_a, const float* lse_a, const void* o_b, const float* lse_b,
                int32_t in_dtype, int32_t n, int32_t H, int32_t D, float* out, float* out_lse) {
  for (int h = 0; h < H; ++h) {
    for (int i = 0; i < n; ++i) {
      float a = lse_a[h * n + i], b = lse_b[h * n + i];
      if (a == INFINITY) a = -INFINITY;
      if (b == INFINITY) b = -INFINITY;
      float m = a > b ? a : b;
      const int both_empty = (m == -INFINITY);
      if (both_empty) m = 0.f;
      float wa = expf(a - m), wb = expf(b - m);
      float tot = wa + wb;
      if (both_empty) tot = 1.f;
      wa = wa / tot;
      wb = wb / tot;
      for (int d = 0; d < D; ++d) {
        const int64_t idx = ((int64_t)i * H + h) * D + d;
        out[idx] = load_elem(o_a, idx, in_dtype) * wa + load_elem(o_b, idx, in_dtype) * wb;
      }
      if (out_lse) out_lse[h * n + i] = both_empty ? -INFINITY : m + logf(tot);
    }
  }
}

/* P-way version over fp32 parts: part p at o + p*part_stride ([n,H,D]) and
 * lse + p*part_stride ([H,n]). */
void fdo_merge_parts(const float* o, const float* lse, int64_t part_stride, int32_t P, int32_t n,
                     int32_t H, int32_t D, float* out, float* out_lse) {
  float* w = (float*)malloc(sizeof(float) * (size_t)P);
  for (int h = 0; h < H; ++h) {
    for (int i = 0; i < n; ++i) {
      float m = -INFINITY;
      for (int p = 0; p < P; ++p) {
        float x = lse[p * part_stride + h * n + i];
        if (x == INFINITY) x = -INFINITY;
        m = x > m ? x : m;
      }
      const int empty = (m == -INFINITY);
      if (empty) m = 0.f;
      float tot = 0.f;
      for (int p = 0; p < P; ++p) {
        float x = lse[p * part_stride + h * n + i];
        if (x == INFINITY) x = -INFINITY;
        w[p] = expf(x - m);
        tot += w[p];
      }
      if (empty) tot = 1.f;
      for (int d = 0; d < D; ++d) {
        const int64_t idx = ((int64_t)i * H + h) * D + d;
        float acc = 0.f;
        for (int p = 0; p < P; ++p) acc += o[p * part_stride + idx] * (w[p] / tot);
        out[idx] = acc;
      }
      if (out_lse) out_lse[h * n + i] = empty ? -INFINITY : m + logf(tot);
    }
  }
  free(w);
}
