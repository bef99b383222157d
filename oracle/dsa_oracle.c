/*
 * CPU oracle for the DSA sparse-MLA decode operator.
 *
 * TEST INFRASTRUCTURE ONLY.  This file checks the CUDA path in the tests and is the
 * timed CPU baseline ("port") of bench.py; nothing in the product path links,
 * loads or calls it.  It restates, in plain C, the reference PyTorch
 * implementation `kernel(...)` in solution/triton/baseline.py of
 * Dogacel/flashinfer-mlsys2026-dsa, step by step:
 *
 *   baseline.py:18-19  flatten the paged caches to [num_slots, 512] / [num_slots, 64]
 *   baseline.py:22-23  valid = idx != -1 ; safe = clamp(idx, min=0)
 *   baseline.py:26-28  gather the selected rows and upcast bf16 -> fp32
 *   baseline.py:30-31  upcast q_nope / q_pe to fp32
 *   baseline.py:34     logits = qn . Kc^T + qp . Kp^T   (two fp32 dot products, then add)
 *   baseline.py:35     logits_scaled = logits * sm_scale   (fp32 multiply)
 *   baseline.py:38     masked_fill(-inf) where idx == -1
 *   baseline.py:41     lse = logsumexp(logits_scaled) / ln(2)     (base-2 LSE)
 *   baseline.py:44     attn = softmax(logits_scaled)
 *   baseline.py:45     out = bf16(attn . Kc)   (round to nearest even)
 *
 * Semantics kept on purpose, including the reference's corner cases:
 *   - an index < -1 is "valid" and reads slot 0 (clamp(min=0) at baseline.py:23);
 *   - a row whose indices are all -1 gets NaN output and lse = -inf (softmax of
 *     an all -inf vector, baseline.py:41,44);
 *   - an index >= num_slots makes the reference raise (out-of-range gather at
 *     baseline.py:27); here the call returns -1 and writes nothing for that row.
 *
 * Accumulation: dot products use 16 independent fp32 partial sums (a BLAS-like
 * order; the reference's fp32 bmm uses its own order), softmax sums use double.
 * The golden fixtures under tests/golden/ (written by the reference itself)
 * pin this file; the differences there are ~1e-6.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define D_CKV 512
#define D_KPE 64

static inline float bf16_to_f32(uint16_t v) {
  uint32_t u = ((uint32_t)v) << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static inline uint16_t f32_to_bf16_rne(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) return 0x7FC0; /* NaN */
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static inline float dot_f32(const float* a, const float* b, int n) {
  float acc[16];
  for (int j = 0; j < 16; ++j) acc[j] = 0.f;
  for (int d = 0; d < n; d += 16)
    for (int j = 0; j < 16; ++j) acc[j] += a[d + j] * b[d + j];
  float s = 0.f;
  for (int j = 0; j < 16; ++j) s += acc[j];
  return s;
}

/* One decode row (all heads).  Scratch: kc [topk*512], kp [topk*64], z [topk]. */
static int oracle_row(const uint16_t* qn_row, const uint16_t* qp_row, const uint16_t* ckv,
                      const uint16_t* kpe, int64_t num_slots, const int32_t* idx_row, int H,
                      int topk, float sm_scale, uint16_t* out_row, float* lse_row, float* kc,
                      float* kp, float* z, unsigned char* valid) {
  for (int k = 0; k < topk; ++k) {
    int32_t i = idx_row[k];
    valid[k] = (i != -1);
    int64_t safe = i < 0 ? 0 : (int64_t)i;
    if (safe >= num_slots) return -1;
    const uint16_t* src_c = ckv + safe * D_CKV;
    const uint16_t* src_p = kpe + safe * D_KPE;
    for (int d = 0; d < D_CKV; ++d) kc[(int64_t)k * D_CKV + d] = bf16_to_f32(src_c[d]);
    for (int d = 0; d < D_KPE; ++d) kp[(int64_t)k * D_KPE + d] = bf16_to_f32(src_p[d]);
  }
  float qn[D_CKV], qp[D_KPE], acc[D_CKV];
  const double ln2 = 0.6931471805599453;
  for (int h = 0; h < H; ++h) {
    for (int d = 0; d < D_CKV; ++d) qn[d] = bf16_to_f32(qn_row[(int64_t)h * D_CKV + d]);
    for (int d = 0; d < D_KPE; ++d) qp[d] = bf16_to_f32(qp_row[(int64_t)h * D_KPE + d]);
    float m = -INFINITY;
    for (int k = 0; k < topk; ++k) {
      float l1 = dot_f32(qn, kc + (int64_t)k * D_CKV, D_CKV);
      float l2 = dot_f32(qp, kp + (int64_t)k * D_KPE, D_KPE);
      float zs = (l1 + l2) * sm_scale;
      z[k] = valid[k] ? zs : -INFINITY;
      if (z[k] > m) m = z[k];
    }
    if (m == -INFINITY) { /* all entries masked: lse = -inf, softmax = NaN */
      lse_row[h] = -INFINITY;
      for (int d = 0; d < D_CKV; ++d) out_row[(int64_t)h * D_CKV + d] = 0x7FC0;
      continue;
    }
    double s = 0.0;
    for (int k = 0; k < topk; ++k) s += exp((double)z[k] - (double)m);
    lse_row[h] = (float)(((double)m + log(s)) / ln2);
    for (int d = 0; d < D_CKV; ++d) acc[d] = 0.f;
    for (int k = 0; k < topk; ++k) {
      if (!valid[k]) continue; /* attn == 0 exactly */
      float a = (float)(exp((double)z[k] - (double)m) / s);
      const float* v = kc + (int64_t)k * D_CKV;
      for (int d = 0; d < D_CKV; ++d) acc[d] += a * v[d];
    }
    for (int d = 0; d < D_CKV; ++d) out_row[(int64_t)h * D_CKV + d] = f32_to_bf16_rne(acc[d]);
  }
  return 0;
}

/*
 * Contiguous layouts: q_nope [B,H,512], q_pe [B,H,64], ckv [num_slots,512],
 * kpe [num_slots,64], idx [B,topk], out [B,H,512] (bf16 bits), lse [B,H].
 * Returns 0, or -1 when an index is >= num_slots (the reference raises there).
 */
int dsa_oracle_decode(const uint16_t* q_nope, const uint16_t* q_pe, const uint16_t* ckv,
                      const uint16_t* kpe, int64_t num_slots, const int32_t* idx, int64_t B,
                      int32_t H, int32_t topk, float sm_scale, uint16_t* out, float* lse,
                      int32_t nthreads) {
  int status = 0;
  if (nthreads < 1) nthreads = 1;
#pragma omp parallel num_threads(nthreads)
  {
    float* kc = (float*)malloc(sizeof(float) * (size_t)topk * D_CKV);
    float* kp = (float*)malloc(sizeof(float) * (size_t)topk * D_KPE);
    float* z = (float*)malloc(sizeof(float) * (size_t)topk);
    unsigned char* valid = (unsigned char*)malloc((size_t)topk);
#pragma omp for schedule(dynamic, 1)
    for (int64_t b = 0; b < B; ++b) {
      int rc = oracle_row(q_nope + b * H * D_CKV, q_pe + b * H * D_KPE, ckv, kpe, num_slots,
                          idx + b * topk, H, topk, sm_scale, out + b * H * D_CKV, lse + b * H, kc,
                          kp, z, valid);
      if (rc != 0) {
#pragma omp atomic write
        status = rc;
      }
    }
    free(kc);
    free(kp);
    free(z);
    free(valid);
  }
  return status;
}

int dsa_oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* ---------------------------------------------------------------- index production
 * Per-row top-k of index scores, translated to slot ids (the step that builds the decode's
 * sparse_indices: slot = page_table[row][pos / page_size] * page_size + pos % page_size, as
 * the reference's callers form page * 64 + offset, baseline.py:17-23; flashinfer publishes
 * the step as top_k_page_table_transform: top k of input[i, :lengths[i]] through the row's
 * table).  Selection: the k largest scores of scores[row, 0:L), L = clamp(lengths[row], 0,
 * max_len), ordered by the IEEE-754 bit pattern (a larger float first, -0.0 below +0.0, NaN
 * below every number), equal scores by the smaller position; the selected positions are
 * written in ascending order, translated, then -1 up to k.  A position past the table or
 * on a negative page gives -1.  Plain sort per row: test sizes only. */
static inline uint32_t score_key(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) return 0u; /* NaN */
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

typedef struct {
  uint32_t key;
  int32_t pos;
} KeyPos;

static int by_key_desc_pos_asc(const void* a, const void* b) {
  const KeyPos* x = (const KeyPos*)a;
  const KeyPos* y = (const KeyPos*)b;
  if (x->key != y->key) return x->key > y->key ? -1 : 1;
  return x->pos < y->pos ? -1 : (x->pos > y->pos ? 1 : 0);
}

static int by_int_asc(const void* a, const void* b) {
  const int32_t x = *(const int32_t*)a, y = *(const int32_t*)b;
  return x < y ? -1 : (x > y ? 1 : 0);
}

int dsa_oracle_topk_slots(const float* scores, int64_t scores_sb, const int32_t* lengths,
                          const int32_t* page_table, int64_t pt_sb, int32_t pt_cols,
                          int32_t page_size, int64_t rows, int32_t max_len, int32_t k,
                          int32_t* out, int64_t out_sb) {
  KeyPos* kp = (KeyPos*)malloc(sizeof(KeyPos) * (size_t)(max_len > 0 ? max_len : 1));
  int32_t* sel = (int32_t*)malloc(sizeof(int32_t) * (size_t)(k > 0 ? k : 1));
  if (!kp || !sel) return -1;
  for (int64_t r = 0; r < rows; ++r) {
    int32_t L = lengths[r];
    if (L < 0) L = 0;
    if (L > max_len) L = max_len;
    const int32_t n = L < k ? L : k;
    if (L <= k) {
      for (int32_t i = 0; i < n; ++i) sel[i] = i;
    } else {
      for (int32_t i = 0; i < L; ++i) {
        kp[i].key = score_key(scores[r * scores_sb + i]);
        kp[i].pos = i;
      }
      qsort(kp, (size_t)L, sizeof(KeyPos), by_key_desc_pos_asc);
      for (int32_t i = 0; i < k; ++i) sel[i] = kp[i].pos;
      qsort(sel, (size_t)k, sizeof(int32_t), by_int_asc);
    }
    for (int32_t i = 0; i < k; ++i) {
      int32_t s = -1;
      if (i < n) {
        const int32_t pos = sel[i], pg = pos / page_size;
        if (pg < pt_cols) {
          const int64_t page = page_table[r * pt_sb + pg];
          const int64_t slot = page * page_size + pos % page_size;
          if (page >= 0 && slot <= 2147483647LL) s = (int32_t)slot;
        }
      }
      out[r * out_sb + i] = s;
    }
  }
  free(kp);
  free(sel);
  return 0;
}
