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
