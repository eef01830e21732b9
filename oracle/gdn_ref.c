/*
 * gdn_ref.c — C restatement of the reference's gated-delta-rule recurrence
 * and chunked prefill (TEST INFRASTRUCTURE ONLY: the checker and the timed
 * CPU baseline, never the product).
 *
 * Follows sileaver/nano-vllm-extend nanovllm/models/qwen3_5.py:
 *   gdn_ref_recurrent_inplace   :616-651 (_torch_recurrent_gated_delta_rule)
 *                               with the slot addressing of :561-613
 *   gdn_ref_chunk_prefill       :152-227 (_torch_chunk_gated_delta_rule),
 *                               per sequence with the state read from and
 *                               written back to its slot (:1039-1077)
 * in fp32, head-mapped by h_k = h_v / (HV / HK) (the repeat_interleave of
 * :1002-1005).  Work is split over (sequence, head) with OpenMP; each unit
 * is computed exactly as the reference's batched tensor ops compute it.
 * Inputs are float32 arrays (bf16 activations already widened by the
 * caller); strides are in elements.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

int gdn_ref_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* Use n threads in later calls (a launcher may have exported OMP_NUM_THREADS=1). */
void gdn_ref_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

static void l2norm_scaled(const float* x, int n, float scale, float* out) {
  float s = 0.f;
  for (int i = 0; i < n; ++i) s += x[i] * x[i];
  const float inv = 1.0f / sqrtf(s + 1e-6f);
  for (int i = 0; i < n; ++i) out[i] = x[i] * inv * scale;
}

/* One decode step for bs sequences; s_pool rows ids[b] updated in place. */
void gdn_ref_recurrent_inplace(const float* q, int64_t qs, const float* k, int64_t ks,
                               const float* v, int64_t vs, const float* g, const float* beta,
                               float* s_pool, int64_t slot_stride, const int64_t* ids,
                               int bs, int HK, int HV, int DK, int DV, float scale,
                               float* out) {
  const int rep = HV / HK;
#pragma omp parallel for schedule(static)
  for (int64_t u = 0; u < (int64_t)bs * HV; ++u) {
    const int b = (int)(u / HV), h = (int)(u % HV), hk = h / rep;
    float qn[256], kn[256], kv[256];
    l2norm_scaled(q + b * qs + hk * DK, DK, scale, qn);
    l2norm_scaled(k + b * ks + hk * DK, DK, 1.0f, kn);
    float* S = s_pool + ids[b] * slot_stride + (int64_t)h * DK * DV;
    const float eg = expf(g[(int64_t)b * HV + h]);
    const float bt = beta[(int64_t)b * HV + h];
    for (int j = 0; j < DV; ++j) kv[j] = 0.f;
    for (int i = 0; i < DK; ++i) {
      float* row = S + (int64_t)i * DV;
      for (int j = 0; j < DV; ++j) {
        row[j] *= eg;
        kv[j] += row[j] * kn[i];
      }
    }
    const float* vv = v + b * vs + h * DV;
    for (int j = 0; j < DV; ++j) kv[j] = (vv[j] - kv[j]) * bt; /* delta */
    float* o = out + ((int64_t)b * HV + h) * DV;
    for (int j = 0; j < DV; ++j) o[j] = 0.f;
    for (int i = 0; i < DK; ++i) {
      float* row = S + (int64_t)i * DV;
      for (int j = 0; j < DV; ++j) {
        row[j] += kn[i] * kv[j];
        o[j] += row[j] * qn[i];
      }
    }
  }
}

#define CH 64

/* Chunked prefill of one (sequence, head) unit: T tokens starting at row t0.
 * Every matrix product keeps the reference's association (the decay factors
 * are applied to an operand before the product, as the batched tensor ops of
 * :201-222 do) and sums over the contracted index in increasing order; the
 * loops run with the output column innermost so they vectorise. */
static void chunk_unit(const float* q, int64_t qs, const float* k, int64_t ks, const float* v,
                       int64_t vs, const float* g, const float* beta, int64_t t0, int64_t T,
                       int h, int hk, int HV, int DK, int DV, float scale, float* S, float* out,
                       float* work) {
  float* Q = work;               /* [CH][DK] */
  float* K = Q + CH * DK;        /* [CH][DK] */
  float* KB = K + CH * DK;       /* k_beta [CH][DK], then k_beta * exp(g) */
  float* VB = KB + CH * DK;      /* v_beta [CH][DV] */
  float* U = VB + CH * DV;       /* value = attn @ v_beta [CH][DV] */
  float* W = U + CH * DV;        /* k_cumdecay [CH][DK] */
  float* VN = W + CH * DK;       /* v_new [CH][DV] */
  float* A = VN + CH * DV;       /* attn [CH][CH] */
  float* DM = A + CH * CH;       /* decay mask [CH][CH] */
  float* QK = DM + CH * CH;      /* [CH][CH] */
  float* SN = QK + CH * CH;      /* new state [DK][DV] */
  float* KE = SN + DK * DV;      /* k * exp(g_last - g) [CH][DK] */
  float* acc = KE + CH * DK;     /* one output row [max(DK, DV)] */
  float G[CH], B[CH], EG[CH];
  const int64_t nch = (T + CH - 1) / CH;
  for (int64_t c = 0; c < nch; ++c) {
    const int64_t base = t0 + c * CH;
    const int nv = (int)((T - c * CH) < CH ? (T - c * CH) : CH);
    for (int i = 0; i < CH; ++i) {
      if (i < nv) {
        l2norm_scaled(q + (base + i) * qs + hk * DK, DK, scale, Q + i * DK);
        l2norm_scaled(k + (base + i) * ks + hk * DK, DK, 1.0f, K + i * DK);
        B[i] = beta[(base + i) * HV + h];
        G[i] = g[(base + i) * HV + h];
        for (int j = 0; j < DV; ++j) VB[i * DV + j] = v[(base + i) * vs + h * DV + j] * B[i];
      } else { /* zero padding (:173-178) */
        memset(Q + i * DK, 0, sizeof(float) * DK);
        memset(K + i * DK, 0, sizeof(float) * DK);
        memset(VB + i * DV, 0, sizeof(float) * DV);
        B[i] = 0.f;
        G[i] = 0.f;
      }
      for (int j = 0; j < DK; ++j) KB[i * DK + j] = K[i * DK + j] * B[i];
    }
    for (int i = 1; i < CH; ++i) G[i] += G[i - 1]; /* cumsum (:193) */
    for (int i = 0; i < CH; ++i) EG[i] = expf(G[i]);
    for (int i = 0; i < CH; ++i)
      for (int j = 0; j < CH; ++j) DM[i * CH + j] = j <= i ? expf(G[i] - G[j]) : 0.f;
    /* attn = -(k_beta k^T * decay), strictly lower (:195) */
    for (int i = 0; i < CH; ++i)
      for (int j = 0; j < CH; ++j) {
        float d = 0.f;
        if (j < i)
          for (int kk = 0; kk < DK; ++kk) d += KB[i * DK + kk] * K[j * DK + kk];
        A[i * CH + j] = j < i ? -(d * DM[i * CH + j]) : 0.f;
      }
    /* forward substitution (:196-199), then + I (:200) */
    for (int i = 1; i < CH; ++i) {
      float row[CH];
      for (int j = 0; j < i; ++j) row[j] = A[i * CH + j];
      for (int j = 0; j < i; ++j) {
        float s = 0.f;
        for (int m = 0; m < i; ++m) s += row[m] * A[m * CH + j];
        A[i * CH + j] = row[j] + s;
      }
    }
    for (int i = 0; i < CH; ++i) A[i * CH + i] += 1.f;
    /* value = attn @ v_beta; k_cumdecay = attn @ (k_beta * exp(g)) (:201-202) */
    for (int m = 0; m < CH; ++m)
      for (int j = 0; j < DK; ++j) KB[m * DK + j] *= EG[m];
    for (int i = 0; i < CH; ++i) {
      float* u = U + i * DV;
      float* w = W + i * DK;
      for (int j = 0; j < DV; ++j) u[j] = 0.f;
      for (int j = 0; j < DK; ++j) w[j] = 0.f;
      for (int m = 0; m < CH; ++m) {
        const float a = A[i * CH + m];
        for (int j = 0; j < DV; ++j) u[j] += a * VB[m * DV + j];
        for (int j = 0; j < DK; ++j) w[j] += a * KB[m * DK + j];
      }
    }
    /* chunk step (:212-222) */
    for (int i = 0; i < CH; ++i)
      for (int j = 0; j < CH; ++j) {
        float d = 0.f;
        for (int kk = 0; kk < DK; ++kk) d += Q[i * DK + kk] * K[j * DK + kk];
        QK[i * CH + j] = d * DM[i * CH + j];
      }
    for (int i = 0; i < CH; ++i) { /* v_new = value - k_cumdecay @ S */
      for (int j = 0; j < DV; ++j) acc[j] = 0.f;
      for (int kk = 0; kk < DK; ++kk) {
        const float w = W[i * DK + kk];
        for (int j = 0; j < DV; ++j) acc[j] += w * S[kk * DV + j];
      }
      for (int j = 0; j < DV; ++j) VN[i * DV + j] = U[i * DV + j] - acc[j];
    }
    for (int i = 0; i < nv; ++i) { /* out = (q * exp(g)) @ S + attn @ v_new */
      float* o = out + ((base + i) * HV + h) * DV;
      for (int j = 0; j < DV; ++j) acc[j] = 0.f;
      for (int kk = 0; kk < DK; ++kk) {
        const float qe = Q[i * DK + kk] * EG[i];
        for (int j = 0; j < DV; ++j) acc[j] += qe * S[kk * DV + j];
      }
      for (int j = 0; j < DV; ++j) o[j] = 0.f;
      for (int m = 0; m < CH; ++m) {
        const float a = QK[i * CH + m];
        for (int j = 0; j < DV; ++j) o[j] += a * VN[m * DV + j];
      }
      for (int j = 0; j < DV; ++j) o[j] += acc[j];
    }
    /* S = S * exp(g_last) + (k * exp(g_last - g))^T @ v_new */
    const float gl = G[CH - 1], egl = expf(gl);
    for (int m = 0; m < CH; ++m) {
      const float e = expf(gl - G[m]);
      for (int kk = 0; kk < DK; ++kk) KE[m * DK + kk] = K[m * DK + kk] * e;
    }
    for (int kk = 0; kk < DK; ++kk) {
      float* sn = SN + kk * DV;
      for (int j = 0; j < DV; ++j) sn[j] = 0.f;
      for (int m = 0; m < CH; ++m) {
        const float a = KE[m * DK + kk];
        for (int j = 0; j < DV; ++j) sn[j] += a * VN[m * DV + j];
      }
      for (int j = 0; j < DV; ++j) sn[j] += S[kk * DV + j] * egl;
    }
    memcpy(S, SN, sizeof(float) * DK * DV);
  }
}

/* Varlen chunked prefill; sequence r owns rows [cu[r], cu[r+1]). */
void gdn_ref_chunk_prefill(const float* q, int64_t qs, const float* k, int64_t ks,
                           const float* v, int64_t vs, const float* g, const float* beta,
                           float* s_pool, int64_t slot_stride, const int64_t* ids,
                           const int32_t* cu, int n_seqs, int HK, int HV, int DK, int DV,
                           float scale, float* out) {
  const int rep = HV / HK;
  const size_t work_floats = (size_t)CH * (5 * DK + 4 * DV) + 3 * CH * CH + (size_t)DK * DV +
                             (size_t)(DK > DV ? DK : DV);
#pragma omp parallel
  {
    float* work = (float*)malloc(sizeof(float) * work_floats);
#pragma omp for schedule(dynamic, 1)
    for (int64_t u = 0; u < (int64_t)n_seqs * HV; ++u) {
      const int r = (int)(u / HV), h = (int)(u % HV);
      const int64_t t0 = cu[r], T = (int64_t)cu[r + 1] - cu[r];
      if (T <= 0) continue;
      float* S = s_pool + ids[r] * slot_stride + (int64_t)h * DK * DV;
      chunk_unit(q, qs, k, ks, v, vs, g, beta, t0, T, h, h / rep, HV, DK, DV, scale, S, out,
                 work);
    }
    free(work);
  }
}
