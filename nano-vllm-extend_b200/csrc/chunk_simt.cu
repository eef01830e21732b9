// (c) Chunked gated-delta-rule prefill — fp32 CUDA-core kernel.
//
// One CTA per (sequence, v-head) walks the sequence's 64-token chunks in
// order, keeping the DK x DV fp32 state in shared memory from the slot read
// to the slot write.  Per chunk, with q^ = l2norm(q)*scale, k^ = l2norm(k),
// gamma = in-chunk cumsum(g) (qwen3_5.py:152-227):
//   L   = -(beta_i k^_i . k^_j) exp(gamma_i - gamma_j)      (j < i)
//   T   = (I - L)^-1                          forward substitution, :196-200
//   R   = beta * (v - exp(gamma) * (k^ S))
//   v'  = T R                                 (= U - W S of :201-202, :215-216)
//   o   = exp(gamma) * (q^ S) + ((q^ k^T) . D) v'             :214, :217-218
//   S   = exp(gamma_L) S + (k^ exp(gamma_L - gamma))^T v'     :219-222
// Rows past the sequence end are zero (k = v = beta = g = 0), the padded-
// chunk convention of the reference, so they leave the state unchanged.
//
// This kernel is the exact-arithmetic path: every product is fp32 on CUDA
// cores.  Shared memory per CTA (DK = DV = 128): raw bf16 q/k (32 KiB),
// fp32 v/R and v' (64 KiB), S (64 KiB), T and L/QK (32 KiB).
#include "common.cuh"

namespace gdn {

constexpr int kChunk = 64;

template <int D>
struct SimtSmem {
  bf16 qb[kChunk][D + 2];  // +2: rows land on distinct banks
  bf16 kb[kChunk][D + 2];
  float vr[kChunk][D];   // v, then R
  float vp[kChunk][D];   // v'
  float S[D][D];
  float T[kChunk][kChunk];
  float A[kChunk][kChunk];  // L, then QK
  float nq[kChunk], nk[kChunk], gam[kChunk], eg[kChunk], bet[kChunk], kd[kChunk];
};

template <int D, int NT>
__global__ void __launch_bounds__(NT) chunk_prefill_simt_kernel(
    const bf16* __restrict__ q, int64_t qs, const bf16* __restrict__ k, int64_t ks,
    const bf16* __restrict__ v, int64_t vs, const float* __restrict__ g,
    const bf16* __restrict__ beta, float* __restrict__ pool, int64_t slot_stride,
    int64_t num_slots, const int64_t* __restrict__ ids, const int32_t* __restrict__ cu,
    int64_t n_tokens, int max_seqlen, bf16* __restrict__ out, int HK, int HV, float scale,
    int32_t* status) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  SimtSmem<D>& sm = *reinterpret_cast<SimtSmem<D>*>(smem_raw);
  const int r = blockIdx.x / HV;
  const int h = blockIdx.x - r * HV;
  const int hk = h / (HV / HK);
  const int tid = threadIdx.x;

  const int64_t slot = ids[r];
  if (!slot_ok(slot, num_slots, status)) return;
  const int64_t start = cu[r];
  int64_t len = (int64_t)cu[r + 1] - start;
  if (start < 0 || len < 0 || start + len > n_tokens) {
    if (tid == 0 && status) atomicOr(status, GDN_STATUS_BAD_SEQLEN);
    return;
  }
  if (len > max_seqlen) {
    if (tid == 0 && status) atomicOr(status, GDN_STATUS_BAD_SEQLEN);
    len = max_seqlen;
  }
  if (len == 0) return;

  float* sp = pool + slot * slot_stride + (int64_t)h * D * D;
  for (int i = tid; i < D * D; i += NT) (&sm.S[0][0])[i] = sp[i];

  const int nchunks = (int)((len + kChunk - 1) / kChunk);
  for (int c = 0; c < nchunks; ++c) {
    const int64_t t0 = start + (int64_t)c * kChunk;
    const int nv = (int)min((int64_t)kChunk, len - (int64_t)c * kChunk);
    __syncthreads();  // previous chunk's readers of the buffers are done
    // (a) load the chunk; rows >= nv are zero
    for (int idx = tid; idx < kChunk * D; idx += NT) {
      const int i = idx / D, j = idx - (idx / D) * D;
      bf16 qv = __float2bfloat16_rn(0.f), kv = qv;
      float vv = 0.f;
      if (i < nv) {
        qv = q[(t0 + i) * qs + (int64_t)hk * D + j];
        kv = k[(t0 + i) * ks + (int64_t)hk * D + j];
        vv = bf2f(v[(t0 + i) * vs + (int64_t)h * D + j]);
      }
      sm.qb[i][j] = qv;
      sm.kb[i][j] = kv;
      sm.vr[i][j] = vv;
    }
    if (tid < kChunk) {
      sm.gam[tid] = tid < nv ? g[(t0 + tid) * HV + h] : 0.f;
      sm.bet[tid] = tid < nv ? bf2f(beta[(t0 + tid) * HV + h]) : 0.f;
    }
    __syncthreads();
    // (b) row norms and the in-chunk cumulative decay
    if (tid < kChunk) {
      float aq = 0.f, ak = 0.f;
      for (int jj = 0; jj < D; ++jj) {
        const int j = (jj + tid) % D;
        const float a = bf2f(sm.qb[tid][j]), b = bf2f(sm.kb[tid][j]);
        aq += a * a;
        ak += b * b;
      }
      sm.nq[tid] = rsqrtf(aq + 1e-6f) * scale;
      sm.nk[tid] = rsqrtf(ak + 1e-6f);
    } else if (tid == kChunk) {
      float acc = 0.f;
      for (int i = 0; i < kChunk; ++i) {
        acc += sm.gam[i];
        sm.gam[i] = acc;
        sm.eg[i] = expf(acc);
      }
    }
    __syncthreads();
    if (tid < kChunk) sm.kd[tid] = sm.nk[tid] * expf(sm.gam[kChunk - 1] - sm.gam[tid]);
    // (c) L = -(beta_i k^_i.k^_j) exp(gamma_i - gamma_j), strictly lower
    for (int idx = tid; idx < kChunk * kChunk; idx += NT) {
      const int i = idx / kChunk, j = idx % kChunk;
      float val = 0.f;
      if (j < i) {
        float dot = 0.f;
        for (int kk = 0; kk < D; ++kk) dot += bf2f(sm.kb[i][kk]) * bf2f(sm.kb[j][kk]);
        val = -(sm.bet[i] * sm.nk[i] * sm.nk[j] * dot) * expf(sm.gam[i] - sm.gam[j]);
      }
      sm.A[i][j] = val;
    }
    __syncthreads();
    // (d) T = (I - L)^-1: column j solved independently by thread j
    if (tid < kChunk) {
      const int j = tid;
      for (int i = 0; i <= j; ++i) sm.T[i][j] = (i == j) ? 1.f : 0.f;
      for (int i = j + 1; i < kChunk; ++i) {
        float x = sm.A[i][j];
        for (int m = j + 1; m < i; ++m) x += sm.A[i][m] * sm.T[m][j];
        sm.T[i][j] = x;
      }
    }
    __syncthreads();
    // (e) QK = (q^_i . k^_j) exp(gamma_i - gamma_j), lower incl. diagonal
    for (int idx = tid; idx < kChunk * kChunk; idx += NT) {
      const int i = idx / kChunk, j = idx % kChunk;
      float val = 0.f;
      if (j <= i) {
        float dot = 0.f;
        for (int kk = 0; kk < D; ++kk) dot += bf2f(sm.qb[i][kk]) * bf2f(sm.kb[j][kk]);
        val = sm.nq[i] * sm.nk[j] * dot * expf(sm.gam[i] - sm.gam[j]);
      }
      sm.A[i][j] = val;
    }
    // (f) R = beta * (v - exp(gamma) * (k^ S))    (elementwise in place)
    for (int idx = tid; idx < kChunk * D; idx += NT) {
      const int i = idx / D, cc = idx - (idx / D) * D;
      float x = 0.f;
      for (int kk = 0; kk < D; ++kk) x += bf2f(sm.kb[i][kk]) * sm.S[kk][cc];
      x *= sm.nk[i];
      sm.vr[i][cc] = sm.bet[i] * (sm.vr[i][cc] - sm.eg[i] * x);
    }
    __syncthreads();
    // (g) v' = T R
    for (int idx = tid; idx < kChunk * D; idx += NT) {
      const int i = idx / D, cc = idx - (idx / D) * D;
      float x = 0.f;
      for (int j = 0; j <= i; ++j) x += sm.T[i][j] * sm.vr[j][cc];
      sm.vp[i][cc] = x;
    }
    __syncthreads();
    // (h) o = exp(gamma) (q^ S) + QK v'
    for (int idx = tid; idx < kChunk * D; idx += NT) {
      const int i = idx / D, cc = idx - (idx / D) * D;
      if (i >= nv) continue;
      float inter = 0.f;
      for (int kk = 0; kk < D; ++kk) inter += bf2f(sm.qb[i][kk]) * sm.S[kk][cc];
      inter *= sm.nq[i] * sm.eg[i];
      float intra = 0.f;
      for (int j = 0; j <= i; ++j) intra += sm.A[i][j] * sm.vp[j][cc];
      out[((t0 + i) * HV + h) * D + cc] = f2bf(inter + intra);
    }
    __syncthreads();
    // (i) S = exp(gamma_L) S + (k^ exp(gamma_L - gamma))^T v'
    const float egl = sm.eg[kChunk - 1];
    for (int idx = tid; idx < D * D; idx += NT) {
      const int kk = idx / D, cc = idx - (idx / D) * D;
      float x = 0.f;
      for (int j = 0; j < kChunk; ++j)
        x += bf2f(sm.kb[j][kk]) * sm.kd[j] * sm.vp[j][cc];
      sm.S[kk][cc] = sm.S[kk][cc] * egl + x;
    }
  }
  __syncthreads();
  for (int i = tid; i < D * D; i += NT) sp[i] = (&sm.S[0][0])[i];
}

template <int D>
static int launch_chunk_simt(int n_seqs, int HV, cudaStream_t s, const bf16* q, int64_t qs,
                             const bf16* k, int64_t ks, const bf16* v, int64_t vs, const float* g,
                             const bf16* beta, float* pool, int64_t slot_stride, int64_t num_slots,
                             const int64_t* ids, const int32_t* cu, int64_t n_tokens,
                             int max_seqlen, bf16* out, int HK, float scale, int32_t* status) {
  constexpr int NT = 256;
  const size_t smem = sizeof(SimtSmem<D>);
  cudaError_t e = cudaFuncSetAttribute(chunk_prefill_simt_kernel<D, NT>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) {
    set_error("gdn_chunk_prefill_varlen: cudaFuncSetAttribute failed: %s", cudaGetErrorString(e));
    return GDN_ERR_CUDA;
  }
  chunk_prefill_simt_kernel<D, NT><<<(unsigned)((int64_t)n_seqs * HV), NT, smem, s>>>(
      q, qs, k, ks, v, vs, g, beta, pool, slot_stride, num_slots, ids, cu, n_tokens, max_seqlen,
      out, HK, HV, scale, status);
  return check_launch("gdn_chunk_prefill_varlen");
}

int chunk_prefill_simt(int n_seqs, int HV, int D, cudaStream_t s, const bf16* q, int64_t qs,
                       const bf16* k, int64_t ks, const bf16* v, int64_t vs, const float* g,
                       const bf16* beta, float* pool, int64_t slot_stride, int64_t num_slots,
                       const int64_t* ids, const int32_t* cu, int64_t n_tokens, int max_seqlen,
                       bf16* out, int HK, float scale, int32_t* status) {
  if (D == 128)
    return launch_chunk_simt<128>(n_seqs, HV, s, q, qs, k, ks, v, vs, g, beta, pool, slot_stride,
                                  num_slots, ids, cu, n_tokens, max_seqlen, out, HK, scale, status);
  return launch_chunk_simt<64>(n_seqs, HV, s, q, qs, k, ks, v, vs, g, beta, pool, slot_stride,
                               num_slots, ids, cu, n_tokens, max_seqlen, out, HK, scale, status);
}

bool chunk_tc_supported(int D, const void* q, int64_t qs, const void* k, int64_t ks,
                        const void* v, int64_t vs, const void* out, const void* pool,
                        int64_t slot_stride, const void* z, int64_t zs, const void* nw);
int chunk_prefill_tc(int n_seqs, int HV, cudaStream_t s, const bf16* q, int64_t qs,
                     const bf16* k, int64_t ks, const bf16* v, int64_t vs, const float* g,
                     const bf16* beta, float* pool, int64_t slot_stride, int64_t num_slots,
                     const int64_t* ids, const int32_t* cu, int64_t n_tokens, int max_seqlen,
                     bf16* out, int HK, float scale, const bf16* z, int64_t zs, const bf16* nw,
                     float eps, int32_t* status);
int64_t chunk_wy_capacity(int64_t n_tokens, int64_t n_seqs);
int64_t chunk_wy_workspace_bytes(int64_t n_tokens, int64_t n_seqs, int64_t HV);
int chunk_prefill_wy(int n_seqs, int HV, cudaStream_t s, const bf16* q, int64_t qs,
                     const bf16* k, int64_t ks, const bf16* v, int64_t vs, const float* g,
                     const bf16* beta, float* pool, int64_t slot_stride, int64_t num_slots,
                     const int64_t* ids, const int32_t* cu, int64_t n_tokens, int max_seqlen,
                     bf16* out, int HK, float scale, void* workspace, int32_t* status);

}  // namespace gdn

using namespace gdn;

extern "C" int gdn_chunk_prefill_varlen(const void* q, int64_t q_row_stride, const void* k,
                                        int64_t k_row_stride, const void* v, int64_t v_row_stride,
                                        const float* g, const void* beta, float* s_pool,
                                        int64_t slot_stride, int64_t num_slots, const int64_t* ids,
                                        const int32_t* cu_seqlens, int32_t n_seqs,
                                        int64_t n_tokens, int32_t max_seqlen, void* out,
                                        int32_t num_k_heads, int32_t num_v_heads,
                                        int32_t head_k_dim, int32_t head_v_dim, float scale,
                                        const void* z, int64_t z_row_stride,
                                        const void* norm_weight, float norm_eps,
                                        void* workspace, int64_t workspace_bytes,
                                        int32_t* status, void* stream) {
  clear_error();
  GDN_REQUIRE(n_seqs >= 0 && n_tokens >= 0 && max_seqlen >= 0 && num_k_heads > 0 &&
                  num_v_heads > 0,
              "gdn_chunk_prefill_varlen: bad sizes");
  GDN_REQUIRE(num_v_heads % num_k_heads == 0,
              "gdn_chunk_prefill_varlen: num_v_heads %d not a multiple of num_k_heads %d",
              num_v_heads, num_k_heads);
  GDN_UNSUPPORTED((head_k_dim == 128 && head_v_dim == 128) || (head_k_dim == 64 && head_v_dim == 64),
                  "gdn_chunk_prefill_varlen: head dims (%d, %d) unsupported", head_k_dim,
                  head_v_dim);
  GDN_REQUIRE(q_row_stride >= (int64_t)num_k_heads * head_k_dim &&
                  k_row_stride >= (int64_t)num_k_heads * head_k_dim &&
                  v_row_stride >= (int64_t)num_v_heads * head_v_dim,
              "gdn_chunk_prefill_varlen: row stride smaller than the heads it holds");
  GDN_REQUIRE(num_slots > 0 && slot_stride >= (int64_t)num_v_heads * head_k_dim * head_v_dim,
              "gdn_chunk_prefill_varlen: slot_stride too small");
  GDN_REQUIRE(z == nullptr || (norm_weight != nullptr &&
                                z_row_stride >= (int64_t)num_v_heads * head_v_dim),
              "gdn_chunk_prefill_varlen: fused norm needs norm_weight and z rows of HV*DV");
  if (n_seqs == 0 || n_tokens == 0) return GDN_OK;
  // token rows are int32 TMA coordinates and (sequence, head) chains one CTA each
  GDN_UNSUPPORTED(n_tokens < (1ll << 31) && (int64_t)n_seqs * num_v_heads < (1ll << 31),
                  "gdn_chunk_prefill_varlen: %lld tokens / %lld chains exceed 2^31",
                  (long long)n_tokens, (long long)n_seqs * num_v_heads);
  GDN_REQUIRE(q && k && v && g && beta && s_pool && ids && cu_seqlens && out,
              "gdn_chunk_prefill_varlen: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  const bool tc = chunk_tc_supported(head_k_dim, q, q_row_stride, k, k_row_stride, v,
                                     v_row_stride, out, s_pool, slot_stride, z, z_row_stride,
                                     norm_weight);
  if (tc && workspace != nullptr) {
    const int64_t need = chunk_wy_workspace_bytes(n_tokens, n_seqs, num_v_heads);
    GDN_REQUIRE(workspace_bytes >= need && aligned16(workspace),
                "gdn_chunk_prefill_varlen: workspace of %lld bytes (16-byte aligned) needed, "
                "got %lld", (long long)need, (long long)workspace_bytes);
    // (chunk, head) blocks are numbered by int32 and launched one CTA each
    GDN_UNSUPPORTED(chunk_wy_capacity(n_tokens, n_seqs) * num_v_heads < (1ll << 31),
                    "gdn_chunk_prefill_varlen: %lld chunk blocks exceed 2^31",
                    (long long)(chunk_wy_capacity(n_tokens, n_seqs) * num_v_heads));
    int rc = chunk_prefill_wy(n_seqs, num_v_heads, s, (const bf16*)q, q_row_stride,
                              (const bf16*)k, k_row_stride, (const bf16*)v, v_row_stride, g,
                              (const bf16*)beta, s_pool, slot_stride, num_slots, ids, cu_seqlens,
                              n_tokens, max_seqlen, (bf16*)out, num_k_heads, scale, workspace,
                              status);
    if (rc == GDN_OK && z != nullptr)
      rc = launch_rms_norm_gated(out, z, z_row_stride, num_v_heads, norm_weight, out,
                                 n_tokens * num_v_heads, head_v_dim, norm_eps, s);
    return rc;
  }
  if (tc)
    return chunk_prefill_tc(n_seqs, num_v_heads, s, (const bf16*)q, q_row_stride, (const bf16*)k,
                            k_row_stride, (const bf16*)v, v_row_stride, g, (const bf16*)beta,
                            s_pool, slot_stride, num_slots, ids, cu_seqlens, n_tokens, max_seqlen,
                            (bf16*)out, num_k_heads, scale, (const bf16*)z, z_row_stride,
                            (const bf16*)norm_weight, norm_eps, status);
  int rc = chunk_prefill_simt(n_seqs, num_v_heads, head_k_dim, s, (const bf16*)q, q_row_stride,
                              (const bf16*)k, k_row_stride, (const bf16*)v, v_row_stride, g,
                              (const bf16*)beta, s_pool, slot_stride, num_slots, ids, cu_seqlens,
                              n_tokens, max_seqlen, (bf16*)out, num_k_heads, scale, status);
  if (rc == GDN_OK && z != nullptr)   // the fp32 kernel stores o; norm it in place
    rc = launch_rms_norm_gated(out, z, z_row_stride, num_v_heads, norm_weight, out,
                               n_tokens * num_v_heads, head_v_dim, norm_eps, s);
  return rc;
}

extern "C" int64_t gdn_chunk_prefill_workspace_bytes(int64_t n_tokens, int32_t n_seqs,
                                                     int32_t num_v_heads, int32_t head_k_dim,
                                                     int32_t head_v_dim) {
  if (n_tokens <= 0 || n_seqs <= 0 || num_v_heads <= 0 || head_k_dim != 128 || head_v_dim != 128)
    return 0;
  return chunk_wy_workspace_bytes(n_tokens, n_seqs, num_v_heads);
}
