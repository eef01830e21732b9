// (c) Chunked gated-delta-rule prefill on tcgen05 tensor cores (sm_100a).
//
// One CTA (128 threads, thread t <-> TMEM lane t) walks one (sequence,
// v-head) chain chunk by chunk (64 tokens).  The fp32 state S [dk x dv] lives
// in TMEM for the whole sequence: read from the pool slot at the start,
// written back at the end.  With q^ = l2norm(q)*scale, k^ = l2norm(k),
// gamma = in-chunk cumsum(g) (qwen3_5.py:152-227), every chunk runs five
// M = 128 MMAs (bf16 operands from 128B-swizzled shared memory, fp32
// accumulators in TMEM):
//
//   1. P   = [K;Q] K^T                 raw bf16 rows: exact products; the
//                                      norms and decays are applied after,
//                                      in fp32, to build
//        L   = -(beta_i nk_i nk_j P_ij e^(gamma_i - gamma_j))   (j < i)
//        QKm =  (nq_i nk_j QK_ij e^(gamma_i - gamma_j))          (j <= i)
//      T = (I - L)^-1 by forward substitution on CUDA cores (fp32)
//   2. M2  = QKm T                     (S-independent)
//   3. XQ  = [K;Q] S_bf16              X = K S (rows 0-63), QS (rows 64-127)
//      R   = beta (v - e^gamma nk X)   split into bf16 hi + lo
//   4. VO  = [T;M2] [R_hi;R_lo]        v' = T R (rows 0-63) and the
//                                      intra-chunk output QKm v' (rows 64-127)
//      out = e^gamma nq QS + QKm v'
//      W   = nk e^(gamma_L - gamma) v' split into bf16 hi + lo
//   5. S  += K^T [W_hi;W_lo]           (S pre-scaled by e^gamma_L in TMEM)
//
// The hi/lo splits keep the state path at ~16-bit operand precision (the
// fp32 relative error of final states stays ~1e-4 over 8k-token sequences,
// where plain bf16 operands give ~2e-3); they cost no extra instructions
// beyond doubling the K extent of MMAs 4 and 5.  The same shared K tile is
// read K-major (MMAs 1, 3) and MN-major as K^T (MMA 5).
//
// TMEM columns: S [0,128), XQ [128,256), VO [256,384), P [384,448),
// M2 [448,512).  Every mbarrier wait is bounded; on timeout the CTA sets
// GDN_STATUS_TIMEOUT, frees its TMEM and returns.
#include "tc_util.cuh"

namespace gdn {
namespace tc {

constexpr int kC = 64;
constexpr int kD = 128;
constexpr int kThreads = 128;
constexpr uint32_t kSpin = 1u << 22;
constexpr uint32_t kColS = 0, kColXQ = 128, kColVO = 256, kColP = 384, kColM2 = 448;

struct __align__(1024) ChunkSmem {
  uint8_t kq[2][2][128 * 128];  // [buffer][dk block][row][128 B]: rows 0-63 K, rows 64-127 Q
  uint8_t sb[2][128 * 128];     // S (bf16) [dv block][dk row][128 B]; T / X (fp32) during the inverse
  uint8_t a4[128 * 128];        // [T ; M2] : row x 64 tokens
  uint8_t qkm[128 * 128];       // QKm rows 0-63 (rows 64-127 zero)
  uint8_t whi[2][64 * 128];     // R, then W, hi part; L (fp32) during the inverse
  uint8_t wlo[2][64 * 128];     // lo part
  uint8_t v[2][64 * 256];       // [buffer] v rows, 16-byte chunk c of row i at (c ^ (i % 16))
  float gam[kC], eg[kC], bet[kC], nk[kC], nq[kC];
  unsigned long long mbar;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ void st8(uint8_t* tile, uint32_t row, uint32_t col, const float* f) {
  *reinterpret_cast<uint4*>(tile + sw128(row, col)) = pack8(f);
}

__device__ __forceinline__ void fma4(float (&acc)[4], float a, const float4& b) {
  acc[0] += a * b.x; acc[1] += a * b.y; acc[2] += a * b.z; acc[3] += a * b.w;
}

// T = (I - L)^-1 for the strictly lower 64x64 L (fp32, shared memory), by
// 16x16 diagonal-block forward substitution in registers followed by two
// recursive-doubling levels: with (I - L) = [A 0; -L21 B],
// T = [A^-1 0; B^-1 L21 A^-1  B^-1], applied at 16 -> 32 and 32 -> 64.
__device__ __forceinline__ void invert_unit_lower(const float (*L)[kC + 1], float (*T)[kC],
                                                  float* X, int tid) {
  const int warp = tid >> 5, lane = tid & 31;
  {  // diagonal 16x16 blocks: warp w owns block w, lane l solves column l % 16
    const int b0 = 16 * warp, j = lane & 15;
    float t[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int m = 0; m < i; ++m) {
        const float pr = L[b0 + i][b0 + m] * t[m];
        if (m & 1) s1 += pr; else s0 += pr;
      }
      t[i] = (i == j) ? 1.f : (i > j ? s0 + s1 : 0.f);
    }
    if (lane < 16) {
#pragma unroll
      for (int i = 0; i < 16; ++i) T[b0 + i][b0 + j] = t[i];
    }
    for (int c = b0 + 16 + lane; c < kC; c += 32)    // blocks right of the diagonal are zero
#pragma unroll
      for (int i = 0; i < 16; ++i) T[b0 + i][c] = 0.f;
  }
  __syncthreads();
  {  // 16 -> 32: for both 32-blocks, X = L21 A^-1, then T21 = B^-1 X
    const int hb = (tid >> 6) * 32, r = (tid >> 2) & 15, c0 = (tid & 3) * 4;
    float* Xh = X + (tid >> 6) * 256;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int s = 0; s < 16; ++s)
      fma4(acc, L[hb + 16 + r][hb + s], *reinterpret_cast<const float4*>(&T[hb + s][hb + c0]));
    *reinterpret_cast<float4*>(&Xh[r * 16 + c0]) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    __syncthreads();
    float acc2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int s = 0; s < 16; ++s)
      fma4(acc2, T[hb + 16 + r][hb + 16 + s], *reinterpret_cast<const float4*>(&Xh[s * 16 + c0]));
    *reinterpret_cast<float4*>(&T[hb + 16 + r][hb + c0]) =
        make_float4(acc2[0], acc2[1], acc2[2], acc2[3]);
  }
  __syncthreads();
  {  // 32 -> 64: X = L21 A^-1 (32x32), then T21 = B^-1 X
    const int p = tid >> 3, c0 = (tid & 7) * 4;
    float a0[4] = {0.f, 0.f, 0.f, 0.f}, a1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
    for (int s = 0; s < 32; ++s) {
      const float4 t4 = *reinterpret_cast<const float4*>(&T[s][c0]);
      fma4(a0, L[32 + 2 * p][s], t4);
      fma4(a1, L[33 + 2 * p][s], t4);
    }
    *reinterpret_cast<float4*>(&X[(2 * p) * 32 + c0]) = make_float4(a0[0], a0[1], a0[2], a0[3]);
    *reinterpret_cast<float4*>(&X[(2 * p + 1) * 32 + c0]) = make_float4(a1[0], a1[1], a1[2], a1[3]);
    __syncthreads();
    float b0[4] = {0.f, 0.f, 0.f, 0.f}, b1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
    for (int s = 0; s < 32; ++s) {
      const float4 x4 = *reinterpret_cast<const float4*>(&X[s * 32 + c0]);
      fma4(b0, T[32 + 2 * p][32 + s], x4);
      fma4(b1, T[33 + 2 * p][32 + s], x4);
    }
    *reinterpret_cast<float4*>(&T[32 + 2 * p][c0]) = make_float4(b0[0], b0[1], b0[2], b0[3]);
    *reinterpret_cast<float4*>(&T[33 + 2 * p][c0]) = make_float4(b1[0], b1[1], b1[2], b1[3]);
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kThreads, 1) chunk_prefill_tc_kernel(
    const bf16* __restrict__ q, int64_t qs, const bf16* __restrict__ k, int64_t ks,
    const bf16* __restrict__ v, int64_t vs, const float* __restrict__ g,
    const bf16* __restrict__ beta, float* __restrict__ pool, int64_t slot_stride,
    int64_t num_slots, const int64_t* __restrict__ ids, const int32_t* __restrict__ cu,
    int64_t n_tokens, int max_seqlen, bf16* __restrict__ out, int HK, int HV, float scale,
    int32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  ChunkSmem& sm = *reinterpret_cast<ChunkSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int r = blockIdx.x / HV;
  const int h = blockIdx.x - r * HV;
  const int hk = h / (HV / HK);

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
  const int nchunks = (int)((len + kC - 1) / kC);

  // async loads of chunk c into buffer b (rows past the sequence end are zero-filled)
  auto issue_loads = [&](int c, int b) {
    const int64_t t0 = start + (int64_t)c * kC;
    const int nv = (int)min((int64_t)kC, len - (int64_t)c * kC);
    const uint32_t kq = smem_u32(sm.kq[b][0]);
#pragma unroll 4
    for (int idx = tid; idx < 128 * 16; idx += kThreads) {
      const int row = idx >> 4, ch = idx & 15, i = row & 63;
      const bf16* src = (row >= 64 ? q + (t0 + i) * qs : k + (t0 + i) * ks) + hk * kD + ch * 8;
      cp_async16(kq + (uint32_t)(ch >> 3) * 16384u + sw128(row, (ch & 7) * 8),
                 i < nv ? src : (const bf16*)q, i < nv ? 16u : 0u);
    }
    const uint32_t vb = smem_u32(sm.v[b]);
#pragma unroll 4
    for (int idx = tid; idx < kC * 16; idx += kThreads) {
      const int i = idx >> 4, ch = idx & 15;
      const bf16* src = v + (t0 + i) * vs + h * kD + ch * 8;
      cp_async16(vb + (uint32_t)i * 256u + (uint32_t)((ch ^ (i & 15)) << 4),
                 i < nv ? src : (const bf16*)v, i < nv ? 16u : 0u);
    }
    cp_async_commit();
  };
  auto load_gb = [&](int c, float& gv, float& bv) {
    const int64_t t0 = start + (int64_t)c * kC;
    const int nv = (int)min((int64_t)kC, len - (int64_t)c * kC);
    gv = 0.f; bv = 0.f;
    if (tid < nv) {
      gv = g[(t0 + tid) * HV + h];
      bv = bf2f(beta[(t0 + tid) * HV + h]);
    }
  };

  issue_loads(0, 0);
  float g_next, b_next;
  load_gb(0, g_next, b_next);

  const uint32_t bar = smem_u32(&sm.mbar);
  if (tid == 0) {
    mbar_init(bar, 1);
    mbar_init_fence();
    sm.abort = 0;
  }
  if (warp == 0) tmem_alloc(smem_u32(&sm.tmem_base), 512);
  for (int i = tid; i < 64 * 128 / 16; i += kThreads)   // qkm rows 64-127 stay zero
    reinterpret_cast<uint4*>(sm.qkm + 64 * 128)[i] = make_uint4(0, 0, 0, 0);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tbase = sm.tmem_base;
  const uint32_t tl = tbase + ((uint32_t)(warp * 32) << 16);   // this warp's lane window
  uint32_t phase = 0;

  auto wait_mma = [&]() -> bool {
    const bool ok = mbar_wait(bar, phase, kSpin);
    phase ^= 1u;
    if (!ok) {
      sm.abort = 1;
      if (status) atomicOr(status, GDN_STATUS_TIMEOUT);
    }
    fence_after();
    __syncthreads();
    return sm.abort == 0;
  };

  // initial state -> TMEM (thread t holds dk row t)
  float* sp = pool + slot * slot_stride + (int64_t)h * kD * kD + (int64_t)tid * kD;
#pragma unroll
  for (int cg = 0; cg < 4; ++cg) {
    float s[32];
    const float4* src = reinterpret_cast<const float4*>(sp + cg * 32);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 x = src[i];
      s[4 * i] = x.x; s[4 * i + 1] = x.y; s[4 * i + 2] = x.z; s[4 * i + 3] = x.w;
    }
    tmem_st32(tl + kColS + cg * 32, s);
  }
  tmem_wait_st();

  const uint32_t sb0 = smem_u32(sm.sb[0]);
  const uint32_t a40 = smem_u32(sm.a4);
  const uint32_t qkm0 = smem_u32(sm.qkm);
  const uint32_t hi0 = smem_u32(sm.whi[0]);
  const uint32_t lo0 = smem_u32(sm.wlo[0]);
  float (*Lm)[kC + 1] = reinterpret_cast<float (*)[kC + 1]>(sm.whi);
  float (*Tm)[kC] = reinterpret_cast<float (*)[kC]>(sm.sb);
  float* Xs = reinterpret_cast<float*>(sm.sb[1]);
  bool ok = true;

  for (int c = 0; c < nchunks && ok; ++c) {
    const int buf = c & 1;
    const int64_t t0 = start + (int64_t)c * kC;
    const int nv = (int)min((int64_t)kC, len - (int64_t)c * kC);
    const float g_cur = g_next, b_cur = b_next;
    if (c + 1 < nchunks) {          // prefetch the next chunk while this one computes
      issue_loads(c + 1, buf ^ 1);
      load_gb(c + 1, g_next, b_next);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    if (tid < kC) {
      sm.gam[tid] = g_cur;
      sm.bet[tid] = b_cur;
    }
    __syncthreads();
    const uint32_t kq0 = smem_u32(sm.kq[buf][0]);
    const uint8_t* vrow = sm.v[buf];

    // ---- row norms (thread t: row t of [K;Q]) and the cumulative decay
    {
      float ss = 0.f;
#pragma unroll 4
      for (int ch = 0; ch < 16; ++ch) {
        float f[8];
        unpack8(*reinterpret_cast<const uint4*>(sm.kq[buf][ch >> 3] + sw128(tid, (ch & 7) * 8)),
                f);
#pragma unroll
        for (int e = 0; e < 8; ++e) ss += f[e] * f[e];
      }
      if (tid < 64) sm.nk[tid] = rsqrtf(ss + 1e-6f);
      else sm.nq[tid - 64] = rsqrtf(ss + 1e-6f) * scale;
      if (warp == 0) {   // inclusive scan of g over 64 tokens (2 per lane)
        const float ga = sm.gam[2 * lane], gb = sm.gam[2 * lane + 1];
        float s = ga + gb;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float y = __shfl_up_sync(0xffffffffu, s, o);
          if (lane >= o) s += y;
        }
        const float ex = s - (ga + gb);
        __syncwarp();
        sm.gam[2 * lane] = ex + ga;
        sm.gam[2 * lane + 1] = s;
        sm.eg[2 * lane] = expf(ex + ga);
        sm.eg[2 * lane + 1] = expf(s);
      }
    }
    fence_async_smem();
    fence_before();
    __syncthreads();
    fence_after();

    // ---- (1) P = [K;Q] K^T : M=128, N=64, K=128 (dk)
    if (tid == 0) {
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        const uint32_t off = (uint32_t)(s >> 2) * 16384u + (uint32_t)(s & 3) * 32u;
        mma_bf16(tbase + kColP, smem_desc(kq0 + off, 16, 1024), smem_desc(kq0 + off, 16, 1024),
                 idesc_bf16(128, 64, false, false), s > 0);
      }
      mma_commit(bar);
    }
    if (!(ok = wait_mma())) break;

    // ---- L (threads 0-63) and QKm (threads 64-127) from P
    {
      const int i = tid & 63;
      const bool isq = tid >= 64;
      const float gi = sm.gam[i];
      const float rowf = isq ? sm.nq[i] : -sm.bet[i] * sm.nk[i];
#pragma unroll
      for (int cg = 0; cg < 2; ++cg) {
        float p[32];
        tmem_ld32(tl + kColP + cg * 32, p);
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
          const int j = cg * 32 + jj;
          const bool keep = isq ? (j <= i) : (j < i);
          p[jj] = keep ? rowf * sm.nk[j] * p[jj] * __expf(gi - sm.gam[j]) : 0.f;
        }
        if (isq) {
#pragma unroll
          for (int q8 = 0; q8 < 4; ++q8) st8(sm.qkm, i, cg * 32 + q8 * 8, p + q8 * 8);
        } else {
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) Lm[i][cg * 32 + jj] = p[jj];
        }
      }
    }
    __syncthreads();

    // ---- T = (I - L)^-1 (fp32), then T -> a4 rows 0-63 (bf16)
    invert_unit_lower(Lm, Tm, Xs, tid);
    for (int idx = tid; idx < kC * 8; idx += kThreads) {
      const int i = idx >> 3, c8 = (idx & 7) * 8;
      st8(sm.a4, i, c8, &Tm[i][c8]);
    }
    fence_async_smem();
    fence_before();
    __syncthreads();
    fence_after();

    // ---- (2) M2 = [QKm;0] T : M=128, N=64, K=64; B = T rows (MN-major)
    if (tid == 0) {
#pragma unroll
      for (int s = 0; s < 4; ++s)
        mma_bf16(tbase + kColM2, smem_desc(qkm0 + s * 32, 16, 1024),
                 smem_desc(a40 + s * 2048, 8192, 1024), idesc_bf16(128, 64, false, true), s > 0);
      mma_commit(bar);
    }
    // S (TMEM) -> bf16 MN-major tile (row = dk, col = dv); S *= e^gamma_L in TMEM
    {
      const float egl = sm.eg[kC - 1];
#pragma unroll
      for (int cg = 0; cg < 4; ++cg) {
        float s[32];
        tmem_ld32(tl + kColS + cg * 32, s);
        const int dv0 = cg * 32;
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) st8(sm.sb[dv0 >> 6], tid, (dv0 & 63) + q8 * 8, s + q8 * 8);
#pragma unroll
        for (int e = 0; e < 32; ++e) s[e] *= egl;
        tmem_st32(tl + kColS + cg * 32, s);
      }
    }
    if (!(ok = wait_mma())) break;
    if (tid < 64) {   // M2 rows -> a4 rows 64-127
#pragma unroll
      for (int cg = 0; cg < 2; ++cg) {
        float m[32];
        tmem_ld32(tl + kColM2 + cg * 32, m);
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) st8(sm.a4, 64 + tid, cg * 32 + q8 * 8, m + q8 * 8);
      }
    }
    tmem_wait_st();
    fence_async_smem();
    fence_before();
    __syncthreads();
    fence_after();

    // ---- (3) XQ = [K;Q] S : M=128, N=128, K=128 (dk); B = S rows (MN-major)
    if (tid == 0) {
#pragma unroll
      for (int s = 0; s < 8; ++s)
        mma_bf16(tbase + kColXQ,
                 smem_desc(kq0 + (uint32_t)(s >> 2) * 16384u + (uint32_t)(s & 3) * 32u, 16, 1024),
                 smem_desc(sb0 + s * 2048, 16384, 1024), idesc_bf16(128, 128, false, true), s > 0);
      mma_commit(bar);
    }
    if (!(ok = wait_mma())) break;

    // ---- R = beta (v - e^gamma nk X) -> hi / lo tiles (threads 0-63, token row i)
    if (tid < 64) {
      const int i = tid;
      const float xs = sm.eg[i] * sm.nk[i];
      const float bi = sm.bet[i];
#pragma unroll
      for (int cg = 0; cg < 4; ++cg) {
        float x[32];
        tmem_ld32(tl + kColXQ + cg * 32, x);
        const int dv0 = cg * 32;
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) {
          float vv[8], hi[8], lo[8];
          const int ch = (dv0 >> 3) + q8;
          unpack8(*reinterpret_cast<const uint4*>(vrow + i * 256 + ((ch ^ (i & 15)) << 4)), vv);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float rr = bi * (vv[e] - xs * x[q8 * 8 + e]);
            hi[e] = round_bf(rr);
            lo[e] = rr - hi[e];
          }
          st8(sm.whi[dv0 >> 6], i, (dv0 & 63) + q8 * 8, hi);
          st8(sm.wlo[dv0 >> 6], i, (dv0 & 63) + q8 * 8, lo);
        }
      }
    }
    fence_async_smem();
    fence_before();
    __syncthreads();
    fence_after();

    // ---- (4) VO = [T;M2] [R_hi;R_lo] : M=128, N=128, K=64+64
    if (tid == 0) {
#pragma unroll
      for (int s = 0; s < 8; ++s)
        mma_bf16(tbase + kColVO, smem_desc(a40 + (s & 3) * 32, 16, 1024),
                 smem_desc((s < 4 ? hi0 : lo0) + (s & 3) * 2048, 8192, 1024),
                 idesc_bf16(128, 128, false, true), s > 0);
      mma_commit(bar);
    }
    if (!(ok = wait_mma())) break;

    // ---- epilogue: W = nk e^(gamma_L-gamma) v' (threads 0-63); out rows (64-127)
    if (tid < 64) {
      const int i = tid;
      const float w = sm.nk[i] * expf(sm.gam[kC - 1] - sm.gam[i]);
#pragma unroll
      for (int cg = 0; cg < 4; ++cg) {
        float vp[32];
        tmem_ld32(tl + kColVO + cg * 32, vp);
        const int dv0 = cg * 32;
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) {
          float hi[8], lo[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float x = w * vp[q8 * 8 + e];
            hi[e] = round_bf(x);
            lo[e] = x - hi[e];
          }
          st8(sm.whi[dv0 >> 6], i, (dv0 & 63) + q8 * 8, hi);
          st8(sm.wlo[dv0 >> 6], i, (dv0 & 63) + q8 * 8, lo);
        }
      }
    } else {
      const int i = tid - 64;
      const float f = sm.eg[i] * sm.nq[i];
      bf16* orow = out + ((t0 + i) * HV + h) * kD;
#pragma unroll
      for (int cg = 0; cg < 4; ++cg) {
        float oi[32], qsv[32];
        tmem_ld32(tl + kColVO + cg * 32, oi);
        tmem_ld32(tl + kColXQ + cg * 32, qsv);
        if (i < nv) {
#pragma unroll
          for (int q8 = 0; q8 < 4; ++q8) {
            float o[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = f * qsv[q8 * 8 + e] + oi[q8 * 8 + e];
            *reinterpret_cast<uint4*>(orow + cg * 32 + q8 * 8) = pack8(o);
          }
        }
      }
    }
    fence_async_smem();
    fence_before();
    __syncthreads();
    fence_after();

    // ---- (5) S += K^T [W_hi;W_lo] : M=128 (dk), N=128, K=64+64; A = K^T (MN-major)
    if (tid == 0) {
#pragma unroll
      for (int s = 0; s < 8; ++s)
        mma_bf16(tbase + kColS, smem_desc(kq0 + (s & 3) * 2048, 16384, 1024),
                 smem_desc((s < 4 ? hi0 : lo0) + (s & 3) * 2048, 8192, 1024),
                 idesc_bf16(128, 128, true, true), 1u);
      mma_commit(bar);
    }
    if (!(ok = wait_mma())) break;
  }
  cp_async_wait<0>();   // no copy may still target shared memory when the CTA exits

  if (ok) {   // final state -> pool slot
#pragma unroll
    for (int cg = 0; cg < 4; ++cg) {
      float s[32];
      tmem_ld32(tl + kColS + cg * 32, s);
      float4* dst = reinterpret_cast<float4*>(sp + cg * 32);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        dst[i] = make_float4(s[4 * i], s[4 * i + 1], s[4 * i + 2], s[4 * i + 3]);
    }
  }
  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 0) tmem_dealloc(tbase, 512);
}

}  // namespace tc

bool chunk_tc_supported(int D, const void* q, int64_t qs, const void* k, int64_t ks,
                        const void* v, int64_t vs, const void* out, const void* pool,
                        int64_t slot_stride) {
  return D == tc::kD && aligned16(q) && aligned16(k) && aligned16(v) && aligned16(out) &&
         aligned16(pool) && qs % 8 == 0 && ks % 8 == 0 && vs % 8 == 0 && slot_stride % 4 == 0;
}

int chunk_prefill_tc(int n_seqs, int HV, cudaStream_t s, const bf16* q, int64_t qs,
                     const bf16* k, int64_t ks, const bf16* v, int64_t vs, const float* g,
                     const bf16* beta, float* pool, int64_t slot_stride, int64_t num_slots,
                     const int64_t* ids, const int32_t* cu, int64_t n_tokens, int max_seqlen,
                     bf16* out, int HK, float scale, int32_t* status) {
  const size_t smem = sizeof(tc::ChunkSmem) + 1024;
  cudaError_t e = cudaFuncSetAttribute(tc::chunk_prefill_tc_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) {
    set_error("gdn_chunk_prefill_varlen: cudaFuncSetAttribute failed: %s", cudaGetErrorString(e));
    return GDN_ERR_CUDA;
  }
  tc::chunk_prefill_tc_kernel<<<(unsigned)((int64_t)n_seqs * HV), tc::kThreads, smem, s>>>(
      q, qs, k, ks, v, vs, g, beta, pool, slot_stride, num_slots, ids, cu, n_tokens, max_seqlen,
      out, HK, HV, scale, status);
  return check_launch("gdn_chunk_prefill_varlen");
}

}  // namespace gdn
