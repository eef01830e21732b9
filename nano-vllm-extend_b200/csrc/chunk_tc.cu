// (c) Chunked gated-delta-rule prefill on tcgen05 tensor cores (sm_100a).
//
// One CTA (128 threads, thread t <-> TMEM lane t; two CTAs per SM) walks one
// (sequence, v-head) chain chunk by chunk (64 tokens), the chains launched
// longest first.  The fp32 state S [dk x dv] lives in TMEM for the whole
// sequence: read from the pool slot at the start, written back at the end.  With q^ = l2norm(q)*scale, k^ = l2norm(k),
// gamma = in-chunk cumsum(g) (qwen3_5.py:152-227), every chunk runs five
// M = 128 MMAs (bf16 operands from 128B-swizzled shared memory, fp32
// accumulators in TMEM):
//
//   1. P   = [K;Q] [K;Q]^T             raw bf16 rows: exact products; its
//                                      diagonal gives the row norms, and the
//                                      norms and decays are applied in fp32
//                                      to build
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
// The decay e^(gamma_i - gamma_j) of entries left of the 16-token diagonal
// block is the product of two factors e^(gamma_i - gamma_end(J)) and
// e^(gamma_end(J) - gamma_j), both <= 1 for g <= 0 (as the gate produces), so
// it never overflows and needs ~5x fewer exponentials than the direct form.
// Every mbarrier wait is bounded; on timeout the CTA sets GDN_STATUS_TIMEOUT,
// frees its TMEM and returns.
#include <cuda.h>

#include "tc_util.cuh"
#include "tmap.cuh"

namespace gdn {
namespace tc {

constexpr int kC = 64;
constexpr int kD = 128;
constexpr int kLptMaxSeqs = 256;   // longest-first chain order up to this many sequences
constexpr int kThreads = 128;
constexpr uint32_t kSpin = 1u << 22;
constexpr uint32_t kTmemCols = 256;
// TMEM columns: S [0,128) for the whole sequence; a 128-column work region
// [128,256) holds, in turn, P = [K;Q][K;Q]^T, M2, and the XQ / VO accumulator.
constexpr uint32_t kColS = 0, kColW = 128;

// Shared memory (~106 KiB: two CTAs fit on an SM).  `scratch` is reused in
// turn: L then T in place (fp32 [64][68]) plus X (fp32 32x32) during the
// inverse; the bf16 S tile for MMA 3; then the R and W hi / lo tiles.
struct __align__(1024) ChunkSmem {
  uint8_t kq[2][128 * 128];   // [dk block][row][128 B]: rows 0-63 K, rows 64-127 Q
  uint8_t scratch[32768];
  uint8_t qkm[64 * 128];      // QKm rows 0-63; MMA 2's rows 64-127 read a4's first rows
  uint8_t a4[128 * 128];      // [T ; M2] : row x 64 tokens
  uint8_t v[2][64 * 128];     // [dv block][token row][128 B] (128B-swizzled, as TMA writes)
  float gam[kC], eg[kC], bet[kC], nk[kC], nq[kC], bcol[kC], cf[kC], gend[4];
  unsigned long long mbar;    // MMA completion
  unsigned long long lbar[3]; // TMA loads: K, Q, V
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ void st8(uint8_t* tile, uint32_t row, uint32_t col, const float* f) {
  *reinterpret_cast<uint4*>(tile + sw128(row, col)) = pack8(f);
}

// x = hi + lo exactly: hi = x truncated to bf16 (upper 16 bits), lo = the
// remainder rounded to bf16 (|lo| < 2^-7 |x|, so hi + lo carries ~16 bits).
__device__ __forceinline__ void split8(const float* x, uint8_t* tile_hi, uint8_t* tile_lo,
                                       uint32_t off) {
  uint4 h, l;
  uint32_t* hp = reinterpret_cast<uint32_t*>(&h);
  __nv_bfloat162* lp = reinterpret_cast<__nv_bfloat162*>(&l);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const uint32_t b0 = __float_as_uint(x[2 * e]), b1 = __float_as_uint(x[2 * e + 1]);
    hp[e] = __byte_perm(b0, b1, 0x7632);
    lp[e] = __floats2bfloat162_rn(x[2 * e] - __uint_as_float(b0 & 0xFFFF0000u),
                                  x[2 * e + 1] - __uint_as_float(b1 & 0xFFFF0000u));
  }
  *reinterpret_cast<uint4*>(tile_hi + off) = h;
  *reinterpret_cast<uint4*>(tile_lo + off) = l;
}

__device__ __forceinline__ void fma4(float (&acc)[4], float a, const float4& b) {
  ffma2(acc[0], acc[1], a, a, b.x, b.y, acc[0], acc[1]);
  ffma2(acc[2], acc[3], a, a, b.z, b.w, acc[2], acc[3]);
}

constexpr int kLP = kC + 4;   // row pitch of L / T (16-byte aligned rows)

// T = (I - L)^-1 for the strictly lower 64x64 L (fp32, shared memory, upper
// triangle zero), computed IN PLACE (T overwrites L): 16x16 diagonal blocks by
// forward substitution in registers, then two recursive-doubling levels —
// with (I - L) = [A 0; -L21 B], T = [A^-1 0; B^-1 L21 A^-1  B^-1] — at
// 16 -> 32 and 32 -> 64.  Each level reads its L21 block before the T21 that
// replaces it is written.  128 threads; X is a 4 KiB fp32 scratch.
__device__ __forceinline__ void invert_unit_lower(float (*LT)[kLP], float* X, int tid) {
  const int warp = tid >> 5, lane = tid & 31;
  {  // diagonal 16x16 blocks: warp w owns block w, lane l solves column l % 16
    const int b0 = 16 * warp, j = lane & 15;
    float t[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int m = 0; m < i; ++m) {
        const float pr = LT[b0 + i][b0 + m] * t[m];
        if (m & 1) s1 += pr; else s0 += pr;
      }
      t[i] = (i == j) ? 1.f : (i > j ? s0 + s1 : 0.f);
    }
    __syncwarp();
    if (lane < 16) {
#pragma unroll
      for (int i = 0; i < 16; ++i) LT[b0 + i][b0 + j] = t[i];
    }
  }
  __syncthreads();
  {  // 16 -> 32: for both 32-blocks, X = L21 A^-1, then T21 = B^-1 X (4 outputs / thread)
    const int hsel = tid >> 6, hb = hsel * 32, r = (tid >> 2) & 15, c0 = (tid & 3) * 4;
    float* Xh = X + hsel * 256;
    float a[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int s = 0; s < 16; ++s)
      fma4(a, LT[hb + 16 + r][hb + s], *reinterpret_cast<const float4*>(&LT[hb + s][hb + c0]));
    *reinterpret_cast<float4*>(&Xh[r * 16 + c0]) = make_float4(a[0], a[1], a[2], a[3]);
    __syncthreads();
    float b[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int s = 0; s < 16; ++s)
      fma4(b, LT[hb + 16 + r][hb + 16 + s], *reinterpret_cast<const float4*>(&Xh[s * 16 + c0]));
    *reinterpret_cast<float4*>(&LT[hb + 16 + r][hb + c0]) = make_float4(b[0], b[1], b[2], b[3]);
  }
  __syncthreads();
  {  // 32 -> 64: X = L21 A^-1 (32x32), then T21 = B^-1 X (8 outputs / thread)
    const int rr = tid >> 2, c0 = (tid & 3) * 8;
    float a0[4] = {0.f, 0.f, 0.f, 0.f}, a1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
    for (int s = 0; s < 32; ++s) {
      const float l = LT[32 + rr][s];
      fma4(a0, l, *reinterpret_cast<const float4*>(&LT[s][c0]));
      fma4(a1, l, *reinterpret_cast<const float4*>(&LT[s][c0 + 4]));
    }
    *reinterpret_cast<float4*>(&X[rr * 32 + c0]) = make_float4(a0[0], a0[1], a0[2], a0[3]);
    *reinterpret_cast<float4*>(&X[rr * 32 + c0 + 4]) = make_float4(a1[0], a1[1], a1[2], a1[3]);
    __syncthreads();
    float b0[4] = {0.f, 0.f, 0.f, 0.f}, b1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
    for (int s = 0; s < 32; ++s) {
      const float t = LT[32 + rr][32 + s];
      fma4(b0, t, *reinterpret_cast<const float4*>(&X[s * 32 + c0]));
      fma4(b1, t, *reinterpret_cast<const float4*>(&X[s * 32 + c0 + 4]));
    }
    *reinterpret_cast<float4*>(&LT[32 + rr][c0]) = make_float4(b0[0], b0[1], b0[2], b0[3]);
    *reinterpret_cast<float4*>(&LT[32 + rr][c0 + 4]) = make_float4(b1[0], b1[1], b1[2], b1[3]);
  }
  __syncthreads();
}

// Longest chains first: CTA rank k (of n_seqs) takes the sequence with the
// k-th largest length (ties by index), so the long serial chains start in the
// first wave and the short ones fill in behind them.  The ranks form a
// permutation for any cu_seqlens, malformed ones included.  Kept out of line so
// it does not weigh on the main loop's register allocation.
__device__ __noinline__ int lpt_sequence(const int32_t* __restrict__ cu, int n_seqs, int rank,
                                         int tid) {
  __shared__ int s_len[kLptMaxSeqs];
  __shared__ int s_seq;
  if (n_seqs > kLptMaxSeqs) return rank;
  for (int i = tid; i < n_seqs; i += kThreads) s_len[i] = cu[i + 1] - cu[i];
  if (tid == 0) s_seq = rank;
  __syncthreads();
  for (int i = tid; i < n_seqs; i += kThreads) {
    const int li = s_len[i];
    int rk = 0;
    for (int j = 0; j < n_seqs; ++j) {
      const int lj = s_len[j];
      rk += (lj > li) || (lj == li && j < i);
    }
    if (rk == rank) s_seq = i;
  }
  __syncthreads();
  return s_seq;
}

__global__ void __launch_bounds__(kThreads, 2) chunk_prefill_tc_kernel(
    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
    const __grid_constant__ CUtensorMap tm_v, const float* __restrict__ g,
    const bf16* __restrict__ beta, float* __restrict__ pool, int64_t slot_stride,
    int64_t num_slots, const int64_t* __restrict__ ids, const int32_t* __restrict__ cu,
    int64_t n_tokens, int max_seqlen, bf16* __restrict__ out, int HK, int HV, float scale,
    int32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  ChunkSmem& sm = *reinterpret_cast<ChunkSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int rank = blockIdx.x / HV;
  const int h = blockIdx.x - rank * HV;
  const int hk = h / (HV / HK);
  const int r = lpt_sequence(cu, gridDim.x / HV, rank, tid);

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

  // TMA loads of chunk c: K / Q into the [K;Q] tile, V into the v tile.  Rows
  // past the sequence end hold the next sequence's rows (or TMA zeros past
  // n_tokens); they are cleared after arrival (clear_tail).
  const uint32_t kq_s = smem_u32(sm.kq[0]);
  auto load_k = [&](int c) {
    if (tid == 0) {
      const uint32_t b = smem_u32(&sm.lbar[0]);
      mbar_expect_tx(b, 2 * 8192);
      for (int blk = 0; blk < 2; ++blk)
        tma_load_2d(kq_s + blk * 16384, &tm_k, hk * kD + blk * 64, (int)(start + c * kC), b);
    }
  };
  auto load_q = [&](int c) {
    if (tid == 0) {
      const uint32_t b = smem_u32(&sm.lbar[1]);
      mbar_expect_tx(b, 2 * 8192);
      for (int blk = 0; blk < 2; ++blk)
        tma_load_2d(kq_s + blk * 16384 + 64 * 128, &tm_q, hk * kD + blk * 64,
                    (int)(start + c * kC), b);
    }
  };
  auto load_v = [&](int c) {
    if (tid == 0) {
      const uint32_t b = smem_u32(&sm.lbar[2]);
      mbar_expect_tx(b, 2 * 8192);
      for (int blk = 0; blk < 2; ++blk)
        tma_load_2d(smem_u32(sm.v[blk]), &tm_v, h * kD + blk * 64, (int)(start + c * kC), b);
    }
  };
  // g and beta of chunk c for thread tid < 64 (raw; converted when used)
  auto load_gb = [&](int c, float& gv, unsigned short& bv) {
    const int64_t t0 = start + (int64_t)c * kC;
    const int nv = (int)min((int64_t)kC, len - (int64_t)c * kC);
    gv = 0.f; bv = 0;
    if (tid < nv) {
      gv = __ldg(g + (t0 + tid) * HV + h);
      bv = __ldg(reinterpret_cast<const unsigned short*>(beta) + (t0 + tid) * HV + h);
    }
  };

  float g_next;
  unsigned short b_next;
  load_gb(0, g_next, b_next);

  const uint32_t bar = smem_u32(&sm.mbar);
  if (tid == 0) {
    mbar_init(bar, 1);
    for (int i = 0; i < 3; ++i) mbar_init(smem_u32(&sm.lbar[i]), 1);
    mbar_init_fence();
    sm.abort = 0;
  }
  __syncthreads();
  load_k(0);
  load_q(0);
  load_v(0);
  uint32_t lphase[3] = {0u, 0u, 0u};
  if (warp == 0) tmem_alloc(smem_u32(&sm.tmem_base), kTmemCols);
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
  auto wait_load = [&](int i) {     // bounded wait for TMA load i (0 K, 1 Q, 2 V)
    if (!mbar_wait(smem_u32(&sm.lbar[i]), lphase[i], kSpin)) {
      sm.abort = 1;
      if (status) atomicOr(status, GDN_STATUS_TIMEOUT);
    }
    lphase[i] ^= 1u;
  };
  auto sync_for_mma = [&]() {      // smem operands + TMEM stores -> visible to the MMA
    fence_async_smem();
    fence_before();
    __syncthreads();
    fence_after();
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

  const uint32_t kq0 = smem_u32(sm.kq[0]);
  const uint32_t scr0 = smem_u32(sm.scratch);
  const uint32_t a40 = smem_u32(sm.a4);
  const uint32_t qkm0 = smem_u32(sm.qkm);
  constexpr uint32_t kLoOff = 16384;                 // W / R lo tiles after the hi tiles
  uint8_t* whi = sm.scratch;                         // [dv block][token row][128 B] x 2
  uint8_t* wlo = sm.scratch + kLoOff;
  float (*Lm)[kLP] = reinterpret_cast<float (*)[kLP]>(sm.scratch);   // L, then T in place
  float* Xs = reinterpret_cast<float*>(sm.scratch + kC * kLP * 4);
  bool ok = true;

  for (int c = 0; c < nchunks && ok; ++c) {
    const int64_t t0 = start + (int64_t)c * kC;
    const int nv = (int)min((int64_t)kC, len - (int64_t)c * kC);
    wait_load(0);
    wait_load(1);
    wait_load(2);
    if (tid < kC) {
      sm.gam[tid] = g_next;
      sm.bet[tid] = __bfloat162float(__ushort_as_bfloat16(b_next));
    }
    if (nv < kC) {   // clear rows past the sequence end in the K, Q and v tiles
      for (int idx = tid; idx < (kC - nv) * 16; idx += kThreads) {
        const int i = nv + idx / 16, ch = idx % 16, blk = ch >> 3, c8 = (ch & 7) * 8;
        const uint4 z = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(sm.kq[blk] + sw128(i, c8)) = z;
        *reinterpret_cast<uint4*>(sm.kq[blk] + sw128(64 + i, c8)) = z;
        *reinterpret_cast<uint4*>(sm.v[blk] + sw128(i, c8)) = z;
      }
    }
    __syncthreads();
    if (sm.abort) { ok = false; break; }
    if (warp == 0) {   // cumulative decay (inclusive scan, 2 tokens per lane) and its factors
      const float ga = sm.gam[2 * lane], gb = sm.gam[2 * lane + 1];
      float s = ga + gb;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, s, o);
        if (lane >= o) s += y;
      }
      const float g0 = s - gb;                      // gamma of token 2*lane
      // gamma at the end of each 16-token block (token 16J+15 = lane 8J+7, second element)
      const float gE = __shfl_sync(0xffffffffu, s, ((2 * lane) >> 4) * 8 + 7);
      __syncwarp();
      sm.gam[2 * lane] = g0;
      sm.gam[2 * lane + 1] = s;
      sm.eg[2 * lane] = expf(g0);
      sm.eg[2 * lane + 1] = expf(s);
      sm.bcol[2 * lane] = __expf(gE - g0);          // <= 1 (g <= 0)
      sm.bcol[2 * lane + 1] = __expf(gE - s);
      if ((lane & 7) == 7) sm.gend[lane >> 3] = s;
    }
    sync_for_mma();

    // ---- (1) P = [K;Q] [K;Q]^T : M=128, N=128, K=128 (dk); diag gives the norms
    if (tid == 0) {
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        const uint32_t off = (uint32_t)(s >> 2) * 16384u + (uint32_t)(s & 3) * 32u;
        mma_bf16(tbase + kColW, smem_desc(kq0 + off, 16, 1024), smem_desc(kq0 + off, 16, 1024),
                 idesc_bf16(128, 128, false, false), s > 0);
      }
      mma_commit(bar);
    }
    if (!(ok = wait_mma())) break;
    {   // norms: P[t][t] sits in this warp's 32-column diagonal window
      float p[32];
      tmem_ld32(tl + kColW + warp * 32, p);
      float d = 0.f;
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) d = (jj == lane) ? p[jj] : d;
      if (tid < 64) {
        const float n = rsqrtf(d + 1e-6f);
        sm.nk[tid] = n;
        sm.cf[tid] = n * sm.bcol[tid];
      } else {
        sm.nq[tid - 64] = rsqrtf(d + 1e-6f) * scale;
      }
    }
    __syncthreads();

    // ---- L (rows 0-63) and QKm (rows 64-127) from P; then scale Q rows by e^gamma nq
    {
      const int i = tid & 63;
      const bool isq = tid >= 64;
      const int I = i >> 4;
      const float gi = sm.gam[i];
      const float rowf = isq ? sm.nq[i] : -sm.bet[i] * sm.nk[i];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        float p[32];
        tmem_ld32(tl + kColW + hh * 32, p);
#pragma unroll
        for (int b2 = 0; b2 < 2; ++b2) {
          const int J = hh * 2 + b2;
          float* pe = p + b2 * 16;
          if (J < I) {
            // left of the diagonal block: e^(gamma_i - gamma_j) =
            // e^(gamma_i - gamma_end(J)) * e^(gamma_end(J) - gamma_j), both <= 1
            const float rf = rowf * __expf(gi - sm.gend[J]);
#pragma unroll
            for (int jj = 0; jj < 16; jj += 2) {
              const float2 c2 = *reinterpret_cast<const float2*>(&sm.cf[J * 16 + jj]);
              float f0, f1;
              fmul2(f0, f1, rf, rf, c2.x, c2.y);
              fmul2(pe[jj], pe[jj + 1], pe[jj], pe[jj + 1], f0, f1);
            }
          } else if (J == I) {
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) {
              const int j = J * 16 + jj;
              const bool keep = isq ? (j <= i) : (j < i);
              pe[jj] = keep ? pe[jj] * rowf * sm.nk[j] * __expf(gi - sm.gam[j]) : 0.f;
            }
          } else {
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) pe[jj] = 0.f;
          }
        }
        if (isq) {
#pragma unroll
          for (int q8 = 0; q8 < 4; ++q8) st8(sm.qkm, i, hh * 32 + q8 * 8, p + q8 * 8);
        } else {
#pragma unroll
          for (int q4 = 0; q4 < 8; ++q4)
            *reinterpret_cast<float4*>(&Lm[i][hh * 32 + q4 * 4]) =
                make_float4(p[4 * q4], p[4 * q4 + 1], p[4 * q4 + 2], p[4 * q4 + 3]);
        }
      }
    }
    __syncthreads();

    // ---- T = (I - L)^-1 (fp32, in place), then T -> a4 rows 0-63 (bf16)
    invert_unit_lower(Lm, Xs, tid);
    for (int idx = tid; idx < kC * 8; idx += kThreads) {
      const int i = idx >> 3, c8 = (idx & 7) * 8;
      st8(sm.a4, i, c8, &Lm[i][c8]);
    }
    sync_for_mma();

    // ---- (2) M2 = [QKm; *] T : M=128, N=64, K=64; B = T rows (MN-major)
    if (tid == 0) {
#pragma unroll
      for (int s = 0; s < 4; ++s)
        mma_bf16(tbase + kColW, smem_desc(qkm0 + s * 32, 16, 1024),
                 smem_desc(a40 + s * 2048, 8192, 1024), idesc_bf16(128, 64, false, true), s > 0);
      mma_commit(bar);
    }
    // S (TMEM) -> bf16 MN-major tile (row = dk, col = dv); S *= e^gamma_L in TMEM
    {
      const float egl = sm.eg[kC - 1];
#pragma unroll
      for (int cg = 0; cg < 4; ++cg) {
        float s[32];
        const int dv0 = cg * 32;
        tmem_ld32(tl + kColS + dv0, s);
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8)
          st8(sm.scratch + (dv0 >> 6) * 16384, tid, (dv0 & 63) + q8 * 8, s + q8 * 8);
#pragma unroll
        for (int e = 0; e < 32; e += 2) fmul2(s[e], s[e + 1], s[e], s[e + 1], egl, egl);
        tmem_st32(tl + kColS + dv0, s);
      }
    }
    if (!(ok = wait_mma())) break;
    if (tid < 64) {   // M2 rows -> a4 rows 64-127
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        float m[32];
        tmem_ld32(tl + kColW + hh * 32, m);
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) st8(sm.a4, 64 + tid, hh * 32 + q8 * 8, m + q8 * 8);
      }
    }
    tmem_wait_st();
    sync_for_mma();

    // ---- (3) XQ = [K; Q] S : M=128, N=128, K=128 (dk); B = S rows (MN-major)
    if (tid == 0) {
#pragma unroll
      for (int s = 0; s < 8; ++s)
        mma_bf16(tbase + kColW,
                 smem_desc(kq0 + (uint32_t)(s >> 2) * 16384u + (uint32_t)(s & 3) * 32u, 16, 1024),
                 smem_desc(scr0 + s * 2048, 16384, 1024), idesc_bf16(128, 128, false, true), s > 0);
      mma_commit(bar);
    }
    if (!(ok = wait_mma())) break;
    if (c + 1 < nchunks) load_q(c + 1);   // Q rows are no longer read this chunk

    // ---- R = beta (v - e^gamma nk X) -> hi / lo tiles (rows 0-63); clear those TMEM rows.
    // Meanwhile the threads of rows 64-127 scale QS by e^gamma nq in TMEM (fp32), so
    // MMA 4 adds the intra-chunk term onto the inter-chunk output.
    if (tid >= 64) {
      const int i = tid - 64;
      const float f = sm.eg[i] * sm.nq[i];
#pragma unroll
      for (int cg = 0; cg < 4; ++cg) {
        float x[32];
        tmem_ld32(tl + kColW + cg * 32, x);
#pragma unroll
        for (int e = 0; e < 32; e += 2) fmul2(x[e], x[e + 1], x[e], x[e + 1], f, f);
        tmem_st32(tl + kColW + cg * 32, x);
      }
    }
    if (tid < 64) {
      const int i = tid;
      const float xs = sm.eg[i] * sm.nk[i];
      const float bi = sm.bet[i];
#pragma unroll
      for (int cg = 0; cg < 4; ++cg) {
        float x[32];
        const int dv0 = cg * 32;
        tmem_ld32(tl + kColW + dv0, x);
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) {
          float vv[8], rr[8];
          const int ch = (dv0 >> 3) + q8;
          unpack8(*reinterpret_cast<const uint4*>(sm.v[ch >> 3] + sw128(i, (ch & 7) * 8)), vv);
#pragma unroll
          for (int e = 0; e < 8; e += 2) {
            ffma2(rr[e], rr[e + 1], -xs, -xs, x[q8 * 8 + e], x[q8 * 8 + e + 1], vv[e], vv[e + 1]);
            fmul2(rr[e], rr[e + 1], rr[e], rr[e + 1], bi, bi);
          }
          split8(rr, whi + (dv0 >> 6) * 8192, wlo + (dv0 >> 6) * 8192,
                 sw128(i, (dv0 & 63) + q8 * 8));
        }
#pragma unroll
        for (int e = 0; e < 32; ++e) x[e] = 0.f;
        tmem_st32(tl + kColW + dv0, x);
      }
    }
    tmem_wait_st();
    sync_for_mma();
    if (c + 1 < nchunks) load_v(c + 1);   // the v tile is free until the next R phase

    // ---- (4) W-region += [T;M2] [R_hi;R_lo] : rows 0-63 -> v', rows 64-127 -> out
    if (tid == 0) {
#pragma unroll
      for (int s = 0; s < 8; ++s)
        mma_bf16(tbase + kColW, smem_desc(a40 + (s & 3) * 32, 16, 1024),
                 smem_desc((s < 4 ? scr0 : scr0 + kLoOff) + (s & 3) * 2048, 8192, 1024),
                 idesc_bf16(128, 128, false, true), 1u);
      mma_commit(bar);
    }
    if (!(ok = wait_mma())) break;

    // ---- epilogue: W = nk e^(gamma_L-gamma) v' (rows 0-63); out (rows 64-127)
    if (tid < 64) {
      const int i = tid;
      const float w = sm.nk[i] * expf(sm.gam[kC - 1] - sm.gam[i]);
#pragma unroll
      for (int cg = 0; cg < 4; ++cg) {
        float vp[32];
        const int dv0 = cg * 32;
        tmem_ld32(tl + kColW + dv0, vp);
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) {
          float x[8];
#pragma unroll
          for (int e = 0; e < 8; e += 2)
            fmul2(x[e], x[e + 1], w, w, vp[q8 * 8 + e], vp[q8 * 8 + e + 1]);
          split8(x, whi + (dv0 >> 6) * 8192, wlo + (dv0 >> 6) * 8192,
                 sw128(i, (dv0 & 63) + q8 * 8));
        }
      }
    } else {
      const int i = tid - 64;
      bf16* orow = out + ((t0 + i) * HV + h) * kD;
#pragma unroll
      for (int cg = 0; cg < 4; ++cg) {
        float o[32];
        tmem_ld32(tl + kColW + cg * 32, o);
        if (i < nv) {
#pragma unroll
          for (int q8 = 0; q8 < 4; ++q8)
            *reinterpret_cast<uint4*>(orow + cg * 32 + q8 * 8) = pack8(o + q8 * 8);
        }
      }
    }
    sync_for_mma();

    // ---- (5) S += K^T [W_hi;W_lo] : M=128 (dk), N=128, K=64+64; A = K^T (MN-major)
    if (tid == 0) {
#pragma unroll
      for (int s = 0; s < 8; ++s)
        mma_bf16(tbase + kColS, smem_desc(kq0 + (s & 3) * 2048, 16384, 1024),
                 smem_desc((s < 4 ? scr0 : scr0 + kLoOff) + (s & 3) * 2048, 8192, 1024),
                 idesc_bf16(128, 128, true, true), 1u);
      mma_commit(bar);
    }
    if (!(ok = wait_mma())) break;
    if (c + 1 < nchunks) {            // the K rows are free: fetch the next chunk
      load_k(c + 1);
      load_gb(c + 1, g_next, b_next);
    }
  }
  if (!ok && tid == 0) {   // drain loads still in flight before the CTA exits (bounded)
    for (int i = 0; i < 3; ++i) mbar_wait(smem_u32(&sm.lbar[i]), lphase[i], kSpin);
  }

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
  if (warp == 0) tmem_dealloc(tbase, kTmemCols);
}

}  // namespace tc

bool chunk_tc_supported(int D, const void* q, int64_t qs, const void* k, int64_t ks,
                        const void* v, int64_t vs, const void* out, const void* pool,
                        int64_t slot_stride, const void*, int64_t, const void*) {
  return D == tc::kD && aligned16(q) && aligned16(k) && aligned16(v) && aligned16(out) &&
         aligned16(pool) && qs % 8 == 0 && ks % 8 == 0 && vs % 8 == 0 && slot_stride % 4 == 0;
}

// bf16 [rows, cols] view with a row stride (elements), 64 x 64 boxes, 128B swizzle.
static bool make_tile_map(CUtensorMap* m, const void* base, int64_t cols, int64_t rows,
                          int64_t row_stride) {
  EncodeTiledFn fn = encode_tiled();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)row_stride * 2};
  const cuuint32_t box[2] = {64, 64};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

int chunk_prefill_tc(int n_seqs, int HV, cudaStream_t s, const bf16* q, int64_t qs,
                     const bf16* k, int64_t ks, const bf16* v, int64_t vs, const float* g,
                     const bf16* beta, float* pool, int64_t slot_stride, int64_t num_slots,
                     const int64_t* ids, const int32_t* cu, int64_t n_tokens, int max_seqlen,
                     bf16* out, int HK, float scale, const bf16* z, int64_t zs, const bf16* nw,
                     float eps, int32_t* status) {
  CUtensorMap tm_q, tm_k, tm_v;
  if (!make_tile_map(&tm_q, q, (int64_t)HK * tc::kD, n_tokens, qs) ||
      !make_tile_map(&tm_k, k, (int64_t)HK * tc::kD, n_tokens, ks) ||
      !make_tile_map(&tm_v, v, (int64_t)HV * tc::kD, n_tokens, vs)) {
    set_error("gdn_chunk_prefill_varlen: cuTensorMapEncodeTiled failed");
    return GDN_ERR_CUDA;
  }
  const size_t smem = sizeof(tc::ChunkSmem) + 1024;
  cudaError_t e = cudaFuncSetAttribute(tc::chunk_prefill_tc_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) {
    set_error("gdn_chunk_prefill_varlen: cudaFuncSetAttribute failed: %s", cudaGetErrorString(e));
    return GDN_ERR_CUDA;
  }
  tc::chunk_prefill_tc_kernel<<<(unsigned)((int64_t)n_seqs * HV), tc::kThreads, smem, s>>>(
      tm_q, tm_k, tm_v, g, beta, pool, slot_stride, num_slots, ids, cu, n_tokens, max_seqlen,
      out, HK, HV, scale, status);
  int rc = check_launch("gdn_chunk_prefill_varlen");
  // gated RMSNorm in place over the output rows (a full-occupancy kernel; an
  // epilogue inside this kernel would run on half its threads)
  if (rc == GDN_OK && z != nullptr)
    rc = launch_rms_norm_gated(out, z, zs, HV, nw, out, n_tokens * HV, tc::kD, eps, s);
  return rc;
}

}  // namespace gdn
