// (c) Chunked gated-delta-rule prefill on tcgen05 tensor cores (sm_100a).
//
// The one-kernel form, run when the caller passes no workspace (the split form
// in chunk_wy.cu gives the same bits).  One CTA (128 threads, thread t <->
// TMEM lane t; two CTAs per SM) walks one (sequence, v-head) chain chunk by
// chunk (64 tokens), the chains launched longest first.  The fp32 state
// S [dk x dv] lives in TMEM for the whole sequence: read from the pool slot at
// the start, written back at the end.  With q^ = l2norm(q)*scale,
// k^ = l2norm(k), gamma = in-chunk cumsum(g) (qwen3_5.py:152-227), every chunk
// runs five M = 128 MMAs (bf16 operands from 128B-swizzled shared memory, fp32
// accumulators in TMEM):
//
//   1. P   = [K;Q] [K;Q]^T             raw bf16 rows: exact products; its
//                                      diagonal gives the k norms (the q
//                                      norms are summed on the CUDA cores);
//                                      norms and decays applied in fp32
//                                      build
//        L   = -(beta_i nk_i nk_j P_ij e^(gamma_i - gamma_j))   (j < i)
//        QKm =  (nq_i nk_j QK_ij e^(gamma_i - gamma_j))          (j <= i)
//      T = (I - L)^-1 in fp32: diagonal blocks by forward substitution,
//      the doubling products on tf32 mma tiles (chunk_common.cuh)
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
#include "chunk_common.cuh"

namespace gdn {
namespace tc {

constexpr int kThreads = 128;
constexpr uint32_t kSpin = 1u << 22;
constexpr uint32_t kTmemCols = 256;
// TMEM columns: S [0,128) for the whole sequence; a 128-column work region
// [128,256) holds, in turn, P = [K;Q][K;Q]^T, M2, and the XQ / VO accumulator.
constexpr uint32_t kColS = 0, kColW = 128;

// Shared memory (~106 KiB: two CTAs fit on an SM).  `scratch` is reused in
// turn: L then T in place (fp32 [64][68]) plus X (fp32 32 x 40) during the
// inverse; the bf16 S tile for MMA 3; then the R and W hi / lo tiles.
struct __align__(1024) ChunkSmem {
  uint8_t kq[2][128 * 128];   // [dk block][row][128 B]: rows 0-63 K, rows 64-127 Q
  uint8_t scratch[32768];
  uint8_t qkm[64 * 128];      // QKm rows 0-63; MMA 2's rows 64-127 read a4's first rows
  uint8_t a4[128 * 128];      // [T ; M2] : row x 64 tokens
  uint8_t v[2][64 * 128];     // [dv block][token row][128 B] (128B-swizzled, as TMA writes)
  ChunkScalars sc;
  unsigned long long mbar;    // MMA completion
  unsigned long long lbar[3]; // TMA loads: K, Q, V
  uint32_t tmem_base;
  int abort;
  int issued[3];              // TMA loads issued per load barrier (K, Q, V)
  int commits;                // MMA commits on mbar
};

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
  const int r = lpt_sequence<kThreads>(cu, gridDim.x / HV, rank, tid);

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
      ++sm.issued[0];
      mbar_expect_tx(b, 2 * 8192);
      for (int blk = 0; blk < 2; ++blk)
        tma_load_2d(kq_s + blk * 16384, &tm_k, hk * kD + blk * 64, (int)(start + c * kC), b);
    }
  };
  auto load_q = [&](int c) {
    if (tid == 0) {
      const uint32_t b = smem_u32(&sm.lbar[1]);
      ++sm.issued[1];
      mbar_expect_tx(b, 2 * 8192);
      for (int blk = 0; blk < 2; ++blk)
        tma_load_2d(kq_s + blk * 16384 + 64 * 128, &tm_q, hk * kD + blk * 64,
                    (int)(start + c * kC), b);
    }
  };
  auto load_v = [&](int c) {
    if (tid == 0) {
      const uint32_t b = smem_u32(&sm.lbar[2]);
      ++sm.issued[2];
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
    for (int i = 0; i < 3; ++i) {
      mbar_init(smem_u32(&sm.lbar[i]), 1);
      sm.issued[i] = 0;
    }
    mbar_init_fence();
    sm.abort = 0;
    sm.commits = 0;
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

  // One thread waits on each barrier; the others wait at the CTA barrier
  // that follows (no issue slots spent polling).
  auto wait_mma = [&]() -> bool {
    if (tid == 0 && !mbar_wait(bar, phase, kSpin)) {
      sm.abort = 1;
      if (status) atomicOr(status, GDN_STATUS_TIMEOUT);
    }
    phase ^= 1u;
    __syncthreads();
    fence_after();
    return sm.abort == 0;
  };
  auto wait_load = [&](int i) {     // TMA load i (0 K, 1 Q, 2 V); thread 0, a CTA barrier follows
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
    if (tid == 0) {
      wait_load(0);
      wait_load(1);
      wait_load(2);
    }
    if (tid < kC) {
      sm.sc.gam[tid] = g_next;
      sm.sc.bet[tid] = __bfloat162float(__ushort_as_bfloat16(b_next));
    }
    if (nv < kC) {   // clear rows past the sequence end in the K, Q and v tiles
      __syncthreads();
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
    if (warp == 0) decay_scan(sm.sc, lane);   // cumulative decay and its factors
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
      ++sm.commits;
    }
    if (!(ok = wait_mma())) break;
    if (tid < 64) k_norm_from_diag(sm.sc, tl, kColW, tid);
    else q_norm(sm.sc, sm.kq[0], tid, nv, scale);
    __syncthreads();

    // ---- L (rows 0-63) and QKm (rows 64-127) from P; then scale Q rows by e^gamma nq
    build_l_qkm(sm.sc, tl, kColW, tid, Lm, sm.qkm);
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
      ++sm.commits;
    }
    // S (TMEM) -> bf16 MN-major tile (row = dk, col = dv); S *= e^gamma_L in TMEM
    {
      const float egl = sm.sc.eg[kC - 1];
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
      ++sm.commits;
    }
    if (!(ok = wait_mma())) break;
    if (c + 1 < nchunks) load_q(c + 1);   // Q rows are no longer read this chunk

    // ---- R = beta (v - e^gamma nk X) -> hi / lo tiles (rows 0-63); clear those TMEM rows.
    // Meanwhile the threads of rows 64-127 scale QS by e^gamma nq in TMEM (fp32), so
    // MMA 4 adds the intra-chunk term onto the inter-chunk output.
    if (tid >= 64) {
      const int i = tid - 64;
      const float f = sm.sc.eg[i] * sm.sc.nq[i];
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
      const float xs = sm.sc.eg[i] * sm.sc.nk[i];
      const float bi = sm.sc.bet[i];
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
      ++sm.commits;
    }
    if (!(ok = wait_mma())) break;

    // ---- epilogue: W = nk e^(gamma_L-gamma) v' (rows 0-63); out (rows 64-127)
    if (tid < 64) {
      const int i = tid;
      const float w = sm.sc.nk[i] * expf(sm.sc.gam[kC - 1] - sm.sc.gam[i]);
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
      ++sm.commits;
    }
    if (!(ok = wait_mma())) break;
    if (c + 1 < nchunks) {            // the K rows are free: fetch the next chunk
      load_k(c + 1);
      load_gb(c + 1, g_next, b_next);
    }
  }
  if (!ok && tid == 0) {   // drain what is in flight before the CTA exits (bounded):
    // loads and MMAs complete in order, so the parity of the last one issued on
    // each barrier covers all (an already completed phase returns at once)
#pragma unroll
    for (int i = 0; i < 3; ++i)
      if (sm.issued[i] > 0)
        mbar_wait(smem_u32(&sm.lbar[i]), (uint32_t)(sm.issued[i] - 1) & 1u, kSpin);
    if (sm.commits > 0) mbar_wait(bar, (uint32_t)(sm.commits - 1) & 1u, kSpin);
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

int chunk_prefill_tc(int n_seqs, int HV, cudaStream_t s, const bf16* q, int64_t qs,
                     const bf16* k, int64_t ks, const bf16* v, int64_t vs, const float* g,
                     const bf16* beta, float* pool, int64_t slot_stride, int64_t num_slots,
                     const int64_t* ids, const int32_t* cu, int64_t n_tokens, int max_seqlen,
                     bf16* out, int HK, float scale, const bf16* z, int64_t zs, const bf16* nw,
                     float eps, int32_t* status) {
  CUtensorMap tm_q, tm_k, tm_v;
  if (!tc::make_tile_map(&tm_q, q, (int64_t)HK * tc::kD, n_tokens, qs) ||
      !tc::make_tile_map(&tm_k, k, (int64_t)HK * tc::kD, n_tokens, ks) ||
      !tc::make_tile_map(&tm_v, v, (int64_t)HV * tc::kD, n_tokens, vs)) {
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
