// (c) Chunked gated-delta-rule prefill, split form (sm_100a): the
// state-independent work of every chunk runs first, fully parallel, and the
// serial chain per (sequence, v-head) keeps only the state-dependent steps.
//
//   chunk_index_kernel  chunk_start[r] = sum over earlier sequences of
//                       ceil(len / 64) (the workspace's block numbering) and
//                       chunk_info[b] = {first row, valid rows} of block b
//   chunk_prep_kernel   one CTA (two warpgroups, three per SM) per (chunk, pair
//                       of v-heads): P = [K;Q] K^T on the tensor core (once per
//                       k-head), the l2 norms, the decays, L and QKm,
//                       T = (I - L)^-1 (fp32; doubling products on tf32 mma
//                       tiles), M2 = QKm T; writes one 17,664-byte block per
//                       (chunk, head): the [T; M2] tile as the 128B-swizzled
//                       shared-memory image MMA 4 reads, and the per-token
//                       factors the chain applies
//   chunk_chain_kernel  one CTA (256 threads, two per SM) per chain, longest
//                       first; the fp32 state in TMEM; per chunk three M = 128
//                       MMAs (XQ = [K;Q] S, [v'; out] += [T;M2] [R_hi;R_lo],
//                       S += K^T [W_hi;W_lo]) and the CUDA-core phases between
//                       them, split over 8 warps (warp w: TMEM lanes of quarter
//                       w % 4, columns of half w / 4; operand rows interleaved,
//                       ilv_row); the output tile leaves by TMA from the
//                       consumed [T; M2] buffer while MMA 5 runs
//
// The arithmetic is the one-kernel form's (chunk_tc.cu) step for step — same
// operands, same roundings, shared code in chunk_common.cuh — so both give the
// same bits; the split only changes where each step runs.  Blocks move by bulk
// copies (one store per prep head, one load per chain chunk).  Every wait is
// bounded (status bit, TMEM freed, return).
#include "chunk_common.cuh"

namespace gdn {
namespace tc {
namespace wy {

constexpr uint32_t kSpin = 1u << 22;
// The chain's loads are issued by one thread of warp 1 (a Q-row warp, light in
// the R phase); thread 0 issues the MMAs, the output stores and does the waits,
// so a TMA issue (hundreds of cycles for four boxes) never delays an MMA.
constexpr int kLoader = 32;
constexpr uint32_t kTile = 16384;                  // [T; M2]: 128 rows x 128 B
constexpr uint32_t kScal = 5 * kC * 4;             // xs, beta, fq, wk, (e^gamma_L, 0 ...)
constexpr uint32_t kBlockBytes = kTile + kScal;    // 17,664 (a multiple of 128)
constexpr int kPrepThreads = 256;
constexpr int kChainThreads = 256;
constexpr int kIndexThreads = 1024;

// The chain's 128-row MMA operands interleave their two 64-row halves by 32
// rows: tile rows [first 0-31; second 0-31; first 32-63; second 32-63] for
// [K;Q] and [T;M2].  An MMA output row lands in the TMEM lane of its operand
// row, and warp w reaches lanes of quarter w % 4 only, so quarters 0 and 2 hold
// the K / T rows (R and W phases) and quarters 1 and 3 the Q / M2 rows (QS
// scaling, output).
__host__ __device__ constexpr int ilv_row(int token, bool second) {
  return token + (token & 32) + (second ? 32 : 0);
}

// ---------------------------------------------------------------- index
// chunk_start[r] = first block of sequence r; chunk_info[b] = {first token row,
// valid rows} of block b (valid rows 0 for the unused tail up to the capacity).
// Sequences that are malformed (negative start or length, past n_tokens) get
// no chunks (the chain kernel flags them); a sequence whose chunks would pass
// the workspace's capacity (only overlapping, malformed cu_seqlens) is cut
// short here and flagged by the chain kernel when its count does not match.
__global__ void __launch_bounds__(kIndexThreads) chunk_index_kernel(
    const int32_t* __restrict__ cu, int n_seqs, int64_t n_tokens, int max_seqlen, int64_t cap,
    int32_t* __restrict__ chunk_start, int2* __restrict__ chunk_info) {
  __shared__ long long wsum[32];
  __shared__ long long carry;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) carry = 0;
  __syncthreads();
  for (int base = 0; base < n_seqs; base += kIndexThreads) {
    const int i = base + tid;
    long long n = 0, s = 0, l = 0;
    if (i < n_seqs) {
      s = cu[i];
      l = (long long)cu[i + 1] - s;
      if (s >= 0 && l > 0 && s + l <= n_tokens) {
        l = min(l, (long long)max_seqlen);
        n = (l + kC - 1) / kC;
      }
    }
    long long x = n;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) wsum[warp] = x;
    __syncthreads();
    if (warp == 0) {
      long long w = wsum[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const long long y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      wsum[lane] = w;
    }
    __syncthreads();
    const long long excl = carry + (warp > 0 ? wsum[warp - 1] : 0) + x - n;
    if (i < n_seqs) {
      chunk_start[i] = (int32_t)min(excl, (long long)cap);
      for (long long c = 0; c < n && excl + c < cap; ++c)
        chunk_info[excl + c] = make_int2((int)(s + c * kC), (int)min((long long)kC, l - c * kC));
    }
    __syncthreads();
    if (tid == 0) carry += wsum[31];
    __syncthreads();
  }
  const long long total = min(carry, (long long)cap);
  if (tid == 0) chunk_start[n_seqs] = (int32_t)total;
  for (long long b = total + tid; b < cap; b += kIndexThreads) chunk_info[b] = make_int2(0, 0);
}

// ---------------------------------------------------------------- prep
// One CTA (256 threads = two warpgroups) per (chunk, pair of v-heads 2p, 2p + 1);
// warpgroup w handles v-head 2p + w.  When the two heads share a k-head (GQA),
// the [K;Q] tile, P = [K;Q] K^T and the l2 norms are made once for both; else
// each warpgroup loads its own tile.  Each warpgroup's 32 KiB region serves in
// turn as its [K;Q] tile (rows interleaved by 16, ilv16_row), as L / T (fp32),
// the QKm tile and X (the inverse), and as its [T; M2] block image (MMA 2 and
// the store) — about 71 KiB and 128 TMEM columns per CTA (256 when the two
// heads have their own k-heads): three CTAs (six heads) per SM.
struct PrepSmem {             // placed at a 1024-byte aligned base (swizzle atoms)
  uint8_t r[2][32768];
  float f[2][5][kC];          // the blocks' factors
  ChunkScalars sc[2];
  unsigned long long mbar, lbar;
  uint32_t tmem_base;
  int abort;
  int commits;                // MMA commits on mbar
};
constexpr uint32_t kQkmOff = 18432;   // QKm tile (1024-aligned) after L / T (17,408 B)
constexpr uint32_t kXOff = 26624;     // X (5 KiB) after QKm; MMA 2's unused A rows 64-127
                                      // read [26624, 34816) of the region: don't-care data
constexpr int kPrepCtasPerSm = 3;

__global__ void __launch_bounds__(kPrepThreads, kPrepCtasPerSm) chunk_prep_kernel(
    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
    const float* __restrict__ g, const bf16* __restrict__ beta,
    const int2* __restrict__ chunk_info, int HK, int HV, float scale,
    uint8_t* __restrict__ blocks, int32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  PrepSmem& sm = *reinterpret_cast<PrepSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int wg = tid >> 7, lt = tid & 127;           // warpgroup, thread within it
  const int n_pairs = (HV + 1) >> 1;
  const int b = blockIdx.x / n_pairs;
  const int pair = blockIdx.x - b * n_pairs;
  const int R = HV / HK;
  const int h0 = 2 * pair, h1 = h0 + 1;
  const bool has1 = h1 < HV;
  const int hk0 = h0 / R, hk1 = has1 ? h1 / R : hk0;
  const bool own1 = has1 && hk1 != hk0;             // head 1 needs its own [K;Q] tile
  const int h = wg ? (has1 ? h1 : h0) : h0;         // this warpgroup's head
  const int2 info = chunk_info[b];
  const int64_t t0 = info.x;
  const int nv = info.y;
  if (nv <= 0) return;                               // past the last chunk

  uint8_t* const rw = sm.r[wg];                      // this warpgroup's region
  const uint32_t r0s = smem_u32(sm.r[0]), r1s = smem_u32(sm.r[1]);
  const uint32_t bar = smem_u32(&sm.mbar), lbar = smem_u32(&sm.lbar);
  if (tid == 0) {
    mbar_init(bar, 1);
    mbar_init(lbar, 1);
    mbar_init_fence();
    sm.abort = 0;
    sm.commits = 0;
    mbar_expect_tx(lbar, (own1 ? 2 : 1) * 4 * 8192);   // the boxes are issued after the barrier
  }
  if (lt < kC) {
    float gv = 0.f, bv = 0.f;
    if (lt < nv) {
      gv = __ldg(g + (t0 + lt) * HV + h);
      bv = __bfloat162float(beta[(t0 + lt) * HV + h]);
    }
    sm.sc[wg].gam[lt] = gv;
    sm.sc[wg].bet[lt] = bv;
  }
  const uint32_t tcols = own1 ? 256u : 128u;          // P (128 columns) per k-head
  if (warp == 0) tmem_alloc(smem_u32(&sm.tmem_base), tcols);
  fence_before();
  __syncthreads();
  fence_after();
  if (lane == 0) {   // 16-row boxes at their interleaved tile rows: warp w -> (dk block, block)
    const int blk = warp & 1, b16 = warp >> 1;
    for (int t = 0; t < (own1 ? 2 : 1); ++t) {
      const uint32_t rs = (t ? r1s : r0s) + blk * 16384;
      const int hk = t ? hk1 : hk0;
      tma_load_2d(rs + ilv16_row(16 * b16, false) * 128, &tm_k, hk * kD + blk * 64,
                  (int)(t0 + 16 * b16), lbar);
      tma_load_2d(rs + ilv16_row(16 * b16, true) * 128, &tm_q, hk * kD + blk * 64,
                  (int)(t0 + 16 * b16), lbar);
    }
  }
  const uint32_t tbase = sm.tmem_base;
  const uint32_t tl = tbase + ((uint32_t)((warp & 3) * 32) << 16);   // lane quarter warp % 4
  const uint32_t colP = own1 ? 128u * wg : 0u;       // this head's P columns
  // one thread waits on each barrier; the others wait at the CTA barrier
  auto wait1 = [&](uint32_t mb, uint32_t ph) -> bool {
    if (tid == 0 && !mbar_wait(mb, ph, kSpin)) {
      sm.abort = 1;
      if (status) atomicOr(status, GDN_STATUS_TIMEOUT);
    }
    __syncthreads();
    fence_after();
    return sm.abort == 0;
  };
  bool ok = wait1(lbar, 0);
  if (ok) {
    if (nv < kC) {   // rows past the sequence end: zero K and Q
      const int nt = own1 ? 2 : 1;
      for (int idx = tid; idx < nt * (kC - nv) * 16; idx += kPrepThreads) {
        const int t = idx / ((kC - nv) * 16), rem = idx - t * (kC - nv) * 16;
        const int i = nv + rem / 16, ch = rem % 16, blk = ch >> 3, c8 = (ch & 7) * 8;
        const uint4 z = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(sm.r[t] + blk * 16384 + sw128(ilv16_row(i, false), c8)) = z;
        *reinterpret_cast<uint4*>(sm.r[t] + blk * 16384 + sw128(ilv16_row(i, true), c8)) = z;
      }
    }
    if ((warp & 3) == 0) decay_scan(sm.sc[wg], lane);   // warps 0 and 4: one head each
    fence_async_smem();
    fence_before();
    __syncthreads();
    fence_after();
    // (1) P = [K;Q] [K;Q]^T (interleaved rows) : M = N = K = 128; once per k-head
    if (tid == 0) {
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        if (t == 1 && !own1) break;
        const uint32_t rs = t ? r1s : r0s;
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          const uint32_t off = (uint32_t)(s >> 2) * 16384u + (uint32_t)(s & 3) * 32u;
          mma_bf16(tbase + 128u * t, smem_desc(rs + off, 16, 1024), smem_desc(rs + off, 16, 1024),
                   idesc_bf16(128, 128, false, false), s > 0);
        }
      }
      mma_commit(bar);
      ++sm.commits;
    }
    if (lt >= 64 && (wg == 0 || own1))          // Q rows: CUDA cores, under MMA 1
      q_norm_row(sm.sc[wg], rw, lt - 64, ilv16_row(lt - 64, true), nv, scale);
    ok = wait1(bar, 0);
  }
  if (ok) {
    if (wg == 0 || own1) k_norm_ilv16(sm.sc[wg], tl, colP, lt);   // P's diagonal (K rows)
    __syncthreads();
    if (wg == 1 && !own1) {                      // head 1 shares head 0's norms
      if (lt < 64) {
        sm.sc[1].nk[lt] = sm.sc[0].nk[lt];
        sm.sc[1].cf[lt] = sm.sc[0].nk[lt] * sm.sc[1].bcol[lt];
      } else {
        sm.sc[1].nq[lt - 64] = sm.sc[0].nq[lt - 64];
      }
    }
    __syncthreads();
    float (*Lm)[kLP] = reinterpret_cast<float (*)[kLP]>(rw);     // K / Q are consumed
    float* Xs = reinterpret_cast<float*>(rw + kXOff);
    build_l_qkm_ilv16(sm.sc[wg], tl, colP, lt, Lm, rw + kQkmOff);
    __syncthreads();
    invert_unit_lower(Lm, Xs, lt);               // both warpgroups pass its barriers together
    {   // T (fp32, rows of 68) -> the bf16 T rows of the block image, over L / T
      float t[4][8];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int idx = lt + k * 128, i = idx >> 3, c8 = (idx & 7) * 8;
        const float4 a = *reinterpret_cast<const float4*>(&Lm[i][c8]);
        const float4 bb = *reinterpret_cast<const float4*>(&Lm[i][c8 + 4]);
        t[k][0] = a.x; t[k][1] = a.y; t[k][2] = a.z; t[k][3] = a.w;
        t[k][4] = bb.x; t[k][5] = bb.y; t[k][6] = bb.z; t[k][7] = bb.w;
      }
      __syncthreads();
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int idx = lt + k * 128, i = idx >> 3, c8 = (idx & 7) * 8;
        st8(rw, ilv_row(i, false), c8, t[k]);
      }
    }
    fence_async_smem();
    fence_before();
    __syncthreads();
    fence_after();
    // (2) M2 = [QKm; *] T per head : M = 128 (rows 64-127 unused), N = 64, K = 64
    if (tid == 0) {
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const uint32_t rs = t ? r1s : r0s;
#pragma unroll
        for (int s = 0; s < 4; ++s)
          mma_bf16(tbase + 64u * t, smem_desc(rs + kQkmOff + s * 32, 16, 1024),
                   smem_desc(rs + ilv_row(16 * s, false) * 128, 8192, 1024),
                   idesc_bf16(128, 64, false, true), s > 0);
      }
      mma_commit(bar);
      ++sm.commits;
    }
    ok = wait1(bar, 1);
    if (ok) {
      if (lt < 64) {   // M2 rows -> the image rows of the second half; the factors
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          float m[32];
          tmem_ld32(tl + 64u * wg + hh * 32, m);
#pragma unroll
          for (int q8 = 0; q8 < 4; ++q8)
            st8(rw, ilv_row(lt, true), hh * 32 + q8 * 8, m + q8 * 8);
        }
        const ChunkScalars& s = sm.sc[wg];
        float (&f)[5][kC] = sm.f[wg];
        f[0][lt] = s.eg[lt] * s.nk[lt];                             // R: e^gamma nk
        f[1][lt] = s.bet[lt];                                       // R: beta
        f[2][lt] = s.eg[lt] * s.nq[lt];                             // QS: e^gamma nq
        f[3][lt] = s.nk[lt] * expf(s.gam[kC - 1] - s.gam[lt]);      // W: nk e^(gL - g)
        f[4][lt] = lt == 0 ? s.eg[kC - 1] : 0.f;                    // S: e^gamma_L
      }
      fence_async_smem();
      __syncthreads();
      if (tid == 0) {
        for (int t = 0; t < (has1 ? 2 : 1); ++t) {
          uint8_t* dst = blocks + ((int64_t)b * HV + h0 + t) * kBlockBytes;
          bulk_store(dst, t ? r1s : r0s, kTile);
          bulk_store(dst + kTile, smem_u32(&sm.f[t][0][0]), kScal);
        }
        bulk_wait_read();
      }
    }
  }
  if (sm.abort && tid == 0) {   // drain what is in flight before TMEM is freed (bounded)
    mbar_wait(lbar, 0, kSpin);    // the one [K;Q] load batch
    if (sm.commits > 0) mbar_wait(bar, (uint32_t)(sm.commits - 1) & 1u, kSpin);
  }
  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 0) tmem_dealloc(tbase, tcols);
}

// ---------------------------------------------------------------- chain
// One CTA per (sequence, v-head, column part): NCOL of the state's 128 value
// columns (128: the whole state; 64: half of it, for launches with too few
// chains to fill the GPU — a long-context prefill of a few sequences).  The
// delta rule's value columns evolve independently given the chunk's K, Q, T
// and M2, so the parts of a chain need no exchange; each loads the shared K /
// Q / [T; M2] tiles itself.  8 warps: warp w owns TMEM lane quarter w % 4 and
// CPT = NCOL / 2 columns of the part (group w / 4).
// CG groups of 32 TMEM columns (starting at `ta`) behind one wait.
template <int CG>
__device__ __forceinline__ void tmem_ld_groups(uint32_t ta, float (&v)[CG][32]) {
  if constexpr (CG == 2) {
    tmem_ld32x2(ta, ta + 32, v[0], v[1]);
  } else {
    tmem_ld32(ta, v[0]);
  }
}

template <int NCOL>
struct __align__(1024) ChainSmem {
  static constexpr int NB = NCOL / 64;   // 64-column blocks of the part
  uint8_t kq[2][128 * 128];   // [dk block][row][128 B]: K / Q rows interleaved (ilv_row)
  uint8_t scratch[NB * 16384];// the bf16 S tile for MMA 3, then R, then W (hi / lo)
  uint8_t a4[128 * 128];      // [T ; M2] from the chunk's block, then the out tile
  uint8_t v[NB][64 * 128];    // [dv block][token row][128 B]
  float f[2][5][kC];          // the blocks' per-token factors, chunks c and c + 1
  unsigned long long mbar;    // MMA completion
  unsigned long long lbar[5]; // loads: K, Q, V, [T;M2] tile, factors
  uint32_t tmem_base;
  int abort;
  int issued[5];              // loads issued per load barrier
  int commits;                // MMA commits on mbar
};

template <int NCOL>
__global__ void __launch_bounds__(kChainThreads, 2) chunk_chain_kernel(
    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_out,
    const uint8_t* __restrict__ blocks,
    const int32_t* __restrict__ chunk_start, float* __restrict__ pool, int64_t slot_stride,
    int64_t num_slots, const int64_t* __restrict__ ids, const int32_t* __restrict__ cu,
    int64_t n_tokens, int max_seqlen, bf16* __restrict__ out, int HK, int HV, int32_t* status) {
  constexpr int PARTS = kD / NCOL;        // column parts per chain
  constexpr int NB = NCOL / 64;           // 64-column blocks per part
  constexpr int CPT = NCOL / 2;           // columns per thread
  constexpr int CG = CPT / 32;            // 32-column TMEM loads per thread
  static_assert(NCOL == 128 || NCOL == 64, "column parts of 128 or 64");
  using Smem = ChainSmem<NCOL>;
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qd = warp & 3, half = warp >> 2;
  const int row = qd * 32 + lane;        // TMEM lane: dk row of S, or row of a 128-row tile
  const bool second = qd & 1;            // interleaved tile row of the second half (Q / M2)
  const int rank = blockIdx.x / (HV * PARTS);
  const int hp = blockIdx.x - rank * (HV * PARTS);
  const int h = hp / PARTS;
  const int cb = (hp - h * PARTS) * NCOL;   // the part's first value column
  const int hk = h / (HV / HK);
  const int n_seqs = gridDim.x / (HV * PARTS);
  const int r = lpt_sequence<kChainThreads>(cu, n_seqs, rank, tid);

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
  const int cs = chunk_start[r];
  if (chunk_start[r + 1] - cs != nchunks) {   // cut short by the index (overlapping cu)
    if (tid == 0 && status) atomicOr(status, GDN_STATUS_BAD_SEQLEN);
    return;
  }

  const uint32_t kq0 = smem_u32(sm.kq[0]);
  // K / Q rows in 32-row boxes at their interleaved tile rows
  auto load_k = [&](int c) {
    const uint32_t b = smem_u32(&sm.lbar[0]);
    ++sm.issued[0];
    mbar_expect_tx(b, 2 * 8192);
    for (int blk = 0; blk < 2; ++blk)
      for (int hf = 0; hf < 2; ++hf)
        tma_load_2d(kq0 + blk * 16384 + ilv_row(32 * hf, false) * 128, &tm_k, hk * kD + blk * 64,
                    (int)(start + c * kC + 32 * hf), b);
  };
  auto load_q = [&](int c) {
    const uint32_t b = smem_u32(&sm.lbar[1]);
    ++sm.issued[1];
    mbar_expect_tx(b, 2 * 8192);
    for (int blk = 0; blk < 2; ++blk)
      for (int hf = 0; hf < 2; ++hf)
        tma_load_2d(kq0 + blk * 16384 + ilv_row(32 * hf, true) * 128, &tm_q, hk * kD + blk * 64,
                    (int)(start + c * kC + 32 * hf), b);
  };
  auto load_v = [&](int c) {        // the part's value columns
    const uint32_t b = smem_u32(&sm.lbar[2]);
    ++sm.issued[2];
    mbar_expect_tx(b, NB * 8192);
    for (int blk = 0; blk < NB; ++blk)
      tma_load_2d(smem_u32(sm.v[blk]), &tm_v, h * kD + cb + blk * 64, (int)(start + c * kC), b);
  };
  auto load_tile = [&](int c) {     // the [T; M2] tile of chunk c's block
    const uint32_t b = smem_u32(&sm.lbar[3]);
    ++sm.issued[3];
    mbar_expect_tx(b, kTile);
    bulk_load(smem_u32(sm.a4), blocks + ((int64_t)(cs + c) * HV + h) * kBlockBytes, kTile, b);
  };
  auto load_f = [&](int c) {        // the factors of chunk c's block, into buffer c % 2
    const uint32_t b = smem_u32(&sm.lbar[4]);
    ++sm.issued[4];
    mbar_expect_tx(b, kScal);
    bulk_load(smem_u32(&sm.f[c & 1][0][0]),
              blocks + ((int64_t)(cs + c) * HV + h) * kBlockBytes + kTile, kScal, b);
  };

  const uint32_t bar = smem_u32(&sm.mbar);
  if (tid == 0) {
    mbar_init(bar, 1);
    for (int i = 0; i < 5; ++i) {
      mbar_init(smem_u32(&sm.lbar[i]), 1);
      sm.issued[i] = 0;
    }
    mbar_init_fence();
    sm.abort = 0;
    sm.commits = 0;
  }
  __syncthreads();
  if (tid == 0) {
    load_f(0);
    load_k(0);
    load_q(0);
    load_tile(0);
    load_v(0);
  }
  uint32_t lphase[5] = {0u, 0u, 0u, 0u, 0u};
  constexpr uint32_t kTmemCols = 2 * NCOL;
  if (warp == 0) tmem_alloc(smem_u32(&sm.tmem_base), kTmemCols);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tbase = sm.tmem_base;
  const uint32_t tl = tbase + ((uint32_t)(qd * 32) << 16);   // this warp's lane window
  constexpr uint32_t kColS = 0, kColW = NCOL;
  const uint32_t c0 = (uint32_t)half * CPT;                 // this warp's columns in the part
  const uint32_t blk0 = c0 >> 6, cin = c0 & 63;              // their 64-column block, offset
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
  auto wait_load = [&](int i) {     // thread 0 only; a CTA barrier must follow
    if (!mbar_wait(smem_u32(&sm.lbar[i]), lphase[i], kSpin)) {
      sm.abort = 1;
      if (status) atomicOr(status, GDN_STATUS_TIMEOUT);
    }
    lphase[i] ^= 1u;
  };
  auto sync_for_mma = [&]() {
    fence_async_smem();
    fence_before();
    __syncthreads();
    fence_after();
  };

  // initial state -> TMEM (thread: dk row `row`, value columns cb + c0 + [0, CPT))
  float* sp = pool + slot * slot_stride + (int64_t)h * kD * kD + (int64_t)row * kD + cb + c0;
#pragma unroll
  for (int cg = 0; cg < CG; ++cg) {
    float s[32];
    const float4* src = reinterpret_cast<const float4*>(sp + cg * 32);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 x = src[i];
      s[4 * i] = x.x; s[4 * i + 1] = x.y; s[4 * i + 2] = x.z; s[4 * i + 3] = x.w;
    }
    tmem_st32(tl + kColS + c0 + cg * 32, s);
  }
  tmem_wait_st();

  const uint32_t scr0 = smem_u32(sm.scratch);
  const uint32_t a40 = smem_u32(sm.a4);
  constexpr uint32_t kLoOff = NB * 8192;             // R / W lo tiles after the hi tiles
  uint8_t* whi = sm.scratch + blk0 * 8192;           // this warp's dv block of R / W
  uint8_t* wlo = whi + kLoOff;
  constexpr uint32_t kIdesc = idesc_bf16(128, NCOL, false, true);
  bool ok = true;

  for (int c = 0; c < nchunks && ok; ++c) {
    const int64_t t0 = start + (int64_t)c * kC;
    const int nv = (int)min((int64_t)kC, len - (int64_t)c * kC);
    const bool full = nv == kC;
    if (tid == 0) wait_load(4);                    // the factors of chunk c
    __syncthreads();
    if (sm.abort) { ok = false; break; }
    const int i = (qd >> 1) * 32 + lane;            // token of this thread's tile row
    const float (&fc)[5][kC] = sm.f[c & 1];
    const float f0 = fc[second ? 2 : 0][i];         // e^gamma nk (R rows) | e^gamma nq (QS rows)
    const float bi = fc[1][i];
    const float wk = fc[3][i];
    const float egl = fc[4][0];
    // the other buffer was last read in chunk c - 1 (barriers since): prefetch c + 1
    if (tid == kLoader && c + 1 < nchunks) {
      load_f(c + 1);
      // the next K into L2: its tile load has to wait for MMA 5
      for (int blk = 0; blk < 2; ++blk)
        for (int hf = 0; hf < 2; ++hf)
          tma_prefetch_2d(&tm_k, hk * kD + blk * 64, (int)(start + (c + 1) * kC + 32 * hf));
    }

    // S (state after the previous chunk) -> bf16 MN-major tile (row = dk,
    // col = dv) for MMA 3; then S *= e^gamma_L in TMEM for MMA 5
    {
      float s[CG][32];
      tmem_ld_groups<CG>(tl + kColS + c0, s);
#pragma unroll
      for (int cg = 0; cg < CG; ++cg) {
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8)
          st8(sm.scratch + blk0 * 16384, row, cin + cg * 32 + q8 * 8, s[cg] + q8 * 8);
#pragma unroll
        for (int e = 0; e < 32; e += 2)
          fmul2(s[cg][e], s[cg][e + 1], s[cg][e], s[cg][e + 1], egl, egl);
        tmem_st32(tl + kColS + c0 + cg * 32, s[cg]);
      }
    }
    tmem_wait_st();
    if (tid == 0) {
      wait_load(0);
      wait_load(1);
    }
    if (nv < kC) {   // clear rows past the sequence end in the K and Q tiles
      __syncthreads();
      for (int idx = tid; idx < (kC - nv) * 16; idx += kChainThreads) {
        const int ii = nv + idx / 16, ch = idx % 16, blk = ch >> 3, c8 = (ch & 7) * 8;
        const uint4 z = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(sm.kq[blk] + sw128(ilv_row(ii, false), c8)) = z;
        *reinterpret_cast<uint4*>(sm.kq[blk] + sw128(ilv_row(ii, true), c8)) = z;
      }
    }
    sync_for_mma();
    if (sm.abort) { ok = false; break; }

    // ---- (3) XQ = [K; Q] S : M=128, N=NCOL, K=128 (dk); B = S rows (MN-major)
    if (tid == 0) {
#pragma unroll
      for (int s = 0; s < 8; ++s)
        mma_bf16(tbase + kColW,
                 smem_desc(kq0 + (uint32_t)(s >> 2) * 16384u + (uint32_t)(s & 3) * 32u, 16, 1024),
                 smem_desc(scr0 + s * 2048, 16384, 1024), kIdesc, s > 0);
      mma_commit(bar);
      ++sm.commits;
    }
    if (tid == 0) {
      if (c > 0) {                 // the previous chunk's out tile has left a4: fetch [T; M2]
        bulk_wait_read();
        load_tile(c);
      }
      wait_load(2);                                    // V, before the barrier in wait_mma
    }
    if (!(ok = wait_mma())) break;
    if (tid == kLoader && c + 1 < nchunks) load_q(c + 1);   // Q rows are no longer read

    // ---- R = beta (v - e^gamma nk X) -> hi / lo tiles (K rows), those TMEM rows cleared;
    // Q rows: QS *= e^gamma nq in TMEM (fp32)
    {
      float xx[CG][32];
      tmem_ld_groups<CG>(tl + kColW + c0, xx);
#pragma unroll
      for (int cg = 0; cg < CG; ++cg) {
        float (&x)[32] = xx[cg];
        if (second) {
#pragma unroll
          for (int e = 0; e < 32; e += 2) fmul2(x[e], x[e + 1], x[e], x[e + 1], f0, f0);
        } else {
#pragma unroll
          for (int q8 = 0; q8 < 4; ++q8) {
            float vv[8], rr[8];
            const uint32_t col = cin + cg * 32 + q8 * 8;   // column within the dv block
            unpack8(i < nv ? *reinterpret_cast<const uint4*>(sm.v[blk0] + sw128(i, col))
                           : make_uint4(0, 0, 0, 0), vv);
#pragma unroll
            for (int e = 0; e < 8; e += 2) {
              ffma2(rr[e], rr[e + 1], -f0, -f0, x[q8 * 8 + e], x[q8 * 8 + e + 1], vv[e],
                    vv[e + 1]);
              fmul2(rr[e], rr[e + 1], rr[e], rr[e + 1], bi, bi);
            }
            split8(rr, whi, wlo, sw128(i, col));
          }
#pragma unroll
          for (int e = 0; e < 32; ++e) x[e] = 0.f;
        }
        tmem_st32(tl + kColW + c0 + cg * 32, x);
      }
    }
    tmem_wait_st();
    if (tid == 0) wait_load(3);                        // the [T; M2] tile of chunk c
    sync_for_mma();
    if (sm.abort) { ok = false; break; }
    if (tid == kLoader && c + 1 < nchunks) load_v(c + 1);   // the v tile is consumed

    // ---- (4) W-region += [T;M2] [R_hi;R_lo] : T rows -> v', M2 rows -> out
    if (tid == 0) {
#pragma unroll
      for (int s = 0; s < 8; ++s)
        mma_bf16(tbase + kColW, smem_desc(a40 + (s & 3) * 32, 16, 1024),
                 smem_desc((s < 4 ? scr0 : scr0 + kLoOff) + (s & 3) * 2048, 8192, 1024), kIdesc,
                 1u);
      mma_commit(bar);
      ++sm.commits;
    }
    if (!(ok = wait_mma())) break;

    // ---- epilogue: W = nk e^(gamma_L-gamma) v' (T rows); out (M2 rows) -> bf16
    // tile in the (consumed) a4 buffer, stored by TMA while MMA 5 runs
    {
      float vv[CG][32];
      tmem_ld_groups<CG>(tl + kColW + c0, vv);
      if (!second) {
#pragma unroll
        for (int cg = 0; cg < CG; ++cg) {
#pragma unroll
          for (int q8 = 0; q8 < 4; ++q8) {
            float x[8];
#pragma unroll
            for (int e = 0; e < 8; e += 2)
              fmul2(x[e], x[e + 1], wk, wk, vv[cg][q8 * 8 + e], vv[cg][q8 * 8 + e + 1]);
            split8(x, whi, wlo, sw128(i, cin + cg * 32 + q8 * 8));
          }
        }
      } else if (full || i < nv) {
#pragma unroll
        for (int cg = 0; cg < CG; ++cg)
#pragma unroll
          for (int q8 = 0; q8 < 4; ++q8) {
            if (full) {
              st8(sm.a4 + blk0 * 8192, i, cin + cg * 32 + q8 * 8, vv[cg] + q8 * 8);
            } else {   // a partial last chunk: rows past the end belong to the next sequence
              *reinterpret_cast<uint4*>(out + ((t0 + i) * HV + h) * kD + cb + c0 + cg * 32 +
                                        q8 * 8) = pack8(vv[cg] + q8 * 8);
            }
          }
      }
    }
    sync_for_mma();

    // ---- (5) S += K^T [W_hi;W_lo] : M=128 (dk), N=NCOL, K=64+64; A = K^T (MN-major)
    if (tid == 0) {
#pragma unroll
      for (int s = 0; s < 8; ++s)
        mma_bf16(tbase + kColS, smem_desc(kq0 + ilv_row(16 * (s & 3), false) * 128, 16384, 1024),
                 smem_desc((s < 4 ? scr0 : scr0 + kLoOff) + (s & 3) * 2048, 8192, 1024),
                 idesc_bf16(128, NCOL, true, true), 1u);
      mma_commit(bar);
      ++sm.commits;
      if (full) {
        for (int blk = 0; blk < NB; ++blk)
          tma_store_2d(&tm_out, h * kD + cb + blk * 64, (int)t0, a40 + blk * 8192);
        bulk_commit();
      }
    }
    if (!(ok = wait_mma())) break;
    if (tid == kLoader && c + 1 < nchunks) load_k(c + 1);   // the K rows are free
  }
  if (!ok && tid == 0) {   // drain what is in flight before the CTA exits (bounded):
    // loads and MMAs complete in order, so the parity of the last one issued on
    // each barrier covers all (an already completed phase returns at once)
#pragma unroll
    for (int i = 0; i < 5; ++i)
      if (sm.issued[i] > 0)
        mbar_wait(smem_u32(&sm.lbar[i]), (uint32_t)(sm.issued[i] - 1) & 1u, kSpin);
    if (sm.commits > 0) mbar_wait(bar, (uint32_t)(sm.commits - 1) & 1u, kSpin);
  }
  if (tid == 0) bulk_wait_all();   // out tiles written before the CTA leaves
  if (ok) {   // final state -> pool slot
#pragma unroll
    for (int cg = 0; cg < CG; ++cg) {
      float s[32];
      tmem_ld32(tl + kColS + c0 + cg * 32, s);
      float4* dst = reinterpret_cast<float4*>(sp + cg * 32);
#pragma unroll
      for (int q = 0; q < 8; ++q)
        dst[q] = make_float4(s[4 * q], s[4 * q + 1], s[4 * q + 2], s[4 * q + 3]);
    }
  }
  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 0) tmem_dealloc(tbase, kTmemCols);
}

}  // namespace wy
}  // namespace tc

int64_t chunk_wy_capacity(int64_t n_tokens, int64_t n_seqs) {
  return (n_tokens + (tc::kC - 1) * n_seqs) / tc::kC;
}

// Workspace: chunk_start (int32 x n_seqs + 1) | chunk_info (int2 x capacity) |
// blocks (capacity x HV x 17,664 B), each part 256-byte aligned.
static int64_t align256(int64_t x) { return (x + 255) / 256 * 256; }

int64_t chunk_wy_workspace_bytes(int64_t n_tokens, int64_t n_seqs, int64_t HV) {
  const int64_t cap = chunk_wy_capacity(n_tokens, n_seqs);
  return align256((n_seqs + 1) * 4) + align256(cap * 8) + cap * HV * tc::wy::kBlockBytes;
}

int chunk_prefill_wy(int n_seqs, int HV, cudaStream_t s, const bf16* q, int64_t qs,
                     const bf16* k, int64_t ks, const bf16* v, int64_t vs, const float* g,
                     const bf16* beta, float* pool, int64_t slot_stride, int64_t num_slots,
                     const int64_t* ids, const int32_t* cu, int64_t n_tokens, int max_seqlen,
                     bf16* out, int HK, float scale, void* workspace, int32_t* status) {
  using namespace tc;
  CUtensorMap tm_q, tm_k, tm_v, tm_q32, tm_k32, tm_out;   // tm_q / tm_k: 16-row boxes (prep)
  if (!make_tile_map(&tm_q, q, (int64_t)HK * kD, n_tokens, qs, 16) ||
      !make_tile_map(&tm_k, k, (int64_t)HK * kD, n_tokens, ks, 16) ||
      !make_tile_map(&tm_q32, q, (int64_t)HK * kD, n_tokens, qs, 32) ||
      !make_tile_map(&tm_k32, k, (int64_t)HK * kD, n_tokens, ks, 32) ||
      !make_tile_map(&tm_v, v, (int64_t)HV * kD, n_tokens, vs) ||
      !make_tile_map(&tm_out, out, (int64_t)HV * kD, n_tokens, (int64_t)HV * kD)) {
    set_error("gdn_chunk_prefill_varlen: cuTensorMapEncodeTiled failed");
    return GDN_ERR_CUDA;
  }
  const int64_t cap = chunk_wy_capacity(n_tokens, n_seqs);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int32_t* chunk_start = reinterpret_cast<int32_t*>(ws);
  int2* chunk_info = reinterpret_cast<int2*>(ws + align256((n_seqs + 1) * 4));
  uint8_t* blocks = ws + align256((n_seqs + 1) * 4) + align256(cap * 8);
  const size_t prep_smem = sizeof(wy::PrepSmem) + 1024;
  // Column parts: with fewer chains than two per SM (a long-context prefill
  // of a few sequences) each chain's state is split into two 64-column parts,
  // which halves the per-chunk work on the serial path of each CTA.
  const int64_t chains = (int64_t)n_seqs * HV;
  const bool split_cols = chains < 2 * (int64_t)sm_count();
  const size_t chain_smem =
      (split_cols ? sizeof(wy::ChainSmem<64>) : sizeof(wy::ChainSmem<128>)) + 1024;
  cudaError_t e = cudaFuncSetAttribute(wy::chunk_prep_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)prep_smem);
  if (e == cudaSuccess)
    e = split_cols ? cudaFuncSetAttribute(wy::chunk_chain_kernel<64>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)chain_smem)
                   : cudaFuncSetAttribute(wy::chunk_chain_kernel<128>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)chain_smem);
  if (e != cudaSuccess) {
    set_error("gdn_chunk_prefill_varlen: cudaFuncSetAttribute failed: %s", cudaGetErrorString(e));
    return GDN_ERR_CUDA;
  }
  wy::chunk_index_kernel<<<1, wy::kIndexThreads, 0, s>>>(cu, n_seqs, n_tokens, max_seqlen, cap,
                                                         chunk_start, chunk_info);
  int rc = check_launch("gdn_chunk_prefill_varlen");
  if (rc != GDN_OK || cap == 0) return rc;
  wy::chunk_prep_kernel<<<(unsigned)(cap * ((HV + 1) / 2)), wy::kPrepThreads, prep_smem, s>>>(
      tm_q, tm_k, g, beta, chunk_info, HK, HV, scale, blocks, status);
  if ((rc = check_launch("gdn_chunk_prefill_varlen")) != GDN_OK) return rc;
  if (split_cols)
    wy::chunk_chain_kernel<64><<<(unsigned)(chains * 2), wy::kChainThreads, chain_smem, s>>>(
        tm_q32, tm_k32, tm_v, tm_out, blocks, chunk_start, pool, slot_stride, num_slots, ids, cu,
        n_tokens, max_seqlen, out, HK, HV, status);
  else
    wy::chunk_chain_kernel<128><<<(unsigned)chains, wy::kChainThreads, chain_smem, s>>>(
        tm_q32, tm_k32, tm_v, tm_out, blocks, chunk_start, pool, slot_stride, num_slots, ids, cu,
        n_tokens, max_seqlen, out, HK, HV, status);
  return check_launch("gdn_chunk_prefill_varlen");
}

}  // namespace gdn
