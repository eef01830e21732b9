// Pieces shared by the two tensor-core forms of the chunked prefill
// (chunk_tc.cu: one kernel per (sequence, v-head) chain; chunk_wy.cu: a
// parallel per-chunk prep kernel plus the chain kernel).  Chunk C = 64 tokens,
// head dim 128, 128B-swizzled bf16 tiles (tc_util.cuh).
#pragma once

#include <cuda.h>

#include "tc_util.cuh"
#include "tmap.cuh"

namespace gdn {
namespace tc {

constexpr int kC = 64;
constexpr int kD = 128;
constexpr int kLptMaxSeqs = 256;   // longest-first chain order up to this many sequences
constexpr int kLP = kC + 4;        // row pitch of L / T (16-byte aligned rows)

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

// Per-token scalars of one chunk (shared memory).  gam holds the raw g on
// entry to decay_scan and the in-chunk cumulative decay gamma after it.
struct ChunkScalars {
  float gam[kC], eg[kC], bet[kC], nk[kC], nq[kC], bcol[kC], cf[kC], gend[4];
};

// Warp 0: gamma = inclusive cumsum of g over the chunk (2 tokens per lane),
// e^gamma, and the factors e^(gamma_end(J) - gamma_j) <= 1 of the 16-token
// blocks J (qwen3_5.py:176-177 decay mask, split at block ends).
__device__ __forceinline__ void decay_scan(ChunkScalars& s, int lane) {
  const float ga = s.gam[2 * lane], gb = s.gam[2 * lane + 1];
  float x = ga + gb;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  const float g0 = x - gb;                      // gamma of token 2*lane
  // gamma at the end of each 16-token block (token 16J+15 = lane 8J+7, second element)
  const float gE = __shfl_sync(0xffffffffu, x, ((2 * lane) >> 4) * 8 + 7);
  __syncwarp();
  s.gam[2 * lane] = g0;
  s.gam[2 * lane + 1] = x;
  s.eg[2 * lane] = expf(g0);
  s.eg[2 * lane + 1] = expf(x);
  s.bcol[2 * lane] = __expf(gE - g0);          // <= 1 (g <= 0)
  s.bcol[2 * lane + 1] = __expf(gE - x);
  if ((lane & 7) == 7) s.gend[lane >> 3] = x;
}

// Row norms from the diagonal of P = [K;Q][K;Q]^T (TMEM columns colP..+128,
// thread t <-> lane t of 128): nk = 1/|k|, nq = scale/|q| (l2norm eps 1e-6,
// qwen3_5.py:160-161), cf = nk * bcol.
__device__ __forceinline__ void norms_from_diag(ChunkScalars& s, uint32_t tl, uint32_t colP,
                                                int tid, float scale) {
  const int warp = tid >> 5, lane = tid & 31;
  float p[32];
  tmem_ld32(tl + colP + warp * 32, p);
  float d = 0.f;
#pragma unroll
  for (int jj = 0; jj < 32; ++jj) d = (jj == lane) ? p[jj] : d;
  if (tid < 64) {
    const float n = rsqrtf(d + 1e-6f);
    s.nk[tid] = n;
    s.cf[tid] = n * s.bcol[tid];
  } else {
    s.nq[tid - 64] = rsqrtf(d + 1e-6f) * scale;
  }
}

// From P (TMEM, thread t <-> lane t of 128): rows 0-63 build
//   L   = -(beta_i nk_i nk_j P_ij e^(gamma_i - gamma_j))   (j < i)   -> Lm (fp32)
// rows 64-127 build
//   QKm =  (nq_i nk_j QK_ij e^(gamma_i - gamma_j))          (j <= i)  -> qkm tile (bf16)
// (qwen3_5.py:176-195).  Left of the 16-token diagonal block the decay is the
// product of two factors <= 1 (no overflow, ~5x fewer exponentials).
__device__ __forceinline__ void build_l_qkm(const ChunkScalars& s, uint32_t tl, uint32_t colP,
                                            int tid, float (*Lm)[kLP], uint8_t* qkm) {
  const int i = tid & 63;
  const bool isq = tid >= 64;
  const int I = i >> 4;
  const float gi = s.gam[i];
  const float rowf = isq ? s.nq[i] : -s.bet[i] * s.nk[i];
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    float p[32];
    tmem_ld32(tl + colP + hh * 32, p);
#pragma unroll
    for (int b2 = 0; b2 < 2; ++b2) {
      const int J = hh * 2 + b2;
      float* pe = p + b2 * 16;
      if (J < I) {
        const float rf = rowf * __expf(gi - s.gend[J]);
#pragma unroll
        for (int jj = 0; jj < 16; jj += 2) {
          const float2 c2 = *reinterpret_cast<const float2*>(&s.cf[J * 16 + jj]);
          float f0, f1;
          fmul2(f0, f1, rf, rf, c2.x, c2.y);
          fmul2(pe[jj], pe[jj + 1], pe[jj], pe[jj + 1], f0, f1);
        }
      } else if (J == I) {
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) {
          const int j = J * 16 + jj;
          const bool keep = isq ? (j <= i) : (j < i);
          pe[jj] = keep ? pe[jj] * rowf * s.nk[j] * __expf(gi - s.gam[j]) : 0.f;
        }
      } else {
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) pe[jj] = 0.f;
      }
    }
    if (isq) {
#pragma unroll
      for (int q8 = 0; q8 < 4; ++q8) st8(qkm, i, hh * 32 + q8 * 8, p + q8 * 8);
    } else {
#pragma unroll
      for (int q4 = 0; q4 < 8; ++q4)
        *reinterpret_cast<float4*>(&Lm[i][hh * 32 + q4 * 4]) =
            make_float4(p[4 * q4], p[4 * q4 + 1], p[4 * q4 + 2], p[4 * q4 + 3]);
    }
  }
}

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
template <int NT>
__device__ __noinline__ int lpt_sequence(const int32_t* __restrict__ cu, int n_seqs, int rank,
                                         int tid) {
  __shared__ int s_len[kLptMaxSeqs];
  __shared__ int s_seq;
  if (n_seqs > kLptMaxSeqs) return rank;
  for (int i = tid; i < n_seqs; i += NT) s_len[i] = cu[i + 1] - cu[i];
  if (tid == 0) s_seq = rank;
  __syncthreads();
  for (int i = tid; i < n_seqs; i += NT) {
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

// bf16 [rows, cols] view with a row stride (elements), boxes of 64 columns x
// box_rows rows, 128B swizzle.
inline bool make_tile_map(CUtensorMap* m, const void* base, int64_t cols, int64_t rows,
                          int64_t row_stride, uint32_t box_rows = 64) {
  EncodeTiledFn fn = encode_tiled();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)row_stride * 2};
  const cuuint32_t box[2] = {64, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

}  // namespace tc
}  // namespace gdn
