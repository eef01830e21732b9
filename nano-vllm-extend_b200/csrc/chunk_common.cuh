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
    float l0, l1;   // x - hi, exact, as one packed fp32x2 operation
    ffma2(l0, l1, __uint_as_float(b0 & 0xFFFF0000u), __uint_as_float(b1 & 0xFFFF0000u), -1.f,
          -1.f, x[2 * e], x[2 * e + 1]);
    lp[e] = __floats2bfloat162_rn(l0, l1);
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

// l2 norms (eps 1e-6, qwen3_5.py:160-161) of the chunk's rows, thread t <-> row
// t of the [K;Q] tile (rows 0-63 K, 64-127 Q; two 64-column dk blocks).
// K rows (t < 64): nk = 1/|k| from the diagonal of P = [K;Q] K^T (TMEM columns
// colP.., exact bf16 products), cf = nk * bcol.
__device__ __forceinline__ void k_norm_from_diag(ChunkScalars& s, uint32_t tl, uint32_t colP,
                                                 int tid) {
  const int warp = tid >> 5, lane = tid & 31;
  float p[32];
  tmem_ld32(tl + colP + warp * 32, p);
  float d = 0.f;
#pragma unroll
  for (int jj = 0; jj < 32; ++jj) d = (jj == lane) ? p[jj] : d;
  const float n = rsqrtf(d + 1e-6f);
  s.nk[tid] = n;
  s.cf[tid] = n * s.bcol[tid];
}
// Q row of token i at tile row `row`: nq = scale/|q| summed on the CUDA cores in
// a fixed order (rows past the sequence end count as zero rows).
__device__ __forceinline__ void q_norm_row(ChunkScalars& s, const uint8_t* kq, int i, int row,
                                           int nv, float scale) {
  float a0 = 0.f, a1 = 0.f;
  if (i < nv) {
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      float f[8];
      unpack8(*reinterpret_cast<const uint4*>(kq + (c >> 3) * 16384 + sw128(row, (c & 7) * 8)),
              f);
#pragma unroll
      for (int e = 0; e < 8; e += 2) ffma2(a0, a1, f[e], f[e + 1], f[e], f[e + 1], a0, a1);
    }
  }
  s.nq[i] = rsqrtf(a0 + a1 + 1e-6f) * scale;
}
// Q rows (t >= 64) of the [K;Q] tile.
__device__ __forceinline__ void q_norm(ChunkScalars& s, const uint8_t* kq, int tid, int nv,
                                       float scale) {
  q_norm_row(s, kq, tid - 64, tid, nv, scale);
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
#pragma unroll 1   // rolled: the unrolled body's code size costs instruction-cache misses
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
        for (int jj = 0; jj < 16; jj += 4) {
          const float4 c4 = *reinterpret_cast<const float4*>(&s.cf[J * 16 + jj]);
          float f0, f1, f2, f3;
          fmul2(f0, f1, rf, rf, c4.x, c4.y);
          fmul2(f2, f3, rf, rf, c4.z, c4.w);
          fmul2(pe[jj], pe[jj + 1], pe[jj], pe[jj + 1], f0, f1);
          fmul2(pe[jj + 2], pe[jj + 3], pe[jj + 2], pe[jj + 3], f2, f3);
        }
      } else if (J == I) {
#pragma unroll
        for (int j4 = 0; j4 < 16; j4 += 4) {
          const float4 n4 = *reinterpret_cast<const float4*>(&s.nk[J * 16 + j4]);
          const float4 g4 = *reinterpret_cast<const float4*>(&s.gam[J * 16 + j4]);
          const float nv4[4] = {n4.x, n4.y, n4.z, n4.w}, gv4[4] = {g4.x, g4.y, g4.z, g4.w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int jj = j4 + k, j = J * 16 + jj;
            const bool keep = isq ? (j <= i) : (j < i);
            pe[jj] = keep ? pe[jj] * rowf * nv4[k] * __expf(gi - gv4[k]) : 0.f;
          }
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

// A [K;Q] tile interleaved by 16 rows, [K 0-15; Q 0-15; K 16-31; Q 16-31; ...]:
// tile row of token i's K row (second = false) or Q row (second = true).  With
// P = [K;Q][K;Q]^T in TMEM, warp w (lane quarter w % 4) then holds the K and Q
// rows of one 16-token block, so the block-structured L / QKm build below runs
// without divergence between the two blocks a plain [K;Q] quarter would mix.
__host__ __device__ constexpr int ilv16_row(int i, bool second) {
  return 32 * (i >> 4) + (i & 15) + (second ? 16 : 0);
}

// nk = 1/|k| from P's diagonal for the interleaved tile: lanes 0-15 of each
// warp (K rows of block w % 4); all 32 lanes load (warp-collective).
__device__ __forceinline__ void k_norm_ilv16(ChunkScalars& s, uint32_t tl, uint32_t colP,
                                             int tid) {
  const int q = (tid >> 5) & 3, lane = tid & 31;
  float p[32];
  tmem_ld32(tl + colP + q * 32, p);
  float d = 0.f;
#pragma unroll
  for (int jj = 0; jj < 32; ++jj) d = (jj == lane) ? p[jj] : d;
  if (lane < 16) {
    const int i = 16 * q + lane;
    const float n = rsqrtf(d + 1e-6f);
    s.nk[i] = n;
    s.cf[i] = n * s.bcol[i];
  }
}

// L (K rows) and QKm (Q rows) from P for the interleaved tile — the arithmetic of
// build_l_qkm, with the row's 16-token block uniform across the warp.  K token
// j's column is ilv16_row(j, false).
__device__ __forceinline__ void build_l_qkm_ilv16(const ChunkScalars& s, uint32_t tl,
                                                  uint32_t colP, int tid, float (*Lm)[kLP],
                                                  uint8_t* qkm) {
  const int I = (tid >> 5) & 3, lane = tid & 31;
  const bool isq = lane >= 16;
  const int i = 16 * I + (lane & 15);
  const float gi = s.gam[i];
  const float rowf = isq ? s.nq[i] : -s.bet[i] * s.nk[i];
#pragma unroll 1   // rolled: code size (instruction-cache pressure)
  for (int J = 0; J < 4; ++J) {
    float pe[16];
    tmem_ld16(tl + colP + 32 * J, pe);
    if (J < I) {                       // warp-uniform
      const float rf = rowf * __expf(gi - s.gend[J]);
#pragma unroll
      for (int jj = 0; jj < 16; jj += 4) {
        const float4 c4 = *reinterpret_cast<const float4*>(&s.cf[J * 16 + jj]);
        float f0, f1, f2, f3;
        fmul2(f0, f1, rf, rf, c4.x, c4.y);
        fmul2(f2, f3, rf, rf, c4.z, c4.w);
        fmul2(pe[jj], pe[jj + 1], pe[jj], pe[jj + 1], f0, f1);
        fmul2(pe[jj + 2], pe[jj + 3], pe[jj + 2], pe[jj + 3], f2, f3);
      }
    } else if (J == I) {
#pragma unroll
      for (int j4 = 0; j4 < 16; j4 += 4) {
        const float4 n4 = *reinterpret_cast<const float4*>(&s.nk[J * 16 + j4]);
        const float4 g4 = *reinterpret_cast<const float4*>(&s.gam[J * 16 + j4]);
        const float nv4[4] = {n4.x, n4.y, n4.z, n4.w}, gv4[4] = {g4.x, g4.y, g4.z, g4.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int jj = j4 + k, j = J * 16 + jj;
          const bool keep = isq ? (j <= i) : (j < i);
          pe[jj] = keep ? pe[jj] * rowf * nv4[k] * __expf(gi - gv4[k]) : 0.f;
        }
      }
    } else {
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) pe[jj] = 0.f;
    }
    if (isq) {
      st8(qkm, i, J * 16, pe);
      st8(qkm, i, J * 16 + 8, pe + 8);
    } else {
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4)
        *reinterpret_cast<float4*>(&Lm[i][J * 16 + q4 * 4]) =
            make_float4(pe[4 * q4], pe[4 * q4 + 1], pe[4 * q4 + 2], pe[4 * q4 + 3]);
    }
  }
}

// m16n8k8 tf32 tensor-core tile product (warp-wide): D += A B, fp32 accumulate.
__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4],
                                         const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
// fp32 -> tf32 (round to nearest, ties away from zero).
__device__ __forceinline__ uint32_t to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

// D[16 x 8*NT] = A[16 x 8*KS] B[8*KS x 8*NT] for one warp, A and B fp32 in
// shared memory (row pitches lda / ldb floats), rounded to tf32 on load;
// fragment layout of mma.m16n8k8 (g = lane / 4, t = lane % 4).
template <int KS, int NT>
__device__ __forceinline__ void warp_mma_tf32(float (&d)[NT][4], const float* A, int lda,
                                              const float* B, int ldb, int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int n = 0; n < NT; ++n) d[n][0] = d[n][1] = d[n][2] = d[n][3] = 0.f;
#pragma unroll
  for (int ks = 0; ks < KS; ++ks) {
    const float* Ak = A + ks * 8;
    const uint32_t a[4] = {to_tf32(Ak[g * lda + t]), to_tf32(Ak[(g + 8) * lda + t]),
                           to_tf32(Ak[g * lda + t + 4]), to_tf32(Ak[(g + 8) * lda + t + 4])};
    const float* Bk = B + ks * 8 * ldb;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const uint32_t bb[2] = {to_tf32(Bk[t * ldb + n * 8 + g]),
                              to_tf32(Bk[(t + 4) * ldb + n * 8 + g])};
      mma_tf32(d[n], a, bb);
    }
  }
}
template <int NT>
__device__ __forceinline__ void warp_store_tile(const float (&d)[NT][4], float* D, int ldd,
                                                int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int n = 0; n < NT; ++n) {
    *reinterpret_cast<float2*>(&D[g * ldd + n * 8 + 2 * t]) = make_float2(d[n][0], d[n][1]);
    *reinterpret_cast<float2*>(&D[(g + 8) * ldd + n * 8 + 2 * t]) = make_float2(d[n][2], d[n][3]);
  }
}

constexpr int kXP = 40;   // row pitch of the X scratch (conflict-free B-fragment reads)

// T = (I - L)^-1 for the strictly lower 64x64 L (fp32, shared memory, upper
// triangle zero), computed IN PLACE (T overwrites L): 16x16 diagonal blocks by
// forward substitution in registers (fp32), then two recursive-doubling levels
// — with (I - L) = [A 0; -L21 B], T = [A^-1 0; B^-1 L21 A^-1  B^-1] — at
// 16 -> 32 and 32 -> 64, their block products on the tensor cores (tf32
// operands, fp32 accumulation; T is rounded to bf16 for its MMAs afterwards).
// Each level reads its L21 block before the T21 that replaces it is written.
// 128 threads (4 warps); X is a 5 KiB fp32 scratch (32 rows of kXP).
__device__ __forceinline__ void invert_unit_lower(float (*LT)[kLP], float* X, int tid) {
  const int warp = tid >> 5, lane = tid & 31;
  {  // diagonal 16x16 blocks: warp w owns block w, lane l solves column l % 16
    const int b0 = 16 * warp, j = lane & 15;
    float t[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int m4 = 0; m4 < (i + 3) / 4; ++m4) {
        const float4 l4 = *reinterpret_cast<const float4*>(&LT[b0 + i][b0 + 4 * m4]);
        const float lv[4] = {l4.x, l4.y, l4.z, l4.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int m = 4 * m4 + k;
          if (m < i) {
            const float pr = lv[k] * t[m];
            if (m & 1) s1 += pr; else s0 += pr;
          }
        }
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
  {  // 16 -> 32: warp w: 32-block hb = 32 (w / 2), column tile 8 (w % 2) of the 16-wide blocks
    const int hb = (warp >> 1) * 32, c = (warp & 1) * 8;
    float* Xh = X + (warp >> 1) * 16;
    float d[1][4];
    warp_mma_tf32<2, 1>(d, &LT[hb + 16][hb], kLP, &LT[hb][hb + c], kLP, lane);   // L21 A^-1
    warp_store_tile<1>(d, Xh + c, kXP, lane);
    __syncthreads();   // every warp has read its L21 block
    warp_mma_tf32<2, 1>(d, &LT[hb + 16][hb + 16], kLP, Xh + c, kXP, lane);       // B^-1 X
    warp_store_tile<1>(d, &LT[hb + 16][hb + c], kLP, lane);
  }
  __syncthreads();
  {  // 32 -> 64: warp w: rows 16 (w / 2) of the 32-row blocks, column tiles 2 (w % 2) + {0, 1}
    const int r = (warp >> 1) * 16, c = (warp & 1) * 16;
    float d[2][4];
    warp_mma_tf32<4, 2>(d, &LT[32 + r][0], kLP, &LT[0][c], kLP, lane);          // L21 A^-1
    warp_store_tile<2>(d, X + r * kXP + c, kXP, lane);
    __syncthreads();   // X complete; every warp has read L21
    warp_mma_tf32<4, 2>(d, &LT[32 + r][32], kLP, X + c, kXP, lane);             // B^-1 X
    warp_store_tile<2>(d, &LT[32 + r][c], kLP, lane);
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
