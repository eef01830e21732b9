// (b) fused g/beta gate and the gated RMSNorm epilogue.
//
// Both are HBM-bound elementwise / row kernels.  The gate reads 2+2 bytes
// and writes 4+2 bytes per (token, v-head); the norm reads x and gate and
// writes y (6 bytes per element).  Grids are sized to a multiple of the SM
// count with grid-stride loops.
#include "common.cuh"

namespace gdn {

template <typename P>
__device__ __forceinline__ float load_param(const P* p, int i);
template <>
__device__ __forceinline__ float load_param<float>(const float* p, int i) { return p[i]; }
template <>
__device__ __forceinline__ float load_param<bf16>(const bf16* p, int i) { return bf2f(p[i]); }

// g = -exp(A_log) * softplus(a + dt_bias) (threshold 20), beta = sigmoid(b).
// Follows qwen3_5.py:320-343 step for step (fp32 arithmetic).
template <typename P>
__global__ void __launch_bounds__(256) gbeta_kernel(
    const bf16* __restrict__ b, const bf16* __restrict__ a, int64_t row_stride,
    int64_t n_rows, int H, const P* __restrict__ a_log, const P* __restrict__ dt_bias,
    const uint8_t* __restrict__ mask, float* __restrict__ g, bf16* __restrict__ beta) {
  const int64_t total = n_rows * H;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / H;
    const int h = (int)(i - r * H);
    float gv, bt;
    gate_value(bf2f(a[r * row_stride + h]), bf2f(b[r * row_stride + h]),
               load_param<P>(a_log, h), load_param<P>(dt_bias, h), gv, bt);
    if (mask != nullptr && mask[r] == 0) gv = 0.0f;
    g[i] = gv;
    beta[i] = f2bf(bt);
  }
}

// Gated RMSNorm, y = bf16(bf16(w * bf16(x * rsqrt(mean x^2 + eps))) * silu(gate)), the
// rounding sequence of qwen3_5.py:121-131 for a bf16 model.  Each lane moves 8
// elements as 16-byte vectors; DIM/8 lanes share a row and reduce by shuffles.
// A warp issues the loads of U row sets (U * 32 / (DIM/8) rows) before it
// computes any of them, so each lane keeps U x 32 bytes in flight.
// x and y may alias: a row's lanes read it fully before any of them writes.
template <int DIM>
__global__ void __launch_bounds__(256, 3) rms_gated_kernel(
    const bf16* x, const bf16* __restrict__ gate, int64_t gate_token_stride,
    int heads, const bf16* __restrict__ w, bf16* y, int64_t n_rows, float eps) {
  constexpr int LPR = DIM / 8;                 // lanes per row
  constexpr int RPW = 32 / LPR;                // rows per warp and row set
  constexpr int U = 4;                         // row sets in flight per warp
  const int lane = threadIdx.x & 31;
  const int sub = lane % LPR;
  float wv[8];
  unpack8(*reinterpret_cast<const uint4*>(w + sub * 8), wv);
  const int64_t rows_per_iter = (int64_t)gridDim.x * (blockDim.x >> 5) * RPW * U;
  // warp-uniform loop bound: every lane of a warp runs the same iterations
  for (int64_t base = ((int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * RPW * U;
       base < n_rows; base += rows_per_iter) {
    const int64_t row0 = base + lane / LPR;
    uint4 xr[U], gr[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t row = row0 + u * RPW;
      xr[u] = make_uint4(0u, 0u, 0u, 0u);
      gr[u] = make_uint4(0u, 0u, 0u, 0u);
      if (row < n_rows) {
        xr[u] = *reinterpret_cast<const uint4*>(x + row * DIM + sub * 8);
        const uint32_t tok = (uint32_t)row / (uint32_t)heads;   // n_rows < 2^32 (host check)
        const uint32_t hh = (uint32_t)row - tok * (uint32_t)heads;
        gr[u] = *reinterpret_cast<const uint4*>(gate + (int64_t)tok * gate_token_stride +
                                                hh * DIM + sub * 8);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t row = row0 + u * RPW;
      float xv[8], gv[8];
      unpack8(xr[u], xv);
      unpack8(gr[u], gv);
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += xv[e] * xv[e];
#pragma unroll
      for (int o = LPR / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float inv = rsqrtf(ss / (float)DIM + eps);
      if (row < n_rows) {
        float yv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) yv[e] = gated_norm_elem(xv[e], inv, wv[e], gv[e]);
        *reinterpret_cast<uint4*>(y + row * DIM + sub * 8) = pack8(yv);
      }
    }
  }
}

int launch_rms_norm_gated(const void* x, const void* gate, int64_t gate_token_stride,
                          int heads_per_token, const void* weight, void* y, int64_t n_rows,
                          int dim, float eps, cudaStream_t s) {
  if (n_rows == 0) return GDN_OK;
  GDN_UNSUPPORTED(n_rows < (1ll << 32), "gated norm: %lld rows (max 2^32 - 1)", (long long)n_rows);
  GDN_UNSUPPORTED(((uintptr_t)x | (uintptr_t)gate | (uintptr_t)weight | (uintptr_t)y) % 16 == 0 &&
                      gate_token_stride % 8 == 0,
                  "gated norm: operands must be 16-byte aligned");
  const int64_t rows_per_block = 8 * (32 / (dim / 8)) * 4;   // warps x rows x row sets
  int64_t blocks = (n_rows + rows_per_block - 1) / rows_per_block;
  const int64_t cap = (int64_t)sm_count() * 8;
  if (blocks > cap) blocks = cap;
#define GDN_NORM_CASE(D)                                                                        \
  case D:                                                                                       \
    rms_gated_kernel<D><<<(unsigned)blocks, 256, 0, s>>>((const bf16*)x, (const bf16*)gate,    \
                                                         gate_token_stride, heads_per_token,    \
                                                         (const bf16*)weight, (bf16*)y, n_rows, \
                                                         eps);                                  \
    break;
  switch (dim) {
    GDN_NORM_CASE(64)
    GDN_NORM_CASE(128)
    GDN_NORM_CASE(256)
    default:
      set_error("gated norm: dim %d unsupported", dim);
      return GDN_ERR_UNSUPPORTED;
  }
#undef GDN_NORM_CASE
  return check_launch("gated norm");
}

}  // namespace gdn

using namespace gdn;

extern "C" int gdn_fused_g_beta(const void* b, const void* a, int64_t ab_row_stride,
                                int64_t n_rows, int32_t num_v_heads, const void* a_log,
                                const void* dt_bias, int32_t param_dtype,
                                const uint8_t* row_mask, float* g, void* beta, void* stream) {
  clear_error();
  GDN_REQUIRE(n_rows >= 0 && num_v_heads > 0, "gdn_fused_g_beta: bad sizes (n_rows=%lld, heads=%d)",
              (long long)n_rows, num_v_heads);
  GDN_REQUIRE(ab_row_stride >= num_v_heads, "gdn_fused_g_beta: row stride %lld < heads %d",
              (long long)ab_row_stride, num_v_heads);
  GDN_REQUIRE(param_dtype == GDN_DTYPE_F32 || param_dtype == GDN_DTYPE_BF16,
              "gdn_fused_g_beta: param_dtype must be F32 or BF16");
  if (n_rows == 0) return GDN_OK;
  GDN_REQUIRE(b && a && a_log && dt_bias && g && beta, "gdn_fused_g_beta: null pointer");
  const int64_t total = n_rows * num_v_heads;
  int64_t blocks = (total + 255) / 256;
  const int64_t cap = (int64_t)sm_count() * 8;
  if (blocks > cap) blocks = cap;
  cudaStream_t s = (cudaStream_t)stream;
  if (param_dtype == GDN_DTYPE_F32)
    gbeta_kernel<float><<<(unsigned)blocks, 256, 0, s>>>(
        (const bf16*)b, (const bf16*)a, ab_row_stride, n_rows, num_v_heads, (const float*)a_log,
        (const float*)dt_bias, row_mask, g, (bf16*)beta);
  else
    gbeta_kernel<bf16><<<(unsigned)blocks, 256, 0, s>>>(
        (const bf16*)b, (const bf16*)a, ab_row_stride, n_rows, num_v_heads, (const bf16*)a_log,
        (const bf16*)dt_bias, row_mask, g, (bf16*)beta);
  return check_launch("gdn_fused_g_beta");
}

extern "C" int gdn_rms_norm_gated(const void* x, const void* gate, int64_t gate_token_stride,
                                  int32_t heads_per_token, const void* weight, void* y,
                                  int64_t n_rows, int32_t dim, float eps, void* stream) {
  clear_error();
  GDN_REQUIRE(n_rows >= 0, "gdn_rms_norm_gated: n_rows < 0");
  GDN_UNSUPPORTED(dim == 64 || dim == 128 || dim == 256,
                  "gdn_rms_norm_gated: dim %d unsupported (64, 128, 256)", dim);
  GDN_REQUIRE(heads_per_token > 0 && n_rows % heads_per_token == 0,
              "gdn_rms_norm_gated: n_rows %lld not a multiple of heads_per_token %d",
              (long long)n_rows, heads_per_token);
  GDN_REQUIRE(gate_token_stride >= (int64_t)heads_per_token * dim,
              "gdn_rms_norm_gated: gate token stride < heads_per_token * dim");
  if (n_rows == 0) return GDN_OK;
  GDN_REQUIRE(x && gate && weight && y, "gdn_rms_norm_gated: null pointer");
  return launch_rms_norm_gated(x, gate, gate_token_stride, heads_per_token, weight, y, n_rows,
                               dim, eps, (cudaStream_t)stream);
}
