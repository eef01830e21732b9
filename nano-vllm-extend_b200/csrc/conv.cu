// (a) Depthwise causal conv1d + SiLU with the prefix state kept in pool slots.
//
// Layouts (the reference engine's, model_runner.py:265-303):
//   x, y        bf16 [rows, C]          row strides given
//   conv_pool   bf16 per-layer view     slot s, channel c, tap j at
//                                       pool[s*slot_stride + c*(K-1) + j]
//   weight      bf16 [C, K]             conv1d.weight viewed [C, K]
//
// Every kernel moves 8 channels per thread as one 16-byte vector (x, y, the
// K-1 taps of 8 channels = (K-1) x 16 bytes, and the K weights of 8 channels
// = K x 16 bytes), so a warp reads 512 contiguous bytes of a token row per
// access.  A scalar kernel covers layouts that are not 16-byte aligned.
//
// The varlen prefill is split in two launches to stay race-free: the conv
// kernel tiles the flat token axis (any number of CTAs per sequence) and only
// READS the prefix state; a second, tiny kernel then rolls each sequence's
// state to its last K-1 inputs.  A single launch would let the CTA holding a
// sequence's tail overwrite the state before the CTA holding its head has
// read it.
//
// The prefill is HBM-bound (2 bytes in + 2 bytes out per element; the K-1 halo
// rows a tile re-reads come from L2).  A tile whose K-1 halo rows and all of
// whose tokens lie inside one sequence (all but a few tiles per sequence)
// copies its K-1+16 rows into shared memory with cp.async at once (each
// thread its own 16-byte column, ~300 bytes in flight per thread without
// holding registers); tiles at sequence boundaries take the general
// per-token path.  Both
// paths evaluate one output with the same conv_point(), so a token's value
// does not depend on where its tile starts (split prefills match one-shot
// prefills bit for bit).
#include "common.cuh"
#include "tc_util.cuh"

namespace gdn {

constexpr int kConvThreads = 128;  // 128 threads x 8 channels = 1024 channels per CTA
constexpr int kConvTileTokens = 16;

// ---------------------------------------------------------------------------
// single-token decode step: qwen3_5.py:515-558
// ---------------------------------------------------------------------------
template <int K>
__global__ void __launch_bounds__(kConvThreads) conv_decode_vec_kernel(
    const bf16* __restrict__ x, int64_t xs, bf16* __restrict__ pool, int64_t slot_stride,
    int64_t num_slots, const int64_t* __restrict__ ids, int C, const bf16* __restrict__ w,
    bf16* __restrict__ y, int64_t ys, int32_t* status) {
  const int n = blockIdx.y;
  const int c0 = (blockIdx.x * kConvThreads + threadIdx.x) * 8;
  const int64_t slot = ids[n];
  if (!slot_ok(slot, num_slots, status)) return;
  if (c0 >= C) return;
  constexpr int T = K - 1;
  float xv[8], sv[8 * T], wv[8 * K], acc[8];
  unpack8(*reinterpret_cast<const uint4*>(x + n * xs + c0), xv);
  uint4* sp = reinterpret_cast<uint4*>(pool + slot * slot_stride + (int64_t)c0 * T);
  uint4 sraw[T];
#pragma unroll
  for (int j = 0; j < T; ++j) sraw[j] = sp[j];
#pragma unroll
  for (int j = 0; j < T; ++j) unpack8(sraw[j], sv + 8 * j);
  const uint4* wp = reinterpret_cast<const uint4*>(w + (int64_t)c0 * K);
#pragma unroll
  for (int j = 0; j < K; ++j) unpack8(wp[j], wv + 8 * j);
#pragma unroll
  for (int ch = 0; ch < 8; ++ch) {
    float win[K];
#pragma unroll
    for (int i = 0; i < T; ++i) win[i] = sv[ch * T + i];
    win[T] = xv[ch];
    acc[ch] = conv_point<K>(win, wv + ch * K);
  }
  *reinterpret_cast<uint4*>(y + n * ys + c0) = pack8(acc);
  // roll: [s1 .. s_{T-1}, x]  (bit copies of bf16 values)
  float ns[8 * T];
#pragma unroll
  for (int ch = 0; ch < 8; ++ch) {
#pragma unroll
    for (int i = 0; i + 1 < T; ++i) ns[ch * T + i] = sv[ch * T + i + 1];
    ns[ch * T + T - 1] = xv[ch];
  }
#pragma unroll
  for (int j = 0; j < T; ++j) sp[j] = pack8(ns + 8 * j);
}

template <int K>
__global__ void __launch_bounds__(kConvThreads) conv_decode_scalar_kernel(
    const bf16* __restrict__ x, int64_t xs, bf16* __restrict__ pool, int64_t slot_stride,
    int64_t num_slots, const int64_t* __restrict__ ids, int C, const bf16* __restrict__ w,
    bf16* __restrict__ y, int64_t ys, int32_t* status) {
  const int n = blockIdx.y;
  const int c = blockIdx.x * kConvThreads + threadIdx.x;
  const int64_t slot = ids[n];
  if (!slot_ok(slot, num_slots, status)) return;
  if (c >= C) return;
  constexpr int T = K - 1;
  bf16* sp = pool + slot * slot_stride + (int64_t)c * T;
  const bf16 xb = x[n * xs + c];
  float win[K], wv[K];
#pragma unroll
  for (int i = 0; i < T; ++i) win[i] = bf2f(sp[i]);
  win[T] = bf2f(xb);
#pragma unroll
  for (int i = 0; i < K; ++i) wv[i] = bf2f(w[(int64_t)c * K + i]);
  y[n * ys + c] = f2bf(conv_point<K>(win, wv));
#pragma unroll
  for (int i = 0; i + 1 < T; ++i) sp[i] = sp[i + 1];
  sp[T - 1] = xb;
}

// ---------------------------------------------------------------------------
// varlen prefill: qwen3_5.py:402-456 (values), tiled over the flat token axis
// ---------------------------------------------------------------------------

// Sequence holding flat row t: largest r with cu[r] <= t (cu non-decreasing).
__device__ __forceinline__ int find_seq(const int32_t* __restrict__ cu, int n_seqs, int64_t t) {
  int lo = 0, hi = n_seqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if ((int64_t)cu[mid] <= t) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// The g / beta gate of the prefill rows, computed by an extra row of the conv
// launch (g == nullptr: no gate row).  b / a are the [rows, H] columns of the
// projection output; g fp32 and beta bf16 are dense [rows, H].
struct GateArgs {
  const bf16* b;
  const bf16* a;
  int64_t ab_stride;
  int H;
  const void* a_log;     // [H] fp32 or bf16 (param_bf16)
  const void* dt_bias;
  bool param_bf16;
  float* g;
  bf16* beta;
};

// g / beta of rows [t_begin, t_end): gbeta_kernel's element order and arithmetic
// (gate_value), so the bits match the separate gate launch.
__device__ __forceinline__ void gate_rows(const GateArgs& ga, int64_t t_begin, int64_t t_end) {
  const int64_t n = (t_end - t_begin) * ga.H;
  for (int64_t i = threadIdx.x; i < n; i += kConvThreads) {
    const int64_t r = t_begin + i / ga.H;
    const int h = (int)(i % ga.H);
    const float al = ga.param_bf16 ? bf2f(static_cast<const bf16*>(ga.a_log)[h])
                                   : static_cast<const float*>(ga.a_log)[h];
    const float db = ga.param_bf16 ? bf2f(static_cast<const bf16*>(ga.dt_bias)[h])
                                   : static_cast<const float*>(ga.dt_bias)[h];
    float gv, bt;
    gate_value(bf2f(ga.a[r * ga.ab_stride + h]), bf2f(ga.b[r * ga.ab_stride + h]), al, db, gv,
               bt);
    ga.g[r * ga.H + h] = gv;
    ga.beta[r * ga.H + h] = f2bf(bt);
  }
}

template <int K, bool VEC>
__global__ void __launch_bounds__(kConvThreads) conv_varlen_kernel(
    const bf16* __restrict__ x, int64_t xs, const bf16* __restrict__ pool, int64_t slot_stride,
    int64_t num_slots, const int64_t* __restrict__ ids, const int32_t* __restrict__ cu,
    int n_seqs, int64_t n_tokens, int C, const bf16* __restrict__ w, bf16* __restrict__ y,
    int64_t ys, int32_t* status, const GateArgs gate) {
  constexpr int T = K - 1;
  constexpr int V = VEC ? 8 : 1;  // channels per thread
  const int64_t t_begin = (int64_t)blockIdx.x * kConvTileTokens;
  if (t_begin >= n_tokens) return;
  const int64_t t_end = min(t_begin + (int64_t)kConvTileTokens, n_tokens);
  if (gate.g != nullptr && blockIdx.y == gridDim.y - 1) {   // the gate row
    gate_rows(gate, t_begin, t_end);
    return;
  }
  const int c0 = (blockIdx.y * kConvThreads + threadIdx.x) * V;
  if (c0 >= C) return;

  float wv[V * K];
  if constexpr (VEC) {
    const uint4* wp = reinterpret_cast<const uint4*>(w + (int64_t)c0 * K);
#pragma unroll
    for (int j = 0; j < K; ++j) unpack8(wp[j], wv + 8 * j);
  } else {
#pragma unroll
    for (int i = 0; i < K; ++i) wv[i] = bf2f(w[(int64_t)c0 * K + i]);
  }

  int r = find_seq(cu, n_seqs, t_begin);
  int64_t seq_start = cu[r], seq_end = cu[r + 1];
  while (t_begin >= seq_end && r + 1 < n_seqs) {  // skip empty sequences
    ++r; seq_start = cu[r]; seq_end = cu[r + 1];
  }

  if constexpr (VEC) {
    constexpr int TT = kConvTileTokens;
    // [row][thread]: a warp's 32 columns of one row are 512 contiguous bytes
    __shared__ uint4 tile[T + TT][kConvThreads];
    // Interior tile: rows t_begin-T .. t_begin+TT-1 all belong to sequence r.
    if (t_begin - T >= seq_start && t_begin >= T && t_begin + TT <= seq_end &&
        seq_end <= n_tokens) {
      const bf16* xp = x + (t_begin - T) * xs + c0;
#pragma unroll
      for (int i = 0; i < T + TT; ++i)
        tc::cp_async16(tc::smem_u32(&tile[i][threadIdx.x]), xp + i * xs, 16);
      tc::cp_async_commit();
      tc::cp_async_wait<0>();  // each thread reads back only its own column
      float win[K][8];  // win[j][ch]: input at t-T+j
#pragma unroll
      for (int j = 0; j < T; ++j) unpack8(tile[j][threadIdx.x], win[j]);
      bf16* yp = y + t_begin * ys + c0;
#pragma unroll
      for (int i = 0; i < TT; ++i) {
        unpack8(tile[T + i][threadIdx.x], win[T]);
        float out[8];
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          float wn[K];
#pragma unroll
          for (int j = 0; j < K; ++j) wn[j] = win[j][ch];
          out[ch] = conv_point<K>(wn, wv + ch * K);
        }
        __stcs(reinterpret_cast<uint4*>(yp + i * ys), pack8(out));
#pragma unroll
        for (int j = 0; j < T; ++j)
#pragma unroll
          for (int ch = 0; ch < 8; ++ch) win[j][ch] = win[j + 1][ch];
      }
      return;
    }
  }

  float win[T][V];  // win[j] = input at position t-T+j
  bool need_init = true;
  for (int64_t t = t_begin; t < t_end; ++t) {
    while (t >= seq_end && r + 1 < n_seqs) {
      ++r; seq_start = cu[r]; seq_end = cu[r + 1]; need_init = true;
    }
    if (need_init) {
      if (seq_start < 0 || seq_end > n_tokens || seq_end < seq_start) {
        if (status) atomicOr(status, GDN_STATUS_BAD_SEQLEN);  // malformed cu_seqlens
        return;
      }
      // Window for token t: positions t-T .. t-1 of sequence r; positions
      // before the sequence start come from the slot's prefix state.
      const int64_t slot = ids[r];
      const bool ok = slot_ok(slot, num_slots, status);
#pragma unroll
      for (int j = 0; j < T; ++j) {
        const int64_t p = t - T + j;
        if (p >= seq_start) {
          if constexpr (VEC) unpack8(*reinterpret_cast<const uint4*>(x + p * xs + c0), win[j]);
          else win[j][0] = bf2f(x[p * xs + c0]);
        } else {
          const int tap = (int)(p - seq_start + T);  // in [0, T)
#pragma unroll
          for (int ch = 0; ch < V; ++ch)
            win[j][ch] = ok ? bf2f(pool[slot * slot_stride + (int64_t)(c0 + ch) * T + tap]) : 0.f;
        }
      }
      need_init = false;
    }
    float xv[V];
    if constexpr (VEC) unpack8(*reinterpret_cast<const uint4*>(x + t * xs + c0), xv);
    else xv[0] = bf2f(x[t * xs + c0]);
    float out[V];
#pragma unroll
    for (int ch = 0; ch < V; ++ch) {
      float wn[K];
#pragma unroll
      for (int i = 0; i < T; ++i) wn[i] = win[i][ch];
      wn[T] = xv[ch];
      out[ch] = conv_point<K>(wn, wv + ch * K);
    }
    if constexpr (VEC) *reinterpret_cast<uint4*>(y + t * ys + c0) = pack8(out);
    else y[t * ys + c0] = f2bf(out[0]);
#pragma unroll
    for (int j = 0; j + 1 < T; ++j)
#pragma unroll
      for (int ch = 0; ch < V; ++ch) win[j][ch] = win[j + 1][ch];
#pragma unroll
    for (int ch = 0; ch < V; ++ch) win[T - 1][ch] = xv[ch];
  }
}

// New state of sequence r = last K-1 entries of [old state | x rows]
// (qwen3_5.py:450-456).  Launched after conv_varlen_kernel on the same stream.
// Every sequence passes through here, so this is where a malformed one (negative
// length, or rows outside [0, n_tokens)) is flagged; its slot is left alone.
template <int K>
__global__ void __launch_bounds__(kConvThreads) conv_state_writeback_kernel(
    const bf16* __restrict__ x, int64_t xs, bf16* __restrict__ pool, int64_t slot_stride,
    int64_t num_slots, const int64_t* __restrict__ ids, const int32_t* __restrict__ cu, int C,
    int64_t n_tokens, int32_t* status) {
  constexpr int T = K - 1;
  const int r = blockIdx.y;
  const int c = blockIdx.x * kConvThreads + threadIdx.x;
  if (c >= C) return;
  const int64_t slot = ids[r];
  if (slot < 0 || slot >= num_slots) return;  // flagged by the conv kernel
  const int64_t start = cu[r], len = (int64_t)cu[r + 1] - start;
  if (len < 0 || start < 0 || start + len > n_tokens) {
    if (status && blockIdx.x == 0 && threadIdx.x == 0) atomicOr(status, GDN_STATUS_BAD_SEQLEN);
    return;
  }
  if (len == 0) return;   // an empty sequence keeps its state
  bf16* sp = pool + slot * slot_stride + (int64_t)c * T;
  bf16 old[T], nw[T];
#pragma unroll
  for (int j = 0; j < T; ++j) old[j] = sp[j];
#pragma unroll
  for (int j = 0; j < T; ++j) {
    const int64_t p = len - T + j;  // position within the sequence
    nw[j] = p >= 0 ? x[(start + p) * xs + c] : old[p + T];
  }
#pragma unroll
  for (int j = 0; j < T; ++j) sp[j] = nw[j];
}

}  // namespace gdn

using namespace gdn;

extern "C" int gdn_conv_decode_step(const void* x, int64_t x_row_stride, void* conv_pool,
                                    int64_t slot_stride, int64_t num_slots, const int64_t* ids,
                                    int32_t n, int32_t channels, int32_t kernel,
                                    const void* weight, void* y, int64_t y_row_stride,
                                    int32_t* status, void* stream) {
  clear_error();
  GDN_REQUIRE(n >= 0 && channels > 0, "gdn_conv_decode_step: bad sizes (n=%d, channels=%d)", n,
              channels);
  GDN_UNSUPPORTED(kernel >= 2 && kernel <= 4, "gdn_conv_decode_step: kernel %d unsupported (2..4)",
                  kernel);
  GDN_REQUIRE(x_row_stride >= channels && y_row_stride >= channels,
              "gdn_conv_decode_step: row stride smaller than channels");
  GDN_REQUIRE(num_slots > 0 && slot_stride >= (int64_t)channels * (kernel - 1),
              "gdn_conv_decode_step: slot_stride %lld < channels*(K-1)", (long long)slot_stride);
  if (n == 0) return GDN_OK;
  GDN_REQUIRE(x && conv_pool && ids && weight && y, "gdn_conv_decode_step: null pointer");
  const bool vec = channels % 8 == 0 && x_row_stride % 8 == 0 && y_row_stride % 8 == 0 &&
                   slot_stride % 8 == 0 && aligned16(x) && aligned16(y) && aligned16(conv_pool) &&
                   aligned16(weight);
  cudaStream_t s = (cudaStream_t)stream;
  const int per_cta = vec ? kConvThreads * 8 : kConvThreads;
  dim3 grid((channels + per_cta - 1) / per_cta, n);
#define GDN_DEC(KK)                                                                            \
  if (kernel == KK) {                                                                          \
    if (vec)                                                                                   \
      conv_decode_vec_kernel<KK><<<grid, kConvThreads, 0, s>>>(                                \
          (const bf16*)x, x_row_stride, (bf16*)conv_pool, slot_stride, num_slots, ids, channels, \
          (const bf16*)weight, (bf16*)y, y_row_stride, status);                                \
    else                                                                                       \
      conv_decode_scalar_kernel<KK><<<grid, kConvThreads, 0, s>>>(                             \
          (const bf16*)x, x_row_stride, (bf16*)conv_pool, slot_stride, num_slots, ids, channels, \
          (const bf16*)weight, (bf16*)y, y_row_stride, status);                                \
  }
  GDN_DEC(2) GDN_DEC(3) GDN_DEC(4)
#undef GDN_DEC
  return check_launch("gdn_conv_decode_step");
}

// The varlen conv (+ the gate row when gate.g is set) and the state roll.
static int launch_conv_varlen(const char* fn, const void* x, int64_t x_row_stride,
                              void* conv_pool, int64_t slot_stride, int64_t num_slots,
                              const int64_t* ids, const int32_t* cu_seqlens, int32_t n_seqs,
                              int64_t n_tokens, int32_t channels, int32_t kernel,
                              const void* weight, void* y, int64_t y_row_stride,
                              const GateArgs& gate, int32_t* status, void* stream) {
  GDN_REQUIRE(n_seqs >= 0 && n_tokens >= 0 && channels > 0,
              "%s: bad sizes (n_seqs=%d, n_tokens=%lld, channels=%d)", fn, n_seqs,
              (long long)n_tokens, channels);
  GDN_UNSUPPORTED(kernel >= 2 && kernel <= 4, "%s: kernel %d unsupported (2..4)", fn, kernel);
  GDN_REQUIRE(x_row_stride >= channels && y_row_stride >= channels,
              "%s: row stride smaller than channels", fn);
  GDN_REQUIRE(num_slots > 0 && slot_stride >= (int64_t)channels * (kernel - 1),
              "%s: slot_stride too small", fn);
  GDN_REQUIRE(n_seqs > 0 || n_tokens == 0, "%s: tokens without sequences", fn);
  if (n_seqs == 0) return GDN_OK;
  GDN_REQUIRE(x && conv_pool && ids && cu_seqlens && weight && y, "%s: null pointer", fn);
  const bool vec = channels % 8 == 0 && x_row_stride % 8 == 0 && y_row_stride % 8 == 0 &&
                   aligned16(x) && aligned16(y) && aligned16(weight);
  cudaStream_t s = (cudaStream_t)stream;
  const int per_cta = vec ? kConvThreads * 8 : kConvThreads;
  const int64_t tiles = (n_tokens + kConvTileTokens - 1) / kConvTileTokens;
  GDN_UNSUPPORTED(tiles < (1ll << 31), "%s: too many tokens", fn);
  const unsigned conv_rows = (unsigned)((channels + per_cta - 1) / per_cta);
  dim3 wgrid((channels + kConvThreads - 1) / kConvThreads, n_seqs);
#define GDN_VL(KK)                                                                               \
  if (kernel == KK) {                                                                            \
    if (tiles > 0) {                                                                             \
      dim3 grid((unsigned)tiles, conv_rows + (gate.g != nullptr ? 1u : 0u));                     \
      if (vec)                                                                                   \
        conv_varlen_kernel<KK, true><<<grid, kConvThreads, 0, s>>>(                              \
            (const bf16*)x, x_row_stride, (const bf16*)conv_pool, slot_stride, num_slots, ids,   \
            cu_seqlens, n_seqs, n_tokens, channels, (const bf16*)weight, (bf16*)y, y_row_stride, \
            status, gate);                                                                       \
      else                                                                                       \
        conv_varlen_kernel<KK, false><<<grid, kConvThreads, 0, s>>>(                             \
            (const bf16*)x, x_row_stride, (const bf16*)conv_pool, slot_stride, num_slots, ids,   \
            cu_seqlens, n_seqs, n_tokens, channels, (const bf16*)weight, (bf16*)y, y_row_stride, \
            status, gate);                                                                       \
    }                                                                                            \
    conv_state_writeback_kernel<KK><<<wgrid, kConvThreads, 0, s>>>(                              \
        (const bf16*)x, x_row_stride, (bf16*)conv_pool, slot_stride, num_slots, ids, cu_seqlens, \
        channels, n_tokens, status);                                                             \
  }
  GDN_VL(2) GDN_VL(3) GDN_VL(4)
#undef GDN_VL
  return check_launch(fn);
}

extern "C" int gdn_causal_conv_silu_varlen(const void* x, int64_t x_row_stride, void* conv_pool,
                                           int64_t slot_stride, int64_t num_slots,
                                           const int64_t* ids, const int32_t* cu_seqlens,
                                           int32_t n_seqs, int64_t n_tokens, int32_t channels,
                                           int32_t kernel, const void* weight, void* y,
                                           int64_t y_row_stride, int32_t* status, void* stream) {
  clear_error();
  const GateArgs none{};
  return launch_conv_varlen("gdn_causal_conv_silu_varlen", x, x_row_stride, conv_pool,
                            slot_stride, num_slots, ids, cu_seqlens, n_seqs, n_tokens, channels,
                            kernel, weight, y, y_row_stride, none, status, stream);
}

extern "C" int gdn_conv_gate_varlen(const void* x, int64_t x_row_stride, void* conv_pool,
                                    int64_t slot_stride, int64_t num_slots, const int64_t* ids,
                                    const int32_t* cu_seqlens, int32_t n_seqs, int64_t n_tokens,
                                    int32_t channels, int32_t kernel, const void* weight, void* y,
                                    int64_t y_row_stride, const void* b, const void* a,
                                    int64_t ab_row_stride, int32_t num_v_heads,
                                    const void* a_log, const void* dt_bias, int32_t param_dtype,
                                    float* g, void* beta, int32_t* status, void* stream) {
  clear_error();
  const char* fn = "gdn_conv_gate_varlen";
  GDN_REQUIRE(num_v_heads > 0, "%s: bad sizes (heads=%d)", fn, num_v_heads);
  GDN_REQUIRE(ab_row_stride >= num_v_heads, "%s: row stride %lld < heads %d", fn,
              (long long)ab_row_stride, num_v_heads);
  GDN_REQUIRE(param_dtype == GDN_DTYPE_F32 || param_dtype == GDN_DTYPE_BF16,
              "%s: param_dtype must be F32 or BF16", fn);
  GDN_REQUIRE(n_tokens == 0 || (b && a && a_log && dt_bias && g && beta), "%s: null pointer", fn);
  GateArgs gate{(const bf16*)b, (const bf16*)a, ab_row_stride, num_v_heads, a_log, dt_bias,
                param_dtype == GDN_DTYPE_BF16, g, (bf16*)beta};
  return launch_conv_varlen(fn, x, x_row_stride, conv_pool, slot_stride, num_slots, ids,
                            cu_seqlens, n_seqs, n_tokens, channels, kernel, weight, y,
                            y_row_stride, gate, status, stream);
}
