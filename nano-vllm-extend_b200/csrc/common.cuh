// Shared helpers for the GDN kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "gdn_b200.h"

namespace gdn {

using bf16 = __nv_bfloat16;

// Thread-local last-error message (read by gdn_last_error()).
void set_error(const char* fmt, ...);
void clear_error();

// After a launch: map a launch failure to GDN_ERR_CUDA with a message.
int check_launch(const char* what);

// Number of SMs of the current device (cached per device).
int sm_count();

// Poll limit for the bounded device waits that honour gdn_set_wait_limit():
// `dflt` unless a test has set an override.
uint32_t wait_limit(uint32_t dflt);

// Gated RMSNorm launch (gate_norm.cu); x and y may alias (in place).
int launch_rms_norm_gated(const void* x, const void* gate, int64_t gate_token_stride,
                          int heads_per_token, const void* weight, void* y, int64_t n_rows,
                          int dim, float eps, cudaStream_t s);

// The reference's gated-norm rounding for one element (qwen3_5.py:127-131):
// y = bf16(bf16(w * bf16(x * inv)) * silu(z)), fp32 arithmetic; silu with the
// hardware exp2 / reciprocal approximations (a few fp32 ulps before the final
// bf16 rounding), which keeps the prefill norm HBM-bound.
__device__ __forceinline__ float gated_norm_elem(float x, float inv, float w, float z);

#define GDN_REQUIRE(cond, ...)                       \
  do {                                               \
    if (!(cond)) {                                   \
      ::gdn::set_error(__VA_ARGS__);                 \
      return GDN_ERR_INVALID_ARGUMENT;               \
    }                                                \
  } while (0)

#define GDN_UNSUPPORTED(cond, ...)                   \
  do {                                               \
    if (!(cond)) {                                   \
      ::gdn::set_error(__VA_ARGS__);                 \
      return GDN_ERR_UNSUPPORTED;                    \
    }                                                \
  } while (0)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

__device__ __forceinline__ float bf2f(bf16 x) { return __bfloat162float(x); }
__device__ __forceinline__ bf16 f2bf(float x) { return __float2bfloat16_rn(x); }
__device__ __forceinline__ float round_bf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float siluf_(float x) { return x * sigmoidf_(x); }

__device__ __forceinline__ float gated_norm_elem(float x, float inv, float w, float z) {
  const float t = __bfloat162float(__float2bfloat16_rn(x * inv));
  const float u = __bfloat162float(__float2bfloat16_rn(w * t));
  return u * __fdividef(z, 1.0f + __expf(-z));
}

// Depthwise conv tap sum + SiLU for one channel: acc = sum_{i<K} w[i] *
// win[i] in tap order, win[K-1] the current input (qwen3_5.py:438-446,
// 540-548); SiLU with the hardware exp2 / reciprocal approximations (a few
// fp32 ulps before the bf16 rounding of the result).  Every conv path uses
// this function, so a token's value does not depend on the kernel that
// computed it.
__device__ __forceinline__ float conv_silu(float a) { return __fdividef(a, 1.0f + __expf(-a)); }

template <int K>
__device__ __forceinline__ float conv_point(const float* win, const float* w) {
  float a = win[0] * w[0];
#pragma unroll
  for (int i = 1; i < K; ++i) a = fmaf(win[i], w[i], a);
  return conv_silu(a);
}

// The decay gate and write strength of one (token, v-head) (qwen3_5.py:320-343):
// g = -exp(A_log) * softplus(a + dt_bias) (softplus threshold 20), beta =
// sigmoid(b) rounded to bf16 (the reference stores beta in the model dtype).
__device__ __forceinline__ void gate_value(float av, float bv, float a_log, float dt_bias,
                                           float& g, float& beta) {
  const float z = av + dt_bias;
  const float sp = z > 20.0f ? z : logf(1.0f + expf(z));
  g = -expf(a_log) * sp;
  beta = round_bf(sigmoidf_(bv));
}

// 8 packed bf16 <-> 8 floats
__device__ __forceinline__ void unpack8(const uint4& u, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float* f) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return u;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Record a bad slot id (never dereferenced) in the optional status word.
__device__ __forceinline__ bool slot_ok(int64_t slot, int64_t num_slots, int32_t* status) {
  if (slot >= 0 && slot < num_slots) return true;
  if (status) atomicOr(status, GDN_STATUS_BAD_SLOT);
  return false;
}

}  // namespace gdn
