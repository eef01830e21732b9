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
