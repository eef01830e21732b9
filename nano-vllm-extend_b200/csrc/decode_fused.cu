// (d) + (a) + (b) + norm: the whole GDN decode core of one layer in one launch.
//
// For every decode row (sequence b) and v-head h it computes, from the fused
// input projection row, what the reference does in four kernels
// (qwen3_5.py:1008-1026 and 1083-1085):
//   conv step  : q, k, v = bf16(silu(conv(state, x)))  and the conv state roll
//   gate       : g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b)
//   recurrence : S' = e^g S; d = beta (v - S'^T k^); S'' = S' + k^ (x) d;
//                o = S''^T q^  (q^, k^ l2-normalised, q^ scaled)
//   norm       : out = bf16(bf16(w * bf16(o * rsqrt(mean o^2 + eps))) * silu(z))
// with the fp32 state read from and written back to its pool slot in place.
//
// Work unit and race freedom.  A CTA owns whole k-head groups (b, hk): the
// R = HV / HK v-heads that share q/k head hk.  The group's conv channels
// (q and k of head hk, v of its R heads) are convolved and their conv state
// rolled once, by that CTA, before its R recurrence units run, so no other CTA
// reads a conv state this one rewrites.
//
// HBM pipeline.  The kernel is persistent (one CTA per SM for D = 128) and
// streams the per-head fp32 states (D x D, contiguous in the pool) through an
// NSTAGE-deep ring of shared-memory buffers with 1-D bulk async copies that
// complete on mbarriers: while a unit computes, the states of the next
// NSTAGE-1 units are already on the way, so HBM always has reads in flight.
// New states go back from registers with streaming 16-byte stores.  The
// recurrence maths, its reduction order, the conv tap order and the gate and
// norm formulas are those of conv_decode_step + fused_g_beta +
// recurrent_inplace + rms_norm_gated, so the fused result is bit-identical
// to that four-launch sequence.
//
// Every mbarrier wait is bounded: on time-out the CTA raises
// GDN_STATUS_TIMEOUT, drains the copies it has in flight (bounded again) and
// returns.
#include <algorithm>

#include "common.cuh"
#include "tc_util.cuh"

namespace gdn {

constexpr int kDecMaxR = 4;                // v-heads per k-head served
constexpr int kDecMaxGroupsPerCta = 512;   // slot table of one CTA
constexpr uint32_t kDecSpin = 1u << 22;

template <int D>
struct DecCfg;
template <>
struct DecCfg<128> {
  static constexpr int NT = 256, NSTAGE = 3, CTAS = 1;
};
template <>
struct DecCfg<64> {
  static constexpr int NT = 128, NSTAGE = 6, CTAS = 2;
};

template <int D>
struct DecSmem {
  static constexpr int NT = DecCfg<D>::NT;
  static constexpr int RG = NT / (D / 4);   // rows per pass
  float state[DecCfg<D>::NSTAGE][D * D];    // the state ring (bulk-copy targets)
  float red[RG][D];
  float delta[D];
  float q[D], k[D];
  float v[kDecMaxR][D];
  float gate_g[kDecMaxR], gate_b[kDecMaxR];
  float norm[2];
  float wsum[NT / 32];
  int64_t slot[kDecMaxGroupsPerCta];
  uint64_t bar[DecCfg<D>::NSTAGE];
  int abort;
};

template <int D, int K>
__global__ void __launch_bounds__(DecCfg<D>::NT, DecCfg<D>::CTAS) decode_fused_kernel(
    const bf16* __restrict__ mixed, int64_t ms, const bf16* __restrict__ zp, int64_t zs,
    const bf16* __restrict__ bp, const bf16* __restrict__ ap, int64_t abs_,
    bf16* __restrict__ conv_pool, int64_t conv_ss, const bf16* __restrict__ conv_w,
    const void* __restrict__ a_log, const void* __restrict__ dt_bias, int param_f32,
    float* __restrict__ pool, int64_t slot_stride, int64_t num_slots,
    const int64_t* __restrict__ ids, const bf16* __restrict__ nw, float eps,
    bf16* __restrict__ out, int bs, int HK, int R, float scale, int32_t* status) {
  constexpr int NT = DecCfg<D>::NT;
  constexpr int NSTAGE = DecCfg<D>::NSTAGE;
  constexpr int CG = D / 4;         // threads across a state row (float4 each)
  constexpr int RG = NT / CG;       // rows per pass
  constexpr int RPT = D / RG;       // rows per thread
  constexpr int T = K - 1;          // conv taps kept in the state
  constexpr uint32_t kStateBytes = D * D * 4;
  static_assert(D <= NT && NT % CG == 0 && D % RG == 0, "bad tiling");

  extern __shared__ __align__(128) unsigned char dsmem[];
  DecSmem<D>& sm = *reinterpret_cast<DecSmem<D>*>(dsmem);

  const int tid = threadIdx.x;
  const int c4 = tid % CG;
  const int r0 = tid / CG;
  const int HV = HK * R;
  const int n_groups = bs * HK;
  const int my_groups =
      n_groups > (int)blockIdx.x ? (n_groups - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int n_units = my_groups * R;

  for (int i = tid; i < my_groups; i += NT) {
    const int G = blockIdx.x + i * gridDim.x;
    sm.slot[i] = ids[G / HK];
  }
  if (tid == 0) {
    for (int s = 0; s < NSTAGE; ++s) tc::mbar_init(tc::smem_u32(&sm.bar[s]), 1);
    tc::mbar_init_fence();
    sm.abort = 0;
  }
  __syncthreads();

  // Producer (thread 0): queue unit u's state copy into stage u % NSTAGE; a
  // unit whose slot is out of range completes the phase without a copy.
  auto issue = [&](int u) {
    const int gi = u / R, j = u - gi * R;
    const int G = blockIdx.x + gi * gridDim.x;
    const int hk = G % HK;
    const int64_t slot = sm.slot[gi];
    const uint32_t bar = tc::smem_u32(&sm.bar[u % NSTAGE]);
    if (slot >= 0 && slot < num_slots) {
      tc::mbar_expect_tx(bar, kStateBytes);
      tc::bulk_load(tc::smem_u32(sm.state[u % NSTAGE]),
                    pool + slot * slot_stride + (int64_t)(hk * R + j) * D * D, kStateBytes, bar);
    } else {
      tc::mbar_arrive(bar);
    }
  };
  if (tid == 0)
    for (int u = 0; u < NSTAGE && u < n_units; ++u) issue(u);

  const float wn = tid < D ? bf2f(nw[tid]) : 0.f;
  int consumed = 0;   // units whose stage has been waited for

  for (int gi = 0; gi < my_groups; ++gi) {
    const int G = blockIdx.x + gi * gridDim.x;
    const int b = G / HK;
    const int hk = G - b * HK;
    const int64_t slot = sm.slot[gi];
    const bool valid = slot >= 0 && slot < num_slots;
    if (!valid && tid == 0 && status) atomicOr(status, GDN_STATUS_BAD_SLOT);

    // ---- group prologue: conv step over q/k of head hk and v of its R heads,
    // conv-state roll, gates of the R heads, z of this thread's column ----
    float zv[kDecMaxR];
    if (valid) {
      const bf16* xrow = mixed + (int64_t)b * ms;
      if (tid < D) {
#pragma unroll
        for (int j = 0; j < kDecMaxR; ++j)
          zv[j] = j < R ? bf2f(zp[(int64_t)b * zs + (int64_t)(hk * R + j) * D + tid]) : 0.f;
      }
      const int n_pairs = (2 + R) * D / 2;
      for (int p = tid; p < n_pairs; p += NT) {
        const int c = 2 * p;   // group-local channel; pairs never straddle q/k/v
        int cg;
        float* dst;
        if (c < D) {
          cg = hk * D + c;
          dst = &sm.q[c];
        } else if (c < 2 * D) {
          cg = HK * D + hk * D + (c - D);
          dst = &sm.k[c - D];
        } else {
          cg = 2 * HK * D + hk * R * D + (c - 2 * D);
          dst = &sm.v[0][0] + (c - 2 * D);
        }
        union { uint32_t u; bf16 h[2]; } xu;
        union { uint32_t u[T]; bf16 h[2 * T]; } tu, nu;
        union { uint32_t u[K]; bf16 h[2 * K]; } wu;
        xu.u = *reinterpret_cast<const uint32_t*>(xrow + cg);
        uint32_t* tp = reinterpret_cast<uint32_t*>(conv_pool + slot * conv_ss + (int64_t)cg * T);
#pragma unroll
        for (int i = 0; i < T; ++i) tu.u[i] = tp[i];
#pragma unroll
        for (int i = 0; i < K; ++i)
          wu.u[i] = reinterpret_cast<const uint32_t*>(conv_w + (int64_t)cg * K)[i];
#pragma unroll
        for (int ch = 0; ch < 2; ++ch) {
          float win[K], wv[K];
#pragma unroll
          for (int i = 0; i < T; ++i) win[i] = bf2f(tu.h[ch * T + i]);
          win[T] = bf2f(xu.h[ch]);
#pragma unroll
          for (int i = 0; i < K; ++i) wv[i] = bf2f(wu.h[ch * K + i]);
          dst[ch] = round_bf(conv_point<K>(win, wv));   // the conv output is bf16
#pragma unroll
          for (int i = 0; i + 1 < T; ++i) nu.h[ch * T + i] = tu.h[ch * T + i + 1];
          nu.h[ch * T + T - 1] = xu.h[ch];
        }
#pragma unroll
        for (int i = 0; i < T; ++i) tp[i] = nu.u[i];
      }
      if (tid < R) {
        const int h = hk * R + tid;
        const float al = param_f32 ? reinterpret_cast<const float*>(a_log)[h]
                                   : bf2f(reinterpret_cast<const bf16*>(a_log)[h]);
        const float db = param_f32 ? reinterpret_cast<const float*>(dt_bias)[h]
                                   : bf2f(reinterpret_cast<const bf16*>(dt_bias)[h]);
        float gv, bt;
        gate_value(bf2f(ap[(int64_t)b * abs_ + h]), bf2f(bp[(int64_t)b * abs_ + h]), al, db, gv,
                   bt);
        sm.gate_g[tid] = gv;
        sm.gate_b[tid] = bt;
      }
    }
    __syncthreads();
    if (valid && tid < 32) {
      float aq = 0.f, ak = 0.f;
      for (int i = tid; i < D; i += 32) {
        aq += sm.q[i] * sm.q[i];
        ak += sm.k[i] * sm.k[i];
      }
      aq = warp_sum(aq);
      ak = warp_sum(ak);
      if (tid == 0) {
        sm.norm[0] = rsqrtf(aq + 1e-6f);
        sm.norm[1] = rsqrtf(ak + 1e-6f);
      }
    }
    __syncthreads();

    // ---- the R recurrence units of the group ----
    for (int j = 0; j < R; ++j) {
      const int u = gi * R + j;
      const int stage = u % NSTAGE;
      float4 s[RPT];
      if (!tc::mbar_wait(tc::smem_u32(&sm.bar[stage]), (uint32_t)(u / NSTAGE) & 1u, kDecSpin)) {
        sm.abort = 1;
        if (status) atomicOr(status, GDN_STATUS_TIMEOUT);
      }
      consumed = u + 1;
      if (valid) {
        const float* st = sm.state[stage] + 4 * c4;
#pragma unroll
        for (int i = 0; i < RPT; ++i)
          s[i] = *reinterpret_cast<const float4*>(st + (r0 + RG * i) * D);
      }
      __syncthreads();   // stage consumed by every thread; abort flag visible
      if (sm.abort) break;
      if (tid == 0 && u + NSTAGE < n_units) issue(u + NSTAGE);
      if (!valid) continue;

      const int h = hk * R + j;
      const float nq = sm.norm[0] * scale;
      const float nk = sm.norm[1];
      const float eg = expf(sm.gate_g[j]);
      const float bt = sm.gate_b[j];

      // S' = S * exp(g); partial (S'^T k^) over this thread's rows.
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int i = 0; i < RPT; ++i) {
        const float kk = sm.k[r0 + RG * i] * nk;
        s[i].x *= eg; s[i].y *= eg; s[i].z *= eg; s[i].w *= eg;
        acc.x += s[i].x * kk; acc.y += s[i].y * kk; acc.z += s[i].z * kk; acc.w += s[i].w * kk;
      }
      *reinterpret_cast<float4*>(&sm.red[r0][4 * c4]) = acc;
      __syncthreads();
      if (tid < D) {
        float kv = 0.f;
#pragma unroll
        for (int jj = 0; jj < RG; ++jj) kv += sm.red[jj][tid];
        sm.delta[tid] = (sm.v[j][tid] - kv) * bt;
      }
      __syncthreads();

      // S'' = S' + k^ (x) d, written back in place; partial (S''^T q^).
      float* sbase = pool + slot * slot_stride + (int64_t)h * D * D + 4 * c4;
      const float4 d = *reinterpret_cast<const float4*>(&sm.delta[4 * c4]);
      acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int i = 0; i < RPT; ++i) {
        const int r = r0 + RG * i;
        const float kk = sm.k[r] * nk;
        const float qq = sm.q[r] * nq;
        s[i].x += kk * d.x; s[i].y += kk * d.y; s[i].z += kk * d.z; s[i].w += kk * d.w;
        __stcs(reinterpret_cast<float4*>(sbase + (int64_t)r * D), s[i]);
        acc.x += s[i].x * qq; acc.y += s[i].y * qq; acc.z += s[i].z * qq; acc.w += s[i].w * qq;
      }
      *reinterpret_cast<float4*>(&sm.red[r0][4 * c4]) = acc;
      __syncthreads();

      // o = S''^T q^, then the gated RMSNorm of the row (bf16 core output first)
      float x = 0.f;
      if (tid < D) {
        float o = 0.f;
#pragma unroll
        for (int jj = 0; jj < RG; ++jj) o += sm.red[jj][tid];
        x = round_bf(o);
      }
      const float ss = warp_sum(x * x);
      if ((tid & 31) == 0) sm.wsum[tid >> 5] = ss;
      __syncthreads();
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < NT / 32; ++w) tot += sm.wsum[w];
      const float inv = rsqrtf(tot / (float)D + eps);
      if (tid < D) {
        float zz = 0.f;
#pragma unroll
        for (int jj = 0; jj < kDecMaxR; ++jj)
          if (jj == j) zz = zv[jj];
        out[((int64_t)b * HV + h) * D + tid] = f2bf(gated_norm_elem(x, inv, wn, zz));
      }
    }
    if (sm.abort) break;
  }

  if (sm.abort && tid == 0) {
    // drain the copies still in flight, bounded: the unit whose wait gave up
    // and those issued after it (a completed phase returns at once)
    const int issued = min(n_units, consumed - 1 + NSTAGE);
    for (int u = max(consumed - 1, 0); u < issued; ++u)
      tc::mbar_wait(tc::smem_u32(&sm.bar[u % NSTAGE]), (uint32_t)(u / NSTAGE) & 1u, kDecSpin);
  }
}

template <int D, int K>
static int launch_decode_fused(int grid, cudaStream_t s, const bf16* mixed, int64_t ms,
                               const bf16* z, int64_t zs, const bf16* b, const bf16* a,
                               int64_t abs_, bf16* conv_pool, int64_t conv_ss, const bf16* conv_w,
                               const void* a_log, const void* dt_bias, int param_f32, float* pool,
                               int64_t slot_stride, int64_t num_slots, const int64_t* ids,
                               const bf16* nw, float eps, bf16* out, int bs, int HK, int R,
                               float scale, int32_t* status) {
  const size_t smem = sizeof(DecSmem<D>);
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(
        decode_fused_kernel<D, K>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) {
      set_error("gdn_decode_fused: cannot reserve %zu bytes of shared memory: %s", smem,
                cudaGetErrorString(e));
      return GDN_ERR_CUDA;
    }
    configured[dev] = 1;
  }
  decode_fused_kernel<D, K><<<grid, DecCfg<D>::NT, smem, s>>>(
      mixed, ms, z, zs, b, a, abs_, conv_pool, conv_ss, conv_w, a_log, dt_bias, param_f32, pool,
      slot_stride, num_slots, ids, nw, eps, out, bs, HK, R, scale, status);
  return check_launch("gdn_decode_fused");
}

}  // namespace gdn

using namespace gdn;

extern "C" int gdn_decode_fused(const void* mixed, int64_t mixed_row_stride, const void* z,
                                int64_t z_row_stride, const void* b, const void* a,
                                int64_t ab_row_stride, void* conv_pool, int64_t conv_slot_stride,
                                const void* conv_weight, int32_t conv_kernel, const void* a_log,
                                const void* dt_bias, int32_t param_dtype, float* s_pool,
                                int64_t slot_stride, int64_t num_slots, const int64_t* ids,
                                const void* norm_weight, float norm_eps, void* out, int32_t bs,
                                int32_t num_k_heads, int32_t num_v_heads, int32_t head_dim,
                                float scale, int32_t* status, void* stream) {
  clear_error();
  GDN_REQUIRE(bs >= 0 && num_k_heads > 0 && num_v_heads > 0,
              "gdn_decode_fused: bad sizes (bs=%d, HK=%d, HV=%d)", bs, num_k_heads, num_v_heads);
  GDN_REQUIRE(num_v_heads % num_k_heads == 0,
              "gdn_decode_fused: num_v_heads %d not a multiple of num_k_heads %d", num_v_heads,
              num_k_heads);
  const int R = num_v_heads / num_k_heads;
  GDN_UNSUPPORTED(head_dim == 128 || head_dim == 64, "gdn_decode_fused: head dim %d unsupported",
                  head_dim);
  GDN_UNSUPPORTED(R <= kDecMaxR, "gdn_decode_fused: %d v-heads per k-head (max %d)", R, kDecMaxR);
  GDN_UNSUPPORTED(conv_kernel >= 2 && conv_kernel <= 4,
                  "gdn_decode_fused: conv kernel %d unsupported (2..4)", conv_kernel);
  GDN_REQUIRE(param_dtype == GDN_DTYPE_F32 || param_dtype == GDN_DTYPE_BF16,
              "gdn_decode_fused: param_dtype must be GDN_DTYPE_F32 or GDN_DTYPE_BF16");
  const int64_t conv_dim = (int64_t)(2 * num_k_heads + num_v_heads) * head_dim;
  const int64_t value_dim = (int64_t)num_v_heads * head_dim;
  GDN_REQUIRE(mixed_row_stride >= conv_dim && z_row_stride >= value_dim &&
                  ab_row_stride >= num_v_heads,
              "gdn_decode_fused: a row stride is smaller than the row it holds");
  GDN_REQUIRE(num_slots > 0 && slot_stride >= value_dim * head_dim && slot_stride % 4 == 0,
              "gdn_decode_fused: slot_stride %lld must be >= HV*D*D and a multiple of 4",
              (long long)slot_stride);
  GDN_REQUIRE(conv_slot_stride >= conv_dim * (conv_kernel - 1),
              "gdn_decode_fused: conv_slot_stride %lld < conv_dim*(K-1)",
              (long long)conv_slot_stride);
  if (bs == 0) return GDN_OK;
  GDN_REQUIRE(mixed && z && b && a && conv_pool && conv_weight && a_log && dt_bias && s_pool &&
                  ids && norm_weight && out,
              "gdn_decode_fused: null pointer");
  GDN_UNSUPPORTED(aligned16(s_pool) && ((uintptr_t)mixed % 4) == 0 && mixed_row_stride % 2 == 0 &&
                      ((uintptr_t)conv_pool % 4) == 0 && conv_slot_stride % 2 == 0 &&
                      ((uintptr_t)conv_weight % 4) == 0,
                  "gdn_decode_fused: s_pool must be 16-byte aligned; mixed rows, conv pool "
                  "slots and conv weight 4-byte aligned");
  const int64_t groups = (int64_t)bs * num_k_heads;
  GDN_UNSUPPORTED(groups < (1ll << 30), "gdn_decode_fused: too many rows");
  const int ctas = head_dim == 128 ? DecCfg<128>::CTAS : DecCfg<64>::CTAS;
  int64_t grid = std::min<int64_t>(groups, (int64_t)sm_count() * ctas);
  const int64_t need = (groups + kDecMaxGroupsPerCta - 1) / kDecMaxGroupsPerCta;
  if (grid < need) grid = need;
  cudaStream_t s = (cudaStream_t)stream;
  const int pf = param_dtype == GDN_DTYPE_F32;
#define GDN_DF(DD, KK)                                                                          \
  if (head_dim == DD && conv_kernel == KK)                                                      \
    return launch_decode_fused<DD, KK>(                                                         \
        (int)grid, s, (const bf16*)mixed, mixed_row_stride, (const bf16*)z, z_row_stride,       \
        (const bf16*)b, (const bf16*)a, ab_row_stride, (bf16*)conv_pool, conv_slot_stride,      \
        (const bf16*)conv_weight, a_log, dt_bias, pf, s_pool, slot_stride, num_slots, ids,      \
        (const bf16*)norm_weight, norm_eps, (bf16*)out, bs, num_k_heads, R, scale, status);
  GDN_DF(128, 4) GDN_DF(128, 3) GDN_DF(128, 2) GDN_DF(64, 4) GDN_DF(64, 3) GDN_DF(64, 2)
#undef GDN_DF
  set_error("gdn_decode_fused: unsupported configuration");
  return GDN_ERR_UNSUPPORTED;
}
