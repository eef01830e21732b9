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
// Work items and race freedom.  A CTA owns whole k-head groups (b, hk): the
// R = HV / HK v-heads that share q/k head hk.  The group's conv channels
// (q and k of head hk, v of its R heads) are convolved and their conv state
// rolled once, by that CTA, before its recurrence units run, so no other CTA
// reads a conv state this one rewrites.
//
// HBM pipeline.  The kernel is persistent (2 CTAs per SM at D = 128, 4 at
// D = 64; 16 warps per SM either way).  A recurrence unit is one 64-column
// part of a head's D x D fp32 state; each CTA streams its units through a
// 3-deep ring of shared-memory tiles loaded by TMA (a [D rows x 64 columns]
// box of the per-layer pool view, completing on an mbarrier), so while a unit
// computes, the next two are in flight.  New state columns go back from
// registers with streaming stores.  The next group's conv inputs, gates and z
// are fetched into registers while the current group runs.
//
// Bit-identical results.  Threads own rows r0 + RG*i of VW adjacent columns,
// RG = 8: the column sums run in the row order of recurrent_inplace's
// full-tile kernels, and the conv, gate and norm formulas are the same device
// functions, so the output and the states equal conv_decode_step +
// fused_g_beta + recurrent_inplace (gated norm fused) bit for bit wherever
// that sequence runs its full-tile recurrent kernel.
//
// Every mbarrier wait is bounded: on time-out the CTA raises
// GDN_STATUS_TIMEOUT, drains the copies it has in flight (bounded again) and
// returns.
#include <algorithm>
#include <atomic>

#include <mutex>

#include "common.cuh"
#include "tc_util.cuh"
#include "tmap.cuh"

namespace gdn {

constexpr int kDecMaxR = 4;                // v-heads per k-head served
constexpr int kDecMaxGroupsPerCta = 256;   // slot table of one CTA
constexpr int kDecPartCols = 64;           // state columns per recurrence unit
constexpr uint32_t kDecSpin = 1u << 22;

template <int D>
struct DecCfg;
template <>
struct DecCfg<128> {
  static constexpr int NT = 256, VW = 2, NSTAGE = 3, CTAS = 2;
};
template <>
struct DecCfg<64> {
  static constexpr int NT = 128, VW = 4, NSTAGE = 3, CTAS = 4;
};

template <int D>
struct DecSmem {
  static constexpr int NT = DecCfg<D>::NT;
  static constexpr int RG = NT / (kDecPartCols / DecCfg<D>::VW);   // rows per pass
  float state[DecCfg<D>::NSTAGE][D * kDecPartCols];   // TMA boxes [D rows][64 cols]
  float red[RG][kDecPartCols];
  float delta[kDecPartCols];
  float q[D], k[D];
  float v[kDecMaxR][D];
  float o[D];                       // the head's core output, before the norm
  // k^ and q^ of the rows each thread owns (rows r0 + RG*i), contiguous per r0
  __align__(16) float kn[RG][D / RG];
  __align__(16) float qn[RG][D / RG];
  float gate_g[kDecMaxR], gate_b[kDecMaxR];
  float wsum[NT / 32];
  int64_t slot[kDecMaxGroupsPerCta];
  uint64_t bar[DecCfg<D>::NSTAGE];
  int abort;
};

// A vector of VW fp32 state columns.
template <int VW>
struct Vec;
template <>
struct Vec<2> {
  float2 v;
  __device__ __forceinline__ float& operator[](int i) { return i == 0 ? v.x : v.y; }
};
template <>
struct Vec<4> {
  float4 v;
  __device__ __forceinline__ float& operator[](int i) {
    return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
  }
};

// The next group's conv inputs, gate inputs and z, held in registers.
template <int K>
struct GroupIn {
  uint32_t x[2];             // two channel pairs per thread at most
  uint32_t taps[2][K - 1];
  uint32_t w[2][K];
  float z[kDecMaxR];         // column tid of each head's z (tid < D)
  float av, bv, al, db;      // a, b, A_log, dt_bias of head tid (tid < R)
};

template <int D, int K>
__global__ void __launch_bounds__(DecCfg<D>::NT, DecCfg<D>::CTAS) decode_fused_kernel(
    const __grid_constant__ CUtensorMap tm_state, const bf16* __restrict__ mixed, int64_t ms,
    const bf16* __restrict__ zp, int64_t zs, const bf16* __restrict__ bp,
    const bf16* __restrict__ ap, int64_t abs_, bf16* __restrict__ conv_pool, int64_t conv_ss,
    const bf16* __restrict__ conv_w, const void* __restrict__ a_log,
    const void* __restrict__ dt_bias, int param_f32, float* __restrict__ pool,
    int64_t slot_stride, int64_t num_slots, const int64_t* __restrict__ ids,
    const bf16* __restrict__ nw, float eps, bf16* __restrict__ out, int bs, int HK, int R,
    float scale, int32_t* status) {
  constexpr int NT = DecCfg<D>::NT;
  constexpr int VW = DecCfg<D>::VW;
  constexpr int NSTAGE = DecCfg<D>::NSTAGE;
  constexpr int PARTS = D / kDecPartCols;
  constexpr int CG = kDecPartCols / VW;   // threads across a part's row
  constexpr int RG = NT / CG;             // rows per pass (8)
  constexpr int RPT = D / RG;             // rows per thread
  constexpr int T = K - 1;                // conv taps kept in the state
  constexpr int MAXP = 2;                 // channel pairs per thread
  constexpr uint32_t kUnitBytes = D * kDecPartCols * 4;
  static_assert(RG == 8 && D <= NT && NT % CG == 0 && D % RG == 0, "bad tiling");
  static_assert((2 + kDecMaxR) * D / 2 <= MAXP * NT, "channel pairs per thread");

  extern __shared__ __align__(16) unsigned char dsmem[];
  // TMA tiles want 128-byte aligned shared memory: round the base up (the
  // launch reserves 128 bytes of slack)
  DecSmem<D>& sm = *reinterpret_cast<DecSmem<D>*>(
      dsmem + ((128u - (tc::smem_u32(dsmem) & 127u)) & 127u));

  const int tid = threadIdx.x;
  const int c4 = tid % CG;
  const int r0 = tid / CG;
  const int HV = HK * R;
  const int n_groups = bs * HK;
  const int my_groups =
      n_groups > (int)blockIdx.x ? (n_groups - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int units_per_group = R * PARTS;
  const int n_units = my_groups * units_per_group;
  const int64_t rows_per_slot = slot_stride / D;   // TMA row coordinate of a slot

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

  // Producer (thread 0): queue unit u's state tile into stage u % NSTAGE; a
  // unit whose slot is out of range completes the phase without a copy.
  auto issue = [&](int u) {
    const int gi = u / units_per_group;
    const int rem = u - gi * units_per_group;
    const int j = rem / PARTS, part = rem - j * PARTS;
    const int G = blockIdx.x + gi * gridDim.x;
    const int hk = G % HK;
    const int64_t slot = sm.slot[gi];
    const uint32_t bar = tc::smem_u32(&sm.bar[u % NSTAGE]);
    if (slot >= 0 && slot < num_slots) {
      tc::mbar_expect_tx(bar, kUnitBytes);
      tc::tma_load_2d(tc::smem_u32(sm.state[u % NSTAGE]), &tm_state, part * kDecPartCols,
                      (int)(slot * rows_per_slot + (int64_t)(hk * R + j) * D), bar);
    } else {
      tc::mbar_arrive(bar);
    }
  };
  if (tid == 0)
    for (int u = 0; u < NSTAGE && u < n_units; ++u) issue(u);

  // Fetch group gi's inputs into registers (plain loads, consumed a group later).
  const int n_pairs = (2 + R) * D / 2;
  auto fetch = [&](int gi, GroupIn<K>& in) {
    const int G = blockIdx.x + gi * gridDim.x;
    const int b = G / HK;
    const int hk = G - b * HK;
    const int64_t slot = sm.slot[gi];
    if (!(slot >= 0 && slot < num_slots)) return;
    const bf16* xrow = mixed + (int64_t)b * ms;
#pragma unroll
    for (int pi = 0; pi < MAXP; ++pi) {
      const int p = tid + pi * NT;
      if (p < n_pairs) {
        const int c = 2 * p;
        const int cg = c < D ? hk * D + c
                             : (c < 2 * D ? HK * D + hk * D + (c - D)
                                          : 2 * HK * D + hk * R * D + (c - 2 * D));
        in.x[pi] = *reinterpret_cast<const uint32_t*>(xrow + cg);
        const uint32_t* tp =
            reinterpret_cast<const uint32_t*>(conv_pool + slot * conv_ss + (int64_t)cg * T);
#pragma unroll
        for (int i = 0; i < T; ++i) in.taps[pi][i] = tp[i];
        const uint32_t* wp = reinterpret_cast<const uint32_t*>(conv_w + (int64_t)cg * K);
#pragma unroll
        for (int i = 0; i < K; ++i) in.w[pi][i] = wp[i];
      }
    }
    if (tid < D) {
#pragma unroll
      for (int j = 0; j < kDecMaxR; ++j)
        in.z[j] = j < R ? bf2f(zp[(int64_t)b * zs + (int64_t)(hk * R + j) * D + tid]) : 0.f;
    }
    if (tid < R) {
      const int h = hk * R + tid;
      in.av = bf2f(ap[(int64_t)b * abs_ + h]);
      in.bv = bf2f(bp[(int64_t)b * abs_ + h]);
      in.al = param_f32 ? reinterpret_cast<const float*>(a_log)[h]
                        : bf2f(reinterpret_cast<const bf16*>(a_log)[h]);
      in.db = param_f32 ? reinterpret_cast<const float*>(dt_bias)[h]
                        : bf2f(reinterpret_cast<const bf16*>(dt_bias)[h]);
    }
  };

  const float wn = tid < D ? bf2f(nw[tid]) : 0.f;
  const int lane = tid & 31;
  GroupIn<K> cur;
  if (my_groups > 0) fetch(0, cur);
  int consumed = 0;   // units whose stage has been waited for

  // The gated RMSNorm of a finished head runs inside the next unit, on that
  // unit's barriers: its sum of squares after the stage barrier, the scaled
  // output after the first reduction barrier.  pend marks such a head, prow
  // its output row, pz this thread's z value of it.
  bool pend = false;
  int64_t prow = 0;
  float pz = 0.f;
  auto norm_store = [&](float x, float inv) {
    if (tid < D) out[prow * D + tid] = f2bf(gated_norm_elem(x, inv, wn, pz));
  };
  auto norm_sumsq = [&](float& x) {
    x = tid < D ? round_bf(sm.o[tid]) : 0.f;   // the core output is bf16 first
    const float ss = warp_sum(x * x);
    if (lane == 0) sm.wsum[tid >> 5] = ss;
  };
  auto norm_inv = [&]() {
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < NT / 32; ++w) tot += sm.wsum[w];
    return rsqrtf(tot / (float)D + eps);
  };

  for (int gi = 0; gi < my_groups; ++gi) {
    const int G = blockIdx.x + gi * gridDim.x;
    const int b = G / HK;
    const int hk = G - b * HK;
    const int64_t slot = sm.slot[gi];
    const bool valid = slot >= 0 && slot < num_slots;
    if (!valid && tid == 0 && status) atomicOr(status, GDN_STATUS_BAD_SLOT);

    // ---- group prologue: conv step over q/k of head hk and v of its R heads
    // (from the prefetched registers), conv-state roll, gates ----
    float zv[kDecMaxR];
    if (valid) {
#pragma unroll
      for (int j = 0; j < kDecMaxR; ++j) zv[j] = cur.z[j];
#pragma unroll
      for (int pi = 0; pi < MAXP; ++pi) {
        const int p = tid + pi * NT;
        if (p < n_pairs) {
          const int c = 2 * p;
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
          xu.u = cur.x[pi];
#pragma unroll
          for (int i = 0; i < T; ++i) tu.u[i] = cur.taps[pi][i];
#pragma unroll
          for (int i = 0; i < K; ++i) wu.u[i] = cur.w[pi][i];
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
          uint32_t* tp =
              reinterpret_cast<uint32_t*>(conv_pool + slot * conv_ss + (int64_t)cg * T);
#pragma unroll
          for (int i = 0; i < T; ++i) tp[i] = nu.u[i];
        }
      }
      if (tid < R) {
        float gv, bt;
        gate_value(cur.av, cur.bv, cur.al, cur.db, gv, bt);
        sm.gate_g[tid] = gv;
        sm.gate_b[tid] = bt;
      }
    }
    if (gi + 1 < my_groups) fetch(gi + 1, cur);   // in flight during this group's units
    __syncthreads();
    // l2 norms of q and k: every warp computes them, identically (the same
    // sums in the same order), so no second barrier is needed
    if (valid) {
      float aq = 0.f, ak = 0.f;
      for (int i = lane; i < D; i += 32) {
        aq += sm.q[i] * sm.q[i];
        ak += sm.k[i] * sm.k[i];
      }
      aq = warp_sum(aq);
      ak = warp_sum(ak);
      const float nq = rsqrtf(aq + 1e-6f) * scale;
      const float nk = rsqrtf(ak + 1e-6f);
      // this warp's rows: 32/CG row sets of RPT rows = 16 entries; lanes 0-15
      // scale k, lanes 16-31 scale q
      const int e = lane & 15;
      const int rr = (tid >> 5) * (32 / CG) + e / RPT;
      const int row = rr + RG * (e % RPT);
      if (lane < 16) sm.kn[rr][e % RPT] = sm.k[row] * nk;
      else sm.qn[rr][e % RPT] = sm.q[row] * nq;
      __syncwarp();
    }

    // ---- the group's recurrence units: R heads x PARTS column parts ----
    for (int j = 0; j < R; ++j) {
      const int h = hk * R + j;
      for (int part = 0; part < PARTS; ++part) {
        const int u = gi * units_per_group + j * PARTS + part;
        const int stage = u % NSTAGE;
        Vec<VW> s[RPT];
        if (!tc::mbar_wait(tc::smem_u32(&sm.bar[stage]), (uint32_t)(u / NSTAGE) & 1u,
                           kDecSpin)) {
          sm.abort = 1;
          if (status) atomicOr(status, GDN_STATUS_TIMEOUT);
        }
        consumed = u + 1;
        if (valid) {
          const float* st = sm.state[stage] + VW * c4;
#pragma unroll
          for (int i = 0; i < RPT; ++i) {
            if constexpr (VW == 2)
              s[i].v = *reinterpret_cast<const float2*>(st + (r0 + RG * i) * kDecPartCols);
            else
              s[i].v = *reinterpret_cast<const float4*>(st + (r0 + RG * i) * kDecPartCols);
          }
        }
        __syncthreads();   // stage consumed by every thread; abort flag visible
        if (sm.abort) break;
        if (tid == 0 && u + NSTAGE < n_units) issue(u + NSTAGE);
        if (!valid) continue;
        float px = 0.f;
        if (pend) norm_sumsq(px);   // the previous head's norm, first half

        const float eg = expf(sm.gate_g[j]);
        const float bt = sm.gate_b[j];
        const int col0 = part * kDecPartCols;

        // S' = S * exp(g); partial (S'^T k^) over this thread's rows.
        float kn[RPT];
#pragma unroll
        for (int i = 0; i < RPT; i += 4)
          *reinterpret_cast<float4*>(&kn[i]) = *reinterpret_cast<const float4*>(&sm.kn[r0][i]);
        Vec<VW> acc;
#pragma unroll
        for (int e = 0; e < VW; ++e) acc[e] = 0.f;
#pragma unroll
        for (int i = 0; i < RPT; ++i) {
          const float kk = kn[i];
#pragma unroll
          for (int e = 0; e < VW; ++e) {
            s[i][e] *= eg;
            acc[e] += s[i][e] * kk;
          }
        }
#pragma unroll
        for (int e = 0; e < VW; ++e) sm.red[r0][VW * c4 + e] = acc[e];
        __syncthreads();
        if (pend) {                 // the previous head's norm, second half
          norm_store(px, norm_inv());
          pend = false;
        }
        if (tid < kDecPartCols) {
          float kv = 0.f;
#pragma unroll
          for (int jj = 0; jj < RG; ++jj) kv += sm.red[jj][tid];
          sm.delta[tid] = (sm.v[j][col0 + tid] - kv) * bt;
        }
        __syncthreads();

        // S'' = S' + k^ (x) d, written back in place; partial (S''^T q^).
        float* sbase = pool + slot * slot_stride + (int64_t)h * D * D + col0 + VW * c4;
        float d[VW];
#pragma unroll
        for (int e = 0; e < VW; ++e) d[e] = sm.delta[VW * c4 + e];
#pragma unroll
        for (int e = 0; e < VW; ++e) acc[e] = 0.f;
        float qn[RPT];
#pragma unroll
        for (int i = 0; i < RPT; i += 4)
          *reinterpret_cast<float4*>(&qn[i]) = *reinterpret_cast<const float4*>(&sm.qn[r0][i]);
#pragma unroll
        for (int i = 0; i < RPT; ++i) {
          const int r = r0 + RG * i;
          const float kk = kn[i];
          const float qq = qn[i];
#pragma unroll
          for (int e = 0; e < VW; ++e) s[i][e] += kk * d[e];
          if constexpr (VW == 2)
            __stcs(reinterpret_cast<float2*>(sbase + (int64_t)r * D), s[i].v);
          else
            __stcs(reinterpret_cast<float4*>(sbase + (int64_t)r * D), s[i].v);
#pragma unroll
          for (int e = 0; e < VW; ++e) acc[e] += s[i][e] * qq;
        }
#pragma unroll
        for (int e = 0; e < VW; ++e) sm.red[r0][VW * c4 + e] = acc[e];
        __syncthreads();
        if (tid < kDecPartCols) {
          float o = 0.f;
#pragma unroll
          for (int jj = 0; jj < RG; ++jj) o += sm.red[jj][tid];
          sm.o[col0 + tid] = o;
        }
      }
      if (sm.abort) break;
      if (!valid) continue;

      // The head's gated RMSNorm: deferred into the next unit when that unit
      // runs (it is valid), else done here on two barriers of its own.
      pend = true;
      prow = (int64_t)b * HV + h;
#pragma unroll
      for (int jj = 0; jj < kDecMaxR; ++jj)
        if (jj == j) pz = zv[jj];
      const bool next_runs =
          j + 1 < R || (gi + 1 < my_groups && sm.slot[gi + 1] >= 0 &&
                        sm.slot[gi + 1] < num_slots);
      if (!next_runs) {
        __syncthreads();
        float x;
        norm_sumsq(x);
        __syncthreads();
        norm_store(x, norm_inv());
        pend = false;
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

// ---------------------------------------------------------------------------
// Head-per-CTA form (the caller passes per-group counters).  One CTA per
// (sequence, v-head) unit: thread 0 brings the head's whole D x D fp32 state
// into shared memory with one 1-D bulk copy at the start, the conv step, gate
// and z are computed while it streams in, and both recurrence passes read the
// state from shared memory, so a thread holds no state in registers and three
// CTAs (3 x 64 KiB in flight) share an SM: measured on B200, this streams a
// read+write of the pool at 6.8 TB/s, where a persistent ring of tiles
// streams at 6.2.  The q/k conv channels of k-head hk are read by the R CTAs
// of its v-heads; the last of them to finish reading (a per-group counter,
// incremented after the reads and reset by that last CTA) writes their
// rolled state.  Reduction orders and formulas as decode_fused_kernel.
// ---------------------------------------------------------------------------
template <int D>
struct HeadCfg;
template <>
struct HeadCfg<128> {
  static constexpr int NT = 256, CTAS = 3;
};
template <>
struct HeadCfg<64> {
  static constexpr int NT = 128, CTAS = 6;
};

template <int D>
struct HeadSmem {
  static constexpr int NT = HeadCfg<D>::NT;
  static constexpr int RG = NT / (D / 4);   // rows per pass
  float state[D * D];                       // the bulk-copy target
  float red[RG][D];
  float delta[D];
  float q[D], k[D], v[D];
  float wsum[NT / 32];
  float gate_g, gate_b;
  uint64_t bar;
  int last, abort;
};

template <int D, int K>
__global__ void __launch_bounds__(HeadCfg<D>::NT) decode_head_kernel(
    const bf16* __restrict__ mixed, int64_t ms, const bf16* __restrict__ zp, int64_t zs,
    const bf16* __restrict__ bp, const bf16* __restrict__ ap, int64_t abs_,
    bf16* __restrict__ conv_pool, int64_t conv_ss, const bf16* __restrict__ conv_w,
    const void* __restrict__ a_log, const void* __restrict__ dt_bias, int param_f32,
    float* __restrict__ pool, int64_t slot_stride, int64_t num_slots,
    const int64_t* __restrict__ ids, const bf16* __restrict__ nw, float eps,
    bf16* __restrict__ out, int HK, int R, float scale, int32_t* __restrict__ group_cnt,
    int32_t* status, uint32_t state_spin) {
  constexpr int NT = HeadCfg<D>::NT;
  constexpr int CG = D / 4;         // threads across a state row (float4 each)
  constexpr int RG = NT / CG;       // rows per pass
  constexpr int RPT = D / RG;       // rows per thread
  constexpr int T = K - 1;
  constexpr uint32_t kStateBytes = D * D * 4;
  static_assert(RG == 8 && 3 * D / 2 <= NT, "bad tiling");

  extern __shared__ __align__(16) unsigned char dsmem[];
  HeadSmem<D>& sm = *reinterpret_cast<HeadSmem<D>*>(
      dsmem + ((128u - (tc::smem_u32(dsmem) & 127u)) & 127u));

  const int tid = threadIdx.x, lane = tid & 31;
  const int c4 = tid % CG, r0 = tid / CG;
  const int HV = HK * R;
  const int b = blockIdx.x / HV;
  const int h = blockIdx.x - b * HV;
  const int hk = h / R;
  const int64_t slot = ids[b];
  if (!slot_ok(slot, num_slots, status)) return;   // the whole CTA: same row
  float* gstate = pool + slot * slot_stride + (int64_t)h * D * D;
  const uint32_t bar = tc::smem_u32(&sm.bar);
  if (tid == 0) {
    tc::mbar_init(bar, 1);
    tc::mbar_init_fence();
    tc::mbar_expect_tx(bar, kStateBytes);
    tc::bulk_load(tc::smem_u32(sm.state), gstate, kStateBytes, bar);
    sm.abort = 0;
  }

  // ---- conv step over this head's q, k (head hk) and v (head h) channels ----
  const bf16* xrow = mixed + (int64_t)b * ms;
  const int p = tid;                 // channel pair of this thread
  const bool has_pair = p < 3 * D / 2;
  const int c = 2 * p;
  const int seg = c / D;             // 0 q, 1 k, 2 v
  const int cc = c - seg * D;
  const int cg = seg == 0 ? hk * D + cc : (seg == 1 ? HK * D + hk * D + cc
                                                    : 2 * HK * D + h * D + cc);
  union { uint32_t u[T]; bf16 h[2 * T]; } nu;   // the rolled taps of the pair
  uint32_t* tp = reinterpret_cast<uint32_t*>(conv_pool + slot * conv_ss + (int64_t)cg * T);
  float zv = 0.f, av = 0.f, bv = 0.f, al = 0.f, db = 0.f;
  if (tid < D) zv = bf2f(zp[(int64_t)b * zs + (int64_t)h * D + tid]);
  if (tid == 0) {
    av = bf2f(ap[(int64_t)b * abs_ + h]);
    bv = bf2f(bp[(int64_t)b * abs_ + h]);
    al = param_f32 ? reinterpret_cast<const float*>(a_log)[h]
                   : bf2f(reinterpret_cast<const bf16*>(a_log)[h]);
    db = param_f32 ? reinterpret_cast<const float*>(dt_bias)[h]
                   : bf2f(reinterpret_cast<const bf16*>(dt_bias)[h]);
  }
  if (has_pair) {
    union { uint32_t u; bf16 h[2]; } xu;
    union { uint32_t u[T]; bf16 h[2 * T]; } tu;
    union { uint32_t u[K]; bf16 h[2 * K]; } wu;
    xu.u = *reinterpret_cast<const uint32_t*>(xrow + cg);
#pragma unroll
    for (int i = 0; i < T; ++i) tu.u[i] = tp[i];
#pragma unroll
    for (int i = 0; i < K; ++i)
      wu.u[i] = reinterpret_cast<const uint32_t*>(conv_w + (int64_t)cg * K)[i];
    float* dst = seg == 0 ? &sm.q[cc] : (seg == 1 ? &sm.k[cc] : &sm.v[cc]);
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
    if (seg == 2) {   // this head's own v channels: roll now
#pragma unroll
      for (int i = 0; i < T; ++i) tp[i] = nu.u[i];
    }
  }
  if (tid == 0) {
    float gv, bt;
    gate_value(av, bv, al, db, gv, bt);
    sm.gate_g = gv;
    sm.gate_b = bt;
  }
  __threadfence();   // this CTA's q/k tap reads are done before its counter bump
  __syncthreads();
  if (tid == 0) {
    int last = 1;
    if (R > 1) {
      const int G = b * HK + hk;
      last = atomicAdd(&group_cnt[G], 1) == R - 1;
      if (last) group_cnt[G] = 0;   // every reader of the group has counted
      __threadfence();
    }
    sm.last = last;
  }
  __syncthreads();
  if (sm.last && has_pair && seg < 2) {   // the group's last reader rolls q and k
#pragma unroll
    for (int i = 0; i < T; ++i) tp[i] = nu.u[i];
  }

  // l2 norms of q and k: every warp computes them identically
  float aq = 0.f, ak = 0.f;
  for (int i = lane; i < D; i += 32) {
    aq += sm.q[i] * sm.q[i];
    ak += sm.k[i] * sm.k[i];
  }
  aq = warp_sum(aq);
  ak = warp_sum(ak);
  const float nq = rsqrtf(aq + 1e-6f) * scale;
  const float nk = rsqrtf(ak + 1e-6f);
  const float eg = expf(sm.gate_g);
  const float bt = sm.gate_b;

  // ---- the state has arrived (bounded wait; state_spin polls, kDecSpin unless a
  // test lowered it through gdn_set_wait_limit) ----
  if (!tc::mbar_wait(bar, 0, state_spin)) {
    sm.abort = 1;
    if (status) atomicOr(status, GDN_STATUS_TIMEOUT);
  }
  __syncthreads();
  if (sm.abort) {
    if (tid == 0) tc::mbar_wait(bar, 0, kDecSpin);   // the copy may still land: wait, bounded
    return;
  }

  // S' = S * exp(g); partial (S'^T k^) over this thread's rows.
  const float* st = sm.state + 4 * c4;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const float kk = sm.k[r0 + RG * i] * nk;
    float4 sv = *reinterpret_cast<const float4*>(st + (r0 + RG * i) * D);
    sv.x *= eg; sv.y *= eg; sv.z *= eg; sv.w *= eg;
    acc.x += sv.x * kk; acc.y += sv.y * kk; acc.z += sv.z * kk; acc.w += sv.w * kk;
  }
  *reinterpret_cast<float4*>(&sm.red[r0][4 * c4]) = acc;
  __syncthreads();
  if (tid < D) {
    float kv = 0.f;
#pragma unroll
    for (int jj = 0; jj < RG; ++jj) kv += sm.red[jj][tid];
    sm.delta[tid] = (sm.v[tid] - kv) * bt;
  }
  __syncthreads();

  // S'' = S' + k^ (x) d, written back in place; partial (S''^T q^).
  float* sbase = gstate + 4 * c4;
  const float4 d = *reinterpret_cast<const float4*>(&sm.delta[4 * c4]);
  acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int r = r0 + RG * i;
    const float kk = sm.k[r] * nk;
    const float qq = sm.q[r] * nq;
    float4 sv = *reinterpret_cast<const float4*>(st + r * D);
    sv.x *= eg; sv.y *= eg; sv.z *= eg; sv.w *= eg;
    sv.x += kk * d.x; sv.y += kk * d.y; sv.z += kk * d.z; sv.w += kk * d.w;
    __stcs(reinterpret_cast<float4*>(sbase + (int64_t)r * D), sv);
    acc.x += sv.x * qq; acc.y += sv.y * qq; acc.z += sv.z * qq; acc.w += sv.w * qq;
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
  if (lane == 0) sm.wsum[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < NT / 32; ++w) tot += sm.wsum[w];
  const float inv = rsqrtf(tot / (float)D + eps);
  if (tid < D) out[((int64_t)b * HV + h) * D + tid] = f2bf(gated_norm_elem(x, inv, bf2f(nw[tid]), zv));
}

template <int D, int K>
static int launch_decode_head(int64_t units, cudaStream_t s, const bf16* mixed, int64_t ms,
                              const bf16* z, int64_t zs, const bf16* b, const bf16* a,
                              int64_t abs_, bf16* conv_pool, int64_t conv_ss, const bf16* conv_w,
                              const void* a_log, const void* dt_bias, int param_f32, float* pool,
                              int64_t slot_stride, int64_t num_slots, const int64_t* ids,
                              const bf16* nw, float eps, bf16* out, int HK, int R, float scale,
                              int32_t* group_cnt, int32_t* status) {
  const size_t smem = sizeof(HeadSmem<D>) + 128;   // + alignment slack
  static_assert(HeadCfg<D>::CTAS * (sizeof(HeadSmem<D>) + 128 + 1024) <= 228 * 1024,
                "the CTAs per SM must fit the shared memory");
  static std::atomic<int> configured[64];   // concurrent first calls set the same limit
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev].load(std::memory_order_relaxed)) {
    const cudaError_t e = cudaFuncSetAttribute(
        decode_head_kernel<D, K>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) {
      set_error("gdn_decode_fused: cannot reserve %zu bytes of shared memory: %s", smem,
                cudaGetErrorString(e));
      return GDN_ERR_CUDA;
    }
    if (dev >= 0 && dev < 64) configured[dev].store(1, std::memory_order_relaxed);
  }
  decode_head_kernel<D, K><<<(unsigned)units, HeadCfg<D>::NT, smem, s>>>(
      mixed, ms, z, zs, b, a, abs_, conv_pool, conv_ss, conv_w, a_log, dt_bias, param_f32, pool,
      slot_stride, num_slots, ids, nw, eps, out, HK, R, scale, group_cnt, status,
      wait_limit(kDecSpin));
  return check_launch("gdn_decode_fused");
}

template <int D, int K>
static int launch_decode_fused(int grid, cudaStream_t s, const CUtensorMap& tm,
                               const bf16* mixed, int64_t ms, const bf16* z, int64_t zs,
                               const bf16* b, const bf16* a, int64_t abs_, bf16* conv_pool,
                               int64_t conv_ss, const bf16* conv_w, const void* a_log,
                               const void* dt_bias, int param_f32, float* pool,
                               int64_t slot_stride, int64_t num_slots, const int64_t* ids,
                               const bf16* nw, float eps, bf16* out, int bs, int HK, int R,
                               float scale, int32_t* status) {
  const size_t smem = sizeof(DecSmem<D>) + 128;   // + alignment slack
  static_assert(DecCfg<D>::CTAS * (sizeof(DecSmem<D>) + 128 + 1024) <= 228 * 1024,
                "the CTAs per SM must fit the shared memory");
  static std::atomic<int> configured[64];   // concurrent first calls set the same limit
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev].load(std::memory_order_relaxed)) {
    const cudaError_t e = cudaFuncSetAttribute(
        decode_fused_kernel<D, K>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) {
      set_error("gdn_decode_fused: cannot reserve %zu bytes of shared memory: %s", smem,
                cudaGetErrorString(e));
      return GDN_ERR_CUDA;
    }
    if (dev >= 0 && dev < 64) configured[dev].store(1, std::memory_order_relaxed);
  }
  decode_fused_kernel<D, K><<<grid, DecCfg<D>::NT, smem, s>>>(
      tm, mixed, ms, z, zs, b, a, abs_, conv_pool, conv_ss, conv_w, a_log, dt_bias, param_f32,
      pool, slot_stride, num_slots, ids, nw, eps, out, bs, HK, R, scale, status);
  return check_launch("gdn_decode_fused");
}

// fp32 [rows, D] view of a per-layer state pool: a (slot, head) tile starts at
// row slot * slot_stride / D + head * D; boxes of [D rows x 64 columns].
static bool make_state_map(CUtensorMap* m, const float* pool, int D, int64_t rows) {
  EncodeTiledFn fn = encode_tiled();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)D * 4};
  const cuuint32_t box[2] = {(cuuint32_t)kDecPartCols, (cuuint32_t)D};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(pool), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
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
                                float scale, int32_t* group_counters, int32_t* status,
                                void* stream) {
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
  GDN_UNSUPPORTED(slot_stride % head_dim == 0,
                  "gdn_decode_fused: slot_stride %lld must be a multiple of the head dim",
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
  cudaStream_t s = (cudaStream_t)stream;
  const int pf = param_dtype == GDN_DTYPE_F32;
  const int64_t units = (int64_t)bs * num_v_heads;
  const int head_ctas = head_dim == 128 ? HeadCfg<128>::CTAS : HeadCfg<64>::CTAS;
  // The head-per-CTA form wins while all units fit one wave (measured on B200:
  // bs 1: 5.8 vs 9.2 us, bs 4: 7.4 vs 10.2 us per config-1 layer); above that
  // the persistent ring streams the pool faster (bs 256: 186 vs 224 us).
  if (group_counters != nullptr && units <= (int64_t)head_ctas * sm_count()) {
#define GDN_DH(DD, KK)                                                                          \
  if (head_dim == DD && conv_kernel == KK)                                                      \
    return launch_decode_head<DD, KK>(                                                          \
        units, s, (const bf16*)mixed, mixed_row_stride, (const bf16*)z, z_row_stride,           \
        (const bf16*)b, (const bf16*)a, ab_row_stride, (bf16*)conv_pool, conv_slot_stride,      \
        (const bf16*)conv_weight, a_log, dt_bias, pf, s_pool, slot_stride, num_slots, ids,      \
        (const bf16*)norm_weight, norm_eps, (bf16*)out, num_k_heads, R, scale, group_counters,  \
        status);
    GDN_DH(128, 4) GDN_DH(128, 3) GDN_DH(128, 2) GDN_DH(64, 4) GDN_DH(64, 3) GDN_DH(64, 2)
#undef GDN_DH
  }
  // the state pool as fp32 rows of head_dim: TMA row coordinates must fit int32
  const int64_t rows = (num_slots - 1) * (slot_stride / head_dim) + value_dim;
  GDN_UNSUPPORTED(rows < (1ll << 31), "gdn_decode_fused: state pool view too large for TMA");
  CUtensorMap tm;
  if (!make_state_map(&tm, s_pool, head_dim, rows)) {
    set_error("gdn_decode_fused: cuTensorMapEncodeTiled failed");
    return GDN_ERR_CUDA;
  }
  const int ctas = head_dim == 128 ? DecCfg<128>::CTAS : DecCfg<64>::CTAS;
  int64_t grid = std::min<int64_t>(groups, (int64_t)sm_count() * ctas);
  const int64_t need = (groups + kDecMaxGroupsPerCta - 1) / kDecMaxGroupsPerCta;
  if (grid < need) grid = need;
#define GDN_DF(DD, KK)                                                                          \
  if (head_dim == DD && conv_kernel == KK)                                                      \
    return launch_decode_fused<DD, KK>(                                                         \
        (int)grid, s, tm, (const bf16*)mixed, mixed_row_stride, (const bf16*)z, z_row_stride,       \
        (const bf16*)b, (const bf16*)a, ab_row_stride, (bf16*)conv_pool, conv_slot_stride,      \
        (const bf16*)conv_weight, a_log, dt_bias, pf, s_pool, slot_stride, num_slots, ids,      \
        (const bf16*)norm_weight, norm_eps, (bf16*)out, bs, num_k_heads, R, scale, status);
  GDN_DF(128, 4) GDN_DF(128, 3) GDN_DF(128, 2) GDN_DF(64, 4) GDN_DF(64, 3) GDN_DF(64, 2)
#undef GDN_DF
  set_error("gdn_decode_fused: unsupported configuration");
  return GDN_ERR_UNSUPPORTED;
}

// ---------------------------------------------------------------------------
// gdn_decode_fused without caller scratch: the group counters live in a
// file-scope device array.  It is zero when the module loads and every launch
// leaves it zero (the last reader of a group resets its counter), so nothing
// has to clear it.  Its address is looked up once per device, on the first call
// made with that device current.
// ---------------------------------------------------------------------------
namespace gdn {

constexpr int64_t kStaticMaxGroups = 16384;   // bs * num_k_heads, 64 KiB of counters
static __device__ __align__(256) int32_t g_static_group_counters[kStaticMaxGroups];

// The lookup is serialised by a mutex (concurrent first calls from several host
// threads are safe).  The address is that of the module's array in the context
// current at the first call on the device, which is the device's primary
// context for a runtime-API caller; a later cudaDeviceReset invalidates it.
static int32_t* static_group_counters() {
  static int32_t* ptr[64] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    set_error("gdn_decode_fused_static: no current CUDA device (or device index >= 64)");
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_static_group_counters);
    if (e != cudaSuccess || p == nullptr) {
      set_error("gdn_decode_fused_static: cudaGetSymbolAddress failed: %s",
                cudaGetErrorString(e));
      return nullptr;
    }
    ptr[dev] = static_cast<int32_t*>(p);
  }
  return ptr[dev];
}

}  // namespace gdn

extern "C" int gdn_decode_fused_static(
    const void* mixed, int64_t mixed_row_stride, const void* z, int64_t z_row_stride,
    const void* b, const void* a, int64_t ab_row_stride, void* conv_pool, int64_t conv_slot_stride,
    const void* conv_weight, int32_t conv_kernel, const void* a_log, const void* dt_bias,
    int32_t param_dtype, float* s_pool, int64_t slot_stride, int64_t num_slots, const int64_t* ids,
    const void* norm_weight, float norm_eps, void* out, int32_t bs, int32_t num_k_heads,
    int32_t num_v_heads, int32_t head_dim, float scale, int32_t* status, void* stream) {
  clear_error();
  GDN_REQUIRE(bs >= 0 && num_k_heads > 0, "gdn_decode_fused_static: bad sizes (bs=%d, HK=%d)",
              bs, num_k_heads);
  const int64_t groups = (int64_t)bs * num_k_heads;
  GDN_UNSUPPORTED(groups <= kStaticMaxGroups,
                  "gdn_decode_fused_static: bs * num_k_heads = %lld exceeds its static scratch "
                  "of %lld groups (use gdn_decode_fused with caller scratch)",
                  (long long)groups, (long long)kStaticMaxGroups);
  if (bs == 0)
    return gdn_decode_fused(mixed, mixed_row_stride, z, z_row_stride, b, a, ab_row_stride,
                            conv_pool, conv_slot_stride, conv_weight, conv_kernel, a_log, dt_bias,
                            param_dtype, s_pool, slot_stride, num_slots, ids, norm_weight,
                            norm_eps, out, bs, num_k_heads, num_v_heads, head_dim, scale, nullptr,
                            status, stream);
  int32_t* counters = static_group_counters();
  if (counters == nullptr) return GDN_ERR_CUDA;
  return gdn_decode_fused(mixed, mixed_row_stride, z, z_row_stride, b, a, ab_row_stride,
                          conv_pool, conv_slot_stride, conv_weight, conv_kernel, a_log, dt_bias,
                          param_dtype, s_pool, slot_stride, num_slots, ids, norm_weight, norm_eps,
                          out, bs, num_k_heads, num_v_heads, head_dim, scale, counters, status,
                          stream);
}
