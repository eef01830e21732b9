// (d) In-place recurrent decode: one gated-delta-rule step per (sequence,
// v-head), the fp32 state read from and written back to its pool slot.
//
// Maths (qwen3_5.py:561-613, 616-651):
//   q^ = l2norm(q) * scale, k^ = l2norm(k)          (eps 1e-6, fp32)
//   S' = S * exp(g);  d = beta * (v - S'^T k^);  S'' = S' + k^ (x) d
//   out = S''^T q^
//
// HBM roofline: the state is the traffic.  Each (sequence, head) unit moves
// its DK x DV fp32 state once in and once out (2 x 64 KiB at DK = DV = 128);
// q, k, v, g, beta and out add < 1 KiB.  A CTA owns one unit (or a column
// slice of it when there are too few units to fill 148 SMs).  Each thread
// keeps RPT rows x 4 columns of the state in registers: the row loads are
// issued before the q/k norms so the whole tile is in flight at once, every
// warp access is a 512-byte (DV = 128) or 256-byte contiguous float4 run,
// and the state is written back from the same registers — one read and one
// write per element, no shared-memory staging of S.  The two column
// reductions (S'^T k^ and S''^T q^) go through a [RG][DVT] shared buffer.
#include "common.cuh"

namespace gdn {

// NORM: the output row (all DV columns live in this CTA, DVT == DV) goes
// through the gated RMSNorm before it is stored (qwen3_5.py:121-131).
template <int DK, int DV, int DVT, int NT, bool NORM>
__global__ void __launch_bounds__(NT) recurrent_inplace_kernel(
    const bf16* __restrict__ q, int64_t qs, const bf16* __restrict__ k, int64_t ks,
    const bf16* __restrict__ v, int64_t vs, const float* __restrict__ g,
    const bf16* __restrict__ beta, float* __restrict__ pool, int64_t slot_stride,
    int64_t num_slots, const int64_t* __restrict__ ids, bf16* __restrict__ out, int HK, int HV,
    float scale, const bf16* __restrict__ z, int64_t zs, const bf16* __restrict__ nw, float eps,
    int32_t* status) {
  static_assert(!NORM || DVT == DV, "the fused norm needs the whole row in one CTA");
  constexpr int VS = DV / DVT;   // column slices per unit
  constexpr int CG = DVT / 4;    // threads across a row (float4 each)
  constexpr int RG = NT / CG;    // rows per pass
  constexpr int RPT = DK / RG;   // rows per thread
  static_assert(NT % CG == 0 && DK % RG == 0 && DVT % 4 == 0, "bad tiling");
  static_assert(DVT <= NT, "one thread per output column");

  // float4 accesses below need 16-byte alignment of red and sdelta
  __shared__ __align__(16) float red[RG][DVT];
  __shared__ __align__(16) float sdelta[DVT];
  __shared__ float sq[DK], sk[DK], sv[DVT];
  __shared__ float snorm[2];
  __shared__ float swsum[NT / 32];

  const int unit = blockIdx.x / VS;
  const int vt = blockIdx.x - unit * VS;
  const int b = unit / HV;
  const int h = unit - b * HV;
  const int hk = h / (HV / HK);
  const int tid = threadIdx.x;
  const int c4 = tid % CG;
  const int r0 = tid / CG;

  const int64_t slot = ids[b];
  if (!slot_ok(slot, num_slots, status)) return;

  // Issue the state loads first: RPT independent 16-byte loads per thread.
  float* sbase = pool + slot * slot_stride + (int64_t)h * DK * DV + vt * DVT + 4 * c4;
  float4 s[RPT];
#pragma unroll
  for (int i = 0; i < RPT; ++i)
    s[i] = __ldcs(reinterpret_cast<const float4*>(sbase + (int64_t)(r0 + RG * i) * DV));

  // the norm epilogue's z and weight are fetched now, not at the tail
  float zval = 0.f, wval = 0.f;
  if constexpr (NORM) {
    if (tid < DVT) {
      zval = bf2f(z[(int64_t)b * zs + h * DV + tid]);
      wval = bf2f(nw[tid]);
    }
  }

  // q, k, v of this unit (fp32 in shared memory); norms by warp 0.
  for (int i = tid; i < DK; i += NT) {
    sq[i] = bf2f(q[(int64_t)b * qs + hk * DK + i]);
    sk[i] = bf2f(k[(int64_t)b * ks + hk * DK + i]);
  }
  for (int i = tid; i < DVT; i += NT) sv[i] = bf2f(v[(int64_t)b * vs + h * DV + vt * DVT + i]);
  __syncthreads();
  if (tid < 32) {
    float aq = 0.f, ak = 0.f;
    for (int i = tid; i < DK; i += 32) {
      aq += sq[i] * sq[i];
      ak += sk[i] * sk[i];
    }
    aq = warp_sum(aq);
    ak = warp_sum(ak);
    if (tid == 0) {
      snorm[0] = rsqrtf(aq + 1e-6f);
      snorm[1] = rsqrtf(ak + 1e-6f);
    }
  }
  __syncthreads();
  const float nq = snorm[0] * scale;
  const float nk = snorm[1];
  const float eg = expf(g[(int64_t)b * HV + h]);
  const float bt = bf2f(beta[(int64_t)b * HV + h]);

  // S' = S * exp(g); partial (S'^T k^) over this thread's rows.
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const float kk = sk[r0 + RG * i] * nk;
    s[i].x *= eg; s[i].y *= eg; s[i].z *= eg; s[i].w *= eg;
    acc.x += s[i].x * kk; acc.y += s[i].y * kk; acc.z += s[i].z * kk; acc.w += s[i].w * kk;
  }
  *reinterpret_cast<float4*>(&red[r0][4 * c4]) = acc;
  __syncthreads();
  if (tid < DVT) {
    float kv = 0.f;
#pragma unroll
    for (int j = 0; j < RG; ++j) kv += red[j][tid];
    sdelta[tid] = (sv[tid] - kv) * bt;
  }
  __syncthreads();

  // S'' = S' + k^ (x) d, written back in place; partial (S''^T q^).
  const float4 d = *reinterpret_cast<const float4*>(&sdelta[4 * c4]);
  acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int r = r0 + RG * i;
    const float kk = sk[r] * nk;
    const float qq = sq[r] * nq;
    s[i].x += kk * d.x; s[i].y += kk * d.y; s[i].z += kk * d.z; s[i].w += kk * d.w;
    __stcs(reinterpret_cast<float4*>(sbase + (int64_t)r * DV), s[i]);
    acc.x += s[i].x * qq; acc.y += s[i].y * qq; acc.z += s[i].z * qq; acc.w += s[i].w * qq;
  }
  *reinterpret_cast<float4*>(&red[r0][4 * c4]) = acc;
  __syncthreads();
  float o = 0.f;
  if (tid < DVT) {
#pragma unroll
    for (int j = 0; j < RG; ++j) o += red[j][tid];
  }
  bf16* orow = out + ((int64_t)b * HV + h) * DV + vt * DVT;
  if constexpr (!NORM) {
    if (tid < DVT) orow[tid] = f2bf(o);
  } else {
    const float x = tid < DVT ? round_bf(o) : 0.f;   // the core output is bf16 first
    const float ss = warp_sum(x * x);
    if ((tid & 31) == 0) swsum[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < NT / 32; ++w) tot += swsum[w];
    const float inv = rsqrtf(tot / (float)DV + eps);
    if (tid < DVT) orow[tid] = f2bf(gated_norm_elem(x, inv, wval, zval));
  }
}

template <int DK, int DV, int DVT, int NT>
static void launch_recurrent(dim3 grid, cudaStream_t s, const bf16* q, int64_t qs, const bf16* k,
                             int64_t ks, const bf16* v, int64_t vs, const float* g,
                             const bf16* beta, float* pool, int64_t slot_stride, int64_t num_slots,
                             const int64_t* ids, bf16* out, int HK, int HV, float scale,
                             const bf16* z, int64_t zs, const bf16* nw, float eps,
                             int32_t* status) {
  if (z != nullptr && DVT == DV)
    recurrent_inplace_kernel<DK, DV, DVT, NT, (DVT == DV)><<<grid, NT, 0, s>>>(
        q, qs, k, ks, v, vs, g, beta, pool, slot_stride, num_slots, ids, out, HK, HV, scale, z,
        zs, nw, eps, status);
  else
    recurrent_inplace_kernel<DK, DV, DVT, NT, false><<<grid, NT, 0, s>>>(
        q, qs, k, ks, v, vs, g, beta, pool, slot_stride, num_slots, ids, out, HK, HV, scale, z,
        zs, nw, eps, status);
}

}  // namespace gdn

using namespace gdn;

extern "C" int gdn_recurrent_inplace(const void* q, int64_t q_row_stride, const void* k,
                                     int64_t k_row_stride, const void* v, int64_t v_row_stride,
                                     const float* g, const void* beta, float* s_pool,
                                     int64_t slot_stride, int64_t num_slots, const int64_t* ids,
                                     void* out, int32_t bs, int32_t num_k_heads,
                                     int32_t num_v_heads, int32_t head_k_dim, int32_t head_v_dim,
                                     float scale, const void* z, int64_t z_row_stride,
                                     const void* norm_weight, float norm_eps, int32_t* status,
                                     void* stream) {
  clear_error();
  GDN_REQUIRE(bs >= 0 && num_k_heads > 0 && num_v_heads > 0,
              "gdn_recurrent_inplace: bad sizes (bs=%d, HK=%d, HV=%d)", bs, num_k_heads,
              num_v_heads);
  GDN_REQUIRE(num_v_heads % num_k_heads == 0,
              "gdn_recurrent_inplace: num_v_heads %d not a multiple of num_k_heads %d",
              num_v_heads, num_k_heads);
  GDN_UNSUPPORTED((head_k_dim == 128 && head_v_dim == 128) || (head_k_dim == 64 && head_v_dim == 64),
                  "gdn_recurrent_inplace: head dims (%d, %d) unsupported", head_k_dim, head_v_dim);
  GDN_REQUIRE(q_row_stride >= (int64_t)num_k_heads * head_k_dim &&
                  k_row_stride >= (int64_t)num_k_heads * head_k_dim &&
                  v_row_stride >= (int64_t)num_v_heads * head_v_dim,
              "gdn_recurrent_inplace: row stride smaller than the heads it holds");
  GDN_REQUIRE(num_slots > 0 && slot_stride >= (int64_t)num_v_heads * head_k_dim * head_v_dim &&
                  slot_stride % 4 == 0,
              "gdn_recurrent_inplace: slot_stride %lld must be >= HV*DK*DV and a multiple of 4",
              (long long)slot_stride);
  GDN_REQUIRE(z == nullptr || (norm_weight != nullptr &&
                                z_row_stride >= (int64_t)num_v_heads * head_v_dim),
              "gdn_recurrent_inplace: fused norm needs norm_weight and z rows of HV*DV");
  if (bs == 0) return GDN_OK;
  GDN_REQUIRE(q && k && v && g && beta && s_pool && ids && out, "gdn_recurrent_inplace: null pointer");
  GDN_REQUIRE(aligned16(s_pool), "gdn_recurrent_inplace: s_pool must be 16-byte aligned");
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t units = (int64_t)bs * num_v_heads;
  // Split each unit's columns when there are too few units to fill the SMs.
  const int64_t target = 4ll * sm_count();
  const bf16 *qb = (const bf16*)q, *kb = (const bf16*)k, *vb = (const bf16*)v;
  const bf16* bb = (const bf16*)beta;
  bf16* ob = (bf16*)out;
  if (head_k_dim == 128) {
    if (units >= target) {
      launch_recurrent<128, 128, 128, 256>(dim3((unsigned)units), s, qb, q_row_stride, kb,
                                           k_row_stride, vb, v_row_stride, g, bb, s_pool,
                                           slot_stride, num_slots, ids, ob, num_k_heads,
                                           num_v_heads, scale, (const bf16*)z, z_row_stride,
                                           (const bf16*)norm_weight, norm_eps, status);
    } else {
      launch_recurrent<128, 128, 32, 128>(dim3((unsigned)(units * 4)), s, qb, q_row_stride, kb,
                                          k_row_stride, vb, v_row_stride, g, bb, s_pool,
                                          slot_stride, num_slots, ids, ob, num_k_heads,
                                          num_v_heads, scale, (const bf16*)z, z_row_stride,
                                           (const bf16*)norm_weight, norm_eps, status);
    }
  } else {
    if (units >= target) {
      launch_recurrent<64, 64, 64, 128>(dim3((unsigned)units), s, qb, q_row_stride, kb,
                                        k_row_stride, vb, v_row_stride, g, bb, s_pool, slot_stride,
                                        num_slots, ids, ob, num_k_heads, num_v_heads, scale,
                                        (const bf16*)z, z_row_stride, (const bf16*)norm_weight,
                                        norm_eps, status);
    } else {
      launch_recurrent<64, 64, 16, 64>(dim3((unsigned)(units * 4)), s, qb, q_row_stride, kb,
                                       k_row_stride, vb, v_row_stride, g, bb, s_pool, slot_stride,
                                       num_slots, ids, ob, num_k_heads, num_v_heads, scale, (const bf16*)z, z_row_stride,
                                           (const bf16*)norm_weight, norm_eps, status);
    }
  }
  int rc = check_launch("gdn_recurrent_inplace");
  if (rc == GDN_OK && z != nullptr && units < target)   // column-split launch: norm after
    rc = launch_rms_norm_gated(out, z, z_row_stride, num_v_heads, norm_weight, out, units,
                               head_v_dim, norm_eps, s);
  return rc;
}
