/*
 * gdn_b200.h — C ABI of the B200-native GatedDeltaNet (GDN) layer kernels.
 *
 * The library (libgdn_b200.so) replaces the GPU kernels the reference's
 * Qwen3.5 GatedDeltaNet layer launches (sileaver/nano-vllm-extend,
 * nanovllm/models/qwen3_5.py).  Each entry point below names the reference
 * function it stands in for.  Conventions shared by every entry point:
 *
 *  - Pointers are CUDA device pointers unless stated otherwise; the caller
 *    owns all memory.  No entry point allocates device memory, synchronises
 *    the device or the stream, or keeps a pointer after it returns, so every
 *    call can be captured into a CUDA graph.
 *  - `stream` is a cudaStream_t passed as void* (NULL = legacy stream).
 *    Work is launched on it asynchronously.
 *  - Strides are in ELEMENTS of the pointed-to type, never bytes.
 *  - Activations are bf16 (the reference's model dtype); recurrent states
 *    and the log-decay g are fp32, as in the reference's state pool
 *    (engine/model_runner.py:265-303).
 *  - Pool arguments are the per-layer views the reference binds to each
 *    layer (module.s_cache / module.conv_cache, model_runner.py:301-303):
 *    the base pointer of slot 0 of that layer plus the distance between
 *    consecutive slots (`slot_stride`).  `num_slots` counts every addressable
 *    slot, the engine's dummy slot included.
 *  - `ids` are int64 slot ids (context.linear_state_ids, utils/context.py:24).
 *    A slot id outside [0, num_slots) is never dereferenced: its row is
 *    skipped and GDN_STATUS_BAD_SLOT is OR-ed into *status (if non-NULL).
 *    Duplicate ids in one call are undefined behaviour, as in the reference.
 *  - Return value: GDN_OK, or an error code with a message available from
 *    gdn_last_error() (thread-local).  Argument errors are detected on the
 *    host before any launch, mirroring the reference's asserts.
 */
#ifndef GDN_B200_H_
#define GDN_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GDN_ABI_VERSION 7

enum gdn_status_code {
  GDN_OK = 0,
  GDN_ERR_INVALID_ARGUMENT = 1, /* shape / stride / alignment contract violated */
  GDN_ERR_UNSUPPORTED = 2,      /* valid, but not a configuration this build supports */
  GDN_ERR_CUDA = 3              /* a CUDA runtime call or launch failed */
};

/* Bits OR-ed into the optional device status word by kernels. */
#define GDN_STATUS_BAD_SLOT 0x1
#define GDN_STATUS_BAD_SEQLEN 0x2
#define GDN_STATUS_TIMEOUT 0x4 /* a bounded device-side wait gave up; outputs invalid */

enum gdn_dtype { GDN_DTYPE_F32 = 0, GDN_DTYPE_BF16 = 1 };

/* Version of this ABI (GDN_ABI_VERSION of the build). */
int gdn_abi_version(void);

/* Message of the last failed call on this host thread ("" if none). */
const char* gdn_last_error(void);

/*
 * Diagnostic for testing the bounded device-side waits (no counterpart in the
 * reference).  Sets, process-wide, the number of polls after which the wait of
 * gdn_decode_fused's head-per-CTA form for its state bulk copy gives up: that
 * launch then ORs GDN_STATUS_TIMEOUT into *status, waits (with the normal
 * limit) for the copy it has in flight, leaves the recurrent state untouched
 * and returns; the context stays usable.  0 makes the wait give up at once;
 * a negative value restores the default.  Not for production use: calls made
 * while an override is set give invalid results by design.
 */
void gdn_set_wait_limit(int64_t polls);

/*
 * (b) Fused gate.  Replaces fused_g_beta / _gdn_g_beta_kernel
 * (qwen3_5.py:320-360).
 *   g[r,h]    = -exp(a_log[h]) * softplus(a[r,h] + dt_bias[h])   (fp32;
 *               softplus(z) = z for z > 20, else log(1 + exp(z)));
 *               0 where row_mask[r] == 0
 *   beta[r,h] = sigmoid(b[r,h])                                  (bf16)
 * b, a: bf16 [n_rows, num_v_heads] with row stride ab_row_stride;
 * a_log, dt_bias: [num_v_heads] of param_dtype (GDN_DTYPE_F32 / _BF16);
 * row_mask: uint8 [n_rows] or NULL; g: fp32 [n_rows, num_v_heads] and
 * beta: bf16 [n_rows, num_v_heads], both contiguous.
 */
int gdn_fused_g_beta(const void* b, const void* a, int64_t ab_row_stride,
                     int64_t n_rows, int32_t num_v_heads,
                     const void* a_log, const void* dt_bias, int32_t param_dtype,
                     const uint8_t* row_mask, float* g, void* beta,
                     void* stream);

/*
 * (a) Single-token causal conv + SiLU, state rolled in place by slot.
 * Replaces conv_decode_step / _conv_decode_step_kernel (qwen3_5.py:515-558).
 *   y[n,c] = silu(x[n,c]*w[c,K-1] + sum_{i<K-1} s[c,i]*w[c,i]),
 *   s <- [s[1..K-2], x]     with s = conv_pool[ids[n]] ([channels, K-1]).
 * x: bf16 [n, channels], row stride x_row_stride; conv_pool: bf16 per-layer
 * view, taps contiguous (channel stride K-1); weight: bf16 [channels, K]
 * contiguous (conv1d.weight); y: bf16 [n, channels], row stride y_row_stride.
 * kernel (K) must be 2, 3 or 4.
 */
int gdn_conv_decode_step(const void* x, int64_t x_row_stride,
                         void* conv_pool, int64_t slot_stride, int64_t num_slots,
                         const int64_t* ids, int32_t n, int32_t channels,
                         int32_t kernel, const void* weight,
                         void* y, int64_t y_row_stride,
                         int32_t* status, void* stream);

/*
 * (a) Varlen causal conv + SiLU with the prefix state read from, and the
 * final state written back to, each sequence's slot.  Replaces
 * causal_conv_silu_varlen / _causal_conv_silu_varlen_kernel
 * (qwen3_5.py:402-473) together with the gather/scatter of the slot states
 * around it (qwen3_5.py:941-946), and the padded variant's role
 * (qwen3_5.py:249-317, 1048-1056).  Sequence r owns rows
 * [cu_seqlens[r], cu_seqlens[r+1]) of x and y; cu_seqlens is int32
 * [n_seqs + 1] on the device, non-decreasing, cu_seqlens[n_seqs] ==
 * n_tokens.  Zero-length sequences leave their slot unchanged.  Unlike the
 * reference kernel there is no channels % 3 restriction and y keeps the
 * [n_tokens, channels] layout (row stride y_row_stride).
 */
int gdn_causal_conv_silu_varlen(const void* x, int64_t x_row_stride,
                                void* conv_pool, int64_t slot_stride,
                                int64_t num_slots, const int64_t* ids,
                                const int32_t* cu_seqlens, int32_t n_seqs,
                                int64_t n_tokens, int32_t channels,
                                int32_t kernel, const void* weight,
                                void* y, int64_t y_row_stride,
                                int32_t* status, void* stream);

/*
 * (a)+(b) The prefill rows' conv and gate in one call: gdn_causal_conv_silu_varlen
 * and gdn_fused_g_beta (no row mask) on the same rows, the gate computed by an
 * extra row of CTAs of the conv launch (two launches instead of three; the
 * results are bit-identical to the two separate calls).  Replaces the
 * fused_g_beta call and the conv of the varlen prefill (qwen3_5.py:929-946).
 * Arguments as the two calls: b, a bf16 [n_tokens, num_v_heads] with row stride
 * ab_row_stride; g fp32 and beta bf16 [n_tokens, num_v_heads] contiguous.
 */
int gdn_conv_gate_varlen(const void* x, int64_t x_row_stride,
                         void* conv_pool, int64_t slot_stride,
                         int64_t num_slots, const int64_t* ids,
                         const int32_t* cu_seqlens, int32_t n_seqs,
                         int64_t n_tokens, int32_t channels,
                         int32_t kernel, const void* weight,
                         void* y, int64_t y_row_stride,
                         const void* b, const void* a, int64_t ab_row_stride,
                         int32_t num_v_heads, const void* a_log,
                         const void* dt_bias, int32_t param_dtype,
                         float* g, void* beta,
                         int32_t* status, void* stream);

/*
 * (d) One decode step of the gated delta rule, state updated in place in
 * its pool slot (no gather / scatter).  Replaces recurrent_gdn_inplace /
 * _recurrent_inplace_kernel (qwen3_5.py:561-613) and the torch recurrence it
 * mirrors (qwen3_5.py:616-651).  For sequence b and v-head h (k-head
 * hk = h / (num_v_heads / num_k_heads), the reference's repeat_interleave):
 *   q^ = l2norm(q[b,hk]) * scale,  k^ = l2norm(k[b,hk])   (eps 1e-6)
 *   S  = s_pool[ids[b], h] * exp(g[b,h])
 *   d  = beta[b,h] * (v[b,h] - S^T k^);  S += k^ (x) d;  out[b,h] = S^T q^
 * q, k: bf16 rows of num_k_heads*head_k_dim; v: bf16 rows of
 * num_v_heads*head_v_dim (each with its own row stride, heads contiguous);
 * g: fp32 [bs, num_v_heads]; beta: bf16 [bs, num_v_heads] (both contiguous);
 * s_pool: fp32 per-layer view [slots, num_v_heads, head_k_dim, head_v_dim]
 * (head, row and column strides dense, as the reference asserts);
 * out: bf16 [bs, num_v_heads, head_v_dim] contiguous.
 * Optional fused gated-RMSNorm epilogue (Qwen3_5RMSNormGated, qwen3_5.py:121-131,
 * 697-709): when z != NULL, out receives rms_norm_gated(o, z, norm_weight, norm_eps)
 * instead of o, with z bf16 rows of num_v_heads*head_v_dim (row stride z_row_stride,
 * heads contiguous) and norm_weight bf16 [head_v_dim].
 * Supported head dims: (head_k_dim, head_v_dim) in {(64,64), (128,128)}.
 */
int gdn_recurrent_inplace(const void* q, int64_t q_row_stride,
                          const void* k, int64_t k_row_stride,
                          const void* v, int64_t v_row_stride,
                          const float* g, const void* beta,
                          float* s_pool, int64_t slot_stride, int64_t num_slots,
                          const int64_t* ids, void* out,
                          int32_t bs, int32_t num_k_heads, int32_t num_v_heads,
                          int32_t head_k_dim, int32_t head_v_dim, float scale,
                          const void* z, int64_t z_row_stride, const void* norm_weight,
                          float norm_eps, int32_t* status, void* stream);

/*
 * (c) Varlen chunked gated-delta-rule prefill.  Replaces the chunk rule
 * (chunk_gated_delta_rule -> fla or _torch_chunk_gated_delta_rule,
 * qwen3_5.py:140-227) together with the slot gather/scatter around it
 * (qwen3_5.py:956-961, 1039-1040, 1077): each sequence's initial state is
 * read from s_pool[ids[r]] and its final state written back there.
 * Layouts as gdn_recurrent_inplace, with q/k/v/g/beta/out holding n_tokens
 * rows (out: bf16 [n_tokens, num_v_heads, head_v_dim] contiguous).
 * max_seqlen bounds the longest sequence (context.max_seqlen_q); a longer
 * sequence is truncated to max_seqlen and flagged GDN_STATUS_BAD_SEQLEN.
 * Chunk size 64, as the reference.  Supported head dims and the optional
 * gated-RMSNorm epilogue (z, z_row_stride, norm_weight, norm_eps) as
 * gdn_recurrent_inplace.
 *
 * workspace: optional device scratch of at least
 * gdn_chunk_prefill_workspace_bytes(n_tokens, n_seqs, num_v_heads, ...) bytes,
 * 16-byte aligned, used only during the call (stream-ordered).  With it, head
 * dim 128 runs the split form: the state-independent factors of every chunk
 * in a parallel pass, then the serial chain per (sequence, head).  NULL runs
 * the one-kernel form.  Both give the same bits.  A non-NULL workspace that is
 * too small is GDN_ERR_INVALID_ARGUMENT.  The reference allocates its chunk
 * intermediates inside the call; here the caller does.
 */
int64_t gdn_chunk_prefill_workspace_bytes(int64_t n_tokens, int32_t n_seqs, int32_t num_v_heads,
                                          int32_t head_k_dim, int32_t head_v_dim);

int gdn_chunk_prefill_varlen(const void* q, int64_t q_row_stride,
                             const void* k, int64_t k_row_stride,
                             const void* v, int64_t v_row_stride,
                             const float* g, const void* beta,
                             float* s_pool, int64_t slot_stride, int64_t num_slots,
                             const int64_t* ids, const int32_t* cu_seqlens,
                             int32_t n_seqs, int64_t n_tokens, int32_t max_seqlen,
                             void* out, int32_t num_k_heads, int32_t num_v_heads,
                             int32_t head_k_dim, int32_t head_v_dim, float scale,
                             const void* z, int64_t z_row_stride, const void* norm_weight,
                             float norm_eps, void* workspace, int64_t workspace_bytes,
                             int32_t* status, void* stream);

/*
 * Gated RMSNorm over the value head dim.  Replaces Qwen3_5RMSNormGated /
 * _rms_gated_forward (qwen3_5.py:121-131, 697-709), with its rounding:
 *   t = bf16(x * rsqrt(mean(x^2) + eps)); u = bf16(weight * t);
 *   y = bf16(u * silu(gate))                      (fp32 arithmetic)
 * x: bf16 [n_rows, dim] contiguous, n_rows = tokens * heads_per_token;
 * gate: bf16, row r = (token t, head hh) at gate[t*gate_token_stride +
 * hh*dim] (a [tokens, heads, dim] view whose token stride may exceed
 * heads*dim, e.g. a column slice of a fused projection output);
 * weight: bf16 [dim]; y: bf16 [n_rows, dim] contiguous.
 */
int gdn_rms_norm_gated(const void* x, const void* gate, int64_t gate_token_stride,
                       int32_t heads_per_token, const void* weight, void* y,
                       int64_t n_rows, int32_t dim, float eps, void* stream);

/*
 * The whole decode core of one layer in one launch: conv step + g/beta gate +
 * in-place recurrence + gated RMSNorm for bs decode rows, from the fused input
 * projection outputs.  Replaces the decode branch of Qwen3_5GatedDeltaNet.forward
 * (qwen3_5.py:1008-1026: conv_decode_step, fused_g_beta, recurrent_gdn_inplace;
 * and :1083-1085: self.norm(core, z)), i.e. the sequence gdn_conv_decode_step +
 * gdn_fused_g_beta + gdn_recurrent_inplace with the fused norm, whose results it
 * reproduces bit for bit.  The reference has no single counterpart.
 * mixed: bf16 rows [q | k | v] of conv_dim = (2*num_k_heads + num_v_heads) *
 * head_dim channels (row stride mixed_row_stride); z: bf16 rows of
 * num_v_heads*head_dim (z_row_stride); b, a: bf16 rows of num_v_heads
 * (ab_row_stride).  conv_pool / conv_weight as gdn_conv_decode_step (channels =
 * conv_dim, kernel = conv_kernel), rolled in place; a_log, dt_bias as
 * gdn_fused_g_beta; s_pool as gdn_recurrent_inplace (head_k_dim = head_v_dim =
 * head_dim); both pools are indexed by the same ids with num_slots slots.
 * out: bf16 [bs, num_v_heads, head_dim] contiguous, the normed core output.
 * Supported: head_dim 64 or 128, num_v_heads / num_k_heads <= 4, conv_kernel
 * 2..4; s_pool 16-byte aligned; mixed rows, conv slots and conv weight 4-byte
 * aligned (even strides).  A row whose slot id is out of range is skipped
 * (GDN_STATUS_BAD_SLOT), its out rows are left unwritten.
 * group_counters: int32 scratch of at least bs * num_k_heads entries, all zero
 * on entry and left all zero on return (the v-heads of a k-head count their
 * reads of the shared q/k conv state there; the last one rolls it).  With it,
 * batches whose bs * num_v_heads units fit one wave of the GPU run one CTA per
 * (row, v-head) with the state staged in shared memory (the low-latency form);
 * larger batches, and every batch when it is NULL, run a persistent form that
 * needs no scratch.  Calls that share a counter array must not overlap in time.
 */
int gdn_decode_fused(const void* mixed, int64_t mixed_row_stride,
                     const void* z, int64_t z_row_stride,
                     const void* b, const void* a, int64_t ab_row_stride,
                     void* conv_pool, int64_t conv_slot_stride,
                     const void* conv_weight, int32_t conv_kernel,
                     const void* a_log, const void* dt_bias, int32_t param_dtype,
                     float* s_pool, int64_t slot_stride, int64_t num_slots,
                     const int64_t* ids, const void* norm_weight, float norm_eps,
                     void* out, int32_t bs, int32_t num_k_heads, int32_t num_v_heads,
                     int32_t head_dim, float scale, int32_t* group_counters,
                     int32_t* status, void* stream);

/*
 * gdn_decode_fused without caller scratch (no counterpart in the reference):
 * the same arguments minus group_counters, the same results.  The group
 * counters live in a static device array of this library, sized for
 * bs * num_k_heads <= 16384; larger batches are rejected with
 * GDN_ERR_UNSUPPORTED.  For callers that hold no device allocator at the call
 * site (a host binding the C ABI that receives the engine's buffers as raw
 * device pointers) or that must not allocate per decode step.  The array is
 * zero when the library loads and each call leaves it zero, so it needs no
 * clearing.  The first call on a device looks its address up (with that device
 * current; the lookup is serialised across host threads and assumes the
 * device's primary context); make that first call before any stream capture.
 * Calls on one device share the array: they must not overlap in time
 * (different streams running it concurrently race on the counters).  The
 * size limit is the array's: only the one-wave head-per-CTA form uses the
 * counters, and a batch that large would run the persistent form anyway, but
 * this entry point rejects it rather than accept sizes its array cannot hold.
 */
int gdn_decode_fused_static(const void* mixed, int64_t mixed_row_stride,
                            const void* z, int64_t z_row_stride,
                            const void* b, const void* a, int64_t ab_row_stride,
                            void* conv_pool, int64_t conv_slot_stride,
                            const void* conv_weight, int32_t conv_kernel,
                            const void* a_log, const void* dt_bias, int32_t param_dtype,
                            float* s_pool, int64_t slot_stride, int64_t num_slots,
                            const int64_t* ids, const void* norm_weight, float norm_eps,
                            void* out, int32_t bs, int32_t num_k_heads, int32_t num_v_heads,
                            int32_t head_dim, float scale, int32_t* status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GDN_B200_H_ */
