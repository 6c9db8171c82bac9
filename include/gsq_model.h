/*
 * gsq_model -- C ABI of the decoder-glue kernels of the Qwen3.5-hybrid model
 * harness (the model the reference wires in mlx_gsq/models/qwen35.py:11-152).
 *
 * The projections of that model are the packed-weight calls of gsq_b200.h
 * (gsq_qmv / gsq_qmm / gsq_embed).  What lies between them is here: the
 * residual add + RMSNorm, the SwiGLU product, the gated-DeltaNet block
 * (causal depthwise conv, q/k normalisation, decay and write gates, the
 * delta-rule recurrence, the gated RMSNorm), and the single-token GQA
 * attention step.  The reference takes these from mlx_lm (qwen3_5 and
 * gated_delta, not part of the reference repository); the formulas each
 * entry point computes are written beside it.
 *
 * Conventions as in gsq_b200.h: device pointers, asynchronous on `stream`,
 * no allocation, GSQ_OK or a negative gsq_status (gsq_last_error()).
 * Fixed head sizes: gated-DeltaNet key and value heads are 128 wide,
 * attention heads 256 wide (the model's dimensions, qwen35.py:18-25).
 */
#ifndef GSQ_MODEL_H
#define GSQ_MODEL_H

#include "gsq_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* resid[r,:] += delta[r,:] (skipped when delta is NULL), then
 * out[r,:] = resid[r,:] * rsqrt(mean(resid[r,:]^2) + eps) * weight,
 * rounded to out_dtype.  resid, delta, weight fp32; rows x dim. */
GSQ_API int gsq_rmsnorm(float* resid, const float* delta, int64_t rows, int64_t dim, const float* weight, float eps,
                        void* out, int out_dtype, gsq_stream_t stream);

/* out[r,i] = silu(gate[r,i]) * up[r,i] from a [rows, 2n] input of gu_dtype
 * (fp32, fp16 or bf16; computed in fp32): with group == 0 the gate
 * projection's n outputs then the up projection's; with group g > 0
 * (n % g == 0) interleaved groups of g gate then g up outputs (the layout of
 * an interleaved gate|up matrix, see gsq_qmv_swiglu). */
GSQ_API int gsq_silu_mul(const void* gu, int gu_dtype, int64_t rows, int64_t n, int64_t group, void* out,
                         int out_dtype, gsq_stream_t stream);

/* The FFN's gate and up projections and their SwiGLU product in one fused
 * matvec (decode, 0 < rows < 8): `packed` is a packed matrix of 2*n_out rows
 * (K inputs) holding, per 16 rows, 8 rows of ffn_gate then the same 8 rows
 * of ffn_up (n_out % 8 == 0); y[r,i] = silu(gate_i . x_r) * (up_i . x_r),
 * [rows, n_out] in y_dtype -- the down projection's input, with no fp32
 * round trip and no separate kernel.  Arguments and workspace as gsq_qmv
 * for a 2*n_out-row matrix (gsq_qmv_workspace_size(qtype, 2*n_out, K,
 * rows)).  Token counts of 8 and more use gsq_qmm on the same matrix, then
 * gsq_silu_mul with group 8. */
GSQ_API int gsq_qmv_swiglu(int qtype, const void* x, int x_dtype, const uint8_t* packed, int64_t n_out, int64_t K,
                           int64_t rows, void* y, int y_dtype, void* workspace, size_t workspace_bytes,
                           gsq_stream_t stream);

/* Gated-DeltaNet block of T consecutive tokens (the GDN layer of
 * qwen35.py:48-101; nk key heads, nv = multiple of nk value heads, value
 * head h reading key head h % nk).
 *
 *   proj   [T, proj_stride] fp32: columns [0, C) the q|k|v projection
 *          (C = 2*nk*128 + nv*128), columns [C, C + nv*128) the gate z
 *   ab     [T, ab_stride] fp16: columns [0, nv) the decay input a,
 *          [nv, 2nv) the write-gate input b; or NULL, and then the kernel
 *          computes them from x [T, x_stride] fp16 (the layer's normalised
 *          input) and ab_w [2nv, hidden] fp16 (ssm_alpha rows, then
 *          ssm_beta rows) -- one launch fewer for a decode token
 *   conv_state [4, C] fp32: ring of the previous q|k|v inputs, slot p & 3
 *          holding position p's (zeros at the start of a sequence); the T
 *          tokens' inputs are written to their slots
 *   pos    device int32: position of the first of the T tokens
 *   conv_w [C, 4] fp32 depthwise causal taps; A [nv] = -exp(A_log)
 *          (GGUF's ssm_a); dt_bias [nv]; norm_w [128]
 *   state  [nv, 128 (value index j), 128 (key index i)] fp32, updated
 *   scratch  >= gsq_gdn_scratch_bytes(T, nk, nv) bytes (none for T == 1:
 *          one token runs as a single kernel, a CTA per value head)
 *   out    [T, nv*128] in out_dtype
 *
 * Per token: c = silu(conv(q|k|v)); q = rmsnorm(c_q)/128,
 * k = rmsnorm(c_k)/sqrt(128) (no weights, eps 1e-6); g = exp(A *
 * softplus(a + dt_bias)), beta = sigmoid(b); per value head
 * S <- g*S; u = (v - S k) * beta; S <- S + u k^T; o = S q;
 * out = rmsnorm(o) * norm_w * silu(z) (eps). */
GSQ_API size_t gsq_gdn_scratch_bytes(int64_t T, int64_t nk, int64_t nv);
GSQ_API int gsq_gdn(const float* proj, int64_t proj_stride, const uint16_t* ab, int64_t ab_stride,
                    const uint16_t* x, int64_t x_stride, const uint16_t* ab_w, int64_t hidden, int64_t T,
                    int64_t nk, int64_t nv, float* conv_state, const int32_t* pos, const float* conv_w, const float* A,
                    const float* dt_bias, const float* norm_w, float eps, float* state, void* scratch,
                    size_t scratch_bytes, void* out, int out_dtype, gsq_stream_t stream);

/* One decode token of each of `batch` sequences (batched decode), all at
 * position *pos: sequence b's token is row b of proj [batch, proj_stride]
 * and of ab [batch, ab_stride] (or of x [batch, x_stride] with ab NULL); its
 * conv ring is conv_state[b] ([batch, 4, C]), its recurrent state state[b]
 * ([batch, nv, 128, 128]) and its output row b of out [batch, nv*128].  The
 * per-token formulas are gsq_gdn's.  No scratch.  Extends the reference's
 * single-sequence GDN call (mlx_gsq/models/qwen35.py:48-106) to a batch. */
GSQ_API int gsq_gdn_batch(const float* proj, int64_t proj_stride, const uint16_t* ab, int64_t ab_stride,
                          const uint16_t* x, int64_t x_stride, const uint16_t* ab_w, int64_t hidden, int64_t batch,
                          int64_t nk, int64_t nv, float* conv_state, const int32_t* pos, const float* conv_w,
                          const float* A, const float* dt_bias, const float* norm_w, float eps, float* state,
                          void* out, int out_dtype, gsq_stream_t stream);

/* One decode token of gated GQA attention (qwen35.py:137-145 with mlx_lm's
 * attention): qkv [nq*512 + 2*nkv*256] fp32 = per query head 256 query
 * values then 256 gate values, then the key heads, then the value heads.
 * q and k are RMS-normalised per head (q_norm_w, k_norm_w [256], eps), the
 * first `rot` dimensions rotated (rotate-half pairs (d, d + rot/2), angle
 * pos * theta^(-2i/rot)), the key and value stored at row *pos of the caches
 * k_cache / v_cache [max_len, nkv, 256] fp32, and
 * out[h] = softmax(q k^T / 16) v * sigmoid(gate) over positions 0..*pos,
 * rounded to out_dtype ([nq*256]).  pos is a device int32, so that a
 * captured graph replays at the current position; *pos < max_len. */
GSQ_API int gsq_attn_decode(const float* qkv, int64_t nq, int64_t nkv, const float* q_norm_w,
                            const float* k_norm_w, float eps, int64_t rot, float theta, float* k_cache,
                            float* v_cache, int64_t max_len, const int32_t* pos, void* out, int out_dtype,
                            gsq_stream_t stream);

/* gsq_attn_decode for one token of each of `batch` sequences at position
 * *pos: sequence b's qkv is row b of qkv [batch, nq*512 + 2*nkv*256], its
 * caches are k_cache[b] / v_cache[b] ([batch, max_len, nkv, 256]) and its
 * output row b of out [batch, nq*256]. */
GSQ_API int gsq_attn_decode_batch(const float* qkv, int64_t nq, int64_t nkv, const float* q_norm_w,
                                  const float* k_norm_w, float eps, int64_t rot, float theta, float* k_cache,
                                  float* v_cache, int64_t max_len, const int32_t* pos, void* out, int out_dtype,
                                  int64_t batch, gsq_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* GSQ_MODEL_H */
