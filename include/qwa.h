/*
 * qwa.h -- C ABI of the B200 (sm_100a) attention hot path for
 * Qwen3-Embedding-0.6B-shaped layers: fused per-head Q/K RMSNorm + RoPE,
 * and causal / sparse (prefix + local window) GQA prefill attention over
 * ragged micro-batches.
 *
 * Shapes are fixed by the model: 16 query heads, 8 key/value heads,
 * head_dim 128, f16 storage, fp32 softmax and accumulation.
 *
 * Reference interface replaced (shihanqu/qwen3-embedding-webgpu-prepacked):
 *   QKNormRopeKernel.createRun + encodeRun     src/webgpu/ops.ts:152-166, :15-19
 *   CausalAttentionKernel.createRun + encode   src/webgpu/ops.ts:320-345
 *   RoPE table build                           src/webgpu/model.ts:76-83
 *
 * Conventions
 *   - All tensor pointers are device pointers owned by the caller; the
 *     library never frees them. f16 tensors are passed as void*.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default).
 *     Launches are asynchronous on that stream.
 *   - Every call returns a qwa_status; on failure qwa_last_error() gives
 *     a message. No entry point aborts or exits the process.
 *   - A qwa_ctx belongs to one device and is not thread-safe; use one
 *     context per device (per host thread).
 *   - cu_seqlens_host is a HOST array of batch+1 int32 offsets
 *     (cu[0] = 0, non-decreasing). The context caches the device-side launch
 *     plan per distinct (cu_seqlens, mode) and reuses it on later calls, so a
 *     repeated shape costs no host->device traffic.
 */
#ifndef QWA_H
#define QWA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define QWA_API __attribute__((visibility("default")))
#else
#define QWA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum qwa_status {
  QWA_OK = 0,
  QWA_ERR_INVALID_ARG = 1,  /* bad pointer, shape, stride or alignment */
  QWA_ERR_UNSUPPORTED = 2,  /* e.g. head counts other than 16/8, not sm_100 */
  QWA_ERR_CUDA = 3,         /* a CUDA runtime/driver call failed */
  QWA_ERR_TIMEOUT = 4,      /* a device-side bounded wait gave up */
  QWA_ERR_NO_DEVICE = 5
} qwa_status;

typedef enum qwa_mode {
  QWA_MODE_AUTO = 0,   /* reference rule (ops.ts:328): sparse iff max_seqlen <= 8192 */
  QWA_MODE_FULL = 1,   /* full causal */
  QWA_MODE_SPARSE = 2  /* causal, keep k < prefix || k + window > q (ops.ts:220) */
} qwa_mode;

typedef struct qwa_ctx qwa_ctx;

/* Create a context on CUDA device `device` (must be compute capability 10.x).
 * Replaces the WebGPU device + pipeline construction of
 * QKNormRopeKernel/CausalAttentionKernel constructors (ops.ts:153-156, :322-326). */
QWA_API qwa_status qwa_create(int device, qwa_ctx **out);

/* Release the context's device memory (plans, RoPE table, status word).
 * Replaces Qwen3ExecutionPlan.destroy's release of AttentionRun.ownedBuffers
 * (src/webgpu/model.ts:108-111). */
QWA_API qwa_status qwa_destroy(qwa_ctx *ctx);

/* Text of the last error on this context ("" if none). */
QWA_API const char *qwa_last_error(const qwa_ctx *ctx);
QWA_API const char *qwa_status_string(qwa_status status);

/* Library version string. */
QWA_API const char *qwa_version(void);

/* Fused per-head RMSNorm + RoPE prologue over a packed ragged batch.
 * Replaces QKNormRopeKernel.createRun + encodeRun (ops.ts:104-166).
 *   qkv        f16 [total_tokens, qkv_stride]; q at column 0 (16x128),
 *              k at column 2048 (8x128)  (inputStride of ops.ts:157)
 *   q_weight, k_weight  f32 [128] each (attn_q_norm / attn_k_norm)
 *   q_out      f16 [total_tokens, 16, 128]
 *   k_out      f16 [total_tokens, 8, 128]
 *   rope_table optional f32 [max_seqlen, 64, 2] (cos, sin) as built by
 *              model.ts:76-83; NULL = the context's own table for `theta`.
 * Position of a token = its index inside its request. */
QWA_API qwa_status qwa_qk_norm_rope(qwa_ctx *ctx, const void *qkv, int64_t qkv_stride,
                            const float *q_weight, const float *k_weight, void *q_out,
                            void *k_out, const int32_t *cu_seqlens_host, int batch,
                            float eps, float theta, const float *rope_table, void *stream);

/* Padded-batch form with the reference's exact signature semantics
 * (ops.ts:157): `tokens` rows, position = row % sequence. */
QWA_API qwa_status qwa_qk_norm_rope_padded(qwa_ctx *ctx, const void *qkv, int64_t qkv_stride,
                                   const float *q_weight, const float *k_weight, void *q_out,
                                   void *k_out, int tokens, int sequence, float eps,
                                   float theta, const float *rope_table, void *stream);

/* Causal GQA prefill attention over a packed ragged batch (tcgen05 + TMA).
 * Replaces CausalAttentionKernel.createRun + encode (ops.ts:168-345).
 *   q    f16 [total_tokens, 16, 128]   (16-byte aligned)
 *   k    f16 [total_tokens, 8, 128]
 *   v    f16, head g of token t at v[t*v_stride + v_offset + g*128]
 *        (valueStride/valueOffset of ops.ts:327; v+v_offset 16-byte aligned,
 *        v_stride a multiple of 8)
 *   out  f16 [total_tokens, 16, 128]
 *   mode qwa_mode; prefix/window the sparse parameters (reference 176/432). */
QWA_API qwa_status qwa_attention(qwa_ctx *ctx, const void *q, const void *k, const void *v,
                         int64_t v_stride, int64_t v_offset, void *out,
                         const int32_t *cu_seqlens_host, int batch, int mode, int prefix,
                         int window, void *stream);

/* Padded-batch form with the reference's createRun parameters (ops.ts:327):
 * `batch` requests of exactly `sequence` rows each; q_heads/kv_heads must be
 * 16/8. Mode AUTO as the reference (sparse iff sequence <= 8192). */
QWA_API qwa_status qwa_attention_padded(qwa_ctx *ctx, const void *q, const void *k, const void *v,
                                void *out, int batch, int sequence, int q_heads, int kv_heads,
                                int64_t value_stride, int64_t value_offset, void *stream);

/* Prologue + attention for one layer, in the order Qwen3ExecutionPlan encodes
 * them (src/webgpu/model.ts:94-95,123). q_buf/k_buf receive the normed+roped
 * q/k (caller-owned scratch, [T,16,128] / [T,8,128]); V is read from
 * qkv[:, 3072:4096]. */
QWA_API qwa_status qwa_prefill_attention_layer(qwa_ctx *ctx, const void *qkv, int64_t qkv_stride,
                                       const float *q_weight, const float *k_weight,
                                       void *q_buf, void *k_buf, void *out,
                                       const int32_t *cu_seqlens_host, int batch, int mode,
                                       int prefix, int window, float eps, float theta,
                                       void *stream);

/* Synchronise `stream` and report any device-side error recorded by the
 * kernels since the last check (e.g. QWA_ERR_TIMEOUT from a bounded wait);
 * clears the recorded error. ctx == NULL checks the status word of
 * qwa_attention_noalloc on the current device instead (no allocation). */
QWA_API qwa_status qwa_check(qwa_ctx *ctx, void *stream);

/* Bounded waits and their test hook. Every wait of the attention kernel on
 * one of its pipeline barriers gives up after wait_limit_ns (<= 0: the
 * default, 2 s), makes the whole CTA stop, lets the copies and MMAs it has
 * already issued complete, frees its tensor memory and records
 * QWA_ERR_TIMEOUT for qwa_check; the context stays usable. skip_kv_load >= 0
 * makes the first CTA of every later attention call on this context leave
 * out its K/V load number skip_kv_load, so a wait runs out (used by the
 * tests to exercise that path); -1 turns it off. No counterpart in the
 * reference, whose shaders have no error reporting (a failed batch is
 * rejected whole by the engine, src/webgpu/embedding-engine.ts:76-81). */
QWA_API qwa_status qwa_set_debug(qwa_ctx *ctx, int64_t wait_limit_ns, int skip_kv_load);

/* Algorithmic work of an attention call: kept (q,k) pairs summed over the
 * batch (per q-head; FLOPs = 8192 * pairs), and key tiles the kernel visits. */
QWA_API qwa_status qwa_attention_work(const int32_t *cu_seqlens_host, int batch, int mode, int prefix,
                              int window, int64_t *kept_pairs, int64_t *visited_tiles);

/* Diagnostic: one 128x128x128 tensor-core tile through the same shared-memory
 * descriptors the attention kernel uses. a [128,128] f16 (row-major, K
 * contiguous), b [128,128] f16 (row-major, K contiguous), c f32 [128,128]
 * = a @ b^T; then d f32 [128,128] = f16(c) @ vt, with the f16 copy of c
 * taken from tensor memory and vt [128 k,128 n] f16 N-contiguous.
 * No counterpart in the reference (it has no tensor-core path). */
QWA_API qwa_status qwa_selftest_tile(qwa_ctx *ctx, const void *a, const void *b, const void *vt,
                             float *c, float *d, void *stream);

/* Attention without any device allocation, for callers that cannot call
 * cudaMalloc on their serving path (runtimes with a fixed, pre-planned memory
 * arena; processes that hold no qwa_ctx). No counterpart in the reference.
 * Same arguments and results as qwa_attention, on the current device, but the
 * work list and status word live in a fixed 1 MiB device array owned by the
 * library (held by every GPU that loads it until exit). The work list is
 * built on the device from cu_seqlens passed in the launch's parameters, so
 * the call enqueues no host-to-device copy. Limits: at most 4096 requests
 * and 65,520 work items -- ceil(len/128) * 8 summed over requests, about one
 * million tokens; a larger call returns QWA_ERR_INVALID_ARG without
 * launching. The first call on each device looks up that array's address;
 * make it before any stream capture. All calls share the array: calls that
 * overlap on the GPU race. A device-side timeout is recorded in the array and
 * reported by qwa_check(NULL, stream). */
QWA_API qwa_status qwa_attention_noalloc(const void *q, const void *k, const void *v,
                                         int64_t v_stride, int64_t v_offset, void *out,
                                         const int32_t *cu_seqlens_host, int batch, int mode,
                                         int prefix, int window, void *stream);

/* Last-token L2 pooling of a packed ragged batch. Replaces poolShader /
 * LastTokenPoolKernel.createRun (src/webgpu/ops.ts:347-379). hidden: f16
 * [cu_seqlens[batch], width] row-major; out: f32 [batch, width]; out[b] =
 * h / sqrt(sum h^2) with h = hidden[cu_seqlens[b+1]-1] (no epsilon, like the
 * reference: an all-zero row gives non-finite values). An empty request
 * (cu_seqlens[b+1] == cu_seqlens[b]) gives a zero row. width must be a
 * positive multiple of 8; hidden and out 16-byte aligned. */
QWA_API qwa_status qwa_last_token_pool(qwa_ctx *ctx, const void *hidden, int width, float *out,
                                       const int32_t *cu_seqlens_host, int batch, void *stream);

/* The reference's padded form, LastTokenPoolKernel.createRun(input, lengths,
 * output, batch, sequence, width) (ops.ts:361-379): lengths is a DEVICE
 * uint32 [batch] buffer, row b*sequence + lengths[b]-1 is pooled (lengths[b]
 * <= sequence; larger values are clamped to sequence; 0 gives a zero row). */
QWA_API qwa_status qwa_last_token_pool_padded(qwa_ctx *ctx, const void *hidden,
                                              const uint32_t *lengths_device, float *out,
                                              int batch, int sequence, int width, void *stream);

/* Residual add + RMSNorm of the residual stream. Replaces rmsNormShader /
 * RmsNormKernel.createRun(x, residual, weight, normalized, rows, width,
 * epsilon, hasResidual) (src/webgpu/ops.ts:21-64). x, residual, normalized:
 * f16 [rows, width]; weight: f32 [width]. With has_residual != 0, x is
 * updated in place to f16(x + residual) and the sum of squares uses the
 * unrounded f32 sums; normalized = f16(x * 1/sqrt(mean(x^2) + eps) * weight).
 * width must be a positive multiple of 8; pointers 16-byte aligned; residual
 * may be NULL when has_residual == 0. */
QWA_API qwa_status qwa_rms_norm(qwa_ctx *ctx, void *x, const void *residual, const float *weight,
                                void *normalized, int rows, int width, float eps,
                                int has_residual, void *stream);

/* SwiGLU of the FFN. Replaces swigluShader / SwiGLUKernel.createRun(combined,
 * output, rows, width) (src/webgpu/ops.ts:74-102): combined f16 [rows,
 * 2*width] (the ffn_gate_up projection: gate columns, then up columns), out
 * f16 [rows, width] = f16(g / (1 + exp(-g)) * u) in f32 arithmetic. width a
 * positive multiple of 8; pointers 16-byte aligned. */
QWA_API qwa_status qwa_swiglu(qwa_ctx *ctx, const void *combined, void *out, int rows, int width,
                              void *stream);

/* Token embedding lookup from a Q6_K matrix. Replaces embeddingShader /
 * EmbeddingLookupKernel.createRun(tokens, weights, output, tokenCount, width)
 * (src/webgpu/ops.ts:381-426): out f16 [tokens, width], row t = row
 * ids[t] of the Q6_K matrix `table` [vocab, width] (210-byte blocks of 256
 * values, src/gguf/quantization.ts:46-72), each value f16((d * scale) * q) in
 * f32 like the shader. ids_device: DEVICE uint32 [tokens]; an id >= vocab
 * gives a zero row (the reference does not check). width a positive
 * multiple of 256; out 16-byte, table 2-byte, ids 4-byte aligned. */
QWA_API qwa_status qwa_embedding_lookup_q6k(qwa_ctx *ctx, const uint32_t *ids_device,
                                            const void *table, int vocab, void *out, int tokens,
                                            int width, void *stream);

/* Projection GEMM, f16: output[m, n] = sum_k input[m, k] * weight[n, k],
 * f32 accumulation on the tensor cores, f16 result. input f16 [m, k] and
 * weight f16 [n, k] row-major, output f16 [m, n] row-major. Replaces the
 * arithmetic of QuantMatmulKernel (src/webgpu/quant-matmul.ts:495-540) once
 * the weight is dequantised. n must be a multiple of 256 and k of 64
 * (QWA_ERR_UNSUPPORTED otherwise); pointers 16-byte aligned. */
QWA_API qwa_status qwa_matmul(qwa_ctx *ctx, const void *input, const void *weight, void *output,
                              int m, int n, int k, void *stream);

/* ffn_gate_up projection fused with the FFN's SwiGLU (model.ts:98-100 with
 * SwiGLUKernel, ops.ts:74-102): output f16 [m, n/2] with
 *   output[r, c] = f16(g / (1 + exp(-g)) * u),  g = f16(gate[r, c]), u = f16(up[r, c]),
 * bit for bit what qwa_matmul followed by qwa_swiglu gives. weight f16 [n, k]
 * holds the gate_up matrix with its rows interleaved in blocks of 128: rows
 * 256b..256b+127 are gate rows 128b.., rows 256b+128..256b+255 up rows 128b..
 * (the reference's layout is gate rows 0..n/2-1, then up rows). n a multiple
 * of 256, k of 64. */
QWA_API qwa_status qwa_matmul_swiglu(qwa_ctx *ctx, const void *input, const void *weight,
                                     void *output, int m, int n, int k, void *stream);

/* Dequantise a Q4_0 "q4_0-tile32-compact" matrix (src/prepacked/format.ts:
 * 65-99; values as quant-matmul.ts:98-107, f16(scale) * (q - 8) in f16) to
 * f16 weight[n, k] row-major. packed: ceil(n/32) * (k/32) * 32 records of 20
 * bytes, 4-byte aligned; k a multiple of 32. Bit-exact with the reference's
 * dequantised values. */
QWA_API qwa_status qwa_q40_dequantize(qwa_ctx *ctx, const void *packed, int n, int k,
                                      void *weight, void *stream);

/* QuantMatmulKernel.createRunFromBuffers(input, weights, m, n, k, output) +
 * encode for the prepacked tile32 layout (quant-matmul.ts:495-540). Like the
 * reference, the pipeline depends on m (quant-matmul.ts:508): for m <= 64 and
 * n <= 2048 the kernel reads the 20-byte records directly (dequantised in
 * shared memory, K split over CTAs, partial sums in a context workspace of
 * up to 16 * m * n floats that grows on first use; make one call of a shape
 * before capturing it); otherwise the first call for a given (packed, n, k)
 * dequantises the matrix into an f16 copy owned by the context (n * k * 2
 * bytes, kept until qwa_q40_forget or qwa_destroy) and every call runs
 * qwa_matmul on that copy. The copy is
 * found by the packed buffer's address: a caller that rewrites the packed
 * buffer in place, or frees it (the address may later hold another matrix),
 * calls qwa_q40_forget first. */
QWA_API qwa_status qwa_q40_matmul(qwa_ctx *ctx, const void *input, const void *packed,
                                  void *output, int m, int n, int k, void *stream);

/* attn_qkv projection fused with the per-head Q/K RMSNorm + RoPE: the
 * matmul(normalized, attn_qkv) + QKNormRopeKernel pair of src/webgpu/
 * model.ts:93-94 (ops.ts:104-166) in one launch. input f16 [T, k] (T =
 * cu_seqlens[batch], requests packed back to back), weight f16 [4096, k]
 * (rows 0..2047 q, 2048..3071 k, 3072..4095 v); writes q f16 [T,16,128] and
 * k f16 [T,8,128] normalised and rotated at each token's position inside its
 * request, and v f16 [T,1024] (pass v_stride 1024, v_offset 0 to
 * qwa_attention). The qkv values are rounded to f16 before the norm exactly
 * as the unfused path stores qkvRaw, and the norm / rotation arithmetic is
 * the prologue's, so results equal qwa_matmul + qwa_qk_norm_rope bit for bit.
 * rope_table as for qwa_qk_norm_rope (NULL: the context's table for theta).
 * k must be a multiple of 64. */
QWA_API qwa_status qwa_qkv_projection(qwa_ctx *ctx, const void *input, const void *weight, int k,
                                      const float *q_weight, const float *k_weight, void *q_out,
                                      void *k_out, void *v_out, const int32_t *cu_seqlens_host,
                                      int batch, float eps, float theta, const float *rope_table,
                                      void *stream);

/* qwa_qkv_projection with the weight as a Q4_0 tile32-compact matrix [4096, k]
 * (dequantised once into the context's cache, as qwa_q40_matmul). */
QWA_API qwa_status qwa_q40_qkv_projection(qwa_ctx *ctx, const void *input, const void *packed,
                                          int k, const float *q_weight, const float *k_weight,
                                          void *q_out, void *k_out, void *v_out,
                                          const int32_t *cu_seqlens_host, int batch, float eps,
                                          float theta, const float *rope_table, void *stream);

/* Drop the context's f16 copies made from `packed`. Never synchronises (safe
 * during stream capture): the memory is released by the next Q4_0 call made
 * outside a capture, or by qwa_destroy. */
QWA_API qwa_status qwa_q40_forget(qwa_ctx *ctx, const void *packed);

#ifdef __cplusplus
}
#endif
#endif /* QWA_H */
