/* epq_decode.h -- decode-step glue around the packed linears (libepq.so).
 *
 * Not part of the reference's op interface (include/epq.h): the reference leaves
 * the non-linear parts of a decoder block to the Hugging Face model around its
 * PackedLinear modules (epure/runtime.py:214-305 swaps only the linears).  These
 * entry points do those parts for one decode token in one launch each, so a
 * whole-token CUDA graph is made of the packed linears, these, and the lm_head.
 * Conventions are those of epq.h: plain pointers, epq_dtype codes, a cudaStream_t
 * passed as void*, EPQ_OK or a negative status with epq_last_error().  Positions
 * are read from device memory (int64), so a captured step replays at any position.
 */
#ifndef EPQ_DECODE_H
#define EPQ_DECODE_H

#include <stdint.h>

#include "epq.h"

#ifdef __cplusplus
extern "C" {
#endif

/* For each of m rows of n values (n <= 12288): h = x + add (rounded to dtype;
 * add may be NULL), optionally stored to h_out (may be NULL), and
 * y = h * rsqrt(mean(h^2) + eps) (RMSNorm with weight 1). */
int epq_add_rmsnorm(const void* x, const void* add, void* h_out, void* y, int64_t m, int64_t n,
                    float eps, int32_t dtype, void* stream);

/* Positions are read on the device, so every call below that takes a KV cache
 * also takes its capacity max_len: a position outside [0, max_len) writes
 * nothing to the cache (and zeros to an attention output) and sets bit 4 of
 * epq_device_error, instead of writing past the cache. */

/* For m rows at positions pos[m] (device): q [m, heads, head_dim] is rotated in
 * place; k, v [m, kv_heads, head_dim] are written to k_cache / v_cache
 * [max_len, kv_heads, head_dim] at those positions, k rotated.  qk_norm != 0
 * first applies RMSNorm (weight 1, eps) over each head of q and k (Qwen3).
 * RoPE is rotate-half with cos_tab / sin_tab [max_len, head_dim / 2] (float32).
 * head_dim 64, 128 or 256. */
int epq_rope_kv(void* q, const void* k, const void* v, const int64_t* pos, int64_t m, int32_t heads,
                int32_t kv_heads, int32_t head_dim, const float* cos_tab, const float* sin_tab,
                void* k_cache, void* v_cache, int64_t max_len, int32_t qk_norm, float eps, int32_t dtype,
                void* stream);

/* One query token: out[h] = softmax(scale * q[h] . K[0..pos[0]]) V for every head h
 * (grouped-query: head h reads kv head h / (heads / kv_heads)); q, out [heads, head_dim],
 * caches [max_len, kv_heads, head_dim]; head_dim 64 or 128.  With bf16 and a
 * workspace (heads / kv_heads of 1, 2, 4 or 8) the positions are split over
 * kv_heads x 16 CTAs and merged by the last one; the workspace
 * (epq_attn_decode_workspace_bytes, 256-byte aligned) must be zeroed once before
 * first use and is left ready for the next call.  Without one, one CTA per head. */
int64_t epq_attn_decode_workspace_bytes(int32_t heads, int32_t kv_heads, int32_t head_dim);
int epq_attn_decode(const void* q, const void* k_cache, const void* v_cache, const int64_t* pos,
                    int64_t max_len, int32_t heads, int32_t kv_heads, int32_t head_dim, float scale, void* out,
                    int32_t dtype, void* workspace, int64_t workspace_bytes, void* stream);

/* epq_rope_kv + epq_attn_decode in one launch (bf16, head_dim 64 or 128, heads /
 * kv_heads of 1, 2, 4 or 8): q, k, v [heads or kv_heads, head_dim] are this token's
 * projections at position pos[0]; q and k get (qk_norm) RMSNorm and RoPE inside,
 * k and v are written into the caches at pos[0], and out receives the attention
 * over positions 0..pos[0].  The positions of each kv head are split over a
 * thread-block cluster of 8 CTAs whose partial softmax records are merged in
 * distributed shared memory.  The workspace of epq_attn_decode is still checked
 * (kept for the ABI) but not used. */
int epq_attn_rope_decode(const void* q, const void* k, const void* v, const int64_t* pos, int32_t heads,
                         int32_t kv_heads, int32_t head_dim, const float* cos_tab, const float* sin_tab,
                         void* k_cache, void* v_cache, int64_t max_len, int32_t qk_norm, float eps, float scale,
                         void* out, int32_t dtype, void* workspace, int64_t workspace_bytes, void* stream);

/* *out = the first index of the maximum of x[0..n) (torch.argmax), on the device.
 * workspace: epq_argmax_workspace_bytes(), 256-byte aligned, zeroed once before first
 * use (left ready for the next call). */
int64_t epq_argmax_workspace_bytes(void);
int epq_argmax(const float* x, int64_t n, int64_t* out, void* workspace, int64_t workspace_bytes,
               void* stream);

/* out = silu(g) * u over n values. */
int epq_silu_mul(const void* g, const void* u, void* out, int64_t n, int32_t dtype, void* stream);

/* Prologue / epilogue options of epq_decode_linear. */
enum epq_prologue { EPQ_PRO_NONE = 0, EPQ_PRO_RMSNORM = 1 };
enum epq_epilogue { EPQ_EPI_STORE = 0, EPQ_EPI_RESIDUAL = 1, EPQ_EPI_SILU_MUL = 2 };

/* A decode-step packed linear with the block glue around it fused in: the
 * tensor-core GEMV of epq_linear_multi (1 <= m <= 16 rows of bf16 / f16
 * activations, EPQ_LAYOUT_MMA16 vector stores sharing k; each weight decoded
 * as dtype(dtype(cb[idx]) * dtype(scale)), the reference's materialize rounding)
 * with
 *   prologue EPQ_PRO_RMSNORM: x is replaced by RMSNorm(x) (weight 1, eps) per
 *            row while it is staged (m * k * 2 <= 64 KiB);
 *   epilogue EPQ_EPI_STORE:    outs[i] = x @ W_i^T (rounded to x_dtype);
 *            EPQ_EPI_RESIDUAL: one store; outs[0] is a residual stream updated
 *                              in place: h = h + dtype(x @ W^T);
 *            EPQ_EPI_SILU_MUL: two stores of equal rows (gate, up);
 *                              outs[0] = dtype(silu(dtype(x @ Wg^T)) * dtype(x @ Wu^T))
 *                              (outs[1] is not written).
 * The reference's block (epure/runtime.py:98-126 PackedLinear inside a Llama /
 * Qwen3 decoder layer) rounds at exactly these points.  No workspace; the launch
 * may overlap the previous kernel on the stream (programmatic dependent launch). */
int epq_decode_linear(const epq_store* stores, int32_t count, const void* x, int32_t x_dtype, int64_t m,
                      int64_t ldx, int32_t prologue, float eps, void* const* outs, const int64_t* ldo,
                      int32_t epilogue, void* stream);

/* A decode program: the steps of one batch-1 decode token -- every layer's
 * epq_decode_linear and epq_attn_rope_decode calls, in order -- recorded once
 * and then run as ONE persistent cooperative kernel per token (one CTA per SM).
 * Its weight stream runs through all linear steps without a break; the steps
 * themselves are separated by grid-wide completion counters.  Results are those
 * of the same calls made one by one (the attention's split merge order aside).
 *
 * Steps keep the pointers they are given: the activation buffers, KV caches,
 * position and stores must stay where they are for the program's lifetime (copy
 * a new token's input into the same buffer, write the position into the same
 * int64).  Linear steps: m = 1, bf16 activations, EPQ_LAYOUT_MMA16 stores,
 * k <= 32768, one scale dtype for the whole program.  Attention steps: bf16,
 * head_dim 64 or 128, heads / kv_heads of 1, 2, 4, 8 or 16, 16-byte aligned
 * caches.
 *
 * Life cycle: epq_program_create; epq_program_add_linear / _add_attention per
 * step; epq_program_workspace_bytes; epq_program_finalize (uploads the step
 * table into the caller's workspace, 256-byte aligned, on `stream`, and
 * synchronizes it); epq_program_run per token (a counter reset and one kernel
 * launch on `stream`; capturable in a CUDA graph); epq_program_destroy.  A
 * program is tied to the device it was finalized on, and two runs of one
 * program must not overlap. */
typedef struct epq_program epq_program;
int epq_program_create(epq_program** out);
int epq_program_add_linear(epq_program* p, const epq_store* stores, int32_t count, const void* x, int64_t ldx,
                           int32_t prologue, float eps, void* const* outs, const int64_t* ldo, int32_t epilogue);
int epq_program_add_attention(epq_program* p, const void* q, const void* k, const void* v, const int64_t* pos,
                              int32_t heads, int32_t kv_heads, int32_t head_dim, const float* cos_tab,
                              const float* sin_tab, void* k_cache, void* v_cache, int64_t max_len, int32_t qk_norm,
                              float eps, float scale, void* out);
int64_t epq_program_workspace_bytes(epq_program* p);
int epq_program_finalize(epq_program* p, void* workspace, int64_t workspace_bytes, void* stream);
int epq_program_run(epq_program* p, void* stream);
void epq_program_destroy(epq_program* p);

#ifdef __cplusplus
}
#endif

#endif /* EPQ_DECODE_H */
