/*
 * siliconed_dit.h — the elementwise stages around the quantized linears in Siliconed's DiT blocks,
 * for B200 (sm_100a): libsiliconed_dit.so.
 *
 * The linears themselves are libsiliconed_cuda (siliconed_cuda.h). These kernels are what the
 * reference runs between them (Sources/Siliconed/Block.swift:286-376 for the single-stream block,
 * Ops.swift for the formulas), fused so that each activation is read and written once: modulated
 * RMSNorm / LayerNorm writing the next product's bf16 operand, QK-norm + RoPE writing the attention's
 * operands in its [batch, heads, tokens, head_dim] layout, the sandwich-norm gated residual, SwiGLU
 * and GELU (tanh).  fp32 arithmetic; bf16 tensors are raw 16-bit words; every function is
 * asynchronous on `stream` (a cudaStream_t) and returns 0, or SD_INVALID_ARG / SD_CUDA_ERROR.
 */
#ifndef SILICONED_DIT_H
#define SILICONED_DIT_H

#include <stdint.h>

#if defined(__GNUC__)
#define SD_API __attribute__((visibility("default")))
#else
#define SD_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum { SD_OK = 0, SD_INVALID_ARG = 1, SD_CUDA_ERROR = 4, SD_TIMEOUT = 5 };

/* out[r, :] = bf16( x[r, :] * rsqrt(mean(x[r, :]^2) + eps) * weight * (1 + scale) ), fp32 x [rows, d];
 * weight and scale [d] may be NULL (ones / zeros).  Ops.rmsNorm then Ops.scaleRows (Ops.swift:16-42),
 * the modulation's 1 + scale (Block.swift:284-285).  d <= 8192, a multiple of 4. */
SD_API int sd_rms_norm_modulate(const float* x, int64_t rows, int d, const float* weight, const float* scale,
                                float eps, uint16_t* out, void* stream);

/* out[r, :] = bf16( (x[r, :] - mean) * rsqrt(mean((x - mean)^2) + eps) * (1 + scale) + shift ), the
 * LayerNorm without affine of the double-stream blocks (Ops.layerNorm, Ops.swift:225-242) with the adaLN
 * shift and scale.  scale / shift [d] may be NULL.  d <= 8192, a multiple of 4. */
SD_API int sd_layer_norm_modulate(const float* x, int64_t rows, int d, const float* scale, const float* shift,
                                  float eps, uint16_t* out, void* stream);

/* x[r, :] = x[r, :] + g * y'[r, :], fp32 x and y [rows, d]: y' = RMSNorm(y) * norm_weight when norm_weight
 * is not NULL (the sandwich norm of Block.swift:8-10), else y; g = tanh(gate) when gate_tanh, else gate
 * (NULL: 1).  Two roundings, as Ops.gatedResidual (Ops.swift:44-54).  d <= 8192, a multiple of 4. */
SD_API int sd_gated_residual(float* x, const float* y, int64_t rows, int d, const float* gate, int gate_tanh,
                             const float* norm_weight, float eps, void* stream);

/* sd_gated_residual, then sd_rms_norm_modulate(x, weight, scale, eps2, out) on the updated rows, in one pass
 * (the Z-Image block's attention residual followed by the feed-forward's input norm): x is read once, updated
 * in place and normalised from the same values; the bits of the two calls. */
SD_API int sd_gated_residual_rms_modulate(float* x, const float* y, int64_t rows, int d, const float* gate,
                                          int gate_tanh, const float* norm_weight, float eps, const float* weight,
                                          const float* scale, float eps2, uint16_t* out, void* stream);

/* One stream's fused QKV rows -> the attention's operands.  qkv bf16 [batch * tokens, 3 * heads * head_dim]
 * (q | k | v per token).  q and k: RMSNorm over head_dim with norm_q / norm_k (eps), then RoPE on adjacent
 * pairs with freqs fp32 [joint_len, head_dim / 2, 2] (cos, sin) at the token's joint position
 * (Ops.rmsNormRope, Ops.swift:116-146).  q, k, v bf16 [batch, heads, joint_len, head_dim], the stream's
 * tokens written at positions token_offset .. token_offset + tokens - 1.  head_dim = 128. */
SD_API int sd_qk_norm_rope(const uint16_t* qkv, int batch, int tokens, int heads, int head_dim,
                           const float* norm_q, const float* norm_k, const float* freqs, float eps, uint16_t* q,
                           uint16_t* k, uint16_t* v, int joint_len, int token_offset, void* stream);

/* The attention's output bf16 [batch, heads, joint_len, head_dim] -> one stream's rows bf16
 * [batch * tokens, heads * head_dim] (positions token_offset .. token_offset + tokens - 1). */
SD_API int sd_attention_merge(const uint16_t* o, int batch, int heads, int head_dim, int joint_len,
                              int token_offset, int tokens, uint16_t* out, void* stream);

/* out[r, j] = bf16( silu(a) * b ), a = h[r, j], b = h[r, hidden + j], h bf16 [rows, 2 * hidden]
 * (the fused gate / up product), silu(a) = a / (1 + exp(-a)) (Ops.siluGate, Ops.swift:64-90). */
SD_API int sd_swiglu(const uint16_t* h, int64_t rows, int hidden, uint16_t* out, void* stream);

/* sd_swiglu on a product whose gate and up columns are interleaved in blocks of `block` (gate block j at
 * h[r, 2 block j ...], up block j right after it): the layout whose SwiGLU a product can apply in its
 * epilogue (SC_EPI_SWIGLU), used below the epilogue's row count.  block a multiple of 8 dividing hidden. */
SD_API int sd_swiglu_blocks(const uint16_t* h, int64_t rows, int hidden, int block, uint16_t* out, void* stream);

/* h = bf16( 0.5 h (1 + tanh(sqrt(2 / pi) (h + 0.044715 h^3))) ) in place, bf16 [count]
 * (nn.GELU(approximate="tanh"), QwenImage21.swift:953-963). */
SD_API int sd_gelu_tanh(uint16_t* h, int64_t count, void* stream);

/* o = softmax(q k^T * scale) v per row of queries, over all seq keys (no mask), bf16 q, k, v, o
 * [bh][seq][head_dim] (bh = batch * heads; the layout sd_qk_norm_rope writes), fp32 scores, sums and
 * accumulation, P rounded to bf16 for the P . v product: the reference's fused attention
 * (TiledAttention.swift:470-610) in its online form on the tensor cores.  head_dim = 128; pointers
 * 16-byte aligned; scale > 0 (the blocks pass 1 / sqrt(head_dim)).  Replaces the library attention the
 * blocks called before.  Device-side waits are bounded: a wait that gives up is reported by
 * sd_attention_errors. */
SD_API int sd_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* o, int bh, int seq,
                        int head_dim, float scale, void* stream);

/* SD_TIMEOUT (and the wait's site in *site) if a wait of sd_attention gave up since the last call, else SD_OK;
 * clears the record.  Synchronous with the device. */
SD_API int sd_attention_errors(int* site);

#ifdef __cplusplus
}
#endif

#endif /* SILICONED_DIT_H */
