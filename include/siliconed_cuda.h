/*
 * siliconed_cuda.h -- the C ABI of libsiliconed_cuda, a B200 (sm_100a) implementation of
 * Siliconed's quantized linear stage: the int8 / fp8 (e4m3fn) weight-only
 * dequantize-and-multiply behind every DiT and text-encoder projection.
 *
 * Plain C: pointers, sizes and integer status codes; no exceptions, aborts or C++ types cross it.
 * A SwiftPM system-library target can wrap this header directly through a module map.
 *
 * Conventions
 *   - Weights are given in the map's layout: q [K, N] row-major, N contiguous, one byte per value
 *     (Sources/Siliconed/Artifact.swift:15-57, linear_weights_transposed = true), with per-output
 *     (per-column) or per-tensor scales in fp32, bf16 or fp16.  SC_WEIGHT_PUBLISHED_NK accepts the
 *     published nn.Linear layout [N, K] instead.
 *   - Activations and outputs are bf16 (uint16 bit patterns), row-major: x [M, K], y [M, N].
 *   - `stream` is a cudaStream_t (NULL = the legacy default stream).  Every compute call is
 *     asynchronous on that stream; sc_sync / sc_poll_errors wait.
 *   - A context is used by one host thread at a time; distinct contexts may run concurrently.
 *   - Products of one context may run on several streams at once when each has its own workspace
 *     (and its own x and y).  The one piece of state they share, the readiness counters of the
 *     widening inside the GEMM (config-1-sized products from 1536 rows), is guarded: a product whose
 *     stream differs from that of the last product that used them, while that product may still be
 *     running, takes the separate widening instead (same bits); so does a product issued under
 *     stream capture.  The counters return to zero at the end of every launch that uses them.
 *   - Every call selects the context's device as the calling thread's current device and leaves
 *     it selected.
 *   - The library never falls back to the CPU: without a usable sm_100 device every call fails.
 */
#ifndef SILICONED_CUDA_H
#define SILICONED_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SC_ABI_VERSION 1

#if defined(__GNUC__)
#define SC_API __attribute__((visibility("default")))
#else
#define SC_API
#endif

/* Status of every call.  Replaces Swift `throws` (Artifact.Failure, WeightProducts.swift:430) and
 * the nil-and-fallback of refused routes (TensorGEMM.swift:204-232): here a refusal is an error. */
typedef enum sc_status {
    SC_OK = 0,
    SC_INVALID_ARG = 1,          /* null pointer, negative size, unknown enum value */
    SC_UNSUPPORTED_SHAPE = 2,    /* a dimension the kernels cannot take (e.g. K not a multiple of 8) */
    SC_UNALIGNED = 3,            /* x / y / bias not 16-byte aligned where a kernel needs it */
    SC_CUDA_ERROR = 4,           /* a CUDA runtime call failed; see sc_last_error_string */
    SC_TIMEOUT = 5,              /* a bounded device-side wait gave up (reported by sc_poll_errors) */
    SC_OUT_OF_MEMORY = 6,        /* a weight's device arena could not be allocated */
    SC_REFUSED = 7,              /* a weight the forge refuses: a scale whose products are subnormal */
    SC_WORKSPACE_TOO_SMALL = 8,  /* the caller's workspace is smaller than sc_workspace_size */
    SC_NO_DEVICE = 9             /* no CUDA device, or not an sm_100 part */
} sc_status;

/* 8-bit weight kinds (Artifact.DType .int8 / .float8_e4m3). */
typedef enum sc_weight_kind { SC_WEIGHT_INT8 = 1, SC_WEIGHT_E4M3 = 2 } sc_weight_kind;

/* Scale element type as published (Artifact.Scale.dtype, Artifact.swift:38-57). */
typedef enum sc_scale_type { SC_SCALE_F32 = 1, SC_SCALE_BF16 = 2, SC_SCALE_F16 = 3 } sc_scale_type;

/* Scale layout (Widen.ScaleLayout .tensor / .columns, Widen.swift:100-110). */
typedef enum sc_scale_layout { SC_SCALE_TENSOR = 0, SC_SCALE_COLUMNS = 1 } sc_scale_layout;

/* Output element type of sc_linear_ex: bf16 (the north star's) or fp32 (the reference's own C,
 * TensorGEMM.linear(... c: MTLBuffer) writes fp32, TensorGEMM.swift:264-267). */
typedef enum sc_out_type { SC_OUT_BF16 = 0, SC_OUT_F32 = 1 } sc_out_type;

/* Activation element type of the W8A8 entries: bf16, or fp32 (the reference's activation). */
typedef enum sc_in_type { SC_IN_BF16 = 0, SC_IN_F32 = 1 } sc_in_type;

/* Flags of sc_weight_create. */
#define SC_WEIGHT_VALUES_ON_DEVICE 0x1u /* values and scales are device pointers (else host) */
#define SC_WEIGHT_PUBLISHED_NK 0x2u     /* values are the published [N, K] rows, not the map's [K, N] */
/* values are already in the arena's own layout (a map stored re-tiled, `"layout": "arena"`): the rows
 * [n_pad][k_pad] bytes of the transposed weight, n_pad = N rounded up to 256, k_pad = K rounded up to 64,
 * int8 stored biased (q + 128), e4m3 as published, every padding byte the code of zero.  Registration is
 * then one copy, no re-tiling kernel; the whole weight only (not with SC_WEIGHT_PUBLISHED_NK, no shard).
 * Host values are checked (padding, NaN codes); device values are trusted, and SC_WEIGHT_NAN_CODES states
 * that an e4m3 weight holds NaN codes (0x7F / 0xFF). */
#define SC_WEIGHT_ARENA_LAYOUT 0x4u
#define SC_WEIGHT_NAN_CODES 0x8u

typedef uint16_t sc_bf16;
typedef struct sc_ctx sc_ctx;
typedef struct sc_weight sc_weight;

/* ---- context ------------------------------------------------------------------------------ */

SC_API int sc_abi_version(void);
SC_API const char* sc_status_string(sc_status status);

/* Opens a context on CUDA device `device` (made current for the calling thread).  Replaces the
 * engine's GEMM/TensorGEMM objects (GEMM.swift:168-225, TensorGEMM.swift:58-80). */
SC_API sc_status sc_ctx_create(int device, sc_ctx** out);
SC_API void sc_ctx_destroy(sc_ctx* ctx);
/* The last error message of this context ("" if none); valid until the next call on it. */
SC_API const char* sc_last_error_string(const sc_ctx* ctx);

/* ---- weights ------------------------------------------------------------------------------ */

/*
 * Registers one 8-bit linear weight: values q (k*n bytes) and scales (1 or n elements of
 * scale_type).  The library copies them once into its own device arena, re-tiled for the kernels
 * (transposed to [N, K], values biased to unsigned for int8, K padded to 64 and N to 256, scales
 * widened to fp32 after the values); the caller keeps ownership of its buffers.  Replaces the map
 * tensor + Scale (Artifact.swift:15-57), Artifact.stageInt8 (Artifact.swift:755-777) and the
 * reserve plan (WeightProducts.int8Plan, WeightProducts.swift:564-610).
 * Refuses (SC_REFUSED) a nonzero scale whose smallest product is subnormal in fp32
 * (QuantizedLayouts.checkSubnormal, Forge/Quantization.swift:387-403).
 * `stream` orders the upload; the weight is usable on any stream once that stream has reached it.
 */
SC_API sc_status sc_weight_create(sc_ctx* ctx, const void* values, sc_weight_kind kind, int64_t k, int64_t n,
                           const void* scales, sc_scale_type scale_type, sc_scale_layout layout, uint32_t flags,
                           void* stream, sc_weight** out);

/*
 * The same for the columns [n_begin, n_end) of a [K, N] weight only: the shard a rank holds in a
 * column-parallel (N-sharded) linear.  `values`/`scales` describe the whole tensor.
 */
SC_API sc_status sc_weight_create_shard(sc_ctx* ctx, const void* values, sc_weight_kind kind, int64_t k, int64_t n,
                                 const void* scales, sc_scale_type scale_type, sc_scale_layout layout,
                                 uint32_t flags, int64_t n_begin, int64_t n_end, void* stream, sc_weight** out);

SC_API sc_status sc_weight_destroy(sc_ctx* ctx, sc_weight* w);

/*
 * Marks an int8 weight as ComfyUI's convrot (Artifact.rotation, Artifact.swift:397-411): the published
 * weight is W = (q . s) . R along K, R block-diagonal with blocks H / sqrt(G), H the regular Hadamard of
 * size G (Kronecker powers of [[1,1,1,-1],[1,1,-1,1],[1,-1,1,1],[-1,1,1,1]]), G a power of 4 from 4 to 256
 * dividing K.  From then on every product rotates its activation first, x . W = (x . R) . q . s
 * (TensorGEMM.swift:53-54, rotate_groups :183-201): in fp32 butterflies, rounded to bf16, into the front
 * of the caller's workspace (sc_workspace_size grows by m * k * 2 bytes, rounded up to 256), and
 * sc_dequantize exports float(H . q) * (s / sqrt(G)) (Widen.dequantizeRotated, Widen.swift:374-428).
 * group 0 clears the mark.  SC_INVALID_ARG for an e4m3 weight, SC_UNSUPPORTED_SHAPE for another group or
 * K not a multiple of it, SC_REFUSED when a nonzero scale over sqrt(G) is subnormal (the smallest
 * rotated product; QuantizedLayouts.checkSubnormal).
 */
SC_API sc_status sc_weight_set_rotation(sc_ctx* ctx, sc_weight* w, int group);

/*
 * out[m, k] = bf16(x . R) for bf16 x [m, k]: the activation's rotation of a convrot product on its own
 * (rotate_groups, TensorGEMM.swift:183-201: fp32 butterflies of spans 1, 4, 16, 64, then times
 * 1/sqrt(G), then nearest-even to bf16).  K a multiple of the group and of 8; x and out 16-byte aligned.
 */
SC_API sc_status sc_rotate_activation(sc_ctx* ctx, const sc_bf16* x, int64_t m, int64_t k, int group, sc_bf16* out,
                                      void* stream);

/* Shape, kind and device bytes of a registered weight (any out pointer may be NULL). */
SC_API sc_status sc_weight_info(const sc_weight* w, int64_t* k, int64_t* n, int* kind, size_t* device_bytes);

/*
 * Exports the dequantized weight, fp32 [K, N] (device pointer `out`), equal bit for bit to
 * Widen.dequantize: float(q) * s, one rounded multiply (Artifact.materialize, Artifact.swift:670-715
 * -> Widen.swift:129-271).
 */
SC_API sc_status sc_dequantize(sc_ctx* ctx, const sc_weight* w, float* out, void* stream);

/* ---- products ----------------------------------------------------------------------------- */

/* Scratch bytes a product of `m` rows on `w` needs (0 when it needs none).  The caller owns the
 * workspace; the library allocates nothing on the product path (WeightProducts.swift:50-53).
 * From m = 1536 rows it is n_pad * k_pad * 2 bytes (N rounded up to 256, K to 64): the weight's
 * codes widened once to bf16, then a GEMM on bf16 operands, which beats converting the codes in
 * every 256-row block of x.  It must be 256-byte aligned; its contents need no initialisation and
 * are overwritten by every call, so products that may run at the same time on the GPU need
 * workspaces of their own.  With a NULL or smaller workspace such a product runs the fused kernel
 * instead; both routes give the same bits. */
SC_API sc_status sc_workspace_size(sc_ctx* ctx, const sc_weight* w, int64_t m, size_t* bytes);

/*
 * y[m, n] = bf16( (sum_k x[m, k] * float(q[k, n])) * s[n] + bias[n] ), fp32 accumulation, the
 * scale applied after the sum as the native int8 route does (linear_int8 + scale_columns,
 * TensorGEMM.swift:125-179), the bias after it (DiT.swift:410-413), nearest-even bf16
 * (TensorGEMMBF16.swift:43-47).  bias may be NULL.  Replaces TensorGEMM.linear(a:int8:...)
 * (TensorGEMM.swift:264-290) / submitRounded (TensorGEMMBF16.swift:208-264) and, for e4m3, the
 * widened route (WeightProducts.swift:995-1001 -> GEMM.linear, GEMM.swift:297-345).
 * Dispatches on the weight's kind and on m: m <= 4 runs the GEMV (an int8 weight of 3 or 4 rows given the
 * workspace sc_workspace_size reports: the integer skinny product), 4 < m <= 32 the skinny tensor-core
 * products, larger m the tensor-core GEMMs.  x, y, bias: device pointers, 16-byte aligned; K a multiple of 8.
 * workspace may be NULL when sc_workspace_size reports 0 (and from 1536 rows, at the cost of speed).
 */
SC_API sc_status sc_linear(sc_ctx* ctx, const sc_weight* w, const sc_bf16* x, int64_t m, const sc_bf16* bias, sc_bf16* y,
                    void* workspace, size_t workspace_bytes, void* stream);

/* sc_linear with the output type chosen: y is bf16 [m, n] (SC_OUT_BF16) or fp32 [m, n] (SC_OUT_F32,
 * the reference's C buffer; the same sum, scale and bias, without the final rounding to bf16). */
SC_API sc_status sc_linear_ex(sc_ctx* ctx, const sc_weight* w, const sc_bf16* x, int64_t m, const sc_bf16* bias, void* y,
                              sc_out_type y_type, void* workspace, size_t workspace_bytes, void* stream);

/*
 * W8A8, the forward of the int8 weight's own author (TensorGEMMInt8.swift, ComfyUI's int8_linear): the
 * activation x [m, k] (bf16 or fp32) rotated by the weight's convrot group if it has one, quantized to
 * int8 per row over the whole row (s_x = max(max|y| / 127, 1e-30), q_x = clamp(rint(y / s_x), -128, 127),
 * correctly rounded divisions, half to even: W8A8.quantize, :198-221), multiplied exactly in int32 by
 * the weight's int8 codes on the tensor cores (tcgen05 kind::i8), then y = float(acc) * (s_x * s_w)
 * (scale_products, :155-160), + bias when given, in fp32 or rounded to bf16.  int8 weights only
 * (SC_INVALID_ARG otherwise); K a multiple of 8, at most 32768.  The workspace
 * (sc_w8a8_workspace_size) holds the weight's codes made signed, x's codes and s_x: 256-byte aligned.
 */
SC_API sc_status sc_w8a8_workspace_size(sc_ctx* ctx, const sc_weight* w, int64_t m, size_t* bytes);
SC_API sc_status sc_linear_w8a8(sc_ctx* ctx, const sc_weight* w, const void* x, sc_in_type x_type, int64_t m,
                                const sc_bf16* bias, void* y, sc_out_type y_type, void* workspace,
                                size_t workspace_bytes, void* stream);
/* The quantization on its own (quantize_rows, TensorGEMMInt8.swift:137-151): codes int8 rows `ld` bytes
 * apart (ld >= k, a multiple of 16), scales fp32 [m].  group 0: no rotation. */
SC_API sc_status sc_quantize_rows(sc_ctx* ctx, const void* x, sc_in_type x_type, int64_t m, int64_t k, int group,
                                  int8_t* codes, int64_t ld, float* scales, void* stream);

/* Operation fused into the epilogue of sc_linear_epilogue, applied to v = acc * s[n] + bias[n] (fp32). */
typedef enum sc_epilogue {
    SC_EPI_GELU_TANH = 1,       /* y bf16 [m, n] = bf16(gelu_tanh(v)): one rounding instead of two */
    SC_EPI_GATED_RESIDUAL = 2,  /* y fp32 [m, n] (read and written) = y + gate[n] * v, two roundings
                                   (Ops.gatedResidual, Ops.swift:44-54) */
    SC_EPI_SWIGLU = 3           /* W's columns in blocks of 128, gate block j then up block j (N a multiple of
                                   256): y bf16 [m, n / 2], y[:, 128 j + c] = bf16(silu(a) * b),
                                   a = v[:, 256 j + c], b = v[:, 256 j + 128 + c], silu(a) = a / (1 + exp(-a)) */
} sc_epilogue;

/* The bf16-operand product of the widened route (see sc_workspace_size) with an elementwise stage of
 * the DiT block fused into its epilogue, so that the product's output never goes through HBM as an
 * intermediate.  No counterpart in the reference, which runs the GELU (AnimaGELU,
 * ElementwiseGPU.swift) and the gated residual (x + gate * y, DiT.swift) as passes of their own.
 * gate: fp32 [n], device memory, used by SC_EPI_GATED_RESIDUAL only (NULL otherwise).  Takes m > 128
 * rows and a 256-byte aligned workspace of at least n_pad * k_pad * 2 bytes (N rounded up to 256, K
 * to 64), whatever m is; otherwise SC_UNSUPPORTED_SHAPE or SC_WORKSPACE_TOO_SMALL.  y must not
 * overlap x. */
SC_API sc_status sc_linear_epilogue(sc_ctx* ctx, const sc_weight* w, const sc_bf16* x, int64_t m, const sc_bf16* bias,
                                    void* y, sc_epilogue op, const float* gate, void* workspace, size_t workspace_bytes,
                                    void* stream);

/*
 * sc_linear_ex from and to host memory: y_host = x_host . W (+ bias), with the copies overlapped with the
 * products.  The rows go in chunks of whole 256-row tiles (chunk_rows, 0 for the library's choice: about
 * m / 4, at least 512 rows, at most 32 chunks); chunk c's copy in (x_host -> x_dev), product (into y_dev)
 * and copy out (y_dev -> y_host) run on the context's two copy streams and on `stream`, so that one
 * chunk's product runs while the next chunk arrives and the last leaves.  Every chunk of a split batch
 * runs the pair GEMM, so each row has the bits the whole batch would give it on the device.  x_dev
 * [m, k] bf16 and y_dev [m, n] are the caller's device buffers (the library allocates nothing); the
 * workspace is sc_workspace_size's for the largest chunk (that of m suffices).  Asynchronous on
 * `stream`: y_host is complete when `stream` reaches the call's end; x_host and y_host must be page-locked
 * for the copies to overlap.  No counterpart in the reference, where the GPU reads the host's memory
 * (Apple silicon's unified memory: the MTLBuffers of WeightProducts.linear are wrapped no-copy).
 * y_dev NULL: the products write y_host themselves (page-locked host memory the GPU can address; needs the
 * widened route's workspace and no rotation), eight chunks by default, nothing copied back.
 */
SC_API sc_status sc_linear_host(sc_ctx* ctx, const sc_weight* w, const sc_bf16* x_host, int64_t m, const sc_bf16* bias,
                                void* y_host, sc_out_type y_type, sc_bf16* x_dev, void* y_dev, void* workspace,
                                size_t workspace_bytes, int64_t chunk_rows, void* stream);

/*
 * The q / k / v product of a DiT block with QK-norm and RoPE in its epilogue (no counterpart in the
 * reference, which runs them as a pass of their own: Block.swift, QwenImage21.swift).  W's N is
 * 3 * heads * 128 (q, then k, then v, head after head); row r of x is token r % tokens of image
 * r / tokens.  q and k heads: v * inv * norm[d] with inv = 1 / sqrt(sum(v^2) / 128 + eps) over the head's
 * fp32 values, then RoPE on adjacent pairs (e0 c - e1 s, e0 s + e1 c), (c, s) = freqs[pos][d / 2][0..1],
 * pos = offset + r % tokens; v heads as they are.  Each head is written bf16 to out[image][head][pos][0..127]
 * of q, k or v, [images, heads, joint, 128] (the attention's layout).  norm_q / norm_k: fp32 [128]; freqs:
 * fp32 [joint][64][2].  Takes m > 128 rows and the workspace of sc_linear_epilogue.
 */
SC_API sc_status sc_linear_qk_norm_rope(sc_ctx* ctx, const sc_weight* w, const sc_bf16* x, int64_t m,
                                        const sc_bf16* bias, sc_bf16* q, sc_bf16* k, sc_bf16* v, int heads,
                                        int64_t tokens, int64_t joint, int64_t offset, const float* norm_q,
                                        const float* norm_k, const float* freqs, float eps, void* workspace,
                                        size_t workspace_bytes, void* stream);

/*
 * The product whose operand is the attention's output o [batch, heads, joint, 128] bf16 itself: row r of the
 * operand is token r % tokens of image r / tokens, at position offset + r % tokens, its K = heads * 128
 * values head after head (the rows a merge pass would gather; no counterpart in the reference, whose
 * attention writes the merged rows).  y [batch * tokens, n]: bf16 or fp32 (y_type) with op 0, or with op
 * SC_EPI_GATED_RESIDUAL the fp32 residual stream += gate[n] * v in place.  tokens a multiple of 128; the
 * workspace of sc_linear_epilogue; not for a convrot weight.
 */
SC_API sc_status sc_linear_heads(sc_ctx* ctx, const sc_weight* w, const sc_bf16* o, int64_t batch, int heads,
                                 int64_t joint, int64_t offset, int64_t tokens, const sc_bf16* bias, void* y,
                                 sc_out_type y_type, sc_epilogue op, const float* gate, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* sc_linear_ex with its scratch in a 32 MiB device array of the library instead of a workspace: it
 * allocates nothing and takes no workspace argument.  No counterpart in the reference: it serves
 * callers that have no scratch buffer to pass (a binding whose linear call carries only the operand,
 * the output and the sizes) and may not allocate per call (cudaMalloc / cudaFree synchronise the
 * device, which a serving loop cannot afford).  A product
 * whose sc_workspace_size exceeds 32 MiB (from 1536 rows: n_pad * k_pad * 2 bytes of widened weight)
 * returns SC_UNSUPPORTED_SHAPE.  The first call on a device sets up the array's address
 * (cudaGetSymbolAddress) and should come before any stream capture.  All calls on a device share the
 * array and leave the last call's contents in it (nothing in it needs to start at zero); calls that
 * overlap on the GPU race on it. */
SC_API sc_status sc_linear_ex_noalloc(sc_ctx* ctx, const sc_weight* w, const sc_bf16* x, int64_t m,
                                      const sc_bf16* bias, void* y, sc_out_type y_type, void* stream);

/* sc_linear for an int8 weight (SC_INVALID_ARG on another kind). */
SC_API sc_status sc_linear_w8(sc_ctx* ctx, const sc_weight* w, const sc_bf16* x, int64_t m, const sc_bf16* bias, sc_bf16* y,
                       void* workspace, size_t workspace_bytes, void* stream);

/* sc_linear for an e4m3 weight (SC_INVALID_ARG on another kind). */
SC_API sc_status sc_linear_fp8(sc_ctx* ctx, const sc_weight* w, const sc_bf16* x, int64_t m, const sc_bf16* bias,
                        sc_bf16* y, void* workspace, size_t workspace_bytes, void* stream);

/*
 * The skinny product for 1 <= m <= 32 rows (token decode, short encoder prompts), either weight
 * kind: split-K over the GPU with partial sums in `workspace` added in a fixed order, so that every
 * run gives the same bits.  Replaces DecodeKernels.gemv (DecodeKernels.swift:458-470, kernel
 * gemv_int8 :67-109, splits :450-453).
 */
SC_API sc_status sc_gemv_w8(sc_ctx* ctx, const sc_weight* w, const sc_bf16* x, int64_t m, const sc_bf16* bias, sc_bf16* y,
                     void* workspace, size_t workspace_bytes, void* stream);

/* ---- several GPUs: the fused column-parallel gather ---------------------------------------- */

/*
 * No counterpart in the reference (it has no multi-device code): the column-parallel linear of one
 * process per GPU, with the all-gather of y fused into the product.  `w` holds this rank's columns
 * [col0, col0 + n) of an [K, n_total] weight (sc_weight_create_shard); every rank multiplies the same
 * x [m, K].  The product (widened route: `workspace` of n_pad * k_pad * 2 bytes, as sc_workspace_size
 * reports from 1536 rows, is required at every m) stores each bf16 output tile straight into the
 * output y_peers[r] [m, n_total] of every rank r over NVLink (peer stores: the pointers come from
 * sc_ipc_open; y_peers[rank] is this rank's own), then raises flag_peers[r][rank] = epoch on every
 * rank.  All ranks call it with the same epoch, which starts at 1 and grows by one per call; the
 * flags [world] uint32 start at zero.  sc_allgather_wait(flags of this rank) then holds this rank's
 * stream until every rank's columns have landed (bounded: SC_TIMEOUT through sc_poll_errors).  The
 * outputs must be double-buffered across consecutive calls (a rank may start call e + 1 while another
 * still reads the result of call e).  world <= 8; col0 and n_total multiples of 8.
 */
SC_API sc_status sc_linear_allgather(sc_ctx* ctx, const sc_weight* w, const sc_bf16* x, int64_t m, const sc_bf16* bias,
                                     void* const* y_peers, uint32_t* const* flag_peers, int world, int rank,
                                     int64_t col0, int64_t n_total, uint32_t epoch, void* workspace,
                                     size_t workspace_bytes, void* stream);
SC_API sc_status sc_allgather_wait(sc_ctx* ctx, const uint32_t* flags, int world, uint32_t epoch, void* stream);

/* sc_linear_allgather with the outputs bound to an NVLink multicast object: y_multicast is the multicast
 * address of this call's output buffer (the same offsets as every rank's y_peers[r]), and each 16-byte
 * piece leaves the GPU once (multimem.st; NVSwitch delivers it to every rank) instead of once per rank.
 * y_peers is still given (checked) and the flags are raised as in sc_linear_allgather.  NULL y_multicast:
 * sc_linear_allgather.  No counterpart in the reference. */
SC_API sc_status sc_linear_allgather_mc(sc_ctx* ctx, const sc_weight* w, const sc_bf16* x, int64_t m,
                                        const sc_bf16* bias, void* y_multicast, void* const* y_peers,
                                        uint32_t* const* flag_peers, int world, int rank, int64_t col0,
                                        int64_t n_total, uint32_t epoch, void* workspace, size_t workspace_bytes,
                                        void* stream);

/* CUDA IPC plumbing for the peer pointers (no counterpart in the reference): the 64-byte handle of the
 * device allocation holding device_ptr in this process and device_ptr's offset in it; the same address
 * mapped in another process (peer access enabled); the unmap (the pointer and offset sc_ipc_open took). */
SC_API sc_status sc_ipc_handle(sc_ctx* ctx, void* device_ptr, void* handle_out, size_t* offset_out);
SC_API sc_status sc_ipc_open(sc_ctx* ctx, const void* handle, size_t offset, void** device_ptr_out);
SC_API sc_status sc_ipc_close(sc_ctx* ctx, void* device_ptr, size_t offset);

/* ---- synchronisation and device-side errors ----------------------------------------------- */

/* Waits for `stream`. */
SC_API sc_status sc_sync(sc_ctx* ctx, void* stream);

/*
 * Waits for `stream`, then reads and clears the context's device error word: SC_TIMEOUT when a
 * bounded wait inside a kernel gave up (the kernel then released its resources and returned),
 * SC_CUDA_ERROR on an asynchronous CUDA error, SC_OK otherwise.
 */
SC_API sc_status sc_poll_errors(sc_ctx* ctx, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* SILICONED_CUDA_H */
