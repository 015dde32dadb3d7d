// Internal definitions shared by the translation units of libsiliconed_cuda.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "siliconed_cuda.h"

// The weight arena's geometry: every weight is stored transposed, [n_pad][k_pad] bytes, K padded
// to the GEMM's K tile and N to its N tile, so that no TMA box ever leaves the arena.
namespace sc {
// cudaFuncSetAttribute(kernel, MaxDynamicSharedMemorySize, bytes) once per device: the attribute belongs to
// the function in the current device's context, so a process that drives several GPUs sets it on each.
template <typename Kernel>
inline cudaError_t set_smem_once(Kernel kernel, int bytes, unsigned long long& done) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = 1ull << (dev & 63);
  if (done & bit) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done |= bit;
  return e;
}

constexpr int kArenaKAlign = 64;    // the GEMM's BK (one 128-byte swizzle row of bf16)
constexpr int kArenaNAlign = 256;   // the GEMM's BN
constexpr int kErrWords = 4;        // device error word: code, site, block, spare
constexpr int kCtxWords = 8;        // the context's device ints: the error word, then the gather counter

// Codes of the padding: q = 0 in the stored encoding of each kind.
constexpr uint8_t kPadInt8 = 0x80;  // int8 is stored biased, u = q + 128
constexpr uint8_t kPadE4M3 = 0x00;  // +0
}  // namespace sc

typedef CUresult (*sc_encode_tiled_fn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                       const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                       CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// A set of device counters that every launch using them returns to zero, and the stream and completion
// event of the last launch that used them: a product on another stream while that launch may still run
// takes a route without them (sc_abi.cu, counters_free).
struct sc_counter_guard {
  cudaStream_t stream = nullptr;
  cudaEvent_t event = nullptr;
  bool launched = false;
};

struct sc_ctx {
  int device = -1;
  int sm_count = 0;
  int* d_err = nullptr;  // sc::kCtxWords ints on the device: the error word (kErrWords), then the
                         // fused gather's CTA counter (zero between launches)
  sc_encode_tiled_fn encode_tiled = nullptr;
  std::string last_error;
  // The fused widening's readiness counters (kWidenCounterWords, then the CTA exit count), zeroed at
  // creation; every launch that uses them returns them to zero as its last CTA leaves.
  uint32_t* d_widen = nullptr;
  sc_counter_guard widen_guard;
  // The int8 skinny product's tile counters (kSkinnyCounterWords), zeroed at creation; the last CTA of
  // each tile returns its counter to zero.
  uint32_t* d_skinny = nullptr;
  sc_counter_guard skinny_guard;
  // sc_linear_host's copy streams and events, created on its first call and kept with the context.
  cudaStream_t copy_in = nullptr, copy_out = nullptr;
  cudaEvent_t host_events[2 * 32 + 2] = {};
};

struct sc_weight {
  int kind = 0;               // SC_WEIGHT_INT8 / SC_WEIGHT_E4M3
  int64_t k = 0, n = 0;       // logical shape [K, N]
  int64_t k_pad = 0, n_pad = 0;
  uint8_t* arena = nullptr;   // one allocation: values, then fp32 scales at a 256-byte boundary
  uint8_t* values = nullptr;  // [n_pad][k_pad] stored codes (int8 biased by 128, e4m3 as is)
  float* scales = nullptr;    // [n_pad] fp32 (0 in the padding)
  size_t bytes = 0;
  bool has_nan_codes = false; // e4m3 weight holding NaN codes (0x7F / 0xFF)
  float min_abs_scale = 0.0f; // the smallest nonzero |s| (0 if every scale is 0)
  int rotation = 0;           // convrot group G (0: none): products rotate x first (sc_rotate.cu)
  int device = -1;
  CUtensorMap tmap_values;    // 2D map over values: inner K (bytes), outer N rows; box 64 x 256
  CUtensorMap tmap_values_half;  // the same, box 64 x 128 (the half tile one CTA of a pair converts)
  CUtensorMap tmap_values_wide;  // the same, box 128 x 128 with 128-byte swizzle (the int8 skinny product's
                                 // MMA operand as stored; 16 KB a copy)
};

namespace sc {

// Sets ctx->last_error and returns `status`.
sc_status fail(sc_ctx* ctx, sc_status status, const std::string& message);
// Maps a CUDA runtime error to SC_CUDA_ERROR with its message (SC_OK if none).
sc_status check_cuda(sc_ctx* ctx, cudaError_t e, const char* what);

// Kernel launchers (host side), defined beside their kernels.
cudaError_t launch_retile(const uint8_t* src, bool published_nk, int kind, int64_t k, int64_t n_total, int64_t n_begin,
                          int64_t n_cols, uint8_t* dst, int64_t k_pad, int64_t n_pad, int* nan_flag,
                          cudaStream_t stream);
cudaError_t launch_dequantize(const sc_weight* w, float* out, cudaStream_t stream);
// convrot (sc_rotate.cu): G a power of 4 in [4, 256]; the rotated activation's scratch; the rotation of
// x [m, k] bf16 into out; the rotated weight's fp32 export.
bool is_rotation_group(int64_t g);
size_t rotated_x_bytes(int64_t m, int64_t k);
cudaError_t launch_rotate(const uint16_t* x, int64_t m, int64_t k, int group, uint16_t* out, cudaStream_t stream);
cudaError_t launch_dequantize_rotated(const sc_weight* w, float* out, cudaStream_t stream);

cudaError_t launch_gemm_tc(const CUtensorMap& tmap_x, const sc_weight* w, const uint16_t* bias, void* y, bool f32_out,
                           int64_t m, int* err, int sm_count, cudaStream_t stream);
cudaError_t launch_gemm_pair(const CUtensorMap& tmap_x, const sc_weight* w, const uint16_t* bias, void* y,
                             bool f32_out, int64_t m, int* err, int sm_count, cudaStream_t stream);
// Rows above which the CTA-pair GEMM takes over from the single-CTA one.
constexpr int64_t kPairMinRows = 128;

// The two-launch large-M route: the codes widened to bf16 [n_pad][k_pad] in the caller's workspace
// (widened_bytes of it), then the pair GEMM on bf16 operands (tmap_w over the widened copy).  Taken
// from kWidenMinRows rows, where converting the codes once beats converting them in every 256-row
// block (measured on B200: even at 256..1024 rows, 10-20 % ahead from 2048).
constexpr int64_t kWidenMinRows = 1536;
size_t widened_bytes(const sc_weight* w);
cudaError_t launch_widen(const sc_weight* w, void* out, int sm_count, cudaStream_t stream);
cudaError_t launch_gemm_bf16(const CUtensorMap& tmap_x, const CUtensorMap& tmap_w, const sc_weight* w,
                             const uint16_t* bias, void* y, bool f32_out, int64_t m, int* err, int sm_count,
                             cudaStream_t stream);

// The fused column-parallel gather (multi-GPU): the bf16-operand pair GEMM whose epilogue stores every
// output tile into the output of each of `world` ranks (peer pointers over NVLink), at columns col0 +
// j of rows of `ld` elements; its last CTA raises flags[r][rank] = epoch on every rank r.  And the
// bounded wait of one rank for the flags of all ranks.
constexpr int kMaxPeers = 8;
struct PeerOut {
  void* y[kMaxPeers];
  void* y_mc;  // the outputs' NVLink multicast address (NVSwitch copies one store to every rank), or null
  uint32_t* flags[kMaxPeers];
  int world, rank;
  int64_t col0, ld;
  uint32_t epoch;
  int* counter;
};
// The q / k / v product's outputs when QK-norm and RoPE run in its epilogue (sc_linear_qk_norm_rope):
// q, k, v [batch, heads, joint, 128] bf16; the product's row r is token r % tokens of image r / tokens,
// at position offset + r % tokens of the joint sequence; freqs [joint][64][2] (cos, sin) per position.
struct HeadOut {
  uint16_t *q, *k, *v;
  const float *norm_q, *norm_k, *freqs;
  float eps;
  int heads, tokens, joint, offset;
};
// x given as the attention's output o [batch, heads, joint, 128] (a 4-D tensor map): the product's row r is
// token r % tokens of image r / tokens at position offset + r % tokens, K = heads * 128.  tokens 0: x is a
// plain [M, K] matrix.
// The widening done inside the bf16 pair GEMM (launch_gemm_bf16_fw): codes -> the workspace's bf16 copy
// by the GEMM's own CTAs, column block by column block, each block's readiness counted in counters[block]
// (zero at launch; the last CTA to leave zeroes them and `done`, its count of CTAs that left).
struct FusedWiden {
  const uint4* codes;
  uint4* out;
  uint32_t* counters;
  uint32_t* done;
  int chunks_per_block;  // 256 * k_pad / 16: 16-code chunks of one 256-column block
  int first_blocks;      // the blocks the first round of tiles reads, widened by every thread first
  int n_blocks;          // n_pad / 256
};
constexpr int kWidenCounterWords = 1024;  // column blocks with a counter (N up to 262144)
cudaError_t launch_gemm_bf16_fw(const CUtensorMap& tmap_x, const CUtensorMap& tmap_w, const sc_weight* w,
                                const uint16_t* bias, void* y, bool f32_out, void* widened, uint32_t* counters,
                                int64_t m, int* err, int sm_count, cudaStream_t stream);
// Whether launch_gemm_bf16_fw serves a product of m rows: two to three rounds of pair tiles, one group of
// the tile order (m_tiles <= 16).
bool fused_widen_fits(const sc_weight* w, int64_t m, int sm_count);

struct XHeads {
  int tokens, offset;
};
cudaError_t launch_gemm_bf16_xheads(const CUtensorMap& tmap_o, const CUtensorMap& tmap_w, const sc_weight* w,
                                    const uint16_t* bias, void* y, bool f32_out, int op, const float* gate,
                                    const XHeads& xh, int64_t m, int* err, int sm_count, cudaStream_t stream);
cudaError_t launch_gemm_bf16_heads(const CUtensorMap& tmap_x, const CUtensorMap& tmap_w, const sc_weight* w,
                                   const uint16_t* bias, const HeadOut& heads, int64_t m, int* err, int sm_count,
                                   cudaStream_t stream);
cudaError_t launch_gemm_bf16_peers(const CUtensorMap& tmap_x, const CUtensorMap& tmap_w, const sc_weight* w,
                                   const uint16_t* bias, const PeerOut& peers, int64_t m, int* err, int sm_count,
                                   cudaStream_t stream);
cudaError_t launch_gather_wait(const uint32_t* flags, int world, uint32_t epoch, int* err, cudaStream_t stream);
// W8A8 (sc_w8a8.cu, sc_gemm_bf16.cu): the weight's codes made signed [n_pad][k_pad] in the workspace;
// x rotated (group > 0) and quantized per row into codes [m][ld] and s_x [m]; the int8 x int8 pair GEMM.
size_t signed_codes_bytes(const sc_weight* w);
cudaError_t launch_sign_codes(const sc_weight* w, void* out, cudaStream_t stream);
cudaError_t launch_quantize_rows(const void* x, bool x_f32, int64_t m, int64_t k, int group, int8_t* codes, int64_t ld,
                                 float* scales, cudaStream_t stream);
cudaError_t launch_gemm_i8(const CUtensorMap& tmap_codes, const CUtensorMap& tmap_w, const sc_weight* w,
                           const uint16_t* bias, void* y, bool f32_out, const float* row_scales, int64_t m, int* err,
                           int sm_count, cudaStream_t stream);
constexpr int64_t kW8A8MaxK = 32768;  // a row held whole in shared memory as fp32 (128 KB)
// The bf16-operand pair GEMM with a fused epilogue operation, op an sc_epilogue value: GELU (tanh) before
// the bf16 store, y (fp32) += gate[n] * v in place (the gated residual), or SwiGLU of gate / up blocks.
cudaError_t launch_gemm_bf16_op(const CUtensorMap& tmap_x, const CUtensorMap& tmap_w, const sc_weight* w,
                                const uint16_t* bias, void* y, int op, const float* gate, int64_t m, int* err,
                                int sm_count, cudaStream_t stream);

// The skinny product on the tensor cores (4 < m <= 32): the x tensor map's box rows for m, and the launch.
int gemm_skinny_box_rows(int64_t m);
cudaError_t launch_gemm_skinny(const CUtensorMap& tmap_x, const sc_weight* w, const uint16_t* bias, void* y,
                               bool f32_out, int64_t m, int* err, int sm_count, cudaStream_t stream);
// Rows above which sc_linear leaves the GEMV for the skinny tensor-core product.
constexpr int64_t kSkinnyMinRows = 4;
// Rows above which an int8 product given the workspace takes the integer skinny product (below: the GEMV).
constexpr int64_t kSkinnyI8MinRows = 2;
// The int8 skinny product on the integer tensor cores (sc_gemm_skinny_sk.cu): x written as three exact 8-bit
// digit planes, the codes multiplied as stored, the work split in equal shares over one CTA per SM, for
// 4 < m <= kSkinnyI8MaxRows (above that the planes' share of the operand traffic makes the cluster kernel
// faster: on B200, 33.5 against 40.6 us a layer of config 4's chain at 24 and 32 rows).  Its grid for a
// weight and m (0: the cluster kernel above serves it), its workspace (the planes, and the tiles' integer
// partials) and the launch (counters: the context's kSkinnyCounterWords tile counters, zero between
// launches).
constexpr int kSkinnyCounterWords = 8192;
constexpr int64_t kSkinnyI8MaxRows = 16;
int skinny_i8_grid(const sc_weight* w, int64_t m, int sm_count);
size_t skinny_i8_workspace_bytes(const sc_weight* w, int64_t m, int grid);
cudaError_t launch_gemm_skinny_i8(sc_encode_tiled_fn encode, const uint16_t* x, const sc_weight* w,
                                  const uint16_t* bias, void* y, bool f32_out, int64_t m, void* workspace,
                                  uint32_t* counters, int grid, int* err, cudaStream_t stream);

// CTA count and workspace of the skinny product.
int gemv_splits(const sc_weight* w, int64_t m, int sm_count);
size_t gemv_workspace_bytes(const sc_weight* w, int64_t m, int sm_count);
cudaError_t launch_gemv(const sc_weight* w, const uint16_t* x, int64_t m, const uint16_t* bias, void* y, bool f32_out,
                        float* workspace, int splits, int* err, cudaStream_t stream);

}  // namespace sc
