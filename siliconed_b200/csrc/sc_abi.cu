// The C ABI of libsiliconed_cuda (include/siliconed_cuda.h): argument checks, the weight arena's
// registration, and dispatch to the kernels.  No entry point throws, traps or falls back to the CPU.
#include <cuda_runtime.h>

#include <cfloat>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <new>
#include <vector>

#include "sc_internal.h"

namespace sc {

sc_status fail(sc_ctx* ctx, sc_status status, const std::string& message) {
  if (ctx != nullptr) ctx->last_error = message;
  return status;
}

sc_status check_cuda(sc_ctx* ctx, cudaError_t e, const char* what) {
  if (e == cudaSuccess) return SC_OK;
  cudaGetLastError();  // clear a sticky launch error of this thread
  std::string m = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
  return fail(ctx, e == cudaErrorMemoryAllocation ? SC_OUT_OF_MEMORY : SC_CUDA_ERROR, m);
}

namespace {

int64_t round_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

// IEEE binary16 -> fp32, exact.
float half_bits_to_f32(uint16_t h) {
  const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
  const int e = (h >> 10) & 0x1F, f = h & 0x3FF;
  uint32_t bits;
  if (e == 0x1F) {
    bits = sign | 0x7F800000u | (static_cast<uint32_t>(f) << 13);
  } else if (e == 0) {
    float v = std::ldexp(static_cast<float>(f), -24);
    std::memcpy(&bits, &v, 4);
    bits |= sign;
  } else {
    bits = sign | (static_cast<uint32_t>(e - 15 + 127) << 23) | (static_cast<uint32_t>(f) << 13);
  }
  float out;
  std::memcpy(&out, &bits, 4);
  return out;
}

float scale_to_f32(const uint8_t* scales, sc_scale_type t, int64_t i) {
  switch (t) {
    case SC_SCALE_F32: {
      float v;
      std::memcpy(&v, scales + 4 * i, 4);
      return v;
    }
    case SC_SCALE_BF16: {
      uint16_t b;
      std::memcpy(&b, scales + 2 * i, 2);
      const uint32_t bits = static_cast<uint32_t>(b) << 16;
      float v;
      std::memcpy(&v, &bits, 4);
      return v;
    }
    default: {
      uint16_t h;
      std::memcpy(&h, scales + 2 * i, 2);
      return half_bits_to_f32(h);
    }
  }
}

size_t scale_size(sc_scale_type t) { return t == SC_SCALE_F32 ? 4 : 2; }

bool is_device_pointer(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

sc_status enter(sc_ctx* ctx) {
  int cur = -1;
  if (cudaGetDevice(&cur) != cudaSuccess) return check_cuda(ctx, cudaGetLastError(), "cudaGetDevice");
  if (cur != ctx->device) return check_cuda(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
  return SC_OK;
}

sc_status make_tmap_x(sc_ctx* ctx, const sc_bf16* x, int64_t m, int64_t k, CUtensorMap* map, int box_rows = 128) {
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(m)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(k) * 2};
  const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = ctx->encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<sc_bf16*>(x), dims, strides, box,
                                 estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ctx, SC_CUDA_ERROR, "cuTensorMapEncodeTiled (activations) failed: " + std::to_string(r));
  return SC_OK;
}

// Map over the widened bf16 copy [n_pad][k_pad] of a weight: box 64 x 128, 128-byte swizzle.
sc_status make_tmap_widened(sc_ctx* ctx, const sc_weight* w, void* widened, CUtensorMap* map) {
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(w->k_pad), static_cast<cuuint64_t>(w->n_pad)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(w->k_pad) * 2};
  const cuuint32_t box[2] = {64, 128};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = ctx->encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, widened, dims, strides, box, estr,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ctx, SC_CUDA_ERROR, "cuTensorMapEncodeTiled (widened weight) failed: " + std::to_string(r));
  return SC_OK;
}

// Map over 8-bit codes [rows][inner] with rows `stride` bytes apart: box 128 x 128, 128-byte swizzle
// (the int8 GEMM's operands: 128 codes of K per stage row).
sc_status make_tmap_codes(sc_ctx* ctx, const void* base, int64_t inner, int64_t rows, int64_t stride, CUtensorMap* map) {
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(stride)};
  const cuuint32_t box[2] = {128, 128};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = ctx->encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
                                 estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ctx, SC_CUDA_ERROR, "cuTensorMapEncodeTiled (codes) failed: " + std::to_string(r));
  return SC_OK;
}

size_t align256(size_t b) { return (b + 255) / 256 * 256; }

// Map over the attention's output o [batch, heads, joint, 128] bf16 as the product's operand: box 64 values
// x 128 tokens of one head of one image, 128-byte swizzle (the same shared-memory tile as make_tmap_x's).
sc_status make_tmap_heads(sc_ctx* ctx, const sc_bf16* o, int64_t batch, int64_t heads, int64_t joint, CUtensorMap* map) {
  const cuuint64_t dims[4] = {128, static_cast<cuuint64_t>(joint), static_cast<cuuint64_t>(heads),
                              static_cast<cuuint64_t>(batch)};
  const cuuint64_t strides[3] = {256, static_cast<cuuint64_t>(joint) * 256, static_cast<cuuint64_t>(heads * joint) * 256};
  const cuuint32_t box[4] = {64, 128, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = ctx->encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<sc_bf16*>(o), dims, strides, box,
                                 estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ctx, SC_CUDA_ERROR, "cuTensorMapEncodeTiled (attention output) failed: " + std::to_string(r));
  return SC_OK;
}
int64_t w8a8_ld(int64_t k) { return (k + 15) / 16 * 16; }
size_t w8a8_workspace(const sc_weight* w, int64_t m) {
  return align256(signed_codes_bytes(w)) + align256(static_cast<size_t>(m * w8a8_ld(w->k))) +
         align256(static_cast<size_t>(m) * 4);
}

sc_status make_tmap_w(sc_ctx* ctx, sc_weight* w) {
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(w->k_pad), static_cast<cuuint64_t>(w->n_pad)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(w->k_pad)};
  const cuuint32_t estr[2] = {1, 1};
  CUtensorMap* maps[3] = {&w->tmap_values, &w->tmap_values_half, &w->tmap_values_wide};
  const cuuint32_t inner[3] = {64, 64, 128}, rows[3] = {256, 128, 128};
  const CUtensorMapSwizzle swz[3] = {CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_SWIZZLE_128B};
  for (int i = 0; i < 3; ++i) {
    const cuuint32_t box[2] = {inner[i], rows[i]};
    CUresult r = ctx->encode_tiled(maps[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, w->values, dims, strides, box, estr,
                                   CU_TENSOR_MAP_INTERLEAVE_NONE, swz[i], CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
      return fail(ctx, SC_CUDA_ERROR, "cuTensorMapEncodeTiled (weights) failed: " + std::to_string(r));
  }
  return SC_OK;
}

sc_status check_product_args(sc_ctx* ctx, const sc_weight* w, const sc_bf16* x, int64_t m, const sc_bf16* bias,
                             const void* y) {
  if (ctx == nullptr) return SC_INVALID_ARG;
  if (w == nullptr) return fail(ctx, SC_INVALID_ARG, "null weight");
  if (m < 0) return fail(ctx, SC_INVALID_ARG, "m < 0");
  if (m == 0) return SC_OK;  // nothing is read or written: x and y may be null
  if (x == nullptr || y == nullptr) return fail(ctx, SC_INVALID_ARG, "null x or y");
  if (m > 0x7FFFFFFF || w->k > 0x7FFFFFFF) return fail(ctx, SC_UNSUPPORTED_SHAPE, "m or k beyond 2^31 - 1");
  if (w->device != ctx->device) return fail(ctx, SC_INVALID_ARG, "weight registered on another device");
  if (w->k % 8 != 0) return fail(ctx, SC_UNSUPPORTED_SHAPE, "K must be a multiple of 8 (16-byte activation rows)");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15u)
    return fail(ctx, SC_UNALIGNED, "x and y must be 16-byte aligned");
  if (bias != nullptr && (reinterpret_cast<uintptr_t>(bias) & 1u)) return fail(ctx, SC_UNALIGNED, "bias must be 2-byte aligned");
  if (m > 0) {
    if (!is_device_pointer(x) || !is_device_pointer(y) || (bias != nullptr && !is_device_pointer(bias)))
      return fail(ctx, SC_INVALID_ARG, "x, y and bias must be device (or managed) memory");
  }
  return SC_OK;
}

// A convrot weight: x . W = (x . R) . q . s, so x is rotated into the front of the workspace first; on
// return x, workspace and workspace_bytes describe the product's operand and the rest of the scratch.
sc_status rotate_operand(sc_ctx* ctx, const sc_weight* w, const sc_bf16*& x, int64_t m, void*& workspace,
                         size_t& workspace_bytes, cudaStream_t st) {
  if (w->rotation == 0 || m == 0) return SC_OK;
  const size_t rx = rotated_x_bytes(m, w->k);
  if (workspace == nullptr || workspace_bytes < rx || (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return fail(ctx, SC_WORKSPACE_TOO_SMALL, "a convrot weight needs a 256-byte aligned workspace (sc_workspace_size)");
  sc_bf16* xr = static_cast<sc_bf16*>(workspace);
  sc_status s = check_cuda(ctx, launch_rotate(x, m, w->k, w->rotation, xr, st), "rotation launch");
  if (s != SC_OK) return s;
  x = xr;
  workspace_bytes -= rx;
  workspace = workspace_bytes > 0 ? static_cast<uint8_t*>(workspace) + rx : nullptr;
  return SC_OK;
}

// Whether a product on stream `st` may use a set of the context's counters (the fused widening's readiness
// counters, the streamed skinny product's tile counters): yes unless the last launch that used them went to
// another stream and may still be running (then the product takes a route without them, which gives the
// same bits and shares nothing).  Under stream capture nothing can be asked of an event, and the route
// without them is taken.
sc_status counters_free(sc_ctx* ctx, const sc_counter_guard& g, cudaStream_t st, bool& free) {
  free = false;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaError_t e = cudaStreamIsCapturing(st, &cap); e != cudaSuccess) return check_cuda(ctx, e, "capture query");
  if (cap != cudaStreamCaptureStatusNone) return SC_OK;
  if (g.launched && g.stream != st) {
    const cudaError_t e = cudaEventQuery(g.event);
    if (e == cudaErrorNotReady) {
      cudaGetLastError();
      return SC_OK;
    }
    if (e != cudaSuccess) return check_cuda(ctx, e, "event query");
  }
  free = true;
  return SC_OK;
}

// Records the stream and completion event of a launch that used a set of counters.
sc_status counters_launched(sc_ctx* ctx, sc_counter_guard& g, cudaStream_t st) {
  if (g.event == nullptr) {
    sc_status s = check_cuda(ctx, cudaEventCreateWithFlags(&g.event, cudaEventDisableTiming), "event");
    if (s != SC_OK) return s;
  }
  sc_status s = check_cuda(ctx, cudaEventRecord(g.event, st), "event record");
  if (s != SC_OK) return s;
  g.stream = st;
  g.launched = true;
  return SC_OK;
}

sc_status run_gemv(sc_ctx* ctx, const sc_weight* w, const sc_bf16* x, int64_t m, const sc_bf16* bias, void* y,
                   bool f32_out, void* workspace, size_t workspace_bytes, cudaStream_t st) {
  const size_t need = gemv_workspace_bytes(w, m, ctx->sm_count);
  if (workspace_bytes < need || (need > 0 && workspace == nullptr))
    return fail(ctx, SC_WORKSPACE_TOO_SMALL, "workspace smaller than sc_workspace_size");
  const int splits = gemv_splits(w, m, ctx->sm_count);
  return check_cuda(ctx, launch_gemv(w, x, m, bias, y, f32_out, static_cast<float*>(workspace), splits, ctx->d_err, st),
                    "gemv launch");
}

sc_status run_linear(sc_ctx* ctx, const sc_weight* w, const sc_bf16* x, int64_t m, const sc_bf16* bias, void* y,
                     bool f32_out, void* workspace, size_t workspace_bytes, void* stream, int want_kind) {
  sc_status s = check_product_args(ctx, w, x, m, bias, y);
  if (s != SC_OK) return s;
  if (want_kind != 0 && w->kind != want_kind)
    return fail(ctx, SC_INVALID_ARG, want_kind == SC_WEIGHT_INT8 ? "not an int8 weight" : "not an e4m3 weight");
  if (m == 0) return SC_OK;
  if ((s = enter(ctx)) != SC_OK) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((s = rotate_operand(ctx, w, x, m, workspace, workspace_bytes, st)) != SC_OK) return s;
  // int8 products of kSkinnyI8MinRows < m <= kSkinnyMinRows go to the integer skinny product when its
  // workspace is there (it reads the weight once whatever m is, where the GEMV's arithmetic grows with m)
  const bool i8_small = m > kSkinnyI8MinRows && m <= kSkinnyMinRows && skinny_i8_grid(w, m, ctx->sm_count) > 0 &&
                        workspace != nullptr;
  if (m <= kSkinnyMinRows && !i8_small)
    return run_gemv(ctx, w, x, m, bias, y, f32_out, workspace, workspace_bytes, st);
  CUtensorMap tmx;
  if (m <= 32) {
    if ((s = make_tmap_x(ctx, x, m, w->k, &tmx, gemm_skinny_box_rows(m))) != SC_OK) return s;
    // int8, m <= 16, with the workspace for x's digit planes and the tiles' partials: the codes straight into
    // the integer tensor cores, every SM an equal share of the weight.  Otherwise (e4m3, m > 16, or no
    // workspace): the cluster kernel, which converts the codes to bf16 and adds its K parts in distributed
    // shared memory.
    const int grid = skinny_i8_grid(w, m, ctx->sm_count);
    bool integer = false;
    if (grid > 0 && workspace != nullptr && workspace_bytes >= skinny_i8_workspace_bytes(w, m, grid) &&
        (reinterpret_cast<uintptr_t>(workspace) & 255u) == 0 &&
        (s = counters_free(ctx, ctx->skinny_guard, st, integer)) != SC_OK)
      return s;
    if (integer) {
      if ((s = check_cuda(ctx, launch_gemm_skinny_i8(ctx->encode_tiled, x, w, bias, y, f32_out, m, workspace,
                                                     ctx->d_skinny, grid, ctx->d_err, st),
                          "int8 skinny gemm launch")) != SC_OK)
        return s;
      return counters_launched(ctx, ctx->skinny_guard, st);
    }
    if (i8_small) return run_gemv(ctx, w, x, m, bias, y, f32_out, workspace, workspace_bytes, st);
    return check_cuda(ctx, launch_gemm_skinny(tmx, w, bias, y, f32_out, m, ctx->d_err, ctx->sm_count, st),
                      "skinny gemm launch");
  }
  if (m <= 128 && w->n_pad / 256 < ctx->sm_count) {
    // 32 < m <= 128 with too few 128 x 256 output tiles to fill the SMs (every weight but the widest): the
    // cluster kernel, whose CTAs split K and own 128 columns each
    if ((s = make_tmap_x(ctx, x, m, w->k, &tmx, gemm_skinny_box_rows(m))) != SC_OK) return s;
    return check_cuda(ctx, launch_gemm_skinny(tmx, w, bias, y, f32_out, m, ctx->d_err, ctx->sm_count, st),
                      "skinny gemm launch");
  }
  if ((s = make_tmap_x(ctx, x, m, w->k, &tmx)) != SC_OK) return s;
  if (m > kPairMinRows) {
    // With a workspace for the widened weight: widen once, then the bf16-operand pair GEMM (the
    // same operands and summation order as the fused kernel, so the same bits).  Without one: the
    // fused pair kernel, which converts the codes in shared memory.
    if (m >= kWidenMinRows && workspace != nullptr && workspace_bytes >= widened_bytes(w) &&
        (reinterpret_cast<uintptr_t>(workspace) & 255u) == 0) {
      CUtensorMap tmw;
      if ((s = make_tmap_widened(ctx, w, workspace, &tmw)) != SC_OK) return s;
      bool fused = false;
      if (fused_widen_fits(w, m, ctx->sm_count) && (s = counters_free(ctx, ctx->widen_guard, st, fused)) != SC_OK) return s;
      if (fused) {
        // a few rounds of tiles: the GEMM's CTAs widen the codes themselves, the first round's columns
        // first, the rest while the pipeline runs
        if ((s = check_cuda(ctx, launch_gemm_bf16_fw(tmx, tmw, w, bias, y, f32_out, workspace, ctx->d_widen, m,
                                                     ctx->d_err, ctx->sm_count, st),
                            "bf16 pair gemm (fused widening) launch")) != SC_OK)
          return s;
        return counters_launched(ctx, ctx->widen_guard, st);
      }
      if ((s = check_cuda(ctx, launch_widen(w, workspace, ctx->sm_count, st), "widen launch")) != SC_OK) return s;
      return check_cuda(ctx, launch_gemm_bf16(tmx, tmw, w, bias, y, f32_out, m, ctx->d_err, ctx->sm_count, st),
                        "bf16 pair gemm launch");
    }
    return check_cuda(ctx, launch_gemm_pair(tmx, w, bias, y, f32_out, m, ctx->d_err, ctx->sm_count, st),
                      "pair gemm launch");
  }
  return check_cuda(ctx, launch_gemm_tc(tmx, w, bias, y, f32_out, m, ctx->d_err, ctx->sm_count, st), "gemm launch");
}

}  // namespace
}  // namespace sc

using namespace sc;

extern "C" {

int sc_abi_version(void) { return SC_ABI_VERSION; }

const char* sc_status_string(sc_status status) {
  switch (status) {
    case SC_OK: return "ok";
    case SC_INVALID_ARG: return "invalid argument";
    case SC_UNSUPPORTED_SHAPE: return "unsupported shape";
    case SC_UNALIGNED: return "unaligned pointer";
    case SC_CUDA_ERROR: return "CUDA error";
    case SC_TIMEOUT: return "device-side wait timed out";
    case SC_OUT_OF_MEMORY: return "out of device memory";
    case SC_REFUSED: return "weight refused";
    case SC_WORKSPACE_TOO_SMALL: return "workspace too small";
    case SC_NO_DEVICE: return "no usable sm_100 device";
  }
  return "unknown status";
}

sc_status sc_ctx_create(int device, sc_ctx** out) {
  if (out == nullptr) return SC_INVALID_ARG;
  *out = nullptr;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
    cudaGetLastError();
    return SC_NO_DEVICE;
  }
  if (device < 0 || device >= count) return SC_INVALID_ARG;
  if (cudaSetDevice(device) != cudaSuccess) {
    cudaGetLastError();
    return SC_NO_DEVICE;
  }
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess || prop.major != 10) {
    cudaGetLastError();
    return SC_NO_DEVICE;
  }
  sc_ctx* ctx = new (std::nothrow) sc_ctx();
  if (ctx == nullptr) return SC_OUT_OF_MEMORY;
  ctx->device = device;
  ctx->sm_count = prop.multiProcessorCount;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || fn == nullptr) {
    cudaGetLastError();
    delete ctx;
    return SC_NO_DEVICE;
  }
  ctx->encode_tiled = reinterpret_cast<sc_encode_tiled_fn>(fn);
  if (cudaMalloc(&ctx->d_err, kCtxWords * sizeof(int)) != cudaSuccess ||
      cudaMemset(ctx->d_err, 0, kCtxWords * sizeof(int)) != cudaSuccess ||
      cudaMalloc(&ctx->d_widen, (kWidenCounterWords + 32) * sizeof(uint32_t)) != cudaSuccess ||
      cudaMemset(ctx->d_widen, 0, (kWidenCounterWords + 32) * sizeof(uint32_t)) != cudaSuccess ||
      cudaMalloc(&ctx->d_skinny, kSkinnyCounterWords * sizeof(uint32_t)) != cudaSuccess ||
      cudaMemset(ctx->d_skinny, 0, kSkinnyCounterWords * sizeof(uint32_t)) != cudaSuccess) {
    cudaGetLastError();
    if (ctx->d_err) cudaFree(ctx->d_err);
    if (ctx->d_widen) cudaFree(ctx->d_widen);
    if (ctx->d_skinny) cudaFree(ctx->d_skinny);
    delete ctx;
    return SC_OUT_OF_MEMORY;
  }
  *out = ctx;
  return SC_OK;
}

void sc_ctx_destroy(sc_ctx* ctx) {
  if (ctx == nullptr) return;
  int cur = -1;
  cudaGetDevice(&cur);
  cudaSetDevice(ctx->device);
  if (ctx->d_err) cudaFree(ctx->d_err);
  if (ctx->d_widen) cudaFree(ctx->d_widen);
  if (ctx->d_skinny) cudaFree(ctx->d_skinny);
  if (ctx->widen_guard.event) cudaEventDestroy(ctx->widen_guard.event);
  if (ctx->skinny_guard.event) cudaEventDestroy(ctx->skinny_guard.event);
  for (cudaEvent_t e : ctx->host_events)
    if (e) cudaEventDestroy(e);
  if (ctx->copy_in) cudaStreamDestroy(ctx->copy_in);
  if (ctx->copy_out) cudaStreamDestroy(ctx->copy_out);
  if (cur >= 0) cudaSetDevice(cur);
  delete ctx;
}

const char* sc_last_error_string(const sc_ctx* ctx) { return ctx ? ctx->last_error.c_str() : "null context"; }

sc_status sc_weight_create_shard(sc_ctx* ctx, const void* values, sc_weight_kind kind, int64_t k, int64_t n,
                                 const void* scales, sc_scale_type scale_type, sc_scale_layout layout, uint32_t flags,
                                 int64_t n_begin, int64_t n_end, void* stream, sc_weight** out) {
  if (ctx == nullptr) return SC_INVALID_ARG;
  if (out == nullptr || values == nullptr || scales == nullptr) return fail(ctx, SC_INVALID_ARG, "null argument");
  *out = nullptr;
  if (kind != SC_WEIGHT_INT8 && kind != SC_WEIGHT_E4M3) return fail(ctx, SC_INVALID_ARG, "unknown weight kind");
  if (scale_type != SC_SCALE_F32 && scale_type != SC_SCALE_BF16 && scale_type != SC_SCALE_F16)
    return fail(ctx, SC_INVALID_ARG, "unknown scale type");
  if (layout != SC_SCALE_TENSOR && layout != SC_SCALE_COLUMNS) return fail(ctx, SC_INVALID_ARG, "unknown scale layout");
  if (flags & ~(SC_WEIGHT_VALUES_ON_DEVICE | SC_WEIGHT_PUBLISHED_NK | SC_WEIGHT_ARENA_LAYOUT | SC_WEIGHT_NAN_CODES))
    return fail(ctx, SC_INVALID_ARG, "unknown flags");
  if (k <= 0 || n <= 0) return fail(ctx, SC_INVALID_ARG, "k and n must be positive");
  if (n_begin < 0 || n_end > n || n_begin >= n_end) return fail(ctx, SC_INVALID_ARG, "bad column range");
  const bool arena_layout = (flags & SC_WEIGHT_ARENA_LAYOUT) != 0;
  if (arena_layout && ((flags & SC_WEIGHT_PUBLISHED_NK) || n_begin != 0 || n_end != n))
    return fail(ctx, SC_INVALID_ARG, "the arena layout is the whole weight's, not a published [N, K] nor a shard");
  if ((flags & SC_WEIGHT_NAN_CODES) && !arena_layout)
    return fail(ctx, SC_INVALID_ARG, "SC_WEIGHT_NAN_CODES goes with SC_WEIGHT_ARENA_LAYOUT");
  sc_status s = enter(ctx);
  if (s != SC_OK) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool on_device = (flags & SC_WEIGHT_VALUES_ON_DEVICE) != 0;
  const bool published = (flags & SC_WEIGHT_PUBLISHED_NK) != 0;
  const int64_t cols = n_end - n_begin;

  // Scales: widened exactly to fp32, checked, padded.
  const int64_t scount = layout == SC_SCALE_TENSOR ? 1 : n;
  std::vector<uint8_t> sbytes(static_cast<size_t>(scount) * scale_size(scale_type));
  if (on_device) {
    if ((s = check_cuda(ctx, cudaMemcpy(sbytes.data(), scales, sbytes.size(), cudaMemcpyDeviceToHost), "scales to host")) != SC_OK)
      return s;
  } else {
    std::memcpy(sbytes.data(), scales, sbytes.size());
  }
  const float smallest = kind == SC_WEIGHT_INT8 ? 1.0f : std::ldexp(1.0f, -9);
  for (int64_t i = 0; i < scount; ++i) {
    const float v = scale_to_f32(sbytes.data(), scale_type, i);
    if (v != 0.0f && std::fabs(v) * smallest < FLT_MIN) {
      char msg[160];
      std::snprintf(msg, sizeof msg, "scale %lld = %g: its products can fall below 2^-126 (subnormal)",
                    static_cast<long long>(i), static_cast<double>(v));
      return fail(ctx, SC_REFUSED, msg);
    }
  }
  sc_weight* w = new (std::nothrow) sc_weight();
  if (w == nullptr) return fail(ctx, SC_OUT_OF_MEMORY, "host allocation");
  w->kind = kind;
  w->k = k;
  w->n = cols;
  w->k_pad = round_up(k, kArenaKAlign);
  w->n_pad = round_up(cols, kArenaNAlign);
  w->device = ctx->device;
  std::vector<float> sf(static_cast<size_t>(w->n_pad), 0.0f);
  for (int64_t j = 0; j < cols; ++j)
    sf[static_cast<size_t>(j)] = scale_to_f32(sbytes.data(), scale_type, layout == SC_SCALE_TENSOR ? 0 : n_begin + j);
  for (int64_t j = 0; j < cols; ++j) {
    const float a = std::fabs(sf[static_cast<size_t>(j)]);
    if (a != 0.0f && (w->min_abs_scale == 0.0f || a < w->min_abs_scale)) w->min_abs_scale = a;
  }

  const size_t vbytes = static_cast<size_t>(w->n_pad * w->k_pad);
  const size_t soff = static_cast<size_t>(round_up(static_cast<int64_t>(vbytes), 256));
  w->bytes = soff + static_cast<size_t>(w->n_pad) * sizeof(float);
  auto cleanup = [&](sc_status st_) {
    if (w->arena) cudaFree(w->arena);
    delete w;
    return st_;
  };
  if (arena_layout) {
    // The codes already lie as the arena keeps them: on the host they are checked here (K and N padding
    // the code of zero, so that no padded product can be a NaN; NaN codes of e4m3 found), then copied once.
    const uint8_t* v = static_cast<const uint8_t*>(values);
    const uint8_t zero = kind == SC_WEIGHT_INT8 ? kPadInt8 : kPadE4M3;
    bool nan_codes = (flags & SC_WEIGHT_NAN_CODES) != 0;
    if (!on_device) {
      nan_codes = false;
      for (int64_t r = 0; r < w->n_pad; ++r) {
        const uint8_t* row = v + r * w->k_pad;
        for (int64_t c = (r < cols ? k : 0); c < w->k_pad; ++c)
          if (row[c] != zero) {
            delete w;
            return fail(ctx, SC_INVALID_ARG, "arena layout: a padding code that is not the code of zero");
          }
        if (kind == SC_WEIGHT_E4M3 && r < cols && !nan_codes)
          for (int64_t c = 0; c < k; ++c)
            if ((row[c] & 0x7Fu) == 0x7Fu) {
              nan_codes = true;
              break;
            }
      }
    }
    if ((s = check_cuda(ctx, cudaMalloc(&w->arena, w->bytes), "weight arena")) != SC_OK) return cleanup(s);
    w->values = w->arena;
    w->scales = reinterpret_cast<float*>(w->arena + soff);
    cudaError_t e = cudaMemcpyAsync(w->values, v, vbytes, on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(w->scales, sf.data(), sf.size() * sizeof(float), cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if ((s = check_cuda(ctx, e, "arena upload")) != SC_OK) return cleanup(s);
    w->has_nan_codes = kind == SC_WEIGHT_E4M3 && nan_codes;
    if ((s = make_tmap_w(ctx, w)) != SC_OK) return cleanup(s);
    *out = w;
    return SC_OK;
  }
  if ((s = check_cuda(ctx, cudaMalloc(&w->arena, w->bytes), "weight arena")) != SC_OK) return cleanup(s);
  w->values = w->arena;
  w->scales = reinterpret_cast<float*>(w->arena + soff);

  // Source codes on the device: the caller's, or a staging copy of the needed part.
  uint8_t* staging = nullptr;
  int* nan_flag = nullptr;
  const uint8_t* src = static_cast<const uint8_t*>(values);
  int64_t src_n_total = n, src_n_begin = n_begin;
  if (!on_device) {
    if ((s = check_cuda(ctx, cudaMalloc(&staging, static_cast<size_t>(k * cols) + 16), "staging")) != SC_OK)
      return cleanup(s);
    cudaError_t e;
    if (published)  // rows [n_begin, n_end) of [N, K] are contiguous
      e = cudaMemcpyAsync(staging, src + n_begin * k, static_cast<size_t>(k * cols), cudaMemcpyHostToDevice, st);
    else  // columns [n_begin, n_end) of [K, N]: a pitched copy
      e = cudaMemcpy2DAsync(staging, static_cast<size_t>(cols), src + n_begin, static_cast<size_t>(n),
                            static_cast<size_t>(cols), static_cast<size_t>(k), cudaMemcpyHostToDevice, st);
    if ((s = check_cuda(ctx, e, "weight upload")) != SC_OK) {
      cudaFree(staging);
      return cleanup(s);
    }
    src = staging;
    src_n_total = cols;
    src_n_begin = 0;
  }
  cudaError_t e = cudaMalloc(&nan_flag, sizeof(int));
  if (e == cudaSuccess) e = cudaMemsetAsync(nan_flag, 0, sizeof(int), st);
  if (e == cudaSuccess)
    e = launch_retile(src, published, kind, k, src_n_total, src_n_begin, cols, w->values, w->k_pad, w->n_pad, nan_flag, st);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(w->scales, sf.data(), sf.size() * sizeof(float), cudaMemcpyHostToDevice, st);
  int nan_host = 0;
  if (e == cudaSuccess) e = cudaMemcpyAsync(&nan_host, nan_flag, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (staging) cudaFree(staging);
  if (nan_flag) cudaFree(nan_flag);
  if ((s = check_cuda(ctx, e, "weight re-tiling")) != SC_OK) return cleanup(s);
  w->has_nan_codes = nan_host != 0;
  if ((s = make_tmap_w(ctx, w)) != SC_OK) return cleanup(s);
  *out = w;
  return SC_OK;
}

sc_status sc_weight_create(sc_ctx* ctx, const void* values, sc_weight_kind kind, int64_t k, int64_t n,
                           const void* scales, sc_scale_type scale_type, sc_scale_layout layout, uint32_t flags,
                           void* stream, sc_weight** out) {
  return sc_weight_create_shard(ctx, values, kind, k, n, scales, scale_type, layout, flags, 0, n, stream, out);
}

sc_status sc_weight_destroy(sc_ctx* ctx, sc_weight* w) {
  if (ctx == nullptr) return SC_INVALID_ARG;
  if (w == nullptr) return SC_OK;
  int cur = -1;
  cudaGetDevice(&cur);
  if (cur != w->device) cudaSetDevice(w->device);
  const cudaError_t e = cudaFree(w->arena);
  if (cur >= 0 && cur != w->device) cudaSetDevice(cur);
  delete w;
  return check_cuda(ctx, e, "cudaFree (weight arena)");
}

sc_status sc_weight_info(const sc_weight* w, int64_t* k, int64_t* n, int* kind, size_t* device_bytes) {
  if (w == nullptr) return SC_INVALID_ARG;
  if (k) *k = w->k;
  if (n) *n = w->n;
  if (kind) *kind = w->kind;
  if (device_bytes) *device_bytes = w->bytes;
  return SC_OK;
}

sc_status sc_dequantize(sc_ctx* ctx, const sc_weight* w, float* out, void* stream) {
  if (ctx == nullptr) return SC_INVALID_ARG;
  if (w == nullptr || out == nullptr) return fail(ctx, SC_INVALID_ARG, "null weight or output");
  if (!is_device_pointer(out)) return fail(ctx, SC_INVALID_ARG, "out must be device (or managed) memory");
  sc_status s = enter(ctx);
  if (s != SC_OK) return s;
  if (w->rotation != 0)
    return check_cuda(ctx, launch_dequantize_rotated(w, out, static_cast<cudaStream_t>(stream)),
                      "rotated dequantize launch");
  return check_cuda(ctx, launch_dequantize(w, out, static_cast<cudaStream_t>(stream)), "dequantize launch");
}

sc_status sc_w8a8_workspace_size(sc_ctx* ctx, const sc_weight* w, int64_t m, size_t* bytes) {
  if (ctx == nullptr) return SC_INVALID_ARG;
  if (w == nullptr || bytes == nullptr || m < 0) return fail(ctx, SC_INVALID_ARG, "bad argument");
  *bytes = m == 0 ? 0 : w8a8_workspace(w, m);
  return SC_OK;
}

sc_status sc_quantize_rows(sc_ctx* ctx, const void* x, sc_in_type x_type, int64_t m, int64_t k, int group,
                           int8_t* codes, int64_t ld, float* scales, void* stream) {
  if (ctx == nullptr) return SC_INVALID_ARG;
  if (x_type != SC_IN_BF16 && x_type != SC_IN_F32) return fail(ctx, SC_INVALID_ARG, "unknown input type");
  if (m < 0 || k <= 0) return fail(ctx, SC_INVALID_ARG, "m < 0 or k <= 0");
  if (group != 0 && (!is_rotation_group(group) || k % group != 0))
    return fail(ctx, SC_UNSUPPORTED_SHAPE, "group must be 0 or a power of 4 from 4 to 256 dividing K");
  if (k % 8 != 0 || k > kW8A8MaxK) return fail(ctx, SC_UNSUPPORTED_SHAPE, "K must be a multiple of 8, at most 32768");
  if (ld < k || ld % 16 != 0) return fail(ctx, SC_INVALID_ARG, "ld must be at least K and a multiple of 16");
  if (m == 0) return SC_OK;
  if (x == nullptr || codes == nullptr || scales == nullptr) return fail(ctx, SC_INVALID_ARG, "null argument");
  if (((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(codes)) & 15u) ||
      (reinterpret_cast<uintptr_t>(scales) & 3u))
    return fail(ctx, SC_UNALIGNED, "x and codes must be 16-byte aligned, scales 4-byte aligned");
  if (!is_device_pointer(x) || !is_device_pointer(codes) || !is_device_pointer(scales))
    return fail(ctx, SC_INVALID_ARG, "x, codes and scales must be device memory");
  sc_status s = enter(ctx);
  if (s != SC_OK) return s;
  return check_cuda(ctx, launch_quantize_rows(x, x_type == SC_IN_F32, m, k, group, codes, ld, scales,
                                              static_cast<cudaStream_t>(stream)),
                    "quantize launch");
}

sc_status sc_linear_w8a8(sc_ctx* ctx, const sc_weight* w, const void* x, sc_in_type x_type, int64_t m,
                         const sc_bf16* bias, void* y, sc_out_type y_type, void* workspace, size_t workspace_bytes,
                         void* stream) {
  if (ctx == nullptr) return SC_INVALID_ARG;
  if (w == nullptr) return fail(ctx, SC_INVALID_ARG, "null weight");
  if (w->kind != SC_WEIGHT_INT8) return fail(ctx, SC_INVALID_ARG, "W8A8 reads int8 weights only");
  if (x_type != SC_IN_BF16 && x_type != SC_IN_F32) return fail(ctx, SC_INVALID_ARG, "unknown input type");
  if (y_type != SC_OUT_BF16 && y_type != SC_OUT_F32) return fail(ctx, SC_INVALID_ARG, "unknown output type");
  if (m < 0) return fail(ctx, SC_INVALID_ARG, "m < 0");
  if (m == 0) return SC_OK;
  if (x == nullptr || y == nullptr) return fail(ctx, SC_INVALID_ARG, "null x or y");
  if (m > 0x7FFFFFFF) return fail(ctx, SC_UNSUPPORTED_SHAPE, "m beyond 2^31 - 1");
  if (w->k % 8 != 0 || w->k > kW8A8MaxK) return fail(ctx, SC_UNSUPPORTED_SHAPE, "K must be a multiple of 8, at most 32768");
  if (w->device != ctx->device) return fail(ctx, SC_INVALID_ARG, "weight registered on another device");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15u)
    return fail(ctx, SC_UNALIGNED, "x and y must be 16-byte aligned");
  if (bias != nullptr && (reinterpret_cast<uintptr_t>(bias) & 1u)) return fail(ctx, SC_UNALIGNED, "bias must be 2-byte aligned");
  if (!is_device_pointer(x) || !is_device_pointer(y) || (bias != nullptr && !is_device_pointer(bias)))
    return fail(ctx, SC_INVALID_ARG, "x, y and bias must be device (or managed) memory");
  if (workspace == nullptr || workspace_bytes < w8a8_workspace(w, m) || (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return fail(ctx, SC_WORKSPACE_TOO_SMALL, "W8A8 needs a 256-byte aligned workspace of sc_w8a8_workspace_size bytes");
  sc_status s = enter(ctx);
  if (s != SC_OK) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* wsigned = static_cast<uint8_t*>(workspace);
  const int64_t ld = w8a8_ld(w->k);
  int8_t* codes = reinterpret_cast<int8_t*>(wsigned + align256(signed_codes_bytes(w)));
  float* sx = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(codes) + align256(static_cast<size_t>(m * ld)));
  if ((s = check_cuda(ctx, launch_sign_codes(w, wsigned, st), "sign launch")) != SC_OK) return s;
  if ((s = check_cuda(ctx, launch_quantize_rows(x, x_type == SC_IN_F32, m, w->k, w->rotation, codes, ld, sx, st),
                      "quantize launch")) != SC_OK)
    return s;
  CUtensorMap tmx, tmw;
  if ((s = make_tmap_codes(ctx, codes, w->k, m, ld, &tmx)) != SC_OK) return s;
  if ((s = make_tmap_codes(ctx, wsigned, w->k_pad, w->n_pad, w->k_pad, &tmw)) != SC_OK) return s;
  return check_cuda(ctx, launch_gemm_i8(tmx, tmw, w, bias, y, y_type == SC_OUT_F32, sx, m, ctx->d_err, ctx->sm_count, st),
                    "int8 gemm launch");
}

sc_status sc_weight_set_rotation(sc_ctx* ctx, sc_weight* w, int group) {
  if (ctx == nullptr) return SC_INVALID_ARG;
  if (w == nullptr) return fail(ctx, SC_INVALID_ARG, "null weight");
  if (group == 0) {
    w->rotation = 0;
    return SC_OK;
  }
  if (w->kind != SC_WEIGHT_INT8) return fail(ctx, SC_INVALID_ARG, "convrot is read on int8 weights only");
  if (!is_rotation_group(group))
    return fail(ctx, SC_UNSUPPORTED_SHAPE, "convrot group must be a power of 4 from 4 to 256");
  if (w->k % group != 0) return fail(ctx, SC_UNSUPPORTED_SHAPE, "K must be a multiple of the convrot group");
  int p = 0;
  while ((1 << (2 * p)) < group) ++p;
  if (w->min_abs_scale != 0.0f && std::ldexp(w->min_abs_scale, -p) < FLT_MIN)
    return fail(ctx, SC_REFUSED, "a scale over sqrt(G) is subnormal: its rotated products can fall below 2^-126");
  w->rotation = group;
  return SC_OK;
}

sc_status sc_rotate_activation(sc_ctx* ctx, const sc_bf16* x, int64_t m, int64_t k, int group, sc_bf16* out,
                               void* stream) {
  if (ctx == nullptr) return SC_INVALID_ARG;
  if (m < 0 || k <= 0) return fail(ctx, SC_INVALID_ARG, "m < 0 or k <= 0");
  if (!is_rotation_group(group)) return fail(ctx, SC_UNSUPPORTED_SHAPE, "group must be a power of 4 from 4 to 256");
  if (k % group != 0 || k % 8 != 0) return fail(ctx, SC_UNSUPPORTED_SHAPE, "K must be a multiple of the group and of 8");
  if (m == 0) return SC_OK;
  if (x == nullptr || out == nullptr) return fail(ctx, SC_INVALID_ARG, "null x or out");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15u)
    return fail(ctx, SC_UNALIGNED, "x and out must be 16-byte aligned");
  if (!is_device_pointer(x) || !is_device_pointer(out)) return fail(ctx, SC_INVALID_ARG, "x and out must be device memory");
  sc_status s = enter(ctx);
  if (s != SC_OK) return s;
  return check_cuda(ctx, launch_rotate(x, m, k, group, out, static_cast<cudaStream_t>(stream)), "rotation launch");
}

sc_status sc_workspace_size(sc_ctx* ctx, const sc_weight* w, int64_t m, size_t* bytes) {
  if (ctx == nullptr) return SC_INVALID_ARG;
  if (w == nullptr || bytes == nullptr || m < 0) return fail(ctx, SC_INVALID_ARG, "bad argument");
  if (m > kSkinnyI8MinRows && m <= kSkinnyMinRows && skinny_i8_grid(w, m, ctx->sm_count) > 0) {
    *bytes = skinny_i8_workspace_bytes(w, m, skinny_i8_grid(w, m, ctx->sm_count));
  } else if (m > kSkinnyMinRows && m <= 32) {
    const int grid = skinny_i8_grid(w, m, ctx->sm_count);
    *bytes = grid > 0 ? skinny_i8_workspace_bytes(w, m, grid) : 0;
  } else if (m >= 1 && m <= 32) {
    *bytes = gemv_workspace_bytes(w, m, ctx->sm_count);
  }
  else if (m >= kWidenMinRows) *bytes = widened_bytes(w);
  else *bytes = 0;
  if (w->rotation != 0 && m >= 1) *bytes += rotated_x_bytes(m, w->k);  // the rotated x comes first
  return SC_OK;
}

sc_status sc_linear(sc_ctx* ctx, const sc_weight* w, const sc_bf16* x, int64_t m, const sc_bf16* bias, sc_bf16* y,
                    void* workspace, size_t workspace_bytes, void* stream) {
  return run_linear(ctx, w, x, m, bias, y, false, workspace, workspace_bytes, stream, 0);
}

sc_status sc_linear_ex(sc_ctx* ctx, const sc_weight* w, const sc_bf16* x, int64_t m, const sc_bf16* bias, void* y,
                       sc_out_type y_type, void* workspace, size_t workspace_bytes, void* stream) {
  if (ctx == nullptr) return SC_INVALID_ARG;
  if (y_type != SC_OUT_BF16 && y_type != SC_OUT_F32) return fail(ctx, SC_INVALID_ARG, "unknown output type");
  return run_linear(ctx, w, x, m, bias, y, y_type == SC_OUT_F32, workspace, workspace_bytes, stream, 0);
}

// sc_linear_host: the rows in chunks, each chunk's copy in, product and copy out on three streams.
constexpr int kHostMaxChunks = 32;

sc_status sc_linear_host(sc_ctx* ctx, const sc_weight* w, const sc_bf16* x_host, int64_t m, const sc_bf16* bias,
                         void* y_host, sc_out_type y_type, sc_bf16* x_dev, void* y_dev, void* workspace,
                         size_t workspace_bytes, int64_t chunk_rows, void* stream) {
  if (ctx == nullptr) return SC_INVALID_ARG;
  if (w == nullptr) return fail(ctx, SC_INVALID_ARG, "null weight");
  if (y_type != SC_OUT_BF16 && y_type != SC_OUT_F32) return fail(ctx, SC_INVALID_ARG, "unknown output type");
  if (m < 0 || chunk_rows < 0) return fail(ctx, SC_INVALID_ARG, "m < 0 or chunk_rows < 0");
  if (m == 0) return SC_OK;
  if (x_host == nullptr || y_host == nullptr) return fail(ctx, SC_INVALID_ARG, "null host buffer");
  // y_dev NULL: the products write y_host themselves (page-locked host memory the GPU can address), so
  // no copy back is queued and the output crosses PCIe while the tiles are computed.
  const bool direct_out = y_dev == nullptr;
  void* y_out = y_dev;
  if (direct_out) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, y_host) != cudaSuccess || a.type != cudaMemoryTypeHost || a.devicePointer == nullptr) {
      cudaGetLastError();
      return fail(ctx, SC_INVALID_ARG, "y_dev NULL needs a page-locked y_host the GPU can address");
    }
    y_out = a.devicePointer;
    if (w->rotation != 0 || workspace == nullptr || workspace_bytes < widened_bytes(w) ||
        (reinterpret_cast<uintptr_t>(workspace) & 255u))
      return fail(ctx, SC_WORKSPACE_TOO_SMALL,
                  "y_dev NULL needs the widened route: a 256-byte aligned workspace of n_pad * k_pad * 2 bytes");
  }
  sc_status s = check_product_args(ctx, w, x_dev, m, bias, direct_out ? static_cast<void*>(x_dev) : y_dev);
  if (s != SC_OK) return s;
  if ((reinterpret_cast<uintptr_t>(y_out) & 15u)) return fail(ctx, SC_UNALIGNED, "y must be 16-byte aligned");
  if ((s = enter(ctx)) != SC_OK) return s;
  if (ctx->copy_in == nullptr) {
    if ((s = check_cuda(ctx, cudaStreamCreateWithFlags(&ctx->copy_in, cudaStreamNonBlocking), "copy stream")) != SC_OK ||
        (s = check_cuda(ctx, cudaStreamCreateWithFlags(&ctx->copy_out, cudaStreamNonBlocking), "copy stream")) != SC_OK)
      return s;
    for (cudaEvent_t& e : ctx->host_events)
      if ((s = check_cuda(ctx, cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "event")) != SC_OK) return s;
  }
  // Chunks of whole 256-row pair tiles, at least 512 rows, at most kHostMaxChunks of them; a remainder
  // of 128 rows or fewer joins the chunk before it, so that every chunk of a split batch runs the pair
  // GEMM and each row comes out with the bits the whole batch would give it.
  // The default: four chunks.  On B200 over PCIe, chunks of 1024 rows of config 1 (6.3 MB each way) took
  // 0.75 ms a step against 0.99 ms unchunked and 0.84 ms with eight chunks (each copy and each cross-stream
  // wait costs a few tens of microseconds; both directions at once move 50 MB in 0.51 ms at best).
  // Writing y directly (no copy back), eight chunks: each chunk's product overlaps the next chunk's copy in.
  int64_t chunk = chunk_rows > 0 ? chunk_rows : (direct_out ? (m + 7) / 8 : (m + 3) / 4);
  chunk = (chunk + 255) / 256 * 256;
  if (chunk < 512) chunk = 512;
  if ((m + chunk - 1) / chunk > kHostMaxChunks) chunk = ((m + kHostMaxChunks - 1) / kHostMaxChunks + 255) / 256 * 256;
  int64_t starts[kHostMaxChunks + 1];
  int chunks = 0;
  for (int64_t r = 0; r < m; r += chunk) starts[chunks++] = r;
  if (chunks > 1 && m - starts[chunks - 1] <= kPairMinRows) --chunks;
  starts[chunks] = m;
  const size_t ysz = y_type == SC_OUT_F32 ? 4 : 2;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaEvent_t* ev_in = ctx->host_events;
  cudaEvent_t* ev_out = ctx->host_events + kHostMaxChunks;
  cudaEvent_t ev_start = ctx->host_events[2 * kHostMaxChunks], ev_end = ctx->host_events[2 * kHostMaxChunks + 1];
  // The copies start after the caller's earlier work on `stream`.
  if ((s = check_cuda(ctx, cudaEventRecord(ev_start, st), "event record")) != SC_OK ||
      (s = check_cuda(ctx, cudaStreamWaitEvent(ctx->copy_in, ev_start, 0), "stream wait")) != SC_OK ||
      (s = check_cuda(ctx, cudaStreamWaitEvent(ctx->copy_out, ev_start, 0), "stream wait")) != SC_OK)
    return s;
  // Every copy in is queued first, so that they run back to back whatever the host takes to queue the
  // products (a few microseconds each: argument checks, tensor maps, launches).
  for (int c = 0; c < chunks; ++c) {
    const int64_t r0 = starts[c], rows = starts[c + 1] - starts[c];
    if ((s = check_cuda(ctx, cudaMemcpyAsync(x_dev + r0 * w->k, x_host + r0 * w->k,
                                             static_cast<size_t>(rows * w->k) * 2, cudaMemcpyHostToDevice, ctx->copy_in),
                        "copy in")) != SC_OK ||
        (s = check_cuda(ctx, cudaEventRecord(ev_in[c], ctx->copy_in), "event record")) != SC_OK)
      return s;
  }
  // With room for the widened weight (and no rotation to stage), the codes are widened once, while the
  // first chunk arrives, and every chunk runs the bf16-operand pair GEMM on them: the widened route's
  // bits, without widening per chunk.  Otherwise each chunk is an ordinary product.
  const bool widen_once = (chunks > 1 || direct_out) && w->rotation == 0 && workspace != nullptr &&
                          workspace_bytes >= widened_bytes(w) && (reinterpret_cast<uintptr_t>(workspace) & 255u) == 0;
  CUtensorMap tmw;
  if (widen_once) {
    if ((s = make_tmap_widened(ctx, w, workspace, &tmw)) != SC_OK) return s;
    if ((s = check_cuda(ctx, launch_widen(w, workspace, ctx->sm_count, st), "widen launch")) != SC_OK) return s;
  }
  for (int c = 0; c < chunks; ++c) {
    const int64_t r0 = starts[c], rows = starts[c + 1] - starts[c];
    if ((s = check_cuda(ctx, cudaStreamWaitEvent(st, ev_in[c], 0), "stream wait")) != SC_OK) return s;
    void* yc = static_cast<uint8_t*>(y_out) + static_cast<size_t>(r0 * w->n) * ysz;
    if (widen_once) {
      CUtensorMap tmx;
      if ((s = make_tmap_x(ctx, x_dev + r0 * w->k, rows, w->k, &tmx)) != SC_OK) return s;
      if ((s = check_cuda(ctx, launch_gemm_bf16(tmx, tmw, w, bias, yc, y_type == SC_OUT_F32, rows, ctx->d_err,
                                                ctx->sm_count, st),
                          "bf16 pair gemm launch")) != SC_OK)
        return s;
    } else if ((s = run_linear(ctx, w, x_dev + r0 * w->k, rows, bias, yc, y_type == SC_OUT_F32, workspace,
                               workspace_bytes, stream, 0)) != SC_OK) {
      return s;
    }
    if (direct_out) continue;
    if ((s = check_cuda(ctx, cudaEventRecord(ev_out[c], st), "event record")) != SC_OK ||
        (s = check_cuda(ctx, cudaStreamWaitEvent(ctx->copy_out, ev_out[c], 0), "stream wait")) != SC_OK ||
        (s = check_cuda(ctx, cudaMemcpyAsync(static_cast<uint8_t*>(y_host) + static_cast<size_t>(r0 * w->n) * ysz, yc,
                                             static_cast<size_t>(rows * w->n) * ysz, cudaMemcpyDeviceToHost,
                                             ctx->copy_out),
                        "copy out")) != SC_OK)
      return s;
  }
  if (direct_out) return SC_OK;  // the products on `stream` wrote y_host themselves
  // The caller's stream holds until the last copy out is done.
  if ((s = check_cuda(ctx, cudaEventRecord(ev_end, ctx->copy_out), "event record")) != SC_OK) return s;
  return check_cuda(ctx, cudaStreamWaitEvent(st, ev_end, 0), "stream wait");
}

sc_status sc_linear_qk_norm_rope(sc_ctx* ctx, const sc_weight* w, const sc_bf16* x, int64_t m, const sc_bf16* bias,
                                 sc_bf16* q, sc_bf16* k, sc_bf16* v, int heads, int64_t tokens, int64_t joint,
                                 int64_t offset, const float* norm_q, const float* norm_k, const float* freqs,
                                 float eps, void* workspace, size_t workspace_bytes, void* stream) {
  sc_status s = check_product_args(ctx, w, x, m, bias, q);
  if (s != SC_OK) return s;
  if (m == 0) return SC_OK;
  if (heads < 1 || w->n != 3LL * heads * 128) return fail(ctx, SC_UNSUPPORTED_SHAPE, "N must be 3 * heads * 128");
  if (tokens < 1 || m % tokens != 0 || offset < 0 || joint < offset + tokens || joint > 0x7FFFFFFF)
    return fail(ctx, SC_INVALID_ARG, "m must be images * tokens and offset + tokens <= joint");
  if (k == nullptr || v == nullptr || norm_q == nullptr || norm_k == nullptr || freqs == nullptr)
    return fail(ctx, SC_INVALID_ARG, "null output, norm weight or frequency table");
  if ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 15u ||
      (reinterpret_cast<uintptr_t>(norm_q) | reinterpret_cast<uintptr_t>(norm_k) | reinterpret_cast<uintptr_t>(freqs)) & 3u)
    return fail(ctx, SC_UNALIGNED, "q, k, v must be 16-byte aligned, the fp32 tables 4-byte aligned");
  if (!is_device_pointer(k) || !is_device_pointer(v) || !is_device_pointer(norm_q) || !is_device_pointer(norm_k) ||
      !is_device_pointer(freqs))
    return fail(ctx, SC_INVALID_ARG, "outputs and tables must be device memory");
  if (m <= kPairMinRows) return fail(ctx, SC_UNSUPPORTED_SHAPE, "sc_linear_qk_norm_rope takes more than 128 rows");
  const size_t rx = w->rotation != 0 ? rotated_x_bytes(m, w->k) : 0;
  if (workspace == nullptr || workspace_bytes < rx + widened_bytes(w) || (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return fail(ctx, SC_WORKSPACE_TOO_SMALL,
                "sc_linear_qk_norm_rope needs a 256-byte aligned workspace of n_pad * k_pad * 2 bytes (+ the rotated x)");
  if ((s = enter(ctx)) != SC_OK) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((s = rotate_operand(ctx, w, x, m, workspace, workspace_bytes, st)) != SC_OK) return s;
  CUtensorMap tmx, tmw;
  if ((s = make_tmap_x(ctx, x, m, w->k, &tmx)) != SC_OK) return s;
  if ((s = make_tmap_widened(ctx, w, workspace, &tmw)) != SC_OK) return s;
  if ((s = check_cuda(ctx, launch_widen(w, workspace, ctx->sm_count, st), "widen launch")) != SC_OK) return s;
  HeadOut ho;
  ho.q = q;
  ho.k = k;
  ho.v = v;
  ho.norm_q = norm_q;
  ho.norm_k = norm_k;
  ho.freqs = freqs;
  ho.eps = eps;
  ho.heads = heads;
  ho.tokens = static_cast<int>(tokens);
  ho.joint = static_cast<int>(joint);
  ho.offset = static_cast<int>(offset);
  return check_cuda(ctx, launch_gemm_bf16_heads(tmx, tmw, w, bias, ho, m, ctx->d_err, ctx->sm_count, st),
                    "qk-norm gemm launch");
}

sc_status sc_linear_heads(sc_ctx* ctx, const sc_weight* w, const sc_bf16* o, int64_t batch, int heads, int64_t joint,
                          int64_t offset, int64_t tokens, const sc_bf16* bias, void* y, sc_out_type y_type,
                          sc_epilogue op, const float* gate, void* workspace, size_t workspace_bytes, void* stream) {
  if (ctx == nullptr) return SC_INVALID_ARG;
  if (w == nullptr || o == nullptr || y == nullptr) return fail(ctx, SC_INVALID_ARG, "null weight, o or y");
  if (y_type != SC_OUT_BF16 && y_type != SC_OUT_F32) return fail(ctx, SC_INVALID_ARG, "unknown output type");
  if (op != 0 && op != SC_EPI_GATED_RESIDUAL) return fail(ctx, SC_INVALID_ARG, "epilogue: none or the gated residual");
  if (op == SC_EPI_GATED_RESIDUAL && (y_type != SC_OUT_F32 || gate == nullptr || !is_device_pointer(gate) ||
                                      (reinterpret_cast<uintptr_t>(gate) & 3u)))
    return fail(ctx, SC_INVALID_ARG, "the gated residual needs an fp32 y and a 4-byte aligned device gate");
  if (batch < 1 || heads < 1 || tokens < 1 || offset < 0 || offset + tokens > joint || joint > 0x7FFFFFFF)
    return fail(ctx, SC_INVALID_ARG, "batch, heads, tokens >= 1 and offset + tokens <= joint");
  if (tokens % 128 != 0) return fail(ctx, SC_UNSUPPORTED_SHAPE, "tokens must be a multiple of 128");
  if (w->k != 128LL * heads) return fail(ctx, SC_UNSUPPORTED_SHAPE, "K must be heads * 128");
  if (w->rotation != 0) return fail(ctx, SC_UNSUPPORTED_SHAPE, "a convrot weight takes its operand through sc_linear");
  if (w->device != ctx->device) return fail(ctx, SC_INVALID_ARG, "weight registered on another device");
  const int64_t m = batch * tokens;
  if (m <= kPairMinRows || m > 0x7FFFFFFF) return fail(ctx, SC_UNSUPPORTED_SHAPE, "sc_linear_heads takes more than 128 rows");
  if ((reinterpret_cast<uintptr_t>(o) | reinterpret_cast<uintptr_t>(y)) & 15u ||
      (bias != nullptr && (reinterpret_cast<uintptr_t>(bias) & 1u)))
    return fail(ctx, SC_UNALIGNED, "o and y must be 16-byte aligned, bias 2-byte aligned");
  if (!is_device_pointer(o) || !is_device_pointer(y) || (bias != nullptr && !is_device_pointer(bias)))
    return fail(ctx, SC_INVALID_ARG, "o, y and bias must be device memory");
  if (workspace == nullptr || workspace_bytes < widened_bytes(w) || (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return fail(ctx, SC_WORKSPACE_TOO_SMALL, "sc_linear_heads needs a 256-byte aligned workspace of n_pad * k_pad * 2 bytes");
  sc_status s = enter(ctx);
  if (s != SC_OK) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUtensorMap tmo, tmw;
  if ((s = make_tmap_heads(ctx, o, batch, heads, joint, &tmo)) != SC_OK) return s;
  if ((s = make_tmap_widened(ctx, w, workspace, &tmw)) != SC_OK) return s;
  if ((s = check_cuda(ctx, launch_widen(w, workspace, ctx->sm_count, st), "widen launch")) != SC_OK) return s;
  const XHeads xh = {static_cast<int>(tokens), static_cast<int>(offset)};
  return check_cuda(ctx, launch_gemm_bf16_xheads(tmo, tmw, w, bias, y, y_type == SC_OUT_F32, static_cast<int>(op), gate,
                                                 xh, m, ctx->d_err, ctx->sm_count, st),
                    "heads gemm launch");
}

sc_status sc_linear_epilogue(sc_ctx* ctx, const sc_weight* w, const sc_bf16* x, int64_t m, const sc_bf16* bias,
                             void* y, sc_epilogue op, const float* gate, void* workspace, size_t workspace_bytes,
                             void* stream) {
  sc_status s = check_product_args(ctx, w, x, m, bias, y);
  if (s != SC_OK) return s;
  if (op != SC_EPI_GELU_TANH && op != SC_EPI_GATED_RESIDUAL && op != SC_EPI_SWIGLU)
    return fail(ctx, SC_INVALID_ARG, "unknown epilogue");
  if (op == SC_EPI_SWIGLU && w->n % 256 != 0)
    return fail(ctx, SC_UNSUPPORTED_SHAPE, "SwiGLU needs N a multiple of 256 (blocks of 128 gate, 128 up)");
  if (op == SC_EPI_GATED_RESIDUAL && (gate == nullptr || !is_device_pointer(gate) ||
                                      (reinterpret_cast<uintptr_t>(gate) & 3u)))
    return fail(ctx, SC_INVALID_ARG, "the gated residual needs a 4-byte aligned device gate of n floats");
  if (m == 0) return SC_OK;
  if (m <= kPairMinRows) return fail(ctx, SC_UNSUPPORTED_SHAPE, "sc_linear_epilogue takes more than 128 rows");
  const size_t rx = w->rotation != 0 ? rotated_x_bytes(m, w->k) : 0;
  if (workspace == nullptr || workspace_bytes < rx + widened_bytes(w) || (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return fail(ctx, SC_WORKSPACE_TOO_SMALL,
                "sc_linear_epilogue needs a 256-byte aligned workspace of n_pad * k_pad * 2 bytes (+ the rotated x)");
  if ((s = enter(ctx)) != SC_OK) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((s = rotate_operand(ctx, w, x, m, workspace, workspace_bytes, st)) != SC_OK) return s;
  CUtensorMap tmx, tmw;
  if ((s = make_tmap_x(ctx, x, m, w->k, &tmx)) != SC_OK) return s;
  if ((s = make_tmap_widened(ctx, w, workspace, &tmw)) != SC_OK) return s;
  if ((s = check_cuda(ctx, launch_widen(w, workspace, ctx->sm_count, st), "widen launch")) != SC_OK) return s;
  return check_cuda(ctx, launch_gemm_bf16_op(tmx, tmw, w, bias, y, static_cast<int>(op), gate, m, ctx->d_err,
                                             ctx->sm_count, st),
                    "epilogue gemm launch");
}

sc_status sc_linear_w8(sc_ctx* ctx, const sc_weight* w, const sc_bf16* x, int64_t m, const sc_bf16* bias, sc_bf16* y,
                       void* workspace, size_t workspace_bytes, void* stream) {
  return run_linear(ctx, w, x, m, bias, y, false, workspace, workspace_bytes, stream, SC_WEIGHT_INT8);
}

sc_status sc_linear_fp8(sc_ctx* ctx, const sc_weight* w, const sc_bf16* x, int64_t m, const sc_bf16* bias, sc_bf16* y,
                        void* workspace, size_t workspace_bytes, void* stream) {
  return run_linear(ctx, w, x, m, bias, y, false, workspace, workspace_bytes, stream, SC_WEIGHT_E4M3);
}

sc_status sc_gemv_w8(sc_ctx* ctx, const sc_weight* w, const sc_bf16* x, int64_t m, const sc_bf16* bias, sc_bf16* y,
                     void* workspace, size_t workspace_bytes, void* stream) {
  sc_status s = check_product_args(ctx, w, x, m, bias, y);
  if (s != SC_OK) return s;
  if (m > 32) return fail(ctx, SC_UNSUPPORTED_SHAPE, "sc_gemv_w8 takes at most 32 rows");
  if (m == 0) return SC_OK;
  if ((s = enter(ctx)) != SC_OK) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((s = rotate_operand(ctx, w, x, m, workspace, workspace_bytes, st)) != SC_OK) return s;
  return run_gemv(ctx, w, x, m, bias, y, false, workspace, workspace_bytes, st);
}

sc_status sc_linear_allgather(sc_ctx* ctx, const sc_weight* w, const sc_bf16* x, int64_t m, const sc_bf16* bias,
                              void* const* y_peers, uint32_t* const* flag_peers, int world, int rank, int64_t col0,
                              int64_t n_total, uint32_t epoch, void* workspace, size_t workspace_bytes, void* stream) {
  return sc_linear_allgather_mc(ctx, w, x, m, bias, nullptr, y_peers, flag_peers, world, rank, col0, n_total, epoch,
                                workspace, workspace_bytes, stream);
}

sc_status sc_linear_allgather_mc(sc_ctx* ctx, const sc_weight* w, const sc_bf16* x, int64_t m, const sc_bf16* bias,
                                 void* y_multicast, void* const* y_peers, uint32_t* const* flag_peers, int world,
                                 int rank, int64_t col0, int64_t n_total, uint32_t epoch, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  if (ctx == nullptr) return SC_INVALID_ARG;
  if (w == nullptr || x == nullptr || y_peers == nullptr || flag_peers == nullptr || m < 1)
    return fail(ctx, SC_INVALID_ARG, "null argument or m < 1");
  if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world)
    return fail(ctx, SC_INVALID_ARG, "world must be 1..8 and 0 <= rank < world");
  if (epoch == 0) return fail(ctx, SC_INVALID_ARG, "epoch 0 is reserved (flags start at 0)");
  if (col0 < 0 || col0 % 8 != 0 || n_total % 8 != 0 || col0 + w->n > n_total)
    return fail(ctx, SC_UNSUPPORTED_SHAPE, "columns must be 8-aligned and inside n_total");
  if (m > 0x7FFFFFFF || w->k > 0x7FFFFFFF || w->k % 8 != 0) return fail(ctx, SC_UNSUPPORTED_SHAPE, "bad m or K");
  if (w->device != ctx->device) return fail(ctx, SC_INVALID_ARG, "weight registered on another device");
  if ((reinterpret_cast<uintptr_t>(x) & 15u) || (bias != nullptr && (reinterpret_cast<uintptr_t>(bias) & 1u)))
    return fail(ctx, SC_UNALIGNED, "x must be 16-byte aligned, bias 2-byte aligned");
  PeerOut peers = {};
  for (int r = 0; r < world; ++r) {
    if (y_peers[r] == nullptr || flag_peers[r] == nullptr || (reinterpret_cast<uintptr_t>(y_peers[r]) & 15u) ||
        (reinterpret_cast<uintptr_t>(flag_peers[r]) & 3u))
      return fail(ctx, SC_INVALID_ARG, "every rank needs a 16-byte aligned output and a 4-byte aligned flag array");
    peers.y[r] = y_peers[r];
    peers.flags[r] = flag_peers[r];
  }
  const size_t rx = w->rotation != 0 ? rotated_x_bytes(m, w->k) : 0;
  if (workspace == nullptr || workspace_bytes < rx + widened_bytes(w) || (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return fail(ctx, SC_WORKSPACE_TOO_SMALL,
                "the fused gather needs a 256-byte aligned workspace of n_pad * k_pad * 2 bytes (+ the rotated x)");
  if (reinterpret_cast<uintptr_t>(y_multicast) & 15u) return fail(ctx, SC_UNALIGNED, "the multicast output must be 16-byte aligned");
  peers.y_mc = y_multicast;
  peers.world = world;
  peers.rank = rank;
  peers.col0 = col0;
  peers.ld = n_total;
  peers.epoch = epoch;
  peers.counter = ctx->d_err + kErrWords;
  sc_status s = enter(ctx);
  if (s != SC_OK) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((s = rotate_operand(ctx, w, x, m, workspace, workspace_bytes, st)) != SC_OK) return s;
  CUtensorMap tmx, tmw;
  if ((s = make_tmap_x(ctx, x, m, w->k, &tmx)) != SC_OK) return s;
  if ((s = make_tmap_widened(ctx, w, workspace, &tmw)) != SC_OK) return s;
  if ((s = check_cuda(ctx, launch_widen(w, workspace, ctx->sm_count, st), "widen launch")) != SC_OK) return s;
  return check_cuda(ctx, launch_gemm_bf16_peers(tmx, tmw, w, bias, peers, m, ctx->d_err, ctx->sm_count, st),
                    "gathering gemm launch");
}

sc_status sc_allgather_wait(sc_ctx* ctx, const uint32_t* flags, int world, uint32_t epoch, void* stream) {
  if (ctx == nullptr) return SC_INVALID_ARG;
  if (flags == nullptr || world < 1 || world > kMaxPeers || epoch == 0) return fail(ctx, SC_INVALID_ARG, "bad argument");
  sc_status s = enter(ctx);
  if (s != SC_OK) return s;
  return check_cuda(ctx, launch_gather_wait(flags, world, epoch, ctx->d_err, static_cast<cudaStream_t>(stream)),
                    "gather wait launch");
}

sc_status sc_ipc_handle(sc_ctx* ctx, void* device_ptr, void* handle_out, size_t* offset_out) {
  if (ctx == nullptr) return SC_INVALID_ARG;
  if (device_ptr == nullptr || handle_out == nullptr || offset_out == nullptr)
    return fail(ctx, SC_INVALID_ARG, "null argument");
  sc_status s = enter(ctx);
  if (s != SC_OK) return s;
  // The handle names the whole allocation that holds device_ptr; the offset locates it inside.
  typedef CUresult (*range_fn)(CUdeviceptr*, size_t*, CUdeviceptr);
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || fn == nullptr) {
    cudaGetLastError();
    return fail(ctx, SC_CUDA_ERROR, "cuMemGetAddressRange is not available");
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (reinterpret_cast<range_fn>(fn)(&base, &size, reinterpret_cast<CUdeviceptr>(device_ptr)) != CUDA_SUCCESS)
    return fail(ctx, SC_INVALID_ARG, "not a device allocation");
  cudaIpcMemHandle_t h;
  if ((s = check_cuda(ctx, cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)), "cudaIpcGetMemHandle")) != SC_OK)
    return s;
  std::memcpy(handle_out, &h, sizeof h);
  *offset_out = static_cast<size_t>(reinterpret_cast<CUdeviceptr>(device_ptr) - base);
  return SC_OK;
}

sc_status sc_ipc_open(sc_ctx* ctx, const void* handle, size_t offset, void** device_ptr_out) {
  if (ctx == nullptr) return SC_INVALID_ARG;
  if (handle == nullptr || device_ptr_out == nullptr) return fail(ctx, SC_INVALID_ARG, "null argument");
  sc_status s = enter(ctx);
  if (s != SC_OK) return s;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof h);
  void* base = nullptr;
  if ((s = check_cuda(ctx, cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle")) !=
      SC_OK)
    return s;
  *device_ptr_out = static_cast<uint8_t*>(base) + offset;
  return SC_OK;
}

sc_status sc_ipc_close(sc_ctx* ctx, void* device_ptr, size_t offset) {
  if (ctx == nullptr) return SC_INVALID_ARG;
  if (device_ptr == nullptr) return fail(ctx, SC_INVALID_ARG, "null argument");
  sc_status s = enter(ctx);
  if (s != SC_OK) return s;
  return check_cuda(ctx, cudaIpcCloseMemHandle(static_cast<uint8_t*>(device_ptr) - offset), "cudaIpcCloseMemHandle");
}

sc_status sc_sync(sc_ctx* ctx, void* stream) {
  if (ctx == nullptr) return SC_INVALID_ARG;
  sc_status s = enter(ctx);
  if (s != SC_OK) return s;
  return check_cuda(ctx, cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "cudaStreamSynchronize");
}

sc_status sc_poll_errors(sc_ctx* ctx, void* stream) {
  if (ctx == nullptr) return SC_INVALID_ARG;
  sc_status s = sc_sync(ctx, stream);
  if (s != SC_OK) return s;
  int h[kErrWords] = {0, 0, 0, 0};
  if ((s = check_cuda(ctx, cudaMemcpy(h, ctx->d_err, sizeof h, cudaMemcpyDeviceToHost), "error word")) != SC_OK) return s;
  if (h[0] == 0) return SC_OK;
  cudaMemset(ctx->d_err, 0, sizeof h);
  char msg[160];
  std::snprintf(msg, sizeof msg, "a bounded device-side wait gave up (site %d, block %d); the kernel returned early",
                h[1], h[2]);
  return fail(ctx, SC_TIMEOUT, msg);
}

}  // extern "C"
