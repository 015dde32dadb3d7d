// sc_linear_ex_noalloc: sc_linear_ex whose scratch (the widened bf16 copy of the weight) lives in a
// file-scope device array of this library instead of a caller's workspace, for callers that have
// no workspace to pass and may not allocate per call.  It allocates nothing: no cudaMalloc, no
// cudaFree, no allocating library routine.
//
// The array holds kStaticScratchBytes (32 MiB).  A product whose scratch (sc_workspace_size: from
// 1536 rows the widened weight, n_pad * k_pad * 2 bytes with N rounded up to 256 and K to 64) is
// larger is rejected with SC_UNSUPPORTED_SHAPE before anything runs.  Set-up runs
// once per device, on that device's first call: cudaGetSymbolAddress of the array with the device
// current; that first call should come before any stream capture.  Every call on a device shares
// the one array and leaves the last call's contents in it.  Nothing in it needs to start at zero:
// the widening writes every byte the GEMM then reads.  Calls that overlap on the GPU (on different
// streams, or from several threads) race on the array.
#include <mutex>

#include "sc_internal.h"

namespace {

constexpr size_t kStaticScratchBytes = static_cast<size_t>(32) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint8_t g_static_scratch[kStaticScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// The array's device address on ctx's device (set-up on first use, with that device current).
sc_status static_scratch(sc_ctx* ctx, void** out) {
  if (ctx->device < 0 || ctx->device >= kMaxDevices) return sc::fail(ctx, SC_INVALID_ARG, "device index out of range");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[ctx->device] == nullptr) {
    int cur = -1;
    cudaError_t e = cudaGetDevice(&cur);
    if (e == cudaSuccess && cur != ctx->device) e = cudaSetDevice(ctx->device);
    if (e != cudaSuccess) return sc::check_cuda(ctx, e, "selecting the context's device");
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return sc::check_cuda(ctx, e, "cudaGetSymbolAddress (static scratch)");
    if (p == nullptr) return sc::fail(ctx, SC_CUDA_ERROR, "cudaGetSymbolAddress returned no address");
    g_scratch_ptr[ctx->device] = p;
  }
  *out = g_scratch_ptr[ctx->device];
  return SC_OK;
}

}  // namespace

extern "C" {

sc_status sc_linear_ex_noalloc(sc_ctx* ctx, const sc_weight* w, const sc_bf16* x, int64_t m, const sc_bf16* bias,
                               void* y, sc_out_type y_type, void* stream) {
  if (ctx == nullptr) return SC_INVALID_ARG;
  size_t need = 0;
  sc_status s = sc_workspace_size(ctx, w, m, &need);
  if (s != SC_OK) return s;
  if (need > kStaticScratchBytes)
    return sc::fail(ctx, SC_UNSUPPORTED_SHAPE,
                    "sc_linear_ex_noalloc: this product needs " + std::to_string(need) +
                        " bytes of scratch (the widened weight); the static scratch holds " +
                        std::to_string(kStaticScratchBytes) + " (use sc_linear_ex with a workspace)");
  void* scratch = nullptr;
  s = static_scratch(ctx, &scratch);
  if (s != SC_OK) return s;
  return sc_linear_ex(ctx, w, x, m, bias, y, y_type, scratch, kStaticScratchBytes, stream);
}

}  // extern "C"
