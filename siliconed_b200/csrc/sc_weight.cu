// The weight arena: re-tiling at registration and the bit-exact dequantization export.
//
// Arena layout of one weight (one cudaMalloc):
//   values  [n_pad][k_pad] bytes   the codes transposed to [N, K] (K contiguous per output), int8
//                                  biased to unsigned (u = q + 128), e4m3 as published; padding
//                                  holds the code of 0.  k_pad = K rounded up to 64, n_pad = N
//                                  rounded up to 256, so every TMA box of the GEMM and every
//                                  128-bit load of the GEMV stays inside the arena.
//   scales  [n_pad] fp32           at the next 256-byte boundary after the values (the map's own
//                                  rule: values, then scales at an aligned offset in one region,
//                                  Sources/Siliconed/Artifact.swift:31-57), widened exactly from
//                                  the published fp32 / bf16 / fp16, 0 in the padding.
#include "sc_codes.cuh"
#include "sc_internal.h"

namespace sc {
namespace {

// Map layout [K, N] (row stride n_total) -> arena [n_pad][k_pad], 32 x 32 tiles through shared memory.
__global__ void retile_kn(const uint8_t* __restrict__ src, int64_t k, int64_t n_total, int64_t n_begin,
                          int64_t n_cols, uint8_t bias_xor, uint8_t pad, bool e4m3, uint8_t* __restrict__ dst,
                          int64_t k_pad, int* nan_flag) {
  __shared__ uint8_t tile[32][33];
  const int64_t k0 = static_cast<int64_t>(blockIdx.y) * 32, j0 = static_cast<int64_t>(blockIdx.x) * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;
  bool nan = false;
  for (int r = ty; r < 32; r += 8) {
    const int64_t kk = k0 + r, j = j0 + tx;
    uint8_t v = pad;
    if (kk < k && j < n_cols) {
      const uint8_t c = src[kk * n_total + n_begin + j];
      nan |= e4m3 && (c & 0x7F) == 0x7F;
      v = c ^ bias_xor;
    }
    tile[r][tx] = v;
  }
  __syncthreads();
  for (int r = ty; r < 32; r += 8) dst[(j0 + r) * k_pad + k0 + tx] = tile[tx][r];
  if (nan) atomicOr(nan_flag, 1);
}

// Published layout [N, K] -> arena rows: a copy with the bias, padded.
__global__ void retile_nk(const uint8_t* __restrict__ src, int64_t k, int64_t n_begin, int64_t n_cols, uint8_t bias_xor,
                          uint8_t pad, bool e4m3, uint8_t* __restrict__ dst, int64_t k_pad, int* nan_flag) {
  const int64_t j = blockIdx.x;  // one arena row per block
  bool nan = false;
  for (int64_t kk = threadIdx.x; kk < k_pad; kk += blockDim.x) {
    uint8_t v = pad;
    if (kk < k && j < n_cols) {
      const uint8_t c = src[(n_begin + j) * k + kk];
      nan |= e4m3 && (c & 0x7F) == 0x7F;
      v = c ^ bias_xor;
    }
    dst[j * k_pad + kk] = v;
  }
  if (nan) atomicOr(nan_flag, 1);
}

// out[kk, j] = float(q[kk, j]) * s[j], one rounded multiply, back in the map's [K, N] layout.
template <int kKind>
__global__ void dequantize_kn(const uint8_t* __restrict__ values, const float* __restrict__ scales, int64_t k,
                              int64_t n, int64_t k_pad, float* __restrict__ out) {
  __shared__ float tile[32][33];
  const int64_t k0 = static_cast<int64_t>(blockIdx.x) * 32, j0 = static_cast<int64_t>(blockIdx.y) * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;
  for (int r = ty; r < 32; r += 8) {
    const int64_t j = j0 + r, kk = k0 + tx;  // read along K (contiguous in the arena)
    tile[r][tx] = __fmul_rn(code_to_f32<kKind>(values[j * k_pad + kk]), scales[j]);
  }
  __syncthreads();
  for (int r = ty; r < 32; r += 8) {
    const int64_t kk = k0 + r, j = j0 + tx;  // write along N (contiguous in the map layout)
    if (kk < k && j < n) out[kk * n + j] = tile[tx][r];
  }
}

}  // namespace

cudaError_t launch_retile(const uint8_t* src, bool published_nk, int kind, int64_t k, int64_t n_total, int64_t n_begin,
                          int64_t n_cols, uint8_t* dst, int64_t k_pad, int64_t n_pad, int* nan_flag,
                          cudaStream_t stream) {
  const bool e4m3 = kind == SC_WEIGHT_E4M3;
  const uint8_t bias_xor = e4m3 ? 0x00 : 0x80;
  const uint8_t pad = e4m3 ? kPadE4M3 : kPadInt8;
  if (!published_nk) {
    const dim3 grid(static_cast<unsigned>(n_pad / 32), static_cast<unsigned>(k_pad / 32));
    retile_kn<<<grid, dim3(32, 8), 0, stream>>>(src, k, n_total, n_begin, n_cols, bias_xor, pad, e4m3, dst, k_pad,
                                                nan_flag);
  } else {
    retile_nk<<<static_cast<unsigned>(n_pad), 256, 0, stream>>>(src, k, n_begin, n_cols, bias_xor, pad, e4m3, dst,
                                                                k_pad, nan_flag);
  }
  return cudaGetLastError();
}

cudaError_t launch_dequantize(const sc_weight* w, float* out, cudaStream_t stream) {
  const dim3 grid(static_cast<unsigned>(w->k_pad / 32), static_cast<unsigned>(w->n_pad / 32));
  if (w->kind == SC_WEIGHT_INT8)
    dequantize_kn<1><<<grid, dim3(32, 8), 0, stream>>>(w->values, w->scales, w->k, w->n, w->k_pad, out);
  else
    dequantize_kn<2><<<grid, dim3(32, 8), 0, stream>>>(w->values, w->scales, w->k, w->n, w->k_pad, out);
  return cudaGetLastError();
}

}  // namespace sc
