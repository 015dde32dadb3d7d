// W8A8: the activation quantized to int8 per row, beside a published int8 weight (TensorGEMMInt8.swift,
// ComfyUI's int8_linear).  quantize_rows is the recipe of W8A8.quantize (TensorGEMMInt8.swift:198-221)
// and quantize_held (:96-126):
//   y   = x rotated by groups of G (convrot on the activation: rotate_groups' butterflies, spans 1, 4,
//         16, 64, then times 1/sqrt(G)), or x itself;
//   s_x = max(max|y| / 127, 1e-30), a correctly rounded division;
//   q_x = clamp(rint(y / s_x), -128, 127), a correctly rounded division, rint half to even.
// One CTA of 256 threads per row holds the row whole in shared memory as fp32 (the scale needs the
// whole row's maximum before any code is written): one read of the row, one write of its codes.  The
// maximum is exact in any order, and every other step is one IEEE operation on the same operands as
// the recipe, so the codes and the scale are the recipe's bits.
#include <cuda_bf16.h>

#include "sc_internal.h"
#include "sc_ptx.cuh"

namespace sc {
namespace {

constexpr int kQThreads = 256;

template <bool kF32In>
__global__ void __launch_bounds__(kQThreads)
    quantize_rows(const void* __restrict__ x, int64_t k, int group, int8_t* __restrict__ codes, int64_t ld,
                  float* __restrict__ scales) {
  extern __shared__ float y[];  // [k rounded up to 256]
  __shared__ float part[kQThreads / 32];
  pdl_launch_dependents();  // the int8 GEMM after it may set up meanwhile
  const int64_t row = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (kF32In) {
    const float* xr = static_cast<const float*>(x) + row * k;
    for (int64_t i = tid * 4; i < k; i += kQThreads * 4) {
      const float4 v = *reinterpret_cast<const float4*>(xr + i);
      y[i] = v.x;
      y[i + 1] = v.y;
      y[i + 2] = v.z;
      y[i + 3] = v.w;
    }
  } else {
    const uint16_t* xr = static_cast<const uint16_t*>(x) + row * k;
    for (int64_t i = tid * 8; i < k; i += kQThreads * 8) {
      const uint4 u = *reinterpret_cast<const uint4*>(xr + i);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        y[i + 2 * e] = __uint_as_float(w[e] << 16);
        y[i + 2 * e + 1] = __uint_as_float(w[e] & 0xFFFF0000u);
      }
    }
  }
  __syncthreads();
  float top = 0.0f;
  if (group > 0) {
    const float norm = __int_as_float((127 - ((31 - __clz(group)) >> 1)) << 23);  // 1 / sqrt(G), a power of two
    for (int64_t c0 = static_cast<int64_t>(warp) * 256; c0 < k; c0 += (kQThreads / 32) * 256) {
      const int len = static_cast<int>(k - c0 < 256 ? k - c0 : 256);  // whole groups (G divides 256 and K)
      float* sv = y + c0;
      for (int span = 1; span < group; span *= 4) {
        for (int t = lane; t < len / 4; t += 32) {
          const int j = (t / span) * 4 * span + t % span;
          const float a = sv[j], b = sv[j + span], c = sv[j + 2 * span], d = sv[j + 3 * span];
          const float p = __fadd_rn(a, b), mm = __fsub_rn(a, b), u = __fadd_rn(c, d), w = __fsub_rn(c, d);
          sv[j] = __fadd_rn(p, w);
          sv[j + span] = __fsub_rn(p, w);
          sv[j + 2 * span] = __fadd_rn(mm, u);
          sv[j + 3 * span] = __fsub_rn(u, mm);
        }
        __syncwarp();
      }
      for (int i = lane; i < len; i += 32) {
        const float v = __fmul_rn(sv[i], norm);
        sv[i] = v;
        top = fmaxf(top, fabsf(v));
      }
      __syncwarp();
    }
  } else {
    for (int64_t i = tid; i < k; i += kQThreads) top = fmaxf(top, fabsf(y[i]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) top = fmaxf(top, __shfl_xor_sync(0xFFFFFFFFu, top, o));
  if (lane == 0) part[warp] = top;
  __syncthreads();  // also orders every warp's rotated values before the codes pass reads them
  top = part[0];
#pragma unroll
  for (int i = 1; i < kQThreads / 32; ++i) top = fmaxf(top, part[i]);
  const float scale = fmaxf(__fdiv_rn(top, 127.0f), 1e-30f);
  int8_t* cr = codes + row * ld;
  for (int64_t i = tid * 4; i < k; i += kQThreads * 4) {
    uint32_t packed = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float q = fminf(fmaxf(rintf(__fdiv_rn(y[i + e], scale)), -128.0f), 127.0f);
      packed |= (static_cast<uint32_t>(static_cast<int>(q)) & 0xFFu) << (8 * e);
    }
    *reinterpret_cast<uint32_t*>(cr + i) = packed;
  }
  if (tid == 0) scales[row] = scale;
}

}  // namespace

cudaError_t launch_quantize_rows(const void* x, bool x_f32, int64_t m, int64_t k, int group, int8_t* codes, int64_t ld,
                                 float* scales, cudaStream_t stream) {
  if (m > 0x7FFFFFFF || k > kW8A8MaxK) return cudaErrorInvalidValue;
  const int smem = static_cast<int>((k + 255) / 256 * 256 * 4);
  static unsigned long long configured[2] = {0, 0};  // per input type and device
  if (cudaError_t e = set_smem_once(x_f32 ? quantize_rows<true> : quantize_rows<false>, static_cast<int>(kW8A8MaxK * 4),
                                    configured[x_f32]);
      e != cudaSuccess)
    return e;
  if (x_f32)
    quantize_rows<true><<<static_cast<unsigned>(m), kQThreads, smem, stream>>>(x, k, group, codes, ld, scales);
  else
    quantize_rows<false><<<static_cast<unsigned>(m), kQThreads, smem, stream>>>(x, k, group, codes, ld, scales);
  return cudaGetLastError();
}

}  // namespace sc
