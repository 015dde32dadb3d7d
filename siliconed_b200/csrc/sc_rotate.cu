// ComfyUI's convrot maps: an int8 weight published rotated, W = (q . s) . R along K, R block-diagonal
// with blocks H / sqrt(G) (H the regular Hadamard of size G, a power of 4 up to 256).  As in the
// reference (TensorGEMM.swift:53-54), the rotation moves to the activation: x . W = (x . R) . q . s,
// and the integers are never touched.
//
// rotate_groups_bf16: the activation's rotation before the product.  One warp per 256 values of a row
// (whole groups: G divides 256 and K); the warp's values sit in shared memory as fp32 and go through
// the radix-4 butterflies of rotate_groups (TensorGEMM.swift:183-201) stage by stage, spans 1, 4, 16, 64,
// each butterfly (a, b, c, d) <- (p + w, p - w, m + u, u - m) with p = a + b, m = a - b, u = c + d,
// w = c - d: the same operations on the same operands as the reference, so the same fp32 bits; then
// times 1/sqrt(G) (a power of two, exact) and rounded to bf16 nearest-even, the product's operand
// (the rounded route rotates, then rounds: TensorGEMMBF16.swift:204-231).  HBM-bound: 2 bytes read
// and 2 written per value.
//
// dequantize_rotated: Widen.dequantizeRotated (Widen.swift:374-428) for the export path: per group of
// G rows and column j, m = H . q in int32 (exact, |m| <= 32648), W = float(m) * (s[j] / sqrt(G)).
#include <cuda_bf16.h>

#include "sc_internal.h"

namespace sc {
namespace {

constexpr int kRotWarps = 8;

__device__ __forceinline__ int rotation_shift(int group) {  // group = 4^p: returns p
  return (31 - __clz(group)) >> 1;
}

__global__ void __launch_bounds__(kRotWarps * 32)
    rotate_groups_bf16(const uint16_t* __restrict__ x, int64_t m, int64_t k, int group, uint16_t* __restrict__ out) {
  __shared__ float v[kRotWarps][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t chunks_per_row = (k + 255) / 256;
  const int64_t chunk = static_cast<int64_t>(blockIdx.x) * kRotWarps + warp;
  if (chunk >= m * chunks_per_row) return;
  const int64_t row = chunk / chunks_per_row, c0 = (chunk % chunks_per_row) * 256;
  const int len = static_cast<int>(k - c0 < 256 ? k - c0 : 256);  // a multiple of the group (K % G == 0)
  const uint16_t* src = x + row * k + c0;
  float* sv = v[warp];
  if (lane * 8 < len) {
    const uint4 u = *reinterpret_cast<const uint4*>(src + lane * 8);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      sv[lane * 8 + 2 * i] = __uint_as_float(w[i] << 16);
      sv[lane * 8 + 2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
  }
  __syncwarp();
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
  if (lane * 8 < len) {
    const float norm = __int_as_float((127 - rotation_shift(group)) << 23);  // 2^-p = 1 / sqrt(G)
    uint32_t packed[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __nv_bfloat162 h =
          __floats2bfloat162_rn(__fmul_rn(sv[lane * 8 + 2 * i], norm), __fmul_rn(sv[lane * 8 + 2 * i + 1], norm));
      packed[i] = *reinterpret_cast<const uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(out + row * k + c0 + lane * 8) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
  }
}

// One block per (group of rows, 32 columns): the group's int8 codes of 32 columns in shared memory as
// int32, the butterflies of Widen.hadamard (exact in any order), then one multiply per value.  The
// arena stores [n_pad][k_pad] codes biased by 128.
__global__ void __launch_bounds__(256)
    dequantize_rotated(const uint8_t* __restrict__ values, const float* __restrict__ scales, int64_t k, int64_t n,
                       int64_t k_pad, int group, float* __restrict__ out) {
  __shared__ int32_t t[256][33];
  const int64_t g0 = static_cast<int64_t>(blockIdx.x) * group, j0 = static_cast<int64_t>(blockIdx.y) * 32;
  const int tid = threadIdx.x;
  for (int i = tid; i < group * 32; i += 256) {
    const int c = i / group, r = i % group;  // read along K (contiguous in the arena)
    const int64_t j = j0 + c;
    t[r][c] = j < n ? static_cast<int32_t>(values[j * k_pad + g0 + r]) - 128 : 0;
  }
  __syncthreads();
  for (int span = 1; span < group; span *= 4) {
    for (int i = tid; i < (group / 4) * 32; i += 256) {
      const int c = i % 32, b = i / 32;
      const int j = (b / span) * 4 * span + b % span;
      const int32_t a = t[j][c], bb = t[j + span][c], cc = t[j + 2 * span][c], d = t[j + 3 * span][c];
      const int32_t p = a + bb, mm = a - bb, u = cc + d, w = cc - d;
      t[j][c] = p + w;
      t[j + span][c] = p - w;
      t[j + 2 * span][c] = mm + u;
      t[j + 3 * span][c] = u - mm;
    }
    __syncthreads();
  }
  const float norm = __int_as_float((127 - rotation_shift(group)) << 23);
  for (int i = tid; i < group * 32; i += 256) {
    const int r = i / 32, c = i % 32;  // write along N (contiguous in the map layout)
    const int64_t j = j0 + c;
    if (j < n) out[(g0 + r) * n + j] = __fmul_rn(static_cast<float>(t[r][c]), __fmul_rn(scales[j], norm));
  }
}

}  // namespace

bool is_rotation_group(int64_t g) {
  int64_t p = 4;
  while (p < g) p *= 4;
  return p == g && g <= 256;
}

size_t rotated_x_bytes(int64_t m, int64_t k) {
  return static_cast<size_t>((m * k * 2 + 255) / 256 * 256);
}

cudaError_t launch_rotate(const uint16_t* x, int64_t m, int64_t k, int group, uint16_t* out, cudaStream_t stream) {
  const int64_t warps = m * ((k + 255) / 256);
  const int64_t blocks = (warps + kRotWarps - 1) / kRotWarps;
  if (blocks > 0x7FFFFFFF) return cudaErrorInvalidValue;
  rotate_groups_bf16<<<static_cast<unsigned>(blocks), kRotWarps * 32, 0, stream>>>(x, m, k, group, out);
  return cudaGetLastError();
}

cudaError_t launch_dequantize_rotated(const sc_weight* w, float* out, cudaStream_t stream) {
  const dim3 grid(static_cast<unsigned>(w->k / w->rotation), static_cast<unsigned>((w->n + 31) / 32));
  dequantize_rotated<<<grid, 256, 0, stream>>>(w->values, w->scales, w->k, w->n, w->k_pad, w->rotation, out);
  return cudaGetLastError();
}

}  // namespace sc
