// The elementwise stages of the DiT blocks (include/siliconed_dit.h), fused so that every activation
// crosses HBM once per stage.  All are memory-bound: row kernels keep their row in registers (one CTA
// of 256 threads per row, float4 per thread, d <= 8192), the others stream 16-byte vectors.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "siliconed_dit.h"

namespace {

constexpr int kRowThreads = 256;
constexpr int kMaxVec = 8;  // float4 per thread: d <= 8192

__device__ __forceinline__ uint16_t to_bf16(float f) {
  const __nv_bfloat16 h = __float2bfloat16_rn(f);
  return *reinterpret_cast<const uint16_t*>(&h);
}

__device__ __forceinline__ float from_bf16(uint16_t u) { return __uint_as_float(static_cast<uint32_t>(u) << 16); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  return static_cast<uint32_t>(to_bf16(lo)) | (static_cast<uint32_t>(to_bf16(hi)) << 16);
}

// Sum over the CTA (256 threads), the same value returned to every thread; `red` holds 8 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, off);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // red is free (an earlier call's readers are done)
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.0f;
#pragma unroll
  for (int w = 0; w < kRowThreads / 32; ++w) s += red[w];
  return s;
}

__device__ __forceinline__ void load_row(const float* row, int d4, float4 (&v)[kMaxVec]) {
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    const int i = threadIdx.x + j * kRowThreads;
    v[j] = i < d4 ? reinterpret_cast<const float4*>(row)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

__device__ __forceinline__ float4 vec_or(const float* p, int i, float dflt) {
  return p != nullptr ? reinterpret_cast<const float4*>(p)[i] : make_float4(dflt, dflt, dflt, dflt);
}

__device__ __forceinline__ void store_bf16x4(uint16_t* out, int i, float a, float b, float c, float d) {
  reinterpret_cast<uint2*>(out)[i] = make_uint2(pack_bf16x2(a, b), pack_bf16x2(c, d));
}

__global__ void __launch_bounds__(kRowThreads) rms_norm_modulate_k(const float* __restrict__ x, int d,
                                                                     const float* __restrict__ weight,
                                                                     const float* __restrict__ scale, float eps,
                                                                     uint16_t* __restrict__ out) {
  __shared__ float red[kRowThreads / 32];
  const int64_t r = blockIdx.x;
  const int d4 = d / 4;
  float4 v[kMaxVec];
  load_row(x + r * d, d4, v);
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
  const float inv = 1.0f / sqrtf(block_sum(ss, red) / static_cast<float>(d) + eps);
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    const int i = threadIdx.x + j * kRowThreads;
    if (i >= d4) break;
    const float4 w = vec_or(weight, i, 1.0f);
    const float4 s = vec_or(scale, i, 0.0f);
    store_bf16x4(out + r * d, i, v[j].x * inv * w.x * (1.0f + s.x), v[j].y * inv * w.y * (1.0f + s.y),
                 v[j].z * inv * w.z * (1.0f + s.z), v[j].w * inv * w.w * (1.0f + s.w));
  }
}

__global__ void __launch_bounds__(kRowThreads) layer_norm_modulate_k(const float* __restrict__ x, int d,
                                                                       const float* __restrict__ scale,
                                                                       const float* __restrict__ shift, float eps,
                                                                       uint16_t* __restrict__ out) {
  __shared__ float red[kRowThreads / 32];
  const int64_t r = blockIdx.x;
  const int d4 = d / 4;
  float4 v[kMaxVec];
  load_row(x + r * d, d4, v);
  float sum = 0.0f;
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) sum += (v[j].x + v[j].y) + (v[j].z + v[j].w);
  const float mean = block_sum(sum, red) / static_cast<float>(d);
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    if (threadIdx.x + j * kRowThreads >= d4) break;
    v[j].x -= mean;
    v[j].y -= mean;
    v[j].z -= mean;
    v[j].w -= mean;
    ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
  }
  const float inv = 1.0f / sqrtf(block_sum(ss, red) / static_cast<float>(d) + eps);
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    const int i = threadIdx.x + j * kRowThreads;
    if (i >= d4) break;
    const float4 s = vec_or(scale, i, 0.0f);
    const float4 b = vec_or(shift, i, 0.0f);
    store_bf16x4(out + r * d, i, v[j].x * inv * (1.0f + s.x) + b.x, v[j].y * inv * (1.0f + s.y) + b.y,
                 v[j].z * inv * (1.0f + s.z) + b.z, v[j].w * inv * (1.0f + s.w) + b.w);
  }
}

__global__ void __launch_bounds__(kRowThreads) gated_residual_k(float* __restrict__ x, const float* __restrict__ y,
                                                                  int d, const float* __restrict__ gate, int gate_tanh,
                                                                  const float* __restrict__ norm_weight, float eps) {
  __shared__ float red[kRowThreads / 32];
  const int64_t r = blockIdx.x;
  const int d4 = d / 4;
  float4 v[kMaxVec];
  load_row(y + r * d, d4, v);
  float inv = 1.0f;
  if (norm_weight != nullptr) {
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < kMaxVec; ++j) ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
    inv = 1.0f / sqrtf(block_sum(ss, red) / static_cast<float>(d) + eps);
  }
  float4* xr = reinterpret_cast<float4*>(x + r * d);
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    const int i = threadIdx.x + j * kRowThreads;
    if (i >= d4) break;
    float4 g = vec_or(gate, i, 1.0f);
    if (gate != nullptr && gate_tanh) g = make_float4(tanhf(g.x), tanhf(g.y), tanhf(g.z), tanhf(g.w));
    float4 o = v[j];
    if (norm_weight != nullptr) {
      const float4 w = reinterpret_cast<const float4*>(norm_weight)[i];
      o = make_float4(o.x * inv * w.x, o.y * inv * w.y, o.z * inv * w.z, o.w * inv * w.w);
    }
    float4 a = xr[i];
    a.x = __fadd_rn(a.x, __fmul_rn(g.x, o.x));  // two roundings, as torch's x + gate * y
    a.y = __fadd_rn(a.y, __fmul_rn(g.y, o.y));
    a.z = __fadd_rn(a.z, __fmul_rn(g.z, o.z));
    a.w = __fadd_rn(a.w, __fmul_rn(g.w, o.w));
    xr[i] = a;
  }
}

// gated_residual_k followed by rms_norm_modulate_k on the updated row, in one pass: the row of x is read
// once, updated, written, and normalised from the same registers (the same operations in the same order
// as the two kernels, so the same bits).
__global__ void __launch_bounds__(kRowThreads)
    gated_residual_rms_modulate_k(float* __restrict__ x, const float* __restrict__ y, int d,
                                  const float* __restrict__ gate, int gate_tanh,
                                  const float* __restrict__ norm_weight, float eps,
                                  const float* __restrict__ weight, const float* __restrict__ scale, float eps2,
                                  uint16_t* __restrict__ out) {
  __shared__ float red[kRowThreads / 32];
  const int64_t r = blockIdx.x;
  const int d4 = d / 4;
  float4 v[kMaxVec];
  load_row(y + r * d, d4, v);
  float inv = 1.0f;
  if (norm_weight != nullptr) {
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < kMaxVec; ++j) ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
    inv = 1.0f / sqrtf(block_sum(ss, red) / static_cast<float>(d) + eps);
  }
  float4* xr = reinterpret_cast<float4*>(x + r * d);
  float ss2 = 0.0f;
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    const int i = threadIdx.x + j * kRowThreads;
    if (i >= d4) {
      v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
      continue;
    }
    float4 g = vec_or(gate, i, 1.0f);
    if (gate != nullptr && gate_tanh) g = make_float4(tanhf(g.x), tanhf(g.y), tanhf(g.z), tanhf(g.w));
    float4 o = v[j];
    if (norm_weight != nullptr) {
      const float4 w = reinterpret_cast<const float4*>(norm_weight)[i];
      o = make_float4(o.x * inv * w.x, o.y * inv * w.y, o.z * inv * w.z, o.w * inv * w.w);
    }
    float4 a = xr[i];
    a.x = __fadd_rn(a.x, __fmul_rn(g.x, o.x));  // two roundings, as torch's x + gate * y
    a.y = __fadd_rn(a.y, __fmul_rn(g.y, o.y));
    a.z = __fadd_rn(a.z, __fmul_rn(g.z, o.z));
    a.w = __fadd_rn(a.w, __fmul_rn(g.w, o.w));
    xr[i] = a;
    v[j] = a;
  }
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) ss2 += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
  const float inv2 = 1.0f / sqrtf(block_sum(ss2, red) / static_cast<float>(d) + eps2);
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    const int i = threadIdx.x + j * kRowThreads;
    if (i >= d4) break;
    const float4 w = vec_or(weight, i, 1.0f);
    const float4 s = vec_or(scale, i, 0.0f);
    store_bf16x4(out + r * d, i, v[j].x * inv2 * w.x * (1.0f + s.x), v[j].y * inv2 * w.y * (1.0f + s.y),
                 v[j].z * inv2 * w.z * (1.0f + s.z), v[j].w * inv2 * w.w * (1.0f + s.w));
  }
}

// One warp per (token, head): lane l holds elements 4l .. 4l + 3 of q, k and v (head_dim 128).
__global__ void __launch_bounds__(256) qk_norm_rope_k(const uint16_t* __restrict__ qkv, int rows, int tokens, int heads,
                                                        const float* __restrict__ norm_q,
                                                        const float* __restrict__ norm_k,
                                                        const float* __restrict__ freqs, float eps,
                                                        uint16_t* __restrict__ q, uint16_t* __restrict__ k,
                                                        uint16_t* __restrict__ v, int joint_len, int token_offset) {
  constexpr int D = 128;
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (gw >= static_cast<int64_t>(rows) * heads) return;
  const int row = static_cast<int>(gw / heads), h = static_cast<int>(gw % heads);
  const int b = row / tokens, t = row % tokens;
  const int pos = token_offset + t;
  const int64_t hd = static_cast<int64_t>(heads) * D;
  const uint16_t* src = qkv + static_cast<int64_t>(row) * 3 * hd + static_cast<int64_t>(h) * D + 4 * lane;
  const int64_t dst = ((static_cast<int64_t>(b) * heads + h) * joint_len + pos) * D + 4 * lane;
  const float4 f = reinterpret_cast<const float4*>(freqs + static_cast<int64_t>(pos) * D)[lane];  // pairs 2l, 2l+1
#pragma unroll
  for (int which = 0; which < 2; ++which) {
    const uint2 raw = *reinterpret_cast<const uint2*>(src + which * hd);
    float e0 = from_bf16(static_cast<uint16_t>(raw.x)), e1 = from_bf16(static_cast<uint16_t>(raw.x >> 16));
    float e2 = from_bf16(static_cast<uint16_t>(raw.y)), e3 = from_bf16(static_cast<uint16_t>(raw.y >> 16));
    float ss = e0 * e0 + e1 * e1 + e2 * e2 + e3 * e3;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, off);
    const float inv = 1.0f / sqrtf(ss / static_cast<float>(D) + eps);
    const float4 w = reinterpret_cast<const float4*>(which == 0 ? norm_q : norm_k)[lane];
    e0 = e0 * inv * w.x;
    e1 = e1 * inv * w.y;
    e2 = e2 * inv * w.z;
    e3 = e3 * inv * w.w;
    const float r0 = e0 * f.x - e1 * f.y, r1 = e0 * f.y + e1 * f.x;
    const float r2 = e2 * f.z - e3 * f.w, r3 = e2 * f.w + e3 * f.z;
    *reinterpret_cast<uint2*>((which == 0 ? q : k) + dst) = make_uint2(pack_bf16x2(r0, r1), pack_bf16x2(r2, r3));
  }
  *reinterpret_cast<uint2*>(v + dst) = *reinterpret_cast<const uint2*>(src + 2 * hd);
}

// One warp per (batch row, head): 256 contiguous bytes in, 256 out.
__global__ void __launch_bounds__(256) attention_merge_k(const uint16_t* __restrict__ o, int batch, int heads,
                                                           int joint_len, int token_offset, int tokens,
                                                           uint16_t* __restrict__ out) {
  constexpr int D = 128;
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (gw >= static_cast<int64_t>(batch) * tokens * heads) return;
  const int64_t row = gw / heads;
  const int h = static_cast<int>(gw % heads);
  const int b = static_cast<int>(row / tokens), t = static_cast<int>(row % tokens);
  const uint2 val =
      reinterpret_cast<const uint2*>(o + ((static_cast<int64_t>(b) * heads + h) * joint_len + token_offset + t) * D)[lane];
  reinterpret_cast<uint2*>(out + row * heads * D + static_cast<int64_t>(h) * D)[lane] = val;
}

__global__ void swiglu_k(const uint16_t* __restrict__ hbuf, int64_t rows, int hidden, uint16_t* __restrict__ out) {
  const int64_t per_row = hidden / 8;
  const int64_t total = rows * per_row;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / per_row, c = (i % per_row) * 8;
    const uint4 a = *reinterpret_cast<const uint4*>(hbuf + r * 2 * hidden + c);
    const uint4 b = *reinterpret_cast<const uint4*>(hbuf + r * 2 * hidden + hidden + c);
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
    uint32_t ow[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float a0 = from_bf16(static_cast<uint16_t>(aw[j])), a1 = from_bf16(static_cast<uint16_t>(aw[j] >> 16));
      const float b0 = from_bf16(static_cast<uint16_t>(bw[j])), b1 = from_bf16(static_cast<uint16_t>(bw[j] >> 16));
      const float s0 = a0 / (1.0f + expf(-a0)), s1 = a1 / (1.0f + expf(-a1));
      ow[j] = pack_bf16x2(s0 * b0, s1 * b1);
    }
    *reinterpret_cast<uint4*>(out + r * hidden + c) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
  }
}

__global__ void gelu_tanh_k(uint16_t* __restrict__ h, int64_t count) {
  const float c = 0.7978845608028654f;  // sqrt(2 / pi)
  const int64_t vecs = count / 8;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < vecs;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    uint4 v = reinterpret_cast<uint4*>(h)[i];
    uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float a = from_bf16(static_cast<uint16_t>(w[j])), b = from_bf16(static_cast<uint16_t>(w[j] >> 16));
      const float ga = 0.5f * a * (1.0f + tanhf(c * (a + 0.044715f * a * a * a)));
      const float gb = 0.5f * b * (1.0f + tanhf(c * (b + 0.044715f * b * b * b)));
      w[j] = pack_bf16x2(ga, gb);
    }
    reinterpret_cast<uint4*>(h)[i] = make_uint4(w[0], w[1], w[2], w[3]);
  }
  // The tail past the last 8-element vector.
  const int64_t first = vecs * 8;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t < count - first) {
    const float a = from_bf16(h[first + t]);
    h[first + t] = to_bf16(0.5f * a * (1.0f + tanhf(c * (a + 0.044715f * a * a * a))));
  }
}

int status_of(cudaError_t e) {
  if (e == cudaSuccess) return SD_OK;
  cudaGetLastError();
  return SD_CUDA_ERROR;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

int grid_for(int64_t work, int per_block) {
  const int64_t g = (work + per_block - 1) / per_block;
  return static_cast<int>(g < 148LL * 64 ? (g > 0 ? g : 1) : 148LL * 64);
}

bool row_args_ok(const void* x, int64_t rows, int d) {
  return x != nullptr && rows >= 0 && d > 0 && d % 4 == 0 && d <= 4 * kMaxVec * kRowThreads && aligned(x, 16);
}

}  // namespace

extern "C" {

int sd_rms_norm_modulate(const float* x, int64_t rows, int d, const float* weight, const float* scale, float eps,
                         uint16_t* out, void* stream) {
  if (!row_args_ok(x, rows, d) || out == nullptr || !aligned(out, 8) || (weight && !aligned(weight, 16)) ||
      (scale && !aligned(scale, 16)) || rows > 0x7FFFFFFF)
    return SD_INVALID_ARG;
  if (rows == 0) return SD_OK;
  rms_norm_modulate_k<<<static_cast<unsigned>(rows), kRowThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      x, d, weight, scale, eps, out);
  return status_of(cudaGetLastError());
}

int sd_layer_norm_modulate(const float* x, int64_t rows, int d, const float* scale, const float* shift, float eps,
                           uint16_t* out, void* stream) {
  if (!row_args_ok(x, rows, d) || out == nullptr || !aligned(out, 8) || (scale && !aligned(scale, 16)) ||
      (shift && !aligned(shift, 16)) || rows > 0x7FFFFFFF)
    return SD_INVALID_ARG;
  if (rows == 0) return SD_OK;
  layer_norm_modulate_k<<<static_cast<unsigned>(rows), kRowThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      x, d, scale, shift, eps, out);
  return status_of(cudaGetLastError());
}

int sd_gated_residual_rms_modulate(float* x, const float* y, int64_t rows, int d, const float* gate, int gate_tanh,
                                   const float* norm_weight, float eps, const float* weight, const float* scale,
                                   float eps2, uint16_t* out, void* stream) {
  if (!row_args_ok(x, rows, d) || y == nullptr || !aligned(y, 16) || (gate && !aligned(gate, 16)) ||
      (norm_weight && !aligned(norm_weight, 16)) || (weight && !aligned(weight, 16)) || (scale && !aligned(scale, 16)) ||
      out == nullptr || !aligned(out, 16) || rows > 0x7FFFFFFF)
    return SD_INVALID_ARG;
  if (rows == 0) return SD_OK;
  gated_residual_rms_modulate_k<<<static_cast<unsigned>(rows), kRowThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      x, y, d, gate, gate_tanh, norm_weight, eps, weight, scale, eps2, out);
  return status_of(cudaGetLastError());
}

int sd_gated_residual(float* x, const float* y, int64_t rows, int d, const float* gate, int gate_tanh,
                      const float* norm_weight, float eps, void* stream) {
  if (!row_args_ok(x, rows, d) || y == nullptr || !aligned(y, 16) || (gate && !aligned(gate, 16)) ||
      (norm_weight && !aligned(norm_weight, 16)) || rows > 0x7FFFFFFF)
    return SD_INVALID_ARG;
  if (rows == 0) return SD_OK;
  gated_residual_k<<<static_cast<unsigned>(rows), kRowThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      x, y, d, gate, gate_tanh, norm_weight, eps);
  return status_of(cudaGetLastError());
}

int sd_qk_norm_rope(const uint16_t* qkv, int batch, int tokens, int heads, int head_dim, const float* norm_q,
                    const float* norm_k, const float* freqs, float eps, uint16_t* q, uint16_t* k, uint16_t* v,
                    int joint_len, int token_offset, void* stream) {
  if (qkv == nullptr || norm_q == nullptr || norm_k == nullptr || freqs == nullptr || q == nullptr || k == nullptr ||
      v == nullptr || head_dim != 128 || batch < 0 || tokens < 0 || heads <= 0 || token_offset < 0 ||
      token_offset + tokens > joint_len || !aligned(qkv, 8) || !aligned(q, 8) || !aligned(k, 8) || !aligned(v, 8) ||
      !aligned(norm_q, 16) || !aligned(norm_k, 16) || !aligned(freqs, 16))
    return SD_INVALID_ARG;
  const int64_t rows = static_cast<int64_t>(batch) * tokens;
  if (rows == 0) return SD_OK;
  if (rows > 0x7FFFFFFF) return SD_INVALID_ARG;
  const int64_t warps = rows * heads;
  qk_norm_rope_k<<<static_cast<unsigned>((warps + 7) / 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      qkv, static_cast<int>(rows), tokens, heads, norm_q, norm_k, freqs, eps, q, k, v, joint_len, token_offset);
  return status_of(cudaGetLastError());
}

int sd_attention_merge(const uint16_t* o, int batch, int heads, int head_dim, int joint_len, int token_offset,
                       int tokens, uint16_t* out, void* stream) {
  if (o == nullptr || out == nullptr || head_dim != 128 || batch < 0 || heads <= 0 || tokens < 0 || token_offset < 0 ||
      token_offset + tokens > joint_len || !aligned(o, 8) || !aligned(out, 8))
    return SD_INVALID_ARG;
  const int64_t warps = static_cast<int64_t>(batch) * tokens * heads;
  if (warps == 0) return SD_OK;
  attention_merge_k<<<static_cast<unsigned>((warps + 7) / 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      o, batch, heads, joint_len, token_offset, tokens, out);
  return status_of(cudaGetLastError());
}

int sd_swiglu(const uint16_t* h, int64_t rows, int hidden, uint16_t* out, void* stream) {
  if (h == nullptr || out == nullptr || rows < 0 || hidden <= 0 || hidden % 8 != 0 || !aligned(h, 16) ||
      !aligned(out, 16))
    return SD_INVALID_ARG;
  if (rows == 0) return SD_OK;
  swiglu_k<<<grid_for(rows * (hidden / 8), 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(h, rows, hidden, out);
  return status_of(cudaGetLastError());
}

// The same with gate and up interleaved in blocks of `block` columns (gate block j, then up block j).
__global__ void swiglu_blocks_k(const uint16_t* __restrict__ hbuf, int64_t rows, int hidden, int block,
                                uint16_t* __restrict__ out) {
  const int64_t per_row = hidden / 8;
  const int64_t total = rows * per_row;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / per_row, c = (i % per_row) * 8;
    const int64_t src = r * 2 * hidden + (c / block) * 2 * block + c % block;
    const uint4 a = *reinterpret_cast<const uint4*>(hbuf + src);
    const uint4 b = *reinterpret_cast<const uint4*>(hbuf + src + block);
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
    uint32_t ow[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float a0 = from_bf16(static_cast<uint16_t>(aw[j])), a1 = from_bf16(static_cast<uint16_t>(aw[j] >> 16));
      const float b0 = from_bf16(static_cast<uint16_t>(bw[j])), b1 = from_bf16(static_cast<uint16_t>(bw[j] >> 16));
      const float s0 = a0 / (1.0f + expf(-a0)), s1 = a1 / (1.0f + expf(-a1));
      ow[j] = pack_bf16x2(s0 * b0, s1 * b1);
    }
    *reinterpret_cast<uint4*>(out + r * hidden + c) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
  }
}

int sd_swiglu_blocks(const uint16_t* h, int64_t rows, int hidden, int block, uint16_t* out, void* stream) {
  if (h == nullptr || out == nullptr || rows < 0 || hidden <= 0 || block <= 0 || block % 8 != 0 ||
      hidden % block != 0 || !aligned(h, 16) || !aligned(out, 16))
    return SD_INVALID_ARG;
  if (rows == 0) return SD_OK;
  swiglu_blocks_k<<<grid_for(rows * (hidden / 8), 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(h, rows, hidden,
                                                                                                   block, out);
  return status_of(cudaGetLastError());
}

int sd_gelu_tanh(uint16_t* h, int64_t count, void* stream) {
  if (h == nullptr || count < 0 || !aligned(h, 16)) return SD_INVALID_ARG;
  if (count == 0) return SD_OK;
  gelu_tanh_k<<<grid_for(count / 8 + 8, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(h, count);
  return status_of(cudaGetLastError());
}

}  // extern "C"
