// The skinny product (1 <= m <= 32): y[m, n] = bf16((sum_k x[m, k] * float(q[k, n])) * s[n] + bias[n]).
//
// Memory-bound: every weight byte is read once per pass.  The arena's transposed layout gives each
// output n a contiguous K row.  A CTA of 8 warps owns a block of rows, split as row groups x K
// slices, and streams it with 128-bit non-allocating loads (32 lanes x 16 bytes = 512 consecutive K
// values per step), all loads of a batch issued before any arithmetic.  Codes are decoded exactly (int8: byte under the
// fp32 pattern 2^23, minus 2^23 + 128; e4m3: magnitude placed and scaled by 2^120) and multiplied
// with Blackwell's packed fp32x2 FMA (each lane rounded as a scalar fma).  The K slices meet in
// shared memory and are added in slice order, so every run gives the same bits; nothing is kept
// outside the CTA (no global scratch, no cross-CTA synchronisation), which is what the reference's
// split GEMV achieves with its fixed-order sum of partials (Sources/Siliconed/DecodeKernels.swift:20-23,
// :67-109).  Launched with programmatic dependent launch: a CTA starts its weight bytes (an L2 prefetch of
// its rows and its first batch of loads) before it waits for the kernel ahead of it, whose output is x in a
// decode step, so consecutive products' weight reads overlap.
#include <cuda_bf16.h>

#include "sc_codes.cuh"
#include "sc_internal.h"
#include "sc_ptx.cuh"

namespace sc {
namespace gemv {


__device__ __forceinline__ unsigned long long pack2(float lo, float hi) {
  return (static_cast<unsigned long long>(__float_as_uint(hi)) << 32) | __float_as_uint(lo);
}

// acc = a * b + acc, lane by lane (two independent fp32 fused multiply-adds).
__device__ __forceinline__ unsigned long long ffma2(unsigned long long a, unsigned long long b, unsigned long long c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

__device__ __forceinline__ unsigned long long fsub2(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

__device__ __forceinline__ unsigned long long fmul2(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// Codes j and j + 1 of `word` (j = 0 or 2) as an fp32 pair, exactly.
template <int kKind, bool kNaN>
__device__ __forceinline__ unsigned long long codes2(uint32_t word, int j) {
  if (kKind == 1) {
    const uint32_t lo = __byte_perm(word, 0x4B000000u, 0x7440u | static_cast<uint32_t>(j));
    const uint32_t hi = __byte_perm(word, 0x4B000000u, 0x7440u | static_cast<uint32_t>(j + 1));
    return fsub2((static_cast<unsigned long long>(hi) << 32) | lo, pack2(kInt8Magic, kInt8Magic));
  } else {
    const uint32_t lo = e4m3_code_scaled_bits(word, j), hi = e4m3_code_scaled_bits(word, j + 1);
    const float two120 = __uint_as_float(kTwoPow120Bits);
    unsigned long long v = fmul2((static_cast<unsigned long long>(hi) << 32) | lo, pack2(two120, two120));
    if (kNaN) {
      const uint32_t m0 = (word >> (8 * j)) & 0x7Fu, m1 = (word >> (8 * (j + 1))) & 0x7Fu;
      if (m0 == 0x7Fu) v = (v & 0xFFFFFFFF00000000ull) | 0x7FC00000u;
      if (m1 == 0x7Fu) v = (v & 0x00000000FFFFFFFFull) | (0x7FC00000ull << 32);
    }
    return v;
  }
}

// One 16-code chunk as 8 exact fp32 pairs.
template <int kKind, bool kNaN>
__device__ __forceinline__ void decode_chunk(const uint4 w, unsigned long long (&q)[8]) {
  const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    q[2 * i] = codes2<kKind, kNaN>(words[i], 0);
    q[2 * i + 1] = codes2<kKind, kNaN>(words[i], 2);
  }
}

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int RW = 2;          // rows per warp
constexpr int kBatch = 4;      // 512-byte steps whose loads are issued together

__device__ __forceinline__ uint4 ld_stream(const uint8_t* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// A CTA owns RB = RG * RW rows; its 8 warps are RG row groups x KS K slices.  Each lane issues all
// the 128-bit loads of a batch (kBatch steps x RW rows) before any arithmetic; per step it decodes
// 16 codes of each row and multiplies them with the 16 activations of each token.  The K slices
// meet in shared memory and are added in slice order.
template <int kKind, bool kNaN, int MT, int KS, bool kF32Out>
__global__ void __launch_bounds__(kThreads) gemv_w8(const uint8_t* __restrict__ values, int k_pad,
                                                     const float* __restrict__ scales, const uint16_t* __restrict__ x,
                                                     int M, int K, const uint16_t* __restrict__ bias,
                                                     void* __restrict__ y, int N, int m0) {
  constexpr int RG = kWarps / KS;
  constexpr int RB = RG * RW;
  __shared__ float part[KS][RB][MT];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rg = warp % RG, ks = warp / RG;
  const int units = k_pad / 16;
  const int kbeg = (ks * units / KS) * 16, kend = ((ks + 1) * units / KS) * 16;
  const int row0 = blockIdx.x * RB + rg * RW;
  const uint8_t* wrow = values + static_cast<int64_t>(row0) * k_pad;

  // In a decode step the products run back to back and x is the previous product's output, while the
  // weight bytes depend on nothing: the next kernel of the stream may launch now, this CTA's rows (RB
  // contiguous rows of the arena) start toward the L2, and its first batch of loads is issued before the
  // wait for the previous kernel (for config 4's shapes the first batch is a warp's whole share).
  pdl_launch_dependents();
  if (threadIdx.x == 0) prefetch_l2_bulk(values + static_cast<int64_t>(blockIdx.x) * RB * k_pad, RB * k_pad);
  bool waited = false;
  unsigned long long acc[RW][MT];
#pragma unroll
  for (int r = 0; r < RW; ++r)
#pragma unroll
    for (int t = 0; t < MT; ++t) acc[r][t] = 0ull;

  for (int base = kbeg + lane * 16; base < kend; base += 512 * kBatch) {
    uint4 wv[kBatch][RW];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int kb = base + u * 512;
#pragma unroll
      for (int r = 0; r < RW; ++r)
        wv[u][r] = kb < kend ? ld_stream(wrow + static_cast<int64_t>(r) * k_pad + kb) : make_uint4(0, 0, 0, 0);
    }
    if (!waited) {  // the first batch of weight bytes is in flight before the wait for the previous kernel
      pdl_wait();
      waited = true;
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int kb = base + u * 512;
      if (kb >= kend) break;
      unsigned long long q[RW][8];
#pragma unroll
      for (int r = 0; r < RW; ++r) decode_chunk<kKind, kNaN>(wv[u][r], q[r]);
      // Each token's 16 activations as 8 fp32 pairs (zero past K; the arena's padding codes are 0).
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        unsigned long long xp[8];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint4 v = make_uint4(0, 0, 0, 0);
          if (m0 + t < M && kb + 8 * h + 8 <= K)
            v = __ldg(reinterpret_cast<const uint4*>(x + static_cast<int64_t>(m0 + t) * K + kb + 8 * h));
          const uint32_t wx[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int j = 0; j < 4; ++j)
            xp[4 * h + j] = pack2(__uint_as_float(wx[j] << 16), __uint_as_float(wx[j] & 0xFFFF0000u));
        }
#pragma unroll
        for (int r = 0; r < RW; ++r)
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[r][t] = ffma2(xp[j], q[r][j], acc[r][t]);
      }
    }
  }

  if (!waited) pdl_wait();
  // Pairs, then lanes (fixed butterfly), then this warp's K slice to shared memory.
#pragma unroll
  for (int r = 0; r < RW; ++r)
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      float v = __uint_as_float(static_cast<uint32_t>(acc[r][t])) +
                __uint_as_float(static_cast<uint32_t>(acc[r][t] >> 32));
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, off);
      if (lane == 0) part[ks][rg * RW + r][t] = v;
    }
  __syncthreads();
  if (threadIdx.x < RB * MT) {
    const int i = threadIdx.x % RB, t = threadIdx.x / RB;
    float sum = part[0][i][t];
#pragma unroll
    for (int sl = 1; sl < KS; ++sl) sum += part[sl][i][t];
    const int n = blockIdx.x * RB + i;
    if (n < N && m0 + t < M) {
      float v = __fmul_rn(sum, scales[n]);
      if (bias != nullptr) v = __fadd_rn(v, __uint_as_float(static_cast<uint32_t>(bias[n]) << 16));
      const int64_t at = static_cast<int64_t>(m0 + t) * N + n;
      if (kF32Out) static_cast<float*>(y)[at] = v;
      else static_cast<uint16_t*>(y)[at] = f32_to_bf16_rne(v);
    }
  }
}

template <int kKind, bool kNaN, int MT, int KS, bool kF32Out>
cudaError_t launch_ks(const sc_weight* w, const uint16_t* x, int64_t m, const uint16_t* bias, void* y, int m0,
                      cudaStream_t stream) {
  constexpr int RB = (kWarps / KS) * RW;
  const unsigned grid = static_cast<unsigned>(w->n_pad / RB);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemv_w8<kKind, kNaN, MT, KS, kF32Out>, static_cast<const uint8_t*>(w->values),
      static_cast<int>(w->k_pad), static_cast<const float*>(w->scales), x, static_cast<int>(m), static_cast<int>(w->k), bias, y,
      static_cast<int>(w->n), m0);
}

template <int kKind, bool kNaN, int MT, bool kF32Out>
cudaError_t launch_pass(const sc_weight* w, const uint16_t* x, int64_t m, const uint16_t* bias, void* y, int m0,
                        int ks, cudaStream_t stream) {
  switch (ks) {
    case 1: return launch_ks<kKind, kNaN, MT, 1, kF32Out>(w, x, m, bias, y, m0, stream);
    case 2: return launch_ks<kKind, kNaN, MT, 2, kF32Out>(w, x, m, bias, y, m0, stream);
    case 4: return launch_ks<kKind, kNaN, MT, 4, kF32Out>(w, x, m, bias, y, m0, stream);
    default: return launch_ks<kKind, kNaN, MT, 8, kF32Out>(w, x, m, bias, y, m0, stream);
  }
}

template <int kKind, bool kNaN, bool kF32Out>
cudaError_t launch_kind(const sc_weight* w, const uint16_t* x, int64_t m, const uint16_t* bias, void* y, int ks,
                        cudaStream_t stream) {
  for (int m0 = 0; m0 < m;) {
    const int left = static_cast<int>(m) - m0;
    // A pass covers up to eight rows; the last pass rounds its row count up (rows past m are guarded).
    const int mt = left >= 5 ? 8 : left >= 3 ? 4 : left;
    cudaError_t e;
    if (mt == 8) e = launch_pass<kKind, kNaN, 8, kF32Out>(w, x, m, bias, y, m0, ks, stream);
    else if (mt == 4) e = launch_pass<kKind, kNaN, 4, kF32Out>(w, x, m, bias, y, m0, ks, stream);
    else if (mt == 2) e = launch_pass<kKind, kNaN, 2, kF32Out>(w, x, m, bias, y, m0, ks, stream);
    else e = launch_pass<kKind, kNaN, 1, kF32Out>(w, x, m, bias, y, m0, ks, stream);
    if (e != cudaSuccess) return e;
    m0 += mt;
  }
  return cudaSuccess;
}

}  // namespace gemv

// K slices per CTA: the fewest that still give at least eight CTAs per SM (a CTA's rows are
// 16 / slices), and no slice shorter than one 512-byte step of a warp.
int gemv_splits(const sc_weight* w, int64_t m, int sm_count) {
  (void)m;
  const int64_t target = static_cast<int64_t>(sm_count) * 8;
  int ks = 1;
  while (ks < gemv::kWarps && w->n_pad / ((gemv::kWarps / ks) * gemv::RW) < target && w->k_pad / (2 * ks) >= 512)
    ks *= 2;
  return ks;
}

size_t gemv_workspace_bytes(const sc_weight*, int64_t, int) { return 0; }

cudaError_t launch_gemv(const sc_weight* w, const uint16_t* x, int64_t m, const uint16_t* bias, void* y, bool f32_out,
                        float* workspace, int splits, int* err, cudaStream_t stream) {
  (void)workspace;
  (void)err;
  if (w->kind == SC_WEIGHT_INT8)
    return f32_out ? gemv::launch_kind<1, false, true>(w, x, m, bias, y, splits, stream)
                   : gemv::launch_kind<1, false, false>(w, x, m, bias, y, splits, stream);
  if (w->has_nan_codes)
    return f32_out ? gemv::launch_kind<2, true, true>(w, x, m, bias, y, splits, stream)
                   : gemv::launch_kind<2, true, false>(w, x, m, bias, y, splits, stream);
  return f32_out ? gemv::launch_kind<2, false, true>(w, x, m, bias, y, splits, stream)
                 : gemv::launch_kind<2, false, false>(w, x, m, bias, y, splits, stream);
}

}  // namespace sc
