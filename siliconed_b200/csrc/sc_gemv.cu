// The skinny product (1 <= m <= 32): y[m, n] = bf16((sum_k x[m, k] * float(q[k, n])) * s[n] + bias[n]).
//
// Memory-bound: every weight byte is read once per pass.  The arena's transposed layout gives each
// output n a contiguous K row, so a warp streams four such rows with 128-bit non-allocating loads
// (32 lanes x 16 bytes = 512 consecutive K values per row per step) and keeps fp32 sums for up to
// eight activation rows.  K is cut into `splits` ranges, one CTA each; the CTAs of one row block
// form a thread-block cluster, and the first CTA of the cluster adds the others' partial sums in
// split order out of their shared memory (distributed shared memory).  The order of every
// addition is fixed, so each run gives the same bits, as the reference's split GEMV does
// (Sources/Siliconed/DecodeKernels.swift:20-23, :67-109); no global scratch is needed.
#include <cuda_bf16.h>

#include "sc_codes.cuh"
#include "sc_internal.h"
#include "sc_ptx.cuh"

namespace sc {
namespace gemv {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kRowsPerWarp = 4;
constexpr int kRowsPerCta = kWarps * kRowsPerWarp;  // 32 outputs n per CTA
constexpr int kMaxSplits = 8;                       // portable cluster size
constexpr int kMaxTokens = 8;                       // activation rows per pass

__device__ __forceinline__ uint4 ld_stream(const uint8_t* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ float ld_peer_f32(const float* local, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

// Word i (0..3) of a 16-code chunk as four fp32 values.
template <int kKind>
__device__ __forceinline__ void word_to_f32(uint32_t w, float (&f)[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) f[j] = kKind == 1 ? int8_code_to_f32(w, j) : e4m3_code_to_f32<true>(w, j);
}

__device__ __forceinline__ void bf16x8_to_f32(const uint4 v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

template <int kKind, int MT, bool kF32Out>
__global__ void __launch_bounds__(kThreads) gemv_w8(const uint8_t* __restrict__ values, int k_pad,
                                                     const float* __restrict__ scales, const uint16_t* __restrict__ x,
                                                     int M, int K, const uint16_t* __restrict__ bias,
                                                     void* __restrict__ y, int N, int m0, int splits) {
  __shared__ float part[MT][kRowsPerCta];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.y;
  const int units = k_pad / 64;  // split boundaries fall on 64-byte units
  const int k_begin = (split * units / splits) * 64, k_end = ((split + 1) * units / splits) * 64;
  const int nrow0 = blockIdx.x * kRowsPerCta + warp * kRowsPerWarp;
  const uint8_t* wrow = values + static_cast<int64_t>(nrow0) * k_pad;

  float acc[kRowsPerWarp][MT];
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
    for (int t = 0; t < MT; ++t) acc[r][t] = 0.0f;

  for (int kb = k_begin + lane * 16; kb < k_end; kb += 512) {
    uint4 wv[kRowsPerWarp];
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r) wv[r] = ld_stream(wrow + static_cast<int64_t>(r) * k_pad + kb);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int kx = kb + h * 8;
      float wf[kRowsPerWarp][8];
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r) {
        const uint32_t w0 = h == 0 ? wv[r].x : wv[r].z, w1 = h == 0 ? wv[r].y : wv[r].w;
        float a[4], b[4];
        word_to_f32<kKind>(w0, a);
        word_to_f32<kKind>(w1, b);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          wf[r][j] = a[j];
          wf[r][4 + j] = b[j];
        }
      }
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        uint4 xv = make_uint4(0, 0, 0, 0);
        if (m0 + t < M && kx + 8 <= K)
          xv = __ldg(reinterpret_cast<const uint4*>(x + static_cast<int64_t>(m0 + t) * K + kx));
        float xf[8];
        bf16x8_to_f32(xv, xf);
#pragma unroll
        for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[r][t] = fmaf(xf[j], wf[r][j], acc[r][t]);
      }
    }
  }

  // Fixed-order warp reduction, then this CTA's partials to shared memory.
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      float v = acc[r][t];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, off);
      if (lane == 0) part[t][warp * kRowsPerWarp + r] = v;
    }
  if (splits > 1) cluster_sync();
  else __syncthreads();

  if (split == 0 && threadIdx.x < MT * kRowsPerCta) {
    const int t = threadIdx.x / kRowsPerCta, i = threadIdx.x % kRowsPerCta;
    float sum = part[t][i];
    for (int sp = 1; sp < splits; ++sp) sum += ld_peer_f32(&part[t][i], static_cast<uint32_t>(sp));
    const int n = blockIdx.x * kRowsPerCta + i;
    if (n < N && m0 + t < M) {
      float v = __fmul_rn(sum, scales[n]);
      if (bias != nullptr) v = __fadd_rn(v, __uint_as_float(static_cast<uint32_t>(bias[n]) << 16));
      const int64_t at = static_cast<int64_t>(m0 + t) * N + n;
      if (kF32Out) static_cast<float*>(y)[at] = v;
      else static_cast<uint16_t*>(y)[at] = f32_to_bf16_rne(v);
    }
  }
  // Peers keep their shared memory until the first CTA has read it.
  if (splits > 1) cluster_sync();
}

template <int kKind, int MT, bool kF32Out>
cudaError_t launch_pass(const sc_weight* w, const uint16_t* x, int64_t m, const uint16_t* bias, void* y, int m0,
                        int splits, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(w->n_pad / kRowsPerCta), static_cast<unsigned>(splits), 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = static_cast<unsigned>(splits);
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemv_w8<kKind, MT, kF32Out>, static_cast<const uint8_t*>(w->values),
                            static_cast<int>(w->k_pad), static_cast<const float*>(w->scales), x, static_cast<int>(m),
                            static_cast<int>(w->k), bias, y, static_cast<int>(w->n), m0, splits);
}

template <int kKind, bool kF32Out>
cudaError_t launch_kind(const sc_weight* w, const uint16_t* x, int64_t m, const uint16_t* bias, void* y,
                        int splits, cudaStream_t stream) {
  for (int m0 = 0; m0 < m;) {
    const int left = static_cast<int>(m) - m0;
    // A pass covers up to eight rows; the last pass rounds its row count up (rows past m are guarded).
    const int mt = left >= 5 ? 8 : left >= 3 ? 4 : left;
    cudaError_t e;
    if (mt == 8) e = launch_pass<kKind, 8, kF32Out>(w, x, m, bias, y, m0, splits, stream);
    else if (mt == 4) e = launch_pass<kKind, 4, kF32Out>(w, x, m, bias, y, m0, splits, stream);
    else if (mt == 2) e = launch_pass<kKind, 2, kF32Out>(w, x, m, bias, y, m0, splits, stream);
    else e = launch_pass<kKind, 1, kF32Out>(w, x, m, bias, y, m0, splits, stream);
    if (e != cudaSuccess) return e;
    m0 += mt;
  }
  return cudaSuccess;
}

}  // namespace gemv

int gemv_splits(const sc_weight* w, int64_t m, int sm_count) {
  (void)m;
  const int64_t blocks = w->n_pad / gemv::kRowsPerCta;
  const int64_t target = static_cast<int64_t>(sm_count) * 8;  // CTAs to keep the memory system busy
  int64_t splits = (target + blocks - 1) / blocks;
  const int64_t units = w->k_pad / 512;                         // at least one 512-byte step per lane row
  if (splits > units) splits = units;
  if (splits > gemv::kMaxSplits) splits = gemv::kMaxSplits;
  if (splits < 1) splits = 1;
  return static_cast<int>(splits);
}

size_t gemv_workspace_bytes(const sc_weight*, int64_t, int) { return 0; }

cudaError_t launch_gemv(const sc_weight* w, const uint16_t* x, int64_t m, const uint16_t* bias, void* y, bool f32_out,
                        float* workspace, int splits, cudaStream_t stream) {
  (void)workspace;
  if (w->kind == SC_WEIGHT_INT8)
    return f32_out ? gemv::launch_kind<1, true>(w, x, m, bias, y, splits, stream)
                   : gemv::launch_kind<1, false>(w, x, m, bias, y, splits, stream);
  return f32_out ? gemv::launch_kind<2, true>(w, x, m, bias, y, splits, stream)
                 : gemv::launch_kind<2, false>(w, x, m, bias, y, splits, stream);
}

}  // namespace sc
