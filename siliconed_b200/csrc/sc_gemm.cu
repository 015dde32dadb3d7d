// The large-M product: y = bf16((x . dequant(q)) * s + bias) on the 5th-generation tensor cores.
//
// One persistent CTA per SM walks output tiles of BM x BN = 128 x 256.  Warp roles:
//   warp 0        TMA producer: x tile (bf16 [128 x 64], 128-byte swizzle) and the weight's code
//                 tile (bytes [256 x 64], the arena's transposed [N, K] layout) per K step, into a
//                 4-stage ring completing on one mbarrier per stage.
//   warps 8..15   converters: code tile -> bf16 tile in the K-major 128-byte-swizzled layout the
//                 MMA reads (exact: every int8 / e4m3 value is a bf16), 2-stage ring.
//   warp 1        MMA issuer (one thread): tcgen05.mma kind::f16, M=128, N=256, K=16, fp32
//                 accumulators in TMEM, two accumulators (512 columns) so the epilogue of one tile
//                 overlaps the main loop of the next.  Also allocates / frees TMEM.
//   warps 4..7    epilogue: tcgen05.ld of the accumulator rows, * scale, + bias (two roundings,
//                 as linear_int8 + scale_columns and the separate bias add), bf16, store.
// The scale multiplies the finished fp32 sum, the order of the reference's native int8 route
// (Sources/Siliconed/TensorGEMM.swift:125-179): the weight never passes through a rounded product.
#include <cuda_bf16.h>

#include "sc_codes.cuh"
#include "sc_internal.h"
#include "sc_ptx.cuh"

namespace sc {
namespace gemm {

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int kStagesIn = 4;   // x + code tiles in flight
constexpr int kStagesB = 2;    // converted bf16 weight tiles
constexpr int kABytes = BM * BK * 2;
constexpr int kWBytes = BN * BK;
constexpr int kBBytes = BN * BK * 2;
constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kEpiWarp0 = 4, kEpiWarps = 4;
constexpr int kConvWarp0 = 8, kConvWarps = 8;
constexpr int kConvThreads = kConvWarps * 32;
constexpr uint32_t kTmemCols = 512;
constexpr int kChunksPerStage = BN * BK / 16;  // 16-byte code chunks per code tile

static_assert(kEpiWarp0 % 4 == 0, "epilogue warps must map warp % 4 onto the four TMEM lane quarters");
static_assert(kChunksPerStage % kConvThreads == 0, "converter work must divide evenly");

struct __align__(1024) Smem {
  uint8_t a[kStagesIn][kABytes];     // x tiles, 128-byte swizzled (TMA)
  uint8_t b[kStagesB][kBBytes];      // converted weight tiles, 128-byte swizzled (converters)
  uint8_t w[kStagesIn][kWBytes];     // code tiles (TMA)
  float sb[kEpiWarps][2][BN];        // per epilogue warp: this tile's scales and biases
  uint64_t in_full[kStagesIn];
  uint64_t in_empty[kStagesIn];
  uint64_t b_full[kStagesB];
  uint64_t b_empty[kStagesB];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

constexpr size_t kSmemBytes = sizeof(Smem) + 1024;  // + slack to align the base to 1024

template <int kKind, bool kNaN, bool kF32Out>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_w8_tc(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
               const float* __restrict__ scales, const uint16_t* __restrict__ bias, void* __restrict__ y_out,
               int M, int N, int k_tiles, int m_tiles, int n_tiles, int* err) {
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_tiles = m_tiles * n_tiles;
  volatile int* abort = &s.abort;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStagesIn; ++i) {
      mbar_init(&s.in_full[i], 1);
      mbar_init(&s.in_empty[i], 1 + kConvWarps);  // the MMA's commit + one per converter warp
    }
    for (int i = 0; i < kStagesB; ++i) {
      mbar_init(&s.b_full[i], kConvWarps);
      mbar_init(&s.b_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.acc_full[i], 1);
      mbar_init(&s.acc_empty[i], kEpiWarps);
    }
    mbar_init(&s.drain, 1);
    s.abort = 0;
    fence_mbar_init();
    prefetch_tensormap(&tm_x);
    prefetch_tensormap(&tm_w);
  }
  if (warp == 1) {
    tmem_alloc(&s.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0, last_parity = 0;  // per-stage bit masks
      for (int tile = blockIdx.x; tile < num_tiles && !*abort; tile += gridDim.x) {
        const int mt = tile % m_tiles, nt = tile / m_tiles;
        for (int kt = 0; kt < k_tiles; ++kt) {
          if (!mbar_wait(&s.in_empty[stage], phase ^ 1u, abort, err, kSiteProducerEmpty)) break;
          mbar_arrive_expect_tx(&s.in_full[stage], kABytes + kWBytes);
          tma_load_2d(s.a[stage], &tm_x, &s.in_full[stage], kt * BK, mt * BM);
          tma_load_2d(s.w[stage], &tm_w, &s.in_full[stage], kt * BK, nt * BN);
          issued |= 1u << stage;
          last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == kStagesIn) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Every load this thread issued has landed before the CTA may exit.
      for (int st = 0; st < kStagesIn; ++st)
        if (issued & (1u << st)) mbar_wait_drain(&s.in_full[st], (last_parity >> st) & 1u);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(BM, BN);
      int stage = 0, bstage = 0, acc = 0;
      uint32_t phase = 0, bphase = 0, acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(&s.acc_empty[acc], acc_phase ^ 1u, abort, err, kSiteMmaAccum)) break;
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(acc * BN);
        for (int kt = 0; kt < k_tiles; ++kt) {
          if (!mbar_wait(&s.in_full[stage], phase, abort, err, kSiteMmaInput) ||
              !mbar_wait(&s.b_full[bstage], bphase, abort, err, kSiteMmaConverted)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(s.a[stage]), b0 = smem_u32(s.b[bstage]);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            tc_mma_f16(d, umma_desc_sw128(a0 + kk * 32), umma_desc_sw128(b0 + kk * 32), idesc,
                       (kt | kk) != 0 ? 1u : 0u);
          tc_commit(&s.in_empty[stage]);
          tc_commit(&s.b_empty[bstage]);
          if (++stage == kStagesIn) {
            stage = 0;
            phase ^= 1u;
          }
          if (++bstage == kStagesB) {
            bstage = 0;
            bphase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(&s.acc_full[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      // Every MMA this thread issued has completed before TMEM is released.
      tc_commit(&s.drain);
      mbar_wait_drain(&s.drain, 0);
    }
  } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + kEpiWarps) {
    // ---------------- epilogue ----------------
    const int ew = warp - kEpiWarp0;  // TMEM lanes [32 ew, 32 ew + 32)
    float* s_scale = s.sb[ew][0];
    float* s_bias = s.sb[ew][1];
    int acc = 0;
    uint32_t acc_phase = 0;
    const bool vec_ok = (N % 8) == 0, vec4_ok = (N % 4) == 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const int mt = tile % m_tiles, nt = tile / m_tiles;
      const int n0 = nt * BN, row = mt * BM + ew * 32 + lane;
      __syncwarp();
      for (int c = lane; c < BN; c += 32) {
        const int n = n0 + c;
        s_scale[c] = scales[n];  // the arena's scales are padded to the N tile
        s_bias[c] = (bias != nullptr && n < N) ? __uint_as_float(static_cast<uint32_t>(bias[n]) << 16) : 0.0f;
      }
      __syncwarp();
      if (!mbar_wait(&s.acc_full[acc], acc_phase, abort, err, kSiteEpilogueFull)) break;
      tc_fence_after();
      const uint32_t tbase = tmem + (static_cast<uint32_t>(ew * 32) << 16) + static_cast<uint32_t>(acc * BN);
#pragma unroll 1
      for (int ch = 0; ch < BN / 32; ++ch) {
        uint32_t r[32];
        tmem_ld_32(tbase + ch * 32, r);
        tmem_wait_ld();
        const int n = n0 + ch * 32;
        if (kF32Out) {
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j)
            v[j] = __fadd_rn(__fmul_rn(__uint_as_float(r[j]), s_scale[ch * 32 + j]), s_bias[ch * 32 + j]);
          if (row < M) {
            float* dst = static_cast<float*>(y_out) + static_cast<int64_t>(row) * N + n;
            if (vec4_ok && n + 32 <= N) {
              float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
              for (int q = 0; q < 8; ++q) d4[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (n + j < N) dst[j] = v[j];
            }
          }
        } else {
          uint32_t packed[16];
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            const float v0 =
                __fadd_rn(__fmul_rn(__uint_as_float(r[j]), s_scale[ch * 32 + j]), s_bias[ch * 32 + j]);
            const float v1 = __fadd_rn(__fmul_rn(__uint_as_float(r[j + 1]), s_scale[ch * 32 + j + 1]),
                                       s_bias[ch * 32 + j + 1]);
            const __nv_bfloat162 h = __floats2bfloat162_rn(v0, v1);
            packed[j / 2] = *reinterpret_cast<const uint32_t*>(&h);
          }
          if (row < M) {
            uint16_t* dst = static_cast<uint16_t*>(y_out) + static_cast<int64_t>(row) * N + n;
            if (vec_ok && n + 32 <= N) {
              uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
              for (int q = 0; q < 4; ++q)
                d4[q] = make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (n + j < N) dst[j] = static_cast<uint16_t>(packed[j / 2] >> (16 * (j & 1)));
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.acc_empty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  } else if (warp >= kConvWarp0) {
    // ---------------- converters ----------------
    const int ct = threadIdx.x - kConvWarp0 * 32;
    int stage = 0, bstage = 0;
    uint32_t phase = 0, bphase = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      for (int kt = 0; kt < k_tiles; ++kt) {
        if (!mbar_wait(&s.in_full[stage], phase, abort, err, kSiteConverterFull) ||
            !mbar_wait(&s.b_empty[bstage], bphase ^ 1u, abort, err, kSiteConverterSlot)) {
          ok = false;
          break;
        }
        const uint8_t* src = s.w[stage];
        uint8_t* dst = s.b[bstage];
#pragma unroll
        for (int i = 0; i < kChunksPerStage / kConvThreads; ++i) {
          const int c = ct + i * kConvThreads;
          const int row = c >> 2, kc = c & 3;  // four 16-byte chunks per 64-byte code row
          const uint4 in = *reinterpret_cast<const uint4*>(src + row * BK + kc * 16);
          uint4 lo, hi;
          codes16_to_bf16<kKind, kNaN>(in, lo, hi);
          uint8_t* drow = dst + row * (BK * 2);
          const int sw = row & 7;
          *reinterpret_cast<uint4*>(drow + (((2 * kc) ^ sw) << 4)) = lo;
          *reinterpret_cast<uint4*>(drow + (((2 * kc + 1) ^ sw) << 4)) = hi;
        }
        fence_async_shared();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&s.b_full[bstage]);
          mbar_arrive(&s.in_empty[stage]);
        }
        if (++stage == kStagesIn) {
          stage = 0;
          phase ^= 1u;
        }
        if (++bstage == kStagesB) {
          bstage = 0;
          bphase ^= 1u;
        }
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <int kKind, bool kNaN, bool kF32Out>
cudaError_t launch_kind(const CUtensorMap& tm_x, const sc_weight* w, const uint16_t* bias, void* y, int64_t m,
                        int* err, int sm_count, cudaStream_t stream) {
  auto kernel = gemm_w8_tc<kKind, kNaN, kF32Out>;
  static unsigned long long configured = 0;  // per template instance and device
  if (cudaError_t e = set_smem_once(kernel, static_cast<int>(kSmemBytes), configured); e != cudaSuccess) return e;
  const int m_tiles = static_cast<int>((m + BM - 1) / BM);
  const int n_tiles = static_cast<int>(w->n_pad / BN);
  const int k_tiles = static_cast<int>(w->k_pad / BK);
  const int tiles = m_tiles * n_tiles;
  const int grid = tiles < sm_count ? tiles : sm_count;
  kernel<<<grid, kThreads, kSmemBytes, stream>>>(tm_x, w->tmap_values, w->scales, bias, y, static_cast<int>(m),
                                                 static_cast<int>(w->n), k_tiles, m_tiles, n_tiles, err);
  return cudaGetLastError();
}

}  // namespace gemm

template <bool kF32Out>
cudaError_t launch_out(const CUtensorMap& tmap_x, const sc_weight* w, const uint16_t* bias, void* y, int64_t m,
                       int* err, int sm_count, cudaStream_t stream) {
  if (w->kind == SC_WEIGHT_INT8)
    return gemm::launch_kind<1, false, kF32Out>(tmap_x, w, bias, y, m, err, sm_count, stream);
  if (w->has_nan_codes) return gemm::launch_kind<2, true, kF32Out>(tmap_x, w, bias, y, m, err, sm_count, stream);
  return gemm::launch_kind<2, false, kF32Out>(tmap_x, w, bias, y, m, err, sm_count, stream);
}

cudaError_t launch_gemm_tc(const CUtensorMap& tmap_x, const sc_weight* w, const uint16_t* bias, void* y, bool f32_out,
                           int64_t m, int* err, int sm_count, cudaStream_t stream) {
  return f32_out ? launch_out<true>(tmap_x, w, bias, y, m, err, sm_count, stream)
                 : launch_out<false>(tmap_x, w, bias, y, m, err, sm_count, stream);
}

}  // namespace sc
