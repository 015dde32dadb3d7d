// The skinny product on the tensor cores: 4 < m <= 128 activation rows (encoder prompts, batched
// decode), where the GEMV's CUDA-core arithmetic, not HBM, sets the pace, and where 128 x 256 output
// tiles would leave most SMs idle (an encoder's [9728, 2560] at 128 rows is 38 such tiles).
//
// Operands swapped: the MMA's M is 128 weight columns (output n), its N the m tokens padded to 16, 32,
// 64 or 128, so D[n, t] = sum_k W[k, n] x[t, k] sits in TMEM with one output column per lane.  A CTA owns
// 128 output columns and one K part; the KS CTAs of a cluster (KS in {1, 2, 4, 8}) take the K parts
// of the same columns, so every SM streams codes even when N / 128 is small.  Per 64-wide K stage:
// TMA brings the x tile (bf16 [MT x 64], 128-byte swizzle) and the code tile (bytes [128 x 64]),
// 8 converter warps decode the codes exactly into the K-major swizzled bf16 layout, and one thread
// issues four tcgen05.mma kind::f16 (M 128, N MT, K 16).  At the end each CTA's 4 epilogue warps
// read their partial D and store it in shared memory; after a cluster barrier the leader CTA adds the
// partials of ranks 0 .. KS - 1 in rank order through distributed shared memory (deterministic, no
// workspace), applies scale and bias, and writes y[t, n].  No load uses cluster multicast; every
// wait is bounded.
#include <cuda_bf16.h>

#include "sc_codes.cuh"
#include "sc_internal.h"
#include "sc_ptx.cuh"

namespace sc {
namespace gemm_skinny {

constexpr int BN = 128, BK = 64;  // weight columns per CTA (the MMA's M), K per stage
constexpr int kStagesB = 2;       // converted bf16 weight tiles
// x + code tiles in flight: 4, or 3 for 128 tokens (16 KB x tiles), so that two CTAs share an SM
template <int MT>
constexpr int stages_in() { return MT >= 128 ? 3 : 4; }
constexpr int kWBytes = BN * BK;
constexpr int kBBytes = BN * BK * 2;
constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kEpiWarp0 = 4, kEpiWarps = 4;
constexpr int kConvWarp0 = 8, kConvWarps = 8;
constexpr int kConvThreads = kConvWarps * 32;
constexpr int kChunksPerStage = BN * BK / 16;

static_assert(kChunksPerStage % kConvThreads == 0, "converter work must divide evenly");
static_assert(kThreads == 8 * (BN / 2), "the sums: a column pair and every eighth token a thread");

template <int MT>
struct __align__(1024) Smem {
  static constexpr int kStagesIn = stages_in<MT>();
  union {
    struct {
      uint8_t b[kStagesB][kBBytes];           // converted weight tiles (the MMA's A), swizzled
      uint8_t a[kStagesIn][MT * BK * 2];      // x tiles (the MMA's B), swizzled (TMA)
      uint8_t w[kStagesIn][kWBytes];          // code tiles (TMA)
    };
    // This CTA's partial D, token-major (rows of the tile's 128 columns, padded to 16-byte units), written once
    // the last MMA has completed, when no copy or conversion writes the pipeline's buffers any more.
    float part[MT][BN + 4];
  };
  uint64_t in_full[kStagesIn];
  uint64_t in_empty[kStagesIn];
  uint64_t b_full[kStagesB];
  uint64_t b_empty[kStagesB];
  uint64_t acc_full;
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

template <int MT>
constexpr size_t smem_bytes() { return sizeof(Smem<MT>) + 1024; }
static_assert(smem_bytes<128>() <= 113 * 1024 && smem_bytes<64>() <= 113 * 1024, "two CTAs an SM");


template <int kKind, bool kNaN, bool kF32Out, int MT>
__global__ void __launch_bounds__(kThreads, 2)
    gemm_w8_skinny(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                   const float* __restrict__ scales, const uint16_t* __restrict__ bias, void* __restrict__ y_out,
                   int M, int N, int k_tiles, int* err) {
  constexpr int kStagesIn = Smem<MT>::kStagesIn;
  constexpr uint32_t kTmemCols = MT < 32 ? 32u : static_cast<uint32_t>(MT);
  extern __shared__ uint8_t smem_raw[];
  Smem<MT>& s = *reinterpret_cast<Smem<MT>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  uint32_t ks_count;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(ks_count));
  const int tile = static_cast<int>(blockIdx.x / ks_count);
  const int kt0 = static_cast<int>(static_cast<int64_t>(rank) * k_tiles / ks_count);
  const int kt1 = static_cast<int>(static_cast<int64_t>(rank + 1) * k_tiles / ks_count);
  constexpr int kABytes = MT * BK * 2;
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
    mbar_init(&s.acc_full, 1);
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
      uint32_t phase = 0, issued = 0, last_parity = 0;
      for (int kt = kt0; kt < kt1 && !*abort; ++kt) {
        if (!mbar_wait(&s.in_empty[stage], phase ^ 1u, abort, err, kSiteProducerEmpty)) break;
        mbar_arrive_expect_tx(&s.in_full[stage], kABytes + kWBytes);
        tma_load_2d(s.a[stage], &tm_x, &s.in_full[stage], kt * BK, 0);
        tma_load_2d(s.w[stage], &tm_w, &s.in_full[stage], kt * BK, tile * BN);
        issued |= 1u << stage;
        last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
        if (++stage == kStagesIn) {
          stage = 0;
          phase ^= 1u;
        }
      }
      for (int st = 0; st < kStagesIn; ++st)
        if (issued & (1u << st)) mbar_wait_drain(&s.in_full[st], (last_parity >> st) & 1u);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(BN, MT);
      int stage = 0, bstage = 0;
      uint32_t phase = 0, bphase = 0;
      bool ok = true;
      for (int kt = kt0; kt < kt1; ++kt) {
        if (!mbar_wait(&s.in_full[stage], phase, abort, err, kSiteMmaInput) ||
            !mbar_wait(&s.b_full[bstage], bphase, abort, err, kSiteMmaConverted)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = smem_u32(s.b[bstage]), b0 = smem_u32(s.a[stage]);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)
          tc_mma_f16(tmem, umma_desc_sw128(a0 + kk * 32), umma_desc_sw128(b0 + kk * 32), idesc,
                     (kt != kt0 || kk != 0) ? 1u : 0u);
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
      if (ok) tc_commit(&s.acc_full);
      tc_commit(&s.drain);
      mbar_wait_drain(&s.drain, 0);
    }
  } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + kEpiWarps) {
    // ---------------- partial D -> shared memory ----------------
    const int ew = warp - kEpiWarp0;  // TMEM lanes [32 ew, 32 ew + 32): output columns
    int got = 0;
    if (lane == 0) got = mbar_wait(&s.acc_full, 0, abort, err, kSiteEpilogueFull) ? 1 : 0;
    got = __shfl_sync(0xFFFFFFFFu, got, 0);
    const int col = ew * 32 + lane;
    if (got) {
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < (MT + 31) / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32(tmem + (static_cast<uint32_t>(ew * 32) << 16) + c * 32, r);
        tmem_wait_ld();
#pragma unroll
        for (int t = 0; t < 32; ++t)
          if (c * 32 + t < MT) s.part[c * 32 + t][col] = __uint_as_float(r[t]);
      }
    } else {
#pragma unroll
      for (int t = 0; t < MT; ++t) s.part[t][col] = 0.0f;
    }
  } else if (warp >= kConvWarp0) {
    // ---------------- converters ----------------
    const int ct = threadIdx.x - kConvWarp0 * 32;
    int stage = 0, bstage = 0;
    uint32_t phase = 0, bphase = 0;
    for (int kt = kt0; kt < kt1; ++kt) {
      if (!mbar_wait(&s.in_full[stage], phase, abort, err, kSiteConverterFull) ||
          !mbar_wait(&s.b_empty[bstage], bphase ^ 1u, abort, err, kSiteConverterSlot))
        break;
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

  // Every CTA's partial is in its shared memory.  Each CTA of the cluster then takes a share of the tokens and
  // adds the KS partials of its tokens in rank order 0 .. KS - 1 (its own from shared memory, the peers' through
  // distributed shared memory): the same sums in the same order whichever CTA adds them.  A thread takes a pair
  // of columns and every eighth token of the share, so a warp reads 256 contiguous bytes of a partial row and
  // writes 128 contiguous bytes of y.
  __syncwarp();
  tc_fence_before();
  cluster_barrier();
  {
    const int cp = threadIdx.x % (BN / 2), tg = threadIdx.x / (BN / 2);  // column pair, token group (0..7)
    const int n = tile * BN + 2 * cp;
    const int t_lo = static_cast<int>(rank) * MT / static_cast<int>(ks_count);
    const int t_hi = static_cast<int>(rank + 1) * MT / static_cast<int>(ks_count);
    const float2 sc = make_float2(n < N ? scales[n] : 0.0f, n + 1 < N ? scales[n + 1] : 0.0f);
    float2 b = make_float2(0.0f, 0.0f);
    if (bias != nullptr) {
      if (n < N) b.x = __uint_as_float(static_cast<uint32_t>(bias[n]) << 16);
      if (n + 1 < N) b.y = __uint_as_float(static_cast<uint32_t>(bias[n + 1]) << 16);
    }
    const bool pair_store = (N & 1) == 0 && n + 1 < N;
    for (int t = t_lo + tg; t < t_hi && t < M; t += kThreads / (BN / 2)) {
      float2 acc = make_float2(0.0f, 0.0f);
      for (uint32_t q = 0; q < ks_count; ++q) {
        float2 v;
        if (q == rank) {
          v = *reinterpret_cast<const float2*>(&s.part[t][2 * cp]);
        } else {
          asm volatile("ld.shared::cluster.v2.f32 {%0, %1}, [%2];"
                       : "=f"(v.x), "=f"(v.y)
                       : "r"(peer_addr(&s.part[t][2 * cp], q))
                       : "memory");
        }
        if (q == 0) {
          acc = v;
        } else {
          acc.x = __fadd_rn(acc.x, v.x);
          acc.y = __fadd_rn(acc.y, v.y);
        }
      }
      const float o0 = __fadd_rn(__fmul_rn(acc.x, sc.x), b.x), o1 = __fadd_rn(__fmul_rn(acc.y, sc.y), b.y);
      const int64_t off = static_cast<int64_t>(t) * N + n;
      if (kF32Out) {
        float* yo = static_cast<float*>(y_out) + off;
        if (pair_store) *reinterpret_cast<float2*>(yo) = make_float2(o0, o1);
        else {
          if (n < N) yo[0] = o0;
          if (n + 1 < N) yo[1] = o1;
        }
      } else {
        uint16_t* yo = static_cast<uint16_t*>(y_out) + off;
        if (pair_store) *reinterpret_cast<uint32_t*>(yo) = static_cast<uint32_t>(f32_to_bf16_rne(o0)) |
                                                            (static_cast<uint32_t>(f32_to_bf16_rne(o1)) << 16);
        else {
          if (n < N) yo[0] = f32_to_bf16_rne(o0);
          if (n + 1 < N) yo[1] = f32_to_bf16_rne(o1);
        }
      }
    }
  }
  // Every CTA's partial stays in place until the other CTAs have read it.
  cluster_barrier();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <int kKind, bool kNaN, bool kF32Out, int MT>
cudaError_t launch_mt(const CUtensorMap& tm_x, const sc_weight* w, const uint16_t* bias, void* y, int64_t m, int* err,
                      int sm_count, cudaStream_t stream) {
  auto kernel = gemm_w8_skinny<kKind, kNaN, kF32Out, MT>;
  static unsigned long long configured = 0;  // per template instance and device
  if (cudaError_t e = set_smem_once(kernel, static_cast<int>(smem_bytes<MT>()), configured); e != cudaSuccess) return e;
  const int n_tiles = static_cast<int>(w->n_pad / BN);
  const int k_tiles = static_cast<int>(w->k_pad / BK);
  int ks = 1;
  while (ks < 8 && n_tiles * ks * 2 <= sm_count * 2 && k_tiles / (ks * 2) >= 2) ks *= 2;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(n_tiles * ks), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem_bytes<MT>();
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(ks);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, tm_x, w->tmap_values_half, static_cast<const float*>(w->scales), bias, y,
                            static_cast<int>(m), static_cast<int>(w->n), k_tiles, err);
}

template <int kKind, bool kNaN, bool kF32Out>
cudaError_t launch_kind(const CUtensorMap& tm_x, const sc_weight* w, const uint16_t* bias, void* y, int64_t m, int* err,
                        int sm_count, cudaStream_t stream) {
  if (m <= 16) return launch_mt<kKind, kNaN, kF32Out, 16>(tm_x, w, bias, y, m, err, sm_count, stream);
  if (m <= 32) return launch_mt<kKind, kNaN, kF32Out, 32>(tm_x, w, bias, y, m, err, sm_count, stream);
  if (m <= 64) return launch_mt<kKind, kNaN, kF32Out, 64>(tm_x, w, bias, y, m, err, sm_count, stream);
  return launch_mt<kKind, kNaN, kF32Out, 128>(tm_x, w, bias, y, m, err, sm_count, stream);
}

}  // namespace gemm_skinny

int gemm_skinny_box_rows(int64_t m) { return m <= 16 ? 16 : m <= 32 ? 32 : m <= 64 ? 64 : 128; }

cudaError_t launch_gemm_skinny(const CUtensorMap& tmap_x, const sc_weight* w, const uint16_t* bias, void* y,
                               bool f32_out, int64_t m, int* err, int sm_count, cudaStream_t stream) {
  using namespace gemm_skinny;
  if (w->kind == SC_WEIGHT_INT8)
    return f32_out ? launch_kind<1, false, true>(tmap_x, w, bias, y, m, err, sm_count, stream)
                   : launch_kind<1, false, false>(tmap_x, w, bias, y, m, err, sm_count, stream);
  if (w->has_nan_codes)
    return f32_out ? launch_kind<2, true, true>(tmap_x, w, bias, y, m, err, sm_count, stream)
                   : launch_kind<2, true, false>(tmap_x, w, bias, y, m, err, sm_count, stream);
  return f32_out ? launch_kind<2, false, true>(tmap_x, w, bias, y, m, err, sm_count, stream)
                 : launch_kind<2, false, false>(tmap_x, w, bias, y, m, err, sm_count, stream);
}

}  // namespace sc
