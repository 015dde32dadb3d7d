// The skinny product (4 < m <= 32) streamed in equal shares: every SM reads the same number of weight
// bytes, however N and K fall into tiles.
//
// The work is the list of units (column tile t of 128 outputs, 64-wide K stage kt), tile-major, split
// evenly over one CTA per SM: CTA c takes units [c U / G, (c + 1) U / G).  Its share crosses at most a
// few tiles; each run of units inside one tile is a segment, summed in TMEM in K order.  A segment that
// covers its whole tile writes y directly.  Otherwise its fp32 partial goes to the caller's workspace and
// the CTA counts itself on the tile's counter (the context's, returned to zero by the last CTA of the
// tile); the last CTA adds the tile's partials in K order (fragment by fragment, whichever CTA arrives
// last), so every run gives the same bits.
//
// Per unit, as in the cluster kernel (sc_gemm_skinny.cu): TMA brings x's tile (bf16 [MT x 64], 128-byte
// swizzle) and the codes' tile (bytes [128 x 64]); 8 converter warps decode the codes exactly to the
// swizzled bf16 layout; one thread issues four tcgen05.mma kind::f16 (M 128 weight columns, N MT tokens,
// K 16).  The ring holds 12 units (96 KB of codes in flight per SM), and the first 12 code tiles are
// requested before the CTA waits for the kernel ahead of it (programmatic dependent launch): in a decode
// step that kernel produced x, while the codes depend on nothing.  Two TMEM accumulators let a segment's
// epilogue overlap the next segment's MMAs.  No load uses cluster multicast; every wait is bounded.
#include <cuda_bf16.h>

#include "sc_codes.cuh"
#include "sc_internal.h"
#include "sc_ptx.cuh"

namespace sc {
namespace skinny_sk {

constexpr int BN = 128, BK = 64;
constexpr int kStagesIn = 12;
constexpr int kStagesB = 3;
constexpr int kWBytes = BN * BK;
constexpr int kBBytes = BN * BK * 2;
constexpr int kMaxTokens = 32;
constexpr int kXBytesMax = kMaxTokens * BK * 2;
constexpr int kWarps = 16, kThreads = kWarps * 32;
constexpr int kEpiWarp0 = 4, kEpiWarps = 4;
constexpr int kConvWarp0 = 8, kConvWarps = 8, kConvThreads = kConvWarps * 32;
constexpr int kChunksPerStage = BN * BK / 16;
constexpr uint32_t kTmemCols = 64;  // two accumulators of 32 columns
constexpr int kMaxSegments = 4;     // tiles a CTA's share may cross (the host checks)

static_assert(kChunksPerStage % kConvThreads == 0, "converter work must divide evenly");

struct __align__(1024) Smem {
  uint8_t b[kStagesB][kBBytes];         // converted weight tiles (the MMA's A), swizzled
  uint8_t a[kStagesIn][kXBytesMax];     // x tiles (the MMA's B), swizzled (TMA)
  uint8_t w[kStagesIn][kWBytes];        // code tiles (TMA)
  uint64_t in_full[kStagesIn];
  uint64_t in_empty[kStagesIn];
  uint64_t b_full[kStagesB];
  uint64_t b_empty[kStagesB];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int last;  // the fix-up decision of the current segment, for the epilogue warps
};

constexpr size_t kSmemBytes = sizeof(Smem) + 1024;

// The CTA whose share holds unit u: the largest c with floor(c U / G) <= u.
__device__ __forceinline__ int owner(int64_t u, int64_t units, int grid) {
  const int c = static_cast<int>(((u + 1) * grid + units - 1) / units) - 1;
  return c < grid - 1 ? c : grid - 1;
}

__device__ __forceinline__ int64_t share_begin(int c, int64_t units, int grid) { return c * units / grid; }

template <int kKind, bool kNaN, bool kF32Out, int MT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_w8_skinny_sk(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                      const float* __restrict__ scales, const uint16_t* __restrict__ bias, void* __restrict__ y_out,
                      int M, int N, int k_tiles, int n_tiles, float* __restrict__ partials,
                      uint32_t* __restrict__ counters, int* err) {
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grid = static_cast<int>(gridDim.x);
  const int64_t units = static_cast<int64_t>(n_tiles) * k_tiles;
  const int64_t u0 = share_begin(blockIdx.x, units, grid), u1 = share_begin(blockIdx.x + 1, units, grid);
  constexpr int kXBytes = MT * BK * 2;
  volatile int* abort = &s.abort;

  pdl_launch_dependents();
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
      uint32_t phase = 0, issued = 0, last_parity = 0;
      const int pre = static_cast<int>(u1 - u0 < kStagesIn ? u1 - u0 : kStagesIn);
      // the first code tiles do not depend on the kernel ahead: requested before waiting for it
      for (int i = 0; i < pre; ++i) {
        const int64_t u = u0 + i;
        const int t = static_cast<int>(u / k_tiles), kt = static_cast<int>(u - static_cast<int64_t>(t) * k_tiles);
        mbar_arrive_expect_tx(&s.in_full[i], kXBytes + kWBytes);
        tma_load_2d(s.w[i], &tm_w, &s.in_full[i], kt * BK, t * BN);
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i) {
        const int64_t u = u0 + i;
        const int t = static_cast<int>(u / k_tiles), kt = static_cast<int>(u - static_cast<int64_t>(t) * k_tiles);
        tma_load_2d(s.a[i], &tm_x, &s.in_full[i], kt * BK, 0);
        issued |= 1u << i;
        last_parity &= ~(1u << i);
      }
      stage = pre % kStagesIn;
      phase = pre == kStagesIn ? 1u : 0u;
      for (int64_t u = u0 + pre; u < u1 && !*abort; ++u) {
        if (!mbar_wait(&s.in_empty[stage], phase ^ 1u, abort, err, kSiteProducerEmpty)) break;
        const int t = static_cast<int>(u / k_tiles), kt = static_cast<int>(u - static_cast<int64_t>(t) * k_tiles);
        mbar_arrive_expect_tx(&s.in_full[stage], kXBytes + kWBytes);
        tma_load_2d(s.w[stage], &tm_w, &s.in_full[stage], kt * BK, t * BN);
        tma_load_2d(s.a[stage], &tm_x, &s.in_full[stage], kt * BK, 0);
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
      int stage = 0, bstage = 0, acc = 0;
      uint32_t phase = 0, bphase = 0, acc_phase = 0;
      bool ok = true;
      for (int64_t u = u0; u < u1 && ok;) {
        const int t = static_cast<int>(u / k_tiles);
        const int64_t seg_end = u1 < static_cast<int64_t>(t + 1) * k_tiles ? u1 : static_cast<int64_t>(t + 1) * k_tiles;
        if (!mbar_wait(&s.acc_empty[acc], acc_phase ^ 1u, abort, err, kSiteMmaAccum)) break;
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(acc * 32);
        for (int64_t v = u; v < seg_end; ++v) {
          if (!mbar_wait(&s.in_full[stage], phase, abort, err, kSiteMmaInput) ||
              !mbar_wait(&s.b_full[bstage], bphase, abort, err, kSiteMmaConverted)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(s.b[bstage]), b0 = smem_u32(s.a[stage]);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            tc_mma_f16(d, umma_desc_sw128(a0 + kk * 32), umma_desc_sw128(b0 + kk * 32), idesc,
                       (v != u || kk != 0) ? 1u : 0u);
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
        u = seg_end;
      }
      tc_commit(&s.drain);
      mbar_wait_drain(&s.drain, 0);
    }
  } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + kEpiWarps) {
    // ---------------- segment epilogue: y, or a partial and the tile's fix-up ----------------
    const int ew = warp - kEpiWarp0;  // TMEM lanes [32 ew, 32 ew + 32): output columns of the tile
    const int row = ew * 32 + lane;
    int acc = 0, seg = 0;
    uint32_t acc_phase = 0;
    const int tile0 = static_cast<int>(u0 / k_tiles);
    for (int64_t u = u0; u < u1; ++seg) {
      const int t = static_cast<int>(u / k_tiles);
      const int64_t tile_end = static_cast<int64_t>(t + 1) * k_tiles;
      const int64_t seg_end = u1 < tile_end ? u1 : tile_end;
      const bool whole = u == static_cast<int64_t>(t) * k_tiles && seg_end == tile_end;
      int got = 0;
      if (lane == 0) got = mbar_wait(&s.acc_full[acc], acc_phase, abort, err, kSiteEpilogueFull) ? 1 : 0;
      got = __shfl_sync(0xFFFFFFFFu, got, 0);
      float v[MT];
      if (got) {
        tc_fence_after();
        uint32_t r[32];
        tmem_ld_32(tmem + (static_cast<uint32_t>(ew * 32) << 16) + static_cast<uint32_t>(acc * 32), r);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < MT; ++i) v[i] = __uint_as_float(r[i]);
      } else {
#pragma unroll
        for (int i = 0; i < MT; ++i) v[i] = 0.0f;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.acc_empty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
      const int n = t * BN + row;
      bool store = whole;
      if (!whole) {
        float* mine = partials + ((static_cast<int64_t>(blockIdx.x) * kMaxSegments + seg) * BN + row) * kMaxTokens;
#pragma unroll
        for (int i = 0; i < MT; i += 4)
          *reinterpret_cast<float4*>(mine + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
        __threadfence();
        named_barrier_sync(1, kEpiWarps * 32);
        const int c_first = owner(static_cast<int64_t>(t) * k_tiles, units, grid);
        const int c_last = owner(tile_end - 1, units, grid);
        if (row == 0) {
          const uint32_t old = atomicAdd(counters + t, 1u);
          const int last = old == static_cast<uint32_t>(c_last - c_first);
          if (last) counters[t] = 0;  // every CTA of the tile has counted: ready for the next launch
          s.last = last;
        }
        named_barrier_sync(1, kEpiWarps * 32);
        store = s.last != 0;
        if (store) {
          __threadfence();
          // the tile's partials in K order (CTA c_first's fragment first), whichever CTA came last
#pragma unroll
          for (int i = 0; i < MT; ++i) v[i] = 0.0f;
          for (int c = c_first; c <= c_last; ++c) {
            const int cseg = t - static_cast<int>(share_begin(c, units, grid) / k_tiles);
            const float* f = partials + ((static_cast<int64_t>(c) * kMaxSegments + cseg) * BN + row) * kMaxTokens;
#pragma unroll
            for (int i = 0; i < MT; i += 4) {
              const float4 q = ld_cg_f4(f + i);
              if (c == c_first) {
                v[i] = q.x;
                v[i + 1] = q.y;
                v[i + 2] = q.z;
                v[i + 3] = q.w;
              } else {
                v[i] = __fadd_rn(v[i], q.x);
                v[i + 1] = __fadd_rn(v[i + 1], q.y);
                v[i + 2] = __fadd_rn(v[i + 2], q.z);
                v[i + 3] = __fadd_rn(v[i + 3], q.w);
              }
            }
          }
        }
      }
      if (store && n < N) {
        const float sc = scales[n];
        const float b = bias != nullptr ? __uint_as_float(static_cast<uint32_t>(bias[n]) << 16) : 0.0f;
#pragma unroll
        for (int i = 0; i < MT; ++i)
          if (i < M) {
            const float o = __fadd_rn(__fmul_rn(v[i], sc), b);
            if (kF32Out) static_cast<float*>(y_out)[static_cast<int64_t>(i) * N + n] = o;
            else static_cast<uint16_t*>(y_out)[static_cast<int64_t>(i) * N + n] = f32_to_bf16_rne(o);
          }
      }
      u = seg_end;
    }
    (void)tile0;
  } else if (warp >= kConvWarp0) {
    // ---------------- converters ----------------
    const int ct = threadIdx.x - kConvWarp0 * 32;
    int stage = 0, bstage = 0;
    uint32_t phase = 0, bphase = 0;
    for (int64_t u = u0; u < u1; ++u) {
      if (!mbar_wait(&s.in_full[stage], phase, abort, err, kSiteConverterFull) ||
          !mbar_wait(&s.b_empty[bstage], bphase ^ 1u, abort, err, kSiteConverterSlot))
        break;
      const uint8_t* src = s.w[stage];
      uint8_t* dst = s.b[bstage];
#pragma unroll
      for (int i = 0; i < kChunksPerStage / kConvThreads; ++i) {
        const int c = ct + i * kConvThreads;
        const int r = c >> 2, kc = c & 3;  // four 16-byte chunks per 64-byte code row
        const uint4 in = *reinterpret_cast<const uint4*>(src + r * BK + kc * 16);
        uint4 lo, hi;
        codes16_to_bf16<kKind, kNaN>(in, lo, hi);
        uint8_t* drow = dst + r * (BK * 2);
        const int sw = r & 7;
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

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <int kKind, bool kNaN, bool kF32Out, int MT>
cudaError_t launch_mt(const CUtensorMap& tm_x, const sc_weight* w, const uint16_t* bias, void* y, int64_t m,
                      float* partials, uint32_t* counters, int grid, int* err, cudaStream_t stream) {
  auto kernel = gemm_w8_skinny_sk<kKind, kNaN, kF32Out, MT>;
  static unsigned long long configured = 0;  // per template instance and device
  if (cudaError_t e = set_smem_once(kernel, static_cast<int>(kSmemBytes), configured); e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, tm_x, w->tmap_values_half, static_cast<const float*>(w->scales), bias, y,
                            static_cast<int>(m), static_cast<int>(w->n), static_cast<int>(w->k_pad / BK),
                            static_cast<int>(w->n_pad / BN), partials, counters, err);
}

template <int kKind, bool kNaN, bool kF32Out>
cudaError_t launch_kind(const CUtensorMap& tm_x, const sc_weight* w, const uint16_t* bias, void* y, int64_t m,
                        float* partials, uint32_t* counters, int grid, int* err, cudaStream_t stream) {
  if (m <= 16) return launch_mt<kKind, kNaN, kF32Out, 16>(tm_x, w, bias, y, m, partials, counters, grid, err, stream);
  return launch_mt<kKind, kNaN, kF32Out, 32>(tm_x, w, bias, y, m, partials, counters, grid, err, stream);
}

}  // namespace skinny_sk

// CTAs of the streamed skinny product for this weight (0 when it does not apply: fewer units than SMs'
// worth of work, a share crossing more tiles than a CTA keeps partials for, or too many tiles to count).
int skinny_sk_grid(const sc_weight* w, int sm_count) {
  using namespace skinny_sk;
  const int64_t k_tiles = w->k_pad / BK, n_tiles = w->n_pad / BN, units = k_tiles * n_tiles;
  if (n_tiles > kSkinnyCounterWords || units < 2 * static_cast<int64_t>(sm_count)) return 0;
  const int64_t per = (units + sm_count - 1) / sm_count;
  if ((per - 1) / k_tiles + 2 > kMaxSegments) return 0;
  return sm_count;
}

size_t skinny_sk_workspace_bytes(int grid) {
  using namespace skinny_sk;
  return static_cast<size_t>(grid) * kMaxSegments * BN * kMaxTokens * sizeof(float);
}

cudaError_t launch_gemm_skinny_sk(const CUtensorMap& tmap_x, const sc_weight* w, const uint16_t* bias, void* y,
                                  bool f32_out, int64_t m, float* partials, uint32_t* counters, int grid, int* err,
                                  cudaStream_t stream) {
  using namespace skinny_sk;
  if (w->kind == SC_WEIGHT_INT8)
    return f32_out ? launch_kind<1, false, true>(tmap_x, w, bias, y, m, partials, counters, grid, err, stream)
                   : launch_kind<1, false, false>(tmap_x, w, bias, y, m, partials, counters, grid, err, stream);
  if (w->has_nan_codes)
    return f32_out ? launch_kind<2, true, true>(tmap_x, w, bias, y, m, partials, counters, grid, err, stream)
                   : launch_kind<2, true, false>(tmap_x, w, bias, y, m, partials, counters, grid, err, stream);
  return f32_out ? launch_kind<2, false, true>(tmap_x, w, bias, y, m, partials, counters, grid, err, stream)
                 : launch_kind<2, false, false>(tmap_x, w, bias, y, m, partials, counters, grid, err, stream);
}

}  // namespace sc
