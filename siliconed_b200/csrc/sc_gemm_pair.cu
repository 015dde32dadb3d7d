// The large-M product on a CTA pair: y = bf16((x . dequant(q)) * s + bias), 5th-generation tensor
// cores with cta_group::2.
//
// A cluster of two CTAs (two SMs of one TPC) owns output tiles of 256 x 256.  Each CTA loads its
// own 128 rows of x and its own 128-column half of the weight's codes, converts only that half to
// bf16, and holds 128 rows x 256 columns of the fp32 accumulator in its TMEM.  The leader CTA
// (rank 0) issues tcgen05.mma.cta_group::2 with M = 256: the tensor cores of both SMs read A from
// each CTA's own shared memory and B from both halves.  Compared with one CTA per 128 x 256 tile,
// every SM converts half as many weight codes per MMA and reads half the B operand, which is what
// bounds this product on B200.
//
// Warp roles in each CTA: warp 0 TMA producer; warp 1 TMEM allocation and (leader only) the MMA
// issuer; warps 4..7 epilogue (TMEM lane quarters 0..3); warps 8..23 converters.  Cross-CTA
// signalling: converters arrive on the leader's b_full; the leader's commits of MMA completion
// arrive on the barriers of both CTAs at once; both epilogues arrive on the leader's acc_empty.  No
// load of this kernel uses cluster multicast (only the completion signal is sent to both CTAs).
// Every wait is bounded.
#include <cuda_bf16.h>

#include "sc_codes.cuh"
#include "sc_internal.h"
#include "sc_ptx.cuh"

// Pipeline timestamps of the first CTA pair, compiled only into diagnostic builds (-DSC_TRACE).
#ifdef SC_TRACE
__device__ unsigned long long g_sc_trace[2][16][512];
#define SC_TRACE_EV(ev, idx) \
  if (blockIdx.x < 2 && (idx) < 512) g_sc_trace[blockIdx.x][(ev)][(idx)] = clock64()
extern "C" __attribute__((visibility("default"))) int sc_debug_trace(void* host, size_t bytes) {
  return static_cast<int>(cudaMemcpyFromSymbol(host, g_sc_trace, bytes < sizeof(g_sc_trace) ? bytes : sizeof(g_sc_trace)));
}
#else
#define SC_TRACE_EV(ev, idx)
#endif

namespace sc {
namespace gemm_pair {

constexpr int BM = 128;            // rows of x per CTA (256 per pair)
constexpr int BN = 256;            // output columns per pair tile (the accumulator's width)
constexpr int BNH = BN / 2;        // weight columns each CTA holds and converts
constexpr int BK = 64;
constexpr int kStages = 5;         // ring of stages: x tile, code half-tile and its bf16 conversion
constexpr int kABytes = BM * BK * 2;
constexpr int kWBytes = BNH * BK;
constexpr int kBBytes = BNH * BK * 2;
constexpr int kWarps = 24;
constexpr int kThreads = kWarps * 32;
constexpr int kEpiWarp0 = 4, kEpiWarps = 4;
constexpr int kConvWarp0 = 8, kConvWarps = 16;  // warps 8..23
constexpr int kConvGroups = 2;                  // groups convert alternate stages concurrently
constexpr int kGroupThreads = kConvWarps * 32 / kConvGroups;
constexpr uint32_t kTmemCols = 512;
constexpr int kChunks = BNH * BK / 8;  // 8-code chunks (one 16-byte bf16 chunk each) per stage

static_assert(kChunks % kGroupThreads == 0, "converter work must divide evenly");

// Converter thread index of warp `warp`, or -1.
__device__ __forceinline__ int converter_index(int warp, int lane) {
  return warp >= kConvWarp0 ? (warp - kConvWarp0) * 32 + lane : -1;
}

struct __align__(1024) Smem {
  uint8_t a[kStages][kABytes];    // x tiles, 128-byte swizzled (TMA)
  uint8_t b[kStages][kBBytes];    // converted weight half-tiles, 128-byte swizzled
  uint8_t w[kStages][kWBytes];    // code half-tiles (TMA)
  float sb[kEpiWarps][2][BN];     // per epilogue warp: the tile's scales and biases
  uint64_t full[kStages];         // this CTA's x and code tiles landed
  uint64_t b_full[kStages];       // leader: both CTAs converted the stage
  uint64_t empty[kStages];        // the pair's MMAs of the stage completed (leader's commit)
  uint64_t acc_full[2];
  uint64_t acc_empty[2];          // leader: both CTAs' epilogues
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int conv_ok[kConvGroups];       // each converter group's elected thread's wait outcome
};

constexpr size_t kSmemBytes = sizeof(Smem) + 1024;

// 8 stored codes (two words, K order) -> 8 bf16 (one 16-byte chunk).
template <int kKind, bool kNaN>
__device__ __forceinline__ uint4 codes8_to_bf16(uint32_t w0, uint32_t w1) {
  float f[8];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (kKind == 1) {
      f[j] = int8_code_to_f32(w0, j);
      f[4 + j] = int8_code_to_f32(w1, j);
    } else {
      f[j] = e4m3_code_to_f32<kNaN>(w0, j);
      f[4 + j] = e4m3_code_to_f32<kNaN>(w1, j);
    }
  }
  return make_uint4(pack_bf16_hi(f[0], f[1]), pack_bf16_hi(f[2], f[3]), pack_bf16_hi(f[4], f[5]),
                    pack_bf16_hi(f[6], f[7]));
}

template <int kKind, bool kNaN, bool kF32Out>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_w8_pair(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                 const float* __restrict__ scales, const uint16_t* __restrict__ bias, void* __restrict__ y_out, int M,
                 int N, int k_tiles, int m_tiles, int n_tiles, int* err) {
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
  const int num_tiles = m_tiles * n_tiles;
  volatile int* abort = &s.abort;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.b_full[i], 2);    // one elected converter thread per CTA
      mbar_init(&s.empty[i], 1);     // the leader's commit
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.acc_full[i], 1);
      mbar_init(&s.acc_empty[i], 2 * kEpiWarps);
    }
    mbar_init(&s.drain, 1);
    s.abort = 0;
    fence_mbar_init();
    prefetch_tensormap(&tm_x);
    prefetch_tensormap(&tm_w);
  }
  if (warp == 1) {
    tmem_alloc_pair(&s.tmem_base, kTmemCols);
    tmem_relinquish_pair();
  }
  __syncwarp();
  tc_fence_before();
  cluster_barrier();  // barriers of both CTAs initialised, TMEM allocated in both
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

  if (warp == 0) {
    // ---------------- TMA producer (each CTA loads its own halves) ----------------
    if (lane == 0) {
      int stage = 0, gcount = 0;
      uint32_t phase = 0, issued = 0, last_parity = 0;
      for (int tile = pair; tile < num_tiles && !*abort; tile += pairs) {
        int mt, nt;
        tile_coords(tile, m_tiles, n_tiles, mt, nt);
        const int row0 = mt * 2 * BM + static_cast<int>(rank) * BM;
        const int col0 = nt * BN + static_cast<int>(rank) * BNH;
        for (int kt = 0; kt < k_tiles; ++kt) {
          if (!mbar_wait(&s.empty[stage], phase ^ 1u, abort, err, kSiteProducerEmpty)) break;
          mbar_arrive_expect_tx(&s.full[stage], kABytes + kWBytes);
          SC_TRACE_EV(0, gcount);
          tma_load_2d(s.a[stage], &tm_x, &s.full[stage], kt * BK, row0);
          tma_load_2d(s.w[stage], &tm_w, &s.full[stage], kt * BK, col0);
          issued |= 1u << stage;
          last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
          ++gcount;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      for (int st = 0; st < kStages; ++st)
        if (issued & (1u << st)) mbar_wait_drain(&s.full[st], (last_parity >> st) & 1u);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader CTA) ----------------
    if (leader && lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(2 * BM, BN);
      int stage = 0, acc = 0, gcount = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += pairs) {
        if (!mbar_wait(&s.acc_empty[acc], acc_phase ^ 1u, abort, err, kSiteMmaAccum)) break;
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(acc * BN);
        // The next stage's barrier is probed before the current stage's MMAs are issued, and the
        // blocking wait runs only when that probe found it incomplete: no barrier operation sits
        // between the last MMA of one stage and the first of the next.
        bool ready = mbar_test_wait(&s.b_full[stage], phase);
        for (int kt = 0; kt < k_tiles; ++kt) {
          // Both CTAs' converters arrive here only after their own x and code tiles landed.
          if (!ready && !mbar_poll(&s.b_full[stage], phase, abort, err, kSiteMmaConverted)) {
            ok = false;
            break;
          }
          SC_TRACE_EV(4, gcount);
          tc_fence_after();
          const int cur = stage;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
          ready = kt + 1 < k_tiles && mbar_test_wait(&s.b_full[stage], phase);
          SC_TRACE_EV(11, gcount);
          const uint32_t a0 = smem_u32(s.a[cur]), b0 = smem_u32(s.b[cur]);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            tc_mma_f16_pair(d, umma_desc_sw128(a0 + kk * 32), umma_desc_sw128(b0 + kk * 32), idesc,
                            (kt | kk) != 0 ? 1u : 0u);
            SC_TRACE_EV(12 + kk, gcount);
          }
          tc_commit_pair_both(&s.empty[cur], 0x3);
          SC_TRACE_EV(5, gcount);
          ++gcount;
        }
        if (!ok) break;
        tc_commit_pair_both(&s.acc_full[acc], 0x3);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      tc_commit_pair(peer_addr(&s.drain, 0));
      mbar_wait_drain(&s.drain, 0);
    }
  } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + kEpiWarps) {
    // ---------------- epilogue (each CTA: its 128 rows x 256 columns) ----------------
    const int ew = warp - kEpiWarp0;
    float* s_scale = s.sb[ew][0];
    float* s_bias = s.sb[ew][1];
    int acc = 0;
    uint32_t acc_phase = 0;
    const bool vec_ok = (N % 8) == 0, vec4_ok = (N % 4) == 0;
    for (int tile = pair; tile < num_tiles; tile += pairs) {
      int mt, nt;
      tile_coords(tile, m_tiles, n_tiles, mt, nt);
      const int n0 = nt * BN;
      const int row = mt * 2 * BM + static_cast<int>(rank) * BM + ew * 32 + lane;
      __syncwarp();
      for (int c = lane; c < BN; c += 32) {
        const int n = n0 + c;
        s_scale[c] = scales[n];
        s_bias[c] = (bias != nullptr && n < N) ? __uint_as_float(static_cast<uint32_t>(bias[n]) << 16) : 0.0f;
      }
      __syncwarp();
      int ready = 0;
      if (lane == 0) ready = mbar_wait(&s.acc_full[acc], acc_phase, abort, err, kSiteEpilogueFull) ? 1 : 0;
      if (!__shfl_sync(0xFFFFFFFFu, ready, 0)) break;
      if (threadIdx.x == kEpiWarp0 * 32) SC_TRACE_EV(6, (tile - pair) / pairs);
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
      if (lane == 0) mbar_arrive_cluster(peer_addr(&s.acc_empty[acc], 0));
      if (threadIdx.x == kEpiWarp0 * 32) SC_TRACE_EV(7, (tile - pair) / pairs);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  } else if (converter_index(warp, lane) >= 0) {
    // ---------------- converters (each CTA: its 128 weight columns) ----------------
    // kConvGroups groups take the K stages in turn (group g: stages g, g + G, ...), so several
    // stages are converted at once.  In a group, one elected thread waits for the stage; a named
    // barrier hands its outcome to the group (all its threads take the same path and always meet at
    // the next barrier); after the conversion a second named barrier gathers the group and the
    // elected thread signals the leader's MMA and this CTA's producer.
    const int cidx = converter_index(warp, lane);
    const int group = cidx / kGroupThreads, ct = cidx % kGroupThreads;
    const int bar_id = 1 + group;
    const int total = ((num_tiles - pair + pairs - 1) / pairs) * k_tiles;  // K stages this CTA runs
    for (int g = group; g < total; g += kConvGroups) {
      // The producer refilled this stage only after the pair's MMAs of its previous round completed,
      // so the bf16 slot of the stage is free as soon as the new code tile has landed.
      const int stage = g % kStages;
      const uint32_t phase = static_cast<uint32_t>(g / kStages) & 1u;
      if (ct == 0) {
        const bool got = mbar_wait(&s.full[stage], phase, abort, err, kSiteConverterFull);
        SC_TRACE_EV(1, g);
        SC_TRACE_EV(2, g);
        s.conv_ok[group] = got;
      }
      named_barrier_sync(bar_id, kGroupThreads);
      if (ct == 0) SC_TRACE_EV(8, g);
      if (!s.conv_ok[group]) break;
      const uint8_t* src = s.w[stage];
      uint8_t* dst = s.b[stage];
      // Eight consecutive threads write the eight 16-byte chunks of one 128-byte row; all loads of a
      // thread are issued before its conversions.
      constexpr int kPer = kChunks / kGroupThreads;
      uint2 in[kPer];
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        const int c = ct + i * kGroupThreads;
        in[i] = *reinterpret_cast<const uint2*>(src + (c >> 3) * BK + (c & 7) * 8);
      }
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        const int c = ct + i * kGroupThreads;
        const int row = c >> 3, j = c & 7;
        *reinterpret_cast<uint4*>(dst + row * (BK * 2) + ((j ^ (row & 7)) << 4)) =
            codes8_to_bf16<kKind, kNaN>(in[i].x, in[i].y);
      }
      if (ct == 0) SC_TRACE_EV(9, g);
      fence_async_shared();
      if (ct == 0) SC_TRACE_EV(10, g);
      named_barrier_sync(bar_id, kGroupThreads);
      if (ct == 0) {
        SC_TRACE_EV(3, g);
        if (leader) mbar_arrive(&s.b_full[stage]);
        else mbar_arrive_cluster(peer_addr(&s.b_full[stage], 0));
      }
    }
  }

  // Neither CTA leaves while the pair's MMAs, TMEM or barriers may still reach its memory.
  __syncwarp();
  tc_fence_before();
  cluster_barrier();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, kTmemCols);
  }
}

template <int kKind, bool kNaN, bool kF32Out>
cudaError_t launch_kind(const CUtensorMap& tm_x, const sc_weight* w, const uint16_t* bias, void* y, int64_t m,
                        int* err, int sm_count, cudaStream_t stream) {
  auto kernel = gemm_w8_pair<kKind, kNaN, kF32Out>;
  static unsigned long long configured = 0;  // per template instance and device
  if (cudaError_t e = set_smem_once(kernel, static_cast<int>(kSmemBytes), configured); e != cudaSuccess) return e;
  const int m_tiles = static_cast<int>((m + 2 * BM - 1) / (2 * BM));
  const int n_tiles = static_cast<int>(w->n_pad / BN);
  const int k_tiles = static_cast<int>(w->k_pad / BK);
  const int tiles = m_tiles * n_tiles;
  const int max_pairs = sm_count / 2;
  const int pairs = tiles < max_pairs ? tiles : max_pairs;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, tm_x, w->tmap_values_half, static_cast<const float*>(w->scales), bias, y,
                            static_cast<int>(m), static_cast<int>(w->n), k_tiles, m_tiles, n_tiles, err);
}

template <bool kF32Out>
cudaError_t launch_out(const CUtensorMap& tm_x, const sc_weight* w, const uint16_t* bias, void* y, int64_t m, int* err,
                       int sm_count, cudaStream_t stream) {
  if (w->kind == SC_WEIGHT_INT8) return launch_kind<1, false, kF32Out>(tm_x, w, bias, y, m, err, sm_count, stream);
  if (w->has_nan_codes) return launch_kind<2, true, kF32Out>(tm_x, w, bias, y, m, err, sm_count, stream);
  return launch_kind<2, false, kF32Out>(tm_x, w, bias, y, m, err, sm_count, stream);
}

}  // namespace gemm_pair

cudaError_t launch_gemm_pair(const CUtensorMap& tmap_x, const sc_weight* w, const uint16_t* bias, void* y,
                             bool f32_out, int64_t m, int* err, int sm_count, cudaStream_t stream) {
  return f32_out ? gemm_pair::launch_out<true>(tmap_x, w, bias, y, m, err, sm_count, stream)
                 : gemm_pair::launch_out<false>(tmap_x, w, bias, y, m, err, sm_count, stream);
}

}  // namespace sc
