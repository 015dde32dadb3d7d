// The int8 skinny product (4 < m <= 16) on the integer tensor cores, the codes read as stored.
//
// Converting every code to bf16 before a kind::f16 MMA is what bounds a skinny product: the conversion runs
// on the CUDA cores at one pass per 64-code sub-tile, and on B200 it held both skinny designs to about
// 0.9 us per 8 KB of codes per SM (33-39 us for config 4's 50 MB weight) with the tensor pipe 3 % busy.
// Here the codes never change form.  Each row of x (bf16) is first written as an exact fixed-point
// integer v = round(x * 2^(21 - e)), e the row's largest exponent (|v| < 2^22: every value whose exponent
// is within 14 of the row's largest is exact, the rest are rounded at 2^-22 of the largest, finer than an
// fp32 sum keeps), split into three signed 8-bit digits v = d0 + 2^8 d1 + 2^16 d2 (x_planes).  The product
// then multiplies the arena's biased codes u = q + 128 (unsigned 8-bit, A) by the digit planes (signed 8-bit,
// B, the 3 MT rows of one MMA of N = 3 MT) with tcgen05.mma kind::i8 into s32 accumulators: sum_d 2^(8d)
// acc_d = sum_k v_k u_k exactly, and subtracting 128 sum_k v_k leaves sum_k v_k q_k, an exact integer.  The
// epilogue turns it into the fp32 sum with one rounding (times 2^(e - 21), exact), then applies the scale
// and the bias as the native route does.  The sum is exact where the fp32 route rounds at every step, so
// the results agree with the oracle's fp32 sums to within their rounding.
//
// The work is the list of units (column tile t of 128 outputs, 256-wide K chunk kt), tile-major, split
// evenly over one CTA per SM: CTA c takes units [c U / G, (c + 1) U / G), so every SM reads the same
// number of weight bytes.  Its share crosses at most a few tiles; each run of units inside one tile is a
// segment, summed in TMEM.  A segment that covers its whole tile writes y directly.  Otherwise its integer
// partial (int64, exact) goes to the caller's workspace and the CTA counts itself on the tile's counter
// (the context's, returned to zero by the tile's last CTA); the last CTA adds the tile's partials, exactly,
// so every run gives the same bits.  Per unit, TMA brings the codes as two 16 KB boxes (128 bytes x 128
// rows, 128-byte swizzle: the MMA's operand layout as stored) and the planes as two [3 MT x 128] boxes; a
// ring of 5 units keeps 160 KB of codes in flight per SM, the first ones requested
// before the CTA waits for the kernel ahead of it (programmatic dependent launch).  No load uses cluster
// multicast; every wait is bounded.
#include <cuda_bf16.h>

#include "sc_codes.cuh"
#include "sc_internal.h"
#include "sc_ptx.cuh"

namespace sc {
namespace skinny_i8 {

constexpr int BN = 128;                 // weight columns per tile (the MMA's M)
constexpr int BKU = 256;                // K of a unit: two 128-byte boxes
constexpr int kBoxBytes = BN * 128;     // 16 KB
constexpr int kCodeBytes = 2 * kBoxBytes;
constexpr int kTokens = 16;            // x rows a launch takes (m <= 16; the rows past m are zeros)
constexpr int kStages = 5;             // ring depth: 5 units, 160 KB of codes and 60 KB of planes
constexpr int kWarps = 8, kThreads = kWarps * 32;
constexpr int kEpiWarp0 = 4, kEpiWarps = 4;
constexpr uint32_t kTmemCols = 256;     // two accumulators of 3 MT columns, 128 apart
constexpr int kSlots = 2;               // partial slots per CTA: its first and its last segment
constexpr int kZeroRow = -100000;       // x_planes' exponent of a row of zeros
constexpr int kBadRow = 100000;         // ... of a row holding an infinity or a NaN

template <int MT>
struct __align__(1024) Smem {
  uint8_t w[kStages][kCodeBytes];           // codes: [2][128 rows][128 bytes], 128-byte swizzled (TMA)
  uint8_t p[kStages][2][3 * MT * 128];      // planes: [2][3 MT rows][128 bytes], 128-byte swizzled (TMA)
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int last;  // the fix-up decision of the current segment, for the epilogue warps
  int shift[kTokens];         // the rows' shifts and corrections, staged once by the epilogue warps
  long long corr[kTokens];
};

template <int MT>
constexpr size_t smem_bytes() { return sizeof(Smem<MT>) + 1024; }
static_assert(smem_bytes<kTokens>() <= 227 * 1024, "shared memory per CTA");

// ---- x_planes: one CTA per token row (MT of them, rows past m all zero) ----------------------------
// planes [3 MT][k_pad] int8 (row d MT + t: digit d of token t), shift[t] = e - 148 (the power of two of
// v's unit, e the row's largest biased bf16 exponent; kZeroRow / kBadRow for a row of zeros / with a
// non-finite value), corr[t] = 128 sum_k v_k.  Each thread takes 8 consecutive values (16-byte loads, 8-byte
// stores per plane); k_pad is a multiple of 64 and K of 8.
constexpr int kPlaneThreads = 1024;

__device__ __forceinline__ int fixed_point(uint32_t b, int E) {
  const int e = (b >> 7) & 0xFF;
  if (e == 0) return 0;                                 // zero (and subnormal: below every kept digit)
  const int a = static_cast<int>(128u | (b & 0x7Fu));   // the significand, 8 bits
  const int sh = e - E + 14;                            // v = a * 2^sh
  int mag;
  if (sh >= 0) {
    mag = a << sh;                                      // sh <= 14: below 2^22
  } else {
    const int r = -sh;                                  // round to nearest, ties to even
    mag = r >= 31 ? 0 : (a >> r) + ((((a >> (r - 1)) & 1) && ((a & ((1 << (r - 1)) - 1)) || ((a >> r) & 1))) ? 1 : 0);
  }
  return (b & 0x8000u) ? -mag : mag;
}

__global__ void __launch_bounds__(kPlaneThreads)
    x_planes(const uint16_t* __restrict__ x, int M, int K, int k_pad, int MT, int8_t* __restrict__ planes,
             int* __restrict__ shift, long long* __restrict__ corr) {
  pdl_launch_dependents();  // the product may launch and request its codes now
  pdl_wait();               // x is the kernel ahead's output
  __shared__ int s_max;
  __shared__ unsigned long long s_sum;
  const int t = blockIdx.x;
  if (threadIdx.x == 0) {
    s_max = 0;
    s_sum = 0ull;
  }
  __syncthreads();
  const uint4* row = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(t) * K);
  const int chunks = K / 8, pad_chunks = k_pad / 8;
  int e_max = 0;
  if (t < M)
    for (int c = threadIdx.x; c < chunks; c += blockDim.x) {
      const uint4 v = __ldg(row + c);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) e_max = max(e_max, max((w[i] >> 7) & 0xFF, (w[i] >> 23) & 0xFF));
    }
  e_max = static_cast<int>(__reduce_max_sync(0xFFFFFFFFu, static_cast<unsigned>(e_max)));
  if ((threadIdx.x & 31) == 0) atomicMax(&s_max, e_max);  // one shared atomic per warp
  __syncthreads();
  const int E = s_max;
  long long sum = 0;
  uint2* p0 = reinterpret_cast<uint2*>(planes + static_cast<int64_t>(t) * k_pad);
  uint2* p1 = reinterpret_cast<uint2*>(planes + static_cast<int64_t>(MT + t) * k_pad);
  uint2* p2 = reinterpret_cast<uint2*>(planes + static_cast<int64_t>(2 * MT + t) * k_pad);
  for (int c = threadIdx.x; c < pad_chunks; c += blockDim.x) {
    uint32_t w[4] = {0, 0, 0, 0};
    if (t < M && c < chunks && E < 255) {
      const uint4 v = __ldg(row + c);
      w[0] = v.x;
      w[1] = v.y;
      w[2] = v.z;
      w[3] = v.w;
    }
    uint32_t d0[2] = {0, 0}, d1[2] = {0, 0}, d2[2] = {0, 0};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t b = (w[i >> 1] >> (16 * (i & 1))) & 0xFFFFu;
      const int v = fixed_point(b, E);
      sum += v;
      const int g0 = ((v + 128) & 255) - 128;
      const int v1 = (v - g0) >> 8;
      const int g1 = ((v1 + 128) & 255) - 128;
      const int g2 = (v1 - g1) >> 8;
      d0[i >> 2] |= (static_cast<uint32_t>(g0) & 0xFFu) << (8 * (i & 3));
      d1[i >> 2] |= (static_cast<uint32_t>(g1) & 0xFFu) << (8 * (i & 3));
      d2[i >> 2] |= (static_cast<uint32_t>(g2) & 0xFFu) << (8 * (i & 3));
    }
    p0[c] = make_uint2(d0[0], d0[1]);
    p1[c] = make_uint2(d1[0], d1[1]);
    p2[c] = make_uint2(d2[0], d2[1]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
  if ((threadIdx.x & 31) == 0) atomicAdd(&s_sum, static_cast<unsigned long long>(sum));
  __syncthreads();
  if (threadIdx.x == 0) {
    corr[t] = 128ll * static_cast<long long>(s_sum);
    shift[t] = t >= M || E == 0 ? kZeroRow : (E == 255 ? kBadRow : E - 148);
  }
}

// The CTA whose share holds unit u: the largest c with floor(c U / G) <= u.
__device__ __forceinline__ int owner(int64_t u, int64_t units, int grid) {
  const int c = static_cast<int>(((u + 1) * grid + units - 1) / units) - 1;
  return c < grid - 1 ? c : grid - 1;
}

__device__ __forceinline__ int64_t share_begin(int c, int64_t units, int grid) { return c * units / grid; }

template <bool kF32Out, int MT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_i8_skinny(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_p,
                   const float* __restrict__ scales, const uint16_t* __restrict__ bias, void* __restrict__ y_out,
                   int M, int N, int k_tiles, int n_tiles, const int* __restrict__ shift,
                   const long long* __restrict__ corr, long long* __restrict__ partials,
                   uint32_t* __restrict__ counters, int* err) {
  constexpr int kRows = 3 * MT;                // the MMA's N: three digit planes of MT tokens
  constexpr int kPlaneBox = kRows * 128;
  extern __shared__ uint8_t smem_raw[];
  Smem<MT>& s = *reinterpret_cast<Smem<MT>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grid = static_cast<int>(gridDim.x);
  const int64_t units = static_cast<int64_t>(n_tiles) * k_tiles;
  const int64_t u0 = share_begin(blockIdx.x, units, grid), u1 = share_begin(blockIdx.x + 1, units, grid);
  volatile int* abort = &s.abort;

  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.acc_full[i], 1);
      mbar_init(&s.acc_empty[i], kEpiWarps);
    }
    mbar_init(&s.drain, 1);
    s.abort = 0;
    fence_mbar_init();
    prefetch_tensormap(&tm_w);
    prefetch_tensormap(&tm_p);
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
      const int pre = static_cast<int>(u1 - u0 < kStages ? u1 - u0 : kStages);
      auto unit_of = [&](int64_t u, int& t, int& kt) {
        t = static_cast<int>(u / k_tiles);
        kt = static_cast<int>(u - static_cast<int64_t>(t) * k_tiles);
      };
      // the first units' codes do not depend on the kernels ahead: requested before waiting for them
      for (int i = 0; i < pre; ++i) {
        int t, kt;
        unit_of(u0 + i, t, kt);
        mbar_arrive_expect_tx(&s.full[i], kCodeBytes + 2 * kPlaneBox);
        tma_load_2d(s.w[i], &tm_w, &s.full[i], kt * BKU, t * BN);
        tma_load_2d(s.w[i] + kBoxBytes, &tm_w, &s.full[i], kt * BKU + 128, t * BN);
      }
      pdl_wait();  // the planes are the kernel ahead's output
      uint32_t issued = 0, last_parity = 0;
      for (int i = 0; i < pre; ++i) {
        int t, kt;
        unit_of(u0 + i, t, kt);
        tma_load_2d(s.p[i][0], &tm_p, &s.full[i], kt * BKU, 0);
        tma_load_2d(s.p[i][1], &tm_p, &s.full[i], kt * BKU + 128, 0);
        issued |= 1u << i;
      }
      int stage = pre % kStages;
      uint32_t phase = pre == kStages ? 1u : 0u;
      for (int64_t u = u0 + pre; u < u1 && !*abort; ++u) {
        if (!mbar_wait(&s.empty[stage], phase ^ 1u, abort, err, kSiteProducerEmpty)) break;
        int t, kt;
        unit_of(u, t, kt);
        mbar_arrive_expect_tx(&s.full[stage], kCodeBytes + 2 * kPlaneBox);
        tma_load_2d(s.w[stage], &tm_w, &s.full[stage], kt * BKU, t * BN);
        tma_load_2d(s.w[stage] + kBoxBytes, &tm_w, &s.full[stage], kt * BKU + 128, t * BN);
        tma_load_2d(s.p[stage][0], &tm_p, &s.full[stage], kt * BKU, 0);
        tma_load_2d(s.p[stage][1], &tm_p, &s.full[stage], kt * BKU + 128, 0);
        issued |= 1u << stage;
        last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      for (int st = 0; st < kStages; ++st)
        if (issued & (1u << st)) mbar_wait_drain(&s.full[st], (last_parity >> st) & 1u);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_u8s8(BN, kRows);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int64_t u = u0; u < u1 && ok;) {
        const int t = static_cast<int>(u / k_tiles);
        const int64_t seg_end = u1 < static_cast<int64_t>(t + 1) * k_tiles ? u1 : static_cast<int64_t>(t + 1) * k_tiles;
        if (!mbar_wait(&s.acc_empty[acc], acc_phase ^ 1u, abort, err, kSiteMmaAccum)) break;
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(acc * 128);
        for (int64_t v = u; v < seg_end; ++v) {
          if (!mbar_wait(&s.full[stage], phase, abort, err, kSiteMmaInput)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int b = 0; b < 2; ++b) {
            const uint32_t a0 = smem_u32(s.w[stage] + b * kBoxBytes), b0 = smem_u32(s.p[stage][b]);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)  // K 32 a step: 32 bytes inside the swizzle atom
              tc_mma_i8(d, umma_desc_sw128(a0 + kk * 32), umma_desc_sw128(b0 + kk * 32), idesc,
                        (v != u || b != 0 || kk != 0) ? 1u : 0u);
          }
          tc_commit(&s.empty[stage]);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
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
    // ---------------- segment epilogue: y, or an integer partial and the tile's fix-up ----------------
    pdl_wait();  // the shifts and corrections are the kernel ahead's output
    const int ew = warp - kEpiWarp0;  // TMEM lanes [32 ew, 32 ew + 32): output columns of the tile
    const int row = ew * 32 + lane;
    // staged while the main loop runs: the y step then reads them from shared memory, not in a chain of loads
    if (row < MT) {
      s.shift[row] = shift[row];
      s.corr[row] = corr[row];
    }
    named_barrier_sync(1, kEpiWarps * 32);
    int acc = 0, seg = 0;
    uint32_t acc_phase = 0;
    for (int64_t u = u0; u < u1; ++seg) {
      const int t = static_cast<int>(u / k_tiles);
      const int64_t tile_end = static_cast<int64_t>(t + 1) * k_tiles;
      const int64_t seg_end = u1 < tile_end ? u1 : tile_end;
      const bool whole = u == static_cast<int64_t>(t) * k_tiles && seg_end == tile_end;
      // this segment's column: scale and bias requested before the wait for its sums
      const int n = t * BN + row;
      const float sc = n < N ? scales[n] : 0.0f;
      const float b = (n < N && bias != nullptr) ? __uint_as_float(static_cast<uint32_t>(bias[n]) << 16) : 0.0f;
      int got = 0;
      if (lane == 0) got = mbar_wait(&s.acc_full[acc], acc_phase, abort, err, kSiteEpilogueFull) ? 1 : 0;
      got = __shfl_sync(0xFFFFFFFFu, got, 0);
      long long v[MT];
#pragma unroll
      for (int i = 0; i < MT; ++i) v[i] = 0;
      if (got) {
        tc_fence_after();
        const uint32_t base = tmem + (static_cast<uint32_t>(ew * 32) << 16) + static_cast<uint32_t>(acc * 128);
#pragma unroll
        for (int c = 0; c < (kRows + 31) / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32(base + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int col = c * 32 + j;
            if (col < kRows) {
              const int d = col / MT, tok = col % MT;
              v[tok] += static_cast<long long>(static_cast<int>(r[j])) << (8 * d);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.acc_empty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
      bool store = whole;
      if (!whole) {
        const int slot = seg == 0 ? 0 : 1;
        long long* mine = partials + ((static_cast<int64_t>(blockIdx.x) * kSlots + slot) * BN + row) * kTokens;
#pragma unroll
        for (int i = 0; i < MT; i += 2)
          *reinterpret_cast<longlong2*>(mine + i) = make_longlong2(v[i], v[i + 1]);
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
#pragma unroll
          for (int i = 0; i < MT; ++i) v[i] = 0;
          // integer sums: exact in any order; plain L2 loads (after the fence above) that the compiler may
          // issue ahead of the adds, so the CTAs' partials arrive together rather than one round trip each
#pragma unroll 2
          for (int c = c_first; c <= c_last; ++c) {
            const int cslot = t == static_cast<int>(share_begin(c, units, grid) / k_tiles) ? 0 : 1;
            const longlong2* f = reinterpret_cast<const longlong2*>(
                partials + ((static_cast<int64_t>(c) * kSlots + cslot) * BN + row) * kTokens);
            longlong2 x[MT / 2];
#pragma unroll
            for (int i = 0; i < MT / 2; ++i) x[i] = __ldcg(f + i);
#pragma unroll
            for (int i = 0; i < MT / 2; ++i) {
              v[2 * i] += x[i].x;
              v[2 * i + 1] += x[i].y;
            }
          }
        }
      }
      if (store && n < N) {
#pragma unroll
        for (int i = 0; i < MT; ++i)
          if (i < M) {
            const int sh = s.shift[i];
            float sum;
            if (sh == kZeroRow) sum = 0.0f;
            else if (sh == kBadRow) sum = __uint_as_float(0x7FC00000u);
            // times 2^sh (sh in [-147, 106]) as a product with that power of two, exact in double; the
            // conversion to fp32 is the one rounding
            else sum = __double2float_rn(static_cast<double>(v[i] - s.corr[i]) *
                                         __longlong_as_double(static_cast<long long>(sh + 1023) << 52));
            const float o = __fadd_rn(__fmul_rn(sum, sc), b);
            if (kF32Out) static_cast<float*>(y_out)[static_cast<int64_t>(i) * N + n] = o;
            else static_cast<uint16_t*>(y_out)[static_cast<int64_t>(i) * N + n] = f32_to_bf16_rne(o);
          }
      }
      u = seg_end;
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

template <bool kF32Out, int MT>
cudaError_t launch_mt(const CUtensorMap& tm_p, const sc_weight* w, const uint16_t* bias, void* y, int64_t m,
                      const int* shift, const long long* corr, long long* partials, uint32_t* counters, int grid,
                      int* err, cudaStream_t stream) {
  auto kernel = gemm_i8_skinny<kF32Out, MT>;
  static unsigned long long configured = 0;  // per template instance and device
  if (cudaError_t e = set_smem_once(kernel, static_cast<int>(smem_bytes<MT>()), configured); e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem_bytes<MT>();
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, w->tmap_values_wide, tm_p, static_cast<const float*>(w->scales), bias, y,
                            static_cast<int>(m), static_cast<int>(w->n), static_cast<int>((w->k_pad + BKU - 1) / BKU),
                            static_cast<int>(w->n_pad / BN), shift, corr, partials, counters, err);
}

}  // namespace skinny_i8

// CTAs of the int8 skinny product for this weight and m (0 when it does not apply: not int8, m beyond 16
// rows, K beyond the s32 accumulators' exact range, fewer units than two per SM, too many tiles to count).
int skinny_i8_grid(const sc_weight* w, int64_t m, int sm_count) {
  using namespace skinny_i8;
  if (w->kind != SC_WEIGHT_INT8 || m > kSkinnyI8MaxRows || w->k_pad > 65536) return 0;
  const int64_t k_tiles = (w->k_pad + BKU - 1) / BKU, n_tiles = w->n_pad / BN, units = k_tiles * n_tiles;
  if (n_tiles > kSkinnyCounterWords || units < 2 * static_cast<int64_t>(sm_count)) return 0;
  return sm_count;
}

// Workspace: the planes [3 MT][k_pad] int8, the rows' shifts and corrections, the CTAs' partial slots.
size_t skinny_i8_workspace_bytes(const sc_weight* w, int64_t m, int grid) {
  using namespace skinny_i8;
  (void)m;
  const size_t planes = (static_cast<size_t>(3 * kTokens) * w->k_pad + 255) / 256 * 256;
  return planes + 1024 + static_cast<size_t>(grid) * kSlots * BN * kTokens * sizeof(long long);
}

cudaError_t launch_gemm_skinny_i8(sc_encode_tiled_fn encode, const uint16_t* x, const sc_weight* w,
                                  const uint16_t* bias, void* y, bool f32_out, int64_t m, void* workspace,
                                  uint32_t* counters, int grid, int* err, cudaStream_t stream) {
  using namespace skinny_i8;
  constexpr int mt = kTokens;
  const size_t planes_bytes = (static_cast<size_t>(3 * mt) * w->k_pad + 255) / 256 * 256;
  int8_t* planes = static_cast<int8_t*>(workspace);
  int* shift = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + planes_bytes);
  long long* corr = reinterpret_cast<long long*>(static_cast<uint8_t*>(workspace) + planes_bytes + 256);
  long long* partials = reinterpret_cast<long long*>(static_cast<uint8_t*>(workspace) + planes_bytes + 1024);
  // the planes as the MMA's B operand: rows of k_pad bytes, boxes of 128 bytes x 3 MT rows, swizzled
  CUtensorMap tm_p;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(w->k_pad), static_cast<cuuint64_t>(3 * mt)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(w->k_pad)};
  const cuuint32_t box[2] = {128, static_cast<cuuint32_t>(3 * mt)};
  const cuuint32_t estr[2] = {1, 1};
  if (encode(&tm_p, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, planes, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
      CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(mt), 1, 1);
    cfg.blockDim = dim3(kPlaneThreads, 1, 1);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaError_t e = cudaLaunchKernelEx(&cfg, x_planes, x, static_cast<int>(m), static_cast<int>(w->k),
                                           static_cast<int>(w->k_pad), mt, planes, shift, corr);
        e != cudaSuccess)
      return e;
  }
  return f32_out ? launch_mt<true, kTokens>(tm_p, w, bias, y, m, shift, corr, partials, counters, grid, err, stream)
                 : launch_mt<false, kTokens>(tm_p, w, bias, y, m, shift, corr, partials, counters, grid, err, stream);
}

}  // namespace sc
