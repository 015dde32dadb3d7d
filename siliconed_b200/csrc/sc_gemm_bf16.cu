// The large-M product in two launches: the weight's codes widened once to bf16 in the caller's
// workspace, then a CTA-pair tcgen05 GEMM whose two operands both arrive by TMA.
//
// In the fused pair kernel (sc_gemm_pair.cu) every CTA pair converts the codes of its weight
// columns for every K stage of every output tile: each code is converted once per 256-row block of
// x, and the conversion sits in the pipeline between the code tile's arrival and the MMA.  For
// large M that costs more than it saves: widening the whole weight once reads K*N bytes and writes
// 2*K*N (a few microseconds of HBM time), after which the GEMM streams both operands with TMA and
// nothing but the tensor cores works between a stage's arrival and its MMA.  The widened values are
// exact (every int8 and e4m3 value is a bf16), the scale and bias are applied in the epilogue after
// the fp32 sum as in the fused kernel, and the MMAs see the same operands in the same order, so the
// two routes give the same bits.
//
// GEMM layout: a cluster of two CTAs owns output tiles of 256 x 256.  Each CTA loads its own 128
// rows of x and 128 of the 256 weight columns (bf16, 128-byte swizzled) into a 6-stage ring; the
// loads use the pair form of the tensor-map copy, so both CTAs' bytes are counted on the leader's
// barrier, and the leader issues tcgen05.mma.cta_group::2 (M = 256, N = 256) into the fp32
// accumulators of both CTAs' TMEM (two buffers of 256 columns: the epilogue of one tile overlaps
// the MMAs of the next).  Warp 0: TMA producer; warp 1: TMEM allocation and (leader) MMA issue;
// warps 4..7: epilogue; warps 2..7 also widen codes in the kFW variant.  No load uses cluster
// multicast; every wait is bounded.
//
// Variants (template parameters): fp32 or bf16 output; the epilogue's operation (kOp: none, GELU, gated
// residual, QK-norm + RoPE into the attention's layout, SwiGLU); the column-parallel gather's peer or
// multicast stores (kPeers); int8 x int8 operands for W8A8 (kI8); the widening inside the kernel (kFW).
// At run time the operand x can also be the attention's output read through a 4-D tensor map (XHeads).
#include <cuda_bf16.h>

#include "sc_codes.cuh"
#include "sc_internal.h"
#include "sc_ptx.cuh"

namespace sc {
namespace gemm_bf16 {

constexpr int BM = 128;      // rows of x per CTA (256 per pair)
constexpr int BN = 256;      // output columns per pair tile
constexpr int BNH = BN / 2;  // weight columns each CTA loads
constexpr int BK = 64;
constexpr int kStages = 6;
constexpr int kABytes = BM * BK * 2;
constexpr int kBBytes = BNH * BK * 2;
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kEpiWarp0 = 4, kEpiWarps = 4;
constexpr uint32_t kTmemCols = 512;

struct __align__(1024) Smem {
  uint8_t a[kStages][kABytes];  // x tiles
  uint8_t b[kStages][kBBytes];  // widened weight half-tiles
  float sb[kEpiWarps][2][BN];   // per epilogue warp: the tile's scales and biases
  float sb2[kEpiWarps][BN];      // kOpResidual: per epilogue warp, the tile's gates
  uint4 stage[kEpiWarps][32 * 8];  // kPeers: per epilogue warp, 32 rows x 64 bf16 (16-byte units, swizzled)
  uint64_t full[kStages];       // leader: both CTAs' operands of the stage landed
  uint64_t empty[kStages];      // the pair's MMAs of the stage completed (leader's commit)
  uint64_t acc_full[2];
  uint64_t acc_empty[2];        // leader: both CTAs' epilogues
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

constexpr size_t kSmemBytes = sizeof(Smem) + 1024;

// kPeers: the fused column-parallel gather.  Each bf16 output tile goes to the output of every rank
// (peers.y[r], rows of peers.ld elements, columns peers.col0 + j) with plain stores over NVLink; after
// its last tile every CTA fences at system scope and counts itself on peers.counter, and the last CTA
// raises peers.flags[r][peers.rank] = peers.epoch on every rank r (release, system scope).
//
// kOp: the epilogue's operation after v = acc * scale + bias (fp32).  kOpNone stores v; kOpGelu stores
// bf16(gelu_tanh(v)) (one rounding, where a separate pass would round v first); kOpResidual adds
// gate[n] * v to the fp32 output in place, x = x + gate * v in two roundings (the gated residual stream).
// kOpQkRope: the q / k / v product of a DiT block; each 128-column half of a tile is one head of q, k or
// v.  For q and k the head is RMS-normalised over its 128 values (sum of squares from a first pass over
// the accumulator, inv = 1 / sqrt(ss / 128 + eps), then * inv * norm[d]) and rotated by RoPE on adjacent
// pairs, (e0 c - e1 s, e0 s + e1 c) with (c, s) = freqs[pos][d / 2]; v is stored as it is.  Every head
// goes to its [batch, heads, joint, 128] row: the attention's layout, written once.
// kOpSwiglu: the gate / up product of a SwiGLU MLP whose weight columns come in blocks of 128, gate block j
// then up block j (each 256-column tile holds one pair); the epilogue stores bf16(silu(a) * b) for the
// tile's 128 outputs, silu(a) = a / (1 + exp(-a)), into y [M, N / 2] at columns n0 / 2 ...
constexpr int kOpNone = 0, kOpGelu = 1, kOpResidual = 2, kOpQkRope = 3, kOpSwiglu = 4;

// gelu_tanh(v) = 0.5 v (1 + tanh(u)), u = sqrt(2 / pi) (v + 0.044715 v^3), through the identity
// 0.5 (1 + tanh(u)) = 1 / (1 + exp(-2u)): one exponential and one approximate division, about 2e-6
// relative error before the bf16 rounding.  exp overflows to +inf for v below about -11: v / inf = -0.
__device__ __forceinline__ float gelu_tanh(float v) {
  const float e = __expf(-1.5957691216057308f * fmaf(0.044715f * v, v * v, v));
  return __fdividef(v, 1.0f + e);
}

// The value of one accumulator element before the epilogue's operation.  bf16 operands: acc * s + b,
// two roundings.  kI8 (W8A8, the int8 x int8 product of TensorGEMMInt8.swift): float(acc) * (s_x * s_w),
// the scales' product first (scale_products, :155-160), then + bias only when there is one (a
// missing bias adds nothing, not +0, which would turn -0 into +0).
template <bool kI8>
__device__ __forceinline__ float epi_value(uint32_t raw, float sc, float bi, float sxr, bool has_bias) {
  if (kI8) {
    const float v = __fmul_rn(__int2float_rn(static_cast<int>(raw)), __fmul_rn(sxr, sc));
    return has_bias ? __fadd_rn(v, bi) : v;
  }
  return __fadd_rn(__fmul_rn(__uint_as_float(raw), sc), bi);
}

// Narrow pieces.  When a product's 256 x 256 tiles would leave most pairs idle and their epilogues carry the
// work that bounds it (the column-parallel gather at 8 GPUs: a rank's 4096 x 384 columns are 24 tiles for 74
// pairs, and each tile is stored to every rank), the output is cut into pieces of 256 rows x `width` columns,
// `per_row` of them per row tile, one per pair, so that more SMs share the stores.  A piece is one pair MMA of
// N = width over the full K: every output is the same sum in the same K order, the same bits as in the whole
// tile.  The weight's box stays 128 rows a CTA (the rows past the piece are loaded and not used).  width 0:
// tiles.
struct Pieces {
  int width;
  int per_row;
  int count;
};

// The work of the pair at `tile` (tile = pair + j pairs): its row tile, first column and width (false when
// the pair has no more work).  Only the gathering kernels (kPieces) take pieces.
template <bool kPieces>
__device__ __forceinline__ bool job_of(int tile, int num_tiles, int m_tiles, int n_tiles, const Pieces& pc, int& mt,
                                       int& n0, int& w) {
  if (!kPieces || pc.width == 0) {
    if (tile >= num_tiles) return false;
    int nt;
    tile_coords(tile, m_tiles, n_tiles, mt, nt);
    n0 = nt * BN;
    w = BN;
    return true;
  }
  if (tile >= pc.count) return false;
  mt = tile / pc.per_row;
  n0 = (tile % pc.per_row) * pc.width;
  w = pc.width;
  return true;
}

// kI8: both operands int8 codes (x's per-row codes, the weight's codes made signed), 128 codes = 128
// bytes per K stage, tcgen05.mma kind::i8 into s32 accumulators; row_scales holds s_x per row.
// kFW (fused widening, 1 int8 / 2 e4m3 / 3 e4m3 with NaN codes): the CTAs widen the codes themselves.
// Every thread first widens the column blocks the first round of tiles reads; then warps 2-7 widen the
// rest, block by block, while the pipeline runs (warps 2 and 3 are otherwise idle, and the epilogue warps
// have nothing to do until the first accumulator is ready).  After its share of a block, a CTA counts
// itself on the block's counter; a producer waits for all CTAs on the block of its tile before the
// tile's first load (acquire, then a proxy fence: the data was written by ordinary stores).
template <bool kF32Out, bool kPeers, int kOp, bool kI8, int kFW = 0>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_pair(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                   const float* __restrict__ scales, const uint16_t* __restrict__ bias, void* __restrict__ y_out,
                   int M, int N, int k_tiles, int m_tiles, int n_tiles, int* err,
                   const __grid_constant__ PeerOut peers, const float* __restrict__ gate,
                   const float* __restrict__ row_scales, const __grid_constant__ HeadOut ho, const XHeads xh,
                   const __grid_constant__ FusedWiden fw, const Pieces pc) {
  static_assert(kOp != kOpResidual || kF32Out, "the residual is fp32");
  static_assert(kOp != kOpGelu || !kF32Out, "the GELU output is bf16");
  static_assert(!kI8 || (kOp == kOpNone && !kPeers), "W8A8 stores plain outputs");
  constexpr int kBKElems = kI8 ? 128 : BK;  // K elements per 128-byte stage row
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
      mbar_init(&s.full[i], 1);   // the leader producer's arrive; the bytes of both CTAs
      mbar_init(&s.empty[i], 1);  // the leader's commit
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
  // Launched early behind the widening (or the int8 passes) of the same product, the set-up above
  // overlapped their end; nothing reads or writes global memory before this point.
  pdl_wait();
  if (kFW != 0) {
    // every thread of the grid: the first round's column blocks
    const int64_t n0 = static_cast<int64_t>(fw.first_blocks) * fw.chunks_per_block;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
    for (int64_t base = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; base < n0; base += 4 * stride) {
      uint4 in[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t i = base + u * stride;
        in[u] = i < n0 ? __ldcs(fw.codes + i) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t i = base + u * stride;
        if (i < n0) {
          uint4 lo, hi;
          codes16_to_bf16<kFW == 1 ? 1 : 2, kFW == 3>(in[u], lo, hi);
          st_global_32b(fw.out + 2 * i, lo, hi);
        }
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      for (int b = 0; b < fw.first_blocks; ++b) atomicAdd(fw.counters + b, 1u);
    }
  }

  if (warp == 0) {
    // ---------------- TMA producer (each CTA loads its own halves) ----------------
    if (lane == 0) {
      int stage = 0, ready_block = -1;
      uint32_t phase = 0, issued = 0, last_parity = 0;
      for (int tile = pair; !*abort; tile += pairs) {
        int mt, n0, wd;
        if (!job_of<kPeers>(tile, num_tiles, m_tiles, n_tiles, pc, mt, n0, wd)) break;
        const int row0 = mt * 2 * BM + static_cast<int>(rank) * BM;
        const int col0 = n0 + static_cast<int>(rank) * (wd / 2);
        const int nt = n0 / BN;  // kFW products have no pieces: the job is the tile of column block nt
        if (kFW != 0 && nt != ready_block) {
          // the tile's column block widened by every CTA (bounded wait)
          const unsigned long long t0 = global_ns();
          while (ld_acquire_gpu(fw.counters + nt) < gridDim.x) {
            if (global_ns() - t0 > kWaitLimitNs) {
              record_error(err, kErrTimeout, kSiteWidened);
              *abort = 1;
              break;
            }
          }
          fence_proxy_async_global();
          ready_block = nt;
        }
        for (int kt = 0; kt < k_tiles; ++kt) {
          if (!mbar_wait(&s.empty[stage], phase ^ 1u, abort, err, kSiteProducerEmpty)) break;
          if (leader) mbar_arrive_expect_tx(&s.full[stage], 2 * (kABytes + kBBytes));
          const uint32_t bar = peer_addr(&s.full[stage], 0);
          if (xh.tokens > 0)  // 64 values of head kt / 2 for 128 tokens of one image (row0 % 128 == 0)
            tma_load_4d_pair(s.a[stage], &tm_x, bar, (kt & 1) * 64, xh.offset + row0 % xh.tokens, kt >> 1,
                             row0 / xh.tokens);
          else
            tma_load_2d_pair(s.a[stage], &tm_x, bar, kt * kBKElems, row0);
          tma_load_2d_pair(s.b[stage], &tm_w, bar, kt * kBKElems, col0);
          issued |= 1u << stage;
          last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // The leader drains its own barriers; the peer's loads complete on the leader's barriers,
      // which the leader's MMA has waited on before the pair's last commit.
      if (leader)
        for (int st = 0; st < kStages; ++st)
          if (issued & (1u << st)) mbar_wait_drain(&s.full[st], (last_parity >> st) & 1u);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader CTA) ----------------
    if (leader && lane == 0) {
      const uint32_t idesc_full = kI8 ? umma_idesc_s8(2 * BM, BN) : umma_idesc_bf16(2 * BM, BN);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int tile = pair; ok; tile += pairs) {
        int mt_, n0_, wd;
        if (!job_of<kPeers>(tile, num_tiles, m_tiles, n_tiles, pc, mt_, n0_, wd)) break;
        const uint32_t idesc = !kPeers || wd == BN ? idesc_full : umma_idesc_bf16(2 * BM, wd);
        if (!mbar_wait(&s.acc_empty[acc], acc_phase ^ 1u, abort, err, kSiteMmaAccum)) break;
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(acc * BN);
        bool ready = mbar_test_wait(&s.full[stage], phase);
        for (int kt = 0; kt < k_tiles; ++kt) {
          if (!ready && !mbar_poll(&s.full[stage], phase, abort, err, kSiteMmaInput)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int cur = stage;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
          ready = kt + 1 < k_tiles && mbar_test_wait(&s.full[stage], phase);
          const uint32_t a0 = smem_u32(s.a[cur]), b0 = smem_u32(s.b[cur]);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            if (kI8)
              tc_mma_i8_pair(d, umma_desc_sw128(a0 + kk * 32), umma_desc_sw128(b0 + kk * 32), idesc,
                             (kt | kk) != 0 ? 1u : 0u);
            else
              tc_mma_f16_pair(d, umma_desc_sw128(a0 + kk * 32), umma_desc_sw128(b0 + kk * 32), idesc,
                              (kt | kk) != 0 ? 1u : 0u);
          tc_commit_pair_both(&s.empty[cur], 0x3);
        }
        if (!ok) break;
        tc_commit_pair_both(&s.acc_full[acc], 0x3);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      tc_commit_pair(peer_addr(&s.drain, 0));
      mbar_wait_drain(&s.drain, 0);
    }
  }
  if (kFW != 0 && warp >= 2) {
    // the remaining column blocks, each CTA its slice of every block, in block order
    const int t = threadIdx.x - 64, nt_threads = kThreads - 64;
    // (no early exit: every warp of 2..7 must reach each block's named barrier)
    for (int b = fw.first_blocks; b < fw.n_blocks; ++b) {
      const int64_t c0 = static_cast<int64_t>(b) * fw.chunks_per_block +
                         static_cast<int64_t>(blockIdx.x) * fw.chunks_per_block / gridDim.x;
      const int64_t c1 = static_cast<int64_t>(b) * fw.chunks_per_block +
                         static_cast<int64_t>(blockIdx.x + 1) * fw.chunks_per_block / gridDim.x;
      for (int64_t base = c0 + t; base < c1; base += 2 * nt_threads) {
        const int64_t i1 = base + nt_threads;
        const uint4 in0 = __ldcs(fw.codes + base);
        const uint4 in1 = i1 < c1 ? __ldcs(fw.codes + i1) : make_uint4(0, 0, 0, 0);
        uint4 lo, hi;
        codes16_to_bf16<kFW == 1 ? 1 : 2, kFW == 3>(in0, lo, hi);
        st_global_32b(fw.out + 2 * base, lo, hi);
        if (i1 < c1) {
          codes16_to_bf16<kFW == 1 ? 1 : 2, kFW == 3>(in1, lo, hi);
          st_global_32b(fw.out + 2 * i1, lo, hi);
        }
      }
      named_barrier_sync(2, kThreads - 64);
      if (t == 0) {
        __threadfence();
        atomicAdd(fw.counters + b, 1u);
      }
    }
  }
  if (warp >= kEpiWarp0 && warp < kEpiWarp0 + kEpiWarps) {
    // ---------------- epilogue (each CTA: its 128 rows x 256 columns) ----------------
    const int ew = warp - kEpiWarp0;
    float* s_scale = s.sb[ew][0];
    float* s_bias = s.sb[ew][1];
    int acc = 0;
    uint32_t acc_phase = 0;
    const bool vec_ok = (N % 8) == 0, vec4_ok = (N % 4) == 0;
    const bool has_bias = bias != nullptr;
    for (int tile = pair;; tile += pairs) {
      int mt, n0, wd;
      if (!job_of<kPeers>(tile, num_tiles, m_tiles, n_tiles, pc, mt, n0, wd)) break;
      const int row = mt * 2 * BM + static_cast<int>(rank) * BM + ew * 32 + lane;
      const float sxr = kI8 && row < M ? row_scales[row] : 0.0f;
      __syncwarp();
      for (int c = lane; c < wd; c += 32) {
        const int n = n0 + c;
        s_scale[c] = scales[n];
        s_bias[c] = (bias != nullptr && n < N) ? __uint_as_float(static_cast<uint32_t>(bias[n]) << 16) : 0.0f;
        if (kOp == kOpResidual) s.sb2[ew][c] = n < N ? gate[n] : 0.0f;
      }
      __syncwarp();
      // Stores leave through the warp's staging buffer: each lane holds one row of a 32-column chunk
      // (its TMEM lane), the chunk is written to shared memory (16-byte units, XOR-swizzled by row)
      // and read back so that 8 lanes cover 128 contiguous bytes of one row: 4 rows per store
      // instruction instead of 32, which the L2 and the memory controllers take far better.
      // kOpResidual reads the residual tile the same way, one chunk ahead of its use (the first
      // chunk before the accumulator is ready): one load round trip per tile is exposed, not one
      // per chunk.  The staged paths need 16-byte aligned rows (N % 8 == 0 for bf16, N % 4 == 0 for
      // fp32); other shapes store one row per lane.
      const int row0 = mt * 2 * BM + static_cast<int>(rank) * BM + ew * 32;
      uint4* st = s.stage[ew];
      float* xres = kOp == kOpResidual ? static_cast<float*>(y_out) : nullptr;
      const bool res_fast = kOp == kOpResidual && vec4_ok && n0 + BN <= N;
      float4 xcur[8];
      if (kOp == kOpResidual && res_fast) {
#pragma unroll
        for (int it = 0; it < 8; ++it) {
          const int grow = row0 + ((it * 32 + lane) >> 3);
          xcur[it] = grow < M ? ld_cg_f4(xres + static_cast<int64_t>(grow) * N + n0 + (lane & 7) * 4)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      int ready = 0;
      if (lane == 0) ready = mbar_wait(&s.acc_full[acc], acc_phase, abort, err, kSiteEpilogueFull) ? 1 : 0;
      if (!__shfl_sync(0xFFFFFFFFu, ready, 0)) break;
      tc_fence_after();
      const uint32_t tbase = tmem + (static_cast<uint32_t>(ew * 32) << 16) + static_cast<uint32_t>(acc * BN);
      if (kOp == kOpQkRope) {
        const int hd = ho.heads * 128;
#pragma unroll 1
        for (int hh = 0; hh < BN / 128; ++hh) {
          const int cb = n0 + hh * 128;
          if (cb >= N) break;
          const int which = cb / hd, head = (cb % hd) / 128;
          const uint32_t tb = tbase + hh * 128;
          float inv = 1.0f;
          if (which < 2) {
            float ss = 0.0f;
#pragma unroll 1
            for (int ch = 0; ch < 4; ++ch) {
              uint32_t r[32];
              tmem_ld_32(tb + ch * 32, r);
              tmem_wait_ld();
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const float v = epi_value<false>(r[j], s_scale[hh * 128 + ch * 32 + j], s_bias[hh * 128 + ch * 32 + j],
                                                 0.0f, true);
                ss = __fmaf_rn(v, v, ss);
              }
            }
            inv = 1.0f / sqrtf(ss / 128.0f + ho.eps);
          }
          const float* wn = which == 0 ? ho.norm_q : ho.norm_k;
          const int tok = row % ho.tokens;
          const float* fr = ho.freqs + static_cast<int64_t>(ho.offset + tok) * 128;
          uint16_t* out = which == 0 ? ho.q : (which == 1 ? ho.k : ho.v);
#pragma unroll 1
          for (int ch = 0; ch < 4; ++ch) {
            uint32_t r[32];
            tmem_ld_32(tb + ch * 32, r);
            tmem_wait_ld();
            uint32_t packed[16];
            const bool rope = which < 2 && row < M;
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
              const int d = ch * 32 + j;
              // two pairs per step: 16-byte loads of the norm weights (the same for the warp) and of the
              // row's (cos, sin) pairs
              const float4 wv = rope ? *reinterpret_cast<const float4*>(wn + d) : make_float4(1.f, 1.f, 1.f, 1.f);
              const float4 fv = rope ? *reinterpret_cast<const float4*>(fr + d) : make_float4(1.f, 0.f, 1.f, 0.f);
              float e[4];
#pragma unroll
              for (int i = 0; i < 4; ++i)
                e[i] = epi_value<false>(r[j + i], s_scale[hh * 128 + d + i], s_bias[hh * 128 + d + i], 0.0f, true);
              if (rope) {
                const float a0 = e[0] * inv * wv.x, a1 = e[1] * inv * wv.y;
                const float a2 = e[2] * inv * wv.z, a3 = e[3] * inv * wv.w;
                e[0] = a0 * fv.x - a1 * fv.y;
                e[1] = a0 * fv.y + a1 * fv.x;
                e[2] = a2 * fv.z - a3 * fv.w;
                e[3] = a2 * fv.w + a3 * fv.z;
              }
              const __nv_bfloat162 h0 = __floats2bfloat162_rn(e[0], e[1]), h1 = __floats2bfloat162_rn(e[2], e[3]);
              packed[j / 2] = *reinterpret_cast<const uint32_t*>(&h0);
              packed[j / 2 + 1] = *reinterpret_cast<const uint32_t*>(&h1);
            }
            // two chunks (64 values of the head) per flush: 8 lanes write 128 contiguous bytes of a row
#pragma unroll
            for (int q = 0; q < 4; ++q)
              st[lane * 8 + (((ch & 1) * 4 + q) ^ (lane & 7))] =
                  make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
            if (ch & 1) {
              __syncwarp();
#pragma unroll
              for (int it = 0; it < 8; ++it) {
                const int u = it * 32 + lane, rr = u >> 3, cu = u & 7;
                const int grow = row0 + rr;
                if (grow < M) {
                  const int b = grow / ho.tokens, t = grow % ho.tokens;
                  uint16_t* dst = out + ((static_cast<int64_t>(b) * ho.heads + head) * ho.joint + ho.offset + t) * 128 +
                                  (ch - 1) * 32 + cu * 8;
                  *reinterpret_cast<uint4*>(dst) = st[rr * 8 + (cu ^ (rr & 7))];
                }
              }
              __syncwarp();
            }
          }
        }
      }
      if (kOp == kOpSwiglu) {
        const int ldy = N / 2, c0 = n0 / 2;
#pragma unroll 1
        for (int ch = 0; ch < 4; ++ch) {
          uint32_t ra[32], rb[32];
          tmem_ld_32(tbase + ch * 32, ra);
          tmem_ld_32(tbase + 128 + ch * 32, rb);
          tmem_wait_ld();
          uint32_t packed[16];
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            float g[2];
#pragma unroll
            for (int i = 0; i < 2; ++i) {
              const int c = ch * 32 + j + i;
              const float a = epi_value<false>(ra[j + i], s_scale[c], s_bias[c], 0.0f, true);
              const float b = epi_value<false>(rb[j + i], s_scale[128 + c], s_bias[128 + c], 0.0f, true);
              g[i] = __fdividef(a, 1.0f + __expf(-a)) * b;
            }
            const __nv_bfloat162 h2 = __floats2bfloat162_rn(g[0], g[1]);
            packed[j / 2] = *reinterpret_cast<const uint32_t*>(&h2);
          }
#pragma unroll
          for (int q = 0; q < 4; ++q)
            st[lane * 8 + (((ch & 1) * 4 + q) ^ (lane & 7))] =
                make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
          if (ch & 1) {
            __syncwarp();
#pragma unroll
            for (int it = 0; it < 8; ++it) {
              const int u = it * 32 + lane, rr = u >> 3, cu = u & 7;
              const int grow = row0 + rr;
              if (grow < M)
                *reinterpret_cast<uint4*>(static_cast<uint16_t*>(y_out) + static_cast<int64_t>(grow) * ldy + c0 +
                                          (ch - 1) * 32 + cu * 8) = st[rr * 8 + (cu ^ (rr & 7))];
            }
            __syncwarp();
          }
        }
      }
#pragma unroll 1
      for (int ch = 0; ch < (kOp == kOpQkRope || kOp == kOpSwiglu ? 0 : wd / 32); ++ch) {
        float4 xnext[8];
        if (kOp == kOpResidual && res_fast && ch + 1 < wd / 32) {
#pragma unroll
          for (int it = 0; it < 8; ++it) {
            const int grow = row0 + ((it * 32 + lane) >> 3);
            xnext[it] = grow < M ? ld_cg_f4(xres + static_cast<int64_t>(grow) * N + n0 + (ch + 1) * 32 + (lane & 7) * 4)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
        uint32_t r[32];
        tmem_ld_32(tbase + ch * 32, r);
        tmem_wait_ld();
        const int n = n0 + ch * 32;
        if (kF32Out) {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            r[j] = __float_as_uint(epi_value<kI8>(r[j], s_scale[ch * 32 + j], s_bias[ch * 32 + j], sxr, has_bias));
          const bool staged = kOp == kOpResidual ? res_fast : vec4_ok;
          if (staged) {
            // 32 rows x 32 fp32: row `lane`'s 16-byte unit q at st[lane * 8 + (q ^ (lane & 7))]
#pragma unroll
            for (int q = 0; q < 8; ++q)
              st[lane * 8 + (q ^ (lane & 7))] = make_uint4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
            __syncwarp();
            const int cu = lane & 7, col = n + cu * 4;
#pragma unroll
            for (int it = 0; it < 8; ++it) {
              const int rr = (it * 32 + lane) >> 3, grow = row0 + rr;
              const uint4 u = st[rr * 8 + (cu ^ (rr & 7))];
              float* dst = static_cast<float*>(y_out) + static_cast<int64_t>(grow) * N + col;
              if (kOp == kOpResidual) {
                // x = x + gate * v in two roundings (torch's x + gate * y, Ops.gatedResidual): the fp32
                // residual stream, in place (the tile lies inside N)
                if (grow < M) {
                  const float* g = s.sb2[ew] + ch * 32 + cu * 4;
                  const float4 xv = xcur[it];
                  *reinterpret_cast<float4*>(dst) = make_float4(
                      __fadd_rn(xv.x, __fmul_rn(g[0], __uint_as_float(u.x))), __fadd_rn(xv.y, __fmul_rn(g[1], __uint_as_float(u.y))),
                      __fadd_rn(xv.z, __fmul_rn(g[2], __uint_as_float(u.z))), __fadd_rn(xv.w, __fmul_rn(g[3], __uint_as_float(u.w))));
                }
              } else if (grow < M) {
                if (col + 4 <= N) {
                  *reinterpret_cast<uint4*>(dst) = u;
                } else {
                  for (int k = 0; col + k < N; ++k)
                    dst[k] = __uint_as_float(k == 0 ? u.x : k == 1 ? u.y : u.z);
                }
              }
            }
            __syncwarp();
            if (kOp == kOpResidual) {
#pragma unroll
              for (int it = 0; it < 8; ++it) xcur[it] = xnext[it];
            }
          } else if (row < M) {
            float* dst = static_cast<float*>(y_out) + static_cast<int64_t>(row) * N + n;
            if (kOp == kOpResidual) {
              const float* g = s.sb2[ew] + ch * 32;
              for (int j = 0; j < 32; ++j)
                if (n + j < N) dst[j] = __fadd_rn(dst[j], __fmul_rn(g[j], __uint_as_float(r[j])));
            } else {
              for (int j = 0; j < 32; ++j)
                if (n + j < N) dst[j] = __uint_as_float(r[j]);
            }
          }
        } else {
          uint32_t packed[16];
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            float v0 = epi_value<kI8>(r[j], s_scale[ch * 32 + j], s_bias[ch * 32 + j], sxr, has_bias);
            float v1 = epi_value<kI8>(r[j + 1], s_scale[ch * 32 + j + 1], s_bias[ch * 32 + j + 1], sxr, has_bias);
            if (kOp == kOpGelu) {
              v0 = gelu_tanh(v0);
              v1 = gelu_tanh(v1);
            }
            const __nv_bfloat162 h = __floats2bfloat162_rn(v0, v1);
            packed[j / 2] = *reinterpret_cast<const uint32_t*>(&h);
          }
          if (kPeers || vec_ok) {
            // Two chunks (64 columns) of the warp's 32 rows gather in the staging buffer, then go out
            // as 128-byte row segments: to this GPU's y, or (kPeers) to every rank's output, its own
            // included, which NVLink carries far better than one 16-byte piece per row.  Peer columns
            // stay 16-byte aligned (col0, ld and the shard's width are multiples of 8, checked by the
            // host).
#pragma unroll
            for (int q = 0; q < 4; ++q)
              st[lane * 8 + (((ch & 1) * 4 + q) ^ (lane & 7))] =
                  make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
            if (ch & 1) {
              __syncwarp();
              const int c0 = n0 + (ch - 1) * 32;
#pragma unroll
              for (int it = 0; it < 8; ++it) {
                const int u = it * 32 + lane, rr = u >> 3, cu = u & 7;
                const int grow = row0 + rr, col = c0 + cu * 8;
                if (grow >= M || col >= N) continue;
                const uint4 v = st[rr * 8 + (cu ^ (rr & 7))];
                if (kPeers) {
                  const int64_t off = static_cast<int64_t>(grow) * peers.ld + peers.col0 + col;
                  if (col + 8 <= N) {
                    if (peers.y_mc != nullptr)
                      multimem_st_v4(static_cast<uint16_t*>(peers.y_mc) + off, v);
                    else
                      for (int r = 0; r < peers.world; ++r) *reinterpret_cast<uint4*>(static_cast<uint16_t*>(peers.y[r]) + off) = v;
                  }
                } else {
                  uint16_t* dst = static_cast<uint16_t*>(y_out) + static_cast<int64_t>(grow) * N + col;
                  if (col + 8 <= N) {
                    *reinterpret_cast<uint4*>(dst) = v;
                  } else {
                    for (int k = 0; col + k < N; ++k) {
                      const uint32_t word = k < 2 ? v.x : k < 4 ? v.y : k < 6 ? v.z : v.w;
                      dst[k] = static_cast<uint16_t>(word >> (16 * (k & 1)));
                    }
                  }
                }
              }
              __syncwarp();
            }
          } else if (row < M) {
            uint16_t* dst = static_cast<uint16_t*>(y_out) + static_cast<int64_t>(row) * N + n;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (n + j < N) dst[j] = static_cast<uint16_t>(packed[j / 2] >> (16 * (j & 1)));
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(peer_addr(&s.acc_empty[acc], 0));
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
    if (kPeers) {
      // The CTA's stores to every rank are done (all four epilogue warps meet here, on every path),
      // then one thread fences them at system scope and counts the CTA; the last CTA signals.
      named_barrier_sync(1, kEpiWarps * 32);
      if (ew == 0 && lane == 0) {
        __threadfence_system();
        const int old = atomicAdd(peers.counter, 1);
        if (old == static_cast<int>(gridDim.x) - 1) {
          atomicExch(peers.counter, 0);
          __threadfence_system();
          for (int r = 0; r < peers.world; ++r) st_release_sys(peers.flags[r] + peers.rank, peers.epoch);
        }
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
  if (kFW != 0 && threadIdx.x == 0) {
    // Every role of this CTA is done, its producer past its last wait on the counters.  The CTA counts its
    // exit; the last one to leave returns the counters to zero, so the next launch (stream-ordered after
    // this one, a graph replay included) starts from zero and no launch depends on another's bookkeeping.
    __threadfence();
    if (atomicAdd(fw.done, 1u) == gridDim.x - 1) {
      __threadfence();
      for (int b = 0; b < fw.n_blocks; ++b) fw.counters[b] = 0;
      *fw.done = 0;
      __threadfence();
    }
  }
}

// Widens the arena's codes [n_pad][k_pad] to bf16 in the same layout.  Each thread takes kPer
// 16-code chunks a block-width apart and issues all their loads before converting (the grid is sized
// so that every thread has kPer chunks, which keeps enough loads in flight for HBM).
constexpr int kWidenPer = 4;

template <int kKind, bool kNaN>
__global__ void __launch_bounds__(256) widen_codes(const uint4* __restrict__ codes, uint4* __restrict__ out,
                                                    int64_t chunks) {
  pdl_launch_dependents();  // the GEMM that reads the widened copy may set up meanwhile
  const int64_t base = static_cast<int64_t>(blockIdx.x) * (256 * kWidenPer) + threadIdx.x;
  uint4 in[kWidenPer];
#pragma unroll
  for (int u = 0; u < kWidenPer; ++u) {
    const int64_t i = base + u * 256;
    in[u] = i < chunks ? __ldcs(codes + i) : make_uint4(0, 0, 0, 0);
  }
#pragma unroll
  for (int u = 0; u < kWidenPer; ++u) {
    const int64_t i = base + u * 256;
    if (i < chunks) {
      uint4 lo, hi;
      codes16_to_bf16<kKind, kNaN>(in[u], lo, hi);
      st_global_32b(out + 2 * i, lo, hi);
    }
  }
}

template <bool kF32Out, bool kPeers, int kOp = kOpNone, bool kI8 = false, int kFW = 0>
cudaError_t launch_gemm(const CUtensorMap& tm_x, const CUtensorMap& tm_w, const sc_weight* w, const uint16_t* bias,
                        void* y, int64_t m, int* err, int sm_count, cudaStream_t stream, const PeerOut& peers,
                        const float* gate = nullptr, const float* row_scales = nullptr, const HeadOut* heads = nullptr,
                        const XHeads* x_heads = nullptr, const FusedWiden* fwp = nullptr) {
  const HeadOut ho = heads != nullptr ? *heads : HeadOut{};
  FusedWiden fw = fwp != nullptr ? *fwp : FusedWiden{};
  const XHeads xh = x_heads != nullptr ? *x_heads : XHeads{0, 0};
  auto kernel = gemm_bf16_pair<kF32Out, kPeers, kOp, kI8, kFW>;
  static unsigned long long configured = 0;  // per template instance and device
  if (cudaError_t e = set_smem_once(kernel, static_cast<int>(kSmemBytes), configured); e != cudaSuccess) return e;
  const int m_tiles = static_cast<int>((m + 2 * BM - 1) / (2 * BM));
  const int n_tiles = static_cast<int>(w->n_pad / BN);
  // kI8: 128 codes per stage; the weight's K padding is a multiple of 64, and a last stage past it
  // reads zeros (the copy's fill), as x's codes are zero past K.
  const int k_tiles = static_cast<int>(kI8 ? (w->k_pad + 127) / 128 : w->k_pad / BK);
  const int tiles = m_tiles * n_tiles;
  int max_pairs = sm_count / 2;
  if (kFW != 0) {
    // The fused widening's waits need every CTA resident at once: no more pairs than the device holds
    // as co-resident clusters of this kernel (asked once per device).
    static int resident[64] = {0};
    int dev = 0;
    if (cudaError_t e = cudaGetDevice(&dev); e != cudaSuccess) return e;
    if (resident[dev & 63] == 0) {
      cudaLaunchConfig_t q = {};
      q.gridDim = dim3(static_cast<unsigned>(2 * max_pairs), 1, 1);
      q.blockDim = dim3(kThreads, 1, 1);
      q.dynamicSmemBytes = kSmemBytes;
      cudaLaunchAttribute qa[1];
      qa[0].id = cudaLaunchAttributeClusterDimension;
      qa[0].val.clusterDim.x = 2;
      qa[0].val.clusterDim.y = 1;
      qa[0].val.clusterDim.z = 1;
      q.attrs = qa;
      q.numAttrs = 1;
      int n = 0;
      if (cudaError_t e = cudaOccupancyMaxActiveClusters(&n, kernel, &q); e != cudaSuccess) return e;
      resident[dev & 63] = n > 0 ? n : 1;
    }
    if (resident[dev & 63] < max_pairs) max_pairs = resident[dev & 63];
  }
  // Pieces of 128 columns (Pieces) for the gathering product when its tiles fill under half the pairs and the
  // pieces still fit them.
  Pieces pc{0, 0, 0};
  if (kPeers && !kI8 && xh.tokens == 0 && 2 * tiles <= max_pairs) {
    const int per_row = static_cast<int>((w->n + 127) / 128);
    if (m_tiles * per_row <= max_pairs && m_tiles * per_row > tiles) pc = Pieces{128, per_row, m_tiles * per_row};
  }
  const int jobs = pc.width != 0 ? pc.count : tiles;
  const int pairs = jobs < max_pairs ? jobs : max_pairs;
  if (kFW != 0) {
    // One group of the tile order (m_tiles <= 16): tile t has column block t / m_tiles, so the first round
    // (tiles 0 .. pairs - 1) reads blocks 0 .. (pairs - 1) / m_tiles.
    fw.first_blocks = (pairs - 1) / m_tiles + 1;
    if (fw.first_blocks > fw.n_blocks) fw.first_blocks = fw.n_blocks;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[3];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // The GEMM may be launched while the kernel before it (the widening) finishes: it sets up its
  // barriers and TMEM, then waits for that kernel's writes (pdl_wait) before its first access.
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  if (kFW != 0) {
    // The fused widening's CTAs wait for one another, so they must all be resident at once: asked of the
    // runtime as a cooperative launch where it takes one beside the cluster shape (tried once per device;
    // a refused launch is an ordinary error, cleared, and the launch then goes without the attribute,
    // sized to the co-resident clusters as above).
    static signed char cooperative[64] = {0};  // 0 untried, 1 accepted, -1 refused
    int dev = 0;
    if (cudaError_t e = cudaGetDevice(&dev); e != cudaSuccess) return e;
    if (cooperative[dev & 63] >= 0) {
      attr[2].id = cudaLaunchAttributeCooperative;
      attr[2].val.cooperative = 1;
      cfg.numAttrs = 3;
      const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, tm_x, tm_w, static_cast<const float*>(w->scales), bias,
                                               y, static_cast<int>(m), static_cast<int>(w->n), k_tiles, m_tiles,
                                               n_tiles, err, peers, gate, row_scales, ho, xh, fw, pc);
      if (e == cudaSuccess) {
        cooperative[dev & 63] = 1;
        return e;
      }
      if (cooperative[dev & 63] == 1) return e;  // accepted before: a real failure
      cudaGetLastError();
      cooperative[dev & 63] = -1;
      cfg.numAttrs = 2;
    }
  }
  return cudaLaunchKernelEx(&cfg, kernel, tm_x, tm_w, static_cast<const float*>(w->scales), bias, y,
                            static_cast<int>(m), static_cast<int>(w->n), k_tiles, m_tiles, n_tiles, err, peers, gate,
                            row_scales, ho, xh, fw, pc);
}

// The weight's arena codes (int8 stored biased by 128) made signed again for the int8 MMA: code ^ 0x80.
__global__ void __launch_bounds__(256) sign_codes(const uint4* __restrict__ codes, uint4* __restrict__ out,
                                                  int64_t chunks) {
  pdl_launch_dependents();
  const int64_t base = static_cast<int64_t>(blockIdx.x) * (256 * kWidenPer) + threadIdx.x;
  uint4 in[kWidenPer];
#pragma unroll
  for (int u = 0; u < kWidenPer; ++u) {
    const int64_t i = base + u * 256;
    in[u] = i < chunks ? __ldcs(codes + i) : make_uint4(0, 0, 0, 0);
  }
#pragma unroll
  for (int u = 0; u < kWidenPer; ++u) {
    const int64_t i = base + u * 256;
    if (i < chunks)
      out[i] = make_uint4(in[u].x ^ 0x80808080u, in[u].y ^ 0x80808080u, in[u].z ^ 0x80808080u, in[u].w ^ 0x80808080u);
  }
}

// One rank waits until every rank's flag for it reached `epoch` (epochs only grow), bounded.
__global__ void gather_wait(const uint32_t* __restrict__ flags, int world, uint32_t epoch, int* err) {
  if (threadIdx.x != 0) return;
  const unsigned long long t0 = global_ns();
  for (int r = 0; r < world; ++r) {
    while (static_cast<int32_t>(ld_acquire_sys(flags + r) - epoch) < 0) {
      if (global_ns() - t0 > kWaitLimitNs) {
        record_error(err, kErrTimeout, kSiteGather);
        return;
      }
    }
  }
}

}  // namespace gemm_bf16

size_t widened_bytes(const sc_weight* w) { return static_cast<size_t>(w->n_pad) * static_cast<size_t>(w->k_pad) * 2; }

cudaError_t launch_widen(const sc_weight* w, void* out, int sm_count, cudaStream_t stream) {
  (void)sm_count;
  const int64_t chunks = w->n_pad * w->k_pad / 16;
  const int64_t per_block = 256LL * gemm_bf16::kWidenPer;
  const int64_t blocks64 = (chunks + per_block - 1) / per_block;
  if (blocks64 > 0x7FFFFFFF) return cudaErrorInvalidValue;
  const int blocks = static_cast<int>(blocks64 > 0 ? blocks64 : 1);
  const uint4* codes = reinterpret_cast<const uint4*>(w->values);
  uint4* dst = static_cast<uint4*>(out);
  if (w->kind == SC_WEIGHT_INT8)
    gemm_bf16::widen_codes<1, false><<<blocks, 256, 0, stream>>>(codes, dst, chunks);
  else if (w->has_nan_codes)
    gemm_bf16::widen_codes<2, true><<<blocks, 256, 0, stream>>>(codes, dst, chunks);
  else
    gemm_bf16::widen_codes<2, false><<<blocks, 256, 0, stream>>>(codes, dst, chunks);
  return cudaGetLastError();
}

cudaError_t launch_gemm_bf16(const CUtensorMap& tmap_x, const CUtensorMap& tmap_w, const sc_weight* w,
                             const uint16_t* bias, void* y, bool f32_out, int64_t m, int* err, int sm_count,
                             cudaStream_t stream) {
  const PeerOut none = {};
  return f32_out ? gemm_bf16::launch_gemm<true, false>(tmap_x, tmap_w, w, bias, y, m, err, sm_count, stream, none)
                 : gemm_bf16::launch_gemm<false, false>(tmap_x, tmap_w, w, bias, y, m, err, sm_count, stream, none);
}

bool fused_widen_fits(const sc_weight* w, int64_t m, int sm_count) {
  using namespace gemm_bf16;
  const int64_t m_tiles = (m + 2 * BM - 1) / (2 * BM), n_tiles = w->n_pad / BN;
  // Two to three rounds of pair tiles: there the separate widening was a sixth of the product (config 1:
  // 10 of 74 us; 70 us with it inside).  With more rounds its share shrinks and the blocks widened during
  // the run fall behind the tiles that need them (config 2, 8.6 rounds: 259 us inside against 233 apart).
  const int64_t tiles = m_tiles * n_tiles, pairs = sm_count / 2;
  return m_tiles <= kTileGroupRows && tiles >= 2 * pairs && tiles <= 3 * pairs && n_tiles <= kWidenCounterWords;
}

cudaError_t launch_gemm_bf16_fw(const CUtensorMap& tmap_x, const CUtensorMap& tmap_w, const sc_weight* w,
                                const uint16_t* bias, void* y, bool f32_out, void* widened, uint32_t* counters,
                                int64_t m, int* err, int sm_count, cudaStream_t stream) {
  using namespace gemm_bf16;
  const PeerOut none = {};
  FusedWiden fw;
  fw.codes = reinterpret_cast<const uint4*>(w->values);
  fw.out = static_cast<uint4*>(widened);
  fw.counters = counters;
  fw.done = counters + kWidenCounterWords;
  fw.chunks_per_block = static_cast<int>(BN * w->k_pad / 16);
  fw.n_blocks = static_cast<int>(w->n_pad / BN);
  fw.first_blocks = 0;  // set by launch_gemm from the pairs it launches
#define SC_FW_LAUNCH(KIND)                                                                                   \
  return f32_out ? launch_gemm<true, false, kOpNone, false, KIND>(tmap_x, tmap_w, w, bias, y, m, err, sm_count, \
                                                                   stream, none, nullptr, nullptr, nullptr,  \
                                                                   nullptr, &fw)                              \
                 : launch_gemm<false, false, kOpNone, false, KIND>(tmap_x, tmap_w, w, bias, y, m, err, sm_count, \
                                                                    stream, none, nullptr, nullptr, nullptr, \
                                                                    nullptr, &fw)
  if (w->kind == SC_WEIGHT_INT8) SC_FW_LAUNCH(1);
  if (w->has_nan_codes) SC_FW_LAUNCH(3);
  SC_FW_LAUNCH(2);
#undef SC_FW_LAUNCH
}

cudaError_t launch_gemm_bf16_xheads(const CUtensorMap& tmap_o, const CUtensorMap& tmap_w, const sc_weight* w,
                                    const uint16_t* bias, void* y, bool f32_out, int op, const float* gate,
                                    const XHeads& xh, int64_t m, int* err, int sm_count, cudaStream_t stream) {
  const PeerOut none = {};
  using namespace gemm_bf16;
  if (op == SC_EPI_GATED_RESIDUAL)
    return launch_gemm<true, false, kOpResidual>(tmap_o, tmap_w, w, bias, y, m, err, sm_count, stream, none, gate,
                                                 nullptr, nullptr, &xh);
  if (op != 0) return cudaErrorInvalidValue;
  return f32_out ? launch_gemm<true, false>(tmap_o, tmap_w, w, bias, y, m, err, sm_count, stream, none, nullptr,
                                            nullptr, nullptr, &xh)
                 : launch_gemm<false, false>(tmap_o, tmap_w, w, bias, y, m, err, sm_count, stream, none, nullptr,
                                             nullptr, nullptr, &xh);
}

cudaError_t launch_gemm_bf16_heads(const CUtensorMap& tmap_x, const CUtensorMap& tmap_w, const sc_weight* w,
                                   const uint16_t* bias, const HeadOut& heads, int64_t m, int* err, int sm_count,
                                   cudaStream_t stream) {
  const PeerOut none = {};
  return gemm_bf16::launch_gemm<false, false, gemm_bf16::kOpQkRope>(tmap_x, tmap_w, w, bias, nullptr, m, err, sm_count,
                                                                    stream, none, nullptr, nullptr, &heads);
}

cudaError_t launch_gemm_bf16_peers(const CUtensorMap& tmap_x, const CUtensorMap& tmap_w, const sc_weight* w,
                                   const uint16_t* bias, const PeerOut& peers, int64_t m, int* err, int sm_count,
                                   cudaStream_t stream) {
  return gemm_bf16::launch_gemm<false, true>(tmap_x, tmap_w, w, bias, nullptr, m, err, sm_count, stream, peers);
}

cudaError_t launch_gemm_bf16_op(const CUtensorMap& tmap_x, const CUtensorMap& tmap_w, const sc_weight* w,
                                const uint16_t* bias, void* y, int op, const float* gate, int64_t m, int* err,
                                int sm_count, cudaStream_t stream) {
  const PeerOut none = {};
  // op: an sc_epilogue value
  if (op == SC_EPI_GELU_TANH)
    return gemm_bf16::launch_gemm<false, false, gemm_bf16::kOpGelu>(tmap_x, tmap_w, w, bias, y, m, err, sm_count,
                                                                    stream, none);
  if (op == SC_EPI_GATED_RESIDUAL)
    return gemm_bf16::launch_gemm<true, false, gemm_bf16::kOpResidual>(tmap_x, tmap_w, w, bias, y, m, err, sm_count,
                                                                       stream, none, gate);
  if (op == SC_EPI_SWIGLU)
    return gemm_bf16::launch_gemm<false, false, gemm_bf16::kOpSwiglu>(tmap_x, tmap_w, w, bias, y, m, err, sm_count,
                                                                      stream, none);
  return cudaErrorInvalidValue;
}

size_t signed_codes_bytes(const sc_weight* w) {
  return static_cast<size_t>(w->n_pad) * static_cast<size_t>(w->k_pad);
}

cudaError_t launch_sign_codes(const sc_weight* w, void* out, cudaStream_t stream) {
  const int64_t chunks = w->n_pad * w->k_pad / 16;
  const int64_t per_block = 256LL * gemm_bf16::kWidenPer;
  const int64_t blocks64 = (chunks + per_block - 1) / per_block;
  if (blocks64 > 0x7FFFFFFF) return cudaErrorInvalidValue;
  gemm_bf16::sign_codes<<<static_cast<int>(blocks64 > 0 ? blocks64 : 1), 256, 0, stream>>>(
      reinterpret_cast<const uint4*>(w->values), static_cast<uint4*>(out), chunks);
  return cudaGetLastError();
}

cudaError_t launch_gemm_i8(const CUtensorMap& tmap_codes, const CUtensorMap& tmap_w, const sc_weight* w,
                           const uint16_t* bias, void* y, bool f32_out, const float* row_scales, int64_t m, int* err,
                           int sm_count, cudaStream_t stream) {
  const PeerOut none = {};
  using namespace gemm_bf16;
  return f32_out ? launch_gemm<true, false, kOpNone, true>(tmap_codes, tmap_w, w, bias, y, m, err, sm_count, stream,
                                                           none, nullptr, row_scales)
                 : launch_gemm<false, false, kOpNone, true>(tmap_codes, tmap_w, w, bias, y, m, err, sm_count, stream,
                                                            none, nullptr, row_scales);
}

cudaError_t launch_gather_wait(const uint32_t* flags, int world, uint32_t epoch, int* err, cudaStream_t stream) {
  gemm_bf16::gather_wait<<<1, 32, 0, stream>>>(flags, world, epoch, err);
  return cudaGetLastError();
}

}  // namespace sc
