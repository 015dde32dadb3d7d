// The DiT blocks' attention on the tensor cores: o = softmax(q k^T * scale) v for head_dim 128, bf16 q, k, v and
// o in the [batch * heads, seq, 128] layout the QK-norm + RoPE stage (or the q / k / v product's epilogue)
// writes and the out projection reads.
//
// The online (flash) form of the reference's fused attention (Sources/Siliconed/TiledAttention.swift:470-610):
// fp32 scores, a running row maximum m and sum l, P = exp(scale s - m) rounded to bf16 unnormalised for the
// P . v product, l summed from the unrounded exponentials, O rescaled when m moves, and O / l at the end.  One
// difference of form: the rescale is lazy.  A row's maximum is only moved when the new tile's maximum exceeds it
// by more than 2^8 (in the exponent's base-2 units); until then the tile's exponentials use the stale maximum
// and may reach 256, which fp32 sums and bf16 P carry without loss of relative precision.  The result is the same
// quotient; fewer O passes.
//
// One CTA per 128 query rows of one head (the grid's CTAs of one head consecutive, so the head's k and v stay in
// L2 while they are read).  Roles:
// - warps 0-3 first write the q tile into TMEM (each thread its row: 128 bf16 as 64 columns of pairs, read from
//   global memory), where it is the A operand of every S MMA: S = q k^T then reads only k from shared memory.
//   With both operands in shared memory the S MMAs (8 KB of operands each) ran at about 60 % of the tensor rate,
//   bound by shared-memory bandwidth beside the TMA's writes of k and v.
// - warp 4: TMA.  Lane 0 loads the k tiles of 128 keys through a ring of three 32 KB stages, lane 1 the v tiles
//   through a ring of three.  Coordinates past seq read zeros.
// - warp 5, one thread: the MMAs.  S_t = q k_t^T (tcgen05.mma kind::f16, M 128, N 128, A from TMEM, B K-major
//   from shared memory) into one of two TMEM buffers of 128 fp32 columns, two key tiles ahead of the softmax;
//   then O += P_t v_t with P_t read from TMEM (the A operand, bf16 pairs in the S buffer's first 64 columns) and
//   v_t from shared memory as an MN-major B operand (its 128-byte rows are keys, 64 dims each: LBO = the 16 KB
//   between the two dim halves, SBO = 1 KB between 8-key groups).  TMEM: S_0, S_1, O, q.
// - warps 0-3: the softmax, one query row per thread (TMEM lane = row).  Each reads its row of S 32 columns at a
//   time (the next load in flight while the last is used) and forms exp2(s c - m) with the row's running maximum m
//   (c = scale log2 e; ex2.approx), their sum and their bf16 pairs.  The maximum itself is only taken when the
//   tile's sum shows it moved far (the first tile; a sum above 2^32): then the tile is redone with the new maximum
//   and O rescaled.  Until then exponentials above 1 are kept (fp32 sums and bf16 P carry them without loss of
//   relative precision) and the result is the same quotient.  P goes back over the columns already read; before
//   handing it over the warp waits for P_{t-1} v, so that a rescale of O sees it whole.  At the end: O / l,
//   rounded to bf16, stored row by row.
// Every wait is bounded (2 s): on expiry the kernel records SD_TIMEOUT's site in a device word, raises the CTA's
// abort flag, drains and frees TMEM.  No load uses cluster multicast.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "../sc_ptx.cuh"
#include "siliconed_dit.h"

namespace {

using namespace sc;

constexpr int kHeadDim = 128;
constexpr int BQ = 128;                         // query rows a CTA
constexpr int BK = 128;                         // keys a tile
constexpr int kK = 3, kV = 3;                   // ring stages for k and for v
constexpr int kTileBytes = BK * kHeadDim * 2;   // 32 KB
constexpr int kBoxBytes = kTileBytes / 2;       // [128 rows][64 dims], 16 KB
constexpr int kThreads = 192;                   // warps 0-3 softmax, 4 TMA, 5 MMA
constexpr int kTmaWarp = 4, kMmaWarp = 5;
constexpr int kSB = 2;                          // S / P buffers in TMEM
constexpr float kMovedSum = 4294967296.0f;      // 2^32: a tile's sum above it means the maximum moved
constexpr uint32_t kTmemCols = 512;

__device__ __forceinline__ uint32_t col_s(int t) { return static_cast<uint32_t>(t % kSB) * 128u; }  // S_t; P_t: first 64
constexpr uint32_t kColO = 256;                                                                    // O: 128 columns
constexpr uint32_t kColQ = 384;                                                                    // q: 64 columns

enum : int { kSiteLoadEmpty = 21, kSiteScores = 22, kSiteProbs = 23, kSiteValues = 24, kSiteQuery = 25, kSiteOut = 26 };

struct __align__(1024) Smem {
  uint8_t k[kK][kTileBytes];
  uint8_t v[kV][kTileBytes];
  uint64_t q_ready;      // q written into TMEM (one arrival per softmax warp)
  uint64_t k_full[kK], k_empty[kK];
  uint64_t v_full[kV], v_empty[kV];
  uint64_t s_full[kSB];  // S_t complete in buffer t % 3 (MMA -> softmax)
  uint64_t p_full[kSB];  // P_t written to buffer t % 3, S_t read (softmax -> MMA; one arrival per softmax warp)
  uint64_t o_done;       // P_t v_t complete (MMA -> softmax), once per key tile
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

constexpr size_t kSmemBytes = sizeof(Smem) + 1024;
static_assert(kSmemBytes <= 227 * 1024, "shared memory per CTA");

__device__ int g_attention_err[4];  // [0] SD_TIMEOUT once set, [1] the wait's site, [2] the CTA

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]: A (bf16 pairs, one row per TMEM lane) from tensor memory.
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 consecutive 32-bit columns of this thread's TMEM lane, written.
__device__ __forceinline__ void tmem_st_32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory descriptor of an MN-major, 128-byte-swizzled bf16 operand: 128-byte rows of 64 MN elements,
// 8-row (K) groups `sbo` bytes apart, the next 64 MN elements `lbo` bytes on.
__device__ __forceinline__ uint64_t umma_desc_mn_sw128(uint32_t start, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((start >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1u) << 46;  // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2u) << 61;  // 128-byte swizzle
  return d;
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// One lane-0 wait broadcast to the warp (tcgen05.ld / st are warp-collective, so the warp moves together).  The
// handoffs between the softmax and the MMA thread are the kernel's critical path, so they poll with the
// non-suspending probe: a suspending wait was seen to notice a completed phase 300-600 cycles late.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int* err, int site) {
  int got = 0;
  if ((threadIdx.x & 31) == 0) got = mbar_poll(bar, parity, abort, err, site) ? 1 : 0;
  return __shfl_sync(0xFFFFFFFFu, got, 0) != 0;
}

// exp2(s c - m) over this row of a tile of S (keys at or past `valid` left out when kMasked), packed to bf16 pairs
// in p (keys 2k, 2k + 1 in p[k]), and their fp32 sum; 32 columns at a time, the next load in flight.
template <bool kMasked>
__device__ __forceinline__ float row_exps(uint32_t sb, int valid, float c_log2, float m, uint32_t (&p)[BK / 2]) {
  float sum4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  uint32_t r[2][32];
  tmem_ld_32(sb, r[0]);
#pragma unroll
  for (int c = 0; c < BK / 32; ++c) {
    tmem_wait_ld();
    if (c + 1 < BK / 32) tmem_ld_32(sb + (c + 1) * 32, r[(c + 1) & 1]);
    const uint32_t* x = r[c & 1];
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      float s0 = __uint_as_float(x[2 * k]), s1 = __uint_as_float(x[2 * k + 1]);
      if (kMasked) {
        if (c * 32 + 2 * k >= valid) s0 = -INFINITY;
        if (c * 32 + 2 * k + 1 >= valid) s1 = -INFINITY;
      }
      const float e0 = ex2(fmaf(s0, c_log2, -m));
      const float e1 = ex2(fmaf(s1, c_log2, -m));
      sum4[k & 3] += e0 + e1;
      p[c * 16 + k] = pack_bf16x2(e0, e1);
    }
  }
  return (sum4[0] + sum4[1]) + (sum4[2] + sum4[3]);
}

// The row's maximum of s over a tile (kMasked: the keys inside the sequence), times c.
template <bool kMasked>
__device__ __forceinline__ float row_max(uint32_t sb, int valid, float c_log2) {
  float mx8[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) mx8[k] = -INFINITY;
#pragma unroll
  for (int c = 0; c < BK / 32; ++c) {
    uint32_t r[32];
    tmem_ld_32(sb + c * 32, r);
    tmem_wait_ld();
#pragma unroll
    for (int k = 0; k < 32; ++k)
      if (!kMasked || c * 32 + k < valid) mx8[k & 7] = fmaxf(mx8[k & 7], __uint_as_float(r[k]));
  }
  return c_log2 * fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])), fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
}

// One tile of this row: P in p, its sum, the running maximum m and the factor alpha that l and O take.
template <bool kMasked>
__device__ __forceinline__ float softmax_tile(uint32_t sb, int valid, float c_log2, bool first, float& m, float& alpha,
                                              uint32_t (&p)[BK / 2]) {
  alpha = 1.0f;
  if (first) {
    m = row_max<kMasked>(sb, valid, c_log2);
    return row_exps<kMasked>(sb, valid, c_log2, m, p);
  }
  float sum = row_exps<kMasked>(sb, valid, c_log2, m, p);
  const bool moved = !(sum <= kMovedSum);  // (a NaN sum takes the slow path too)
  if (__any_sync(0xFFFFFFFFu, moved)) {  // rare: S is still in TMEM, P not yet written back
    // one call for the whole warp: tcgen05.ld is warp-collective (.sync.aligned), so every lane must reach the
    // same instruction; the lanes whose maximum did not move keep theirs
    const float mt = row_max<kMasked>(sb, valid, c_log2);
    if (moved && mt > m) {
      alpha = ex2(m - mt);
      m = mt;
    }
    sum = row_exps<kMasked>(sb, valid, c_log2, m, p);
  }
  return sum;
}

__global__ void __launch_bounds__(kThreads, 1)
    attention_fwd(const uint16_t* __restrict__ q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, uint16_t* __restrict__ o, int seq, int q_tiles,
                  float c_log2, int* err) {
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = static_cast<int>(blockIdx.x) / q_tiles, q0 = (static_cast<int>(blockIdx.x) % q_tiles) * BQ;
  const int n = (seq + BK - 1) / BK;
  volatile int* abort = &s.abort;

  if (threadIdx.x == 0) {
    mbar_init(&s.q_ready, 4);
    for (int i = 0; i < kK; ++i) {
      mbar_init(&s.k_full[i], 1);
      mbar_init(&s.k_empty[i], 1);
    }
    for (int i = 0; i < kV; ++i) {
      mbar_init(&s.v_full[i], 1);
      mbar_init(&s.v_empty[i], 1);
    }
    for (int i = 0; i < kSB; ++i) {
      mbar_init(&s.s_full[i], 1);
      mbar_init(&s.p_full[i], 4);
    }
    mbar_init(&s.o_done, 1);
    mbar_init(&s.drain, 1);
    s.abort = 0;
    fence_mbar_init();
    prefetch_tensormap(&tm_k);
    prefetch_tensormap(&tm_v);
  }
  if (warp == kMmaWarp) {
    tmem_alloc(&s.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

  if (warp == kTmaWarp) {
    // ---------------- TMA producers: q and k (lane 0), v (lane 1) ----------------
    if (lane < 2) {
      const bool keys = lane == 0;
      const int stages = keys ? kK : kV;
      uint64_t* full = keys ? s.k_full : s.v_full;
      uint64_t* empty = keys ? s.k_empty : s.v_empty;
      const CUtensorMap* map = keys ? &tm_k : &tm_v;
      uint32_t issued = 0, last_parity = 0;
      for (int t = 0; t < n && !*abort; ++t) {
        const int st = t % stages;
        const uint32_t ph = static_cast<uint32_t>(t / stages) & 1u;
        if (!mbar_wait(&empty[st], ph ^ 1u, abort, err, kSiteLoadEmpty)) break;
        uint8_t* dst = keys ? s.k[st] : s.v[st];
        mbar_arrive_expect_tx(&full[st], kTileBytes);
        tma_load_3d(dst, map, &full[st], 0, t * BK, bh);
        tma_load_3d(dst + kBoxBytes, map, &full[st], 64, t * BK, bh);
        issued |= 1u << st;
        last_parity = (last_parity & ~(1u << st)) | (ph << st);
      }
      // no copy may still be landing when the CTA leaves (on the normal path the MMA thread consumed them all)
      for (int st = 0; st < stages; ++st)
        if (issued & (1u << st)) mbar_wait_drain(&full[st], (last_parity >> st) & 1u);
    }
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc_s = umma_idesc_bf16(BQ, BK);                     // both K-major
      const uint32_t idesc_o = umma_idesc_bf16(BQ, kHeadDim) | (1u << 16);  // B (v) MN-major
      auto issue_scores = [&](int t) -> bool {
        const int st = t % kK;
        if (!mbar_wait(&s.k_full[st], static_cast<uint32_t>(t / kK) & 1u, abort, err, kSiteScores)) return false;
        tc_fence_after();
        const uint32_t d = tmem + col_s(t);
        const uint32_t kb = smem_u32(s.k[st]);
#pragma unroll
        for (int kk = 0; kk < kHeadDim / 16; ++kk) {  // 16 dims a step: 8 columns of q, 32 bytes of k's swizzle atom
          const uint32_t off = static_cast<uint32_t>((kk >> 2) * kBoxBytes + (kk & 3) * 32);
          tc_mma_ts(d, tmem + kColQ + kk * 8, umma_desc_sw128(kb + off), idesc_s, kk > 0 ? 1u : 0u);
        }
        tc_commit(&s.k_empty[st]);
        tc_commit(&s.s_full[t % kSB]);
        return true;
      };
      bool ok = mbar_poll(&s.q_ready, 0, abort, err, kSiteQuery);
      if (ok) tc_fence_after();
      for (int t = 0; t < kSB && t < n && ok; ++t) ok = issue_scores(t);
      for (int t = 0; t < n && ok; ++t) {
        if (!mbar_poll(&s.p_full[t % kSB], static_cast<uint32_t>(t / kSB) & 1u, abort, err, kSiteProbs)) break;
        const int st = t % kV;
        if (!mbar_wait(&s.v_full[st], static_cast<uint32_t>(t / kV) & 1u, abort, err, kSiteValues)) break;
        tc_fence_after();
        const uint32_t a = tmem + col_s(t);  // P: 64 columns of bf16 pairs, keys 2c and 2c + 1 in column c
        const uint32_t vb = smem_u32(s.v[st]);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)  // 16 keys a step: two 8-key groups of 1 KB
          tc_mma_ts(tmem + kColO, a + kk * 8, umma_desc_mn_sw128(vb + kk * 2048, kBoxBytes, 1024), idesc_o,
                    (t > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&s.v_empty[st]);
        tc_commit(&s.o_done);
        if (t + kSB < n) ok = issue_scores(t + kSB);
      }
      tc_commit(&s.drain);
      mbar_wait_drain(&s.drain, 0);
    }
  } else {
    // ---------------- q into TMEM, the softmax, then the output ----------------
    const int row = warp * 32 + lane;
    const uint32_t lanes = static_cast<uint32_t>(warp * 32) << 16;
    const uint32_t ob = tmem + lanes + kColO;
    {
      // this row of q (zeros past seq) as 64 columns of bf16 pairs: dims 2c and 2c + 1 in column c
      uint32_t qv[kHeadDim / 2];
      const bool in_seq = q0 + row < seq;
      const uint4* src = reinterpret_cast<const uint4*>(q + (static_cast<int64_t>(bh) * seq + (in_seq ? q0 + row : 0)) * kHeadDim);
#pragma unroll
      for (int i = 0; i < kHeadDim / 8; ++i) {
        const uint4 v4 = in_seq ? __ldg(src + i) : make_uint4(0, 0, 0, 0);
        qv[4 * i] = v4.x;
        qv[4 * i + 1] = v4.y;
        qv[4 * i + 2] = v4.z;
        qv[4 * i + 3] = v4.w;
      }
      tmem_st_32(tmem + lanes + kColQ, qv);
      tmem_st_32(tmem + lanes + kColQ + 32, qv + 32);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.q_ready);
    }
    float m = 0.0f, l = 0.0f;
    bool ok = true;
    for (int t = 0; t < n; ++t) {
      if (!warp_wait(&s.s_full[t % kSB], static_cast<uint32_t>(t / kSB) & 1u, abort, err, kSiteScores)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t sb = tmem + lanes + col_s(t);
      const int valid = seq - t * BK;  // keys of this tile inside the sequence
      uint32_t p[BK / 2];
      float alpha;
      const float sum = valid < BK ? softmax_tile<true>(sb, valid, c_log2, t == 0, m, alpha, p)
                                   : softmax_tile<false>(sb, valid, c_log2, t == 0, m, alpha, p);
      l = fmaf(l, alpha, sum);
      tmem_st_32(sb, p);
      tmem_st_32(sb + 32, p + 32);
      if (t > 0) {
        // P_{t-1} v_{t-1} complete: O is whole for a rescale
        if (!warp_wait(&s.o_done, static_cast<uint32_t>(t - 1) & 1u, abort, err, kSiteOut)) {
          ok = false;
          tmem_wait_st();
          break;
        }
        tc_fence_after();
        if (__any_sync(0xFFFFFFFFu, alpha != 1.0f)) {
#pragma unroll 1
          for (int c = 0; c < kHeadDim / 32; ++c) {
            uint32_t x[32];
            tmem_ld_32(ob + c * 32, x);
            tmem_wait_ld();
#pragma unroll
            for (int k = 0; k < 32; ++k) x[k] = __float_as_uint(__uint_as_float(x[k]) * alpha);
            tmem_st_32(ob + c * 32, x);
          }
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.p_full[t % kSB]);
    }
    if (ok && warp_wait(&s.o_done, static_cast<uint32_t>(n - 1) & 1u, abort, err, kSiteOut)) {
      tc_fence_after();
      const float inv = 1.0f / l;
      const int qrow = q0 + row;
      uint4* dst = reinterpret_cast<uint4*>(o + (static_cast<int64_t>(bh) * seq + qrow) * kHeadDim);
#pragma unroll 1
      for (int c = 0; c < kHeadDim / 32; ++c) {
        uint32_t x[32];
        tmem_ld_32(ob + c * 32, x);
        tmem_wait_ld();
        uint32_t h[16];
#pragma unroll
        for (int k = 0; k < 16; ++k)
          h[k] = pack_bf16x2(__uint_as_float(x[2 * k]) * inv, __uint_as_float(x[2 * k + 1]) * inv);
        if (qrow < seq) {
#pragma unroll
          for (int k = 0; k < 4; ++k) dst[c * 4 + k] = make_uint4(h[4 * k], h[4 * k + 1], h[4 * k + 2], h[4 * k + 3]);
        }
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

typedef CUresult (*encode_fn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                              const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                              CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

encode_fn encoder() {
  static encode_fn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<encode_fn>(p);
  }
  return fn;
}

// [bh][seq][128] bf16 as a 3-D tensor map with boxes of 64 dims x 128 rows, 128-byte swizzle (zeros past seq).
bool make_map(CUtensorMap* map, encode_fn enc, const uint16_t* base, int bh, int seq) {
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kHeadDim), static_cast<cuuint64_t>(seq), static_cast<cuuint64_t>(bh)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(kHeadDim) * 2, static_cast<cuuint64_t>(seq) * kHeadDim * 2};
  const cuuint32_t box[3] = {64, static_cast<cuuint32_t>(BK), 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<uint16_t*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

extern "C" {

SD_API int sd_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* o, int bh, int seq,
                        int head_dim, float scale, void* stream) {
  if (q == nullptr || k == nullptr || v == nullptr || o == nullptr || bh < 1 || seq < 1 || head_dim != kHeadDim ||
      !(scale > 0.0f) || !std::isfinite(scale))
    return SD_INVALID_ARG;
  for (const void* p : {static_cast<const void*>(q), static_cast<const void*>(k), static_cast<const void*>(v),
                        static_cast<const void*>(o)})
    if ((reinterpret_cast<uintptr_t>(p) & 15u) != 0) return SD_INVALID_ARG;
  const int64_t q_tiles = (seq + BQ - 1) / BQ;
  if (q_tiles * bh > 0x7FFFFFFF) return SD_INVALID_ARG;
  encode_fn enc = encoder();
  if (enc == nullptr) return SD_CUDA_ERROR;
  CUtensorMap tk, tv;
  if (!make_map(&tk, enc, k, bh, seq) || !make_map(&tv, enc, v, bh, seq)) return SD_INVALID_ARG;
  static unsigned long long configured = 0;  // one bit per device
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return SD_CUDA_ERROR;
  if (dev < 64 && !(configured & (1ull << dev))) {
    if (cudaFuncSetAttribute(attention_fwd, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemBytes)) !=
        cudaSuccess)
      return SD_CUDA_ERROR;
    configured |= 1ull << dev;
  }
  int* err = nullptr;
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&err), g_attention_err) != cudaSuccess) return SD_CUDA_ERROR;
  const float c_log2 = static_cast<float>(static_cast<double>(scale) * 1.4426950408889634);  // scale * log2(e)
  attention_fwd<<<static_cast<unsigned>(q_tiles * bh), kThreads, kSmemBytes, static_cast<cudaStream_t>(stream)>>>(
      q, tk, tv, o, seq, static_cast<int>(q_tiles), c_log2, err);
  return cudaGetLastError() == cudaSuccess ? SD_OK : SD_CUDA_ERROR;
}

SD_API int sd_attention_errors(int* site) {
  int h[4] = {0, 0, 0, 0};
  const int zero[4] = {0, 0, 0, 0};
  if (cudaMemcpyFromSymbol(h, g_attention_err, sizeof(h)) != cudaSuccess) return SD_CUDA_ERROR;
  if (h[0] != 0 && cudaMemcpyToSymbol(g_attention_err, zero, sizeof(zero)) != cudaSuccess) return SD_CUDA_ERROR;
  if (site != nullptr) *site = h[1];
  return h[0] != 0 ? SD_TIMEOUT : SD_OK;
}

}  // extern "C"
