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
// One CTA per 128 query rows of one head (the grid's tiles of one head consecutive, so the head's k and v stay in
// L2 while they are read).  Roles:
// - warp 0, one thread: TMA.  q's tile once ([128 rows][128 dims] as two 128-byte-swizzled boxes of 64 dims), then
//   k and v tiles of 128 keys through rings of two 32 KB stages each.  Coordinates past seq read zeros.
// - warp 1, one thread: the MMAs.  S_j = q k_j^T (tcgen05.mma kind::f16, M 128, N 128, both operands K-major from
//   shared memory) into one of two TMEM buffers of 128 fp32 columns, two tiles ahead of the softmax; then
//   O += P_j v_j with P_j read from TMEM (the A operand, bf16 pairs in the S buffer's first 64 columns) and v_j
//   from shared memory as an MN-major B operand (its 128-byte rows are keys, 64 dims each: LBO = the 16 KB between
//   the two dim halves, SBO = 1 KB between 8-key groups).  O lives in TMEM for the CTA's whole run.
// - warps 4-7: the softmax, one query row per thread (TMEM lane = row).  Each reads its row of S_j (128 fp32),
//   masks keys past seq, takes the maximum, forms exp2(s c - m) (c = scale log2 e; ex2.approx), adds them to l,
//   packs them to bf16 pairs and writes them back into the buffer for the MMA.  Before writing P_j it waits for
//   P_{j-1} v_{j-1} to finish, so that a rescale of O (a warp reads, scales and writes its rows' O) sees it whole.
//   At the end: O / l, rounded to bf16, stored row by row.
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
constexpr int kKV = 2;                          // ring stages for k and for v
constexpr int kTileBytes = BK * kHeadDim * 2;   // 32 KB
constexpr int kBoxBytes = kTileBytes / 2;       // [128 rows][64 dims], 16 KB
constexpr int kThreads = 256;
constexpr int kSoftWarp0 = 4;                   // warps 4-7: TMEM lanes 0-127
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 256;                 // O: 128 fp32 columns (S / P buffers: columns 0 and 128)
constexpr float kLazyLog2 = 8.0f;               // a row's maximum moves when exceeded by more than 2^8

__device__ __forceinline__ uint32_t col_s(int j) { return (j & 1) ? 128u : 0u; }

enum : int { kSiteLoadEmpty = 21, kSiteScores = 22, kSiteProbs = 23, kSiteValues = 24, kSiteQuery = 25, kSiteOut = 26 };

struct __align__(1024) Smem {
  uint8_t q[kTileBytes];
  uint8_t k[kKV][kTileBytes];
  uint8_t v[kKV][kTileBytes];
  uint64_t q_full;
  uint64_t k_full[kKV], k_empty[kKV];
  uint64_t v_full[kKV], v_empty[kKV];
  uint64_t s_full[2];  // S_j complete in buffer j % 2 (MMA -> softmax)
  uint64_t p_full[2];  // P_j written to buffer j % 2, S_j read (softmax -> MMA; one arrival per softmax warp)
  uint64_t o_done;     // P_j v_j complete (MMA -> softmax), once per tile
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

// One lane-0 wait broadcast to the warp (tcgen05.ld / st are warp-collective, so the warp moves together).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int* err, int site) {
  int got = 0;
  if ((threadIdx.x & 31) == 0) got = mbar_wait(bar, parity, abort, err, site) ? 1 : 0;
  return __shfl_sync(0xFFFFFFFFu, got, 0) != 0;
}

__global__ void __launch_bounds__(kThreads, 1)
    attention_fwd(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, uint16_t* __restrict__ o, int seq, int q_tiles,
                  float c_log2, int* err) {
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = static_cast<int>(blockIdx.x) / q_tiles, q0 = (static_cast<int>(blockIdx.x) % q_tiles) * BQ;
  const int n = (seq + BK - 1) / BK;
  volatile int* abort = &s.abort;

  if (threadIdx.x == 0) {
    mbar_init(&s.q_full, 1);
    for (int i = 0; i < kKV; ++i) {
      mbar_init(&s.k_full[i], 1);
      mbar_init(&s.k_empty[i], 1);
      mbar_init(&s.v_full[i], 1);
      mbar_init(&s.v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.s_full[i], 1);
      mbar_init(&s.p_full[i], 4);
    }
    mbar_init(&s.o_done, 1);
    mbar_init(&s.drain, 1);
    s.abort = 0;
    fence_mbar_init();
    prefetch_tensormap(&tm_q);
    prefetch_tensormap(&tm_k);
    prefetch_tensormap(&tm_v);
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
      mbar_arrive_expect_tx(&s.q_full, kTileBytes);
      tma_load_3d(s.q, &tm_q, &s.q_full, 0, q0, bh);
      tma_load_3d(s.q + kBoxBytes, &tm_q, &s.q_full, 64, q0, bh);
      uint32_t issued = 0, last_parity = 0;
      for (int j = 0; j < n && !*abort; ++j) {
        const int st = j % kKV;
        const uint32_t ph = static_cast<uint32_t>(j / kKV) & 1u;
        if (!mbar_wait(&s.k_empty[st], ph ^ 1u, abort, err, kSiteLoadEmpty)) break;
        mbar_arrive_expect_tx(&s.k_full[st], kTileBytes);
        tma_load_3d(s.k[st], &tm_k, &s.k_full[st], 0, j * BK, bh);
        tma_load_3d(s.k[st] + kBoxBytes, &tm_k, &s.k_full[st], 64, j * BK, bh);
        issued |= 1u << st;
        last_parity = (last_parity & ~(1u << st)) | (ph << st);
        if (!mbar_wait(&s.v_empty[st], ph ^ 1u, abort, err, kSiteLoadEmpty)) break;
        mbar_arrive_expect_tx(&s.v_full[st], kTileBytes);
        tma_load_3d(s.v[st], &tm_v, &s.v_full[st], 0, j * BK, bh);
        tma_load_3d(s.v[st] + kBoxBytes, &tm_v, &s.v_full[st], 64, j * BK, bh);
        issued |= 1u << (st + kKV);
        last_parity = (last_parity & ~(1u << (st + kKV))) | (ph << (st + kKV));
      }
      // no copy may still be landing when the CTA leaves (on the normal path the MMA thread consumed them all)
      mbar_wait_drain(&s.q_full, 0);
      for (int st = 0; st < kKV; ++st) {
        if (issued & (1u << st)) mbar_wait_drain(&s.k_full[st], (last_parity >> st) & 1u);
        if (issued & (1u << (st + kKV))) mbar_wait_drain(&s.v_full[st], (last_parity >> (st + kKV)) & 1u);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc_s = umma_idesc_bf16(BQ, BK);                 // both K-major
      const uint32_t idesc_o = umma_idesc_bf16(BQ, kHeadDim) | (1u << 16);  // B (v) MN-major
      auto issue_scores = [&](int j) -> bool {
        const int st = j % kKV;
        if (!mbar_wait(&s.k_full[st], static_cast<uint32_t>(j / kKV) & 1u, abort, err, kSiteScores)) return false;
        tc_fence_after();
        const uint32_t d = tmem + col_s(j);
        const uint32_t qa = smem_u32(s.q), kb = smem_u32(s.k[st]);
#pragma unroll
        for (int kk = 0; kk < kHeadDim / 16; ++kk) {  // 16 dims a step: 32 bytes inside a swizzle atom
          const uint32_t off = static_cast<uint32_t>((kk >> 2) * kBoxBytes + (kk & 3) * 32);
          tc_mma_f16(d, umma_desc_sw128(qa + off), umma_desc_sw128(kb + off), idesc_s, kk > 0 ? 1u : 0u);
        }
        tc_commit(&s.k_empty[st]);
        tc_commit(&s.s_full[j & 1]);
        return true;
      };
      bool ok = mbar_wait(&s.q_full, 0, abort, err, kSiteQuery);
      if (ok) {
        tc_fence_after();
        ok = issue_scores(0);
      }
      if (ok && n > 1) ok = issue_scores(1);
      for (int j = 0; j < n && ok; ++j) {
        if (!mbar_wait(&s.p_full[j & 1], static_cast<uint32_t>(j >> 1) & 1u, abort, err, kSiteProbs)) break;
        const int st = j % kKV;
        if (!mbar_wait(&s.v_full[st], static_cast<uint32_t>(j / kKV) & 1u, abort, err, kSiteValues)) break;
        tc_fence_after();
        const uint32_t a = tmem + col_s(j);  // P_j: 64 columns of bf16 pairs, keys 2c and 2c + 1 in column c
        const uint32_t vb = smem_u32(s.v[st]);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)  // 16 keys a step: two 8-key groups of 1 KB
          tc_mma_ts(tmem + kColO, a + kk * 8, umma_desc_mn_sw128(vb + kk * 2048, kBoxBytes, 1024), idesc_o,
                    (j > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&s.v_empty[st]);
        tc_commit(&s.o_done);
        if (j + 2 < n) ok = issue_scores(j + 2);
      }
      tc_commit(&s.drain);
      mbar_wait_drain(&s.drain, 0);
    }
  } else if (warp >= kSoftWarp0) {
    // ---------------- softmax, then the output ----------------
    const int sw = warp - kSoftWarp0;
    const int row = sw * 32 + lane;
    const uint32_t lanes = static_cast<uint32_t>(sw * 32) << 16;
    float m = 0.0f, l = 0.0f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      if (!warp_wait(&s.s_full[j & 1], static_cast<uint32_t>(j >> 1) & 1u, abort, err, kSiteScores)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t sb = tmem + lanes + col_s(j);
      uint32_t r[BK];
#pragma unroll
      for (int c = 0; c < BK / 32; ++c) tmem_ld_32(sb + c * 32, *reinterpret_cast<uint32_t(*)[32]>(r + c * 32));
      tmem_wait_ld();
      const int valid = seq - j * BK;  // keys of this tile inside the sequence
      if (valid < BK) {
#pragma unroll
        for (int i = 0; i < BK; ++i)
          if (i >= valid) r[i] = 0xFF800000u;  // -inf: P = 0
      }
      float mx8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mx8[i] = __uint_as_float(r[i]);
#pragma unroll
      for (int i = 8; i < BK; ++i) mx8[i & 7] = fmaxf(mx8[i & 7], __uint_as_float(r[i]));
      const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                             fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      const float mt = mx * c_log2;
      float alpha = 1.0f;
      if (j == 0) {
        m = mt;
      } else if (mt > m + kLazyLog2) {
        alpha = ex2(m - mt);
        m = mt;
      }
      uint32_t p[BK / 2];
      float sum4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int i = 0; i < BK / 2; ++i) {
        const float e0 = ex2(fmaf(__uint_as_float(r[2 * i]), c_log2, -m));
        const float e1 = ex2(fmaf(__uint_as_float(r[2 * i + 1]), c_log2, -m));
        sum4[i & 3] += e0 + e1;
        p[i] = pack_bf16x2(e0, e1);
      }
      l = fmaf(l, alpha, (sum4[0] + sum4[1]) + (sum4[2] + sum4[3]));
      if (j > 0) {
        // P_{j-1} v_{j-1} complete: O is whole (for a rescale), and nothing reads the buffer P_j goes to
        if (!warp_wait(&s.o_done, static_cast<uint32_t>(j - 1) & 1u, abort, err, kSiteOut)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xFFFFFFFFu, alpha != 1.0f)) {
          const uint32_t ob = tmem + lanes + kColO;
#pragma unroll 1
          for (int c = 0; c < kHeadDim / 32; ++c) {
            uint32_t t[32];
            tmem_ld_32(ob + c * 32, t);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) t[i] = __float_as_uint(__uint_as_float(t[i]) * alpha);
            tmem_st_32(ob + c * 32, t);
          }
        }
      }
      tmem_st_32(sb, p);
      tmem_st_32(sb + 32, p + 32);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.p_full[j & 1]);
    }
    if (ok && warp_wait(&s.o_done, static_cast<uint32_t>(n - 1) & 1u, abort, err, kSiteOut)) {
      tc_fence_after();
      const float inv = 1.0f / l;
      const int qrow = q0 + row;
      uint4* dst = reinterpret_cast<uint4*>(o + (static_cast<int64_t>(bh) * seq + qrow) * kHeadDim);
#pragma unroll 1
      for (int c = 0; c < kHeadDim / 32; ++c) {
        uint32_t t[32];
        tmem_ld_32(tmem + lanes + kColO + c * 32, t);
        tmem_wait_ld();
        uint32_t h[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          h[i] = pack_bf16x2(__uint_as_float(t[2 * i]) * inv, __uint_as_float(t[2 * i + 1]) * inv);
        if (qrow < seq) {
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[c * 4 + i] = make_uint4(h[4 * i], h[4 * i + 1], h[4 * i + 2], h[4 * i + 3]);
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
  CUtensorMap tq, tk, tv;
  if (!make_map(&tq, enc, q, bh, seq) || !make_map(&tk, enc, k, bh, seq) || !make_map(&tv, enc, v, bh, seq))
    return SD_INVALID_ARG;
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
      tq, tk, tv, o, seq, static_cast<int>(q_tiles), c_log2, err);
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
