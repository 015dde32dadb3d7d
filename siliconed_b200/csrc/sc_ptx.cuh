// Inline-PTX building blocks for sm_100a: shared-memory mbarriers with bounded waits, tensor-map
// (TMA) bulk loads, the async-proxy fence, and the tcgen05 family (TMEM allocation, MMA issue,
// commit, TMEM loads).  Every wait here is bounded in time: a wait that gives up records an error
// in the caller's error word and returns false, so no kernel of this library can spin forever.
#pragma once

#include <cstdint>
#include <cuda.h>

namespace sc {

// A wait on an mbarrier gives up after this long (global timer, nanoseconds).
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

// Error codes written to the device error word (sc_ctx::d_err[0]).
constexpr int kErrTimeout = 1;

// Sites recorded beside a timeout (d_err[1]).
enum WaitSite : int {
  kSiteProducerEmpty = 1,
  kSiteConverterFull = 2,
  kSiteConverterSlot = 3,
  kSiteMmaInput = 4,
  kSiteMmaConverted = 5,
  kSiteMmaAccum = 6,
  kSiteEpilogueFull = 7,
  kSiteDrain = 8,
  kSiteGather = 9,
  kSiteWidened = 10,
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-suspending probe of a phase (the thread keeps its issue slot; for latency-critical pollers).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Records the first error of a launch: code, site, block.
__device__ __forceinline__ void record_error(int* err, int code, int site) {
  if (err != nullptr && atomicCAS(err, 0, code) == 0) {
    err[1] = site;
    err[2] = static_cast<int>(blockIdx.x);
  }
}

// Waits for the phase of `bar` with parity `parity` to complete.  Returns false (and raises the
// CTA's abort flag) when `abort` is raised by another role or when the time limit passes.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int* err, int site) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 31u) == 0u) {
      if (*abort) return false;
      if (global_ns() - t0 > kWaitLimitNs) {
        record_error(err, kErrTimeout, site);
        *abort = 1;
        return false;
      }
    }
  }
}

// Flags between GPUs (the fused gather): system-scope acquire load and release store.
// Output-tile order of the persistent GEMMs: groups of kTileGroupRows row tiles, and inside a group
// the row tile fastest, so that the tiles in flight at one time (one per CTA pair) share a few row
// blocks of x and a few column blocks of the weight, which stay in L2.  With x larger than L2 (the
// DiT blocks' 32768-row products) a plain column-major order re-read all of x from HBM once per
// column block.  Products with at most kTileGroupRows row tiles keep the column-major order.
constexpr int kTileGroupRows = 16;

__device__ __forceinline__ void tile_coords(int tile, int m_tiles, int n_tiles, int& mt, int& nt) {
  const int group = tile / (kTileGroupRows * n_tiles);
  const int first = group * kTileGroupRows;
  const int rows = min(m_tiles - first, kTileGroupRows);
  const int t = tile - first * n_tiles;
  mt = first + t % rows;
  nt = t / rows;
}

// Programmatic dependent launch.  The kernel launched after this one on the stream (with the
// programmatic-serialization attribute) may start once every CTA of this grid has issued this, or exited.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
// Waits until the grid this one depends on has completed and its writes are visible; returns at once for a
// kernel launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// One 16-byte store to a multicast address: NVSwitch delivers it to the same offset of every GPU bound
// to the multicast object (the bits are moved, not converted).
__device__ __forceinline__ void multimem_st_v4(void* mc, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc), "f"(__uint_as_float(v.x)),
               "f"(__uint_as_float(v.y)), "f"(__uint_as_float(v.z)), "f"(__uint_as_float(v.w))
               : "memory");
}

// Two 16-byte values to 32 contiguous bytes of global memory: one 256-bit store (st.global.v8.b32,
// sm_100) when the address is 32-byte aligned, so that a warp's store covers whole 32-byte sectors in
// one instruction; two 128-bit stores otherwise.
__device__ __forceinline__ void st_global_32b(uint4* p, uint4 lo, uint4 hi) {
  if ((reinterpret_cast<uintptr_t>(p) & 31u) == 0) {
    asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(lo.x), "r"(lo.y),
                 "r"(lo.z), "r"(lo.w), "r"(hi.x), "r"(hi.y), "r"(hi.z), "r"(hi.w)
                 : "memory");
  } else {
    p[0] = lo;
    p[1] = hi;
  }
}

// 16-byte global load cached in L2 only (data this kernel also writes: not the read-only path).
__device__ __forceinline__ float4 ld_cg_f4(const float* p) {
  float4 v;
  asm volatile("ld.global.cg.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
  return v;
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Orders this thread's earlier global accesses (the acquire of a flag) before its later async-proxy
// accesses (TMA reads of data other CTAs wrote with ordinary stores).
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// mbar_wait by polling with the non-suspending probe.
__device__ __forceinline__ bool mbar_poll(uint64_t* bar, uint32_t parity, volatile int* abort, int* err, int site) {
  if (mbar_test_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_test_wait(bar, parity)) return true;
    if ((i & 255u) == 0u) {
      if (*abort) return false;
      if (global_ns() - t0 > kWaitLimitNs) {
        record_error(err, kErrTimeout, site);
        *abort = 1;
        return false;
      }
    }
  }
}

// The same without an abort flag, for a drain at exit: gives up quietly after the limit.
__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity) {
  const unsigned long long t0 = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_ns() - t0 > kWaitLimitNs) return false;
  }
  return true;
}

// Generic-proxy writes to shared memory made visible to the async proxy (TMA, tensor cores).
__device__ __forceinline__ void fence_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 2D tensor-map load into this CTA's shared memory, completing on `bar` (no multicast).
// c0 is the innermost coordinate; c0 * element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// 2D tensor-map load into this CTA's shared memory for a CTA-pair MMA (.cta_group::2, no
// multicast): the bytes are counted on the mbarrier at shared::cluster address `bar_cluster`, which
// may be the leader CTA's, so one barrier sees both CTAs' operands land.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int c0,
                                                 int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1)
      : "memory");
}

// The same with a 4-D tensor map (the attention's output [batch, heads, joint, 128] read as the rows of a
// product's operand).
__device__ __forceinline__ void tma_load_4d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int c0,
                                                 int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// 1D bulk copy global -> this CTA's shared memory, completing on `bar` (no multicast).  Both addresses
// 16-byte aligned, `bytes` a multiple of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// `bytes` (a multiple of 16) of global memory from `p` (16-byte aligned) brought toward the L2; nothing
// reaches shared memory and nothing waits for it.
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---- tcgen05 -------------------------------------------------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, bf16 inputs, fp32 accumulate (kind::f16).
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on `bar` when every tcgen05 operation this thread issued before it has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane (lane = the warp's 32-lane slice).
__device__ __forceinline__ void tmem_ld_32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Named barrier `id` (1..15) over `threads` threads (a multiple of 32); every thread named must arrive.
__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---- clusters and CTA pairs ---------------------------------------------------------------

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// The shared::cluster address of the variable at `local` in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t peer_addr(const void* local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(local)), "r"(rank));
  return r;
}

// Arrive on an mbarrier given by its shared::cluster address (this CTA's or the peer's).  Default
// (CTA-scope release) semantics: the data it announces is in the arriving CTA's own shared memory,
// made visible to the tensor cores beforehand by the async-proxy fence.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// mbar_wait for barriers that the other CTA of the pair arrives on (acquire at cluster scope).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort, int* err,
                                                  int site) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((i & 31u) == 0u) {
      if (*abort) return false;
      if (global_ns() - t0 > kWaitLimitNs) {
        record_error(err, kErrTimeout, site);
        *abort = 1;
        return false;
      }
    }
  }
}

__device__ __forceinline__ void cluster_barrier() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Generic-proxy shared-memory writes made visible to the async proxy of either CTA of the pair.
__device__ __forceinline__ void fence_async_all() { asm volatile("fence.proxy.async;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem of both CTAs] (+)= A[both CTAs' smem] * B[both CTAs' smem]^T, M = 256 across the pair.
__device__ __forceinline__ void tc_mma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, 8-bit integer operands, s32 accumulate (kind::i8, one CTA).
__device__ __forceinline__ void tc_mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tc_mma_i8_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on the mbarrier at shared::cluster address `bar` (this CTA's or the peer's) when the
// pair MMAs this thread issued have completed.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar_cluster_addr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster_addr)
               : "memory");
}

// Arrives once on the mbarrier at the same shared-memory offset in each CTA of `cta_mask` when the
// pair MMAs this thread issued have completed (a commit, not a load: no data moves).
__device__ __forceinline__ void tc_commit_pair_both(const uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

// Shared-memory matrix descriptor of a K-major, 128-byte-swizzled bf16 tile: rows of 64 elements
// (128 bytes), groups of 8 rows 1024 bytes apart.  The tile must start on a 1024-byte boundary;
// moving `start` by 32 bytes steps K by 16 inside the swizzle atom.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t start) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((start >> 4) & 0x3FFFu);        // start address, 16-byte units
  d |= static_cast<uint64_t>(1u) << 16;                       // leading byte offset (unused when swizzled)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;               // stride byte offset: 8-row groups
  d |= static_cast<uint64_t>(1u) << 46;                       // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2u) << 61;                       // layout: 128-byte swizzle
  return d;
}

// Instruction descriptor: bf16 x bf16 -> fp32, both operands K-major, tile M x N.
// kind::i8: D s32, A and B signed 8-bit, both K-major, no saturation (the int32 sums wrap, as the
// exact sums of int8 products do not for K below 2^17).
// kind::i8 with A unsigned 8-bit (the arena's biased int8 codes, u = q + 128) and B signed 8-bit.
__host__ __device__ constexpr uint32_t umma_idesc_u8s8(int m, int n) {
  return (2u << 4)                                  // D format: s32
         | (0u << 7)                                // A format: unsigned 8-bit
         | (1u << 10)                               // B format: signed 8-bit
         | (static_cast<uint32_t>(n >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);   // M / 16
}

__host__ __device__ constexpr uint32_t umma_idesc_s8(int m, int n) {
  return (2u << 4)                                  // D format: s32
         | (1u << 7)                                // A format: signed 8-bit
         | (1u << 10)                               // B format: signed 8-bit
         | (static_cast<uint32_t>(n >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);   // M / 16
}

__host__ __device__ constexpr uint32_t umma_idesc_bf16(int m, int n) {
  return (1u << 4)                                  // D format: fp32
         | (1u << 7)                                // A format: bf16
         | (1u << 10)                               // B format: bf16
         | (static_cast<uint32_t>(n >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);   // M / 16
}

}  // namespace sc
