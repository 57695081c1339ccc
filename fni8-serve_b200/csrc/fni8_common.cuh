// Shared device helpers for the sm_100a W8A8 path: mbarriers, TMA bulk-tensor loads,
// tcgen05 (TMEM alloc, MMA kind::i8, commit, ld) and a bounded wait that gives up after
// a fixed wall-clock budget instead of spinning forever.
//
// Everything here is inline PTX written for sm_100a; there is no fallback for other
// architectures.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdlib.h>

#include <atomic>

#include "../../include/fni8_b200.h"
#include "tuning.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "fni8-serve_b200 kernels target sm_100a only"
#endif

namespace fni8b {

// ---------------------------------------------------------------------------------
// Watchdog: every spin-wait in the library is bounded. A wait that exceeds
// kWaitBudgetNs records an error code into the caller's per-file status word and
// returns false; the caller then abandons its loop, drains what it issued (bounded),
// frees TMEM and exits. The host reads the word with fni8_device_status().
// ---------------------------------------------------------------------------------
constexpr uint64_t kWaitBudgetNs = 1000ull * 1000ull * 1000ull;  // 1 s

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
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

// Bounded wait for the phase with the given parity to complete. Returns false (and
// records `code` in *status unless one is already there) after kWaitBudgetNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0u && globaltimer_ns() - t0 > kWaitBudgetNs) {
      atomicCAS(status, 0, code);
      return false;
    }
  }
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// 2-D tiled load; x is the innermost (contiguous) coordinate in elements.
__device__ __forceinline__ void tma_load_2d(const CUtensorMap* map, uint64_t* bar, void* dst, int32_t x,
                                            int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
// Prefetch a 2-D tile into L2 only (no shared memory, no barrier).
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap* map, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global [%0, {%1, %2}];" ::"l"(reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void tma_load_3d(const CUtensorMap* map, uint64_t* bar, void* dst, int32_t x,
                                            int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// 2-D tiled store shared -> global (bulk async group); rows/columns past the tensor's
// extent are not written.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// 16-byte asynchronous global -> shared copy through L2 only (no L1 allocation).
__device__ __forceinline__ void cp_async_16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// Wait until at most N committed groups of this thread's cp.async copies are in flight.
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// Wait until at most N committed bulk groups still read their shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Wait until at most N committed bulk groups are still in flight (writes done).
template <int N>
__device__ __forceinline__ void bulk_wait_group() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Instruction descriptor for tcgen05.mma kind::i8: D = s32, A = B = signed 8-bit,
// both operands K-major, dense, no negate, shape M x N (M in {64,128}, N % 16 == 0).
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N) {
  return (2u << 4)                                   // D format: s32
         | (1u << 7)                                 // A format: signed 8-bit
         | (1u << 10)                                // B format: signed 8-bit
         | (static_cast<uint32_t>(N >> 3) << 17)     // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);    // M / 16
}

// Shared-memory matrix descriptor for a K-major operand stored with the 128-byte
// swizzle that a TMA load with CU_TENSOR_MAP_SWIZZLE_128B produces: rows of 128 bytes,
// 8-row (1024-byte) swizzle atoms stacked along M/N. LBO is unused for this layout (1),
// SBO = 1024 bytes between 8-row groups, version 1 (sm_100), layout code 2 (128B swizzle).
// sbo_bytes = 0 makes every 8-row group read the first one (rows 8.. alias rows 0..7).
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t saddr, uint32_t sbo_bytes = 1024u) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(sbo_bytes >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread.
__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on `bar` when every tcgen05 op previously issued by this thread completes.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// ---------------------------------------------------------------- CTA pairs (cta_group::2)
// Two CTAs of a cluster (ranks 2i, 2i+1) run one MMA of M=256 rows: each holds its 128 A
// rows and half of the B rows in its own shared memory and receives its 128 accumulator
// rows in its own TMEM. The even CTA issues the MMAs; both allocate TMEM collectively.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void umma_i8_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on the barrier at `bar`'s offset in every CTA of `cta_mask` when the pair's
// tcgen05 ops issued so far complete.
__device__ __forceinline__ void umma_commit_pair_to(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// Tiled loads into this CTA's shared memory whose completion is counted on an mbarrier
// of the pair's even CTA (`bar_cluster`: a shared::cluster address).
__device__ __forceinline__ void tma_load_2d_pair(const CUtensorMap* map, uint32_t bar_cluster, void* dst, int32_t x,
                                                 int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d_pair(const CUtensorMap* map, uint32_t bar_cluster, void* dst, int32_t x,
                                                 int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
      "%5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp gets lane (base+i).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, uint32_t (&r)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// After tmem_ld_wait: marks the destination registers of the waited-for loads as written
// here, so the compiler schedules no use of them before the wait (an empty statement).
__device__ __forceinline__ void tmem_regs_ready(uint32_t (&r)[32]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

// ---------------------------------------------------------------- clusters / DSMEM
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same variable in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t local_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(rank));
  return r;
}
// Arrive (release at cluster scope) on an mbarrier that may live in another CTA.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
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
// Bounded wait that also acquires the writes other CTAs of the cluster released.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* status, int code) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((i & 63u) == 0u && globaltimer_ns() - t0 > kWaitBudgetNs) {
      atomicCAS(status, 0, code);
      return false;
    }
  }
}
__device__ __forceinline__ uint32_t ld_dsmem_u32(uint32_t cluster_addr) {
  uint32_t v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(cluster_addr) : "memory");
  return v;
}
__device__ __forceinline__ uint4 ld_dsmem_v4(uint32_t cluster_addr) {
  uint4 v;
  asm volatile("ld.shared::cluster.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(cluster_addr)
               : "memory");
  return v;
}
// Store into the shared memory of a CTA of this cluster (a local address works too).
__device__ __forceinline__ void st_dsmem_v4(uint32_t cluster_addr, uint4 v) {
  asm volatile("st.shared::cluster.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(cluster_addr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}
// Whole-cluster barrier; every thread of every CTA of the cluster must execute it.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// ---------------------------------------------------------------- misc
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
// AND of `pred` over the `nthreads` threads that meet at named barrier `id`.
__device__ __forceinline__ int named_bar_and(int id, int nthreads, int pred) {
  int out;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 q, %3, 0;\n\t"
      "bar.red.and.pred p, %1, %2, q;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(out)
      : "r"(id), "r"(nthreads), "r"(pred)
      : "memory");
  return out;
}
__device__ __forceinline__ void red_add_s32(int32_t* p, int32_t v) {
  asm volatile("red.relaxed.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Programmatic dependent launch: wait for the upstream grid's memory to be visible,
// and allow the downstream grid to begin its prologue.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// fp32 -> output element, and fp16/bf16 -> fp32, without contraction surprises.
template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) {
  return __half2float(v);
}
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) {
  return __float2half_rn(v);
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// Round to the storage type and back (the value the unfused chain would re-read).
template <typename T>
__device__ __forceinline__ float round_trip(float v) {
  return to_f32<T>(from_f32<T>(v));
}

// g / d for d >= 1 (or +inf) in straight-line code: the hardware reciprocal estimate of d,
// one Newton-Raphson step r' = r + r (1 - d r) (the classical reciprocal iteration, which
// doubles the correct bits), the quotient q0 = g r', and Markstein's correction step
// q = q0 + r' (g - q0 d) with fused multiply-adds (P. Markstein, "IA-64 and Elementary
// Functions", 2000), which leaves q the correctly rounded quotient except in rare
// double-rounding cases. d = +inf gives g * 0 (the IEEE quotient of a finite g). Unlike an
// IEEE division it has no slow-path branch, so an unrolled epilogue can interleave many
// elements.
__device__ __forceinline__ float div_by_ge1(float g, float d) {
  float r;
  asm("rcp.approx.f32 %0, %1;" : "=f"(r) : "f"(d));
  r = __fmaf_rn(__fmaf_rn(-d, r, 1.0f), r, r);
  const float q0 = __fmul_rn(g, r);
  const float q = __fmaf_rn(__fmaf_rn(-q0, d, g), r, q0);
  return isinf(d) ? __fmul_rn(g, 0.0f) : q;
}

// act(g) of act_and_mul (fni8serve/layers/activation.py:21-45) in fp32: SiLU g / (1 + e^-g),
// or the tanh-approximated GELU 0.5 g (1 + tanh(sqrt(2/pi) (g + 0.044715 g^3))); CUDA's
// expf / tanhf, no contraction outside the quotient. Shared by the row kernels and the GEMM
// epilogue that applies it, so both round identically.
template <int ACT>
__device__ __forceinline__ float act_fn(float g) {
  if constexpr (ACT == FNI8_ACT_SILU) {
    return div_by_ge1(g, __fadd_rn(1.0f, expf(-g)));
  } else {
    const float k0 = 0.7978845608028654f, k1 = 0.044715f;
    float inner = __fmul_rn(k0, __fadd_rn(g, __fmul_rn(k1, __fmul_rn(g, __fmul_rn(g, g)))));
    return __fmul_rn(__fmul_rn(0.5f, g), __fadd_rn(1.0f, tanhf(inner)));
  }
}

// One element of act_and_mul on the rounded gate and up values: act(g) rounded to T, times
// u, rounded to T (the reference's F.silu(gate) * up on fp16 tensors).
template <typename T, int ACT>
__device__ __forceinline__ T act_mul_one(float g, float u) {
  return from_f32<T>(__fmul_rn(round_trip<T>(act_fn<ACT>(g)), u));
}

}  // namespace fni8b

// ---------------------------------------------------------------------------------
// Host-side helpers shared by the entry points (defined in capi.cu).
// ---------------------------------------------------------------------------------
namespace fni8h {
// Record a human-readable message for fni8_last_error_message() and return `status`.
int fail(int status, const char* fmt, ...);
int cuda_status(cudaError_t e, const char* what);
int num_sms(int device);
int current_device();
// cuTensorMapEncodeTiled via the runtime's driver entry point (no libcuda link).
int encode_tmap_2d_i8(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                      uint32_t box_inner, uint32_t box_outer);
// 16-bit elements (fp16 / bf16); swizzle64 selects the 64-byte swizzle (box rows of 64 B).
int encode_tmap_2d_16_sw(CUtensorMap* map, const void* base, bool bf16, uint64_t inner, uint64_t outer,
                         uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, bool swizzle64);
// 16-bit elements (fp16 / bf16), no swizzle: rows of box_inner elements land contiguously.
int encode_tmap_2d_16(CUtensorMap* map, const void* base, bool bf16, uint64_t inner, uint64_t outer,
                      uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer);
// 8-bit elements with the 64-byte swizzle (box rows of 64 B: packed int4 weight tiles).
int encode_tmap_2d_u8_sw64(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                           uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer);
int encode_tmap_3d_i8(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1,
                      uint64_t stride2, uint32_t box0, uint32_t box1);
}  // namespace fni8h

namespace fni8h {
// Programmatic dependent launch between the library's kernels (FNI8_TUNE_PDL, on).
inline int pdl_enabled() { return FNI8_TUNE_PDL != 0 ? 1 : 0; }

// Launch with programmatic dependent launch allowed: the kernel may be scheduled while
// the previous kernel on the stream drains; it must execute griddepcontrol.wait before
// touching that kernel's results. Also pins the shared-memory carveout to the maximum so
// consecutive kernels of the library never force an L1/shared reconfiguration.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args);

// First failed launch_pdl of this host thread since FNI8_CHECK_LAUNCH last looked
// (cudaLaunchKernelEx returns a refused launch, e.g. too many registers for the block,
// without leaving it for cudaGetLastError).
inline thread_local cudaError_t t_launch_error = cudaSuccess;
inline cudaError_t take_launch_error() {
  const cudaError_t e = t_launch_error;
  t_launch_error = cudaSuccess;
  return e != cudaSuccess ? e : cudaGetLastError();
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = fni8h::pdl_enabled();
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  static std::atomic<bool> carveout_set[64] = {};  // per kernel instantiation and device (host threads may race)
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < 64 && !carveout_set[dev]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    carveout_set[dev] = true;
  }
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
  if (e != cudaSuccess && t_launch_error == cudaSuccess) t_launch_error = e;
  return e;
}
}  // namespace fni8h

#define FNI8_CHECK_LAUNCH(what)                                  \
  do {                                                           \
    cudaError_t _e = fni8h::take_launch_error();                 \
    if (_e != cudaSuccess) return fni8h::cuda_status(_e, what);  \
  } while (0)
