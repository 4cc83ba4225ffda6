// Shared device/host helpers for the sm_100a W8A16 / LoRA-delta kernels.
//
// * PTX wrappers for mbarriers, TMA (cp.async.bulk.tensor; every CTA loads its own tiles),
//   and the 5th-generation tensor core (tcgen05.mma / TMEM).
// * Bounded waits: every spin on an mbarrier gives up after the wait limit
//   (default BW_WAIT_LIMIT_NS, settable per device with bw_set_wait_limit_ns),
//   records a site id in the device status word and lets the caller unwind,
//   so a lost arrival never hangs the GPU.
// * Host-side status plumbing shared by all entry points.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/bw_ops.h"

#ifndef BW_WAIT_LIMIT_NS
#define BW_WAIT_LIMIT_NS 4000000000ull  // default, 4 s: far beyond any legitimate wait
#endif

namespace bw {

// GEMM workspaces start with a tile-counter region of this size for every split plan; the counters
// are zero at rest, and anything else a caller keeps in a shared workspace must stay out of it.
constexpr int kGemmCounterSlots = 1024;
constexpr size_t kGemmCounterBytes = kGemmCounterSlots * sizeof(int);

// ---------------------------------------------------------------------------
// device status word (first failure wins) and the wait limit
// ---------------------------------------------------------------------------
extern __device__ int g_status;  // 0 = ok, else wait-site id
// Bound of every spin wait, in SM cycles: the limit in ns x 2.5 (no SM clock is
// above 2.5 GHz, so a wait never gives up before the limit).  Set per device by
// bw_set_wait_limit_ns; read only once a wait has not completed at first try.
extern __device__ long long g_wait_limit_cycles;
__device__ __forceinline__ long long wait_limit_cycles() {
  return *static_cast<volatile long long*>(&g_wait_limit_cycles);
}

__device__ __forceinline__ void record_timeout(int site) { atomicCAS(&g_status, 0, site); }

// ---------------------------------------------------------------------------
// device-side phase trace (off unless bw_trace_enable gave a buffer)
//
// Each CTA of a traced kernel claims one 128-byte record and fills it with
// globaltimer stamps of its phases:
//   u64 rec[16] = {gridid, blockIdx.x | gridDim.x << 32, kernel id | smid << 32, stamp[0..12]}
// (stamp 0 = phase not reached).  The host groups records by gridid (one
// launch) and reads the phases; nothing is written while tracing is off.
// ---------------------------------------------------------------------------
struct TraceState {
  unsigned long long* buf;  // null: tracing off
  unsigned int records;     // capacity
  unsigned int next;        // next free record
};
extern __device__ TraceState g_trace;
constexpr int kTraceStamps = 13;
constexpr int kTraceRecordWords = 16;

// Claim a record (call from one thread per CTA); null when tracing is off or full.
__device__ __forceinline__ unsigned long long* trace_claim(int kernel_id) {
  unsigned long long* buf = *static_cast<unsigned long long* volatile*>(&g_trace.buf);
  if (buf == nullptr) return nullptr;
  const unsigned int i = atomicAdd(&g_trace.next, 1u);
  if (i >= g_trace.records) return nullptr;
  unsigned long long* r = buf + static_cast<size_t>(i) * kTraceRecordWords;
  unsigned long long gid;
  asm volatile("mov.u64 %0, %%gridid;" : "=l"(gid));
  r[0] = gid;
  r[1] = static_cast<unsigned long long>(blockIdx.x) | (static_cast<unsigned long long>(gridDim.x) << 32);
  unsigned smid;
  asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
  r[2] = static_cast<unsigned long long>(kernel_id) | (static_cast<unsigned long long>(smid) << 32);
  for (int e = 0; e < kTraceStamps; ++e) r[3 + e] = 0ull;
  return r;
}
__device__ __forceinline__ uint64_t globaltimer_now();
__device__ __forceinline__ void trace_stamp(unsigned long long* rec, int e) {
  if (rec != nullptr) rec[3 + e] = globaltimer_now();
}

// Acquire load at GPU scope (a flag another CTA publishes with a release or a fence).
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ uint64_t globaltimer_now() { return globaltimer(); }

// ---------------------------------------------------------------------------
// shared memory addressing
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
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
#ifndef BW_MBAR_SUSPEND_NS
#define BW_MBAR_SUSPEND_NS 0
#endif
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
#if BW_MBAR_SUSPEND_NS > 0
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(BW_MBAR_SUSPEND_NS)
      : "memory");
#else
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
#endif
  return ok != 0;
}

// Wait for the phase with the given parity to complete.  Returns false (and
// records `site`) if it did not within the wait limit (measured with the SM
// cycle counter, assuming at most 2.5 GHz so the bound is never shorter), or if
// another thread of the CTA has already flagged an abort through `abort_flag`.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int site) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long limit = wait_limit_cycles();
  const long long t0 = clock64();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0u) {
      if (abort_flag != nullptr && *abort_flag) return false;
      if (clock64() - t0 > limit) {
        record_timeout(site);
        if (abort_flag != nullptr) *abort_flag = 1;
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// thread-block clusters: distributed shared memory (every CTA loads its own TMA tiles)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// All threads of all CTAs of the cluster; used once, right after barrier init,
// when every CTA of the (co-scheduled) cluster is certain to arrive.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of the same shared-memory variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_shared_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void fence_acq_rel_cluster() { asm volatile("fence.acq_rel.cluster;" ::: "memory"); }
// Release-arrive on an mbarrier of another CTA of the cluster.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                                  int site) {
  const long long limit = wait_limit_cycles();
  const long long t0 = clock64();
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((i & 63u) == 63u && clock64() - t0 > limit) {
      record_timeout(site);
      if (abort_flag != nullptr) *abort_flag = 1;
      return false;
    }
  }
}

// ---------------------------------------------------------------------------
// named barriers
// ---------------------------------------------------------------------------
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
// Named barrier that also ORs a predicate over the participating threads, so
// every participant takes the same abort decision (a thread that left a loop
// alone would otherwise leave its siblings waiting at a later bar.sync).
__device__ __forceinline__ bool named_bar_any(int id, int nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"(pred ? 1u : 0u), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

// ---------------------------------------------------------------------------
// proxies / fences
// ---------------------------------------------------------------------------
// Make this thread's generic-proxy shared-memory writes visible to the async
// proxy (TMA store engine, tensor core operand reads).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// TMA (tensor maps passed as __grid_constant__ kernel parameters)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// 2-D tiled load global -> this CTA's shared memory, completion counted on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}
// 1-D bulk copy global -> this CTA's shared memory (both addresses 16-byte
// aligned, `bytes` a multiple of 16), completion counted on `bar`.
__device__ __forceinline__ void bulk_load_1d(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                             uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
// 2-D tiled store shared -> global (bulk-group completion).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void tma_store_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void tma_store_wait_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void tma_store_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// At most one committed store group may still be reading shared memory.
__device__ __forceinline__ void tma_store_wait_read1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05 (5th-gen tensor core, accumulators in tensor memory)
// ---------------------------------------------------------------------------
// Whole warp: allocate `ncols` TMEM columns (power of two >= 32); the base
// address is written to shared memory at `dst`.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
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

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (f16/bf16 in, fp32 accumulate).
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16.  A lives in TMEM: lane = row
// of A, two consecutive 16-bit K elements per 32-bit column.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// 32 lanes x 32 bit, 32 consecutive columns per thread (register -> TMEM).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Programmatic dependent launch: wait for the preceding grid's memory to be
// visible (no-op without PDL), and allow the next grid to start launching.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Arrive once on `bar` when all previously issued tcgen05 ops of this thread complete.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 bit, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// 32 lanes x 32 bit, 32 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// Shared-memory matrix descriptor (sm_100 UMMA format):
//   [0,14) start>>4, [16,30) LBO>>4, [32,46) SBO>>4, [46,48) version=1,
//   [49,52) base offset (0: tiles are 1024-byte aligned), [61,64) layout.
constexpr uint32_t kLayoutSW128 = 2;
__device__ __forceinline__ uint64_t make_sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(layout & 7u) << 61;
  return d;
}

// Instruction descriptor, kind::f16 with fp32 accumulator.
//   [4,6) D fmt (1 = f32), [7,10) A fmt, [10,13) B fmt (0 f16, 1 bf16),
//   [15] A major, [16] B major (0 = K-major, 1 = MN-major),
//   [17,23) N>>3, [24,29) M>>4.
__host__ __device__ constexpr uint32_t make_idesc_f16(int M, int N, bool bf16, bool b_mn_major) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((b_mn_major ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// ---------------------------------------------------------------------------
// small numeric helpers
// ---------------------------------------------------------------------------
// Four int8 codes (one 32-bit word) -> two f16x2 words, exactly.  Each byte is
// biased to u = q + 128 in [1, 255], placed in the mantissa of 1024.0
// (0x6400 | u == 1024 + u) and 1152 = 1024 + 128 is subtracted.
__device__ __forceinline__ void i8x4_to_f16x4(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t u = w ^ 0x80808080u;
  uint32_t a, b;
  asm("prmt.b32 %0, %1, %2, 0x5140;" : "=r"(a) : "r"(u), "r"(0x64646464u));
  asm("prmt.b32 %0, %1, %2, 0x5342;" : "=r"(b) : "r"(u), "r"(0x64646464u));
  const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
  __half2 ha = __hsub2(*reinterpret_cast<__half2*>(&a), bias);
  __half2 hb = __hsub2(*reinterpret_cast<__half2*>(&b), bias);
  lo = *reinterpret_cast<uint32_t*>(&ha);
  hi = *reinterpret_cast<uint32_t*>(&hb);
}

// Four int8 codes -> two bf16x2 words, exactly.  The low 7 bits go into the
// mantissa of 128.0 (0x4300 | m == 128 + m); non-negative codes subtract 128,
// negative ones (m = q + 128) subtract 256 (0x4380).
__device__ __forceinline__ void i8x4_to_bf16x4(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t m = w & 0x7F7F7F7Fu;
  const uint32_t s = w & 0x80808080u;
  uint32_t a, b, sa, sb;
  asm("prmt.b32 %0, %1, %2, 0x5140;" : "=r"(a) : "r"(m), "r"(0x43434343u));
  asm("prmt.b32 %0, %1, %2, 0x5342;" : "=r"(b) : "r"(m), "r"(0x43434343u));
  asm("prmt.b32 %0, %1, %2, 0x5140;" : "=r"(sa) : "r"(s), "r"(0x43434343u));
  asm("prmt.b32 %0, %1, %2, 0x5342;" : "=r"(sb) : "r"(s), "r"(0x43434343u));
  __nv_bfloat162 va = __hsub2(*reinterpret_cast<__nv_bfloat162*>(&a), *reinterpret_cast<__nv_bfloat162*>(&sa));
  __nv_bfloat162 vb = __hsub2(*reinterpret_cast<__nv_bfloat162*>(&b), *reinterpret_cast<__nv_bfloat162*>(&sb));
  lo = *reinterpret_cast<uint32_t*>(&va);
  hi = *reinterpret_cast<uint32_t*>(&vb);
}

__device__ __forceinline__ float load_as_float(const void* p, int64_t i, int dtype) {
  if (dtype == BW_DTYPE_F16) return __half2float(static_cast<const __half*>(p)[i]);
  if (dtype == BW_DTYPE_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  return static_cast<const float*>(p)[i];
}

}  // namespace bw

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace bw {
// Record a detail message for the calling thread and return `status`.
int fail(int status, const char* fmt, ...);
// Map a CUDA error to BW_ERR_CUDA with a message (BW_OK if e == cudaSuccess).
int check_cuda(cudaError_t e, const char* what);
int check_launch(const char* what);
// sm_100 check for the current device (cached per device).
int require_sm100();
int dtype_size(int dtype);
// Encode a 2-D tiled tensor map: rows x cols (cols contiguous), row stride
// `ld_bytes`, box box_rows x box_cols, 128-byte swizzle.
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint64_t rows, uint64_t cols,
                 uint64_t ld_bytes, uint32_t box_rows, uint32_t box_cols, CUtensorMapSwizzle swz);
int num_sms();
}  // namespace bw
