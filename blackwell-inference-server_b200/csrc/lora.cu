// LoRA delta / merge / requantisation on the 5th-generation tensor core, sm_100a.
//
// Replaces the reference's CUDA-core kernels:
//   lora_delta_kernel        src/blackwell_ops/cuda/lora_ops.cu:16-27
//   lora_delta_tiled_kernel  src/blackwell_ops/cuda/lora_tiled.cu:20-83
//   add_delta_kernel         src/blackwell_ops/cuda/lora_ops.cu:32-38
// and fuses them with quantize_weight_int8 (src/blackwell_ops/kernels/int8_gemm.py:63-68)
// for per-adapter requantisation.
//
//   delta[n,k] = fp16( fp32(sum_j B[n,j] A[j,k]) * s )                 (lora_ops.cu:26)
//   merged     = fp16( fp32(W[n,k]) + fp32(delta[n,k]) )               (lora_ops.cu:36)
//   (q, scale) = quantize_weight_int8(merged)                          (int8_gemm.py:63-68)
//
// Delta and merge: one kernel, two epilogues.  A CTA owns a 128-row x
// 128-column output tile: TMA brings B[128 rows, r] (K-major, 128-byte swizzle;
// the rank dimension is zero-filled up to a multiple of 16), A[r, 128 cols]
// (MN-major, 128-byte swizzle: TMA writes A's natural row-major layout and the
// UMMA descriptor reads it transposed, so A is never transposed in memory) and,
// for the merge, the W tile.  One thread issues r/16 tcgen05.mma (M=128, N=128,
// K=16) into a 128-column TMEM accumulator; 128 epilogue threads (thread = row)
// read it back, round, merge, and write the result through swizzled shared
// memory and a TMA store.
//
// Requantisation (the cooperative kernel below) needs each row's absolute
// maximum over all of K before any code can be written: it computes the merged
// panels twice, once for the row maxima and once for the codes, so the merged
// fp16 weight never touches HBM.
#include <stdio.h>

#include <string.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "quant_math.cuh"

namespace bw {

enum LoraMode : int { kModeDelta = 0, kModeMerge = 1 };

constexpr int kLoraMaxR = 128;

__device__ __forceinline__ float h2f_lo(uint32_t w) { return __half2float(__ushort_as_half(static_cast<unsigned short>(w & 0xFFFFu))); }
__device__ __forceinline__ float h2f_hi(uint32_t w) { return __half2float(__ushort_as_half(static_cast<unsigned short>(w >> 16))); }
__device__ __forceinline__ uint32_t pack_h2(__half a, __half b) {
  return static_cast<uint32_t>(__half_as_ushort(a)) | (static_cast<uint32_t>(__half_as_ushort(b)) << 16);
}

// Epilogue for one 128x128 tile; thread = tile row.  The result overwrites the
// W tile in shared memory (the TMA store's source).
template <int MODE>
__device__ __forceinline__ void lora_tile_epilogue(uint32_t taddr, uint8_t* sW, int row, float scaling) {
  const int sw = row & 7;
#pragma unroll 1
  for (int c0 = 0; c0 < 128; c0 += 16) {
    uint32_t r[16];
    tmem_ld16(taddr + c0, r);
    tmem_ld_wait();
    const int p = c0 >> 6;
    const int j = (c0 & 63) >> 3;
    uint4* w0 = reinterpret_cast<uint4*>(sW + p * 16384 + row * 128 + ((j ^ sw) << 4));
    uint4* w1 = reinterpret_cast<uint4*>(sW + p * 16384 + row * 128 + (((j + 1) ^ sw) << 4));
    __half d[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) d[e] = __float2half_rn(__uint_as_float(r[e]) * scaling);
    uint32_t o[8];
    if constexpr (MODE == kModeDelta) {
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = pack_h2(d[2 * e], d[2 * e + 1]);
    } else {
      const uint4 a = *w0, b = *w1;
      const uint32_t win[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
      for (int e = 0; e < 8; ++e)
        o[e] = pack_h2(__float2half_rn(h2f_lo(win[e]) + __half2float(d[2 * e])),
                       __float2half_rn(h2f_hi(win[e]) + __half2float(d[2 * e + 1])));
    }
    *w0 = make_uint4(o[0], o[1], o[2], o[3]);
    *w1 = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

// ---------------------------------------------------------------------------
// Persistent ΔW / merge: one CTA per SM walks a contiguous range of 128 x 128 output tiles in
// row-major order, so a CTA keeps the row block's B[128, r] resident across its k-tiles and
// streams only A[r, 128] panels (from L2: A is shared by every row block) and, for the merge,
// the W tiles.  The MMA of tile i+1 runs while the epilogues of earlier tiles convert and store
// them (one TMEM accumulator per epilogue group), and TMA stores overlap the next tile's epilogue.
//   warp 0      TMA producer (B when the row block changes, A panels, W tiles)
//   warp 1      TMEM owner and tcgen05.mma issuer (r/16 MMAs of M=N=128, K=16 per tile)
//   warps 4-15  epilogue, kLsGroups = 3 groups of four taking the tiles in turn, thread = row:
//               fp16(acc * s) (delta) or fp16(W + fp16(acc * s)) (merge), staged in the
//               128-byte-swizzled layout and written by TMA stores.  The epilogue bounds the
//               launch (ΔW writes 32 KB per tile, read-modify-write for the merge): a third group
//               measured faster than two on the 70B shapes.
// ---------------------------------------------------------------------------
constexpr int kLsGroups = 3;
constexpr int kLsThreads = 128 + 128 * kLsGroups;
constexpr int kLsSmemBudget = 220 * 1024;
// barriers (A ring 2 x 6, B 2, W 2 x (kLsGroups + 1), accumulators 2 x kLsGroups, final) + 8 bytes
static_assert((12 + 2 + 2 * (kLsGroups + 1) + 2 * kLsGroups + 1) * 8 + 8 <= 256, "barrier area");

struct LoraStreamSmem {
  int rp, nbp, a_bytes, b_bytes, wslots, aslots, off_a, off_b, off_w, off_bar, total;
  __host__ __device__ LoraStreamSmem(int r, int mode) {
    rp = (r + 15) / 16 * 16;
    nbp = (rp + 63) / 64;
    a_bytes = ((2 * rp * 128 + 1023) / 1024) * 1024;
    b_bytes = nbp * 16384;
    // output staging (delta) / W tiles updated in place (merge), one per group; the merge takes a
    // slot more (its producer one W tile ahead of the groups) where two A panels still fit
    wslots = kLsGroups;
    if (mode != kModeDelta && kLsSmemBudget - b_bytes - (kLsGroups + 1) * 32768 >= 2 * a_bytes) wslots = kLsGroups + 1;
    const int left = kLsSmemBudget - b_bytes - wslots * 32768;
    aslots = left / a_bytes > 6 ? 6 : left / a_bytes;
    off_a = 0;
    off_b = off_a + aslots * a_bytes;
    off_w = off_b + b_bytes;
    off_bar = off_w + wslots * 32768;
    total = off_bar + 256 + 1024;
  }
};

enum LoraStreamSite : int {
  kSiteLsProd = 221,
  kSiteLsMma = 222,
  kSiteLsEpi = 223,
  kSiteLsDrain = 224,
};

template <int MODE>
__global__ void __launch_bounds__(kLsThreads, 1)
    lora_stream_kernel(const __grid_constant__ CUtensorMap tm_b, const __grid_constant__ CUtensorMap tm_a,
                       const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_out, int N,
                       int K, int r, float scaling) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const LoraStreamSmem L(r, MODE);
  const int SA = L.aslots, SW = L.wslots;
  uint64_t* afull = reinterpret_cast<uint64_t*>(smem + L.off_bar);  // [6]
  uint64_t* aempty = afull + 6;                                      // [6]
  uint64_t* bfull = aempty + 6;
  uint64_t* bempty = bfull + 1;
  uint64_t* wfull = bempty + 1;   // [kLsGroups + 1] merge: W tile landed
  uint64_t* wempty = wfull + kLsGroups + 1;  // [kLsGroups + 1] merge: the tile's TMA store has read the slot
  uint64_t* dfull = wempty + kLsGroups + 1;  // [kLsGroups]
  uint64_t* dempty = dfull + kLsGroups;
  uint64_t* final_bar = dempty + kLsGroups;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(final_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_cb = (K + 127) / 128;
  const long long tiles = static_cast<long long>((N + 127) / 128) * n_cb;
  const long long t_begin = tiles * blockIdx.x / gridDim.x, t_end = tiles * (blockIdx.x + 1) / gridDim.x;
  const int ntile = static_cast<int>(t_end - t_begin);

  if (threadIdx.x == 0) {
    for (int i = 0; i < 6; ++i) {
      mbar_init(&afull[i], 1);
      mbar_init(&aempty[i], 1);
    }
    mbar_init(bfull, 1);
    mbar_init(bempty, 1);
    for (int i = 0; i < kLsGroups + 1; ++i) {
      mbar_init(&wfull[i], 1);
      mbar_init(&wempty[i], 1);
    }
    for (int i = 0; i < kLsGroups; ++i) {
      mbar_init(&dfull[i], 1);
      mbar_init(&dempty[i], 4);
    }
    mbar_init(final_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);  // kLsGroups x 128 accumulator columns
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t keep = l2_policy_evict_last();   // A and B are re-read by many tiles
      const uint64_t once = l2_policy_evict_first();  // W is read once
      int prev_rb = -1, nb = 0, issued_a = 0, issued_w = 0;
      bool ok = true;
      for (int i = 0; i < ntile && ok; ++i) {
        const long long t = t_begin + i;
        const int rb = static_cast<int>(t / n_cb), cb = static_cast<int>(t % n_cb);
        if (rb != prev_rb) {  // new row block: B once the MMAs of the previous one are done
          if (nb > 0 && !mbar_wait(bempty, (nb - 1) & 1, abort_flag, kSiteLsProd)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(bfull, L.b_bytes);
          for (int p = 0; p < L.nbp; ++p) tma_load_2d(smem + L.off_b + p * 16384, &tm_b, bfull, p * 64, rb * 128, keep);
          ++nb;
          prev_rb = rb;
        }
        const int sa = i % SA;
        if (i >= SA && !mbar_wait(&aempty[sa], ((i / SA) & 1) ^ 1, abort_flag, kSiteLsProd)) {
          ok = false;
          break;
        }
        uint8_t* sA = smem + L.off_a + sa * L.a_bytes;
        mbar_arrive_expect_tx(&afull[sa], 2 * L.rp * 128);
        tma_load_2d(sA, &tm_a, &afull[sa], cb * 128, 0, keep);
        tma_load_2d(sA + L.rp * 128, &tm_a, &afull[sa], cb * 128 + 64, 0, keep);
        issued_a = i + 1;
        if constexpr (MODE != kModeDelta) {
          const int sw = i % SW;
          if (i >= SW && !mbar_wait(&wempty[sw], ((i / SW) & 1) ^ 1, abort_flag, kSiteLsProd)) {
            ok = false;
            break;
          }
          uint8_t* sWt = smem + L.off_w + sw * 32768;
          mbar_arrive_expect_tx(&wfull[sw], 32768);
          tma_load_2d(sWt, &tm_w, &wfull[sw], cb * 128, rb * 128, once);
          tma_load_2d(sWt + 16384, &tm_w, &wfull[sw], cb * 128 + 64, rb * 128, once);
          issued_w = i + 1;
        }
      }
      if (!ok) {  // the copies still in flight land before the CTA may exit
        for (int j = issued_a > SA ? issued_a - SA : 0; j < issued_a; ++j)
          mbar_wait(&afull[j % SA], (j / SA) & 1, nullptr, kSiteLsDrain);
        for (int j = issued_w > SW ? issued_w - SW : 0; j < issued_w; ++j)
          mbar_wait(&wfull[j % SW], (j / SW) & 1, nullptr, kSiteLsDrain);
        if (nb > 0) mbar_wait(bfull, (nb - 1) & 1, nullptr, kSiteLsDrain);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = make_idesc_f16(128, 128, false, true);
      int prev_rb = -1, nb = 0;
      for (int i = 0; i < ntile; ++i) {
        const long long t = t_begin + i;
        const int rb = static_cast<int>(t / n_cb);
        const int db = i % kLsGroups;
        if (!mbar_wait(&dempty[db], ((i / kLsGroups) & 1) ^ 1, abort_flag, kSiteLsMma)) break;
        if (rb != prev_rb) {
          if (!mbar_wait(bfull, nb & 1, abort_flag, kSiteLsMma)) break;
          ++nb;
          prev_rb = rb;
        }
        const int sa = i % SA;
        if (!mbar_wait(&afull[sa], (i / SA) & 1, abort_flag, kSiteLsMma)) break;
        tc_fence_after();
        const uint32_t b_base = smem_u32(smem + L.off_b);
        const uint32_t a_base = smem_u32(smem + L.off_a + sa * L.a_bytes);
        for (int kk = 0; kk < L.rp / 16; ++kk) {
          const uint64_t ad = make_sdesc(b_base + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024, kLayoutSW128);
          const uint64_t bd = make_sdesc(a_base + kk * 2048, L.rp * 128, 1024, kLayoutSW128);
          umma_f16(tmem + db * 128, ad, bd, idesc, kk > 0 ? 1u : 0u);
        }
        umma_commit(&aempty[sa]);
        umma_commit(&dfull[db]);
        // the last tile of this row block in the CTA's range: B may be replaced once it completes
        const bool last_of_rb = i + 1 == ntile || static_cast<int>((t + 1) / n_cb) != rb;
        if (last_of_rb) umma_commit(bempty);
      }
      umma_commit(final_bar);
      mbar_wait(final_bar, 0, nullptr, kSiteLsDrain);
    }
  } else if (warp >= 4) {
    // kLsGroups epilogue groups (warps 4-7, 8-11, 12-15) take the tiles in turn, each with its own
    // accumulator (tile i: buffer i % kLsGroups) and named barrier; a group's leader issues its TMA
    // stores and waits for them to read the staging slot before the group writes that slot again
    const int grp = (warp - 4) >> 2;
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const int bar_id = 1 + grp;
    const bool leader = (warp & 3) == 0 && lane == 0 && (warp >> 2) == 1 + grp;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
    for (int i = grp; i < ntile; i += kLsGroups) {
      const long long t = t_begin + i;
      const int rb = static_cast<int>(t / n_cb), cb = static_cast<int>(t % n_cb);
      const int db = i % kLsGroups;
      const int sw = i % SW;
      uint8_t* sWt = smem + L.off_w + sw * 32768;
      bool ok = mbar_wait(&dfull[db], (i / kLsGroups) & 1, abort_flag, kSiteLsEpi);
      if constexpr (MODE != kModeDelta) ok = ok && mbar_wait(&wfull[sw], (i / SW) & 1, abort_flag, kSiteLsEpi);
      // one decision for the group; the leader's wait for its previous store is ordered before it
      if (named_bar_any(bar_id, 128, !ok || *abort_flag)) break;
      tc_fence_after();
      lora_tile_epilogue<MODE>(lane_base + db * 128, sWt, row, scaling);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dempty[db]);  // accumulator read: the MMA may reuse it
      fence_proxy_async_smem();
      named_bar_sync(bar_id, 128);
      if (leader) {
        tma_store_2d(&tm_out, sWt, cb * 128, rb * 128);
        if (cb * 128 + 64 < K) tma_store_2d(&tm_out, sWt + 16384, cb * 128 + 64, rb * 128);  // never past K
        tma_store_commit();
        tma_store_wait_read0();  // the store has read the slot
        if constexpr (MODE != kModeDelta) mbar_arrive(&wempty[sw]);
      }
    }
    if (leader) tma_store_wait0();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// Grouped, cooperative merge + requantisation.
//
// One launch covers up to kReqMaxProblems projections (e.g. every projection an
// adapter touches).  The work is cut into uniform items, one 128-row x 64-column
// panel each, numbered problem-major then row block then panel, and dealt to a
// grid of co-resident CTAs (one per SM, cooperative launch) in contiguous
// ranges.  Each CTA walks its range twice:
//   pass 1: TMA brings the W panel and the A[r, 64] panel into a ring of
//           stages sized to fill shared memory (and B[128, r] when the row
//           block changes, double-buffered); tcgen05.mma (M=128, N=64,
//           K=16 x r/16) -> one of eight TMEM accumulator slots; the epilogue
//           merges W' = fp16(W + fp16(acc*s)) in registers (__hadd2 is the
//           correctly rounded fp16 sum = fp16(fp32(W) + fp32(delta))) and keeps
//           each row's running |W'| maximum, merged into the workspace's
//           per-row maxima with one atomicMax per row block;
//   grid barrier (a self-resetting generation barrier in the workspace; every
//           CTA is resident, the wait is bounded);
//   pass 2: the same panels again (W hits L2, delta recomputed on the tensor
//           core), row scale from one load of the row maximum, packed exact
//           quantiser, int8 stored by each warp with its own TMA store.
// The epilogue is four groups of four warps (thread = row) that take the
// items in turn, so four items are in flight there while the producer and the
// MMA run up to a full ring ahead (into pass 2 while the epilogue waits at the
// grid barrier).  The merged weight never touches memory.  The workspace holds
// the barrier's count and generation and two sets of row maxima: a call uses
// the set of its generation's parity and clears the other one for the next
// call, so no CTA does clean-up work after its own items.
// ---------------------------------------------------------------------------
constexpr int kReqMaxProblems = 16;
constexpr int kReqGroups = 4;                      // epilogue groups of 4 warps, items taken in turn
constexpr int kReqSlots = 2 * kReqGroups;          // TMEM accumulator slots, 64 columns each
constexpr int kReqTmemCols = kReqSlots * 64 <= 256 ? 256 : 512;  // allocation: a power of two
static_assert(kReqSlots * 64 <= 512, "TMEM holds 512 columns");
// warp 0 TMA, warp 1 MMA/TMEM, then the epilogue groups, then a second MMA warp: the two issuers take
// alternate items, so one item's r/16 MMAs and commit overlap the other's (r=128 launch 41.9 -> 37.4 us).
constexpr int kReqMmaWarp2 = 2 + 4 * kReqGroups;
constexpr int kReqThreads = 64 + 128 * kReqGroups + 32;
constexpr int kReqEpiThreads = 128 * kReqGroups;
constexpr int kReqMaxStages = 12;
constexpr int kReqSmemLimit = 232448;              // 227 KB of dynamic shared memory per CTA
constexpr int kReqBarBytes = 1536;                 // mbarriers and flags (512 B), then the problem table

struct ReqProblem {
  __half* scale;
  float s;
  int n, k, r, rp, nbp, npanel, rb, item0, row0;  // rp: r rounded to 16; item0/row0: first item/row of the problem
};

struct ReqBatch {
  CUtensorMap tm_w[kReqMaxProblems];
  CUtensorMap tm_a[kReqMaxProblems];
  CUtensorMap tm_b[kReqMaxProblems];
  CUtensorMap tm_q[kReqMaxProblems];
  ReqProblem p[kReqMaxProblems];
  int count;
  int total_items;
  int* sync;           // [0] grid-barrier arrivals (reset by the last arrival), [1] barrier generation
  unsigned* rowmax;    // [cap_rows][2] |W'| maxima as float bits (non-negative floats order as
                       // unsigned integers, NaN above +inf), two sets chosen by the generation's
                       // parity: a call uses one and clears the other for the next call
  int cap_rows;        // rows the workspace holds
  int b_bytes;         // one B buffer (nbp_max * 16 KB)
  int stage_bytes;     // 16 KB W panel + rp_max*128 B A panel, rounded to 1 KB
  int stages;
  int off_ring, off_q, off_bar;
};

enum ReqWaitSite : int {
  kSiteReqB = 211,
  kSiteReqEmpty = 212,
  kSiteReqFull = 213,
  kSiteReqD = 214,
  kSiteReqDE = 215,
  kSiteReqGrid = 216,
  kSiteReqFinal = 217,
  kSiteReqBEmpty = 218,
};

// Position of an item in the batch: problem, row block, panel.  The roles walk
// their items with these, reading the problem table from shared memory (the
// kernel-parameter copy is reached through generic loads that every asm
// "memory" clobber would force to be re-issued).
struct ReqWalk {
  int pi, rb, panel;
};

__device__ __forceinline__ ReqWalk req_walk_at(const ReqProblem* sp, int count, int item) {
  int pi = 0;
  while (pi + 1 < count && sp[pi + 1].item0 <= item) ++pi;
  const int local = item - sp[pi].item0;
  const int np = sp[pi].npanel;
  ReqWalk w;
  w.pi = pi;
  w.rb = local / np;
  w.panel = local - w.rb * np;
  return w;
}

__device__ __forceinline__ void req_walk_next(ReqWalk& w, const ReqProblem* sp, int count) {
  if (w.pi >= count) return;
  if (++w.panel == sp[w.pi].npanel) {
    w.panel = 0;
    if (++w.rb == sp[w.pi].rb) {
      w.rb = 0;
      ++w.pi;
    }
  }
}

// 32 merged values of a row and their 32 codes.
struct ReqHalfRow {
  __half2 v[16];
};
struct ReqCodes {
  uint32_t w[8];
};

// Codes of a row whose scale is not a normal fp16 number: subnormal (packed
// quantiser with its clamp) or zero / inf / NaN (closed form).  Inline: as an
// out-of-line call it took a 64-byte argument through the stack and left the
// kernel with register spills (cfg2 2.6 % slower); inline, the kernel has none.
static __device__ __forceinline__ ReqCodes req_codes_rare(ReqHalfRow m, float scale, float rcp, bool fast_row) {
  ReqCodes q;
  if (fast_row) {
#pragma unroll
    for (int e = 0; e < 8; ++e) q.w[e] = quant4_f16<true>(m.v[2 * e], m.v[2 * e + 1], scale, rcp);
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) q.w[e] = quant4_special(m.v[2 * e], m.v[2 * e + 1], scale);
  }
  return q;
}

// |W'| maximum of a half2 running max as float bits, NaN if either half is NaN.
__device__ __forceinline__ unsigned req_max_bits(__half2 hm) {
  const float l = __low2float(hm), h = __high2float(hm);
  return (l != l || h != h) ? 0x7fc00000u : __float_as_uint(fmaxf(l, h));
}

static_assert(512 + kReqMaxProblems * sizeof(ReqProblem) <= kReqBarBytes, "problem table does not fit");
// mbarriers (B full/empty, accumulator full/empty, ring full/empty, final), then 24 bytes of slots
// (TMEM address, abort flag, barrier generation, trace record)
static_assert((4 + 2 * kReqSlots + 2 * kReqMaxStages + 2) * 8 + 24 <= 512, "barrier area");

__global__ void __launch_bounds__(kReqThreads, 1) lora_requant_coop_kernel(const __grid_constant__ ReqBatch batch) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // kernel-wide values in registers
  const int S = batch.stages;
  const int count = batch.count;
  const int b_bytes = batch.b_bytes;
  const int stage_bytes = batch.stage_bytes;
  const int T = batch.total_items;
  int* const gsync = batch.sync;
  unsigned* const rowmax = batch.rowmax;
  const int cap_rows = batch.cap_rows;
  uint8_t* sB = smem;                                  // 2 x b_bytes
  uint8_t* sRing = smem + batch.off_ring;              // S x stage_bytes
  uint8_t* sQ = smem + batch.off_q;                    // one 2 KB int8 staging buffer per epilogue warp
  uint64_t* bfull = reinterpret_cast<uint64_t*>(smem + batch.off_bar);  // 2
  uint64_t* bempty = bfull + 2;          // 2
  uint64_t* dfull = bempty + 2;          // kReqSlots
  uint64_t* dempty = dfull + kReqSlots;  // kReqSlots
  uint64_t* full = dempty + kReqSlots;   // S
  uint64_t* empty = full + S;            // S
  uint64_t* final_bar = empty + S;       // 2, one per MMA issuer
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(final_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* s_gen = abort_flag + 1;  // barrier generation seen at entry
  unsigned long long** trace_slot = reinterpret_cast<unsigned long long**>(tmem_slot + 4);
  ReqProblem* sp = reinterpret_cast<ReqProblem*>(smem + batch.off_bar + 512);  // problem table

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = static_cast<int>(gridDim.x);
  const int lo = static_cast<int>((static_cast<long long>(T) * blockIdx.x) / G);
  const int hi = static_cast<int>((static_cast<long long>(T) * (blockIdx.x + 1)) / G);
  const int nmine = hi - lo;    // >= 1: the host launches at most one CTA per item
  const int steps = 2 * nmine;  // pass 1 items, then pass 2 items

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bfull[b], 1);
      mbar_init(&bempty[b], 2);  // both MMA issuers release a B buffer
    }
    for (int d = 0; d < kReqSlots; ++d) {
      mbar_init(&dfull[d], 1);
      mbar_init(&dempty[d], 4);  // the 4 warps of the group that owns the slot
    }
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1 + 4);  // MMA commit + the 4 warps of the item's group
    }
    mbar_init(&final_bar[0], 1);
    mbar_init(&final_bar[1], 1);
    *abort_flag = 0;
    *s_gen = ld_acquire_gpu(&gsync[1]);  // before this CTA arrives: the same value in every CTA
    *trace_slot = trace_claim(3);
    fence_mbar_init();
  }
  if (warp == 0 && lane < count) {
    tma_prefetch_desc(&batch.tm_w[lane]);
    tma_prefetch_desc(&batch.tm_a[lane]);
    tma_prefetch_desc(&batch.tm_b[lane]);
    tma_prefetch_desc(&batch.tm_q[lane]);
  }
  if (threadIdx.x >= 64 && threadIdx.x < 64 + count) sp[threadIdx.x - 64] = batch.p[threadIdx.x - 64];
  if (warp == 1) {
    tmem_alloc(tmem_slot, kReqTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // phase stamps: 0 start, 1 first accumulator ready, 2 pass 1 done (grid-barrier arrival),
  // 3 grid barrier passed, 4 first pass-2 accumulator ready, 5 last code block stored,
  // 6 / 7 the TMA producer has issued every pass-1 / every load, 8 / 9 MMA issuer 0 reached
  // pass 2 / its MMAs completed
  unsigned long long* const trec = *trace_slot;
  if (threadIdx.x == 0) trace_stamp(trec, 0);

  // B buffer use: a new buffer whenever (problem, row block) changes along the walk
  // or pass 2 starts; the walk repeats identically in pass 2.
  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      const uint64_t keep = l2_policy_evict_last();
      const uint64_t once = l2_policy_evict_first();
      int bseq = -1;
      ReqWalk w = req_walk_at(sp, count, lo);
      int prev_pi = -1, prev_rb = -1;
      for (int it = 0; it < steps; ++it) {
        if (it == nmine) {
          w = req_walk_at(sp, count, lo);
          prev_pi = -1;  // pass 2 starts with a fresh B buffer
          trace_stamp(trec, 6);
        }
        const int pi = w.pi, rb = w.rb, panel = w.panel;
        const int nbp = sp[pi].nbp;
        const int a_bytes = sp[pi].rp * 128;
        if (pi != prev_pi || rb != prev_rb) {
          prev_pi = pi;
          prev_rb = rb;
          ++bseq;
          const int bb = bseq & 1;
          // the buffer's previous row block must be finished by the MMA
          if (!mbar_wait(&bempty[bb], ((bseq >> 1) & 1) ^ 1, abort_flag, kSiteReqBEmpty)) break;
          mbar_arrive_expect_tx(&bfull[bb], nbp * 16384);
          for (int p = 0; p < nbp; ++p)
            tma_load_2d(sB + bb * b_bytes + p * 16384, &batch.tm_b[pi], &bfull[bb], p * 64, rb * 128, keep);
        }
        const int st = it % S;
        if (!mbar_wait(&empty[st], ((it / S) & 1) ^ 1, abort_flag, kSiteReqEmpty)) break;
        uint8_t* slot = sRing + st * stage_bytes;
        mbar_arrive_expect_tx(&full[st], 16384 + a_bytes);
        tma_load_2d(slot, &batch.tm_w[pi], &full[st], panel * 64, rb * 128, it < nmine ? keep : once);
        tma_load_2d(slot + 16384, &batch.tm_a[pi], &full[st], panel * 64, 0, keep);
        req_walk_next(w, sp, count);
      }
      trace_stamp(trec, 7);
    }
  } else if (warp == 1 || warp == kReqMmaWarp2) {
    // ---------------- MMA issuers: items alternate between the two ----------------
    // Both walk every item so that they take the same B-buffer steps; each item's MMAs
    // come from one thread in one accumulator, so its sums are those of lora_merge.
    if (lane == 0) {
      const int me = warp == 1 ? 0 : 1;
      const uint32_t idesc = make_idesc_f16(128, 64, false, true);
      const uint32_t sB_u32 = smem_u32(sB);
      const uint32_t ring_u32 = smem_u32(sRing) + 16384;  // A panel of stage 0
      int bseq = -1;
      ReqWalk w = req_walk_at(sp, count, lo);
      int prev_pi = -1, prev_rb = -1;
      for (int it = 0; it < steps; ++it) {
        if (it == nmine) {
          w = req_walk_at(sp, count, lo);
          prev_pi = -1;
          if (me == 0) trace_stamp(trec, 8);
        }
        const int pi = w.pi, rb = w.rb;
        const int rp = sp[pi].rp;
        if (pi != prev_pi || rb != prev_rb) {
          if (bseq >= 0) umma_commit(&bempty[bseq & 1]);  // previous row block's MMAs release its B buffer
          prev_pi = pi;
          prev_rb = rb;
          ++bseq;
          if (!mbar_wait(&bfull[bseq & 1], (bseq >> 1) & 1, abort_flag, kSiteReqB)) break;
        }
        if ((it & 1) != me) {
          req_walk_next(w, sp, count);
          continue;
        }
        const int st = it % S;
        const int d = it % kReqSlots;
        if (!mbar_wait(&full[st], (it / S) & 1, abort_flag, kSiteReqFull) ||
            !mbar_wait(&dempty[d], ((it / kReqSlots) & 1) ^ 1, abort_flag, kSiteReqDE))
          break;
        tc_fence_after();
        const uint32_t b_base = sB_u32 + (bseq & 1) * b_bytes;
        const uint32_t a_base = ring_u32 + st * stage_bytes;
        for (int kk = 0; kk < rp / 16; ++kk) {
          const uint64_t ad = make_sdesc(b_base + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024, kLayoutSW128);
          const uint64_t bd = make_sdesc(a_base + kk * 2048, rp * 128, 1024, kLayoutSW128);
          umma_f16(tmem + d * 64, ad, bd, idesc, kk > 0 ? 1u : 0u);
        }
        umma_commit(&dfull[d]);
        umma_commit(&empty[st]);
        req_walk_next(w, sp, count);
      }
      umma_commit(&final_bar[me]);  // every issued MMA has completed before TMEM is freed
      mbar_wait(&final_bar[me], 0, nullptr, kSiteReqFinal);
      if (me == 0) trace_stamp(trec, 9);
    }
  } else {
    // ---------------- epilogue: warps 2 .. 2 + 4*kReqGroups - 1 ----------------
    const int ew = warp - 2;
    const int grp = ew >> 2;             // items it with it % kReqGroups == grp
    const int q = warp & 3;              // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;       // row of the 128-row block
    const int sw = row & 7;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(q * 32) << 16);
    uint8_t* buf = sQ + ew * 2048;       // [32 rows x 64 B] int8, 64-byte swizzle
    const int sz = (lane >> 1) & 3;      // chunk c of staging row r sits at c ^ ((r >> 1) & 3)
    const int gen = *s_gen;
    const int set = gen & 1;
    {
      // clear the other set of row maxima for the next call (nothing reads it in this one)
      const int r0 = static_cast<int>((static_cast<long long>(cap_rows) * blockIdx.x) / G);
      const int r1 = static_cast<int>((static_cast<long long>(cap_rows) * (blockIdx.x + 1)) / G);
      for (int i = r0 + static_cast<int>(threadIdx.x) - 64; i < r1; i += kReqEpiThreads) __stcg(&rowmax[2 * i + (set ^ 1)], 0u);
    }
    bool bad = false;
    for (int pass = 0; pass < 2; ++pass) {
      if (pass == 1) {
        // ---- grid barrier: every CTA's pass-1 maxima are in the workspace ----
        __threadfence();
        if (named_bar_any(1, kReqEpiThreads, bad || *abort_flag)) bad = true;
        // only the spinning thread knows the outcome: it alone votes, the OR spreads it
        bool grid_failed = false;
        if (ew == 0 && lane == 0) {
          trace_stamp(trec, 2);
          // self-resetting barrier: the last arrival clears the count and opens the next generation
          if (atomicAdd(&gsync[0], 1) == G - 1) {
            __threadfence();
            atomicAdd(&gsync[1], 1);   // open the waiters first
            atomicExch(&gsync[0], 0);  // the count is next needed by the next call
          } else {
            const long long limit = wait_limit_cycles();
            const long long t0 = clock64();
            while (ld_acquire_gpu(&gsync[1]) == gen) {
              if (clock64() - t0 > limit) {
                record_timeout(kSiteReqGrid);
                grid_failed = true;
                *abort_flag = 1;
                break;
              }
            }
          }
        }
        if (named_bar_any(1, kReqEpiThreads, grid_failed)) bad = true;
        __threadfence();
        if (ew == 0 && lane == 0) trace_stamp(trec, 3);
      }
      int cur_pi = -1, cur_rb = -1, cur_row = -1;
      __half2 hm = __float2half2_rn(0.0f);
      float scale = 0.f, rcp = 0.f, s = 0.f;
      bool fast_row = false, normal_row = false;
      int pn = 0;
      const int it0 = pass * nmine;
      const int first = it0 + ((grp - it0 % kReqGroups) + kReqGroups) % kReqGroups;
      ReqWalk w = req_walk_at(sp, count, lo + (first - it0));
      for (int it = first; it < it0 + nmine; it += kReqGroups) {
        if (bad) break;
        const int st = it % S;
        const int d = it % kReqSlots;
        const int n = w.rb * 128 + row;
        if (w.pi != cur_pi || w.rb != cur_rb) {
          if (w.pi != cur_pi) {
            s = sp[w.pi].s;
            pn = sp[w.pi].n;
          }
          const int grow = sp[w.pi].row0 + n;
          if (pass == 0) {
            // fold the finished row block's maximum into the workspace
            if (cur_row >= 0) atomicMax(&rowmax[2 * cur_row + set], req_max_bits(hm));
            hm = __float2half2_rn(0.0f);
          } else if (n < pn) {
            const float m = __uint_as_float(__ldcg(&rowmax[2 * grow + set]));
            scale = scale_from_amax<BW_DTYPE_F16>(m, m != m);
            rcp = __frcp_rn(scale);
            // finite, non-zero scale: every quotient is finite and the packed path applies
            fast_row = scale > 0.0f && scale < __int_as_float(0x7f800000) && rcp < 1.0e30f;
            normal_row = fast_row && scale >= 6.103515625e-05f;  // no clamp needed (quant4_f16<false>)
            if (w.panel == 0) sp[w.pi].scale[n] = scale_to_f16(scale);
          }
          cur_pi = w.pi;
          cur_rb = w.rb;
          cur_row = n < pn ? grow : -1;
        }
        bool ok = mbar_wait(&dfull[d], (it / kReqSlots) & 1, abort_flag, kSiteReqD) &&
                  mbar_wait(&full[st], (it / S) & 1, abort_flag, kSiteReqFull);
        ok = __all_sync(0xffffffffu, ok);  // one decision per warp before the warp-wide steps below
        if (!ok) {
          bad = true;
          break;
        }
        if ((ew & 3) == 0 && lane == 0 && it == it0) trace_stamp(trec, 1 + 3 * pass);  // the pass's first item
        tc_fence_after();
        const uint8_t* wrow = sRing + st * stage_bytes + row * 128;
        if (pass == 1) {
          if (lane == 0) tma_store_wait_read0();  // the previous store from this warp's buffer has read it
          __syncwarp();
        }
        // two 32-column halves: half the registers of a 64-column pass, so four groups fit
        // (not unrolled: a smaller loop body keeps the instruction cache and registers in reach)
#pragma unroll 1
        for (int h = 0; h < 2; ++h) {
          uint32_t acc[32];
          tmem_ld32(lane_addr + d * 64 + h * 32, acc);
          uint4 wv[4];
#pragma unroll
          for (int c = 0; c < 4; ++c) wv[c] = *reinterpret_cast<const uint4*>(wrow + (((4 * h + c) ^ sw) << 4));
          tmem_ld_wait();
          if (h == 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
              mbar_arrive(&dempty[d]);
              mbar_arrive(&empty[st]);  // this warp is done with the accumulator slot and the stage
            }
          }
          __half2 merged[16];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint32_t* w32 = reinterpret_cast<const uint32_t*>(&wv[c]);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 p = __fmul2_rn(make_float2(__uint_as_float(acc[8 * c + 2 * e]),
                                                      __uint_as_float(acc[8 * c + 2 * e + 1])),
                                          make_float2(s, s));
              merged[4 * c + e] = __hadd2(*reinterpret_cast<const __half2*>(&w32[e]), __float22half2_rn(p));
            }
          }
          if (pass == 0) {
#pragma unroll
            for (int e = 0; e < 16; ++e) hm = __hmax2_nan(hm, __habs2(merged[e]));
            continue;
          }
          ReqCodes qw;
          if (normal_row) {
#pragma unroll
            for (int e = 0; e < 8; ++e) qw.w[e] = quant4_f16<false>(merged[2 * e], merged[2 * e + 1], scale, rcp);
          } else {
            qw = req_codes_rare(*reinterpret_cast<const ReqHalfRow*>(merged), scale, rcp, fast_row);
          }
#pragma unroll
          for (int c = 0; c < 2; ++c)
            *reinterpret_cast<uint4*>(buf + lane * 64 + (((2 * h + c) ^ sz) << 4)) =
                make_uint4(qw.w[4 * c], qw.w[4 * c + 1], qw.w[4 * c + 2], qw.w[4 * c + 3]);
        }
        if (pass == 1) {
          fence_proxy_async_smem();
          __syncwarp();
          const int y0 = w.rb * 128 + q * 32;
          if (lane == 0 && y0 < pn) {
            tma_store_2d(&batch.tm_q[w.pi], buf, w.panel * 64, y0);
            tma_store_commit();
          }
        }
#pragma unroll
        for (int j = 0; j < kReqGroups; ++j) req_walk_next(w, sp, count);
      }
      if (pass == 0 && !bad && cur_row >= 0) atomicMax(&rowmax[2 * cur_row + set], req_max_bits(hm));
    }
    if (lane == 0) tma_store_wait0();
    named_bar_sync(1, kReqEpiThreads);
    if (ew == 0 && lane == 0) trace_stamp(trec, 5);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kReqTmemCols);
  }
}

// ---------------------------------------------------------------------------
// CUDA-core kernels: add_delta_ and the fallbacks for shapes TMA cannot address
// ---------------------------------------------------------------------------
__global__ void add_delta_kernel(__half* __restrict__ w, const __half* __restrict__ d, int64_t numel, int vec) {
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  if (vec) {
    const int64_t nv = numel / 8;
    uint4* wv = reinterpret_cast<uint4*>(w);
    const uint4* dv = reinterpret_cast<const uint4*>(d);
    for (int64_t i = tid; i < nv; i += stride) {
      uint4 a = wv[i];
      const uint4 b = __ldcs(dv + i);
      uint32_t* pa = reinterpret_cast<uint32_t*>(&a);
      const uint32_t* pb = reinterpret_cast<const uint32_t*>(&b);
#pragma unroll
      for (int e = 0; e < 4; ++e)
        pa[e] = pack_h2(__float2half_rn(h2f_lo(pa[e]) + h2f_lo(pb[e])), __float2half_rn(h2f_hi(pa[e]) + h2f_hi(pb[e])));
      wv[i] = a;
    }
    for (int64_t i = nv * 8 + tid; i < numel; i += stride)
      w[i] = __float2half_rn(__half2float(w[i]) + __half2float(d[i]));
  } else {
    for (int64_t i = tid; i < numel; i += stride) w[i] = __float2half_rn(__half2float(w[i]) + __half2float(d[i]));
  }
}

// delta / merge with the reference kernels' own j-ordered fp32 accumulation.
// mode 0: out = delta; mode 1: out = fp16(W + delta).
__global__ void lora_simt_kernel(const __half* __restrict__ A, const __half* __restrict__ B, const __half* __restrict__ W,
                                 int64_t ldw, __half* __restrict__ out, int64_t ldo, int N, int K, int r, float s,
                                 int mode) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  const int n = blockIdx.y;
  if (k >= K || n >= N) return;
  float acc = 0.f;
  for (int j = 0; j < r; ++j)
    acc = fmaf(__half2float(B[static_cast<int64_t>(n) * r + j]), __half2float(A[static_cast<int64_t>(j) * K + k]), acc);
  __half d = __float2half_rn(acc * s);
  if (mode == 1) d = __float2half_rn(__half2float(W[static_cast<int64_t>(n) * ldw + k]) + __half2float(d));
  out[static_cast<int64_t>(n) * ldo + k] = d;
}

// Reference-order delta / merge on the CUDA cores (the `exact` entry points): every output is the
// reference kernels' own j-ordered fp32 accumulation, acc = fmaf(B[n,j], A[j,k], acc) for
// j = 0 .. r-1, rounded as they round it (lora_ops.cu:16-27, :32-38), so delta, the merged weight
// and its requantisation equal the reference pipeline bit for bit.  A thread computes 8 rows x 4
// columns; the block's 32 rows of B sit in shared memory as fp32, transposed ([j][row], a padded
// row of 36 so a thread's 8 values of one j are two 16-byte reads shared by its warp), and A is
// read 4 columns at a time.
constexpr int kExactRows = 32;
constexpr int kExactLd = kExactRows + 4;  // padded [j] stride of the transposed B rows
constexpr int kExactMaxR = 1024;          // 144 KB of B in shared memory

template <int MODE, bool VEC>
__global__ void __launch_bounds__(128) lora_exact_kernel(const __half* __restrict__ A, const __half* __restrict__ B,
                                                         const __half* W, int64_t ldw, __half* out, int64_t ldo, int N,
                                                         int K, int r, float s) {
  extern __shared__ float4 sB4[];  // [r][kExactLd / 4]
  float* sB = reinterpret_cast<float*>(sB4);
  const int n0 = blockIdx.y * kExactRows;
  for (int i = threadIdx.x; i < kExactRows * r; i += blockDim.x) {
    const int j = i / kExactRows, rr = i - j * kExactRows;
    sB[j * kExactLd + rr] = n0 + rr < N ? __half2float(B[static_cast<int64_t>(n0 + rr) * r + j]) : 0.f;
  }
  __syncthreads();
  const int cg = threadIdx.x & 31, rg = threadIdx.x >> 5;  // rows rg*8 .. rg*8+7 of the block
  const int k0 = blockIdx.x * 128 + cg * 4;
  if (k0 >= K) return;
  float acc[8][4];
#pragma unroll
  for (int rr = 0; rr < 8; ++rr)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[rr][e] = 0.f;
  for (int j = 0; j < r; ++j) {
    float a[4];
    const __half* ap = A + static_cast<int64_t>(j) * K + k0;
    if constexpr (VEC) {
      const uint2 v = __ldg(reinterpret_cast<const uint2*>(ap));
      a[0] = h2f_lo(v.x);
      a[1] = h2f_hi(v.x);
      a[2] = h2f_lo(v.y);
      a[3] = h2f_hi(v.y);
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) a[e] = k0 + e < K ? __half2float(ap[e]) : 0.f;
    }
    const float4 b0 = sB4[(j * kExactLd + rg * 8) / 4], b1 = sB4[(j * kExactLd + rg * 8) / 4 + 1];
    const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
    for (int rr = 0; rr < 8; ++rr)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[rr][e] = fmaf(b[rr], a[e], acc[rr][e]);
  }
#pragma unroll
  for (int rr = 0; rr < 8; ++rr) {
    const int n = n0 + rg * 8 + rr;
    if (n >= N) break;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int k = k0 + e;
      if (k >= K) break;
      __half d = __float2half_rn(acc[rr][e] * s);
      if constexpr (MODE == kModeMerge)
        d = __float2half_rn(__half2float(W[static_cast<int64_t>(n) * ldw + k]) + __half2float(d));
      out[static_cast<int64_t>(n) * ldo + k] = d;
    }
  }
}

// Fused merge + requantise for layouts TMA cannot address: one block per row,
// two passes that both recompute the merged row (the reference's j-ordered
// fp32 accumulation), so no scratch memory is needed.
__global__ void __launch_bounds__(256) lora_requant_simt_kernel(const __half* __restrict__ A, const __half* __restrict__ B,
                                                                const __half* __restrict__ W, int64_t ldw,
                                                                int8_t* __restrict__ q, int64_t ldq,
                                                                __half* __restrict__ scale, int K, int r, float s) {
  __shared__ float red[8];
  __shared__ int redn[8];
  const int64_t n = blockIdx.x;
  const __half* brow = B + n * r;
  auto merged = [&](int k) {
    float acc = 0.f;
    for (int j = 0; j < r; ++j) acc = fmaf(__half2float(brow[j]), __half2float(A[static_cast<int64_t>(j) * K + k]), acc);
    const __half d = __float2half_rn(acc * s);
    return __half2float(__float2half_rn(__half2float(W[n * ldw + k]) + __half2float(d)));
  };
  float amax = 0.f;
  bool nan = false;
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    const float v = merged(k);
    nan |= (v != v);
    amax = fmaxf(amax, fabsf(v));
  }
  for (int o = 16; o > 0; o >>= 1) {
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    nan = __any_sync(0xffffffffu, nan);
  }
  if ((threadIdx.x & 31) == 0) {
    red[threadIdx.x >> 5] = amax;
    redn[threadIdx.x >> 5] = nan;
  }
  __syncthreads();
  float m = 0.f;
  bool nn = false;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) {
    m = fmaxf(m, red[i]);
    nn |= redn[i] != 0;
  }
  const float sc = scale_from_amax<BW_DTYPE_F16>(m, nn);
  if (threadIdx.x == 0) scale[n] = scale_to_f16(sc);
  for (int k = threadIdx.x; k < K; k += blockDim.x) q[n * ldq + k] = quant_one<BW_DTYPE_F16>(merged(k), sc);
}

// ---------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------
static bool lora_tc_ok(const void* a, const void* b, int64_t k, int64_t r) {
  const auto al16 = [](const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  return al16(a) && al16(b) && r >= 1 && r <= kLoraMaxR && r % 8 == 0 && k % 8 == 0;
}

template <int MODE>
static int launch_lora_stream(const CUtensorMap& tb, const CUtensorMap& ta, const CUtensorMap& tw,
                              const CUtensorMap& to, int N, int K, int r, float s, cudaStream_t st) {
  const LoraStreamSmem L(r, MODE);
  static std::once_flag once[64];
  static cudaError_t err[64];
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 63], [&] {
    // every rank's layout fits in the planning budget plus barriers and alignment slack
    err[dev & 63] = cudaFuncSetAttribute(lora_stream_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kLsSmemBudget + 256 + 1024);
  });
  if (int rc = check_cuda(err[dev & 63], "cudaFuncSetAttribute(lora_stream_kernel)")) return rc;
  const long long tiles = static_cast<long long>((N + 127) / 128) * ((K + 127) / 128);
  const int grid = static_cast<int>(tiles < num_sms() ? tiles : num_sms());
  lora_stream_kernel<MODE><<<grid, kLsThreads, L.total, st>>>(tb, ta, tw, to, N, K, r, s);
  return check_launch("lora_stream_kernel");
}

static int lora_maps(CUtensorMap* tb, CUtensorMap* ta, const void* a, const void* b, int64_t n, int64_t k, int64_t r) {
  const int rp = static_cast<int>((r + 15) / 16 * 16);
  if (int s = make_tmap_2d(tb, b, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, n, r, r * 2, 128, 64, CU_TENSOR_MAP_SWIZZLE_128B))
    return s;
  return make_tmap_2d(ta, a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, r, k, k * 2, rp, 64, CU_TENSOR_MAP_SWIZZLE_128B);
}

static int check_lora_args(const char* op, const void* a, const void* b, int64_t n, int64_t k, int64_t r) {
  if (n < 0 || k < 0 || r < 1) return fail(BW_ERR_INVALID_ARGUMENT, "%s: need n, k >= 0 and r >= 1", op);
  if (n > (1LL << 30) || k > (1LL << 30) || r > (1LL << 20))
    return fail(BW_ERR_INVALID_ARGUMENT, "%s: dimension too large", op);
  if ((n > 0 && k > 0) && (!a || !b)) return fail(BW_ERR_INVALID_ARGUMENT, "%s: null pointer", op);
  return BW_OK;
}

// ---- grouped cooperative requant: host side ----
static bool req_tc_eligible(const bw_lora_requant_problem& P) {
  const auto al16 = [](const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  return lora_tc_ok(P.a, P.b, P.k, P.r) && al16(P.w) && al16(P.q) && (P.ldw * 2) % 16 == 0 && P.ldq % 16 == 0 &&
         P.n >= 1 && P.k >= 1;
}

// Items (128-row x 64-column panels) of one problem.
static int64_t req_items(const bw_lora_requant_problem& P) { return ((P.n + 127) / 128) * ((P.k + 63) / 64); }

// Barrier count and generation, then two words per row of the launch.
static size_t req_workspace_bytes(int64_t rows) { return 256 + static_cast<size_t>(rows) * 2 * sizeof(unsigned); }

struct ReqPlan {
  int smem = 0, stages = 0;
  int b_bytes = 0, stage_bytes = 0, off_ring = 0, off_q = 0, off_bar = 0;
};

// Shared memory: 2 B buffers, as many ring stages as fit, int8 staging, barriers + problem table.
static ReqPlan req_plan(int rp_max) {
  ReqPlan pl;
  const int nbp_max = (rp_max + 63) / 64;
  pl.b_bytes = nbp_max * 16384;
  pl.stage_bytes = 16384 + (rp_max * 128 + 1023) / 1024 * 1024;
  pl.off_ring = 2 * pl.b_bytes;
  const int staging = 4 * kReqGroups * 2048;
  const int fixed = pl.off_ring + staging + kReqBarBytes + 1024;
  pl.stages = std::min(kReqMaxStages, (kReqSmemLimit - fixed) / pl.stage_bytes);
  pl.off_q = pl.off_ring + pl.stages * pl.stage_bytes;
  pl.off_bar = pl.off_q + staging;
  pl.smem = pl.off_bar + kReqBarBytes + 1024;
  return pl;
}

static int launch_req_coop(const bw_lora_requant_problem* probs, const int* idx, int count, void* workspace,
                           size_t ws_bytes, cudaStream_t st) {
  ReqBatch b;
  memset(&b, 0, sizeof(b));
  b.count = count;
  int rp_max = 16;
  int64_t items = 0, rows = 0;
  for (int j = 0; j < count; ++j) {
    const bw_lora_requant_problem& P = probs[idx[j]];
    ReqProblem& R = b.p[j];
    R.scale = static_cast<__half*>(P.scale);
    R.s = P.scaling;
    R.n = static_cast<int>(P.n);
    R.k = static_cast<int>(P.k);
    R.r = static_cast<int>(P.r);
    R.rp = (R.r + 15) / 16 * 16;
    R.nbp = (R.rp + 63) / 64;
    R.npanel = (R.k + 63) / 64;
    R.rb = (R.n + 127) / 128;
    R.item0 = static_cast<int>(items);
    R.row0 = static_cast<int>(rows);
    items += req_items(P);
    rows += P.n;
    rp_max = std::max(rp_max, R.rp);
    if (int e = make_tmap_2d(&b.tm_w[j], P.w, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, P.n, P.k, P.ldw * 2, 128, 64,
                             CU_TENSOR_MAP_SWIZZLE_128B))
      return e;
    if (int e = make_tmap_2d(&b.tm_a[j], P.a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, P.r, P.k, P.k * 2, R.rp, 64,
                             CU_TENSOR_MAP_SWIZZLE_128B))
      return e;
    if (int e = make_tmap_2d(&b.tm_b[j], P.b, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, P.n, P.r, P.r * 2, 128, 64,
                             CU_TENSOR_MAP_SWIZZLE_128B))
      return e;
    if (int e = make_tmap_2d(&b.tm_q[j], P.q, CU_TENSOR_MAP_DATA_TYPE_UINT8, P.n, P.k, P.ldq, 32, 64,
                             CU_TENSOR_MAP_SWIZZLE_64B))
      return e;
  }
  if (items > (1LL << 30) || rows > (1LL << 30))
    return fail(BW_ERR_INVALID_ARGUMENT, "lora_merge_requant: problem too large");
  const size_t need = req_workspace_bytes(rows);
  if (workspace == nullptr || ws_bytes < need || reinterpret_cast<uintptr_t>(workspace) % 256 != 0)
    return fail(BW_ERR_WORKSPACE, "lora_merge_requant: workspace of %zu bytes (256-byte aligned) required, %zu given",
                need, ws_bytes);
  b.total_items = static_cast<int>(items);
  b.cap_rows = static_cast<int>(std::min<size_t>((ws_bytes - 256) / (2 * sizeof(unsigned)), size_t(1) << 30));
  b.sync = static_cast<int*>(workspace);
  b.rowmax = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(workspace) + 256);
  const ReqPlan pl = req_plan(rp_max);
  if (pl.stages < 2) return fail(BW_ERR_UNSUPPORTED, "lora_merge_requant: shared memory holds %d stages", pl.stages);
  b.b_bytes = pl.b_bytes;
  b.stage_bytes = pl.stage_bytes;
  b.stages = pl.stages;
  b.off_ring = pl.off_ring;
  b.off_q = pl.off_q;
  b.off_bar = pl.off_bar;
  int per_sm = 0;
  if (int e = check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, lora_requant_coop_kernel, kReqThreads,
                                                                      pl.smem),
                         "cudaOccupancyMaxActiveBlocksPerMultiprocessor(lora_requant_coop_kernel)"))
    return e;
  if (per_sm < 1) return fail(BW_ERR_UNSUPPORTED, "lora_merge_requant: kernel does not fit on an SM");
  // one CTA per SM (the shared memory plan allows no more), never more CTAs than items
  const int grid = static_cast<int>(std::min<int64_t>(items, num_sms()));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kReqThreads);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs co-resident: the grid barrier cannot deadlock
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return check_cuda(cudaLaunchKernelEx(&cfg, lora_requant_coop_kernel, b),
                    "cudaLaunchKernelEx(lora_requant_coop_kernel)");
}

// Kernel attributes, once per device (dynamic shared memory above 48 KB).
static int req_setup() {
  static std::once_flag once[64];
  static cudaError_t err[64];
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 63], [&] {
    err[dev & 63] =
        cudaFuncSetAttribute(lora_requant_coop_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kReqSmemLimit);
  });
  return check_cuda(err[dev & 63], "cudaFuncSetAttribute(lora_requant_coop_kernel)");
}

}  // namespace bw

extern "C" int bw_add_delta(void* w, const void* delta, int64_t numel, void* stream) {
  using namespace bw;
  if (numel < 0) return fail(BW_ERR_INVALID_ARGUMENT, "add_delta_: negative numel");
  if (numel == 0) return BW_OK;
  if (!w || !delta) return fail(BW_ERR_INVALID_ARGUMENT, "add_delta_: null pointer");
  if (int s = require_sm100()) return s;
  const int vec = (reinterpret_cast<uintptr_t>(w) % 16 == 0) && (reinterpret_cast<uintptr_t>(delta) % 16 == 0);
  int64_t blocks = (numel / (vec ? 8 : 1) + 255) / 256;
  const int64_t cap = static_cast<int64_t>(num_sms()) * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  add_delta_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<__half*>(w), static_cast<const __half*>(delta), numel, vec);
  return check_launch("add_delta_kernel");
}

extern "C" int bw_lora_delta(const void* a, const void* b, void* delta, int64_t n, int64_t k, int64_t r, float scaling,
                             void* stream) {
  using namespace bw;
  if (int s = check_lora_args("lora_delta", a, b, n, k, r)) return s;
  if (n == 0 || k == 0) return BW_OK;
  if (!delta) return fail(BW_ERR_INVALID_ARGUMENT, "lora_delta: null output");
  if (int s = require_sm100()) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (!lora_tc_ok(a, b, k, r) || reinterpret_cast<uintptr_t>(delta) % 16 != 0) {
    dim3 grid(static_cast<unsigned>((k + 127) / 128), static_cast<unsigned>(n));
    lora_simt_kernel<<<grid, 128, 0, st>>>(static_cast<const __half*>(a), static_cast<const __half*>(b), nullptr, 0,
                                           static_cast<__half*>(delta), k, (int)n, (int)k, (int)r, scaling, 0);
    return check_launch("lora_simt_kernel");
  }
  CUtensorMap tb, ta, to;
  if (int s = lora_maps(&tb, &ta, a, b, n, k, r)) return s;
  if (int s = make_tmap_2d(&to, delta, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, n, k, k * 2, 128, 64, CU_TENSOR_MAP_SWIZZLE_128B))
    return s;
  return launch_lora_stream<kModeDelta>(tb, ta, to, to, (int)n, (int)k, (int)r, scaling, st);
}

extern "C" int bw_lora_merge(const void* w, int64_t ldw, const void* a, const void* b, float scaling, void* w_out,
                             int64_t ldo, int64_t n, int64_t k, int64_t r, void* stream) {
  using namespace bw;
  if (int s = check_lora_args("lora_merge", a, b, n, k, r)) return s;
  if (n == 0 || k == 0) return BW_OK;
  if (!w || !w_out) return fail(BW_ERR_INVALID_ARGUMENT, "lora_merge: null pointer");
  if (ldw < k || ldo < k) return fail(BW_ERR_INVALID_ARGUMENT, "lora_merge: row stride smaller than k");
  if (int s = require_sm100()) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool aligned = reinterpret_cast<uintptr_t>(w) % 16 == 0 && reinterpret_cast<uintptr_t>(w_out) % 16 == 0 &&
                       (ldw * 2) % 16 == 0 && (ldo * 2) % 16 == 0;
  if (!lora_tc_ok(a, b, k, r) || !aligned) {
    dim3 grid(static_cast<unsigned>((k + 127) / 128), static_cast<unsigned>(n));
    lora_simt_kernel<<<grid, 128, 0, st>>>(static_cast<const __half*>(a), static_cast<const __half*>(b),
                                           static_cast<const __half*>(w), ldw, static_cast<__half*>(w_out), ldo, (int)n,
                                           (int)k, (int)r, scaling, 1);
    return check_launch("lora_simt_kernel");
  }
  CUtensorMap tb, ta, tw, to;
  if (int s = lora_maps(&tb, &ta, a, b, n, k, r)) return s;
  if (int s = make_tmap_2d(&tw, w, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, n, k, ldw * 2, 128, 64, CU_TENSOR_MAP_SWIZZLE_128B))
    return s;
  if (int s = make_tmap_2d(&to, w_out, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, n, k, ldo * 2, 128, 64, CU_TENSOR_MAP_SWIZZLE_128B))
    return s;
  return launch_lora_stream<kModeMerge>(tb, ta, tw, to, (int)n, (int)k, (int)r, scaling, st);
}

namespace bw {
static int launch_lora_exact(int mode, const void* a, const void* b, const void* w, int64_t ldw, void* out,
                             int64_t ldo, int64_t n, int64_t k, int64_t r, float s, cudaStream_t st) {
  if (r > kExactMaxR) {  // B rows beyond shared memory: the one-output-per-thread kernel (same order)
    dim3 grid(static_cast<unsigned>((k + 127) / 128), static_cast<unsigned>(n));
    lora_simt_kernel<<<grid, 128, 0, st>>>(static_cast<const __half*>(a), static_cast<const __half*>(b),
                                           static_cast<const __half*>(w), ldw, static_cast<__half*>(out), ldo, (int)n,
                                           (int)k, (int)r, s, mode);
    return check_launch("lora_simt_kernel");
  }
  const dim3 grid(static_cast<unsigned>((k + 127) / 128), static_cast<unsigned>((n + kExactRows - 1) / kExactRows));
  const size_t smem = static_cast<size_t>(kExactLd) * r * sizeof(float);
  const bool vec = k % 4 == 0 && reinterpret_cast<uintptr_t>(a) % 8 == 0;
  const __half* A = static_cast<const __half*>(a);
  const __half* B = static_cast<const __half*>(b);
  const __half* W = static_cast<const __half*>(w);
  __half* O = static_cast<__half*>(out);
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 63], [] {
    const int bytes = kExactLd * kExactMaxR * sizeof(float);
    cudaFuncSetAttribute(lora_exact_kernel<kModeDelta, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(lora_exact_kernel<kModeDelta, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(lora_exact_kernel<kModeMerge, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(lora_exact_kernel<kModeMerge, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  });
  if (mode == kModeDelta) {
    if (vec) lora_exact_kernel<kModeDelta, true><<<grid, 128, smem, st>>>(A, B, W, ldw, O, ldo, (int)n, (int)k, (int)r, s);
    else lora_exact_kernel<kModeDelta, false><<<grid, 128, smem, st>>>(A, B, W, ldw, O, ldo, (int)n, (int)k, (int)r, s);
  } else {
    if (vec) lora_exact_kernel<kModeMerge, true><<<grid, 128, smem, st>>>(A, B, W, ldw, O, ldo, (int)n, (int)k, (int)r, s);
    else lora_exact_kernel<kModeMerge, false><<<grid, 128, smem, st>>>(A, B, W, ldw, O, ldo, (int)n, (int)k, (int)r, s);
  }
  return check_launch("lora_exact_kernel");
}
}  // namespace bw

extern "C" int bw_lora_delta_exact(const void* a, const void* b, void* delta, int64_t n, int64_t k, int64_t r,
                                   float scaling, void* stream) {
  using namespace bw;
  if (int s = check_lora_args("lora_delta", a, b, n, k, r)) return s;
  if (n == 0 || k == 0) return BW_OK;
  if (!delta) return fail(BW_ERR_INVALID_ARGUMENT, "lora_delta: null output");
  if (int s = require_sm100()) return s;
  return launch_lora_exact(kModeDelta, a, b, nullptr, 0, delta, k, n, k, r, scaling, static_cast<cudaStream_t>(stream));
}

extern "C" int bw_lora_merge_exact(const void* w, int64_t ldw, const void* a, const void* b, float scaling,
                                   void* w_out, int64_t ldo, int64_t n, int64_t k, int64_t r, void* stream) {
  using namespace bw;
  if (int s = check_lora_args("lora_merge", a, b, n, k, r)) return s;
  if (n == 0 || k == 0) return BW_OK;
  if (!w || !w_out) return fail(BW_ERR_INVALID_ARGUMENT, "lora_merge: null pointer");
  if (ldw < k || ldo < k) return fail(BW_ERR_INVALID_ARGUMENT, "lora_merge: row stride smaller than k");
  if (int s = require_sm100()) return s;
  return launch_lora_exact(kModeMerge, a, b, w, ldw, w_out, ldo, n, k, r, scaling, static_cast<cudaStream_t>(stream));
}

namespace bw {
// Layouts TMA cannot address: the CUDA-core kernel, one problem at a time.
static int merge_requant_simt(const bw_lora_requant_problem& P, cudaStream_t st) {
  lora_requant_simt_kernel<<<static_cast<unsigned>(P.n), 256, 0, st>>>(
      static_cast<const __half*>(P.a), static_cast<const __half*>(P.b), static_cast<const __half*>(P.w), P.ldw, P.q,
      P.ldq, static_cast<__half*>(P.scale), (int)P.k, (int)P.r, P.scaling);
  return check_launch("lora_requant_simt_kernel");
}
}  // namespace bw

extern "C" size_t bw_lora_merge_requant_batched_workspace_size(const bw_lora_requant_problem* problems, int count) {
  using namespace bw;
  // the largest launch: up to kReqMaxProblems eligible problems at a time
  int64_t best = 0, run = 0;
  int inrun = 0;
  for (int i = 0; i < count; ++i) {
    const bw_lora_requant_problem& P = problems[i];
    if (P.n <= 0 || P.k <= 0 || !req_tc_eligible(P)) continue;
    if (inrun == kReqMaxProblems) {
      best = std::max(best, run);
      run = 0;
      inrun = 0;
    }
    run += P.n;
    ++inrun;
  }
  best = std::max(best, run);
  return best > 0 ? req_workspace_bytes(best) : 0;
}

extern "C" int bw_lora_merge_requant_batched(const bw_lora_requant_problem* problems, int count, void* workspace,
                                             size_t workspace_bytes, void* stream) {
  using namespace bw;
  if (count < 0 || (count > 0 && problems == nullptr))
    return fail(BW_ERR_INVALID_ARGUMENT, "lora_merge_requant: bad problem list");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  std::vector<int> grouped;
  for (int i = 0; i < count; ++i) {
    const bw_lora_requant_problem& P = problems[i];
    if (int e = check_lora_args("lora_merge_requant", P.a, P.b, P.n, P.k, P.r)) return e;
    if (P.k < 1) return fail(BW_ERR_INVALID_ARGUMENT, "lora_merge_requant: k must be >= 1 (problem %d)", i);
    if (P.n == 0) continue;
    if (!P.w || !P.q || !P.scale) return fail(BW_ERR_INVALID_ARGUMENT, "lora_merge_requant: null pointer (problem %d)", i);
    if (P.ldw < P.k || P.ldq < P.k)
      return fail(BW_ERR_INVALID_ARGUMENT, "lora_merge_requant: row stride smaller than k (problem %d)", i);
  }
  if (int e = require_sm100()) return e;
  if (int e = req_setup()) return e;
  for (int i = 0; i < count; ++i) {
    const bw_lora_requant_problem& P = problems[i];
    if (P.n == 0) continue;
    if (req_tc_eligible(P)) {
      grouped.push_back(i);
    } else if (int e = merge_requant_simt(P, st)) {
      return e;
    }
  }
  for (size_t j = 0; j < grouped.size(); j += kReqMaxProblems) {
    const int c = static_cast<int>(std::min<size_t>(kReqMaxProblems, grouped.size() - j));
    if (int e = launch_req_coop(problems, grouped.data() + j, c, workspace, workspace_bytes, st)) return e;
  }
  return BW_OK;
}

extern "C" size_t bw_lora_merge_requant_workspace_size(int64_t n, int64_t k, int64_t r) {
  bw_lora_requant_problem P = {};
  P.w = P.a = P.b = reinterpret_cast<const void*>(uintptr_t(256));
  P.q = reinterpret_cast<int8_t*>(uintptr_t(256));
  P.ldw = P.ldq = k;
  P.n = n;
  P.k = k;
  P.r = r;
  return bw_lora_merge_requant_batched_workspace_size(&P, 1);
}

extern "C" int bw_lora_merge_requant(const void* w, int64_t ldw, const void* a, const void* b, float scaling, int8_t* q,
                                     int64_t ldq, void* scale, int64_t n, int64_t k, int64_t r, void* workspace,
                                     size_t workspace_bytes, void* stream) {
  bw_lora_requant_problem P;
  P.w = w;
  P.ldw = ldw;
  P.a = a;
  P.b = b;
  P.scaling = scaling;
  P.q = q;
  P.ldq = ldq;
  P.scale = scale;
  P.n = n;
  P.k = k;
  P.r = r;
  return bw_lora_merge_requant_batched(&P, 1, workspace, workspace_bytes, stream);
}
