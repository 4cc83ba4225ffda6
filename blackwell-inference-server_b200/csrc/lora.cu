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
// One kernel, three epilogues.  A CTA owns a 128-row x 128-column output tile:
// TMA brings B[128 rows, r] (K-major, 128-byte swizzle; the rank dimension is
// zero-filled up to a multiple of 16), A[r, 128 cols] (MN-major, 128-byte
// swizzle: TMA writes A's natural row-major layout and the UMMA descriptor
// reads it transposed, so A is never transposed in memory) and, for the
// merge, the W tile.  One thread issues r/16 tcgen05.mma (M=128, N=128, K=16)
// into a 128-column TMEM accumulator; 128 epilogue threads (thread = row)
// read it back, round, merge, and write the result through swizzled shared
// memory and a TMA store.
//
// Requantisation needs each row's absolute maximum over all of K before any
// code can be written.  The CTAs that share a 128-row block form a thread-block
// cluster along K: pass 1 computes merged tiles and per-row partial maxima
// (nothing is written to memory), the partial maxima are pushed to every CTA of
// the cluster through distributed shared memory (bounded mbarrier wait), and
// pass 2 recomputes the merged tiles (the W re-read hits L2) and writes int8
// codes.  The merged fp16 weight never touches HBM.
#include <stdio.h>

#include <string.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "quant_math.cuh"

namespace bw {

enum LoraMode : int { kModeDelta = 0, kModeMerge = 1, kModeRequant = 2 };

enum LoraWaitSite : int {
  kSiteLoraB = 201,
  kSiteLoraTile = 202,
  kSiteLoraMma = 203,
  kSiteLoraXchg = 204,
};

constexpr int kLoraMaxCluster = 8;
constexpr int kLoraMaxR = 128;

struct LoraSmem {
  int rp;  // rank rounded up to 16
  int nbp;  // 64-wide rank panels of the B tile
  int off_b, off_a, off_w, off_q, off_red, off_bar, total;
  __host__ __device__ LoraSmem(int r, int mode) {
    rp = (r + 15) / 16 * 16;
    nbp = (rp + 63) / 64;
    off_b = 0;
    off_a = off_b + nbp * 16384;
    off_w = off_a + ((2 * rp * 128 + 1023) / 1024) * 1024;
    off_q = off_w + 32768;
    off_red = off_q + (mode == kModeRequant ? 16384 : 0);
    off_bar = off_red + (mode == kModeRequant ? kLoraMaxCluster * 128 * 4 : 0);
    total = off_bar + 128 + 1024;
  }
};

__device__ __forceinline__ float h2f_lo(uint32_t w) { return __half2float(__ushort_as_half(static_cast<unsigned short>(w & 0xFFFFu))); }
__device__ __forceinline__ float h2f_hi(uint32_t w) { return __half2float(__ushort_as_half(static_cast<unsigned short>(w >> 16))); }
__device__ __forceinline__ uint32_t pack_h2(__half a, __half b) {
  return static_cast<uint32_t>(__half_as_ushort(a)) | (static_cast<uint32_t>(__half_as_ushort(b)) << 16);
}

// Epilogue for one 128x128 tile; thread = tile row.
template <int MODE, int PASS>
__device__ __forceinline__ void lora_tile_epilogue(uint32_t taddr, uint8_t* sW, uint8_t* sQ, int row, float scaling,
                                                   float qscale, float& pmax, bool& nan) {
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
    if constexpr (MODE == kModeDelta) {
      uint32_t o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = pack_h2(d[2 * e], d[2 * e + 1]);
      *w0 = make_uint4(o[0], o[1], o[2], o[3]);
      *w1 = make_uint4(o[4], o[5], o[6], o[7]);
    } else {
      const uint4 a = *w0, b = *w1;
      const uint32_t win[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
      float wp[16];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        wp[2 * e] = __half2float(__float2half_rn(h2f_lo(win[e]) + __half2float(d[2 * e])));
        wp[2 * e + 1] = __half2float(__float2half_rn(h2f_hi(win[e]) + __half2float(d[2 * e + 1])));
      }
      if constexpr (MODE == kModeMerge) {
        uint32_t o[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = pack_h2(__float2half_rn(wp[2 * e]), __float2half_rn(wp[2 * e + 1]));
        *w0 = make_uint4(o[0], o[1], o[2], o[3]);
        *w1 = make_uint4(o[4], o[5], o[6], o[7]);
      } else if constexpr (PASS == 0) {
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          nan |= (wp[e] != wp[e]);
          pmax = fmaxf(pmax, fabsf(wp[e]));
        }
      } else {
        int8_t qv[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) qv[e] = quant_fast<BW_DTYPE_F16>(wp[e], qscale, __frcp_rn(qscale));
        *reinterpret_cast<uint4*>(sQ + row * 128 + (((c0 >> 4) ^ sw) << 4)) = *reinterpret_cast<uint4*>(qv);
      }
    }
  }
}

template <int MODE>
__global__ void __launch_bounds__(128)
    lora_tc_kernel(const __grid_constant__ CUtensorMap tm_b, const __grid_constant__ CUtensorMap tm_a,
                   const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_out,
                   __half* __restrict__ scale_out, int N, int K, int r, float scaling, int k_tiles) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const LoraSmem L(r, MODE);
  uint8_t* sB = smem + L.off_b;
  uint8_t* sA = smem + L.off_a;
  uint8_t* sW = smem + L.off_w;
  uint8_t* sQ = smem + L.off_q;
  float* xred = reinterpret_cast<float*>(smem + L.off_red);
  uint64_t* bar_b = reinterpret_cast<uint64_t*>(smem + L.off_bar);
  uint64_t* bar_t = bar_b + 1;
  uint64_t* bar_mma = bar_b + 2;
  uint64_t* bar_x = bar_b + 3;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_b + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int row = warp * 32 + lane;  // 128 threads: warp w owns TMEM lanes 32w..32w+31
  const int n0 = blockIdx.y * 128;
  const int rp = L.rp;

  int cl_rank = 0, cl_size = 1;
  if constexpr (MODE == kModeRequant) {
    cl_rank = static_cast<int>(cluster_ctarank());
    cl_size = static_cast<int>(gridDim.x);  // the cluster spans the whole x extent
  }

  if (tid == 0) {
    mbar_init(bar_b, 1);
    mbar_init(bar_t, 1);
    mbar_init(bar_mma, 1);
    mbar_init(bar_x, static_cast<uint32_t>(cl_size));
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_b);
    tma_prefetch_desc(&tm_a);
    if (MODE != kModeDelta) tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_out);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 128);
    tmem_relinquish();
  }
  tc_fence_before();
  if constexpr (MODE == kModeRequant) cluster_sync_all();  // peers' barriers are initialised
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t taddr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
  const uint32_t idesc = make_idesc_f16(128, 128, false, true);

  // tiles of this CTA: delta/merge -> exactly blockIdx.x; requant -> rank, rank + C, ...
  const int first = MODE == kModeRequant ? cl_rank : static_cast<int>(blockIdx.x);
  const int stride = MODE == kModeRequant ? cl_size : k_tiles;
  const int passes = MODE == kModeRequant ? 2 : 1;
  float pmax = 0.f;
  bool nan = false;
  float qscale = 0.f;
  int it = 0;
  bool ok = true;

  for (int pass = 0; pass < passes && ok; ++pass) {
    if (MODE == kModeRequant && pass == 1) {
      // ---- exchange the per-row partial maxima across the cluster ----
      const uint32_t slot = smem_u32(&xred[cl_rank * 128 + row]);
      const float mine = nan ? __int_as_float(0x7fc00000) : pmax;
      for (int d = 0; d < cl_size; ++d) st_shared_cluster_f32(mapa_shared(slot, d), mine);
      __syncthreads();
      if (tid == 0) {
        fence_acq_rel_cluster();
        for (int d = 0; d < cl_size; ++d) mbar_arrive_remote(mapa_shared(smem_u32(bar_x), d));
      }
      ok = mbar_wait_cluster(bar_x, 0, abort_flag, kSiteLoraXchg);
      ok = !__syncthreads_or(!ok || *abort_flag);  // one decision for the whole CTA
      if (!ok) break;
      float m = 0.f;
      bool nn = false;
      for (int d = 0; d < cl_size; ++d) {
        const float v = xred[d * 128 + row];
        nn |= (v != v);
        m = fmaxf(m, v);
      }
      qscale = scale_from_amax<BW_DTYPE_F16>(m, nn);
      if (cl_rank == 0 && n0 + row < N) scale_out[n0 + row] = __float2half_rn(qscale);
    }
    for (int kt = first; kt < k_tiles; kt += stride, ++it) {
      const int k0 = kt * 128;
      const uint32_t ph = it & 1;
      if (tid == 0) {
        if (it == 0) {
          mbar_arrive_expect_tx(bar_b, L.nbp * 16384);
          for (int p = 0; p < L.nbp; ++p) tma_load_2d(sB + p * 16384, &tm_b, bar_b, p * 64, n0, l2_policy_evict_last());
        }
        const uint32_t bytes = 2 * rp * 128 + (MODE != kModeDelta ? 32768 : 0);
        mbar_arrive_expect_tx(bar_t, bytes);
        const uint64_t pol = l2_policy_evict_last();
        tma_load_2d(sA, &tm_a, bar_t, k0, 0, pol);
        tma_load_2d(sA + rp * 128, &tm_a, bar_t, k0 + 64, 0, pol);
        if (MODE != kModeDelta) {
          const uint64_t polw = (MODE == kModeRequant && pass == 0) ? l2_policy_evict_last() : l2_policy_evict_first();
          tma_load_2d(sW, &tm_w, bar_t, k0, n0, polw);
          tma_load_2d(sW + 16384, &tm_w, bar_t, k0 + 64, n0, polw);
        }
        bool good = mbar_wait(bar_b, 0, abort_flag, kSiteLoraB) && mbar_wait(bar_t, ph, abort_flag, kSiteLoraTile);
        if (good) {
          tc_fence_after();
          const uint32_t b_base = smem_u32(sB);
          const uint32_t a_base = smem_u32(sA);
          for (int kk = 0; kk < rp / 16; ++kk) {
            const uint64_t ad = make_sdesc(b_base + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024, kLayoutSW128);
            const uint64_t bd = make_sdesc(a_base + kk * 2048, rp * 128, 1024, kLayoutSW128);
            umma_f16(tmem, ad, bd, idesc, kk > 0 ? 1u : 0u);
          }
        }
        umma_commit(bar_mma);  // always, so waiters never wait on an op that was not issued
      }
      ok = mbar_wait(bar_t, ph, abort_flag, kSiteLoraTile) && mbar_wait(bar_mma, ph, abort_flag, kSiteLoraMma);
      tc_fence_after();
      ok = !__syncthreads_or(!ok || *abort_flag);  // one decision for the whole CTA
      if (ok) {
        if (MODE == kModeRequant && pass == 0) lora_tile_epilogue<MODE, 0>(taddr, sW, sQ, row, scaling, 0.f, pmax, nan);
        else lora_tile_epilogue<MODE, 1>(taddr, sW, sQ, row, scaling, qscale, pmax, nan);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncthreads();
      if (tid == 0 && ok && !(MODE == kModeRequant && pass == 0)) {
        if (MODE == kModeRequant) {
          tma_store_2d(&tm_out, sQ, k0, n0);
        } else {
          tma_store_2d(&tm_out, sW, k0, n0);
          if (k0 + 64 < K) tma_store_2d(&tm_out, sW + 16384, k0 + 64, n0);  // never start a store past K
        }
        tma_store_commit();
        tma_store_wait_read0();
      }
      __syncthreads();
      if (!ok) break;
    }
  }
  if (tid == 0) tma_store_wait0();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
}

// ---------------------------------------------------------------------------
// Grouped, cooperative merge + requantisation.
//
// One launch covers up to kReqMaxProblems projections (e.g. every projection an
// adapter touches).  The work is cut into uniform items, one 128-row x 64-column
// panel each, numbered problem-major then row block then panel, and dealt to a
// grid of co-resident CTAs in contiguous ranges (cooperative launch).  Each CTA
// walks its range twice:
//   pass 1: TMA brings the W panel and the A[r, 64] panel (and B[128, r] when
//           the row block changes, double-buffered); tcgen05.mma (M=128, N=64,
//           K=16 x r/16) -> TMEM; 8 epilogue warps merge
//           W' = fp16(W + fp16(acc*s)) in registers (__hadd2 is the correctly
//           rounded fp16 sum = fp16(fp32(W) + fp32(delta))) and write each
//           row's |W'| maximum of the panel half to the workspace;
//   grid barrier (bounded spin on a workspace counter; every CTA is resident);
//   pass 2: the same panels again (W hits L2, ΔW recomputed on the tensor
//           core), row scale from the panel maxima, packed exact quantiser,
//           int8 stored by each warp with its own TMA store (no CTA barrier).
// The producer and MMA run ahead into pass 2 while the epilogue waits at the
// grid barrier, so the weight stream does not stall.  The merged weight never
// touches memory; the workspace holds 2 floats per row per panel + a counter.
// ---------------------------------------------------------------------------
constexpr int kReqMaxProblems = 16;
constexpr int kReqThreads = 320;  // warp 0 TMA, warp 1 MMA/TMEM, warps 2-9 epilogue
constexpr int kReqStages = 3;

struct ReqProblem {
  __half* scale;
  float s;
  int n, k, r, rp, nbp, npanel, rb, item0;  // rp: r rounded to 16; item0: first item of this problem
};

struct ReqBatch {
  CUtensorMap tm_w[kReqMaxProblems];
  CUtensorMap tm_a[kReqMaxProblems];
  CUtensorMap tm_b[kReqMaxProblems];
  CUtensorMap tm_q[kReqMaxProblems];
  ReqProblem p[kReqMaxProblems];
  int count;
  int total_items;
  float* maxima;   // [total_items][2][128]
  int* counter;    // grid barrier, zeroed before the launch
  int b_bytes;     // one B buffer (nbp_max * 16 KB)
  int stage_bytes; // 16 KB W panel + rp_max*128 B A panel, rounded to 1 KB
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

struct ReqItem {
  int pi, rb, panel;
};

__device__ __forceinline__ ReqItem req_item(const ReqBatch& bt, int item) {
  int pi = 0;
  while (pi + 1 < bt.count && bt.p[pi + 1].item0 <= item) ++pi;
  const int local = item - bt.p[pi].item0;
  ReqItem r;
  r.pi = pi;
  r.rb = local / bt.p[pi].npanel;
  r.panel = local % bt.p[pi].npanel;
  return r;
}

__global__ void __launch_bounds__(kReqThreads, 2) lora_requant_coop_kernel(const __grid_constant__ ReqBatch batch) {
  constexpr int S = kReqStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sB = smem;                                  // 2 x b_bytes
  uint8_t* sRing = smem + batch.off_ring;              // S x stage_bytes
  uint8_t* sQ = smem + batch.off_q;                    // 8 warps x 2 x 1 KB int8 staging
  uint64_t* bfull = reinterpret_cast<uint64_t*>(smem + batch.off_bar);  // 2
  uint64_t* bempty = bfull + 2;      // 2
  uint64_t* full = bempty + 2;       // S
  uint64_t* empty = full + S;        // S
  uint64_t* dfull = empty + S;       // 2
  uint64_t* dempty = dfull + 2;      // 2
  uint64_t* final_bar = dempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(final_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = static_cast<int>(gridDim.x);
  const int T = batch.total_items;
  const int lo = static_cast<int>((static_cast<long long>(T) * blockIdx.x) / G);
  const int hi = static_cast<int>((static_cast<long long>(T) * (blockIdx.x + 1)) / G);
  const int nmine = hi - lo;
  const int steps = 2 * nmine;  // pass 1 items, then pass 2 items

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bfull[b], 1);
      mbar_init(&bempty[b], 1);
      mbar_init(&dfull[b], 1);
      mbar_init(&dempty[b], 8);
    }
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1 + 8);  // MMA commit + 8 epilogue warps
    }
    mbar_init(final_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 128);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // B buffer use: a new buffer whenever (problem, row block) changes along the walk;
  // the walk repeats identically in pass 2.
  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      const uint64_t keep = l2_policy_evict_last();
      int prev_key = -1, bseq = -1;
      for (int it = 0; it < steps; ++it) {
        const int item = lo + (it % nmine);
        const ReqItem I = req_item(batch, item);
        const ReqProblem& P = batch.p[I.pi];
        const int key = item - I.panel;  // first item of the row block: identifies (problem, row block)
        if (key != prev_key || it == nmine) {
          prev_key = key;
          ++bseq;
          const int bb = bseq & 1;
          // the buffer's previous row block must be finished by the MMA
          if (!mbar_wait(&bempty[bb], ((bseq >> 1) & 1) ^ 1, abort_flag, kSiteReqBEmpty)) break;
          mbar_arrive_expect_tx(&bfull[bb], P.nbp * 16384);
          for (int p = 0; p < P.nbp; ++p)
            tma_load_2d(sB + bb * batch.b_bytes + p * 16384, &batch.tm_b[I.pi], &bfull[bb], p * 64, I.rb * 128, keep);
        }
        const int st = it % S;
        if (!mbar_wait(&empty[st], ((it / S) & 1) ^ 1, abort_flag, kSiteReqEmpty)) break;
        uint8_t* slot = sRing + st * batch.stage_bytes;
        mbar_arrive_expect_tx(&full[st], 16384 + P.rp * 128);
        const int kx = I.panel * 64;
        tma_load_2d(slot, &batch.tm_w[I.pi], &full[st], kx, I.rb * 128, it < nmine ? keep : l2_policy_evict_first());
        tma_load_2d(slot + 16384, &batch.tm_a[I.pi], &full[st], kx, 0, keep);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = make_idesc_f16(128, 64, false, true);
      int prev_key = -1, bseq = -1;
      bool ok = true;
      for (int it = 0; it < steps && ok; ++it) {
        const int item = lo + (it % nmine);
        const ReqItem I = req_item(batch, item);
        const ReqProblem& P = batch.p[I.pi];
        const int key = item - I.panel;
        if (key != prev_key || it == nmine) {
          if (bseq >= 0) umma_commit(&bempty[bseq & 1]);  // previous row block's MMAs release its B buffer
          prev_key = key;
          ++bseq;
          if (!mbar_wait(&bfull[bseq & 1], (bseq >> 1) & 1, abort_flag, kSiteReqB)) break;
        }
        const int st = it % S;
        const int d = it & 1;
        if (!mbar_wait(&full[st], (it / S) & 1, abort_flag, kSiteReqFull) ||
            !mbar_wait(&dempty[d], ((it >> 1) & 1) ^ 1, abort_flag, kSiteReqDE)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t b_base = smem_u32(sB + (bseq & 1) * batch.b_bytes);
        const uint32_t a_base = smem_u32(sRing + st * batch.stage_bytes + 16384);
        for (int kk = 0; kk < P.rp / 16; ++kk) {
          const uint64_t ad = make_sdesc(b_base + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024, kLayoutSW128);
          const uint64_t bd = make_sdesc(a_base + kk * 2048, P.rp * 128, 1024, kLayoutSW128);
          umma_f16(tmem + d * 64, ad, bd, idesc, kk > 0 ? 1u : 0u);
        }
        umma_commit(&dfull[d]);
        umma_commit(&empty[st]);
      }
      umma_commit(final_bar);  // every issued MMA has completed before TMEM is freed
      mbar_wait(final_bar, 0, nullptr, kSiteReqFinal);
    }
  } else {
    // ---------------- epilogue warps 2-9 ----------------
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;  // columns [32*half, 32*half + 32) of each panel
    const int row = q * 32 + lane;
    const int sw = row & 7;
    const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16) + half * 32;
    uint8_t* stage_q = sQ + (warp - 2) * 2048;  // this warp's two 1 KB staging buffers
    bool bad = false;
    int qbuf = 0;
    int cur_key = -1;
    float scale = 0.f, rcp = 0.f;
    bool fast_row = false;
    for (int it = 0; it < steps; ++it) {
      if (it == nmine) {
        // ---- grid barrier: every CTA's pass-1 maxima are in the workspace ----
        __threadfence();
        if (named_bar_any(1, 256, bad || *abort_flag)) bad = true;
        // only the spinning thread knows the outcome: it alone votes, the OR spreads it
        bool grid_failed = false;
        if (warp == 2 && lane == 0) {
          atomicAdd(batch.counter, 1);
          const long long limit = static_cast<long long>(BW_WAIT_LIMIT_NS) * 5 / 2;
          const long long t0 = clock64();
          while (atomicAdd(batch.counter, 0) < G) {
            if (clock64() - t0 > limit) {
              record_timeout(kSiteReqGrid);
              grid_failed = true;
              *abort_flag = 1;
              break;
            }
            __nanosleep(64);
          }
        }
        if (named_bar_any(1, 256, grid_failed)) bad = true;
        __threadfence();
      }
      if (bad) continue;  // keep walking so every barrier above is reached the same number of times
      const int item = lo + (it % nmine);
      const ReqItem I = req_item(batch, item);
      const ReqProblem& P = batch.p[I.pi];
      const bool pass2 = it >= nmine;
      const int st = it % S;
      const int d = it & 1;
      const bool ok = mbar_wait(&dfull[d], (it >> 1) & 1, abort_flag, kSiteReqD) &&
                      mbar_wait(&full[st], (it / S) & 1, abort_flag, kSiteReqFull);
      if (!ok) {
        bad = true;
        continue;
      }
      tc_fence_after();
      uint32_t acc[32];
      tmem_ld32(taddr + d * 64, acc);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dempty[d]);
      const uint8_t* wrow = sRing + st * batch.stage_bytes + row * 128;
      uint4 wv[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) wv[c] = *reinterpret_cast<const uint4*>(wrow + (((4 * half + c) ^ sw) << 4));
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);  // this warp is done with the stage
      __half2 merged[16];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint32_t* w32 = reinterpret_cast<const uint32_t*>(&wv[c]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const __half2 dl = __floats2half2_rn(__uint_as_float(acc[8 * c + 2 * e]) * P.s,
                                               __uint_as_float(acc[8 * c + 2 * e + 1]) * P.s);
          merged[4 * c + e] = __hadd2(*reinterpret_cast<const __half2*>(&w32[e]), dl);
        }
      }
      const int n = I.rb * 128 + row;
      if (!pass2) {
        __half2 hm = __float2half2_rn(0.0f);
#pragma unroll
        for (int e = 0; e < 16; ++e) hm = __hmax2_nan(hm, __habs2(merged[e]));
        const float l = __low2float(hm), h = __high2float(hm);
        batch.maxima[(static_cast<size_t>(item) * 2 + half) * 128 + row] =
            (l != l || h != h) ? __int_as_float(0x7fc00000) : fmaxf(l, h);
      } else {
        const int key = item - I.panel;
        if (key != cur_key) {
          // scale of this row from every panel's maxima of the row block
          cur_key = key;
          float m = 0.f;
          bool nn = false;
          const float* mx = batch.maxima + static_cast<size_t>(key) * 2 * 128 + row;
          for (int j = 0; j < 2 * P.npanel; ++j) {
            const float v = __ldcg(mx + j * 128);
            nn |= (v != v);
            m = fmaxf(m, v);
          }
          scale = scale_from_amax<BW_DTYPE_F16>(m, nn);
          rcp = __frcp_rn(scale);
          fast_row = scale > 0.0f && rcp < 1.0e30f;  // finite, non-zero scale: every quotient is finite
        }
        if (I.panel == 0 && half == 0 && n < P.n) P.scale[n] = __float2half_rn(scale);
        uint32_t qw[8];
        if (fast_row) {
#pragma unroll
          for (int e = 0; e < 8; ++e) qw[e] = quant4_f16(merged[2 * e], merged[2 * e + 1], scale, rcp);
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            uint32_t v = 0;
#pragma unroll
            for (int t = 0; t < 2; ++t) {
              const __half2 hh = merged[2 * e + t];
              v |= static_cast<uint32_t>(static_cast<uint8_t>(quant_one<BW_DTYPE_F16>(__low2float(hh), scale)))
                   << (16 * t);
              v |= static_cast<uint32_t>(static_cast<uint8_t>(quant_one<BW_DTYPE_F16>(__high2float(hh), scale)))
                   << (16 * t + 8);
            }
            qw[e] = v;
          }
        }
        // this warp's [32 rows x 32 B] int8 block, 32-byte swizzle: chunk c of row r at c ^ ((r >> 2) & 1)
        uint8_t* buf = stage_q + qbuf * 1024;
        if (lane == 0) tma_store_wait_read1();  // the store issued from this buffer two panels ago has read it
        __syncwarp();
        const int sz = (lane >> 2) & 1;
#pragma unroll
        for (int c = 0; c < 2; ++c)
          *reinterpret_cast<uint4*>(buf + lane * 32 + ((c ^ sz) << 4)) =
              make_uint4(qw[4 * c], qw[4 * c + 1], qw[4 * c + 2], qw[4 * c + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        const int x0 = I.panel * 64 + 32 * half;
        const int y0 = I.rb * 128 + q * 32;
        if (lane == 0 && x0 < P.k && y0 < P.n) {
          tma_store_2d(&batch.tm_q[I.pi], buf, x0, y0);
          tma_store_commit();
        }
        qbuf ^= 1;
      }
    }
    if (nmine == 0) {
      // a CTA without items still takes part in the grid barrier
      __threadfence();
      named_bar_sync(1, 256);
      if (warp == 2 && lane == 0) atomicAdd(batch.counter, 1);
    }
    if (lane == 0) tma_store_wait0();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 128);
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
  if (threadIdx.x == 0) scale[n] = __float2half_rn(sc);
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
static int launch_lora_tc(const CUtensorMap& tb, const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& to,
                          __half* scale_out, int N, int K, int r, float s, cudaStream_t st) {
  const LoraSmem L(r, MODE);
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t e = cudaSuccess;
  std::call_once(once[dev & 63], [&] {
    e = cudaFuncSetAttribute(lora_tc_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e == cudaSuccess && MODE == kModeRequant)
      e = cudaFuncSetAttribute(lora_tc_kernel<MODE>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  });
  if (int rc = check_cuda(e, "cudaFuncSetAttribute(lora_tc_kernel)")) return rc;
  const int k_tiles = (K + 127) / 128;
  const int n_blocks = (N + 127) / 128;
  if (MODE != kModeRequant) {
    dim3 grid(k_tiles, n_blocks);
    lora_tc_kernel<MODE><<<grid, 128, L.total, st>>>(tb, ta, tw, to, scale_out, N, K, r, s, k_tiles);
    return check_launch("lora_tc_kernel");
  }
  const int cl = k_tiles < kLoraMaxCluster ? k_tiles : kLoraMaxCluster;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cl, n_blocks);
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cl;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, lora_tc_kernel<MODE>, tb, ta, tw, to, scale_out, N, K, r, s, k_tiles);
  return check_cuda(e, "cudaLaunchKernelEx(lora_tc_kernel requant)");
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

// ---- grouped cluster requant: host side ----
static bool req_cluster_eligible(const bw_lora_requant_problem& P) {
  const auto al16 = [](const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  return lora_tc_ok(P.a, P.b, P.k, P.r) && al16(P.w) && al16(P.q) && (P.ldw * 2) % 16 == 0 && P.ldq % 16 == 0 &&
         P.n >= 1 && P.k >= 1;
}

// Items (128-row x 64-column panels) of one problem.
static int64_t req_items(const bw_lora_requant_problem& P) { return ((P.n + 127) / 128) * ((P.k + 63) / 64); }

static size_t req_workspace_bytes(int64_t items) { return 256 + static_cast<size_t>(items) * 2 * 128 * sizeof(float); }

struct ReqPlan {
  int smem = 0;
  int b_bytes = 0, stage_bytes = 0, off_ring = 0, off_q = 0, off_bar = 0;
};

static ReqPlan req_plan(int rp_max) {
  ReqPlan pl;
  const int nbp_max = (rp_max + 63) / 64;
  pl.b_bytes = nbp_max * 16384;
  pl.stage_bytes = 16384 + (rp_max * 128 + 1023) / 1024 * 1024;
  pl.off_ring = 2 * pl.b_bytes;
  pl.off_q = pl.off_ring + kReqStages * pl.stage_bytes;
  pl.off_bar = pl.off_q + 8 * 2048;
  pl.smem = pl.off_bar + 256 + 1024;
  return pl;
}

static int launch_req_coop(const bw_lora_requant_problem* probs, const int* idx, int count, void* workspace,
                           size_t ws_bytes, cudaStream_t st) {
  ReqBatch b;
  memset(&b, 0, sizeof(b));
  b.count = count;
  int rp_max = 16;
  int64_t items = 0;
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
    items += req_items(P);
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
    if (int e = make_tmap_2d(&b.tm_q[j], P.q, CU_TENSOR_MAP_DATA_TYPE_UINT8, P.n, P.k, P.ldq, 32, 32,
                             CU_TENSOR_MAP_SWIZZLE_32B))
      return e;
  }
  if (items > (1LL << 30)) return fail(BW_ERR_INVALID_ARGUMENT, "lora_merge_requant: problem too large");
  const size_t need = req_workspace_bytes(items);
  if (workspace == nullptr || ws_bytes < need || reinterpret_cast<uintptr_t>(workspace) % 256 != 0)
    return fail(BW_ERR_WORKSPACE, "lora_merge_requant: workspace of %zu bytes (256-byte aligned) required, %zu given",
                need, ws_bytes);
  b.total_items = static_cast<int>(items);
  b.counter = static_cast<int*>(workspace);
  b.maxima = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + 256);
  const ReqPlan pl = req_plan(rp_max);
  b.b_bytes = pl.b_bytes;
  b.stage_bytes = pl.stage_bytes;
  b.off_ring = pl.off_ring;
  b.off_q = pl.off_q;
  b.off_bar = pl.off_bar;
  if (pl.smem > 232448) return fail(BW_ERR_UNSUPPORTED, "lora_merge_requant: shared memory plan of %d bytes", pl.smem);
  int per_sm = 0;
  if (int e = check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, lora_requant_coop_kernel, kReqThreads,
                                                                      pl.smem),
                         "cudaOccupancyMaxActiveBlocksPerMultiprocessor(lora_requant_coop_kernel)"))
    return e;
  if (per_sm < 1) return fail(BW_ERR_UNSUPPORTED, "lora_merge_requant: kernel does not fit on an SM");
  const int grid = static_cast<int>(std::min<int64_t>(items, static_cast<int64_t>(per_sm) * num_sms()));
  if (int e = check_cuda(cudaMemsetAsync(b.counter, 0, sizeof(int), st), "clear requant grid counter")) return e;
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
    err[dev & 63] = cudaFuncSetAttribute(lora_requant_coop_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         232448 - 2048);
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
  return launch_lora_tc<kModeDelta>(tb, ta, to, to, nullptr, (int)n, (int)k, (int)r, scaling, st);
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
  return launch_lora_tc<kModeMerge>(tb, ta, tw, to, nullptr, (int)n, (int)k, (int)r, scaling, st);
}

namespace bw {
// One problem through the two-pass cluster kernel (any K) or, for layouts TMA
// cannot address, the CUDA-core kernel.
static int merge_requant_single(const bw_lora_requant_problem& Pr, cudaStream_t st) {
  const void* w = Pr.w; const int64_t ldw = Pr.ldw; const void* a = Pr.a; const void* b = Pr.b;
  const float scaling = Pr.scaling; int8_t* q = Pr.q; const int64_t ldq = Pr.ldq; void* scale = Pr.scale;
  const int64_t n = Pr.n, k = Pr.k, r = Pr.r;
  const bool aligned = reinterpret_cast<uintptr_t>(w) % 16 == 0 && reinterpret_cast<uintptr_t>(q) % 16 == 0 &&
                       (ldw * 2) % 16 == 0 && ldq % 16 == 0;
  if (!lora_tc_ok(a, b, k, r) || !aligned) {
    lora_requant_simt_kernel<<<static_cast<unsigned>(n), 256, 0, st>>>(
        static_cast<const __half*>(a), static_cast<const __half*>(b), static_cast<const __half*>(w), ldw, q, ldq,
        static_cast<__half*>(scale), (int)k, (int)r, scaling);
    return check_launch("lora_requant_simt_kernel");
  }
  CUtensorMap tb, ta, tw, tq;
  if (int s = lora_maps(&tb, &ta, a, b, n, k, r)) return s;
  if (int s = make_tmap_2d(&tw, w, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, n, k, ldw * 2, 128, 64, CU_TENSOR_MAP_SWIZZLE_128B))
    return s;
  if (int s = make_tmap_2d(&tq, q, CU_TENSOR_MAP_DATA_TYPE_UINT8, n, k, ldq, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B))
    return s;
  return launch_lora_tc<kModeRequant>(tb, ta, tw, tq, static_cast<__half*>(scale), (int)n, (int)k, (int)r, scaling, st);
}
}  // namespace bw

extern "C" size_t bw_lora_merge_requant_batched_workspace_size(const bw_lora_requant_problem* problems, int count) {
  using namespace bw;
  // the largest launch: up to kReqMaxProblems eligible problems at a time
  int64_t best = 0, run = 0;
  int inrun = 0;
  for (int i = 0; i < count; ++i) {
    const bw_lora_requant_problem& P = problems[i];
    if (P.n <= 0 || P.k <= 0 || !req_cluster_eligible(P)) continue;
    if (inrun == kReqMaxProblems) {
      best = std::max(best, run);
      run = 0;
      inrun = 0;
    }
    run += req_items(P);
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
    if (req_cluster_eligible(P)) {
      grouped.push_back(i);
    } else if (int e = merge_requant_single(P, st)) {
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
