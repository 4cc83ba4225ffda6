// W8A16 GEMM on the 5th-generation tensor core (tcgen05), sm_100a.
//
// Replaces the Triton int8_gemm of the reference
// (src/blackwell_ops/kernels/int8_gemm.py:15-60 kernel, :71-107 launcher):
//     y[m, n] = dt( fp32( sum_k x[m,k] * w_int8[n,k] ) * fp32(scale[n]) ),  dt = x.dtype
//
// Formulation ("swap AB"): a work unit is 128 weight rows (the UMMA M
// dimension) x BM tokens (the UMMA N dimension, 16..128) x a K range, so a
// decode call with M = 1..16 tokens still fills the 128-row tensor-core
// datapath and the op streams the int8 weight from HBM exactly once.  One
// persistent kernel serves every M (details above its definition).  Split-K
// (few tiles for the SMs) writes fp32 partials to the workspace; the last CTA
// of a tile (atomic ticket) sums the splits in split order (deterministic) and
// resets the tile's counter to zero.
//
// Layouts that TMA cannot address (unaligned base, row strides that are not
// multiples of 16 bytes) go to a CUDA-core kernel with the same arithmetic.
#include <stdio.h>

#include <mutex>

#include "common.cuh"

namespace bw {

template <bool BF16>
__device__ __forceinline__ void convert_chunk(const uint4& v, uint4& o0, uint4& o1) {
  if constexpr (BF16) {
    i8x4_to_bf16x4(v.x, o0.x, o0.y);
    i8x4_to_bf16x4(v.y, o0.z, o0.w);
    i8x4_to_bf16x4(v.z, o1.x, o1.y);
    i8x4_to_bf16x4(v.w, o1.z, o1.w);
  } else {
    i8x4_to_f16x4(v.x, o0.x, o0.y);
    i8x4_to_f16x4(v.y, o0.z, o0.w);
    i8x4_to_f16x4(v.z, o1.x, o1.y);
    i8x4_to_f16x4(v.w, o1.z, o1.w);
  }
}

template <bool BF16>
__device__ __forceinline__ void store_out(void* y, int64_t idx, float v) {
  if constexpr (BF16) static_cast<__nv_bfloat16*>(y)[idx] = __float2bfloat16_rn(v);
  else static_cast<__half*>(y)[idx] = __float2half_rn(v);
}

// Column-parallel N-split with the all-gather fused into the epilogue: every
// output element is stored into every rank's Y (peer memory over NVLink, plain
// stores), guarded by two flag handshakes on the ranks' signal pads.
struct GatherArgs {
  unsigned long long y[8];    // each rank's Y [M, ldy]; this rank's columns start at col0
  unsigned long long sig[8];  // each rank's signal pad (u32): [0,G) ready, [G,2G) done, [2G] CTA ticket,
                              // [2G+1] epoch of the last completed call (all zero before the first call)
  long long col0;
  int world, rank;            // world == 0: a plain GEMM into y
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Bounded wait until every word of flags[0, n) equals v; false (and the site recorded) on timeout.
__device__ __forceinline__ bool wait_flags(const uint32_t* flags, int n, uint32_t v, int site) {
  const long long limit = static_cast<long long>(BW_WAIT_LIMIT_NS) * 5 / 2;
  const long long t0 = clock64();
  for (int p = 0; p < n; ++p) {
    while (ld_acquire_sys(flags + p) != v) {
      if (clock64() - t0 > limit) {
        record_timeout(site);
        return false;
      }
    }
  }
  return true;
}

template <bool BF16>
__device__ __forceinline__ void store_y(void* y, const GatherArgs& g, int64_t ldy, int m, int n, float v) {
  if (g.world == 0) {
    store_out<BF16>(y, static_cast<int64_t>(m) * ldy + n, v);
  } else {
    const int64_t idx = static_cast<int64_t>(m) * ldy + g.col0 + n;
    for (int r = 0; r < g.world; ++r) store_out<BF16>(reinterpret_cast<void*>(g.y[r]), idx, v);
  }
}

// ---------------------------------------------------------------------------
// Persistent W8A16 GEMM for every M (decode, prefill).
//
// One CTA per SM walks work units (m_tile fastest, then n_tile, then k-split)
// with a stride of gridDim.x; the TMA producer streams W/x stages continuously
// across units, so the weight stream never drains between tiles, and the units
// that share a weight tile run side by side (one DRAM read, the rest from L2).
// 448 threads:
//   warp 0       TMA producer (STAGES-deep ring of [W int8 128x128 B | x BM x 128])
//   warp 1       TMEM owner (512 columns) + tcgen05.mma issuer
//   warps 2-9    dequantisers in two groups of four that take alternate k-blocks
//                (thread = weight row, all 128 columns of the stage); int8 ->
//                f16/bf16 straight into a TMEM A buffer (tcgen05.st), 4 x 64 cols
//   warps 10-13  epilogue: double-buffered TMEM accumulators (2 x BM cols), so a
//                unit's epilogue overlaps the next unit's mainloop
// The MMA is the TS form: A (dequantised W) from TMEM, B (x) from shared memory.
// Programmatic dependent launch: the producer waits (griddepcontrol.wait) only
// before its first x load and the epilogue before its first global access, so
// a dependent launch can stream weights while its predecessor finishes.
// ---------------------------------------------------------------------------
template <int BM>
struct PCfg {
  static constexpr int BK = 128;
  static constexpr int W_BYTES = 128 * 128;
  static constexpr int X_PANEL = BM * 128;
  static constexpr int X_BYTES = 2 * X_PANEL;
  static constexpr int STAGE_BYTES = W_BYTES + X_BYTES;
  static constexpr int STAGES = (200 * 1024) / STAGE_BYTES > 8 ? 8 : (200 * 1024) / STAGE_BYTES;
  static constexpr int ASTAGES = 4;  // TMEM A buffers, 64 columns each
  static constexpr int A_COL0 = 0;
  static constexpr int D_COL0 = ASTAGES * 64;
  static constexpr int TMEM_COLS = 512;
  static constexpr int OFF_W = 0;
  static constexpr int OFF_X = STAGES * W_BYTES;
  static constexpr int OFF_BAR = OFF_X + STAGES * X_BYTES;
  static constexpr int BAR_BYTES = 512;
  static constexpr int SMEM = OFF_BAR + BAR_BYTES + 1024;
  static constexpr int THREADS = 448;
  static_assert(BM >= 16 && BM <= 128 && BM % 16 == 0, "UMMA N for M=128");
  static_assert(D_COL0 + 2 * BM <= TMEM_COLS, "TMEM budget");
  static_assert(SMEM <= 232448, "shared memory budget");
  static_assert((3 * STAGES + 2 * ASTAGES + 4 + 1) * 8 + 16 <= BAR_BYTES, "barrier area");
};

enum PersistentWaitSite : int {
  kSitePProd = 111,
  kSitePConvFull = 112,
  kSitePConvA = 113,
  kSitePMmaA = 114,
  kSitePMmaFull = 115,
  kSitePMmaD = 116,
  kSitePEpi = 117,
  kSitePDrain = 118,
  kSitePFinal = 119,
  kSiteGReady = 130,
  kSiteGDone = 131,
};

template <int BM, bool BF16>
__global__ void __launch_bounds__(448, 1)
    w8a16_persistent_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                            const void* __restrict__ scale, int sdtype, void* __restrict__ y, int64_t ldy, int M,
                            int N, int n_tiles, int kblocks, int kb_per_split, int splits, int units,
                            float* __restrict__ ws, int* __restrict__ counters, const GatherArgs g) {
  using C = PCfg<BM>;
  constexpr int STAGES = C::STAGES;
  constexpr int ASTAGES = C::ASTAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sW = smem + C::OFF_W;
  uint8_t* sX = smem + C::OFF_X;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* empty = full + STAGES;
  uint64_t* afull = empty + STAGES;
  uint64_t* aempty = afull + ASTAGES;
  uint64_t* dfull = aempty + ASTAGES;    // 2
  uint64_t* dempty = dfull + 2;          // 2
  uint64_t* final_bar = dempty + 2;      // 1
  uint64_t* xfull = final_bar + 1;       // STAGES: the x tiles of a stage (full[] covers its W tile)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xfull + STAGES);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* ticket = abort_flag + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&xfull[s], 1);
      mbar_init(&empty[s], 4 + 1);  // one group of 4 dequantiser warps + 1 MMA commit
    }
    for (int t = 0; t < ASTAGES; ++t) {
      mbar_init(&afull[t], 4);
      mbar_init(&aempty[t], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&dfull[b], 1);
      mbar_init(&dempty[b], 4);
    }
    mbar_init(final_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_x);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (threadIdx.x == 0) pdl_launch_dependents();

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      // a weight tile used by several M-tiles stays in L2 for the neighbours that share it
      const int m_tiles = units / (n_tiles * splits);
      const uint64_t pol_w = m_tiles > 1 ? l2_policy_evict_normal() : l2_policy_evict_first();
      const uint64_t pol_x = l2_policy_evict_last();
      // (unit, k-block) walk of this CTA
      int u = blockIdx.x, i = 0;
      auto unit_kb = [&](int uu, int& nt, int& mt, int& kb0, int& nkb) {
        const int sp = uu % splits;
        const int t = uu / splits;
        // M-tile fastest: the units that share a weight tile are consecutive
        const int m_tiles_u = units / (n_tiles * splits);
        mt = t % m_tiles_u;
        nt = t / m_tiles_u;
        kb0 = sp * kb_per_split;
        nkb = min(kb_per_split, kblocks - kb0);
      };
      // Weights do not depend on the preceding kernel: fill the ring with weight
      // tiles first, then wait for the predecessor (PDL) before loading x.
      int pre = 0;
      {
        int uu = u, ii = 0;
        while (uu < units && pre < STAGES) {
          int nt, mt, kb0, nkb;
          unit_kb(uu, nt, mt, kb0, nkb);
          mbar_arrive_expect_tx(&full[pre], C::W_BYTES);
          tma_load_2d(sW + pre * C::W_BYTES, &tm_w, &full[pre], (kb0 + ii) * C::BK, nt * 128, pol_w);
          ++pre;
          if (++ii == nkb) {
            ii = 0;
            uu += gridDim.x;
          }
        }
      }
      pdl_wait();
      int it = 0;
      bool ok = true;
      while (u < units && ok) {
        int nt, mt, kb0, nkb;
        unit_kb(u, nt, mt, kb0, nkb);
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        const int kx = (kb0 + i) * C::BK;
        if (it >= pre) {
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, kSitePProd)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], C::W_BYTES);
          tma_load_2d(sW + s * C::W_BYTES, &tm_w, &full[s], kx, nt * 128, pol_w);
        }
        mbar_arrive_expect_tx(&xfull[s], C::X_BYTES);
        tma_load_2d(sX + s * C::X_BYTES, &tm_x, &xfull[s], kx, mt * BM, pol_x);
        tma_load_2d(sX + s * C::X_BYTES + C::X_PANEL, &tm_x, &xfull[s], kx + 64, mt * BM, pol_x);
        ++it;
        if (++i == nkb) {
          i = 0;
          u += gridDim.x;
        }
      }
      if (!ok) {
        for (int j = (it > STAGES ? it - STAGES : 0); j < it; ++j)
        {
          mbar_wait(&full[j % STAGES], (j / STAGES) & 1, nullptr, kSitePDrain);
          mbar_wait(&xfull[j % STAGES], (j / STAGES) & 1, nullptr, kSitePDrain);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_f16(128, BM, BF16, false);
      int it = 0, j = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++j) {
        const int sp = u % splits;
        const int kb0 = sp * kb_per_split;
        const int nkb = min(kb_per_split, kblocks - kb0);
        const int b = j & 1;
        if (!mbar_wait(&dempty[b], ((j >> 1) & 1) ^ 1, abort_flag, kSitePMmaD)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + C::D_COL0 + b * BM;
        for (int i = 0; i < nkb; ++i, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          const int t = it % ASTAGES;
          const uint32_t pa = (it / ASTAGES) & 1;
          if (!mbar_wait(&afull[t], pa, abort_flag, kSitePMmaA) || !mbar_wait(&xfull[s], ph, abort_flag, kSitePMmaFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t x_base = smem_u32(sX + s * C::X_BYTES);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t bd = make_sdesc(x_base + (kk >> 2) * C::X_PANEL + (kk & 3) * 32, 16, 1024, kLayoutSW128);
            umma_f16_ts(d_tmem, tmem + C::A_COL0 + t * 64 + kk * 8, bd, idesc, (i | kk) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[s]);
          umma_commit(&aempty[t]);
        }
        if (ok) umma_commit(&dfull[b]);
      }
      // every issued MMA has completed before TMEM is released
      umma_commit(final_bar);
      mbar_wait(final_bar, 0, nullptr, kSitePFinal);
    }
  } else if (warp < 10) {
    // ---------------- dequantisers ----------------
    // Two groups of four warps take alternate k-blocks, so two stages are
    // dequantised at once; within a group, thread = weight row (all 128 columns).
    const int q = warp & 3;
    const int grp = (warp - 2) >> 2;
    const int row = q * 32 + lane;
    const int sw = row & 7;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16) + C::A_COL0;
    int it = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
      const int sp = u % splits;
      const int kb0 = sp * kb_per_split;
      const int nkb = min(kb_per_split, kblocks - kb0);
      for (int i = 0; i < nkb; ++i, ++it) {
        if ((it & 1) != grp) continue;
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        const int t = it % ASTAGES;
        const uint32_t pa = (it / ASTAGES) & 1;
        if (!mbar_wait(&full[s], ph, abort_flag, kSitePConvFull) ||
            !mbar_wait(&aempty[t], pa ^ 1, abort_flag, kSitePConvA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint8_t* src = sW + s * C::W_BYTES + row * 128;
        uint4 v[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) v[c] = *reinterpret_cast<const uint4*>(src + ((c ^ sw) << 4));
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t out[32];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint4 o0, o1;
            convert_chunk<BF16>(v[4 * h + c], o0, o1);
            out[8 * c + 0] = o0.x;
            out[8 * c + 1] = o0.y;
            out[8 * c + 2] = o0.z;
            out[8 * c + 3] = o0.w;
            out[8 * c + 4] = o1.x;
            out[8 * c + 5] = o1.y;
            out[8 * c + 6] = o1.z;
            out[8 * c + 7] = o1.w;
          }
          tmem_st32(lane_base + t * 64 + h * 32, out);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&afull[t]);
          mbar_arrive(&empty[s]);
        }
      }
    }
  } else {
    // ---------------- epilogue ----------------
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(q * 32) << 16) + C::D_COL0;
    pdl_wait();
    bool gather_ok = true;
    uint32_t epoch = 0;
    if (g.world > 0) {
      // this call's epoch: one past the last completed call (kept on the device, so a captured
      // graph replays correctly); ready handshake: this rank's Y may be overwritten now (its
      // earlier readers are done), and no store goes to a peer before that peer has said the same
      if (warp == 10 && lane == 0) {
        const uint32_t* mine = reinterpret_cast<const uint32_t*>(g.sig[g.rank]);
        epoch = ld_acquire_sys(mine + 2 * g.world + 1) + 1u;
        if (blockIdx.x == 0)
          for (int p = 0; p < g.world; ++p) st_release_sys(reinterpret_cast<uint32_t*>(g.sig[p]) + g.rank, epoch);
        gather_ok = wait_flags(mine, g.world, epoch, kSiteGReady);
        if (!gather_ok) *abort_flag = 1;
      }
      gather_ok = !named_bar_any(1, 128, !gather_ok);
    }
    int j = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++j) {
      const int sp = u % splits;
      const int t = u / splits;
      const int m_tiles_u = units / (n_tiles * splits);
      const int mt = t % m_tiles_u;
      const int nt = t / m_tiles_u;
      const int n = nt * 128 + row;
      const int m0 = mt * BM;
      const int b = j & 1;
      const bool ok = mbar_wait(&dfull[b], (j >> 1) & 1, abort_flag, kSitePEpi);
      if (named_bar_any(1, 128, !ok || *abort_flag)) break;  // same decision in all 4 warps
      tc_fence_after();
      const uint32_t taddr = lane_addr + b * BM;
      if (splits == 1) {
        const float sc = n < N ? load_as_float(scale, n, sdtype) : 0.f;
#pragma unroll 1
        for (int c0 = 0; c0 < BM; c0 += 16) {
          uint32_t r[16];
          tmem_ld16(taddr + c0, r);
          tmem_ld_wait();
          if (n < N) {
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const int m = m0 + c0 + e;
              if (m < M) store_y<BF16>(y, g, ldy, m, n, __uint_as_float(r[e]) * sc);
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&dempty[b]);
      } else {
        float* mine = ws + (static_cast<size_t>(t) * splits + sp) * (128 * BM) + static_cast<size_t>(row) * BM;
#pragma unroll 1
        for (int c0 = 0; c0 < BM; c0 += 16) {
          uint32_t r[16];
          tmem_ld16(taddr + c0, r);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 16; e += 4)
            *reinterpret_cast<float4*>(mine + c0 + e) = make_float4(
                __uint_as_float(r[e]), __uint_as_float(r[e + 1]), __uint_as_float(r[e + 2]), __uint_as_float(r[e + 3]));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&dempty[b]);  // accumulator free; partials are in global memory
        __threadfence();
        named_bar_sync(1, 128);
        if (warp == 10 && lane == 0) *ticket = atomicAdd(&counters[t], 1);
        named_bar_sync(1, 128);
        const bool last = *ticket == splits - 1;
        named_bar_sync(1, 128);  // every thread has read the ticket before the next unit overwrites it
        if (last) {
          __threadfence();
          const float sc = n < N ? load_as_float(scale, n, sdtype) : 0.f;
          const float* base = ws + static_cast<size_t>(t) * splits * (128 * BM) + static_cast<size_t>(row) * BM;
          // 8 columns at a time; the loads of four partials are issued together, then
          // summed in split order (partial 0 first, as the result must not depend on timing)
#pragma unroll 1
          for (int c0 = 0; c0 < BM; c0 += 8) {
            float a[8];
#pragma unroll 1
            for (int p0 = 0; p0 < splits; p0 += 4) {
              float4 v[4][2];
#pragma unroll
              for (int pp = 0; pp < 4; ++pp)
#pragma unroll
                for (int e = 0; e < 2; ++e)
                  v[pp][e] = p0 + pp < splits ? __ldcg(reinterpret_cast<const float4*>(
                                                    base + static_cast<size_t>(p0 + pp) * 128 * BM + c0 + 4 * e))
                                              : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
              for (int pp = 0; pp < 4; ++pp) {
                if (p0 + pp >= splits) break;
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                  const float f[4] = {v[pp][e].x, v[pp][e].y, v[pp][e].z, v[pp][e].w};
#pragma unroll
                  for (int g = 0; g < 4; ++g) a[4 * e + g] = (p0 + pp == 0) ? f[g] : a[4 * e + g] + f[g];
                }
              }
            }
            if (n < N) {
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const int m = m0 + c0 + e;
                if (m < M) store_y<BF16>(y, g, ldy, m, n, a[e] * sc);
              }
            }
          }
          if (warp == 10 && lane == 0) counters[t] = 0;
        }
      }
    }
    if (g.world > 0) {
      // done handshake: the last CTA of this rank tells every peer that this rank's columns
      // are in its Y, then waits until every peer has said the same (bounded)
      named_bar_sync(1, 128);
      if (warp == 10 && lane == 0) {
        __threadfence_system();
        uint32_t* mine = reinterpret_cast<uint32_t*>(g.sig[g.rank]);
        if (atomicAdd(mine + 2 * g.world, 1u) == gridDim.x - 1) {
          // every CTA of this call has read the epoch (it took a ticket after doing so)
          __threadfence_system();
          for (int p = 0; p < g.world; ++p)
            st_release_sys(reinterpret_cast<uint32_t*>(g.sig[p]) + g.world + g.rank, epoch);
          wait_flags(mine + g.world, g.world, epoch, kSiteGDone);
          atomicExch(mine + 2 * g.world, 0u);  // the CTA ticket, for the next call
          st_release_sys(mine + 2 * g.world + 1, epoch);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// CUDA-core fallback for layouts TMA cannot address: one thread per output.
template <bool BF16>
__global__ void __launch_bounds__(128) w8a16_simt_kernel(const void* __restrict__ x, int64_t ldx,
                                                         const int8_t* __restrict__ w, int64_t ldw,
                                                         const void* __restrict__ scale, int sdtype,
                                                         void* __restrict__ y, int64_t ldy, int M, int N, int K) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  const int m = blockIdx.y;
  if (n >= N || m >= M) return;
  const int xdt = BF16 ? BW_DTYPE_BF16 : BW_DTYPE_F16;
  float acc = 0.f;
  for (int k = 0; k < K; ++k)
    acc = fmaf(load_as_float(x, static_cast<int64_t>(m) * ldx + k, xdt),
               static_cast<float>(w[static_cast<int64_t>(n) * ldw + k]), acc);
  store_out<BF16>(y, static_cast<int64_t>(m) * ldy + n, acc * load_as_float(scale, n, sdtype));
}

// ---------------------------------------------------------------------------
// host planning
// ---------------------------------------------------------------------------
struct GemmPlan {
  int bm = 16;
  int n_tiles = 0, m_tiles = 0, kblocks = 0, splits = 1, kb_per_split = 0, units = 0, grid = 0;
  size_t counter_bytes = 0, partial_bytes = 0;
};

// Persistent path: pick the split count that minimises the busiest CTA's work,
// counting each k-block as 16 KB of weights and each unit a fixed overhead
// (epilogue, pipeline hand-off) plus, when split, its fp32 partial round trip.
static GemmPlan plan_gemm(int64_t m, int64_t n, int64_t k) {
  GemmPlan p;
  const int sms = num_sms();
  p.n_tiles = static_cast<int>((n + 127) / 128);
  p.kblocks = static_cast<int>((k + 127) / 128);
  p.bm = m <= 16 ? 16 : m <= 32 ? 32 : m <= 64 ? 64 : 128;
  p.m_tiles = static_cast<int>((m + p.bm - 1) / p.bm);
  const int64_t tiles = static_cast<int64_t>(p.n_tiles) * p.m_tiles;
  // split-K count: cost model over the units each CTA walks (weight bytes per unit,
  // a fixed per-unit cost, the partials a split writes)
  double best = 1e300;
  for (int sp = 1; sp <= p.kblocks && sp <= 32; ++sp) {
    const int kbps = (p.kblocks + sp - 1) / sp;
    const int real = (p.kblocks + kbps - 1) / kbps;
    if (real != sp) continue;
    const int64_t units = tiles * sp;
    const int64_t per_cta = (units + sms - 1) / sms;
    const double unit_cost = kbps * 16384.0 + 6000.0 + (sp > 1 ? 2.0 * 128 * p.bm * 4 : 0.0);
    const double cost = static_cast<double>(per_cta) * unit_cost;
    if (cost < best * 0.97) {
      best = cost;
      p.splits = sp;
      p.kb_per_split = kbps;
    }
  }
  const int64_t units = tiles * p.splits;
  p.units = units > INT32_MAX ? -1 : static_cast<int>(units);  // -1: too many units (refused by the caller)
  p.grid = units < sms ? static_cast<int>(units) : sms;
  if (p.splits > 1) {
    p.counter_bytes = ((static_cast<size_t>(tiles) * sizeof(int) + 255) / 256) * 256;
    p.partial_bytes = static_cast<size_t>(tiles) * p.splits * 128 * p.bm * sizeof(float);
  }
  return p;
}

static bool g_use_pdl = true;

template <int BM, bool BF16>
static int launch_persistent(const GemmPlan& p, const CUtensorMap& tw, const CUtensorMap& tx, const void* scale,
                             int sdt, void* y, int64_t ldy, int M, int N, float* ws, int* counters,
                             const GatherArgs& g, cudaStream_t st) {
  using C = PCfg<BM>;
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t attr_err = cudaSuccess;
  std::call_once(once[dev & 63], [&] {
    attr_err = cudaFuncSetAttribute(w8a16_persistent_kernel<BM, BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    C::SMEM);
  });
  if (int s = check_cuda(attr_err, "cudaFuncSetAttribute(w8a16_persistent_kernel)")) return s;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(C::THREADS);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = g_use_pdl ? 1 : 0;
  return check_cuda(cudaLaunchKernelEx(&cfg, w8a16_persistent_kernel<BM, BF16>, tw, tx, scale, sdt, y, ldy, M, N,
                                       p.n_tiles, p.kblocks, p.kb_per_split, p.splits, p.units, ws, counters, g),
                    "cudaLaunchKernelEx(w8a16_persistent_kernel)");
}

template <bool BF16>
static int dispatch_gemm(const GemmPlan& p, const CUtensorMap& tw, const CUtensorMap& tx, const void* scale, int sdt,
                         void* y, int64_t ldy, int M, int N, float* ws, int* counters, const GatherArgs& g,
                         cudaStream_t st) {
  switch (p.bm) {
    case 16: return launch_persistent<16, BF16>(p, tw, tx, scale, sdt, y, ldy, M, N, ws, counters, g, st);
    case 32: return launch_persistent<32, BF16>(p, tw, tx, scale, sdt, y, ldy, M, N, ws, counters, g, st);
    case 64: return launch_persistent<64, BF16>(p, tw, tx, scale, sdt, y, ldy, M, N, ws, counters, g, st);
    default: return launch_persistent<128, BF16>(p, tw, tx, scale, sdt, y, ldy, M, N, ws, counters, g, st);
  }
}

static bool tma_ok(const void* p, int64_t ld_bytes) {
  return p != nullptr && (reinterpret_cast<uintptr_t>(p) % 16 == 0) && (ld_bytes % 16 == 0) && ld_bytes > 0;
}

}  // namespace bw

extern "C" size_t bw_w8a16_gemm_workspace_size(int64_t m, int64_t n, int64_t k) {
  if (m <= 0 || n <= 0 || k <= 0) return 0;
  const bw::GemmPlan p = bw::plan_gemm(m, n, k);
  return p.counter_bytes + p.partial_bytes;
}

extern "C" size_t bw_w8a16_gemm_workspace_zeroed_bytes(int64_t m, int64_t n, int64_t k) {
  if (m <= 0 || n <= 0 || k <= 0) return 0;
  return bw::plan_gemm(m, n, k).counter_bytes;
}

namespace bw {
static int gemm_impl(const void* x, int x_dtype, int64_t ldx, const int8_t* w, int64_t ldw, const void* scale,
                     int scale_dtype, void* y, int64_t ldy, int64_t m, int64_t n, int64_t k, void* workspace,
                     size_t workspace_bytes, const GatherArgs& g, void* stream) {
  if (m < 0 || n < 0 || k < 1)
    return fail(BW_ERR_INVALID_ARGUMENT, "int8_gemm: need m, n >= 0 and k >= 1 (got %lld, %lld, %lld)",
                (long long)m, (long long)n, (long long)k);
  if (x_dtype != BW_DTYPE_F16 && x_dtype != BW_DTYPE_BF16)
    return fail(BW_ERR_INVALID_ARGUMENT, "int8_gemm: x must be fp16 or bf16 (dtype %d)", x_dtype);
  if (scale_dtype < BW_DTYPE_F16 || scale_dtype > BW_DTYPE_F32)
    return fail(BW_ERR_INVALID_ARGUMENT, "int8_gemm: unsupported scale dtype %d", scale_dtype);
  if (m == 0 || n == 0) return BW_OK;
  if (!x || !w || !scale || !y) return fail(BW_ERR_INVALID_ARGUMENT, "int8_gemm: null pointer");
  if (ldx < k || ldw < k || ldy < n) return fail(BW_ERR_INVALID_ARGUMENT, "int8_gemm: row stride too small");
  if (m > (1LL << 30) || n > (1LL << 30) || k > (1LL << 30))
    return fail(BW_ERR_INVALID_ARGUMENT, "int8_gemm: dimension too large");
  if (int s = require_sm100()) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool bf16 = x_dtype == BW_DTYPE_BF16;

  if (!tma_ok(x, ldx * 2) || !tma_ok(w, ldw)) {
    if (g.world > 0)
      return fail(BW_ERR_UNSUPPORTED, "int8_gemm (all-gather): x and w must be 16-byte aligned with 16-byte row strides");
    dim3 grid(static_cast<unsigned>((n + 127) / 128), static_cast<unsigned>(m));
    if (bf16)
      w8a16_simt_kernel<true><<<grid, 128, 0, st>>>(x, ldx, w, ldw, scale, scale_dtype, y, ldy, (int)m, (int)n, (int)k);
    else
      w8a16_simt_kernel<false><<<grid, 128, 0, st>>>(x, ldx, w, ldw, scale, scale_dtype, y, ldy, (int)m, (int)n, (int)k);
    return check_launch("w8a16_simt_kernel");
  }

  const GemmPlan p = plan_gemm(m, n, k);
  if (p.units < 0) return fail(BW_ERR_INVALID_ARGUMENT, "int8_gemm: m=%lld n=%lld is too many output tiles",
                               (long long)m, (long long)n);
  float* ws = nullptr;
  int* counters = nullptr;
  if (p.splits > 1) {
    if (workspace == nullptr || workspace_bytes < p.counter_bytes + p.partial_bytes)
      return fail(BW_ERR_WORKSPACE, "int8_gemm: workspace of %zu bytes required, %zu given",
                  p.counter_bytes + p.partial_bytes, workspace_bytes);
    if (reinterpret_cast<uintptr_t>(workspace) % 16 != 0)
      return fail(BW_ERR_WORKSPACE, "int8_gemm: workspace must be 16-byte aligned");
    counters = static_cast<int*>(workspace);
    ws = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + p.counter_bytes);
  }
  CUtensorMap tw, tx;
  if (int s = make_tmap_2d(&tw, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, n, k, ldw, 128, 128,
                           CU_TENSOR_MAP_SWIZZLE_128B))
    return s;
  if (int s = make_tmap_2d(&tx, x, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, m, k,
                           ldx * 2, p.bm, 64, CU_TENSOR_MAP_SWIZZLE_128B))
    return s;
  if (bf16) return dispatch_gemm<true>(p, tw, tx, scale, scale_dtype, y, ldy, (int)m, (int)n, ws, counters, g, st);
  return dispatch_gemm<false>(p, tw, tx, scale, scale_dtype, y, ldy, (int)m, (int)n, ws, counters, g, st);
}
}  // namespace bw

extern "C" int bw_w8a16_gemm(const void* x, int x_dtype, int64_t ldx, const int8_t* w, int64_t ldw,
                             const void* scale, int scale_dtype, void* y, int64_t ldy, int64_t m, int64_t n,
                             int64_t k, void* workspace, size_t workspace_bytes, void* stream) {
  bw::GatherArgs g = {};
  return bw::gemm_impl(x, x_dtype, ldx, w, ldw, scale, scale_dtype, y, ldy, m, n, k, workspace, workspace_bytes, g,
                       stream);
}

// Column-parallel N-split GEMM with the all-gather in the epilogue: this rank's output columns
// [col0, col0 + n) are stored into every rank's Y over peer memory, then the ranks exchange
// completion flags (bounded waits; a timeout shows in bw_device_status).
extern "C" int bw_w8a16_gemm_allgather(const void* x, int x_dtype, int64_t ldx, const int8_t* w, int64_t ldw,
                                       const void* scale, int scale_dtype, void* const* y_ranks, int64_t ldy,
                                       int64_t col0, int64_t m, int64_t n, int64_t k, void* const* signal_ranks,
                                       int world, int rank, void* workspace, size_t workspace_bytes, void* stream) {
  using namespace bw;
  if (world < 1 || world > 8 || rank < 0 || rank >= world)
    return fail(BW_ERR_INVALID_ARGUMENT, "int8_gemm (all-gather): need 1 <= world <= 8 and 0 <= rank < world");
  if (!y_ranks || !signal_ranks) return fail(BW_ERR_INVALID_ARGUMENT, "int8_gemm (all-gather): null pointer list");
  if (col0 < 0 || col0 + n > ldy)
    return fail(BW_ERR_INVALID_ARGUMENT, "int8_gemm (all-gather): columns [%lld, %lld) outside the row stride %lld",
                (long long)col0, (long long)(col0 + n), (long long)ldy);
  GatherArgs g = {};
  for (int r = 0; r < world; ++r) {
    if (!y_ranks[r] || !signal_ranks[r])
      return fail(BW_ERR_INVALID_ARGUMENT, "int8_gemm (all-gather): null pointer for rank %d", r);
    if (reinterpret_cast<uintptr_t>(signal_ranks[r]) % 4 != 0)
      return fail(BW_ERR_INVALID_ARGUMENT, "int8_gemm (all-gather): signal pad of rank %d is not 4-byte aligned", r);
    g.y[r] = reinterpret_cast<unsigned long long>(y_ranks[r]);
    g.sig[r] = reinterpret_cast<unsigned long long>(signal_ranks[r]);
  }
  g.col0 = col0;
  g.world = world;
  g.rank = rank;
  return gemm_impl(x, x_dtype, ldx, w, ldw, scale, scale_dtype, y_ranks[rank], ldy, m, n, k, workspace,
                   workspace_bytes, g, stream);
}

// ---------------------------------------------------------------------------
// GEMM entry point that allocates nothing (no counterpart in the reference).
//
// Some callers cannot give this library device memory: a serving runtime whose
// memory manager reserves the whole GPU at start-up and refuses allocations
// from plug-ins, or a foreign-language binding that has no handle on any CUDA
// allocator.  For them the split-K scratch (tile counters + fp32 partials) is
// this fixed array, one per GPU that loads the library, held until the process
// exits.  Host code never uses the symbol directly: its device address is
// looked up once per device with cudaGetSymbolAddress.
// ---------------------------------------------------------------------------
namespace bw {
constexpr size_t kStaticScratchBytes = size_t(8) << 20;  // 8 MiB
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

// Device address of g_static_scratch on the current device (looked up on the
// first call per device, with that device current).
static int static_scratch_address(void** out) {
  static std::mutex mu;
  static void* addr[64] = {};
  int dev = 0;
  if (int s = check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) return s;
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev & 63] == nullptr) {
    void* p = nullptr;
    if (int s = check_cuda(cudaGetSymbolAddress(&p, g_static_scratch), "cudaGetSymbolAddress(static scratch)"))
      return s;
    addr[dev & 63] = p;
  }
  *out = addr[dev & 63];
  return BW_OK;
}
}  // namespace bw

extern "C" size_t bw_w8a16_gemm_static_scratch_bytes(void) { return bw::kStaticScratchBytes; }

extern "C" int bw_w8a16_gemm_noalloc(const void* x, int x_dtype, int64_t ldx, const int8_t* w, int64_t ldw,
                                     const void* scale, int scale_dtype, void* y, int64_t ldy, int64_t m, int64_t n,
                                     int64_t k, void* stream) {
  using namespace bw;
  if (m > 0 && n > 0 && k > 0) {
    const size_t need = bw_w8a16_gemm_workspace_size(m, n, k);
    if (need > kStaticScratchBytes)
      return fail(BW_ERR_WORKSPACE,
                  "int8_gemm (no-alloc): m=%lld n=%lld k=%lld needs %zu bytes of split-K scratch, more than the "
                  "%zu-byte static array",
                  (long long)m, (long long)n, (long long)k, need, kStaticScratchBytes);
    if (need > 0) {
      void* scratch = nullptr;
      if (int s = static_scratch_address(&scratch)) return s;
      // the array keeps the previous call's contents: the tile counters must start at zero
      const size_t zeroed = bw_w8a16_gemm_workspace_zeroed_bytes(m, n, k);
      if (int s = check_cuda(cudaMemsetAsync(scratch, 0, zeroed, static_cast<cudaStream_t>(stream)),
                             "clear static scratch counters"))
        return s;
      return bw_w8a16_gemm(x, x_dtype, ldx, w, ldw, scale, scale_dtype, y, ldy, m, n, k, scratch,
                           kStaticScratchBytes, stream);
    }
  }
  return bw_w8a16_gemm(x, x_dtype, ldx, w, ldw, scale, scale_dtype, y, ldy, m, n, k, nullptr, 0, stream);
}
