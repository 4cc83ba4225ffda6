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
// (few tiles for the SMs) or stream-K (many tiles: equal k-ranges per CTA)
// writes fp32 pieces of split tiles to the workspace; the last CTA of a tile
// (atomic ticket) sums them in k order (deterministic) and resets the tile's
// counter to zero.
//
// Layouts that TMA cannot address (unaligned base, row strides that are not
// multiples of 16 bytes) go to a CUDA-core kernel with the same arithmetic.
#include <stdio.h>

#include <algorithm>
#include <mutex>
#include <type_traits>

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

// Column-parallel N-split with the all-gather fused into the epilogue.  Rank p's
// output columns are [base0 + p*n, base0 + (p+1)*n) of every rank's Y.  A CTA
// stores the outputs it produces into its own rank's Y and, for every peer, into
// that peer's mailbox as 8-byte words {2 outputs, call epoch} (plain peer stores
// over NVLink, no fence: a word is read whole, so its epoch says its data has
// arrived).  Each rank copies its peers' words into its Y as they arrive.
struct GatherArgs {
  unsigned long long ybase;    // this rank's Y at rank 0's first column (rank p's columns: ybase + p*n)
  unsigned long long pad[8];   // each rank's signal pad: u32 [0] CTA ticket, [1] epoch of the last call
                               // (zero before the first call); u64 mailbox from byte kMailbox0:
                               // [epoch parity][source rank][M][rowwords] words {data, epoch}
  int n;                       // columns per rank
  int rowwords;                // mailbox words per token row (ceil(n / 128) * 64)
  int world, rank;             // world == 0: a plain GEMM into y
  int vec;                     // plain GEMM: Y base 16-byte aligned, ldy and the tile columns multiples of 8
  int vec4;                    // gather: ybase 8-byte aligned, ldy and n multiples of 4
};

constexpr int kMailbox0 = 256;    // byte offset of the mailbox in a signal pad
constexpr int kGatherMaxM = 256;  // largest M of the fused all-gather (the mailbox grows with M)

__host__ __device__ inline size_t gather_pad_bytes(long long m, long long n, int world) {
  const long long rowwords = (n + 127) / 128 * 64;
  return kMailbox0 + static_cast<size_t>(2) * world * m * rowwords * 8;
}

// Grouped launch: up to kMaxGroup GEMMs that share x (same M, K, dtypes), e.g. the q/k/v or
// gate/up projections of a layer, as one schedule over the union of their n-tiles.  Problem p owns
// n-tiles [tile0[p], tile0[p+1]); count == 0 is a single GEMM (the kernel's own tm_w, scale, y).
constexpr int kMaxGroup = 4;
struct GroupArgs {
  CUtensorMap w[kMaxGroup];
  unsigned long long scale[kMaxGroup], y[kMaxGroup];
  long long ldy[kMaxGroup];
  int n[kMaxGroup];
  int tile0[kMaxGroup + 1];
  int count;
};

__device__ __forceinline__ int group_of(const GroupArgs& grp, int nt) {
  int p = 0;
  while (p + 1 < grp.count && nt >= grp.tile0[p + 1]) ++p;
  return p;
}

// 8 consecutive outputs of one token row, already rounded, as one 16-byte store.
__device__ __forceinline__ void store_y8(void* y, int64_t idx, const uint4& v) {
  *reinterpret_cast<uint4*>(static_cast<uint16_t*>(y) + idx) = v;
}

__device__ __forceinline__ void st_ll2(uint64_t* p, uint32_t a, uint32_t b, uint32_t ep) {
  const unsigned long long wa = (static_cast<unsigned long long>(ep) << 32) | a;
  const unsigned long long wb = (static_cast<unsigned long long>(ep) << 32) | b;
  asm volatile("st.relaxed.sys.global.v2.b64 [%0], {%1, %2};" ::"l"(p), "l"(wa), "l"(wb) : "memory");
}
__device__ __forceinline__ void ld_ll2(const uint64_t* p, unsigned long long& a, unsigned long long& b) {
  asm volatile("ld.relaxed.sys.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ uint32_t ld_relaxed_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

template <bool BF16>
__device__ __forceinline__ void store_y(void* y, int64_t ldy, int m, int n, float v) {
  store_out<BF16>(y, static_cast<int64_t>(m) * ldy + n, v);
}

// dt(v): the value an unfused int8_gemm would have written.
template <bool BF16>
__device__ __forceinline__ float round_out(float v) {
  if constexpr (BF16) return __bfloat162float(__float2bfloat16_rn(v));
  else return __half2float(__float2half_rn(v));
}

// ---------------------------------------------------------------------------
// Persistent W8A16 GEMM for every M (decode, prefill).
//
// One CTA per SM walks its work (split-K units b, b + grid, ... or one contiguous stream-K range
// of the tiles' k-blocks laid end to end); the TMA producers stream W/x stages continuously
// across units, so the weight stream never drains between tiles.
// 512 threads:
//   warp 0       TMA producer of the weight tiles (STAGES-deep ring, 128 x 128 B boxes, requested
//                BW_GEMM_W_GROUP k-blocks at a time)
//   warp 15      TMA producer of the activation tiles (their own XSTAGES-deep ring)
//   warp 1       TMEM owner (512 columns) + tcgen05.mma issuer 0
//   warp 14      tcgen05.mma issuer 1 (BM <= 64)
//   warps 2-9    dequantisers in two groups of four that take alternate k-blocks
//                (thread = weight row, all 128 columns of the stage); int8 ->
//                f16/bf16 straight into a TMEM A buffer (tcgen05.st), up to six of 64 columns
//   warps 10-13  epilogue
// The MMA is the TS form: A (dequantised W) from TMEM, B (x) from shared memory.
// A weight slot is released as soon as a dequantiser group has the row in registers, before it
// converts and waits for a free TMEM buffer, and an x slot when the MMAs that read it complete,
// so the weight ring stays full of loads in flight.  With two issuers, issuer h takes every other
// k-block into its own accumulator and the epilogue adds the two in issuer order (a fixed order,
// so the result does not depend on timing).  Accumulators are double-buffered (DBUF = 2), so a
// tile's epilogue overlaps the next tile's mainloop.  After the main loop all 512 threads sum the
// stream-K tiles this CTA finished last and, for the all-gather, receive the peers' tiles.
// A grouped launch (GroupArgs) runs up to four GEMMs that share x over the union of their tiles.
// Programmatic dependent launch: the weight producer never waits for the
// preceding kernel (weights do not depend on it); the activation producer and
// the epilogue wait (griddepcontrol.wait) before their first global access.
// ---------------------------------------------------------------------------
#ifndef BW_GEMM_STREAMK
#define BW_GEMM_STREAMK 1
#endif
// MMA issuer threads.  A thread issuing tcgen05.mma (M=128, N=16, K=16, A from TMEM slices that
// change every k-block) completes one per ~81 cycles however many accumulators it uses, plus
// ~120 cycles per tcgen05.commit; the tensor pipe overlaps the MMAs of different issuer threads
// (microbenchmark, 148 CTAs: 1, 2, 3, 4 issuers -> 81, 40, 27, 20 cycles per MMA aggregate).  A
// 16 KB k-block is eight MMAs, so one issuer caps a CTA near 2.5 TB/s-equivalent of weights.
// Decode tiles (BM <= 64) run two issuers (warps 1, 14), each taking every other k-block into
// its own accumulator; BM = 128 one.  A third issuer (warp 15, with the weight producer also
// loading the activation tiles) measured slower on the Llama-3-70B MLP decode shapes (3.1 against
// 4.0 TB/s; the single producer then issued one weight tile per ~1250 cycles) and is not kept.
// Shared memory (KB) of the two decode rings together.
#ifndef BW_GEMM_DEC_SMEM_KB
#define BW_GEMM_DEC_SMEM_KB 208
#endif
// Activation ring depth at BM = 16 (the weight ring takes the rest of the decode rings' budget).
#ifndef BW_GEMM_XSTAGES16
#define BW_GEMM_XSTAGES16 16
#endif
// The weight producer requests this many consecutive k-blocks of the same rows back to back
// (waiting for that many free slots), so a row's adjacent 128-byte blocks reach DRAM together.
#ifndef BW_GEMM_W_GROUP
#define BW_GEMM_W_GROUP 4
#endif
#ifndef BW_GEMM_W_GROUP_PRE  // the same for prefill tiles (BM = 128)
#define BW_GEMM_W_GROUP_PRE 1
#endif
// Loads in flight per thread in the deferred stream-K reduction (a tile cut into up to ~20
// pieces at small per-rank N).
#ifndef BW_GEMM_RED_BATCH
#define BW_GEMM_RED_BATCH 12
#endif
template <int BM>
struct PCfg {
  static constexpr int BK = 128;
  static constexpr int W_BYTES = 128 * 128;
  static constexpr int X_PANEL = BM * 128;
  static constexpr int X_BYTES = 2 * X_PANEL;
  static constexpr int STAGE_BYTES = W_BYTES + X_BYTES;
  static constexpr int NI = BM <= 64 ? 2 : 1;
  // Prefill ring: weight + activation tiles per stage, up to 4 stages of 48 KB.
  static constexpr int STAGES_PRE = (220 * 1024) / STAGE_BYTES > 8 ? 8 : (220 * 1024) / STAGE_BYTES;
  // Decode rings.  The weight stream is bound by the bytes a CTA keeps in flight (Little's law:
  // under a full stream a 16 KB tile lands ~3-5 us after its TMA issue; probes streaming the same
  // boxes reach ~6 TB/s with 8 x 16 KB in flight per SM when slots are released at once), so the
  // weight ring takes most of shared memory.  The activations get their own ring, deeper than the
  // weight ring by the k-blocks the MMAs may lag the dequantisers: a TMA load queues behind the
  // weight tiles already issued, so an activation tile must be issued with (or before) its
  // k-block's weight tile; with a shallow ring its slot frees only when an MMA completes, and the
  // tile then landed a full loaded latency after the MMA was due (one stage per ~900 cycles).
  static constexpr int XSTAGES_DEC = BM == 16 ? BW_GEMM_XSTAGES16 : BM == 32 ? 12 : 5;
  static constexpr int STAGES_DEC = (BW_GEMM_DEC_SMEM_KB * 1024 - XSTAGES_DEC * X_BYTES) / W_BYTES;
  static constexpr int STAGES = BM < 128 ? STAGES_DEC : STAGES_PRE;
  static constexpr int XSTAGES = BM < 128 ? XSTAGES_DEC : STAGES_PRE;
  // TMEM: A buffers (64 columns each) between the dequantisers and the MMAs, as many as the
  // double-buffered accumulators (DBUF x NI x BM columns) leave room for, up to 6.
  static constexpr int DBUF = 2;
  static constexpr int AFIT = (512 - DBUF * NI * BM) / 64;
  static constexpr int ASTAGES = AFIT < 6 ? AFIT : 6;
  static constexpr int A_COL0 = 0;
  static constexpr int D_COL0 = ASTAGES * 64;
  static constexpr int TMEM_COLS = 512;
  static constexpr int OFF_W = 0;
  static constexpr int OFF_X = STAGES * W_BYTES;
  static constexpr int OFF_BAR = OFF_X + XSTAGES * X_BYTES;
  static constexpr int BAR_BYTES = 1024;
  static constexpr int OFF_XCH = OFF_BAR + BAR_BYTES;  // SwiGLU epilogue: 64 rows x 16 fp32 (4 KB)
  static constexpr int SMEM = OFF_XCH + 4096 + 1024;
  static constexpr int THREADS = 512;
  static_assert(BM >= 16 && BM <= 128 && BM % 16 == 0, "UMMA N for M=128");
  static_assert(NI >= 1 && NI <= 2, "one or two MMA issuers");
  static_assert(ASTAGES >= 2, "TMEM A buffers");
  static_assert(D_COL0 + DBUF * NI * BM <= TMEM_COLS, "TMEM budget");
  static_assert(SMEM <= 232448, "shared memory budget");
  // barriers, then 32 bytes of slots (TMEM address, abort flag, ticket, epoch, trace record) and the
  // deferred-reduction list (count + two entries of four ints)
  static_assert((2 * STAGES + 2 * XSTAGES + 2 * ASTAGES + 4 + 1) * 8 + 32 + 48 <= BAR_BYTES, "barrier area");
  static_assert(X_PANEL % 1024 == 0 && OFF_X % 1024 == 0, "128-byte swizzled x tiles are 1024-byte aligned");
};

// The workspace starts with a counter region of the same size for every shape,
// so the fp32 pieces of one call never land where another shape keeps counters
// (a workspace is shared by calls of different shapes): counters stay zero at
// rest across any sequence of calls.

// Work schedule of the persistent kernel.  A tile is 128 weight rows x BM tokens
// (M-tile fastest: t = nt * m_tiles + mt) over `kblocks` k-blocks of 128.
//   mode 0  split-K units: unit u = (tile u / splits, k-split u % splits), CTA b
//           takes units b, b + grid, ...; a split tile's piece lives in slot
//           [tile][split]
//   mode 1  stream-K: the tiles' k-blocks laid end to end (tile-major) and cut
//           into `grid` equal contiguous ranges, one per CTA, so every CTA
//           streams the same number of weight bytes whatever the tile count; a
//           tile cut by a range boundary is finished by the CTAs that share it,
//           each writing its piece to slot [cta][0] (the CTA's first segment) or
//           [cta][1] (its last)
// Either way the last CTA to finish a split tile (atomic ticket) sums the
// pieces in k order, so the result does not depend on timing.
struct Sched {
  int mode;
  int n_tiles, m_tiles, kblocks;
  int splits, kb_per_split, units;  // mode 0
  long long work;                   // mode 1: tiles * kblocks
};

// One (tile, k-range) piece of a CTA's work.
struct Seg {
  int t, k0, nkb, split;  // split: k-split index (mode 0); 0 = first / 1 = later segment of the CTA (mode 1)
};

// Stream-K plans keep work * grid below 2^31 (checked by the planner), so the
// range arithmetic is 32-bit.
__host__ __device__ __forceinline__ long long sk_start(long long b, const Sched& s, int grid) {
  return static_cast<long long>(static_cast<unsigned>(b) * static_cast<unsigned>(s.work) / static_cast<unsigned>(grid));
}
// the CTA whose stream-K range holds k-block x of the flattened work
__host__ __device__ __forceinline__ int sk_owner(long long x, const Sched& s, int grid) {
  const unsigned w = static_cast<unsigned>(s.work);
  return static_cast<int>((static_cast<unsigned>(x + 1) * static_cast<unsigned>(grid) + w - 1) / w) - 1;
}

struct SegWalk {
  long long x, end;
  int u, grid;
  bool first;
  __host__ __device__ __forceinline__ SegWalk(const Sched& s, int b, int g) : x(0), end(0), u(b), grid(g), first(true) {
    if (s.mode == 1) {
      x = sk_start(b, s, g);
      end = sk_start(b + 1, s, g);
    }
  }
  __host__ __device__ __forceinline__ bool next(const Sched& s, Seg& sg) {
    if (s.mode == 0) {
      if (u >= s.units) return false;
      sg.split = u % s.splits;
      sg.t = u / s.splits;
      sg.k0 = sg.split * s.kb_per_split;
      sg.nkb = min(s.kb_per_split, s.kblocks - sg.k0);
      u += grid;
      return true;
    }
    if (x >= end) return false;
    const long long kb = s.kblocks;
    sg.t = static_cast<int>(x / kb);
    const long long tile0 = static_cast<long long>(sg.t) * kb;
    sg.k0 = static_cast<int>(x - tile0);
    sg.nkb = static_cast<int>(min(kb, end - tile0)) - sg.k0;
    sg.split = first ? 0 : 1;
    first = false;
    x = tile0 + sg.k0 + sg.nkb;
    return true;
  }
};

// Where the pieces of a cut stream-K tile t live: the first contributor `c_first` (whose counter
// the contributors count on), the number of contributors, and the slot (0: the CTA's first
// segment, 1: a later one) of the first contributor's piece; every later contributor starts its
// range inside the tile, so its piece is in its slot 0.
struct PieceLoc {
  int c_first, n_parts, slot0;
};
__host__ __device__ __forceinline__ PieceLoc sk_pieces(const Sched& s, int t, int grid) {
  const long long kb = s.kblocks;
  PieceLoc p;
  p.c_first = sk_owner(t * kb, s, grid);
  p.n_parts = sk_owner(t * kb + kb - 1, s, grid) - p.c_first + 1;
  p.slot0 = sk_start(p.c_first, s, grid) / kb == t ? 0 : 1;
  return p;
}

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
  kSiteGRecv = 131,
};

// GLU = true: the fused gate/up + SwiGLU variant.  A tile is 64 rows of the gate
// weight and the same 64 rows of the up weight (two 64-row TMA boxes stacked into
// one 128-row stage, so both weights keep the reference's layout); the epilogue's
// up-row warps hand their dt-rounded values to the gate-row warps through shared
// memory, which write y = dt(silu(g) * u) for 64 output columns:
// swiglu(int8_gemm(x, w_gate, s_gate), int8_gemm(x, w_up, s_up)) in one launch
// (reference swiglu_kernel, src/blackwell_ops/cuda/basic_ops.cu:112-122).
template <int BM, bool BF16, bool GLU>
__global__ void __launch_bounds__(512, 1)
    w8a16_persistent_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_w2,
                            const __grid_constant__ CUtensorMap tm_x, const void* __restrict__ scale_in,
                            const void* __restrict__ scale2, int sdtype, void* __restrict__ y_in, int64_t ldy_in,
                            int M, int N_in, const Sched sc, float* __restrict__ ws, int* __restrict__ counters,
                            const __grid_constant__ GatherArgs g, const __grid_constant__ GroupArgs grp) {
  using C = PCfg<BM>;
  constexpr int STAGES = C::STAGES;
  constexpr int XSTAGES = C::XSTAGES;
  constexpr int ASTAGES = C::ASTAGES;
  constexpr int NI = C::NI;
  constexpr int DBUF = C::DBUF;
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
  uint64_t* xfull = final_bar + 1;       // XSTAGES: the x tiles of a k-block (full[] covers its W tile)
  uint64_t* xempty = xfull + XSTAGES;    // XSTAGES: the MMAs that read a k-block's x tiles are done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xempty + XSTAGES);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* ticket = abort_flag + 1;
  volatile uint32_t* sh_epoch = reinterpret_cast<volatile uint32_t*>(tmem_slot + 3);
  unsigned long long** trace_slot = reinterpret_cast<unsigned long long**>(tmem_slot + 4);
  // stream-K tiles this CTA finishes last, reduced by all 512 threads after the main loop:
  // pend[0] = count (<= 2: a CTA's first and last segments), entries {t, n_parts, c_first, poff0}
  volatile int* pend = reinterpret_cast<volatile int*>(tmem_slot + 8);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    *trace_slot = trace_claim(GLU ? 2 : 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 4);       // W tile read into registers by one group of 4 dequantiser warps
    }
    for (int s = 0; s < XSTAGES; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&xempty[s], 1);      // x tiles: a commit by the k-block's issuer
    }
    for (int t = 0; t < ASTAGES; ++t) {
      mbar_init(&afull[t], 4);
      mbar_init(&aempty[t], 1);
    }
    for (int b = 0; b < DBUF; ++b) {
      mbar_init(&dfull[b], NI);
      mbar_init(&dempty[b], 4);
    }
    mbar_init(final_bar, NI);
    *abort_flag = 0;
    pend[0] = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_w);
    for (int pg = 0; pg < grp.count; ++pg) tma_prefetch_desc(&grp.w[pg]);
    if (GLU) tma_prefetch_desc(&tm_w2);
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
  unsigned long long* const trec = *trace_slot;
  if (threadIdx.x == 0) {
    trace_stamp(trec, 0);
    pdl_launch_dependents();
  }

  if (warp == 0) {
    // ---------------- TMA producer: weight tiles ----------------
    // Weights do not depend on the preceding kernel (no griddepcontrol.wait here), and a
    // slot is free as soon as a dequantiser group has read it into registers.
    if (lane == 0) {
      // a weight tile used by several M-tiles stays in L2 for the CTAs that share it
      const uint64_t pol_w = sc.m_tiles > 1 ? l2_policy_evict_normal() : l2_policy_evict_first();
      int it = 0;
      bool ok = true;
      SegWalk wk(sc, blockIdx.x, gridDim.x);
      Seg sg;
      while (ok && wk.next(sc, sg)) {
        const int nt = sg.t / sc.m_tiles;
        for (int i = 0; i < sg.nkb; ++i, ++it) {
          const int s = it % STAGES;
          constexpr int WG = BM < 128 ? BW_GEMM_W_GROUP : BW_GEMM_W_GROUP_PRE;
          if constexpr (WG > 1) {
            // wait for the group's last slot before issuing its first k-block (each slot's own wait follows)
            const int jl = it + min(WG, sg.nkb - i) - 1;
            if (i % WG == 0 && jl >= STAGES &&
                !mbar_wait(&empty[jl % STAGES], ((jl / STAGES) & 1) ^ 1, abort_flag, kSitePProd)) {
              ok = false;
              break;
            }
          }
          if (it >= STAGES && !mbar_wait(&empty[s], ((it / STAGES) & 1) ^ 1, abort_flag, kSitePProd)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], C::W_BYTES);
          if constexpr (GLU) {
            tma_load_2d(sW + s * C::W_BYTES, &tm_w, &full[s], (sg.k0 + i) * C::BK, nt * 64, pol_w);
            tma_load_2d(sW + s * C::W_BYTES + C::W_BYTES / 2, &tm_w2, &full[s], (sg.k0 + i) * C::BK, nt * 64, pol_w);
          } else {
            const CUtensorMap* wm = &tm_w;
            int wrow = nt * 128;
            if (grp.count > 0) {  // grouped launch: the tile's problem and its rows there
              const int pg = group_of(grp, nt);
              wm = &grp.w[pg];
              wrow = (nt - grp.tile0[pg]) * 128;
            }
            tma_load_2d(sW + s * C::W_BYTES, wm, &full[s], (sg.k0 + i) * C::BK, wrow, pol_w);
          }
        }
      }
      if (!ok)  // wait (bounded) for the copies still in flight into this CTA's shared memory
        for (int j = (it > STAGES ? it - STAGES : 0); j < it; ++j)
          mbar_wait(&full[j % STAGES], (j / STAGES) & 1, nullptr, kSitePDrain);
    }
  } else if (warp == 15) {
    // ---------------- TMA producer: activation tiles (after the predecessor) ----------------
    if (lane == 0) {
      const uint64_t pol_x = l2_policy_evict_last();
      pdl_wait();
      int it = 0;
      bool ok = true;
      SegWalk wk(sc, blockIdx.x, gridDim.x);
      Seg sg;
      while (ok && wk.next(sc, sg)) {
        const int mt = sg.t % sc.m_tiles;
        for (int i = 0; i < sg.nkb; ++i, ++it) {
          const int s = it % XSTAGES;
          const int kx = (sg.k0 + i) * C::BK;
          if (it >= XSTAGES && !mbar_wait(&xempty[s], ((it / XSTAGES) & 1) ^ 1, abort_flag, kSitePProd)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&xfull[s], C::X_BYTES);
          tma_load_2d(sX + s * C::X_BYTES, &tm_x, &xfull[s], kx, mt * BM, pol_x);
          tma_load_2d(sX + s * C::X_BYTES + C::X_PANEL, &tm_x, &xfull[s], kx + 64, mt * BM, pol_x);
        }
      }
      if (!ok)
        for (int j = (it > XSTAGES ? it - XSTAGES : 0); j < it; ++j)
          mbar_wait(&xfull[j % XSTAGES], (j / XSTAGES) & 1, nullptr, kSitePDrain);
    }
  } else if (warp == 1 || (NI >= 2 && warp == 14)) {
    // ---------------- MMA issuers ----------------
    if (lane == 0) {
      // Issuer h takes the k-blocks it with it % NI == h, all eight K=16 slices of each, into
      // its own accumulator, so the issuers' MMA streams, waits and commits run side by side.
      // The epilogue adds the accumulators in a fixed order.
      constexpr uint32_t idesc = make_idesc_f16(128, BM, BF16, false);
      const int h = warp == 1 ? 0 : 1;  // issuer index
      int it = 0, j = 0;
      bool ok = true;
      SegWalk wk(sc, blockIdx.x, gridDim.x);
      Seg sg;
      for (; ok && wk.next(sc, sg); ++j) {
        const int b = j % DBUF;
        if (!mbar_wait(&dempty[b], ((j / DBUF) & 1) ^ 1, abort_flag, kSitePMmaD)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + C::D_COL0 + (b * NI + h) * BM;
        uint32_t acc = 0;  // 0 until this issuer's first MMA of the segment
        for (int i = 0; i < sg.nkb; ++i, ++it) {
          if (NI > 1 && it % NI != h) continue;
          const int s = it % XSTAGES;
          const uint32_t ph = (it / XSTAGES) & 1;
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
            umma_f16_ts(d_tmem, tmem + C::A_COL0 + t * 64 + kk * 8, bd, idesc, acc);
            acc = 1u;
          }
          umma_commit(&xempty[s]);
          umma_commit(&aempty[t]);
        }
        if (ok) umma_commit(&dfull[b]);
      }
      // every issued MMA has completed before TMEM is released
      umma_commit(final_bar);
      mbar_wait(final_bar, 0, nullptr, kSitePFinal);
      if (h == 0) trace_stamp(trec, 2);
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
    SegWalk wk(sc, blockIdx.x, gridDim.x);
    Seg sg;
    while (ok && wk.next(sc, sg)) {
      for (int i = 0; i < sg.nkb; ++i, ++it) {
        if ((it & 1) != grp) continue;
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        const int t = it % ASTAGES;
        const uint32_t pa = (it / ASTAGES) & 1;
        if (!mbar_wait(&full[s], ph, abort_flag, kSitePConvFull)) {
          ok = false;
          break;
        }
        if (it == 0 && threadIdx.x == 64) trace_stamp(trec, 1);
        const uint8_t* src = sW + s * C::W_BYTES + row * 128;
        uint32_t out[2][32];
        // The row in registers, then the slot released before the conversion: the OR over every
        // loaded word makes the arrive wait for the loads themselves (an arrive right after
        // issuing them let a fast refill land under reads still in flight).  Releasing here
        // instead of after the conversion measured +2.5 % on the 70B decode shapes (with
        // BW_GEMM_W_GROUP = 4).
        uint4 raw[8];
        uint32_t dep = 0;
#pragma unroll
        for (int c = 0; c < 8; ++c) raw[c] = *reinterpret_cast<const uint4*>(src + ((c ^ sw) << 4));
#pragma unroll
        for (int c = 0; c < 8; ++c) dep |= raw[c].x | raw[c].y | raw[c].z | raw[c].w;
        asm volatile("" ::"r"(dep));  // `dep` (so every load) is complete before the arrive below
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 v = raw[c];
          uint4 o0, o1;
          convert_chunk<BF16>(v, o0, o1);
          uint32_t* o = &out[c >> 2][8 * (c & 3)];
          o[0] = o0.x;
          o[1] = o0.y;
          o[2] = o0.z;
          o[3] = o0.w;
          o[4] = o1.x;
          o[5] = o1.y;
          o[6] = o1.z;
          o[7] = o1.w;
        }
        if (!mbar_wait(&aempty[t], pa ^ 1, abort_flag, kSitePConvA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        tmem_st32(lane_base + t * 64, out[0]);
        tmem_st32(lane_base + t * 64 + 32, out[1]);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&afull[t]);
      }
    }
  } else if (warp < 14) {
    // ---------------- epilogue: warps 10-13 ----------------
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(q * 32) << 16) + C::D_COL0;
    float* xch = reinterpret_cast<float*>(smem + C::OFF_XCH);
    pdl_wait();
    if (warp == 10 && lane == 0) trace_stamp(trec, 7);
    uint32_t epoch = 0;
    if (g.world > 0) {
      // this call's epoch: one past the last completed call's (kept on the device, so a captured
      // graph replays correctly); the last CTA to read it stores it for the next call, which reads
      // it after this grid has completed, and resets the ticket
      if (warp == 10 && lane == 0) {
        uint32_t* mine = reinterpret_cast<uint32_t*>(g.pad[g.rank]);
        const uint32_t e = ld_relaxed_gpu(mine + 1) + 1u;
        if (atomicAdd(mine, 1u) == gridDim.x - 1) {
          atomicExch(mine, 0u);
          atomicExch(mine + 1, e);
        }
        *sh_epoch = e;
        trace_stamp(trec, 5);
      }
      named_bar_sync(1, 128);
      epoch = *sh_epoch;
    }
    int j = 0;
    int it0 = 0;  // this CTA's k-block count before the segment
    SegWalk wk(sc, blockIdx.x, gridDim.x);
    Seg sg;
    for (; wk.next(sc, sg); it0 += sg.nkb, ++j) {
      const int t = sg.t;
      const int nt_all = t / sc.m_tiles;
      const int mt = t - nt_all * sc.m_tiles;
      // the tile's GEMM (a grouped launch holds several) and its n-tile there
      int nt = nt_all;
      const void* scale = scale_in;
      void* y = y_in;
      int64_t ldy = ldy_in;
      int N = N_in;
      if (grp.count > 0) {
        const int pg = group_of(grp, nt_all);
        nt = nt_all - grp.tile0[pg];
        scale = reinterpret_cast<const void*>(grp.scale[pg]);
        y = reinterpret_cast<void*>(grp.y[pg]);
        ldy = grp.ldy[pg];
        N = grp.n[pg];
      }
      // issuer h holds part of this segment iff one of its k-blocks (it % NI == h) lies in it
      auto has = [&](int h) { return sg.nkb >= NI || (h - it0 % NI + NI) % NI < sg.nkb; };
      const int n = GLU ? nt * 64 + (row & 63) : nt * 128 + row;
      const int m0 = mt * BM;
      const void* srow = GLU && row >= 64 ? scale2 : scale;
      const int b = j % DBUF;
      const bool ok = mbar_wait(&dfull[b], (j / DBUF) & 1, abort_flag, kSitePEpi);
      if (named_bar_any(1, 128, !ok || *abort_flag)) break;  // same decision in all 4 warps
      tc_fence_after();
      const uint32_t taddr = lane_addr + b * NI * BM;
      // 16 accumulator columns of this thread's row: the sum over the issuers that took part
      // of the segment, in issuer order (a fixed order, so results do not depend on timing)
      auto load_acc = [&](int c0, float (&v)[16]) {
        bool first = true;
#pragma unroll
        for (int h = 0; h < NI; ++h) {
          if (!has(h)) continue;
          uint32_t r[16];
          tmem_ld16(taddr + h * BM + c0, r);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 16; ++e) v[e] = first ? __uint_as_float(r[e]) : v[e] + __uint_as_float(r[e]);
          first = false;
        }
      };
      // Output of CH consecutive tokens [c0, c0 + CH) of this thread's row, already scaled.
      // SwiGLU: up rows (warps of lane quarters 2, 3) pass dt(up) through shared memory; gate
      // rows write dt(silu(dt(gate)) * dt(up)).  Every epilogue thread calls this (barriers).
      auto emit = [&](const float* v, int c0, auto ch_tag) {
        constexpr int CH = decltype(ch_tag)::value;
        if constexpr (!GLU) {
          if (g.vec || g.world > 0) {
            // Stage the CH x 128 outputs of the chunk as dt values in shared memory (token-major),
            // then store 16-byte rows of 8 outputs: one vector store per 8 outputs instead of eight
            // 2-byte stores (outputs past N or a misaligned Y: element by element).  All-gather:
            // the same 8 outputs go to every peer's mailbox as four {2 outputs, epoch} words.
            uint16_t* st = reinterpret_cast<uint16_t*>(xch);
#pragma unroll
            for (int e = 0; e < CH; ++e) {
              if constexpr (BF16) st[e * 128 + row] = __bfloat16_as_ushort(__float2bfloat16_rn(v[e]));
              else st[e * 128 + row] = __half_as_ushort(__float2half_rn(v[e]));
            }
            named_bar_sync(1, 128);
            const int n0 = nt * 128;
#pragma unroll
            for (int cc = row; cc < CH * 16; cc += 128) {
              const int e = cc >> 4, c8 = (cc & 15) * 8;
              const int m = m0 + c0 + e;
              if (m < M) {
                const uint4 val = *reinterpret_cast<const uint4*>(st + e * 128 + c8);
                if (g.world > 0) {
                  const size_t off = (static_cast<size_t>((epoch & 1u) * g.world + g.rank) * M + m) * g.rowwords +
                                     ((n0 + c8) >> 1);
                  for (int r = 0; r < g.world; ++r) {
                    if (r == g.rank) continue;
                    uint64_t* mb = reinterpret_cast<uint64_t*>(g.pad[r] + kMailbox0) + off;
                    st_ll2(mb, val.x, val.y, epoch);
                    st_ll2(mb + 2, val.z, val.w, epoch);
                  }
                }
                const int64_t idx = static_cast<int64_t>(m) * ldy + n0 + c8;
                if (g.vec && n0 + c8 + 8 <= N) {
                  store_y8(y, idx, val);
                } else {
                  const uint16_t* h = reinterpret_cast<const uint16_t*>(&val);
                  for (int q8 = 0; q8 < 8 && n0 + c8 + q8 < N; ++q8) static_cast<uint16_t*>(y)[idx + q8] = h[q8];
                }
              }
            }
            named_bar_sync(1, 128);  // the stage is read before the next chunk overwrites it
          } else if (n < N) {
#pragma unroll
            for (int e = 0; e < CH; ++e) {
              const int m = m0 + c0 + e;
              if (m < M) store_y<BF16>(y, ldy, m, n, v[e]);
            }
          }
        } else {
          if (row >= 64) {
#pragma unroll
            for (int e = 0; e < CH; ++e) xch[(row - 64) * 16 + e] = round_out<BF16>(v[e]);
          }
          named_bar_sync(1, 128);
          if (row < 64 && n < N) {
#pragma unroll
            for (int e = 0; e < CH; ++e) {
              const int m = m0 + c0 + e;
              const float gt = round_out<BF16>(v[e]);
              const float up = xch[row * 16 + e];
              if (m < M) store_y<BF16>(y, ldy, m, n, gt / (1.0f + expf(-gt)) * up);
            }
          }
          named_bar_sync(1, 128);  // the buffer is read before the next chunk overwrites it
        }
      };
      if (sg.nkb == sc.kblocks) {  // this CTA computes the tile's full K
        const float scl = n < N ? load_as_float(srow, n, sdtype) : 0.f;
#pragma unroll 1
        for (int c0 = 0; c0 < BM; c0 += 16) {
          float v[16];
          load_acc(c0, v);
#pragma unroll
          for (int e = 0; e < 16; ++e) v[e] *= scl;
          emit(v, c0, std::integral_constant<int, 16>{});
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&dempty[b]);
      } else {
        // piece slots: [tile][split] (mode 0) or [cta][first/last segment] (mode 1)
        const PieceLoc loc = sc.mode == 0 ? PieceLoc{0, sc.splits, 0} : sk_pieces(sc, t, gridDim.x);
        const int c_first = loc.c_first;
        const int n_parts = loc.n_parts;
        // piece c of the tile sits at base + c * stride (+ off0 for piece 0): in mode 1 every
        // contributor after the first starts its range inside the tile (its slot 0), and only
        // the first may hold the tile as its last segment (slot 1).  Branch-free addresses keep
        // the reduction's loads of four pieces in flight together.
        constexpr size_t kPiece = static_cast<size_t>(128) * BM;
        const float* pbase;
        size_t pstride, poff0 = 0;
        if (sc.mode == 0) {
          pbase = ws + static_cast<size_t>(t) * sc.splits * kPiece + static_cast<size_t>(row) * BM;
          pstride = kPiece;
        } else {
          pbase = ws + static_cast<size_t>(c_first) * 2 * kPiece + static_cast<size_t>(row) * BM;
          pstride = 2 * kPiece;
          poff0 = loc.slot0 ? kPiece : 0;
        }
        // tile counter: the tile itself (mode 0) or the CTA holding its first k-block, which
        // heads at most one cut tile (mode 1); either way an index below kGemmCounterSlots
        const int cidx = sc.mode == 0 ? t : c_first;
        float* mine = ws + (sc.mode == 0 ? static_cast<size_t>(t) * sc.splits + sg.split
                                         : static_cast<size_t>(blockIdx.x) * 2 + sg.split) * kPiece +
                      static_cast<size_t>(row) * BM;
#pragma unroll 1
        for (int c0 = 0; c0 < BM; c0 += 16) {
          float v[16];
          load_acc(c0, v);
#pragma unroll
          for (int e = 0; e < 16; e += 4)
            *reinterpret_cast<float4*>(mine + c0 + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&dempty[b]);  // accumulator free; the piece is in global memory
        __threadfence();
        named_bar_sync(1, 128);
        if (warp == 10 && lane == 0) *ticket = atomicAdd(&counters[cidx], 1);
        named_bar_sync(1, 128);
        const bool last = *ticket == n_parts - 1;
        named_bar_sync(1, 128);  // every thread has read the ticket before the next segment overwrites it
        if (!GLU && sc.mode == 1 && last) {
          // the whole CTA sums this tile's pieces after the main loop
          if (warp == 10 && lane == 0) {
            const int i = pend[0];
            pend[1 + 4 * i] = t;
            pend[2 + 4 * i] = n_parts;
            pend[3 + 4 * i] = c_first;
            pend[4 + 4 * i] = static_cast<int>(poff0);
            pend[0] = i + 1;
          }
        } else if (last) {
          __threadfence();
          const float scl = n < N ? load_as_float(srow, n, sdtype) : 0.f;
          // 8 columns at a time; the loads of four pieces are issued together, then summed
          // in k order (piece 0 first, as the result must not depend on timing).  Issuing
          // 16 columns of four pieces at once measured slower (register-bound load batching).
#pragma unroll 1
          for (int c0 = 0; c0 < BM; c0 += 8) {
            float a[8];
#pragma unroll 1
            for (int p0 = 0; p0 < n_parts; p0 += 4) {
              float4 v[4][2];
#pragma unroll
              for (int pp = 0; pp < 4; ++pp)
#pragma unroll
                for (int e = 0; e < 2; ++e)
                  v[pp][e] = p0 + pp < n_parts
                                 ? __ldcg(reinterpret_cast<const float4*>(pbase + (p0 + pp) * pstride +
                                                                          (p0 + pp == 0 ? poff0 : 0) + c0 + 4 * e))
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
              for (int pp = 0; pp < 4; ++pp) {
                if (p0 + pp >= n_parts) break;
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                  const float f[4] = {v[pp][e].x, v[pp][e].y, v[pp][e].z, v[pp][e].w};
#pragma unroll
                  for (int g = 0; g < 4; ++g) a[4 * e + g] = (p0 + pp == 0) ? f[g] : a[4 * e + g] + f[g];
                }
              }
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) a[e] *= scl;
            emit(a, c0, std::integral_constant<int, 8>{});
          }
          if (warp == 10 && lane == 0) counters[cidx] = 0;
        }
      }
    }
    if (warp == 10 && lane == 0) trace_stamp(trec, 3);
  }

  // ---------------- all 512 threads, after the main loop ----------------
  // (1) The stream-K tiles this CTA finished last: their pieces (up to ~20 at small per-rank N)
  //     are summed with a float4 per thread and all loads of a batch in flight, in k order
  //     (piece 0 first), so the result is the in-loop reduction's, bit for bit.
  // (2) All-gather receive: the (tile, peer) pairs are dealt to the CTAs round robin (the same on
  //     every rank; which peer CTA produced a tile does not matter).  A word belongs to this call
  //     when its epoch does; stale words (an older call of this parity) never do.  Bounded: a peer
  //     that never sends records the site and stops this CTA's receive.
  // A CTA sends all it owns (its tiles and these reductions) before it receives anything.
  if constexpr (!GLU) {
    if (sc.mode == 1 || g.world > 0) {
      __syncthreads();  // the pending list, the producers' drained rings
      if (!__syncthreads_or(*abort_flag != 0)) {
        const int tid = threadIdx.x;
        const uint32_t ep = g.world > 0 ? *sh_epoch : 0u;
        const int npend = pend[0];
        uint16_t* stage = reinterpret_cast<uint16_t*>(sW);  // the weight ring is idle now
        fence_proxy_async_smem();                          // its last writer was the TMA engine
        constexpr size_t kPiece = static_cast<size_t>(128) * BM;
        constexpr int kRedBatch = BW_GEMM_RED_BATCH;  // pieces loaded together per thread
        for (int i = 0; i < npend; ++i) {
          const int t = pend[1 + 4 * i], n_parts = pend[2 + 4 * i], c_first = pend[3 + 4 * i];
          const size_t poff0 = static_cast<size_t>(pend[4 + 4 * i]);
          const int nt_all = t / sc.m_tiles;
          const int m0 = (t - nt_all * sc.m_tiles) * BM;
          int nt = nt_all;
          const void* scale = scale_in;
          void* y = y_in;
          int64_t ldy = ldy_in;
          int N = N_in;
          if (grp.count > 0) {
            const int pg = group_of(grp, nt_all);
            nt = nt_all - grp.tile0[pg];
            scale = reinterpret_cast<const void*>(grp.scale[pg]);
            y = reinterpret_cast<void*>(grp.y[pg]);
            ldy = grp.ldy[pg];
            N = grp.n[pg];
          }
          const float* base = ws + static_cast<size_t>(c_first) * 2 * kPiece;
          __threadfence();  // the contributors' pieces, published before their tickets
          for (int f = tid; f < 32 * BM; f += C::THREADS) {
            const int r = f / (BM / 4), c4 = (f % (BM / 4)) * 4;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
            for (int p0 = 0; p0 < n_parts; p0 += kRedBatch) {
              float4 v[kRedBatch];
#pragma unroll
              for (int pp = 0; pp < kRedBatch; ++pp)
                if (p0 + pp < n_parts)
                  v[pp] = __ldcg(reinterpret_cast<const float4*>(base + (p0 + pp) * 2 * kPiece +
                                                                 (p0 + pp == 0 ? poff0 : 0) + r * BM + c4));
#pragma unroll
              for (int pp = 0; pp < kRedBatch; ++pp) {
                if (p0 + pp >= n_parts) break;
                if (p0 + pp == 0) {
                  acc = v[0];
                } else {
                  acc.x += v[pp].x;
                  acc.y += v[pp].y;
                  acc.z += v[pp].z;
                  acc.w += v[pp].w;
                }
              }
            }
            const int n = nt * 128 + r;
            const float scl = n < N ? load_as_float(scale, n, sdtype) : 0.f;
            const float o[4] = {acc.x * scl, acc.y * scl, acc.z * scl, acc.w * scl};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              if constexpr (BF16) stage[(c4 + e) * 128 + r] = __bfloat16_as_ushort(__float2bfloat16_rn(o[e]));
              else stage[(c4 + e) * 128 + r] = __half_as_ushort(__float2half_rn(o[e]));
            }
          }
          __syncthreads();
          const int n0 = nt * 128;
          for (int cc = tid; cc < BM * 16; cc += C::THREADS) {
            const int e = cc >> 4, c8 = (cc & 15) * 8;
            const int m = m0 + e;
            if (m >= M) continue;
            const uint4 val = *reinterpret_cast<const uint4*>(stage + e * 128 + c8);
            if (g.world > 0) {
              const size_t off =
                  (static_cast<size_t>((ep & 1u) * g.world + g.rank) * M + m) * g.rowwords + ((n0 + c8) >> 1);
              for (int q = 0; q < g.world; ++q) {
                if (q == g.rank) continue;
                uint64_t* mb = reinterpret_cast<uint64_t*>(g.pad[q] + kMailbox0) + off;
                st_ll2(mb, val.x, val.y, ep);
                st_ll2(mb + 2, val.z, val.w, ep);
              }
            }
            const int64_t idx = static_cast<int64_t>(m) * ldy + n0 + c8;
            if (g.vec && n0 + c8 + 8 <= N) {
              store_y8(y, idx, val);
            } else {
              const uint16_t* h = reinterpret_cast<const uint16_t*>(&val);
              for (int q8 = 0; q8 < 8 && n0 + c8 + q8 < N; ++q8) static_cast<uint16_t*>(y)[idx + q8] = h[q8];
            }
          }
          __syncthreads();  // the stage is read before the next tile overwrites it
          if (tid == 0) counters[c_first] = 0;
        }
        if (tid == 0) trace_stamp(trec, 4);
        if (g.world > 0) {
          const int peers = g.world - 1;
          const int tiles = sc.m_tiles * sc.n_tiles;
          const uint64_t* mbox = reinterpret_cast<const uint64_t*>(g.pad[g.rank] + kMailbox0);
          const long long limit = wait_limit_cycles();
          const long long tw0 = clock64();
          bool ok = true;
          for (int q = blockIdx.x; ok && q < tiles * peers; q += gridDim.x) {
            const int t = q / peers;
            const int p = q - t * peers + (q - t * peers >= g.rank ? 1 : 0);
            const int nt = t / sc.m_tiles, mt = t - nt * sc.m_tiles;
            const int rows = min(BM, M - mt * BM);
            const uint64_t* src =
                mbox + (static_cast<size_t>((ep & 1u) * g.world + p) * M + mt * BM) * g.rowwords + nt * 64;
            uint16_t* dst = reinterpret_cast<uint16_t*>(g.ybase) + static_cast<int64_t>(mt * BM) * ldy_in +
                            static_cast<int64_t>(p) * g.n + nt * 128;
            const int cols = min(128, g.n - nt * 128);
            // 2 words (4 outputs) per thread per load, four loads in flight
            for (int w0 = tid * 2; ok && w0 < rows * 64; w0 += 4 * 2 * C::THREADS) {
              unsigned long long v[4][2];
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int w = w0 + i * 2 * C::THREADS;
                if (w < rows * 64) ld_ll2(src + static_cast<size_t>(w >> 6) * g.rowwords + (w & 63), v[i][0], v[i][1]);
              }
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int w = w0 + i * 2 * C::THREADS;
                if (!ok || w >= rows * 64) continue;  // no break: the loop stays unrolled, v in registers
                const uint64_t* a = src + static_cast<size_t>(w >> 6) * g.rowwords + (w & 63);
                while (static_cast<uint32_t>(v[i][0] >> 32) != ep || static_cast<uint32_t>(v[i][1] >> 32) != ep) {
                  if (clock64() - tw0 > limit) {
                    record_timeout(kSiteGRecv);
                    *abort_flag = 1;
                    ok = false;
                    break;
                  }
                  ld_ll2(a, v[i][0], v[i][1]);
                }
                if (!ok) continue;
                // 4 outputs: token w / 64, columns 2 (w % 64) .. + 3 of the tile
                const int c = 2 * (w & 63);
                uint16_t* d = dst + static_cast<int64_t>(w >> 6) * ldy_in + c;
                const uint32_t lo = static_cast<uint32_t>(v[i][0]), hi = static_cast<uint32_t>(v[i][1]);
                if (g.vec4 && c + 4 <= cols) {
                  *reinterpret_cast<uint2*>(d) = make_uint2(lo, hi);
                } else {
                  const uint16_t h4[4] = {static_cast<uint16_t>(lo), static_cast<uint16_t>(lo >> 16),
                                          static_cast<uint16_t>(hi), static_cast<uint16_t>(hi >> 16)};
                  for (int u = 0; u < 4 && c + u < cols; ++u) d[u] = h4[u];
                }
              }
            }
          }
          __syncthreads();
          if (tid == 0) trace_stamp(trec, 6);
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

// CUDA-core fallback of the fused gate/up + SwiGLU op: one thread per output.
template <bool BF16>
__global__ void __launch_bounds__(128) w8a16_swiglu_simt_kernel(const void* __restrict__ x, int64_t ldx,
                                                                const int8_t* __restrict__ wg,
                                                                const int8_t* __restrict__ wu, int64_t ldw,
                                                                const void* __restrict__ sg,
                                                                const void* __restrict__ su, int sdtype,
                                                                void* __restrict__ y, int64_t ldy, int M, int N,
                                                                int K) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  const int m = blockIdx.y;
  if (n >= N || m >= M) return;
  const int xdt = BF16 ? BW_DTYPE_BF16 : BW_DTYPE_F16;
  float ag = 0.f, au = 0.f;
  for (int k = 0; k < K; ++k) {
    const float xv = load_as_float(x, static_cast<int64_t>(m) * ldx + k, xdt);
    ag = fmaf(xv, static_cast<float>(wg[static_cast<int64_t>(n) * ldw + k]), ag);
    au = fmaf(xv, static_cast<float>(wu[static_cast<int64_t>(n) * ldw + k]), au);
  }
  const float gt = round_out<BF16>(ag * load_as_float(sg, n, sdtype));
  const float up = round_out<BF16>(au * load_as_float(su, n, sdtype));
  store_out<BF16>(y, static_cast<int64_t>(m) * ldy + n, gt / (1.0f + expf(-gt)) * up);
}

// ---------------------------------------------------------------------------
// host planning
// ---------------------------------------------------------------------------
struct GemmPlan {
  int bm = 16;
  int n_tiles = 0, m_tiles = 0, kblocks = 0, splits = 1, kb_per_split = 0, units = 0, grid = 0;
  int mode = 0;         // 0: split-K units, 1: stream-K ranges
  long long work = 0;   // tiles * kblocks
  size_t counter_bytes = 0, partial_bytes = 0;
};

// Persistent path.  Cost model: the busiest CTA's work, counting each k-block as
// 16 KB of weights, each unit or segment a fixed overhead (epilogue, pipeline
// hand-off) and each fp32 piece written a round trip.  Split-K (mode 0) picks
// the split count; when CTAs would walk several units each, stream-K (mode 1)
// removes the last round's imbalance (e.g. 1187 LM-head tiles on 148 SMs:
// 9 units for some CTAs against 8.02 on average).
// gather = true (the fused all-gather): stream-K over all SMs whatever the shape, so every rank
// runs the same grid (its CTAs pair up with the peers' CTAs of the same index).
static GemmPlan plan_gemm(int64_t m, int64_t n, int64_t k, bool glu = false, bool gather = false) {
  GemmPlan p;
  const int sms = num_sms();
  const int rows = glu ? 64 : 128;  // output columns per tile
  p.n_tiles = static_cast<int>((n + rows - 1) / rows);
  p.kblocks = static_cast<int>((k + 127) / 128);
  p.bm = m <= 16 ? 16 : m <= 32 ? 32 : m <= 64 ? 64 : 128;
  p.m_tiles = static_cast<int>((m + p.bm - 1) / p.bm);
  const int64_t tiles = static_cast<int64_t>(p.n_tiles) * p.m_tiles;
#ifndef BW_GEMM_PART_COST_SCALE
#define BW_GEMM_PART_COST_SCALE 1.0
#endif
  const double part_cost = BW_GEMM_PART_COST_SCALE * 2.0 * 128 * p.bm * 4;
  // Small decode GEMMs (at most 8 k-blocks per CTA even on `cap` CTAs, e.g. every Qwen3-0.6B
  // projection) use at most `cap` CTAs: they are bound by per-launch latency, and the SMs left
  // over host the next launch's CTAs, which stream their weights while this launch finishes
  // (programmatic dependent launch).  32 measured cfg1 415 -> 567 GB/s, cfg3 337 -> 425 GB/s
  // against all 148 SMs.
#ifndef BW_GEMM_SPLITK_CAP
#define BW_GEMM_SPLITK_CAP 32
#endif
  const int64_t work_kb = tiles * p.kblocks;
  const int cap = p.bm < 128 && BW_GEMM_SPLITK_CAP > 0 && BW_GEMM_SPLITK_CAP < sms &&
                          work_kb <= 8LL * BW_GEMM_SPLITK_CAP
                      ? BW_GEMM_SPLITK_CAP
                      : sms;
  double best = 1e300;
  int64_t best_per_cta = 1;
  for (int sp = 1; sp <= p.kblocks && sp <= 32; ++sp) {
    const int kbps = (p.kblocks + sp - 1) / sp;
    const int real = (p.kblocks + kbps - 1) / kbps;
    if (real != sp) continue;
    const int64_t units = tiles * sp;
    const int64_t per_cta = (units + cap - 1) / cap;
    const double unit_cost = kbps * 16384.0 + 6000.0 + (sp > 1 ? part_cost : 0.0);
    const double cost = static_cast<double>(per_cta) * unit_cost;
    if (cost < best * 0.97) {
      best = cost;
      best_per_cta = per_cta;
      p.splits = sp;
      p.kb_per_split = kbps;
    }
  }
  p.work = tiles * p.kblocks;
  // split-K counters are per tile: more split tiles than counter slots go to stream-K
  const bool force_sk = p.splits > 1 && tiles > kGemmCounterSlots;
  // prefill tiles (BM = 128) keep split-K units unless forced: measured 809 against 784 TFLOPS on
  // the Llama-3-8B MLP, as the 64 KB pieces of cut tiles and their end-of-range reductions cost
  // more than the last round's imbalance
  if (BW_GEMM_STREAMK && ((best_per_cta >= 2 && p.bm < 128) || force_sk || gather) &&
      (p.work >= sms || gather) && p.work * sms < (1LL << 31)) {
    const int64_t per = (p.work + sms - 1) / sms;
    const double seg = static_cast<double>((per + p.kblocks - 1) / p.kblocks + 1);
    const double cost = per * 16384.0 + seg * 6000.0 + 2.0 * part_cost;
    if (cost < best || force_sk || gather) {
      // every CTA's range must hold at least one k-block (the owner arithmetic assumes it), so
      // a gather plan with less work than SMs runs one CTA per k-block
      const int grid = p.work < sms ? static_cast<int>(p.work) : sms;
      p.mode = 1;
      p.grid = grid;
      p.splits = 1;
      p.kb_per_split = p.kblocks;
      p.units = 0;
      bool cut = false;  // does a range boundary fall inside a tile?
      for (int b = 1; b < grid && !cut; ++b) cut = (static_cast<int64_t>(b) * p.work / grid) % p.kblocks != 0;
      if (cut) {
        p.counter_bytes = kGemmCounterBytes;
        p.partial_bytes = static_cast<size_t>(grid) * 2 * 128 * p.bm * sizeof(float);
      }
      return p;
    }
  }
  const int64_t units = tiles * p.splits;
  p.units = units > INT32_MAX ? -1 : static_cast<int>(units);  // -1: too many units (refused by the caller)
  p.grid = units < cap ? static_cast<int>(units) : cap;
  if (p.splits > 1) {
    if (tiles > kGemmCounterSlots) {  // unreachable for realistic shapes: work < sms with > 1024 tiles
      p.splits = 1;
      p.kb_per_split = p.kblocks;
      p.units = tiles > INT32_MAX ? -1 : static_cast<int>(tiles);
      p.grid = tiles < sms ? static_cast<int>(tiles) : sms;
      return p;
    }
    p.counter_bytes = kGemmCounterBytes;
    p.partial_bytes = static_cast<size_t>(tiles) * p.splits * 128 * p.bm * sizeof(float);
  }
  return p;
}

static bool g_use_pdl = true;

template <int BM, bool BF16, bool GLU>
static int launch_persistent(const GemmPlan& p, const CUtensorMap& tw, const CUtensorMap& tw2, const CUtensorMap& tx,
                             const void* scale, const void* scale2, int sdt, void* y, int64_t ldy, int M, int N,
                             float* ws, int* counters, const GatherArgs& g, const GroupArgs& grp, cudaStream_t st) {
  using C = PCfg<BM>;
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t attr_err = cudaSuccess;
  std::call_once(once[dev & 63], [&] {
    attr_err = cudaFuncSetAttribute(w8a16_persistent_kernel<BM, BF16, GLU>, cudaFuncAttributeMaxDynamicSharedMemorySize,
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
  Sched sc;
  sc.mode = p.mode;
  sc.n_tiles = p.n_tiles;
  sc.m_tiles = p.m_tiles;
  sc.kblocks = p.kblocks;
  sc.splits = p.splits;
  sc.kb_per_split = p.kb_per_split;
  sc.units = p.units;
  sc.work = p.work;
  return check_cuda(cudaLaunchKernelEx(&cfg, w8a16_persistent_kernel<BM, BF16, GLU>, tw, tw2, tx, scale, scale2, sdt,
                                       y, ldy, M, N, sc, ws, counters, g, grp),
                    "cudaLaunchKernelEx(w8a16_persistent_kernel)");
}

template <bool BF16, bool GLU>
static int dispatch_gemm(const GemmPlan& p, const CUtensorMap& tw, const CUtensorMap& tw2, const CUtensorMap& tx,
                         const void* scale, const void* scale2, int sdt, void* y, int64_t ldy, int M, int N, float* ws,
                         int* counters, const GatherArgs& g, const GroupArgs& grp, cudaStream_t st) {
  switch (p.bm) {
    case 16:
      return launch_persistent<16, BF16, GLU>(p, tw, tw2, tx, scale, scale2, sdt, y, ldy, M, N, ws, counters, g, grp, st);
    case 32:
      return launch_persistent<32, BF16, GLU>(p, tw, tw2, tx, scale, scale2, sdt, y, ldy, M, N, ws, counters, g, grp, st);
    case 64:
      return launch_persistent<64, BF16, GLU>(p, tw, tw2, tx, scale, scale2, sdt, y, ldy, M, N, ws, counters, g, grp, st);
    default:
      return launch_persistent<128, BF16, GLU>(p, tw, tw2, tx, scale, scale2, sdt, y, ldy, M, N, ws, counters, g, grp,
                                               st);
  }
}

static const GroupArgs& no_group() {
  static const GroupArgs z = {};
  return z;
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

extern "C" size_t bw_w8a16_gemm_allgather_workspace_size(int64_t m, int64_t n, int64_t k) {
  if (m <= 0 || n <= 0 || k <= 0) return 0;
  const bw::GemmPlan p = bw::plan_gemm(m, n, k, false, true);
  return p.counter_bytes + p.partial_bytes;
}

extern "C" size_t bw_w8a16_gemm_workspace_zeroed_bytes(int64_t m, int64_t n, int64_t k) {
  if (m <= 0 || n <= 0 || k <= 0) return 0;
  return bw::plan_gemm(m, n, k).counter_bytes;
}

namespace bw {
// w2 / scale2 non-null: the fused gate (w, scale) / up (w2, scale2) + SwiGLU op.
static int gemm_impl(const void* x, int x_dtype, int64_t ldx, const int8_t* w, int64_t ldw, const void* scale,
                     int scale_dtype, void* y, int64_t ldy, int64_t m, int64_t n, int64_t k, void* workspace,
                     size_t workspace_bytes, const GatherArgs& g, void* stream, const int8_t* w2 = nullptr,
                     const void* scale2 = nullptr, const GroupArgs* grp = nullptr) {
  const bool glu = w2 != nullptr;
  if (m < 0 || n < 0 || k < 1)
    return fail(BW_ERR_INVALID_ARGUMENT, "int8_gemm: need m, n >= 0 and k >= 1 (got %lld, %lld, %lld)",
                (long long)m, (long long)n, (long long)k);
  if (x_dtype != BW_DTYPE_F16 && x_dtype != BW_DTYPE_BF16)
    return fail(BW_ERR_INVALID_ARGUMENT, "int8_gemm: x must be fp16 or bf16 (dtype %d)", x_dtype);
  if (scale_dtype < BW_DTYPE_F16 || scale_dtype > BW_DTYPE_F32)
    return fail(BW_ERR_INVALID_ARGUMENT, "int8_gemm: unsupported scale dtype %d", scale_dtype);
  if (m == 0 || n == 0) return BW_OK;
  if (!x || !w || !scale || !y) return fail(BW_ERR_INVALID_ARGUMENT, "int8_gemm: null pointer");
  if (glu && !scale2) return fail(BW_ERR_INVALID_ARGUMENT, "int8_gemm_swiglu: null pointer");
  if (glu && g.world > 0) return fail(BW_ERR_UNSUPPORTED, "int8_gemm_swiglu: no all-gather variant");
  if (ldx < k || ldw < k || (grp == nullptr && ldy < n))
    return fail(BW_ERR_INVALID_ARGUMENT, "int8_gemm: row stride too small");
  if (m > (1LL << 30) || n > (1LL << 30) || k > (1LL << 30))
    return fail(BW_ERR_INVALID_ARGUMENT, "int8_gemm: dimension too large");
  if (int s = require_sm100()) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool bf16 = x_dtype == BW_DTYPE_BF16;

  if (!tma_ok(x, ldx * 2) || !tma_ok(w, ldw) || (glu && !tma_ok(w2, ldw))) {
    if (g.world > 0)
      return fail(BW_ERR_UNSUPPORTED, "int8_gemm (all-gather): x and w must be 16-byte aligned with 16-byte row strides");
    dim3 grid(static_cast<unsigned>((n + 127) / 128), static_cast<unsigned>(m));
    if (glu) {
      if (bf16)
        w8a16_swiglu_simt_kernel<true><<<grid, 128, 0, st>>>(x, ldx, w, w2, ldw, scale, scale2, scale_dtype, y, ldy,
                                                             (int)m, (int)n, (int)k);
      else
        w8a16_swiglu_simt_kernel<false><<<grid, 128, 0, st>>>(x, ldx, w, w2, ldw, scale, scale2, scale_dtype, y, ldy,
                                                              (int)m, (int)n, (int)k);
      return check_launch("w8a16_swiglu_simt_kernel");
    }
    if (bf16)
      w8a16_simt_kernel<true><<<grid, 128, 0, st>>>(x, ldx, w, ldw, scale, scale_dtype, y, ldy, (int)m, (int)n, (int)k);
    else
      w8a16_simt_kernel<false><<<grid, 128, 0, st>>>(x, ldx, w, ldw, scale, scale_dtype, y, ldy, (int)m, (int)n, (int)k);
    return check_launch("w8a16_simt_kernel");
  }

  const GemmPlan p = plan_gemm(m, n, k, glu, g.world > 0);
  if (p.units < 0) return fail(BW_ERR_INVALID_ARGUMENT, "int8_gemm: m=%lld n=%lld is too many output tiles",
                               (long long)m, (long long)n);
  if (g.world > 0 && p.mode != 1)
    return fail(BW_ERR_UNSUPPORTED, "int8_gemm (all-gather): shape m=%lld n=%lld k=%lld has no stream-K plan",
                (long long)m, (long long)n, (long long)k);
  float* ws = nullptr;
  int* counters = nullptr;
  if (p.partial_bytes > 0) {
    if (workspace == nullptr || workspace_bytes < p.counter_bytes + p.partial_bytes)
      return fail(BW_ERR_WORKSPACE, "int8_gemm: workspace of %zu bytes required, %zu given",
                  p.counter_bytes + p.partial_bytes, workspace_bytes);
    if (reinterpret_cast<uintptr_t>(workspace) % 16 != 0)
      return fail(BW_ERR_WORKSPACE, "int8_gemm: workspace must be 16-byte aligned");
    counters = static_cast<int*>(workspace);
    ws = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + p.counter_bytes);
  }
  CUtensorMap tw, tw2, tx;
  if (grp != nullptr) {
    tw = grp->w[0];  // the grouped kernel reads its problems' maps; this one is not used
  } else if (int s = make_tmap_2d(&tw, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, n, k, ldw, glu ? 64 : 128, 128,
                                  CU_TENSOR_MAP_SWIZZLE_128B)) {
    return s;
  }
  if (glu) {
    if (int s = make_tmap_2d(&tw2, w2, CU_TENSOR_MAP_DATA_TYPE_UINT8, n, k, ldw, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B))
      return s;
  } else {
    tw2 = tw;  // unused
  }
  if (int s = make_tmap_2d(&tx, x, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, m, k,
                           ldx * 2, p.bm, 64, CU_TENSOR_MAP_SWIZZLE_128B))
    return s;
  if (glu) {
    if (bf16)
      return dispatch_gemm<true, true>(p, tw, tw2, tx, scale, scale2, scale_dtype, y, ldy, (int)m, (int)n, ws, counters,
                                       g, no_group(), st);
    return dispatch_gemm<false, true>(p, tw, tw2, tx, scale, scale2, scale_dtype, y, ldy, (int)m, (int)n, ws, counters,
                                      g, no_group(), st);
  }
  const GroupArgs& ga = grp != nullptr ? *grp : no_group();
  if (bf16)
    return dispatch_gemm<true, false>(p, tw, tw2, tx, scale, scale, scale_dtype, y, ldy, (int)m, (int)n, ws, counters,
                                      g, ga, st);
  return dispatch_gemm<false, false>(p, tw, tw2, tx, scale, scale, scale_dtype, y, ldy, (int)m, (int)n, ws, counters,
                                     g, ga, st);
}
}  // namespace bw

extern "C" int bw_w8a16_gemm(const void* x, int x_dtype, int64_t ldx, const int8_t* w, int64_t ldw,
                             const void* scale, int scale_dtype, void* y, int64_t ldy, int64_t m, int64_t n,
                             int64_t k, void* workspace, size_t workspace_bytes, void* stream) {
  bw::GatherArgs g = {};
  g.vec = reinterpret_cast<uintptr_t>(y) % 16 == 0 && ldy % 8 == 0;
  return bw::gemm_impl(x, x_dtype, ldx, w, ldw, scale, scale_dtype, y, ldy, m, n, k, workspace, workspace_bytes, g,
                       stream);
}

// Grouped W8A16 GEMM: up to kMaxGroup GEMMs sharing x (y_i = x @ (w_i * scale_i)^T, e.g. the q/k/v
// projections of a layer) in one persistent launch over the union of their tiles.
namespace bw {
static bool group_shape_ok(const int64_t* n, int count, int64_t* tiles) {
  if (count < 1 || count > kMaxGroup || n == nullptr) return false;
  int64_t t = 0;
  for (int i = 0; i < count; ++i) {
    if (n[i] < 1 || n[i] > (1LL << 30)) return false;
    t += (n[i] + 127) / 128;
  }
  *tiles = t;
  return true;
}
}  // namespace bw

extern "C" size_t bw_w8a16_gemm_grouped_workspace_size(int64_t m, const int64_t* n, int count, int64_t k) {
  int64_t tiles = 0;
  if (m <= 0 || k <= 0 || !bw::group_shape_ok(n, count, &tiles)) return 0;
  // the union's plan, or (layouts TMA cannot address) the largest single GEMM's
  size_t need = bw_w8a16_gemm_workspace_size(m, 128 * tiles, k);
  for (int i = 0; i < count; ++i) need = std::max(need, bw_w8a16_gemm_workspace_size(m, n[i], k));
  return need;
}

extern "C" int bw_w8a16_gemm_grouped(const void* x, int x_dtype, int64_t ldx, int count, const int8_t* const* w,
                                     const int64_t* ldw, const void* const* scale, int scale_dtype, void* const* y,
                                     const int64_t* ldy, const int64_t* n, int64_t m, int64_t k, void* workspace,
                                     size_t workspace_bytes, void* stream) {
  using namespace bw;
  int64_t tiles = 0;
  if (!group_shape_ok(n, count, &tiles) || !w || !ldw || !scale || !y || !ldy)
    return fail(BW_ERR_INVALID_ARGUMENT, "int8_gemm_grouped: need 1..%d problems with n >= 1 and their arrays",
                kMaxGroup);
  if (m < 0 || k < 1) return fail(BW_ERR_INVALID_ARGUMENT, "int8_gemm_grouped: need m >= 0 and k >= 1");
  for (int i = 0; i < count; ++i) {
    if (!w[i] || !scale[i] || !y[i])
      return fail(BW_ERR_INVALID_ARGUMENT, "int8_gemm_grouped: null pointer (problem %d)", i);
    if (ldw[i] < k || ldy[i] < n[i])
      return fail(BW_ERR_INVALID_ARGUMENT, "int8_gemm_grouped: row stride too small (problem %d)", i);
  }
  if (m == 0) return BW_OK;
  bool tma = tma_ok(x, ldx * 2);
  for (int i = 0; i < count; ++i) tma = tma && tma_ok(w[i], ldw[i]);
  if (!tma || count == 1) {  // one launch per GEMM (each picks its own path)
    for (int i = 0; i < count; ++i)
      if (int s = bw_w8a16_gemm(x, x_dtype, ldx, w[i], ldw[i], scale[i], scale_dtype, y[i], ldy[i], m, n[i], k,
                                workspace, workspace_bytes, stream))
        return s;
    return BW_OK;
  }
  GroupArgs ga = {};
  ga.count = count;
  GatherArgs g = {};
  g.vec = 1;
  int t0 = 0;
  for (int i = 0; i < count; ++i) {
    if (int s = make_tmap_2d(&ga.w[i], w[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, n[i], k, ldw[i], 128, 128,
                             CU_TENSOR_MAP_SWIZZLE_128B))
      return s;
    ga.scale[i] = reinterpret_cast<unsigned long long>(scale[i]);
    ga.y[i] = reinterpret_cast<unsigned long long>(y[i]);
    ga.ldy[i] = ldy[i];
    ga.n[i] = static_cast<int>(n[i]);
    ga.tile0[i] = t0;
    t0 += static_cast<int>((n[i] + 127) / 128);
    g.vec &= reinterpret_cast<uintptr_t>(y[i]) % 16 == 0 && ldy[i] % 8 == 0;
  }
  ga.tile0[count] = t0;
  return gemm_impl(x, x_dtype, ldx, w[0], ldw[0], scale[0], scale_dtype, y[0], ldy[0], m, 128 * tiles, k, workspace,
                   workspace_bytes, g, stream, nullptr, nullptr, &ga);
}

extern "C" size_t bw_w8a16_gemm_swiglu_workspace_size(int64_t m, int64_t n, int64_t k) {
  if (m <= 0 || n <= 0 || k <= 0) return 0;
  const bw::GemmPlan p = bw::plan_gemm(m, n, k, true);
  return p.counter_bytes + p.partial_bytes;
}

// Fused gate/up W8A16 GEMM with the SwiGLU epilogue:
// y = dt(silu(dt(x @ (w_gate * s_gate)^T)) * dt(x @ (w_up * s_up)^T)).
extern "C" int bw_w8a16_gemm_swiglu(const void* x, int x_dtype, int64_t ldx, const int8_t* w_gate,
                                    const int8_t* w_up, int64_t ldw, const void* scale_gate, const void* scale_up,
                                    int scale_dtype, void* y, int64_t ldy, int64_t m, int64_t n, int64_t k,
                                    void* workspace, size_t workspace_bytes, void* stream) {
  bw::GatherArgs g = {};
  if (!w_up) return bw::fail(BW_ERR_INVALID_ARGUMENT, "int8_gemm_swiglu: null pointer");
  return bw::gemm_impl(x, x_dtype, ldx, w_gate, ldw, scale_gate, scale_dtype, y, ldy, m, n, k, workspace,
                       workspace_bytes, g, stream, w_up, scale_up);
}

// Column-parallel N-split GEMM with the all-gather in the epilogue: this rank's output columns
// [col0, col0 + n) of y are computed here and sent to every peer's signal-pad mailbox; the peers'
// columns (rank p: [col0 + (p - rank) n, ... + n)) arrive in this rank's mailbox and are copied
// into y before the kernel ends.  Waits are bounded; a timeout shows in bw_device_status.
extern "C" size_t bw_w8a16_gemm_allgather_signal_bytes(int64_t m, int64_t n, int world) {
  if (m <= 0 || n <= 0 || world < 1 || world > 8) return 0;
  return bw::gather_pad_bytes(m, n, world);
}

extern "C" int bw_w8a16_gemm_allgather(const void* x, int x_dtype, int64_t ldx, const int8_t* w, int64_t ldw,
                                       const void* scale, int scale_dtype, void* y, int64_t ldy, int64_t col0,
                                       int64_t m, int64_t n, int64_t k, void* const* signal_ranks,
                                       size_t signal_bytes, int world, int rank, void* workspace,
                                       size_t workspace_bytes, void* stream) {
  using namespace bw;
  if (world < 1 || world > 8 || rank < 0 || rank >= world)
    return fail(BW_ERR_INVALID_ARGUMENT, "int8_gemm (all-gather): need 1 <= world <= 8 and 0 <= rank < world");
  if (!y || !signal_ranks) return fail(BW_ERR_INVALID_ARGUMENT, "int8_gemm (all-gather): null pointer");
  if (m < 0 || n < 0 || m > kGatherMaxM)
    return fail(BW_ERR_UNSUPPORTED, "int8_gemm (all-gather): m = %lld outside [0, %d]", (long long)m, kGatherMaxM);
  if (n > (1LL << 30) || col0 < rank * n || col0 + (world - rank) * n > ldy)
    return fail(BW_ERR_INVALID_ARGUMENT,
                "int8_gemm (all-gather): the %d ranks' columns around [%lld, %lld) do not fit the row stride %lld",
                world, (long long)col0, (long long)(col0 + n), (long long)ldy);
  if (m == 0 || n == 0) return BW_OK;
  if (signal_bytes < gather_pad_bytes(m, n, world))
    return fail(BW_ERR_WORKSPACE, "int8_gemm (all-gather): signal pads of %zu bytes required, %zu given",
                gather_pad_bytes(m, n, world), signal_bytes);
  GatherArgs g = {};
  for (int r = 0; r < world; ++r) {
    if (!signal_ranks[r]) return fail(BW_ERR_INVALID_ARGUMENT, "int8_gemm (all-gather): null signal pad for rank %d", r);
    if (reinterpret_cast<uintptr_t>(signal_ranks[r]) % 16 != 0)
      return fail(BW_ERR_INVALID_ARGUMENT, "int8_gemm (all-gather): signal pad of rank %d is not 16-byte aligned", r);
    g.pad[r] = reinterpret_cast<unsigned long long>(signal_ranks[r]);
  }
  uint16_t* yl = static_cast<uint16_t*>(y) + col0;
  g.ybase = reinterpret_cast<unsigned long long>(yl - rank * n);
  g.n = static_cast<int>(n);
  g.rowwords = static_cast<int>((n + 127) / 128 * 64);
  g.world = world;
  g.rank = rank;
  g.vec = reinterpret_cast<uintptr_t>(yl) % 16 == 0 && ldy % 8 == 0;
  g.vec4 = g.ybase % 8 == 0 && ldy % 4 == 0 && n % 4 == 0;
  return gemm_impl(x, x_dtype, ldx, w, ldw, scale, scale_dtype, yl, ldy, m, n, k, workspace, workspace_bytes, g,
                   stream);
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

// ---------------------------------------------------------------------------
// Stream-K schedule introspection (host only, for tests): the same sk_start / sk_owner / SegWalk /
// sk_pieces code the kernel runs, on a plan of `tiles` tiles of `kblocks` k-blocks over `grid` CTAs.
// ---------------------------------------------------------------------------
static bool streamk_plan(int64_t kblocks, int64_t tiles, int grid, bw::Sched* s) {
  if (kblocks < 1 || tiles < 1 || grid < 1 || kblocks * tiles < grid || kblocks * tiles * grid >= (1LL << 31))
    return false;
  *s = bw::Sched{};
  s->mode = 1;
  s->n_tiles = static_cast<int>(tiles);
  s->m_tiles = 1;
  s->kblocks = static_cast<int>(kblocks);
  s->work = kblocks * tiles;
  return true;
}

extern "C" int bw_debug_streamk_walk(int64_t kblocks, int64_t tiles, int grid, int cta, int32_t* segs,
                                     int max_segs) {
  bw::Sched s;
  if (!streamk_plan(kblocks, tiles, grid, &s) || cta < 0 || cta >= grid || !segs) return -1;
  bw::SegWalk wk(s, cta, grid);
  bw::Seg sg;
  int n = 0;
  while (wk.next(s, sg)) {
    if (n >= max_segs) return -1;
    segs[4 * n] = sg.t;
    segs[4 * n + 1] = sg.k0;
    segs[4 * n + 2] = sg.nkb;
    segs[4 * n + 3] = sg.split;
    ++n;
  }
  return n;
}

extern "C" int64_t bw_debug_streamk_start(int64_t kblocks, int64_t tiles, int grid, int cta) {
  bw::Sched s;
  if (!streamk_plan(kblocks, tiles, grid, &s) || cta < 0 || cta > grid) return -1;
  return bw::sk_start(cta, s, grid);
}

extern "C" int bw_debug_streamk_owner(int64_t kblocks, int64_t tiles, int grid, int64_t x) {
  bw::Sched s;
  if (!streamk_plan(kblocks, tiles, grid, &s) || x < 0 || x >= s.work) return -1;
  return bw::sk_owner(x, s, grid);
}

extern "C" int bw_debug_streamk_pieces(int64_t kblocks, int64_t tiles, int grid, int tile, int32_t* loc) {
  bw::Sched s;
  if (!streamk_plan(kblocks, tiles, grid, &s) || tile < 0 || tile >= tiles || !loc) return -1;
  const bw::PieceLoc p = bw::sk_pieces(s, tile, grid);
  loc[0] = p.c_first;
  loc[1] = p.n_parts;
  loc[2] = p.slot0;
  return 0;
}
