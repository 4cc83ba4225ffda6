// Per-output-channel symmetric int8 quantisation, bit-exact with the
// reference quantize_weight_int8 (src/blackwell_ops/kernels/int8_gemm.py:63-68):
//
//   amax  = max_k |w[n,k]|                         (exact in the weight dtype)
//   amaxc = dt(max(fp32(amax), 1e-8f))             (.clamp(min=1e-8), :65)
//   scale = dt(fp32(amaxc) / 127.0f)               (IEEE division, :66)
//   q     = clamp(rint(dt(fp32(w) / fp32(scale))), -127, 127)   (:67)
//           NaN -> 0 (torch's NaN -> int8 cast), +-inf -> +-127
//
// dt() rounds to the weight's dtype (fp16 / bf16 / fp32) with round-to-nearest-
// even.  The division must be IEEE (__fdiv_rn), never an approximate reciprocal.
//
// HBM-bound: each row is read once into registers (16-byte vector loads,
// `VPT` vectors per thread, a power-of-two group of threads per row), reduced,
// quantised from registers and written with 8-byte (4-byte for fp32) stores.
// Rows that do not fit in registers, or unaligned layouts, use a two-pass
// kernel that re-reads the row (from L2) instead.
#include <stdio.h>

#include <algorithm>
#include <type_traits>
#include <mutex>

#include "quant_math.cuh"

namespace bw {

constexpr int kElemBytes[3] = {2, 2, 4};

// Unpack the values of one 16-byte chunk.
template <int DT>
__device__ __forceinline__ void chunk_values(const uint4& v, float* out) {
  if constexpr (DT == BW_DTYPE_F32) {
    out[0] = __uint_as_float(v.x);
    out[1] = __uint_as_float(v.y);
    out[2] = __uint_as_float(v.z);
    out[3] = __uint_as_float(v.w);
  } else {
    const uint32_t words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (DT == BW_DTYPE_F16) {
        const __half2 h = *reinterpret_cast<const __half2*>(&words[i]);
        out[2 * i] = __low2float(h);
        out[2 * i + 1] = __high2float(h);
      } else {
        const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&words[i]);
        out[2 * i] = __low2float(h);
        out[2 * i + 1] = __high2float(h);
      }
    }
  }
}

// Max-reduce (amax, nan) over the `group` threads of a row.  `red` holds
// one float per warp of the block.
__device__ __forceinline__ void group_reduce(float& amax, bool& nan, int group, float* red, int* redn) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    nan = __any_sync(0xffffffffu, nan);
  }
  if (group > 32) {
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    if (lane == 0) {
      red[warp] = amax;
      redn[warp] = nan ? 1 : 0;
    }
    __syncthreads();
    const int wpg = group >> 5;  // warps per group
    const int first = (warp / wpg) * wpg;
    float m = 0.f;
    int nn = 0;
    for (int i = 0; i < wpg; ++i) {
      m = fmaxf(m, red[first + i]);
      nn |= redn[first + i];
    }
    amax = m;
    nan = nn != 0;
  }
}

// Row held in registers: each thread of the row's group holds up to VPT
// 16-byte chunks (chunk index = g + i*group).
template <int DT, int VPT>
__global__ void __launch_bounds__(512) quantize_rows_reg_kernel(const uint8_t* __restrict__ w, int64_t ldw_bytes,
                                                                int64_t n, int64_t k, int8_t* __restrict__ q,
                                                                int64_t ldq, void* __restrict__ scale, int group) {
  constexpr int EB = kElemBytes[DT];
  constexpr int E = 16 / EB;  // elements per chunk
  __shared__ float red[32];
  __shared__ int redn[32];
  const int rows_per_block = blockDim.x / group;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * rows_per_block + threadIdx.x / group;
  const int g = threadIdx.x % group;
  const bool active = row < n;
  const int64_t nchunks = (k + E - 1) / E;
  const uint8_t* wr = w + (active ? row : 0) * ldw_bytes;

  uint4 v[VPT];
  float amax = 0.f;
  bool nan = false;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t c = g + static_cast<int64_t>(i) * group;
    v[i] = make_uint4(0u, 0u, 0u, 0u);
    if (active && c < nchunks) {
      if ((c + 1) * E <= k) {
        v[i] = __ldcs(reinterpret_cast<const uint4*>(wr) + c);
      } else {  // ragged tail chunk: element loads, zero padding (|0| never raises the max)
        uint8_t tmp[16] = {0};
        for (int64_t e = c * E; e < k; ++e)
          for (int b = 0; b < EB; ++b) tmp[(e - c * E) * EB + b] = wr[e * EB + b];
        v[i] = *reinterpret_cast<uint4*>(tmp);
      }
    }
    float f[E];
    chunk_values<DT>(v[i], f);
#pragma unroll
    for (int e = 0; e < E; ++e) {
      nan |= (f[e] != f[e]);
      amax = fmaxf(amax, fabsf(f[e]));
    }
  }
  group_reduce(amax, nan, group, red, redn);
  const float s = scale_from_amax<DT>(amax, nan);
  const float rcp = __frcp_rn(s);
  if (!active) return;
  if (g == 0) store_scale<DT>(scale, row, s);

  int8_t* qr = q + row * ldq;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t c = g + static_cast<int64_t>(i) * group;
    if (c >= nchunks) continue;
    float f[E];
    chunk_values<DT>(v[i], f);
    int8_t out[E];
#pragma unroll
    for (int e = 0; e < E; ++e) out[e] = quant_fast<DT>(f[e], s, rcp);
    if ((c + 1) * E <= k) {
      if constexpr (E == 8) {
        *reinterpret_cast<uint2*>(qr + c * E) = *reinterpret_cast<uint2*>(out);
      } else {
        *reinterpret_cast<uint32_t*>(qr + c * E) = *reinterpret_cast<uint32_t*>(out);
      }
    } else {
      for (int64_t e = c * E; e < k; ++e) qr[e] = out[e - c * E];
    }
  }
}

// Streaming kernel for aligned rows of up to a few tens of KB: one or two CTAs
// per SM walk rows blockIdx.x, + gridDim.x, ...; thread 0 keeps `stages` rows in
// flight with 1-D bulk copies into a shared-memory ring.  Four groups of 64
// threads take rows in turn (a stage count that is a multiple of four keeps each
// stage with one group), so four rows are reduced and quantised at once per CTA:
// a row's two passes and its reduction are a latency chain.  Llama-3-8B MLP bf16
// weights: one row per CTA 2791 GB/s, two groups 3210, four groups 3470 (a ring
// of 16 stages instead of 8 changed nothing).  The arithmetic is the register kernel's (fp16
// rows with a normal scale use the packed quantiser, proved equal to it).
constexpr int kQsThreads = 256;
#ifndef BW_QS_GROUPS
#define BW_QS_GROUPS 4
#endif
#ifndef BW_QS_MAX_STAGES
#define BW_QS_MAX_STAGES 8
#endif
constexpr int kQsGroups = BW_QS_GROUPS;
constexpr int kQsGroupThreads = kQsThreads / kQsGroups;
constexpr int kQsMaxStages = BW_QS_MAX_STAGES;
enum QuantWaitSite : int { kSiteQsFull = 301 };

template <int DT>
__global__ void __launch_bounds__(kQsThreads) quantize_rows_stream_kernel(const uint8_t* __restrict__ w,
                                                                        int64_t ldw_bytes, int64_t n, int64_t k,
                                                                        int8_t* __restrict__ q, int64_t ldq,
                                                                        void* __restrict__ scale, int stage_bytes,
                                                                        int stages) {
  constexpr int EB = kElemBytes[DT];
  constexpr int E = 16 / EB;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + static_cast<size_t>(stages) * stage_bytes);
  __shared__ float red[kQsGroups][kQsGroupThreads / 32];
  __shared__ int redn[kQsGroups][kQsGroupThreads / 32];
  __shared__ int abort_flag_s;
  volatile int* abort_flag = &abort_flag_s;
  const int grp = threadIdx.x / kQsGroupThreads;
  const int tid = threadIdx.x % kQsGroupThreads;  // thread within the row group
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int bar = 1 + grp;                         // the group's named barrier
  const uint32_t row_bytes = static_cast<uint32_t>(k * EB);
  const int nchunks = static_cast<int>(row_bytes / 16);
  const int64_t G = gridDim.x;
  const int64_t mine = n > blockIdx.x ? (n - blockIdx.x + G - 1) / G : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) mbar_init(&full[s], 1);
    abort_flag_s = 0;
    fence_mbar_init();
    const uint64_t once = l2_policy_evict_first();
    for (int64_t i = 0; i < mine && i < stages; ++i) {
      const int64_t row = blockIdx.x + i * G;
      mbar_arrive_expect_tx(&full[i], row_bytes);
      bulk_load_1d(ring + i * stage_bytes, w + row * ldw_bytes, row_bytes, &full[i], once);
    }
  }
  __syncthreads();
  const uint64_t once = l2_policy_evict_first();
  int64_t i = grp;
  for (; i < mine; i += kQsGroups) {
    const int st = static_cast<int>(i % stages);
    const int64_t row = blockIdx.x + i * G;
    const bool ok = mbar_wait(&full[st], static_cast<uint32_t>((i / stages) & 1), abort_flag, kSiteQsFull);
    if (named_bar_any(bar, kQsGroupThreads, !ok)) break;  // one decision for the group
    const uint4* src = reinterpret_cast<const uint4*>(ring + static_cast<size_t>(st) * stage_bytes);
    // pass 1: row maximum of |w| (NaN-propagating flag)
    float amax = 0.f;
    bool nan = false;
    if constexpr (DT == BW_DTYPE_F32) {
      for (int c = tid; c < nchunks; c += kQsGroupThreads) {
        float f[E];
        chunk_values<DT>(src[c], f);
#pragma unroll
        for (int e = 0; e < E; ++e) {
          nan |= (f[e] != f[e]);
          amax = fmaxf(amax, fabsf(f[e]));
        }
      }
    } else {
      // packed |w| maxima in the weight dtype (exact), NaN carried by the _nan max
      using T2 = typename std::conditional<DT == BW_DTYPE_F16, __half2, __nv_bfloat162>::type;
      T2 hm;
      *reinterpret_cast<uint32_t*>(&hm) = 0u;  // +0, +0
      for (int c = tid; c < nchunks; c += kQsGroupThreads) {
        const uint4 v = src[c];
        const T2* h = reinterpret_cast<const T2*>(&v);
#pragma unroll
        for (int e = 0; e < 4; ++e) hm = __hmax2_nan(hm, __habs2(h[e]));
      }
      const float l = __low2float(hm), hh = __high2float(hm);
      nan = (l != l) || (hh != hh);
      amax = nan ? 0.f : fmaxf(l, hh);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    nan = __any_sync(0xffffffffu, nan);
    if (lane == 0) {
      red[grp][warp] = amax;
      redn[grp][warp] = nan ? 1 : 0;
    }
    named_bar_sync(bar, kQsGroupThreads);
    amax = 0.f;
    nan = false;
#pragma unroll
    for (int j = 0; j < kQsGroupThreads / 32; ++j) {
      amax = fmaxf(amax, red[grp][j]);
      nan |= redn[grp][j] != 0;
    }
    const float s = scale_from_amax<DT>(amax, nan);
    const float rcp = __frcp_rn(s);
    if (tid == 0) store_scale<DT>(scale, row, s);
    // pass 2: codes
    int8_t* qr = q + row * ldq;
    if constexpr (DT == BW_DTYPE_F16) {
      if (s >= 6.103515625e-05f && s < __int_as_float(0x7f800000)) {  // normal scale: packed, clamp-free
        for (int c = tid; c < nchunks; c += kQsGroupThreads) {
          const uint4 v = src[c];
          const __half2* h = reinterpret_cast<const __half2*>(&v);
          uint2 o;
          o.x = quant4_f16<false>(h[0], h[1], s, rcp);
          o.y = quant4_f16<false>(h[2], h[3], s, rcp);
          *reinterpret_cast<uint2*>(qr + c * 8) = o;
        }
      } else {
        for (int c = tid; c < nchunks; c += kQsGroupThreads) {
          float f[E];
          chunk_values<DT>(src[c], f);
          int8_t out[E];
#pragma unroll
          for (int e = 0; e < E; ++e) out[e] = quant_fast<DT>(f[e], s, rcp);
          *reinterpret_cast<uint2*>(qr + c * E) = *reinterpret_cast<uint2*>(out);
        }
      }
    } else if constexpr (DT == BW_DTYPE_BF16) {
      if (s > 0.0f && s < __int_as_float(0x7f800000) && rcp < 1.0e30f) {  // packed quantiser
        for (int c = tid; c < nchunks; c += kQsGroupThreads) {
          const uint4 v = src[c];
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
          uint2 o;
          o.x = quant4_bf16(h[0], h[1], s, rcp);
          o.y = quant4_bf16(h[2], h[3], s, rcp);
          *reinterpret_cast<uint2*>(qr + c * 8) = o;
        }
      } else {
        for (int c = tid; c < nchunks; c += kQsGroupThreads) {
          float f[E];
          chunk_values<DT>(src[c], f);
          int8_t out[E];
#pragma unroll
          for (int e = 0; e < E; ++e) out[e] = quant_fast<DT>(f[e], s, rcp);
          *reinterpret_cast<uint2*>(qr + c * E) = *reinterpret_cast<uint2*>(out);
        }
      }
    } else {
      for (int c = tid; c < nchunks; c += kQsGroupThreads) {
        float f[E];
        chunk_values<DT>(src[c], f);
        int8_t out[E];
#pragma unroll
        for (int e = 0; e < E; ++e) out[e] = quant_fast<DT>(f[e], s, rcp);
        *reinterpret_cast<uint32_t*>(qr + c * E) = *reinterpret_cast<uint32_t*>(out);
      }
    }
    named_bar_sync(bar, kQsGroupThreads);  // the group is done with this stage and with red[grp]
    if (tid == 0 && i + stages < mine) {  // stages is even: row i + stages belongs to this group too
      const int64_t nrow = blockIdx.x + (i + stages) * G;
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(&full[st], row_bytes);
      bulk_load_1d(ring + static_cast<size_t>(st) * stage_bytes, w + nrow * ldw_bytes, row_bytes, &full[st], once);
    }
  }
  if (i < mine && tid == 0) {
    // a wait gave up: let this group's copies still in flight land before the CTA's shared memory
    // is released (rows i, i + 2, ... below i + stages were issued for it)
    const int64_t issued = mine < i + stages ? mine : i + stages;
    for (int64_t j = i; j < issued; j += kQsGroups)
      mbar_wait(&full[j % stages], static_cast<uint32_t>((j / stages) & 1), nullptr, kSiteQsFull);
  }
}

// Any layout, any length: one block of 256 threads per row, two passes.
template <int DT>
__global__ void __launch_bounds__(256) quantize_rows_generic_kernel(const uint8_t* __restrict__ w, int64_t ldw_bytes,
                                                                    int64_t n, int64_t k, int8_t* __restrict__ q,
                                                                    int64_t ldq, void* __restrict__ scale) {
  __shared__ float red[32];
  __shared__ int redn[32];
  const int64_t row = blockIdx.x;
  if (row >= n) return;
  const uint8_t* wr = w + row * ldw_bytes;
  float amax = 0.f;
  bool nan = false;
  for (int64_t i = threadIdx.x; i < k; i += blockDim.x) {
    const float f = elem_at<DT>(wr, i);
    nan |= (f != f);
    amax = fmaxf(amax, fabsf(f));
  }
  group_reduce(amax, nan, blockDim.x, red, redn);
  const float s = scale_from_amax<DT>(amax, nan);
  if (threadIdx.x == 0) store_scale<DT>(scale, row, s);
  const float rcp = __frcp_rn(s);
  int8_t* qr = q + row * ldq;
  for (int64_t i = threadIdx.x; i < k; i += blockDim.x) qr[i] = quant_fast<DT>(elem_at<DT>(wr, i), s, rcp);
}

template <int DT, int VPT>
static void launch_reg(const void* w, int64_t ldw_bytes, int64_t n, int64_t k, int8_t* q, int64_t ldq,
                       void* scale, int group, cudaStream_t st) {
  const int block = group > 256 ? group : 256;
  const int rows_per_block = block / group;
  const int64_t grid = (n + rows_per_block - 1) / rows_per_block;
  // groups wider than 256 threads run one row per block with the group's width
  quantize_rows_reg_kernel<DT, VPT><<<static_cast<unsigned>(grid), block, 0, st>>>(
      static_cast<const uint8_t*>(w), ldw_bytes, n, k, q, ldq, scale, group);
}

// Streaming plan: stage size and count, CTAs per SM; false if the rows do not suit it.
struct QsPlan {
  int stage_bytes = 0, stages = 0, per_sm = 0, smem = 0;
};
static bool qs_plan(int64_t row_bytes, QsPlan& p) {
  if (row_bytes % 16 != 0 || row_bytes > 96 * 1024) return false;
  p.stage_bytes = static_cast<int>((row_bytes + 127) / 128 * 128);
  for (int cps = 2; cps >= 1; --cps) {
    const int budget = (cps == 2 ? 112 : 224) * 1024;
    // an even stage count keeps every stage with one row group
    const int s = std::min(kQsMaxStages, (budget - 256) / p.stage_bytes) / kQsGroups * kQsGroups;
    if (s >= 2 * kQsGroups || (cps == 1 && s >= kQsGroups)) {
      p.stages = s;
      p.per_sm = cps;
      p.smem = s * p.stage_bytes + s * 8 + 128;
      return true;
    }
  }
  return false;
}

template <int DT>
static int launch_stream(const void* w, int64_t ldw_bytes, int64_t n, int64_t k, int8_t* q, int64_t ldq, void* scale,
                         const QsPlan& p, cudaStream_t st) {
  static std::once_flag once[64];
  static cudaError_t err[64];
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 63], [&] {
    // the kernel's static shared memory (reduction scratch) comes out of the same 227 KB
    err[dev & 63] = cudaFuncSetAttribute(quantize_rows_stream_kernel<DT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         226 * 1024);
  });
  if (int s = check_cuda(err[dev & 63], "cudaFuncSetAttribute(quantize_rows_stream_kernel)")) return s;
  const int64_t grid = std::min<int64_t>(n, static_cast<int64_t>(p.per_sm) * num_sms());
  quantize_rows_stream_kernel<DT><<<static_cast<unsigned>(grid), kQsThreads, p.smem, st>>>(
      static_cast<const uint8_t*>(w), ldw_bytes, n, k, q, ldq, scale, p.stage_bytes, p.stages);
  return check_launch("quantize_rows_stream_kernel");
}

template <int DT>
static int quantize_dispatch(const void* w, int64_t n, int64_t k, int64_t ldw, int8_t* q, int64_t ldq,
                             void* scale, cudaStream_t st) {
  constexpr int EB = kElemBytes[DT];
  constexpr int E = 16 / EB;
  const int64_t ldw_bytes = ldw * EB;
  const bool aligned = (reinterpret_cast<uintptr_t>(w) % 16 == 0) && (ldw_bytes % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(q) % 16 == 0) && (ldq % 16 == 0);
  QsPlan qp;
  if (aligned && n >= 2 * num_sms() && qs_plan(k * EB, qp)) return launch_stream<DT>(w, ldw_bytes, n, k, q, ldq, scale, qp, st);
  const int64_t nchunks = (k + E - 1) / E;
  int group = 32;
  while (group < 512 && (nchunks + group - 1) / group > 8) group <<= 1;
  const int64_t vpt = (nchunks + group - 1) / group;
  if (!aligned || vpt > 8) {
    quantize_rows_generic_kernel<DT><<<static_cast<unsigned>(n), 256, 0, st>>>(
        static_cast<const uint8_t*>(w), ldw_bytes, n, k, q, ldq, scale);
    return check_launch("quantize_rows_generic_kernel");
  }
  if (vpt <= 1) launch_reg<DT, 1>(w, ldw_bytes, n, k, q, ldq, scale, group, st);
  else if (vpt <= 2) launch_reg<DT, 2>(w, ldw_bytes, n, k, q, ldq, scale, group, st);
  else if (vpt <= 4) launch_reg<DT, 4>(w, ldw_bytes, n, k, q, ldq, scale, group, st);
  else launch_reg<DT, 8>(w, ldw_bytes, n, k, q, ldq, scale, group, st);
  return check_launch("quantize_rows_reg_kernel");
}

}  // namespace bw

extern "C" int bw_quantize_rowwise_int8(const void* w, int w_dtype, int64_t n, int64_t k, int64_t ldw, int8_t* q,
                                        int64_t ldq, void* scale, void* stream) {
  using namespace bw;
  if (n < 0 || k < 1) return fail(BW_ERR_INVALID_ARGUMENT, "quantize: need n >= 0 and k >= 1 (got n=%lld k=%lld)",
                                  (long long)n, (long long)k);
  if (n == 0) return BW_OK;
  if (!w || !q || !scale) return fail(BW_ERR_INVALID_ARGUMENT, "quantize: null pointer");
  if (ldw < k || ldq < k) return fail(BW_ERR_INVALID_ARGUMENT, "quantize: row stride smaller than k");
  if (n > 0x7fffffffLL) return fail(BW_ERR_INVALID_ARGUMENT, "quantize: too many rows");
  if (int s = require_sm100()) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (w_dtype) {
    case BW_DTYPE_F16: return quantize_dispatch<BW_DTYPE_F16>(w, n, k, ldw, q, ldq, scale, st);
    case BW_DTYPE_BF16: return quantize_dispatch<BW_DTYPE_BF16>(w, n, k, ldw, q, ldq, scale, st);
    case BW_DTYPE_F32: return quantize_dispatch<BW_DTYPE_F32>(w, n, k, ldw, q, ldq, scale, st);
    default: return fail(BW_ERR_INVALID_ARGUMENT, "quantize: unsupported dtype %d", w_dtype);
  }
}
