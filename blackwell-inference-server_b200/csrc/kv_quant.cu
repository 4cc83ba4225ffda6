// Per-channel int8 quantisation for KV caches (the shared quantiser family's
// second member), sm_100a.  Replaces the reference's
//   quantize_per_channel_kernel    src/blackwell_ops/cuda/kv_quant.cu:17-42
//   dequantize_per_channel_kernel  src/blackwell_ops/cuda/kv_quant.cu:47-58
// whose semantics differ from the weight quantiser's (quantize_weight_int8):
//   amax  = max over the channel of |x| in fp32, NaN elements ignored (fmaxf), 0 for an empty max
//   scale = amax / 127 in fp32 (no clamp, stored as fp32)
//   q     = clamp(lrint(x / scale), -127, 127)       (fp32 quotient, round half to even, NaN -> 0)
//   x'    = fp16(fp32(q) * scale)                    (dequantise)
// Divisions are IEEE (__fdiv_rn, or the reciprocal fast path of quant_math.cuh
// that falls back to it near a rounding boundary), so a CPU restatement in
// float32 reproduces every bit.
//
// Quantise: a channel is split over a thread-block cluster of CL CTAs (CL <= 8),
// each holding its part of the row in registers (16-byte loads, read from HBM
// once); the CTAs exchange their partial maxima through distributed shared
// memory and quantise from registers.  Channels of more than 8 x 8192 elements,
// or layouts without 16-byte alignment, use a two-pass kernel that re-reads
// the row.
#include <stdio.h>

#include <mutex>

#include "quant_math.cuh"

namespace bw {

constexpr int kKvThreads = 256;
constexpr int kKvMaxCluster = 8;
constexpr int kKvMaxVpt = 4;  // 16-byte chunks per thread

// |x| maximum of 8 halves, NaN ignored (fmaxf returns the other operand)
__device__ __forceinline__ float kv_absmax8(const uint4& v, float m) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
    m = fmaxf(m, fmaxf(fabsf(f.x), fabsf(f.y)));
  }
  return m;
}

// 8 codes of 8 halves, packed in a uint2
__device__ __forceinline__ uint2 kv_quant8(const uint4& v, float s, float rcp) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t out[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint32_t packed = 0;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[2 * h + i]));
      const uint32_t c0 = static_cast<uint8_t>(quant_fast<BW_DTYPE_F32>(f.x, s, rcp));
      const uint32_t c1 = static_cast<uint8_t>(quant_fast<BW_DTYPE_F32>(f.y, s, rcp));
      packed |= (c0 | (c1 << 8)) << (16 * i);
    }
    out[h] = packed;
  }
  return make_uint2(out[0], out[1]);
}

template <int VPT>
__global__ void __launch_bounds__(kKvThreads) kv_quant_cluster_kernel(const __half* __restrict__ x, int64_t ldx,
                                                                      int64_t n, int8_t* __restrict__ q, int64_t ldq,
                                                                      float* __restrict__ scale, int seg) {
  __shared__ float red[kKvThreads / 32];
  __shared__ float part[kKvMaxCluster];  // partial maxima of the cluster's CTAs
  const int cl = static_cast<int>(cluster_ctarank());
  int nclus;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(nclus));
  const int64_t c = blockIdx.x / nclus;  // channel
  const int64_t e0 = static_cast<int64_t>(cl) * seg;
  const int64_t e1 = e0 + seg < n ? e0 + seg : n;
  const __half* xr = x + c * ldx;
  uint4 v[VPT];
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t e = e0 + (static_cast<int64_t>(i) * kKvThreads + threadIdx.x) * 8;
    v[i] = make_uint4(0u, 0u, 0u, 0u);
    if (e < e1) v[i] = __ldcs(reinterpret_cast<const uint4*>(xr + e));
    m = kv_absmax8(v[i], m);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float mm = 0.f;
    for (int w = 0; w < kKvThreads / 32; ++w) mm = fmaxf(mm, red[w]);
    // this CTA's maximum into slot `cl` of every CTA of the cluster
    for (int r = 0; r < nclus; ++r) st_shared_cluster_f32(mapa_shared(smem_u32(&part[cl]), r), mm);
  }
  cluster_sync_all();  // every partial maximum is in every CTA's shared memory
  float amax = 0.f;
  for (int r = 0; r < nclus; ++r) amax = fmaxf(amax, part[r]);
  const float s = __fdiv_rn(amax, 127.0f);
  const float rcp = __frcp_rn(s);
  if (cl == 0 && threadIdx.x == 0) scale[c] = s;
  int8_t* qr = q + c * ldq;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t e = e0 + (static_cast<int64_t>(i) * kKvThreads + threadIdx.x) * 8;
    if (e < e1) *reinterpret_cast<uint2*>(qr + e) = kv_quant8(v[i], s, rcp);
  }
  cluster_sync_all();  // no CTA exits while a peer may still write its shared memory
}

// Any layout: one CTA per channel, two passes over the row.
__global__ void __launch_bounds__(kKvThreads) kv_quant_rows_kernel(const __half* __restrict__ x, int64_t ldx,
                                                                   int64_t n, int8_t* __restrict__ q, int64_t ldq,
                                                                   float* __restrict__ scale) {
  __shared__ float red[kKvThreads / 32];
  const int64_t c = blockIdx.x;
  const __half* xr = x + c * ldx;
  float m = 0.f;
  for (int64_t e = threadIdx.x; e < n; e += kKvThreads) m = fmaxf(m, fabsf(__half2float(xr[e])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  float amax = 0.f;
  for (int w = 0; w < kKvThreads / 32; ++w) amax = fmaxf(amax, red[w]);
  const float s = __fdiv_rn(amax, 127.0f);
  const float rcp = __frcp_rn(s);
  if (threadIdx.x == 0) scale[c] = s;
  int8_t* qr = q + c * ldq;
  for (int64_t e = threadIdx.x; e < n; e += kKvThreads) qr[e] = quant_fast<BW_DTYPE_F32>(__half2float(xr[e]), s, rcp);
}

// x'[c, e] = fp16(fp32(q[c, e]) * scale[c]); 8 elements per thread when aligned.
__global__ void __launch_bounds__(256) kv_dequant_kernel(const int8_t* __restrict__ q, int64_t ldq,
                                                         const float* __restrict__ scale, int64_t c_rows, int64_t n,
                                                         __half* __restrict__ x, int64_t ldx, int vec) {
  const int64_t per_row = vec ? n / 8 : n;
  const int64_t total = c_rows * per_row;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t c = i / per_row, j = i - c * per_row;
    const float s = scale[c];
    if (vec) {
      const uint2 codes = *reinterpret_cast<const uint2*>(q + c * ldq + j * 8);
      const uint32_t w[2] = {codes.x, codes.y};
      uint32_t o[4];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const uint32_t word = w[h >> 1] >> (16 * (h & 1));
        const float a = static_cast<float>(static_cast<int8_t>(word & 0xFF)) * s;
        const float b = static_cast<float>(static_cast<int8_t>((word >> 8) & 0xFF)) * s;
        const __half2 hv = __halves2half2(__float2half_rn(a), __float2half_rn(b));
        o[h] = *reinterpret_cast<const uint32_t*>(&hv);
      }
      *reinterpret_cast<uint4*>(x + c * ldx + j * 8) = make_uint4(o[0], o[1], o[2], o[3]);
    } else {
      x[c * ldx + j] = __float2half_rn(static_cast<float>(q[c * ldq + j]) * s);
    }
  }
}

template <int VPT>
static int launch_kv_cluster(const __half* x, int64_t ldx, int64_t c, int64_t n, int8_t* q, int64_t ldq, float* scale,
                             int cl, int seg, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(c * cl));
  cfg.blockDim = dim3(kKvThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cl;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return check_cuda(cudaLaunchKernelEx(&cfg, kv_quant_cluster_kernel<VPT>, x, ldx, n, q, ldq, scale, seg),
                    "cudaLaunchKernelEx(kv_quant_cluster_kernel)");
}

}  // namespace bw

extern "C" int bw_quantize_kv_int8(const void* x, int64_t c, int64_t n, int64_t ldx, int8_t* q, int64_t ldq,
                                   float* scale, void* stream) {
  using namespace bw;
  if (c < 0 || n < 0) return fail(BW_ERR_INVALID_ARGUMENT, "quantize_kv_int8: need c, n >= 0");
  if (c == 0) return BW_OK;
  if (!x || !q || !scale) return fail(BW_ERR_INVALID_ARGUMENT, "quantize_kv_int8: null pointer");
  if (ldx < n || ldq < n) return fail(BW_ERR_INVALID_ARGUMENT, "quantize_kv_int8: row stride too small");
  if (c > INT32_MAX / kKvMaxCluster) return fail(BW_ERR_INVALID_ARGUMENT, "quantize_kv_int8: too many channels");
  if (int s = require_sm100()) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const __half* xh = static_cast<const __half*>(x);
  const bool vec = n > 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0 && ldx % 8 == 0 && n % 8 == 0 &&
                   reinterpret_cast<uintptr_t>(q) % 8 == 0 && ldq % 8 == 0;
  const int64_t per_cta = static_cast<int64_t>(kKvThreads) * 8;  // elements one chunk per thread covers
  if (vec && n <= static_cast<int64_t>(kKvMaxCluster) * kKvMaxVpt * per_cta) {
    // at least one chunk per thread, at most kKvMaxVpt; spread a channel over up to 8 CTAs
    int cl = static_cast<int>((n + per_cta - 1) / per_cta);
    cl = cl < 1 ? 1 : (cl > kKvMaxCluster ? kKvMaxCluster : cl);
    int64_t seg = (n + cl - 1) / cl;
    seg = (seg + 7) / 8 * 8;
    const int vpt = static_cast<int>((seg + per_cta - 1) / per_cta);
    switch (vpt) {
      case 1: return launch_kv_cluster<1>(xh, ldx, c, n, q, ldq, scale, cl, static_cast<int>(seg), st);
      case 2: return launch_kv_cluster<2>(xh, ldx, c, n, q, ldq, scale, cl, static_cast<int>(seg), st);
      default: return launch_kv_cluster<4>(xh, ldx, c, n, q, ldq, scale, cl, static_cast<int>(seg), st);
    }
  }
  kv_quant_rows_kernel<<<static_cast<unsigned>(c), kKvThreads, 0, st>>>(xh, ldx, n, q, ldq, scale);
  return check_launch("kv_quant_rows_kernel");
}

extern "C" int bw_dequantize_kv_int8(const int8_t* q, int64_t ldq, const float* scale, int64_t c, int64_t n, void* x,
                                     int64_t ldx, void* stream) {
  using namespace bw;
  if (c < 0 || n < 0) return fail(BW_ERR_INVALID_ARGUMENT, "dequantize_kv_int8: need c, n >= 0");
  if (c == 0 || n == 0) return BW_OK;
  if (!x || !q || !scale) return fail(BW_ERR_INVALID_ARGUMENT, "dequantize_kv_int8: null pointer");
  if (ldx < n || ldq < n) return fail(BW_ERR_INVALID_ARGUMENT, "dequantize_kv_int8: row stride too small");
  if (int s = require_sm100()) return s;
  const int vec = reinterpret_cast<uintptr_t>(x) % 16 == 0 && ldx % 8 == 0 && n % 8 == 0 &&
                  reinterpret_cast<uintptr_t>(q) % 8 == 0 && ldq % 8 == 0;
  const int64_t total = c * (vec ? n / 8 : n);
  const int64_t blocks = (total + 255) / 256;
  const int grid = static_cast<int>(blocks < 4L * num_sms() ? blocks : 4L * num_sms());
  kv_dequant_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(q, ldq, scale, c, n,
                                                                         static_cast<__half*>(x), ldx, vec);
  return check_launch("kv_dequant_kernel");
}
