// Residual + RMSNorm, alone and as the prologue of the W8A16 GEMM, sm_100a.
//
// Replaces the reference's
//   rmsnorm_kernel                 src/blackwell_ops/cuda/basic_ops.cu:16-46
//   fused_residual_rmsnorm_kernel  src/blackwell_ops/cuda/basic_ops.cu:49-78
// and feeds the normalised rows straight into the W8A16 GEMM (bw_w8a16_gemm_rmsnorm):
//   v[k]  = fp32(x[m,k]) (+ fp32(residual[m,k]))                          (:56, :73)
//   ss    = sum_k v[k]^2, summed as the reference's 256-thread block does: thread t adds
//           k = t, t+256, ... in order, then the tree smem[t] += smem[t+s], s = 128 .. 1 (:57-67)
//   rstd  = 1 / sqrt(ss / K + eps)                                         (:68)
//   out   = T(v[k] * rstd * fp32(w[k]))                                     (:71-74)
// Every operation is IEEE fp32 (no contraction: products and sums rounded separately), so a
// float32 CPU restatement reproduces every bit.  The prologue writes the normalised rows into
// the caller's workspace and the GEMM follows with programmatic dependent launch: the GEMM's
// weight stream starts while the rows are normalised (they are M x K, tiny next to the weights).
#include <stdio.h>

#include <type_traits>

#include "common.cuh"

namespace bw {

constexpr int kNormThreads = 256;

template <typename T>
__device__ __forceinline__ float norm_ld(const void* p, int64_t i) {
  if constexpr (std::is_same<T, __half>::value) return __half2float(static_cast<const __half*>(p)[i]);
  else return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}
template <typename T>
__device__ __forceinline__ void norm_st(void* p, int64_t i, float v) {
  if constexpr (std::is_same<T, __half>::value) static_cast<__half*>(p)[i] = __float2half_rn(v);
  else static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
}

// One CTA per row.  residual may be null (plain RMSNorm).
template <typename T>
__global__ void __launch_bounds__(kNormThreads) residual_rmsnorm_kernel(const void* __restrict__ x,
                                                                        const void* __restrict__ res, int64_t ldx,
                                                                        const void* __restrict__ w, float eps,
                                                                        void* __restrict__ out, int64_t ldo, int K) {
  __shared__ float red[kNormThreads];
  pdl_launch_dependents();
  pdl_wait();  // x / residual may come from the preceding kernel
  const int64_t row = blockIdx.x;
  const int t = threadIdx.x;
  float local = 0.f;
  for (int k = t; k < K; k += kNormThreads) {
    float v = norm_ld<T>(x, row * ldx + k);
    if (res != nullptr) v = __fadd_rn(v, norm_ld<T>(res, row * ldx + k));
    local = __fadd_rn(local, __fmul_rn(v, v));
  }
  red[t] = local;
  __syncthreads();
  for (int s = kNormThreads / 2; s > 0; s >>= 1) {
    if (t < s) red[t] = __fadd_rn(red[t], red[t + s]);
    __syncthreads();
  }
  const float rstd = __frcp_rn(__fsqrt_rn(__fadd_rn(__fdiv_rn(red[0], static_cast<float>(K)), eps)));
  for (int k = t; k < K; k += kNormThreads) {
    float v = norm_ld<T>(x, row * ldx + k);
    if (res != nullptr) v = __fadd_rn(v, norm_ld<T>(res, row * ldx + k));
    norm_st<T>(out, row * ldo + k, __fmul_rn(__fmul_rn(v, rstd), norm_ld<T>(w, k)));
  }
}

static int launch_norm(const void* x, const void* res, int dtype, int64_t ldx, const void* w, float eps, void* out,
                       int64_t ldo, int64_t m, int64_t k, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(m));
  cfg.blockDim = dim3(kNormThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int kk = static_cast<int>(k);
  if (dtype == BW_DTYPE_BF16)
    return check_cuda(cudaLaunchKernelEx(&cfg, residual_rmsnorm_kernel<__nv_bfloat16>, x, res, ldx, w, eps, out, ldo, kk),
                      "cudaLaunchKernelEx(residual_rmsnorm_kernel)");
  return check_cuda(cudaLaunchKernelEx(&cfg, residual_rmsnorm_kernel<__half>, x, res, ldx, w, eps, out, ldo, kk),
                    "cudaLaunchKernelEx(residual_rmsnorm_kernel)");
}

static int check_norm_args(const void* x, int dtype, int64_t ldx, const void* w, const void* out, int64_t ldo,
                           int64_t m, int64_t k, const char* op) {
  if (m < 0 || k < 1) return fail(BW_ERR_INVALID_ARGUMENT, "%s: need m >= 0 and k >= 1", op);
  if (dtype != BW_DTYPE_F16 && dtype != BW_DTYPE_BF16)
    return fail(BW_ERR_INVALID_ARGUMENT, "%s: x must be fp16 or bf16 (dtype %d)", op, dtype);
  if (m > 0 && (!x || !w || !out)) return fail(BW_ERR_INVALID_ARGUMENT, "%s: null pointer", op);
  if (ldx < k || ldo < k) return fail(BW_ERR_INVALID_ARGUMENT, "%s: row stride too small", op);
  if (m > INT32_MAX || k > INT32_MAX) return fail(BW_ERR_INVALID_ARGUMENT, "%s: dimension too large", op);
  return BW_OK;
}

// Normalised rows go to the workspace after the GEMM's own scratch, 256-byte aligned, and never
// into the GEMM counter region: a plan without split tiles needs no scratch, but a workspace is
// shared with other calls, whose tile counters at its start must stay zero.
static size_t norm_offset(int64_t m, int64_t n, int64_t k) {
  const size_t g = bw_w8a16_gemm_workspace_size(m, n, k);
  return ((g > kGemmCounterBytes ? g : kGemmCounterBytes) + 255) / 256 * 256;
}

}  // namespace bw

extern "C" int bw_residual_rmsnorm(const void* x, const void* residual, int dtype, int64_t ldx, const void* w,
                                   float eps, void* out, int64_t ldo, int64_t m, int64_t k, void* stream) {
  using namespace bw;
  if (int s = check_norm_args(x, dtype, ldx, w, out, ldo, m, k, "fused_residual_rmsnorm")) return s;
  if (m == 0) return BW_OK;
  if (int s = require_sm100()) return s;
  return launch_norm(x, residual, dtype, ldx, w, eps, out, ldo, m, k, static_cast<cudaStream_t>(stream));
}

extern "C" size_t bw_w8a16_gemm_rmsnorm_workspace_size(int64_t m, int64_t n, int64_t k) {
  if (m <= 0 || n <= 0 || k <= 0) return 0;
  return bw::norm_offset(m, n, k) + static_cast<size_t>(m) * static_cast<size_t>(k) * 2;
}

extern "C" int bw_w8a16_gemm_rmsnorm(const void* x, const void* residual, int x_dtype, int64_t ldx,
                                     const void* norm_w, float eps, const int8_t* w, int64_t ldw, const void* scale,
                                     int scale_dtype, void* y, int64_t ldy, int64_t m, int64_t n, int64_t k,
                                     void* workspace, size_t workspace_bytes, void* stream) {
  using namespace bw;
  if (int s = check_norm_args(x, x_dtype, ldx, norm_w, y, k, m, k, "int8_gemm_rmsnorm")) return s;
  if (m == 0 || n == 0) return BW_OK;
  const size_t need = bw_w8a16_gemm_rmsnorm_workspace_size(m, n, k);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(BW_ERR_WORKSPACE, "int8_gemm_rmsnorm: workspace of %zu bytes required, %zu given", need,
                workspace_bytes);
  if (reinterpret_cast<uintptr_t>(workspace) % 256 != 0)
    return fail(BW_ERR_WORKSPACE, "int8_gemm_rmsnorm: workspace must be 256-byte aligned");
  if (int s = require_sm100()) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  void* xn = static_cast<uint8_t*>(workspace) + norm_offset(m, n, k);
  if (int s = launch_norm(x, residual, x_dtype, ldx, norm_w, eps, xn, k, m, k, st)) return s;
  return bw_w8a16_gemm(xn, x_dtype, k, w, ldw, scale, scale_dtype, y, ldy, m, n, k, workspace,
                       norm_offset(m, n, k), stream);
}
