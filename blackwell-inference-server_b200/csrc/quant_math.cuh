// Quantiser arithmetic shared by the quantise kernel and the fused LoRA
// merge + requantise kernel, so both produce the reference's bits
// (src/blackwell_ops/kernels/int8_gemm.py:63-68):
//   amaxc = dt(max(fp32(amax), 1e-8f)); scale = dt(fp32(amaxc) / 127.0f)
//   q     = clamp(rint(dt(fp32(w) / fp32(scale))), -127, 127); NaN -> 0
// dt() rounds to the weight dtype (RNE); divisions are IEEE (__fdiv_rn).
#pragma once

#include "common.cuh"

namespace bw {

template <int DT>
__device__ __forceinline__ float round_dt(float x) {
  if constexpr (DT == BW_DTYPE_F16) return __half2float(__float2half_rn(x));
  else if constexpr (DT == BW_DTYPE_BF16) return __bfloat162float(__float2bfloat16_rn(x));
  else return x;
}

template <int DT>
__device__ __forceinline__ float elem_at(const uint8_t* row, int64_t i) {
  if constexpr (DT == BW_DTYPE_F16) return __half2float(reinterpret_cast<const __half*>(row)[i]);
  else if constexpr (DT == BW_DTYPE_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(row)[i]);
  else return reinterpret_cast<const float*>(row)[i];
}

// A NaN scale is stored as the positive quiet NaN that torch produces on the
// CPU (fp16 0x7E00, bf16 0x7FC0, fp32 0x7FC00000); CUDA's conversions would
// give 0x7FFF.
__device__ __forceinline__ __half scale_to_f16(float s) {
  return s != s ? __ushort_as_half(static_cast<unsigned short>(0x7E00)) : __float2half_rn(s);
}

template <int DT>
__device__ __forceinline__ void store_scale(void* scale, int64_t row, float s) {
  if constexpr (DT == BW_DTYPE_F16) {
    static_cast<__half*>(scale)[row] = scale_to_f16(s);
  } else if constexpr (DT == BW_DTYPE_BF16) {
    static_cast<__nv_bfloat16*>(scale)[row] =
        s != s ? __ushort_as_bfloat16(static_cast<unsigned short>(0x7FC0)) : __float2bfloat16_rn(s);
  } else {
    static_cast<float*>(scale)[row] = s != s ? __int_as_float(0x7fc00000) : s;
  }
}

// scale from the row's absolute maximum (NaN-propagating like torch.amax)
template <int DT>
__device__ __forceinline__ float scale_from_amax(float amax, bool has_nan) {
  if (has_nan) return __int_as_float(0x7fc00000);
  const float amaxc = round_dt<DT>(fmaxf(amax, 1e-8f));
  return round_dt<DT>(__fdiv_rn(amaxc, 127.0f));
}

template <int DT>
__device__ __forceinline__ int8_t quant_one(float w, float s) {
  const float x = round_dt<DT>(__fdiv_rn(w, s));
  if (x != x) return 0;
  return static_cast<int8_t>(fminf(fmaxf(rintf(x), -127.0f), 127.0f));
}

// Same result as quant_one<DT>(w, s), faster.  With rcp = RN32(1/s),
// x = RN32(w * rcp) lies within 2.5 fp32 ulps of RN32(w / s).  Rounding x to
// dt (then to an integer) therefore gives the exact path's code unless x is
// within 4 fp32 ulps of a dt rounding midpoint (fp16: low 13 mantissa bits
// 0x1000; bf16: low 16 bits 0x8000), of an integer + 1/2 (fp32), or is not
// finite.  Those lanes take the IEEE division.  Quotients below 1/2 in
// magnitude give code 0 on both paths, so the fp16 subnormal range needs no
// check.
template <int DT>
__device__ __forceinline__ int8_t quant_fast(float w, float s, float rcp) {
  const float x = __fmul_rn(w, rcp);
  const float ax = fabsf(x);
  bool slow = !(ax < 1.0e30f);  // inf or NaN (zero scale, NaN input)
  if constexpr (DT == BW_DTYPE_F16) {
    const int d = static_cast<int>(__float_as_uint(x) & 0x1FFFu) - 0x1000;
    slow |= (ax >= 0.5f) && (d >= -4 && d <= 4);
  } else if constexpr (DT == BW_DTYPE_BF16) {
    const int d = static_cast<int>(__float_as_uint(x) & 0xFFFFu) - 0x8000;
    slow |= (ax >= 0.5f) && (d >= -4 && d <= 4);
  } else {
    slow |= fabsf(ax - floorf(ax) - 0.5f) <= 4.0e-5f;  // > 4 ulps for |x| < 256
  }
  if (slow) return quant_one<DT>(w, s);
  return static_cast<int8_t>(fminf(fmaxf(rintf(round_dt<DT>(x)), -127.0f), 127.0f));
}

// Four fp16 values (two half2 words) -> four int8 codes packed in one word,
// bit-identical to quant_fast / quant_one with dt = fp16, for a row whose
// scale is finite and non-zero (so every quotient is finite).  x = RN32(w * rcp)
// is rounded to fp16 in packed form, clamped to +-127 and rounded to an
// integer by adding 1536 (fp16 spacing is exactly 1 on [1024, 2048), so the
// addition is round-to-nearest-even, and the half's low byte is the code).
//
// No lane needs the exact division.  x differs from RN32(w / s) by at most a few
// fp32 ulps, so the two could only round to different fp16 values if w / s lay
// at or next to an fp16 rounding midpoint m.  It is never at one: w = m * s
// would make w's odd significand (at most 11 bits) a multiple of m's (12 bits,
// odd).  That it is never close enough to one is not argued but enumerated: for
// every finite fp16 w and every positive finite fp16 s (2.0e9 pairs, subnormal
// scales included) this packed path gives quant_one's code
// (tests/quant_fast_check.cpp, f16packed and f16packed_noclamp at stride 1).
// A midpoint check with an out-of-line fix-up cost the fused merge +
// requantisation kernel 16 % of its time.
//
// CLAMP = false is for rows whose scale is a normal fp16 number (>= 2^-14):
// then every |w| <= the row maximum gives |x| < 127.07, fp16(x) stays within
// +-127.0625 and the rounding lands on codes -127..127 without the clamp.
template <bool CLAMP = true>
__device__ __forceinline__ uint32_t quant4_f16(__half2 w01, __half2 w23, float s, float rcp) {
  (void)s;
  // packed fp32 multiplies: each lane is the IEEE round-to-nearest product
  const float2 x01 = __fmul2_rn(__half22float2(w01), make_float2(rcp, rcp));
  const float2 x23 = __fmul2_rn(__half22float2(w23), make_float2(rcp, rcp));
  const __half2 bias = __float2half2_rn(1536.0f);
  __half2 y01 = __float22half2_rn(x01);
  __half2 y23 = __float22half2_rn(x23);
  if constexpr (CLAMP) {
    const __half2 lim = __float2half2_rn(127.0f);
    const __half2 nlim = __float2half2_rn(-127.0f);
    y01 = __hmin2(__hmax2(y01, nlim), lim);
    y23 = __hmin2(__hmax2(y23, nlim), lim);
  }
  y01 = __hadd2(y01, bias);
  y23 = __hadd2(y23, bias);
  uint32_t packed;
  asm("prmt.b32 %0, %1, %2, 0x6420;" : "=r"(packed) : "r"(*reinterpret_cast<uint32_t*>(&y01)),
      "r"(*reinterpret_cast<uint32_t*>(&y23)));
  return packed;
}

// bf16 counterpart of quant4_f16, for a row whose scale is finite, non-zero and
// has a finite reciprocal: x = RN32(w * rcp) rounded to bf16 in packed form,
// clamped to +-127 in bf16, rounded to an integer by adding 1.5 * 2^23 in fp32
// (spacing 1 there, so the add is round-to-nearest-even) and the code is the low
// byte of the sum.  As for fp16, no lane needs the exact division: enumerated
// for every finite bf16 weight and every such scale (1.9e9 pairs,
// tests/quant_fast_check.cpp bf16packed at stride 1).
__device__ __forceinline__ uint32_t quant4_bf16(__nv_bfloat162 w01, __nv_bfloat162 w23, float s, float rcp) {
  (void)s;
  const float2 x01 = __fmul2_rn(__bfloat1622float2(w01), make_float2(rcp, rcp));
  const float2 x23 = __fmul2_rn(__bfloat1622float2(w23), make_float2(rcp, rcp));
  const __nv_bfloat162 lim = __float2bfloat162_rn(127.0f);
  const __nv_bfloat162 nlim = __float2bfloat162_rn(-127.0f);
  const __nv_bfloat162 y01 = __hmin2(__hmax2(__float22bfloat162_rn(x01), nlim), lim);
  const __nv_bfloat162 y23 = __hmin2(__hmax2(__float22bfloat162_rn(x23), nlim), lim);
  const float2 m = make_float2(12582912.0f, 12582912.0f);
  const float2 z01 = __fadd2_rn(__bfloat1622float2(y01), m);
  const float2 z23 = __fadd2_rn(__bfloat1622float2(y23), m);
  uint32_t t01, t23, packed;
  asm("prmt.b32 %0, %1, %2, 0x0040;" : "=r"(t01) : "r"(__float_as_uint(z01.x)), "r"(__float_as_uint(z01.y)));
  asm("prmt.b32 %0, %1, %2, 0x0040;" : "=r"(t23) : "r"(__float_as_uint(z23.x)), "r"(__float_as_uint(z23.y)));
  asm("prmt.b32 %0, %1, %2, 0x5410;" : "=r"(packed) : "r"(t01), "r"(t23));
  return packed;
}

// quant_one<fp16>'s codes, four at a time, for a row whose scale is not a
// finite positive number, in closed form: a NaN or +inf scale gives 0 for
// every element (w / inf = 0, inf / inf = NaN -> 0); a zero scale (a row of
// zeros and values below fp16's subnormal step) gives +-127 by sign and 0 for
// +-0 (0 / 0 = NaN -> 0).  Such a row holds no NaN or inf when its scale is 0.
__device__ __forceinline__ uint32_t quant4_special(__half2 w01, __half2 w23, float s) {
  if (s != 0.0f) return 0u;
  const float2 f01 = __half22float2(w01);
  const float2 f23 = __half22float2(w23);
  const float f[4] = {f01.x, f01.y, f23.x, f23.y};
  uint32_t packed = 0;
#pragma unroll
  for (int e = 0; e < 4; ++e) packed |= (f[e] > 0.0f ? 0x7Fu : (f[e] < 0.0f ? 0x81u : 0u)) << (8 * e);
  return packed;
}

}  // namespace bw
