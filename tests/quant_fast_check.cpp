// Exhaustive CPU check of the fast quantiser path used by the kernels
// (csrc/quant_math.cuh: quant_fast vs quant_one).  Test infrastructure only.
//
// For every finite weight w and every positive finite scale s of the dtype,
// the fast path (x = RN32(w * RN32(1/s)), exact division only when x is within
// 4 fp32 ulps of a rounding midpoint, non-finite, or (fp32) near an integer +
// 1/2; the packed fp16 and bf16 paths have no such fix-up at all) must give the
// same int8 code as the exact path
// (clamp(rint(dt(RN32(w / s))), -127, 127), NaN -> 0).  x86-64 SSE float
// arithmetic is IEEE single precision; build without fast-math or FP
// contraction.
//
// usage: quant_fast_check f16|bf16|f32|f16packed|f16packed_noclamp|bf16packed [scale_stride]
//   -> prints "mismatches=<n> slow=<n> total=<n>"; scale_stride > 1 checks every
//   stride-th scale (all weights) to bound the run time.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <vector>

static float bits_to_f(uint32_t b) { float f; std::memcpy(&f, &b, 4); return f; }
static uint32_t f_to_bits(float f) { uint32_t b; std::memcpy(&b, &f, 4); return b; }

static float f16_to_f(uint16_t h) { _Float16 v; std::memcpy(&v, &h, 2); return static_cast<float>(v); }
static float round_f16(float x) { return static_cast<float>(static_cast<_Float16>(x)); }
static float bf16_to_f(uint16_t h) { return bits_to_f(static_cast<uint32_t>(h) << 16); }
static float round_bf16(float x) {
  uint32_t u = f_to_bits(x);
  if (std::isnan(x)) return x;
  u = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
  return bits_to_f(u);
}

enum { F16 = 0, BF16 = 1, F32 = 2 };

template <int DT> static float round_dt(float x) {
  if (DT == F16) return round_f16(x);
  if (DT == BF16) return round_bf16(x);
  return x;
}

template <int DT> static int8_t quant_exact(float w, float s) {
  volatile float q = w / s;  // IEEE division
  const float x = round_dt<DT>(q);
  if (x != x) return 0;
  return static_cast<int8_t>(std::fmin(std::fmax(std::rint(x), -127.0f), 127.0f));
}

template <int DT> static int8_t quant_fast(float w, float s, float rcp, long* slow_count) {
  volatile float x = w * rcp;
  const float ax = std::fabs(x);
  bool slow = !(ax < 1.0e30f);
  if (DT == F16) {
    const int d = static_cast<int>(f_to_bits(x) & 0x1FFFu) - 0x1000;
    slow |= (ax >= 0.5f) && (d >= -4 && d <= 4);
  } else if (DT == BF16) {
    const int d = static_cast<int>(f_to_bits(x) & 0xFFFFu) - 0x8000;
    slow |= (ax >= 0.5f) && (d >= -4 && d <= 4);
  } else {
    slow |= std::fabs(ax - std::floor(ax) - 0.5f) <= 4.0e-5f;
  }
  if (slow) {
    ++*slow_count;
    return quant_exact<DT>(w, s);
  }
  return static_cast<int8_t>(std::fmin(std::fmax(std::rint(round_dt<DT>(x)), -127.0f), 127.0f));
}

// Emulation of quant4_f16 (csrc/quant_math.cuh) for one element: packed fp16
// rounding, fp16 clamp to +-127, +1536 in fp16 (round-to-nearest-even to an
// integer), code = low byte of the half.  No exact-division fix-up: the kernel
// has none, and the sweep shows that none is needed.  Valid for finite, non-zero
// scales.
static int8_t quant_packed_f16(float w, float s, float rcp, long* slow_count) {
  (void)s;
  (void)slow_count;
  volatile float x = w * rcp;
  _Float16 y = static_cast<_Float16>(x);
  if (y > static_cast<_Float16>(127.0f)) y = static_cast<_Float16>(127.0f);
  if (y < static_cast<_Float16>(-127.0f)) y = static_cast<_Float16>(-127.0f);
  volatile _Float16 z = static_cast<_Float16>(static_cast<float>(y) + 1536.0f);
  uint16_t bits;
  _Float16 zz = z;
  std::memcpy(&bits, &zz, 2);
  return static_cast<int8_t>(bits & 0xFF);
}

// quant4_f16 without the +-127 clamp, used for rows whose scale is a normal
// fp16 number: every |w| <= amax of the row gives |x| < 127.07, so fp16(x)
// stays within +-127.0625 and the +1536 rounding lands on 1409..1663.  No
// midpoint check and no exact-division fix-up, as in the kernel.
static int8_t quant_packed_f16_noclamp(float w, float s, float rcp, long* slow_count) {
  (void)s;
  (void)slow_count;
  volatile float x = w * rcp;
  const _Float16 y = static_cast<_Float16>(x);
  volatile _Float16 z = static_cast<_Float16>(static_cast<float>(y) + 1536.0f);
  uint16_t bits;
  _Float16 zz = z;
  std::memcpy(&bits, &zz, 2);
  return static_cast<int8_t>(bits & 0xFF);
}

// Every (w, s) a row can hold: s = the quantiser's scale of the row maximum a
// (csrc/quant_math.cuh: scale_from_amax), |w| <= a, s normal (>= 2^-14).
static void run_packed_noclamp(int stride) {
  std::vector<float> scale_of, amax_of;  // distinct scales with the largest row maximum giving each
  for (uint32_t h = 1; h < 0x7C00u; ++h) {
    const float a = f16_to_f(static_cast<uint16_t>(h));
    volatile float den = 127.0f;
    const float amaxc = round_f16(std::fmax(a, 1e-8f));
    const float s = round_f16(amaxc / den);
    if (!(s >= 6.103515625e-05f) || !std::isfinite(s)) continue;
    if (!scale_of.empty() && scale_of.back() == s) amax_of.back() = a;
    else { scale_of.push_back(s); amax_of.push_back(a); }
  }
  std::vector<float> weights;
  for (uint32_t h = 0; h < 0x10000u; ++h) {
    const float v = f16_to_f(static_cast<uint16_t>(h));
    if (std::isfinite(v)) weights.push_back(v);
  }
  const int nt = std::max(1u, std::thread::hardware_concurrency());
  std::vector<long> mism(nt, 0), slow(nt, 0), total(nt, 0);
  std::vector<std::thread> th;
  for (int t = 0; t < nt; ++t) {
    th.emplace_back([&, t] {
      for (size_t i = static_cast<size_t>(t) * stride; i < scale_of.size(); i += static_cast<size_t>(nt) * stride) {
        const float s = scale_of[i], a = amax_of[i];
        volatile float one = 1.0f;
        const float rcp = one / s;
        for (float w : weights) {
          if (std::fabs(w) > a) continue;
          if (quant_packed_f16_noclamp(w, s, rcp, &slow[t]) != quant_exact<F16>(w, s)) ++mism[t];
          ++total[t];
        }
      }
    });
  }
  for (auto& x : th) x.join();
  long m = 0, sl = 0, tot = 0;
  for (int t = 0; t < nt; ++t) { m += mism[t]; sl += slow[t]; tot += total[t]; }
  std::printf("mismatches=%ld slow=%ld total=%ld\n", m, sl, tot);
}

// Emulation of quant4_bf16 (csrc/quant_math.cuh) for one element: x = RN32(w*rcp)
// rounded to bf16, clamped to +-127 in bf16, rounded to an integer by adding
// 1.5*2^23 in fp32 (spacing 1 there: round-to-nearest-even), code = low byte of
// the sum's bits.  No exact-division fix-up, as in the kernel.  Valid for
// finite, non-zero scales.
static int8_t quant_packed_bf16(float w, float s, float rcp, long* slow_count) {
  (void)s;
  (void)slow_count;
  volatile float x = w * rcp;
  float y = round_bf16(x);
  if (y > 127.0f) y = 127.0f;
  if (y < -127.0f) y = -127.0f;
  volatile float z = y + 12582912.0f;
  return static_cast<int8_t>(f_to_bits(z) & 0xFF);
}

static void run_packed_bf16(int stride) {
  std::vector<float> scales, weights;
  for (uint32_t h = 1; h < 0x7F80u; ++h) scales.push_back(bf16_to_f(static_cast<uint16_t>(h)));
  for (uint32_t h = 0; h < 0x10000u; ++h) {
    const float v = bf16_to_f(static_cast<uint16_t>(h));
    if (std::isfinite(v)) weights.push_back(v);
  }
  const int nt = std::max(1u, std::thread::hardware_concurrency());
  std::vector<long> mism(nt, 0), slow(nt, 0), total(nt, 0);
  std::vector<std::thread> th;
  for (int t = 0; t < nt; ++t) {
    th.emplace_back([&, t] {
      for (size_t i = static_cast<size_t>(t) * stride; i < scales.size(); i += static_cast<size_t>(nt) * stride) {
        const float s = scales[i];
        volatile float one = 1.0f;
        const float rcp = one / s;
        if (!(rcp < 1.0e30f)) continue;  // the kernel takes the exact path for such scales
        for (float w : weights) {
          if (quant_packed_bf16(w, s, rcp, &slow[t]) != quant_exact<BF16>(w, s)) ++mism[t];
          ++total[t];
        }
      }
    });
  }
  for (auto& x : th) x.join();
  long m = 0, sl = 0, tot = 0;
  for (int t = 0; t < nt; ++t) { m += mism[t]; sl += slow[t]; tot += total[t]; }
  std::printf("mismatches=%ld slow=%ld total=%ld\n", m, sl, tot);
}

static void run_packed(int stride) {
  std::vector<float> scales, weights;
  for (uint32_t h = 1; h < 0x7C00u; ++h) scales.push_back(f16_to_f(static_cast<uint16_t>(h)));
  for (uint32_t h = 0; h < 0x10000u; ++h) {
    const float v = f16_to_f(static_cast<uint16_t>(h));
    if (std::isfinite(v)) weights.push_back(v);
  }
  const int nt = std::max(1u, std::thread::hardware_concurrency());
  std::vector<long> mism(nt, 0), slow(nt, 0), total(nt, 0);
  std::vector<std::thread> th;
  for (int t = 0; t < nt; ++t) {
    th.emplace_back([&, t] {
      for (size_t i = static_cast<size_t>(t) * stride; i < scales.size(); i += static_cast<size_t>(nt) * stride) {
        const float s = scales[i];
        volatile float one = 1.0f;
        const float rcp = one / s;
        for (float w : weights) {
          if (quant_packed_f16(w, s, rcp, &slow[t]) != quant_exact<F16>(w, s)) ++mism[t];
          ++total[t];
        }
      }
    });
  }
  for (auto& x : th) x.join();
  long m = 0, sl = 0, tot = 0;
  for (int t = 0; t < nt; ++t) { m += mism[t]; sl += slow[t]; tot += total[t]; }
  std::printf("mismatches=%ld slow=%ld total=%ld\n", m, sl, tot);
}

template <int DT> static void run(int stride) {
  // scales: every non-negative finite value of the dtype (fp32: a dense log sweep)
  std::vector<float> scales, weights;
  if (DT == F32) {
    for (int e = -30; e <= 10; ++e)
      for (int m = 0; m < 64; ++m) scales.push_back(std::ldexp(1.0f + m / 64.0f + 1.0f / 8192, e));
    scales.push_back(0.0f);
    for (uint32_t b = 0; b < 0x7F800000u; b += 99991) {  // ~21K magnitudes x 2 signs over all finite floats
      weights.push_back(bits_to_f(b));
      weights.push_back(-bits_to_f(b));
    }
  } else {
    for (uint32_t h = 0; h < 0x7C00u + (DT == BF16 ? 0x0380u : 0u); ++h) {
      const float v = DT == F16 ? f16_to_f(static_cast<uint16_t>(h)) : bf16_to_f(static_cast<uint16_t>(h));
      if (std::isfinite(v)) scales.push_back(v);
    }
    for (uint32_t h = 0; h < 0x10000u; ++h) {
      const float v = DT == F16 ? f16_to_f(static_cast<uint16_t>(h)) : bf16_to_f(static_cast<uint16_t>(h));
      if (std::isfinite(v)) weights.push_back(v);
    }
  }
  const int nt = std::max(1u, std::thread::hardware_concurrency());
  std::vector<long> mism(nt, 0), slow(nt, 0), total(nt, 0);
  std::vector<std::thread> th;
  for (int t = 0; t < nt; ++t) {
    th.emplace_back([&, t] {
      for (size_t i = static_cast<size_t>(t) * stride; i < scales.size(); i += static_cast<size_t>(nt) * stride) {
        const float s = scales[i];
        volatile float one = 1.0f;
        const float rcp = one / s;  // RN32(1/s)
        for (float w : weights) {
          if (quant_fast<DT>(w, s, rcp, &slow[t]) != quant_exact<DT>(w, s)) ++mism[t];
          ++total[t];
        }
      }
    });
  }
  for (auto& x : th) x.join();
  long m = 0, sl = 0, tot = 0;
  for (int t = 0; t < nt; ++t) { m += mism[t]; sl += slow[t]; tot += total[t]; }
  std::printf("mismatches=%ld slow=%ld total=%ld\n", m, sl, tot);
}

int main(int argc, char** argv) {
  if (argc < 2) return 2;
  const int stride = argc > 2 ? std::atoi(argv[2]) : 1;
  if (!std::strcmp(argv[1], "f16")) run<F16>(stride);
  else if (!std::strcmp(argv[1], "bf16")) run<BF16>(stride);
  else if (!std::strcmp(argv[1], "f32")) run<F32>(stride);
  else if (!std::strcmp(argv[1], "f16packed")) run_packed(stride);
  else if (!std::strcmp(argv[1], "f16packed_noclamp")) run_packed_noclamp(stride);
  else if (!std::strcmp(argv[1], "bf16packed")) run_packed_bf16(stride);
  else return 2;
  return 0;
}
