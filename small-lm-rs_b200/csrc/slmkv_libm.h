// The host C library's single-precision exp and tanh, restated so that the
// GPU computes the same bits as the reference's CPU path.
//
// The reference calls f32::exp (softmax.rs:29, situ_glu.rs:131-138) and
// f32::tanh (situ_glu.rs:59-67); on Linux these lower to glibc's expf and
// tanhf. Neither is correctly rounded in glibc 2.39 (the image's C library),
// so CUDA's expf/tanhf, or a correctly rounded evaluation, differ from them
// in the last bit for some inputs; where the reference then rounds the value
// to bf16 (every projection input, linear.rs:14-23) one such bit can move a
// logit by ~1e-3. These functions restate the published algorithms glibc
// uses, operation by operation with explicit roundings, and are checked
// against the host's expf/tanhf for every float input by the tests:
//   slm_expf   glibc sysdeps/ieee754/flt-32/e_expf.c (Szabolcs Nagy's
//              algorithm from ARM's optimized-routines): k = round(x N/ln2),
//              2^(k/N) from a 32-entry table, a cubic in double precision,
//              one final rounding to float; in the x86-64 FMA build.
//   slm_expm1f glibc sysdeps/ieee754/flt-32/s_expm1f.c (Sun fdlibm).
//   slm_tanhf  glibc sysdeps/ieee754/flt-32/s_tanhf.c (Sun fdlibm), from
//              slm_expm1f.
// Header-only, __host__ __device__: the host build (compiled with
// -ffp-contract=off) is the one the tests compare with glibc; every
// operation is an explicitly rounded IEEE operation, so the device computes
// the same bits.
#pragma once

#include <cstdint>
#include <cstring>

#if defined(__CUDACC__)
#define SLM_HD __host__ __device__ __forceinline__
#else
#define SLM_HD inline
#endif

namespace slmkv {
namespace libm {

SLM_HD uint32_t f2u(float f) {
#if defined(__CUDA_ARCH__)
  return __float_as_uint(f);
#else
  uint32_t u;
  std::memcpy(&u, &f, 4);
  return u;
#endif
}
SLM_HD float u2f(uint32_t u) {
#if defined(__CUDA_ARCH__)
  return __uint_as_float(u);
#else
  float f;
  std::memcpy(&f, &u, 4);
  return f;
#endif
}
SLM_HD uint64_t d2u(double d) {
#if defined(__CUDA_ARCH__)
  return static_cast<uint64_t>(__double_as_longlong(d));
#else
  uint64_t u;
  std::memcpy(&u, &d, 8);
  return u;
#endif
}
SLM_HD double u2d(uint64_t u) {
#if defined(__CUDA_ARCH__)
  return __longlong_as_double(static_cast<long long>(u));
#else
  double d;
  std::memcpy(&d, &u, 8);
  return d;
#endif
}

// Explicitly rounded operations (no contraction on either side).
#if defined(__CUDA_ARCH__)
SLM_HD double dmul(double a, double b) { return __dmul_rn(a, b); }
SLM_HD double dadd(double a, double b) { return __dadd_rn(a, b); }
SLM_HD double dsub(double a, double b) { return __dsub_rn(a, b); }
SLM_HD double dfma(double a, double b, double c) { return __fma_rn(a, b, c); }
SLM_HD float fmul(float a, float b) { return __fmul_rn(a, b); }
SLM_HD float fadd(float a, float b) { return __fadd_rn(a, b); }
SLM_HD float fsub(float a, float b) { return __fsub_rn(a, b); }
SLM_HD float fdiv(float a, float b) { return __fdiv_rn(a, b); }
SLM_HD float d2f(double a) { return __double2float_rn(a); }
#else
SLM_HD double dmul(double a, double b) { return a * b; }
SLM_HD double dadd(double a, double b) { return a + b; }
SLM_HD double dsub(double a, double b) { return a - b; }
SLM_HD double dfma(double a, double b, double c) { return __builtin_fma(a, b, c); }
SLM_HD float fmul(float a, float b) { return a * b; }
SLM_HD float fadd(float a, float b) { return a + b; }
SLM_HD float fsub(float a, float b) { return a - b; }
SLM_HD float fdiv(float a, float b) { return a / b; }
SLM_HD float d2f(double a) { return static_cast<float>(a); }
#endif

// 2^(i/32) rounded to double, minus i << 47 (so that adding k << 47 to the
// bits of entry k % 32 gives 2^(k/32) for any integer k in range). The
// entries are the correctly rounded powers; the tests rederive them.
#define SLMKV_EXP2_TAB                                                                          \
  {0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull, \
   0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull, \
   0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull, \
   0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull, \
   0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull, \
   0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull, \
   0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull, \
   0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull}
#if defined(__CUDACC__)
__device__ __constant__ static const uint64_t kExp2TabDevice[32] = SLMKV_EXP2_TAB;
#endif
static const uint64_t kExp2TabHost[32] = SLMKV_EXP2_TAB;
#undef SLMKV_EXP2_TAB

SLM_HD uint64_t exp2_tab(uint32_t i) {
#if defined(__CUDA_ARCH__)
  return kExp2TabDevice[i];
#else
  return kExp2TabHost[i];
#endif
}

// e^x for a float x, as glibc's expf returns it.
SLM_HD float slm_expf(float x) {
  constexpr double kN = 32.0;
  constexpr double kInvLn2N = 0x1.71547652b82fep+0 * kN;
  constexpr double kShift = 0x1.8p+52;
  constexpr double kC0 = 0x1.c6af84b912394p-5 / kN / kN / kN;
  constexpr double kC1 = 0x1.ebfce50fac4f3p-3 / kN / kN;
  constexpr double kC2 = 0x1.62e42ff0c52d6p-1 / kN;
  const uint32_t ux = f2u(x);
  const uint32_t abstop = (ux >> 20) & 0x7ff;
  if (abstop >= (f2u(88.0f) >> 20)) {
    if (ux == f2u(-__builtin_inff())) return 0.0f;
    if (abstop >= (f2u(__builtin_inff()) >> 20)) return fadd(x, x);  // inf or NaN
    if (x > 0x1.62e42ep6f) return __builtin_inff();                 // overflow
    if (x < -0x1.9fe368p6f) return 0.0f;                             // underflow
  }
  const double xd = static_cast<double>(x);
  double z = dmul(kInvLn2N, xd);
  double kd = dadd(z, kShift);  // round to an integer (ties to even) in the low bits
  const uint64_t ki = d2u(kd);
  kd = dsub(kd, kShift);
  // z - kd with z's product unrounded: the x86-64 FMA build contracts it
  const double r = dfma(kInvLn2N, xd, -kd);
  uint64_t t = exp2_tab(static_cast<uint32_t>(ki % 32));
  t += ki << (52 - 5);
  const double s = u2d(t);
  z = dfma(kC0, r, kC1);
  const double r2 = dmul(r, r);
  double y = dfma(kC2, r, 1.0);
  y = dfma(z, r2, y);
  y = dmul(y, s);
  return d2f(y);
}

// e^x - 1 for a float x, as glibc's expm1f returns it (finite x).
SLM_HD float slm_expm1f(float x) {
  const float o_threshold = 8.8721679688e+01f;
  const float ln2_hi = 6.9313812256e-01f;
  const float ln2_lo = 9.0580006145e-06f;
  const float invln2 = 1.4426950216e+00f;
  const float Q1 = -3.3333335072e-02f, Q2 = 1.5873016091e-03f, Q3 = -7.9365076090e-05f,
              Q4 = 4.0082177293e-06f, Q5 = -2.0109921195e-07f;
  float y, hi, lo, c = 0.0f, t, e, hxs, hfx, r1;
  int32_t k;
  uint32_t hx = f2u(x);
  const uint32_t xsb = hx & 0x80000000u;
  y = xsb == 0 ? x : -x;
  (void)y;
  hx &= 0x7fffffffu;
  if (hx >= 0x4195b844u) {          // |x| >= 27 ln2
    if (hx >= 0x42b17218u) {        // |x| >= 88.72...
      if (hx > 0x7f800000u) return fadd(x, x);
      if (hx == 0x7f800000u) return xsb == 0 ? x : -1.0f;
      if (x > o_threshold) return __builtin_inff();
    }
    if (xsb != 0) return -1.0f;     // tiny - one
  }
  if (hx > 0x3eb17218u) {           // |x| > 0.5 ln2
    if (hx < 0x3F851592u) {         // and |x| < 1.5 ln2
      if (xsb == 0) {
        hi = fsub(x, ln2_hi);
        lo = ln2_lo;
        k = 1;
      } else {
        hi = fadd(x, ln2_hi);
        lo = -ln2_lo;
        k = -1;
      }
    } else {
      k = static_cast<int32_t>(fadd(fmul(invln2, x), xsb == 0 ? 0.5f : -0.5f));
      t = static_cast<float>(k);
      hi = fsub(x, fmul(t, ln2_hi));
      lo = fmul(t, ln2_lo);
    }
    x = fsub(hi, lo);
    c = fsub(fsub(hi, x), lo);
  } else if (hx < 0x33000000u) {    // |x| < 2^-25: x
    return x;
  } else {
    k = 0;
  }
  hfx = fmul(0.5f, x);
  hxs = fmul(x, hfx);
  r1 = fadd(1.0f, fmul(hxs, fadd(Q1, fmul(hxs, fadd(Q2, fmul(hxs, fadd(Q3, fmul(hxs,
                                                           fadd(Q4, fmul(hxs, Q5))))))))));
  t = fsub(3.0f, fmul(r1, hfx));
  e = fmul(hxs, fdiv(fsub(r1, t), fsub(6.0f, fmul(x, t))));
  if (k == 0) return fsub(x, fsub(fmul(x, e), hxs));
  e = fsub(fmul(x, fsub(e, c)), c);
  e = fsub(e, hxs);
  if (k == -1) return fsub(fmul(0.5f, fsub(x, e)), 0.5f);
  if (k == 1) {
    if (x < -0.25f) return fmul(-2.0f, fsub(e, fadd(x, 0.5f)));
    return fadd(1.0f, fmul(2.0f, fsub(x, e)));
  }
  if (k <= -2 || k > 56) {          // exp(x) - 1 suffices
    y = fsub(1.0f, fsub(e, x));
    y = u2f(f2u(y) + (static_cast<uint32_t>(k) << 23));
    return fsub(y, 1.0f);
  }
  if (k < 23) {
    t = u2f(0x3f800000u - (0x1000000u >> k));  // 1 - 2^-k
    y = fsub(t, fsub(e, x));
    y = u2f(f2u(y) + (static_cast<uint32_t>(k) << 23));
  } else {
    t = u2f(static_cast<uint32_t>(0x7f - k) << 23);  // 2^-k
    y = fsub(x, fadd(e, t));
    y = fadd(y, 1.0f);
    y = u2f(f2u(y) + (static_cast<uint32_t>(k) << 23));
  }
  return y;
}

// tanh(x) for a float x, as glibc's tanhf returns it.
SLM_HD float slm_tanhf(float x) {
  const uint32_t jx = f2u(x);
  const uint32_t ix = jx & 0x7fffffffu;
  float z;
  if (ix >= 0x7f800000u) {  // inf or NaN
    if ((jx & 0x80000000u) == 0) return fadd(fdiv(1.0f, x), 1.0f);
    return fsub(fdiv(1.0f, x), 1.0f);
  }
  if (ix < 0x41b00000u) {   // |x| < 22
    if (ix == 0) return x;
    if (ix < 0x24000000u) return fmul(x, fadd(1.0f, x));  // |x| < 2^-55
    const float ax = u2f(ix);
    if (ix >= 0x3f800000u) {  // |x| >= 1
      const float t = slm_expm1f(fmul(2.0f, ax));
      z = fsub(1.0f, fdiv(2.0f, fadd(t, 2.0f)));
    } else {
      const float t = slm_expm1f(fmul(-2.0f, ax));
      z = fdiv(-t, fadd(t, 2.0f));
    }
  } else {
    z = 1.0f;  // one - tiny
  }
  return (jx & 0x80000000u) == 0 ? z : -z;
}

}  // namespace libm
}  // namespace slmkv
