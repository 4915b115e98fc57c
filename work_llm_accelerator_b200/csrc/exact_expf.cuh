// exact_expf: the host C library's single-precision exp, restated for the GPU (used wherever a kernel must
// reproduce the reference host code's std::exp on floats bit for bit).
#pragma once

#include <cstdint>

namespace qb {

// ------------------------------------------------------------------------------------------------
// exact_expf: glibc's expf (sysdeps/ieee754/flt-32/e_expf.c since glibc 2.27), which is the algorithm of
// ARM's optimized-routines expf (Szabolcs Nagy, 2017; MIT / Apache-2.0), restated:
//   x / ln2 * 32 = k + r with k = round-to-nearest integer (the 1.5 * 2^52 shift trick), |r| <= 1/2;
//   2^(k/32) = double(T[k % 32] + (k << 47)) with T[i] = bits(RN(2^(i/32))) - (i << 47);
//   2^(r/32) ~= C0 r^3 + C1 r^2 + C2 r + 1 (a degree-3 fit published with the routine, here pre-divided by
//   32^3, 32^2 and 32);  expf = float(s * poly), everything but the last rounding in double.
// The reference host library resolves expf to glibc's FMA build on FMA-capable x86-64 hosts, whose code
// fuses the multiply-adds marked below; with those fusions this restatement equals that expf on every one
// of the 2^32 fp32 inputs (checked exhaustively against glibc 2.39), and the GPU test compares it with the
// host's expf again. The table values are RN(2^(i/32)) computed with 60-digit decimal arithmetic.
// ------------------------------------------------------------------------------------------------
static __constant__ unsigned long long c_exp2_tab[32] = {
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull};

__device__ __forceinline__ float exact_expf(float x) {
  constexpr double kInvLn2N = 0x1.71547652b82fep+5;  // 32 / ln 2
  constexpr double kShift = 0x1.8p+52;
  constexpr double kC0 = 0x1.c6af84b912394p-20;  // 0x1.c6af84b912394p-5 / 32^3
  constexpr double kC1 = 0x1.ebfce50fac4f3p-13;  // 0x1.ebfce50fac4f3p-3 / 32^2
  constexpr double kC2 = 0x1.62e42ff0c52d6p-6;   // 0x1.62e42ff0c52d6p-1 / 32
  const uint32_t ux = __float_as_uint(x);
  const uint32_t abstop = (ux >> 20) & 0x7ffu;
  if (abstop >= 0x42bu) {  // |x| >= 88, inf or nan
    if (ux == 0xff800000u) return 0.0f;                      // -inf
    if (abstop >= 0x7f8u) return __fadd_rn(x, x);            // +inf, nan
    if (x > 0x1.62e42ep6f) return __uint_as_float(0x7f800000u);  // overflow
    if (x < -0x1.9fe368p6f) return 0.0f;                     // underflow
  }
  const double xd = (double)x;
  double kd = __fma_rn(kInvLn2N, xd, kShift);  // fused in the FMA build
  const unsigned long long ki = (unsigned long long)__double_as_longlong(kd);
  kd = __dsub_rn(kd, kShift);
  const double r = __fma_rn(kInvLn2N, xd, -kd);  // fused in the FMA build
  const unsigned long long t = c_exp2_tab[ki % 32] + (ki << 47);
  const double s = __longlong_as_double((long long)t);
  const double z = __fma_rn(kC0, r, kC1);
  const double r2 = __dmul_rn(r, r);
  double y = __fma_rn(kC2, r, 1.0);
  y = __fma_rn(z, r2, y);
  y = __dmul_rn(y, s);
  return __double2float_rn(y);
}

}  // namespace qb
