// vtq_libm.h -- the software single-precision transcendentals the reference's
// decode path uses, restated so their bits are the same on every machine.
//
// The reference calls the Rust `libm` crate (version "0.2", Cargo.toml:23; a
// port of musl's libm, whose single-precision functions are Bruce Evans'
// FreeBSD msun algorithms): expf (SiLU forward_quantized.rs:559, softmax :934),
// sqrtf (rms_norm.rs:102, attention scale :486), powf/cosf/sinf (RoPE :453-456).
// The algorithms below follow those published methods -- argument reduction by
// ln2 / pi/2 split constants, the msun minimax polynomials, the same evaluation
// order -- written for this project. The bits are pinned by the reference's
// own sweep hash (tests/transcendental_determinism.rs:14-67), checked in
// tests/test_libm.py.
//
// sqrtf is correctly rounded in every IEEE implementation (sqrtf on the host,
// __fsqrt_rn on the device), so it needs no restatement.
//
// expf is __host__ __device__ (the device computes SiLU and softmax with it);
// sinf/cosf/powf run on the host only (RoPE tables are precomputed per position).
// Host code must be built without FMA contraction (-ffp-contract=off).
//
// Notices of the published algorithms these functions restate:
//   FreeBSD msun (e_expf.c, k_sinf.c, k_cosf.c, e_powf.c, e_rem_pio2f.c):
//     Copyright (C) 1993 by Sun Microsystems, Inc. All rights reserved.
//     Developed at SunPro, a Sun Microsystems, Inc. business.
//     Permission to use, copy, modify, and distribute this software is freely
//     granted, provided that this notice is preserved.
//     Float versions by Ian Lance Taylor, Cygnus Support, and Bruce D. Evans.
//   musl libm (the C sources the Rust `libm` crate ports): Copyright (c)
//     2005-2020 Rich Felker, et al., MIT licence: permission is granted, free
//     of charge, to deal in the software without restriction, provided the
//     copyright notice and this permission notice are included.
#pragma once
#include <cmath>
#include <cstdint>
#include <cstring>

#ifdef __CUDACC__
#define VTQ_HD __host__ __device__ __forceinline__
#else
#define VTQ_HD inline
#endif

namespace vtq {
namespace libm {

VTQ_HD uint32_t fbits(float f) {
#ifdef __CUDA_ARCH__
  return __float_as_uint(f);
#else
  uint32_t u;
  std::memcpy(&u, &f, 4);
  return u;
#endif
}
VTQ_HD float ffrom(uint32_t u) {
#ifdef __CUDA_ARCH__
  return __uint_as_float(u);
#else
  float f;
  std::memcpy(&f, &u, 4);
  return f;
#endif
}

// Round-to-nearest single operations that the device compiler may not fuse.
#ifdef __CUDA_ARCH__
VTQ_HD float fmul(float a, float b) { return __fmul_rn(a, b); }
VTQ_HD float fadd(float a, float b) { return __fadd_rn(a, b); }
VTQ_HD float fsub(float a, float b) { return __fsub_rn(a, b); }
VTQ_HD float fdiv(float a, float b) { return __fdiv_rn(a, b); }
#else
VTQ_HD float fmul(float a, float b) { return a * b; }
VTQ_HD float fadd(float a, float b) { return a + b; }
VTQ_HD float fsub(float a, float b) { return a - b; }
VTQ_HD float fdiv(float a, float b) { return a / b; }
#endif

// x * 2^n with the steps of a correct scalbnf: pre-scale by 2^127 or
// 2^-102 (at most twice) when 2^n is not a normal float, then one multiply.
VTQ_HD float scalbnf(float x, int n) {
  float y = x;
  if (n > 127) {
    y = fmul(y, ffrom(0x7f000000u));  // 2^127
    n -= 127;
    if (n > 127) {
      y = fmul(y, ffrom(0x7f000000u));
      n -= 127;
      if (n > 127) n = 127;
    }
  } else if (n < -126) {
    y = fmul(y, ffrom(0x0c800000u));  // 2^-126 * 2^24 = 2^-102
    n += 126 - 24;
    if (n < -126) {
      y = fmul(y, ffrom(0x0c800000u));
      n += 126 - 24;
      if (n < -126) n = -126;
    }
  }
  return fmul(y, ffrom((uint32_t)(0x7f + n) << 23));
}

// exp(x) (msun e_expf method): k = round(x / ln2); r = x - k*ln2 (ln2 split
// hi/lo so k*ln2hi is exact); exp(r) from the degree-2 minimax R(r) of
// r*(exp(r)+1)/(exp(r)-1) on [-0.34568, 0.34568]; scale by 2^k.
VTQ_HD float expf(float x) {
  const float ln2hi = ffrom(0x3f317200u);   // 6.9314575195e-01
  const float ln2lo = ffrom(0x35bfbe8eu);   // 1.4286067653e-06
  const float invln2 = ffrom(0x3fb8aa3bu);  // 1.4426950216e+00
  const float P1 = ffrom(0x3e2aaa8fu);      // 1.6666625440e-01
  const float P2 = ffrom(0xbb355215u);      // -2.7667332906e-03
  uint32_t hx = fbits(x);
  const int sign = (int)(hx >> 31);
  hx &= 0x7fffffffu;
  if (hx >= 0x42aeac50u) {                 // |x| >= 87.33655 or NaN
    if (hx > 0x7f800000u) return x;        // NaN
    if (hx >= 0x42b17218u && !sign) return fmul(x, ffrom(0x7f000000u));  // overflow
    if (sign && hx >= 0x42cff1b5u) return 0.0f;  // x <= -103.972084: underflow to 0
  }
  float hi, lo;
  int k;
  if (hx > 0x3eb17218u) {                  // |x| > 0.5 ln2
    if (hx > 0x3f851592u)                  // |x| > 1.5 ln2
      k = (int)fadd(fmul(invln2, x), sign ? -0.5f : 0.5f);
    else
      k = 1 - sign - sign;
    const float kf = (float)k;
    hi = fsub(x, fmul(kf, ln2hi));
    lo = fmul(kf, ln2lo);
    x = fsub(hi, lo);
  } else if (hx > 0x39000000u) {           // |x| > 2^-14
    k = 0;
    hi = x;
    lo = 0.0f;
  } else {
    return fadd(1.0f, x);
  }
  const float xx = fmul(x, x);
  const float c = fsub(x, fmul(xx, fadd(P1, fmul(xx, P2))));
  const float y = fadd(1.0f, fadd(fsub(fdiv(fmul(x, c), fsub(2.0f, c)), lo), hi));
  return k == 0 ? y : scalbnf(y, k);
}

// Host-only functions below (RoPE tables); nvcc parses them in the device
// pass but never generates device code for them.

// sin / cos on [-pi/4, pi/4] in double (msun k_sinf / k_cosf minimax
// polynomials, evaluated in the published grouping), rounded once to float.
inline float sin_kernel(double x) {
  const double S1 = -0x15555554cbac77.0p-55, S2 = 0x111110896efbb2.0p-59,
               S3 = -0x1a00f9e2cae774.0p-65, S4 = 0x16cd878c3b46a7.0p-71;
  const double z = x * x, w = z * z, r = S3 + z * S4, s = z * x;
  return (float)((x + s * (S1 + z * S2)) + s * w * r);
}
inline float cos_kernel(double x) {
  const double C0 = -0x1ffffffd0c5e81.0p-54, C1 = 0x155553e1053a42.0p-57,
               C2 = -0x16c087e80f1e27.0p-62, C3 = 0x199342e0ee5069.0p-68;
  const double z = x * x, w = z * z, r = C2 + z * C3;
  return (float)(((1.0 + z * C0) + w * C1) + (w * z) * r);
}

// 2/pi as a binary fraction: 320 bits, most significant first (computed from
// Machin's formula; 0.A2F9836E4E44... in hex).
static const uint32_t kTwoOverPi[10] = {0xA2F9836Eu, 0x4E441529u, 0xFC2757D1u, 0xF534DDC0u,
                                        0xDB629599u, 0x3C439041u, 0xFE5163ABu, 0xDEBBC561u,
                                        0xB7246E3Au, 0x424DD2E0u};

// Bits [pos, pos + 64) of 2/pi (bit 1 = first fraction bit) as a 64-bit word.
inline uint64_t two_over_pi_bits(int pos) {
  uint64_t v = 0;
  for (int i = 0; i < 64; i++) {
    const int b = pos + i;  // 1-based
    const int w = (b - 1) >> 5, o = 31 - ((b - 1) & 31);
    const uint64_t bit = (b >= 1 && w < 10) ? ((kTwoOverPi[w] >> o) & 1u) : 0u;
    v = (v << 1) | bit;
  }
  return v;
}

// Reduce a float to (quadrant n, y in about [-pi/4, pi/4]) with x = n*pi/2 + y.
// |x| < 2^28 * pi/2: one double-precision step with pi/2 split into a 33-bit
// head and its tail (as msun's __rem_pio2f). Larger |x|: exact integer
// multiplication by the bits of 2/pi (Payne-Hanek), remainder rounded to double.
inline int rem_pio2f(float x, double* y) {
  const double toint = 1.5 / 2.220446049250313e-16;  // 1.5 * 2^52
  const double pio4 = 0x1.921fb6p-1;
  const double invpio2 = 6.36619772367581382433e-01;
  const double pio2_1 = 1.57079631090164184570e+00;   // first 33 bits of pi/2
  const double pio2_1t = 1.58932547735281966916e-08;  // pi/2 - pio2_1
  const uint32_t ix = fbits(x) & 0x7fffffffu;
  if (ix < 0x4dc90fdbu) {
    double fn = (double)x * invpio2 + toint - toint;
    int n = (int)fn;
    *y = x - fn * pio2_1 - fn * pio2_1t;
    if (*y < -pio4) {
      n--;
      fn--;
      *y = x - fn * pio2_1 - fn * pio2_1t;
    } else if (*y > pio4) {
      n++;
      fn++;
      *y = x - fn * pio2_1 - fn * pio2_1t;
    }
    return n;
  }
  if (ix >= 0x7f800000u) {
    *y = (double)(x - x);
    return 0;
  }
  // |x| = m * 2^e, m < 2^24, e >= 5. x*(2/pi) = m * 2^e * T. Bits of T at
  // positions <= e - 2 contribute multiples of 4 (whole turns) and are dropped.
  const int e = (int)(ix >> 23) - 127 - 23;
  const uint64_t m = (ix & 0x7fffffu) | 0x800000u;
  // Window: bits (e-1) .. (e+126) of T as a 128-bit integer W; the kept part
  // of x*T is m * W * 2^-126.
  const uint64_t hiw = two_over_pi_bits(e - 1), low = two_over_pi_bits(e + 63);
  const unsigned __int128 p_lo = (unsigned __int128)m * low;
  const unsigned __int128 p_hi = (unsigned __int128)m * hiw + (uint64_t)(p_lo >> 64);
  // value = (p_hi * 2^64 + (uint64)p_lo) * 2^-126: integer part = p_hi >> 62.
  const int quad = (int)((p_hi >> 62) & 3u);
  const unsigned __int128 f128 = ((p_hi & ((((unsigned __int128)1) << 62) - 1)) << 66) |
                                 ((unsigned __int128)(uint64_t)p_lo << 2);
  long double f = (long double)(uint64_t)(f128 >> 64) / 18446744073709551616.0L +
                  (long double)(uint64_t)f128 / 18446744073709551616.0L / 18446744073709551616.0L;
  int n = quad;
  if (f >= 0.5L) {
    f -= 1.0L;
    n = (n + 1) & 3;
  }
  const long double pio2l = 1.5707963267948966192313216916397514L;
  double r = (double)(f * pio2l);
  if (fbits(x) >> 31) {
    r = -r;
    n = -n;
  }
  *y = r;
  return n;
}

// sin(x) (msun s_sinf method): |x| <= 9pi/4 reduced by the nearest multiple of
// pi/2 in double; beyond that through rem_pio2f.
inline float sinf(float x) {
  const double p1 = 1 * 1.57079632679489661923, p2 = 2 * 1.57079632679489661923,
               p3 = 3 * 1.57079632679489661923, p4 = 4 * 1.57079632679489661923;
  const uint32_t hx = fbits(x), ix = hx & 0x7fffffffu;
  const bool neg = hx >> 31;
  if (ix <= 0x3f490fdau) {                   // |x| <= ~pi/4
    if (ix < 0x39800000u) return x;          // |x| < 2^-12
    return sin_kernel(x);
  }
  if (ix <= 0x407b53d1u) {                   // |x| <= ~5pi/4
    if (ix <= 0x4016cbe3u)                   // |x| <= ~3pi/4
      return neg ? -cos_kernel(x + p1) : cos_kernel(x - p1);
    return sin_kernel(neg ? -(x + p2) : -(x - p2));
  }
  if (ix <= 0x40e231d5u) {                   // |x| <= ~9pi/4
    if (ix <= 0x40afeddfu)                   // |x| <= ~7pi/4
      return neg ? cos_kernel(x + p3) : -cos_kernel(x - p3);
    return sin_kernel(neg ? x + p4 : x - p4);
  }
  if (ix >= 0x7f800000u) return x - x;
  double y;
  const int n = rem_pio2f(x, &y);
  switch (n & 3) {
    case 0: return sin_kernel(y);
    case 1: return cos_kernel(y);
    case 2: return sin_kernel(-y);
    default: return -cos_kernel(y);
  }
}

// cos(x) (msun s_cosf method).
inline float cosf(float x) {
  const double p1 = 1 * 1.57079632679489661923, p2 = 2 * 1.57079632679489661923,
               p3 = 3 * 1.57079632679489661923, p4 = 4 * 1.57079632679489661923;
  const uint32_t hx = fbits(x), ix = hx & 0x7fffffffu;
  const bool neg = hx >> 31;
  if (ix <= 0x3f490fdau) {
    if (ix < 0x39800000u) return 1.0f;
    return cos_kernel(x);
  }
  if (ix <= 0x407b53d1u) {
    if (ix > 0x4016cbe3u) return -cos_kernel(neg ? x + p2 : x - p2);
    return neg ? sin_kernel(x + p1) : sin_kernel(p1 - x);
  }
  if (ix <= 0x40e231d5u) {
    if (ix > 0x40afeddfu) return cos_kernel(neg ? x + p4 : x - p4);
    return neg ? sin_kernel(-x - p3) : sin_kernel(x - p3);
  }
  if (ix >= 0x7f800000u) return x - x;
  double y;
  const int n = rem_pio2f(x, &y);
  switch (n & 3) {
    case 0: return cos_kernel(y);
    case 1: return sin_kernel(-y);
    case 2: return -cos_kernel(y);
    default: return sin_kernel(y);
  }
}

// pow(x, y) (msun e_powf method): log2|x| as t1 + t2 from s = (x-b)/(x+b) and
// a degree-6 polynomial in s^2 (b = 1 or 1.5), with 12-bit head/tail splits;
// y * log2|x| split the same way; 2^z by k = round(z), a degree-5 polynomial
// for 2^r, and an exponent add (scalbnf when the result is subnormal).
inline float powf(float x, float y) {
  const float bp[2] = {1.0f, 1.5f};
  const float dp_h[2] = {0.0f, ffrom(0x3f15c000u)};  // 5.84960938e-01
  const float dp_l[2] = {0.0f, ffrom(0x35d1cfdcu)};  // 1.56322085e-06
  const float two24 = 16777216.0f, huge = 1.0e30f, tiny = 1.0e-30f;
  const float L1 = ffrom(0x3f19999au), L2 = ffrom(0x3edb6db7u), L3 = ffrom(0x3eaaaaabu),
              L4 = ffrom(0x3e8ba305u), L5 = ffrom(0x3e6c3255u), L6 = ffrom(0x3e53f142u);
  const float P1 = ffrom(0x3e2aaaabu), P2 = ffrom(0xbb360b61u), P3 = ffrom(0x388ab355u),
              P4 = ffrom(0xb5ddea0eu), P5 = ffrom(0x3331bb4cu);
  const float lg2 = ffrom(0x3f317218u), lg2_h = ffrom(0x3f317200u), lg2_l = ffrom(0x35bfbe8cu);
  const float ovt = 4.2995665694e-08f;
  const float cp = ffrom(0x3f76384fu), cp_h = ffrom(0x3f764000u), cp_l = ffrom(0xb8f623c6u);
  const float ivln2 = ffrom(0x3fb8aa3bu), ivln2_h = ffrom(0x3fb8aa00u),
              ivln2_l = ffrom(0x36eca570u);

  const int32_t hx = (int32_t)fbits(x), hy = (int32_t)fbits(y);
  int32_t ix = hx & 0x7fffffff;
  const int32_t iy = hy & 0x7fffffff;
  if (iy == 0) return 1.0f;
  if (hx == 0x3f800000) return 1.0f;
  if (ix > 0x7f800000 || iy > 0x7f800000) return x + y;

  int yisint = 0;  // 0: not an integer, 1: odd, 2: even (only when x < 0)
  if (hx < 0) {
    if (iy >= 0x4b800000) {
      yisint = 2;
    } else if (iy >= 0x3f800000) {
      const int k = (iy >> 23) - 0x7f;
      const int32_t j = iy >> (23 - k);
      if ((j << (23 - k)) == iy) yisint = 2 - (j & 1);
    }
  }
  if (iy == 0x7f800000) {  // y = +-inf
    if (ix == 0x3f800000) return 1.0f;
    if (ix > 0x3f800000) return hy >= 0 ? y : 0.0f;
    return hy < 0 ? -y : 0.0f;
  }
  if (iy == 0x3f800000) return hy < 0 ? 1.0f / x : x;
  if (hy == 0x40000000) return x * x;
  if (hy == 0x3f000000 && hx >= 0) return std::sqrt(x);

  float ax = std::fabs(x);
  if (ix == 0x7f800000 || ix == 0 || ix == 0x3f800000) {  // x = +-0, +-inf, +-1
    float z = ax;
    if (hy < 0) z = 1.0f / z;
    if (hx < 0) {
      if (((ix - 0x3f800000) | yisint) == 0)
        z = (z - z) / (z - z);
      else if (yisint == 1)
        z = -z;
    }
    return z;
  }
  float sn = 1.0f;
  if (hx < 0) {
    if (yisint == 0) return (x - x) / (x - x);
    if (yisint == 1) sn = -1.0f;
  }

  float t1, t2;
  if (iy > 0x4d000000) {  // |y| > 2^27
    if (ix < 0x3f7ffff8) return hy < 0 ? sn * huge * huge : sn * tiny * tiny;
    if (ix > 0x3f800007) return hy > 0 ? sn * huge * huge : sn * tiny * tiny;
    const float t = ax - 1.0f;
    const float w = (t * t) * (0.5f - t * (ffrom(0x3eaaaaabu) - t * 0.25f));
    const float u = ivln2_h * t;
    const float v = t * ivln2_l - w * ivln2;
    t1 = ffrom(fbits(u + v) & 0xfffff000u);
    t2 = v - (t1 - u);
  } else {
    int n = 0;
    if (ix < 0x00800000) {  // subnormal x
      ax *= two24;
      n -= 24;
      ix = (int32_t)fbits(ax);
    }
    n += ((ix) >> 23) - 0x7f;
    const int32_t j = ix & 0x007fffff;
    int k;
    ix = j | 0x3f800000;
    if (j <= 0x1cc471) {
      k = 0;
    } else if (j < 0x5db3d7) {
      k = 1;
    } else {
      k = 0;
      n += 1;
      ix -= 0x00800000;
    }
    ax = ffrom((uint32_t)ix);
    // s = s_h + s_l = (ax - bp) / (ax + bp)
    const float u = ax - bp[k];
    const float v = 1.0f / (ax + bp[k]);
    const float s = u * v;
    const float s_h = ffrom(fbits(s) & 0xfffff000u);
    const float t_h0 =
        ffrom((uint32_t)(((((uint32_t)ix >> 1) & 0xfffff000u) | 0x20000000u) + 0x00400000u +
                         ((uint32_t)k << 21)));
    const float t_l0 = ax - (t_h0 - bp[k]);
    const float s_l = v * ((u - s_h * t_h0) - s_h * t_l0);
    // log(ax)
    float s2 = s * s;
    float r = s2 * s2 * (L1 + s2 * (L2 + s2 * (L3 + s2 * (L4 + s2 * (L5 + s2 * L6)))));
    r += s_l * (s_h + s);
    s2 = s_h * s_h;
    const float t_h = ffrom(fbits(3.0f + s2 + r) & 0xfffff000u);
    const float t_l = r - ((t_h - 3.0f) - s2);
    const float uu = s_h * t_h;
    const float vv = s_l * t_h + t_l * s;
    const float p_h = ffrom(fbits(uu + vv) & 0xfffff000u);
    const float p_l = vv - (p_h - uu);
    const float z_h = cp_h * p_h;
    const float z_l = cp_l * p_h + p_l * cp + dp_l[k];
    const float t = (float)n;
    t1 = ffrom(fbits(((z_h + z_l) + dp_h[k]) + t) & 0xfffff000u);
    t2 = z_l - (((t1 - t) - dp_h[k]) - z_h);
  }

  // (y1 + y2) * (t1 + t2)
  const float y1 = ffrom(fbits(y) & 0xfffff000u);
  float p_l = (y - y1) * t1 + y * t2;
  float p_h = y1 * t1;
  float z = p_l + p_h;
  int32_t j = (int32_t)fbits(z);
  if (j > 0x43000000) return sn * huge * huge;
  if (j == 0x43000000) {
    if (p_l + ovt > z - p_h) return sn * huge * huge;
  } else if ((j & 0x7fffffff) > 0x43160000) {
    return sn * tiny * tiny;
  } else if ((uint32_t)j == 0xc3160000u) {
    if (p_l <= z - p_h) return sn * tiny * tiny;
  }
  // 2^(p_h + p_l)
  const int32_t i = j & 0x7fffffff;
  int k = (i >> 23) - 0x7f;
  int n = 0;
  if (i > 0x3f000000) {  // |z| > 0.5: n = nearest integer
    n = j + (0x00800000 >> (k + 1));
    k = ((n & 0x7fffffff) >> 23) - 0x7f;
    const float t = ffrom((uint32_t)(n & ~(0x007fffff >> k)));
    n = ((n & 0x007fffff) | 0x00800000) >> (23 - k);
    if (j < 0) n = -n;
    p_h -= t;
  }
  float t = ffrom(fbits(p_l + p_h) & 0xffff8000u);
  const float u = t * lg2_h;
  const float v = (p_l - (t - p_h)) * lg2 + t * lg2_l;
  z = u + v;
  const float w = v - (z - u);
  t = z * z;
  const float tt1 = z - t * (P1 + t * (P2 + t * (P3 + t * (P4 + t * P5))));
  const float r = (z * tt1) / (tt1 - 2.0f) - (w + z * w);
  z = 1.0f - (r - z);
  j = (int32_t)fbits(z);
  j += (int32_t)((uint32_t)n << 23);
  if ((j >> 23) <= 0)
    z = scalbnf(z, n);
  else
    z = ffrom((uint32_t)j);
  return sn * z;
}

}  // namespace libm
}  // namespace vtq
