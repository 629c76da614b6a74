// exp_f32.h -- exp of an f32 argument, rounded to f32, with the same bits on
// the host and on the GPU.
//
// The router needs exp(v) for the softmax over all experts
// (gpt_oss.rs:174, candle's softmax_last_dim) and for the sigmoid router
// (lfm2moe_q.rs:242); the reference evaluates both with the C library's expf.
// Expert selection compares the resulting probabilities, and two experts whose
// probabilities round to the same f32 are ordered by index, so the last bit of
// every exp matters.  This function is written to be the correctly rounded
// exp(x): it evaluates exp in double precision and rounds once to f32.
//
// Method (Cody and Waite's argument reduction, then the Taylor series):
//   n = rint(x / ln 2), r = x - n ln 2 with ln 2 split into the double nearest
//   ln 2 and its remainder, both subtractions as fused multiply-adds, so
//   |r| <= ln 2 / 2 with an error below 2^-54;
//   exp(r) = sum_{k=0..13} r^k / k!  by Horner's rule with fused multiply-adds
//   (truncation below 2^-56 relative for |r| <= ln 2 / 2);
//   exp(x) = exp(r) * 2^n, exact in double for the arguments that reach it;
//   one rounding of the double to f32 (subnormal results included).
// The double carries an error of about 2^-51 relative, so the f32 result is
// the correctly rounded exp(x) except when exp(x) lies within that distance of
// a rounding boundary between two f32 values (about one argument in 10^8).
// Every step is an IEEE-754 operation with one rounding (fma, rint, multiply,
// conversion), so host and device results agree bit for bit.
//
// Plain C++ when not compiled by nvcc (the CPU tests build it with g++).
#pragma once

#include <math.h>
#include <stdint.h>
#include <string.h>

#ifdef __CUDACC__
#define GB_HD __host__ __device__ __forceinline__
#else
#define GB_HD inline
#endif

namespace gb {

GB_HD double pow2_double(int n) {  // 2^n for -1022 <= n <= 1023
  const uint64_t bits = (uint64_t)(n + 1023) << 52;
  double d;
#ifdef __CUDA_ARCH__
  d = __longlong_as_double((long long)bits);
#else
  memcpy(&d, &bits, sizeof d);
#endif
  return d;
}

GB_HD float exp_f32(float x) {
  if (!(x == x)) return x + x;      // NaN
  if (x > 89.0f) return INFINITY;   // exp(89) > FLT_MAX
  if (x < -104.0f) return 0.0f;     // exp(-104) < 2^-150: rounds to +0
  const double xd = (double)x;
  // constants as hexadecimal literals so that every compiler reads the same
  // doubles: 1/ln 2, ln 2 rounded to double, ln 2 minus that double, 1/k!
  const double n = rint(xd * 0x1.71547652b82fep+0);  // nearest integer to x / ln 2
  double r = fma(-n, 0x1.62e42fefa39efp-1, xd);
  r = fma(-n, 0x1.abc9e3b39803fp-56, r);
  double p = 0x1.6124613a86d09p-33;  // 1/13!
  p = fma(p, r, 0x1.1eed8eff8d898p-29);  // 1/12!
  p = fma(p, r, 0x1.ae64567f544e4p-26);  // 1/11!
  p = fma(p, r, 0x1.27e4fb7789f5cp-22);  // 1/10!
  p = fma(p, r, 0x1.71de3a556c734p-19);  // 1/9!
  p = fma(p, r, 0x1.a01a01a01a01ap-16);  // 1/8!
  p = fma(p, r, 0x1.a01a01a01a01ap-13);  // 1/7!
  p = fma(p, r, 0x1.6c16c16c16c17p-10);  // 1/6!
  p = fma(p, r, 0x1.1111111111111p-7);   // 1/5!
  p = fma(p, r, 0x1.5555555555555p-5);   // 1/4!
  p = fma(p, r, 0x1.5555555555555p-3);   // 1/3!
  p = fma(p, r, 0.5);
  p = fma(p, r, 1.0);
  p = fma(p, r, 1.0);
  return (float)(p * pow2_double((int)n));
}

}  // namespace gb
