// pieces.cuh -- activation rows as four E4M3 pieces (the B operand of the
// block-scaled expert GEMM).
//
// x' = x * 2^-s with max |x'| in [128, 256) is written as q0 + q1/16 +
// q2/256 + q3/4096, each piece the E4M3 rounding of 16^p times the remaining
// part (representation error below 2^-19 of the row max).
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "common.cuh"
#include "umma.cuh"

namespace gb {

constexpr int kActPieces = 4;

// E4M3 of one f32 (round to nearest even, saturating) and back.
__device__ __forceinline__ uint32_t e4m3_of(float v) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(0.0f), "f"(v));
  return r & 0xffu;
}

__device__ __forceinline__ uint32_t e4m3x2_of(float hi, float lo) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ float2 e4m3x2_value(uint32_t v) {
  uint32_t h;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"((uint16_t)v));
  const __half2 hv = *reinterpret_cast<const __half2*>(&h);
  return __half22float2(hv);  // .x = low byte, .y = high byte
}

__device__ __forceinline__ float e4m3_value(uint32_t v) { return e4m3x2_value(v).x; }

// One activation row -> exponent s and the four pieces of x * 2^-s, written
// [4][K] at each of the `ndst` destinations (a token routed to several
// experts has one grouped position per expert).  Every thread of the CTA
// (a multiple of 32, at most 1024) calls it; it may be called repeatedly.
__device__ __forceinline__ void row_pieces(const float* __restrict__ xrow, int K,
                                           uint8_t* __restrict__ q,
                                           float* __restrict__ xscale, const int* dst_pos,
                                           int ndst) {
  const float4* src = reinterpret_cast<const float4*>(xrow);
  const int n4 = K / 4;
  __shared__ float red[32];
  float mx = 0.0f;
  for (int i = threadIdx.x; i < n4; i += blockDim.x) {
    const float4 v = src[i];
    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFullMask, mx, s));
  __syncthreads();  // a previous call's readers of red are done
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = red[0];
  for (int w = 1; w < (int)(blockDim.x >> 5); ++w) mx = fmaxf(mx, red[w]);
  // max |x'| in [128, 256); exponents kept where 2^-s stays a normal f32
  int s = mx > 0.0f ? ilogbf(mx) - 7 : 0;
  s = max(-120, min(120, s));
  const float inv = pow2f(-s);
  if ((int)threadIdx.x < ndst) xscale[dst_pos[threadIdx.x]] = (float)s;
  for (int i = threadIdx.x; i < n4; i += blockDim.x) {
    const float4 v = src[i];
    float r[4] = {__fmul_rn(v.x, inv), __fmul_rn(v.y, inv), __fmul_rn(v.z, inv),
                  __fmul_rn(v.w, inv)};
    uint32_t w[kActPieces];
#pragma unroll
    for (int p = 0; p < kActPieces; ++p) {
      const uint32_t lo = e4m3x2_of(r[1], r[0]), hi = e4m3x2_of(r[3], r[2]);
      w[p] = lo | (hi << 16);
      const float2 a = e4m3x2_value(lo), b = e4m3x2_value(hi);
      r[0] = __fmul_rn(__fsub_rn(r[0], a.x), 16.0f);
      r[1] = __fmul_rn(__fsub_rn(r[1], a.y), 16.0f);
      r[2] = __fmul_rn(__fsub_rn(r[2], b.x), 16.0f);
      r[3] = __fmul_rn(__fsub_rn(r[3], b.y), 16.0f);
    }
    for (int d = 0; d < ndst; ++d) {
      uint32_t* dst = reinterpret_cast<uint32_t*>(q + (int64_t)dst_pos[d] * kActPieces * K);
#pragma unroll
      for (int p = 0; p < kActPieces; ++p) dst[p * n4 + i] = w[p];
    }
  }
}

}  // namespace gb
