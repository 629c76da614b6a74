// common.cuh -- device helpers shared by the MoE kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/gallium_b200.h"

namespace gb {

constexpr unsigned kFullMask = 0xffffffffu;

// bf16 bits -> f32 (exact).
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

// E8M0 scale byte -> 2^(s-127) as an f32 with exponent field s and zero
// mantissa; s == 255 gives +inf like 2f32.powi(128).  s == 0 has no such
// encoding (it would be f32 zero): the caller's format decides its value
// (0 for safetensors, 2^-127 for GGUF), passed in as zero_scale.
__device__ __forceinline__ float e8m0_scale(uint32_t s, float zero_scale) {
  return s == 0 ? zero_scale : __uint_as_float(s << 23);
}

// Two E2M1 codes packed in one byte (low nibble = even element) -> f16x2
// (low half = even element), exact.  Uses the sm_100 hardware conversion.
__device__ __forceinline__ uint32_t e2m1x2_to_f16x2(uint32_t byte) {
  uint32_t out;
  asm("{\n\t.reg .b8 lo8, hi8;\n\t"
      "mov.b16 {lo8, hi8}, %1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, lo8;\n\t}"
      : "=r"(out)
      : "h"(static_cast<uint16_t>(byte)));
  return out;
}

// 32 E2M1 codes (one 16-byte MXFP4 block, byte j = elements 2j, 2j+1) ->
// 32 floats of the code values (before the block scale).
__device__ __forceinline__ void decode_block_f32(const uint4& q, float (&v)[32]) {
  const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int wd = 0; wd < 4; ++wd) {
#pragma unroll
    for (int by = 0; by < 4; ++by) {
      const uint32_t h2 = e2m1x2_to_f16x2((words[wd] >> (8 * by)) & 0xffu);
      const __half2 hv = *reinterpret_cast<const __half2*>(&h2);
      const float2 f = __half22float2(hv);
      v[wd * 8 + by * 2] = f.x;
      v[wd * 8 + by * 2 + 1] = f.y;
    }
  }
}

__device__ __forceinline__ float warp_sum_butterfly(float v) {
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) v = v + __shfl_xor_sync(kFullMask, v, s);
  return v;
}

// Read-only streaming 128-bit load (weights are read once per forward).
__device__ __forceinline__ uint4 ld_stream_u4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// GPT-OSS clamped SwiGLU, step for step as gpt_oss.rs:202-212 evaluates it
// through candle ops (clamp = maximum(-1e38) then minimum(limit); sigmoid(1.702 g)
// as (tanh(0.851 g) + 1) * 0.5 through affine ops; up clamped both sides and
// shifted by one).  The _rn intrinsics keep every product and sum separately
// rounded, as the reference's ops are.
__device__ __forceinline__ float act_gptoss(float g, float u, float limit) {
  g = fmaxf(g, -1e38f);
  g = fminf(g, limit);
  float s = __fadd_rn(__fmul_rn(g, 0.851f), 0.0f);
  s = tanhf(s);
  s = __fadd_rn(__fmul_rn(s, 1.0f), 1.0f);
  s = __fadd_rn(__fmul_rn(s, 0.5f), 0.0f);
  const float glu = __fmul_rn(g, s);
  u = fminf(fmaxf(u, -limit), limit);
  const float u1 = __fadd_rn(__fmul_rn(u, 1.0f), 1.0f);
  return __fmul_rn(glu, u1);
}

// silu(g) * u with silu(v) = v / (1 + exp(-v)) (lfm2moe_q.rs:288-290).
__device__ __forceinline__ float act_silu(float g, float u) {
  const float sg = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
  return __fmul_rn(sg, u);
}

// gallium-core's Activation (ffn.rs:16-24) on the gate, clamped to
// [-clamp, clamp] when clamp > 0 (ffn.rs:58-62): SiLU, GELU (erf, candle
// gelu_erf), GELU (tanh, candle gelu; also Gemma-4's GEGLU,
// gemma4_q.rs:305), ReLU.
__device__ __forceinline__ float act_generic(int kind, float g, float clamp) {
  float a;
  switch (kind) {
    case GB_ACT_GELU:
      a = __fmul_rn(__fmul_rn(0.5f, g), __fadd_rn(1.0f, erff(__fmul_rn(g, 0.70710678118654752f))));
      break;
    case GB_ACT_GELU_TANH: {
      const float inner = __fmul_rn(0.79788456080286536f,
                                    __fadd_rn(g, __fmul_rn(0.044715f, __fmul_rn(g, __fmul_rn(g, g)))));
      a = __fmul_rn(__fmul_rn(0.5f, g), __fadd_rn(1.0f, tanhf(inner)));
      break;
    }
    case GB_ACT_RELU:
      a = fmaxf(g, 0.0f);
      break;
    default:
      a = __fdiv_rn(g, __fadd_rn(expf(-g), 1.0f));
  }
  return clamp > 0.0f ? fminf(fmaxf(a, -clamp), clamp) : a;
}

// The expert activation h(gate, up) of every kind (gb_act_kind).
__device__ __forceinline__ float act_apply(int kind, float g, float u, float limit, float clamp) {
  if (kind == GB_ACT_GPTOSS_CLAMP) return act_gptoss(g, u, limit);
  if (kind == GB_ACT_SILU && !(clamp > 0.0f)) return act_silu(g, u);
  return __fmul_rn(act_generic(kind, g, clamp), u);
}

}  // namespace gb
