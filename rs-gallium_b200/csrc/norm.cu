// norm.cu -- the RMS norms around Gemma-4's routed experts
// (QGemmaMoe::forward, crates/gallium-models/src/gemma4_q.rs:262-328).
//
// Router input:  rms(x) * hidden^-0.5 * router_input_scale   (gemma4_q.rs:267-270,
//                rms_norm_no_scale at :27-33)
// Expert input:  rms(x) * expert_input_norm                  (pre_ffw_norm_2, :274)
// Output:        rms(out) * output_norm, in place            (post_ffw_norm_2, :327)
// with rms(v) = v / sqrt(mean(v^2) + eps) (candle_nn::ops::rms_norm).  One CTA
// per token; the sum of squares is reduced in a fixed order (per-thread
// strided partial sums, then a butterfly per warp, then the warps in order).
#include <math.h>

#include "common.cuh"
#include "moe_internal.h"
#include "ptx.cuh"

namespace gb {
namespace {

constexpr int kNormThreads = 256;

__device__ __forceinline__ float inv_rms_row(const float* __restrict__ v, int H, float eps) {
  __shared__ float warp_ss[kNormThreads / 32];
  float ss = 0.0f;
  for (int k = threadIdx.x; k < H; k += blockDim.x) ss = __fmaf_rn(v[k], v[k], ss);
  ss = warp_sum_butterfly(ss);
  if ((threadIdx.x & 31) == 0) warp_ss[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) tot = __fadd_rn(tot, warp_ss[w]);
  __syncthreads();  // warp_ss may be reused by the caller's next row
  return __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)H), eps));
}

__global__ void __launch_bounds__(kNormThreads)
    input_norms_kernel(const float* __restrict__ x, int H, float eps,
                       const float* __restrict__ rscale, const float* __restrict__ enorm,
                       float* __restrict__ xr, float* __restrict__ xe) {
  pdl_trigger();
  pdl_wait();
  const int64_t t = blockIdx.x;
  const float* row = x + t * H;
  const float m = inv_rms_row(row, H, eps);
  const float inv_sqrt_h = (float)(1.0 / sqrt((double)H));  // hidden^-0.5 as candle's affine rounds it
  for (int k = threadIdx.x; k < H; k += blockDim.x) {
    const float n = __fdiv_rn(row[k], m);
    xr[t * H + k] = __fmul_rn(__fmul_rn(n, inv_sqrt_h), rscale[k]);
    xe[t * H + k] = __fmul_rn(n, enorm[k]);
  }
}

__global__ void __launch_bounds__(kNormThreads)
    output_norm_kernel(float* __restrict__ out, int H, float eps, const float* __restrict__ w) {
  pdl_trigger();
  pdl_wait();
  float* row = out + (int64_t)blockIdx.x * H;
  const float m = inv_rms_row(row, H, eps);
  for (int k = threadIdx.x; k < H; k += blockDim.x) row[k] = __fmul_rn(__fdiv_rn(row[k], m), w[k]);
}

}  // namespace

cudaError_t launch_input_norms(const Moe& m, const float* x, int64_t T, float* x_route,
                               float* x_expert, cudaStream_t st) {
  if (T <= 0) return cudaSuccess;
  return launch_pdl(input_norms_kernel, dim3((unsigned)T), dim3(kNormThreads), 0, st, x,
                    m.desc.hidden, m.desc.rms_eps, (const float*)m.w.router_in_scale,
                    (const float*)m.w.expert_in_norm, x_route, x_expert);
}

cudaError_t launch_output_norm(const Moe& m, float* out, int64_t T, cudaStream_t st) {
  if (T <= 0 || !m.w.out_norm) return cudaSuccess;
  return launch_pdl(output_norm_kernel, dim3((unsigned)T), dim3(kNormThreads), 0, st, out,
                    m.desc.hidden, m.desc.rms_eps, (const float*)m.w.out_norm);
}

}  // namespace gb
