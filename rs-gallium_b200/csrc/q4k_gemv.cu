// q4k_gemv.cu -- grouped GGML Q4_K expert products (LFM2.5 experts).
//
// Reference: lfm2moe_q.rs:279-296 (h = silu(x Wg^T) * (x Wu^T), y = h Wd^T, no
// biases) with candle's Q4_K dequantiser reached through QExperts
// (quantized.rs:139-178).  A 144-byte super-block holds 256 elements: f16 d,
// f16 dmin, 12 bytes of 6-bit sub-block scales and mins, 128 bytes of 4-bit
// quants; sub-block j (32 elements) has value d*sc_j*q - dmin*m_j, and quant
// bytes serve two sub-blocks (low nibbles 2c, high nibbles 2c+1).
//
// Layout on the device: the caller's row-major blocks, with gate and up rows
// interleaved into one fused matrix (row 2i = gate_i, 2i+1 = up_i) like the
// MXFP4 path: q4_gu [E_loc][2I][H/256][144], q4_dn [E_loc][H][I/256][144].
//
// Kernel: one CTA per (active expert, 16 row pairs); a warp owns row pairs,
// lane l takes sub-blocks l, l+32, ... of a row.  For each sub-block the lane
// loads the super-block header (16 bytes) and its 32 quant bytes, and adds
// d1 * sum(x q) - m1 * sum(x) to the row sum (sum(x) per 32-element block is
// computed once per staged token); a butterfly folds the lanes.
#include <algorithm>

#include "common.cuh"
#include "moe_internal.h"

namespace gb {
namespace {

constexpr int kQWarps = 4;
constexpr int kQPairs = 4;
constexpr int kQRowsPerCta = kQWarps * 2 * kQPairs;
constexpr int kQPitch = 36;  // floats per staged 32-element block (+4 pad)
constexpr int kQTok = 4;

enum Mode { GATE_UP = 0, DOWN = 1 };

struct QArgs {
  const float* in;
  int K;
  int rows;
  int top_k;
  const uint8_t* q;      // [E_loc][rows][K/256][144]
  const int32_t* counts;
  const int32_t* offsets;
  const int32_t* active;
  const int32_t* meta;
  const int32_t* perm;
  int e_begin;
  int act_kind;
  float limit;
  const int32_t* out_rows;
  float* out;
  int out_stride;
};

// The 6-bit (scale, min) pair of sub-block j from the 12 packed bytes.
__device__ __forceinline__ void q4k_scale_min(int j, const uint8_t* s, int& sc, int& m) {
  if (j < 4) {
    sc = s[j] & 63;
    m = s[j + 4] & 63;
  } else {
    sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
    m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
}

__device__ __forceinline__ float half_bits_to_f32(uint16_t h) {
  return __half2float(*reinterpret_cast<const __half*>(&h));
}

template <int MODE>
__global__ void __launch_bounds__(kQWarps * 32) q4k_rows_kernel(const QArgs a) {
  extern __shared__ float qsm[];
  const int K = a.K;
  const int NB = K >> 5;        // 32-element sub-blocks per row
  const int nsb = K >> 8;       // super-blocks per row
  const int xstride = NB * kQPitch;
  float* xs = qsm;                      // [kQTok][NB][kQPitch]
  float* xsum = xs + kQTok * xstride;   // [kQTok][NB]

  const int slot = blockIdx.y;
  if (slot >= a.meta[0]) return;
  const int e = a.active[slot];
  const int le = e - a.e_begin;
  const int n = a.counts[e];
  const int p0 = a.offsets[e];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * kQRowsPerCta + warp * 2 * kQPairs;
  const int npairs = max(0, min(kQPairs, (a.rows - row0) >> 1));
  const int64_t erow = (int64_t)le * a.rows;
  const int64_t row_bytes = (int64_t)nsb * 144;

  for (int c0 = 0; c0 < n; c0 += kQTok) {
    const int nc = min(kQTok, n - c0);
    __syncthreads();
    for (int j = 0; j < nc; ++j) {
      const float* src = MODE == GATE_UP
                             ? a.in + (int64_t)(a.perm[p0 + c0 + j] / a.top_k) * K
                             : a.in + (int64_t)(p0 + c0 + j) * K;
      for (int k4 = threadIdx.x; k4 < (K >> 2); k4 += blockDim.x) {
        const int k = k4 << 2;
        *reinterpret_cast<float4*>(xs + j * xstride + (k >> 5) * kQPitch + (k & 31)) =
            reinterpret_cast<const float4*>(src)[k4];
      }
    }
    __syncthreads();
    for (int jb = warp; jb < nc * NB; jb += kQWarps) {
      const int j = jb / NB, b = jb - j * NB;
      float v = xs[j * xstride + b * kQPitch + lane];
      v = warp_sum_butterfly(v);
      if (lane == 0) xsum[j * NB + b] = v;
    }
    __syncthreads();

    for (int p = 0; p < npairs; ++p) {
      float acc[2][kQTok];
#pragma unroll
      for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int t = 0; t < kQTok; ++t) acc[r][t] = 0.0f;
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const uint8_t* rowp = a.q + (erow + row0 + 2 * p + r) * row_bytes;
        for (int sbk = lane; sbk < NB; sbk += 32) {
          const int sb = sbk >> 3, jj = sbk & 7;
          const uint8_t* blk = rowp + sb * 144;
          const uint4 hdr = __ldg(reinterpret_cast<const uint4*>(blk));
          const uint4 qa = __ldg(reinterpret_cast<const uint4*>(blk + 16 + 32 * (jj >> 1)));
          const uint4 qb = __ldg(reinterpret_cast<const uint4*>(blk + 32 + 32 * (jj >> 1)));
          const uint8_t* hb = reinterpret_cast<const uint8_t*>(&hdr);
          const float d = half_bits_to_f32((uint16_t)(hb[0] | (hb[1] << 8)));
          const float dmin = half_bits_to_f32((uint16_t)(hb[2] | (hb[3] << 8)));
          int sc, mn;
          q4k_scale_min(jj, hb + 4, sc, mn);
          const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)mn);
          const int shift = (jj & 1) ? 4 : 0;
          const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
          float qv[32];
#pragma unroll
          for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int bb = 0; bb < 4; ++bb) qv[i * 4 + bb] = (float)((w[i] >> (8 * bb + shift)) & 0xF);
#pragma unroll
          for (int t = 0; t < kQTok; ++t) {
            if (t < nc) {
              const float4* x4 = reinterpret_cast<const float4*>(xs + t * xstride + sbk * kQPitch);
              float f0 = 0.0f, f1 = 0.0f, f2 = 0.0f, f3 = 0.0f;
#pragma unroll
              for (int q4 = 0; q4 < 8; ++q4) {
                const float4 xv = x4[q4];
                f0 = __fmaf_rn(xv.x, qv[4 * q4], f0);
                f1 = __fmaf_rn(xv.y, qv[4 * q4 + 1], f1);
                f2 = __fmaf_rn(xv.z, qv[4 * q4 + 2], f2);
                f3 = __fmaf_rn(xv.w, qv[4 * q4 + 3], f3);
              }
              const float sxq = __fadd_rn(__fadd_rn(f0, f1), __fadd_rn(f2, f3));
              const float part = __fsub_rn(__fmul_rn(d1, sxq), __fmul_rn(m1, xsum[t * NB + sbk]));
              acc[r][t] = __fadd_rn(acc[r][t], part);
            }
          }
        }
      }
      const int row = row0 + 2 * p;
#pragma unroll
      for (int t = 0; t < kQTok; ++t) {
        if (t >= nc) break;
        const float s0 = warp_sum_butterfly(acc[0][t]);
        const float s1 = warp_sum_butterfly(acc[1][t]);
        if (lane == 0) {
          const int64_t pos = p0 + c0 + t;
          if (MODE == GATE_UP) {
            a.out[pos * a.out_stride + (row >> 1)] =
                a.act_kind == GB_ACT_GPTOSS_CLAMP ? act_gptoss(s0, s1, a.limit) : act_silu(s0, s1);
          } else {
            const int64_t orow = a.out_rows ? a.out_rows[pos] : pos;
            a.out[orow * a.out_stride + row] = s0;
            a.out[orow * a.out_stride + row + 1] = s1;
          }
        }
      }
    }
  }
}

template <int MODE>
cudaError_t launch_q(const Groups& g, const QArgs& a, cudaStream_t st) {
  if (g.max_active <= 0) return cudaSuccess;
  dim3 grid((unsigned)((a.rows + kQRowsPerCta - 1) / kQRowsPerCta), (unsigned)g.max_active);
  const int NB = a.K / 32;
  const size_t smem = (size_t)kQTok * NB * kQPitch * sizeof(float) + (size_t)kQTok * NB * sizeof(float);
  auto kern = q4k_rows_kernel<MODE>;
  cudaError_t err = set_smem_limit(kern, smem);
  if (err != cudaSuccess) return err;
  kern<<<grid, kQWarps * 32, smem, st>>>(a);
  return cudaGetLastError();
}

QArgs q_args(const Moe& m, const Groups& g) {
  QArgs a{};
  a.top_k = g.perm_div;
  a.counts = g.counts;
  a.offsets = g.offsets;
  a.active = g.active;
  a.meta = g.meta;
  a.perm = g.perm;
  a.e_begin = m.e_begin;
  a.act_kind = m.desc.act_kind;
  a.limit = m.desc.swiglu_limit;
  return a;
}

// Element values of one matrix, bit-identical to the GGML dequantiser:
// thread per 32-element sub-block, value = d*sc*q - dmin*m with each product
// and the difference rounded separately.
__global__ void q4k_dequant_kernel(const uint8_t* __restrict__ q, int64_t row_base, int row_step,
                                   int nrows, int K, float* __restrict__ out) {
  const int NB = K >> 5, nsb = K >> 8;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)nrows * NB) return;
  const int r = (int)(i / NB), sbk = (int)(i % NB);
  const int64_t row = row_base + (int64_t)r * row_step;
  const uint8_t* blk = q + row * nsb * 144 + (sbk >> 3) * 144;
  const int jj = sbk & 7;
  const float d = half_bits_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
  const float dmin = half_bits_to_f32((uint16_t)(blk[2] | (blk[3] << 8)));
  int sc, mn;
  q4k_scale_min(jj, blk + 4, sc, mn);
  const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)mn);
  const uint8_t* qs = blk + 16 + 32 * (jj >> 1);
  const int shift = (jj & 1) ? 4 : 0;
  float* dst = out + (int64_t)r * K + sbk * 32;
  for (int l = 0; l < 32; ++l) dst[l] = __fsub_rn(__fmul_rn(d1, (float)((qs[l] >> shift) & 0xF)), m1);
}

}  // namespace

cudaError_t launch_q4k_gate_up(const Moe& m, const Groups& g, const float* x, ExpertBufs& eb,
                               cudaStream_t st) {
  QArgs a = q_args(m, g);
  a.in = x;
  a.K = m.desc.hidden;
  a.rows = 2 * m.desc.inter;
  a.q = m.w.q4_gu;
  a.out = eb.h;
  a.out_stride = m.desc.inter;
  return launch_q<GATE_UP>(g, a, st);
}

cudaError_t launch_q4k_down(const Moe& m, const Groups& g, ExpertBufs& eb, cudaStream_t st) {
  QArgs a = q_args(m, g);
  a.in = eb.h;
  a.K = m.desc.inter;
  a.rows = m.desc.hidden;
  a.q = m.w.q4_dn;
  a.out_rows = g.out_rows;
  a.out = eb.y;
  a.out_stride = m.desc.hidden;
  return launch_q<DOWN>(g, a, st);
}

cudaError_t launch_q4k_dequant(const Moe& m, int which, int local_expert, float* out,
                               cudaStream_t st) {
  const int H = m.desc.hidden, I = m.desc.inter;
  const uint8_t* q;
  int64_t row_base;
  int row_step, nrows, K;
  if (which == 2) {
    q = m.w.q4_dn;
    row_base = (int64_t)local_expert * H;
    row_step = 1;
    nrows = H;
    K = I;
  } else {
    q = m.w.q4_gu;
    row_base = (int64_t)local_expert * 2 * I + which;
    row_step = 2;
    nrows = I;
    K = H;
  }
  const int64_t n = (int64_t)nrows * (K / 32);
  q4k_dequant_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(q, row_base, row_step, nrows, K,
                                                                   out);
  return cudaGetLastError();
}

}  // namespace gb
