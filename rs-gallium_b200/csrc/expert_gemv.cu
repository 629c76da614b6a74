// expert_gemv.cu -- grouped MXFP4 expert products on CUDA cores, combine,
// and the weight-format helpers.
//
// Reference math: gpt_oss.rs:189-223 (gate_up + bias, interleaved split,
// clamped SwiGLU, down + bias, weighted sum), gpt_oss_q.rs:194-266,
// lfm2moe_q.rs:279-311.
//
// expert_rows_kernel<MODE, TC>: one CTA per (active expert, tile of rows).
// A warp owns two weight rows (the gate/up pair 2i, 2i+1 in GATE_UP mode;
// two consecutive output rows in DOWN mode).  Lane l holds blocks l, l+32,
// l+64, ... of both rows in registers (16-byte streaming loads, read from HBM
// once per forward), and the expert's tokens stream through shared memory in
// chunks of TC rows.  Each 32-element block is decoded with the hardware
// E2M1 -> f16x2 conversion, dotted with the activations in f32 FMAs, and the
// block sum is scaled by its E8M0 scale into the row accumulator; the 32 lane
// sums are folded with a butterfly.
#include <algorithm>

#include "common.cuh"
#include "moe_internal.h"
#include "ptx.cuh"

namespace gb {
namespace {

constexpr int kWarps = 8;

enum Mode { GATE_UP = 0, DOWN = 1 };

template <int MODE, int TC, int NBQ>
__global__ void __launch_bounds__(kWarps * 32)
    expert_rows_kernel(const float* __restrict__ in, int K_in, int n_rows_total, int top_k,
                       const uint8_t* __restrict__ blocks, const uint8_t* __restrict__ scales,
                       int sp, const float* __restrict__ bias, float zero_scale,
                       const int32_t* __restrict__ counts, const int32_t* __restrict__ offsets,
                       const int32_t* __restrict__ active, const int32_t* __restrict__ meta,
                       const int32_t* __restrict__ perm, int e_begin, int act_kind, float limit,
                       float clamp, const int32_t* __restrict__ out_rows, float* __restrict__ out,
                       int out_stride) {
  extern __shared__ float xs[];  // [TC][33 * NB], element k at k + k/32
  const int slot = blockIdx.y;
  if (slot >= meta[0]) return;
  const int e = active[slot];
  const int le = e - e_begin;
  const int n = counts[e];
  const int p0 = offsets[e];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NB = K_in >> 5;
  const int PH = 33 * NB;

  // Rows of this warp.
  const int pair = blockIdx.x * kWarps + warp;
  const int row0 = 2 * pair;  // GATE_UP: gate row 2i / up row 2i+1; DOWN: rows 2p, 2p+1
  const bool valid = row0 < n_rows_total;
  const bool valid1 = row0 + 1 < n_rows_total;

  uint4 wq[2][NBQ];
  float sc[2][NBQ];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int64_t row = (int64_t)le * n_rows_total + row0 + r;
    const bool rv = r == 0 ? valid : valid1;
#pragma unroll
    for (int q = 0; q < NBQ; ++q) {
      const int b = lane + 32 * q;
      if (rv && b < NB) {
        wq[r][q] = ld_stream_u4(blocks + (row * NB + b) * 16);
        sc[r][q] = e8m0_scale(scales[row * sp + b], zero_scale);
      } else {
        wq[r][q] = make_uint4(0, 0, 0, 0);
        sc[r][q] = 0.0f;
      }
    }
  }

  for (int c0 = 0; c0 < n; c0 += TC) {
    const int nc = min(TC, n - c0);
    __syncthreads();
    // Stage the chunk's activation rows (padded layout, conflict-free reads).
    for (int j = 0; j < nc; ++j) {
      const float* src;
      if (MODE == GATE_UP) {
        const int tok = perm[p0 + c0 + j] / top_k;
        src = in + (int64_t)tok * K_in;
      } else {
        src = in + (int64_t)(p0 + c0 + j) * K_in;
      }
      for (int k4 = threadIdx.x; k4 < (K_in >> 2); k4 += blockDim.x) {
        const float4 v = reinterpret_cast<const float4*>(src)[k4];
        const int k = k4 << 2;
        float* d = xs + j * PH + k + (k >> 5);
        d[0] = v.x;
        d[1] = v.y;
        d[2] = v.z;
        d[3] = v.w;
      }
    }
    __syncthreads();
    if (!valid) continue;

    float acc[2][TC];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int j = 0; j < TC; ++j) acc[r][j] = 0.0f;

#pragma unroll
    for (int r = 0; r < 2; ++r) {
#pragma unroll
      for (int q = 0; q < NBQ; ++q) {
        const int b = lane + 32 * q;
        if (b >= NB) continue;
        float v[32];
        decode_block_f32(wq[r][q], v);
        const float* xb = xs + b * 33;
#pragma unroll
        for (int j = 0; j < TC; ++j) {
          if (j < nc) {
            float part = 0.0f;
#pragma unroll
            for (int el = 0; el < 32; ++el) part = __fmaf_rn(xb[j * PH + el], v[el], part);
            acc[r][j] = __fmaf_rn(part, sc[r][q], acc[r][j]);
          }
        }
      }
    }
#pragma unroll
    for (int j = 0; j < TC; ++j) {
      if (j >= nc) break;
      const float s0 = warp_sum_butterfly(acc[0][j]);
      const float s1 = warp_sum_butterfly(acc[1][j]);
      if (lane == 0) {
        const int64_t pos = p0 + c0 + j;
        if (MODE == GATE_UP) {
          float g = s0, u = s1;
          if (bias) {
            g = __fadd_rn(g, bias[(int64_t)le * n_rows_total + row0]);
            u = __fadd_rn(u, bias[(int64_t)le * n_rows_total + row0 + 1]);
          }
          out[pos * out_stride + pair] = act_apply(act_kind, g, u, limit, clamp);
        } else {
          float y0 = s0, y1 = s1;
          if (bias) {
            y0 = __fadd_rn(y0, bias[(int64_t)le * n_rows_total + row0]);
            if (valid1) y1 = __fadd_rn(y1, bias[(int64_t)le * n_rows_total + row0 + 1]);
          }
          const int64_t orow = out_rows ? out_rows[pos] : pos;
          out[orow * out_stride + row0] = y0;
          if (valid1) out[orow * out_stride + row0 + 1] = y1;
        }
      }
    }
  }
}

template <int MODE, int TC>
cudaError_t launch_rows(const Moe& m, const Groups& g, const float* in, int K_in, int n_rows_total,
                        const uint8_t* blocks, const uint8_t* scales, int sp, const float* bias,
                        float* out, int out_stride, cudaStream_t st) {
  const gb_moe_desc& d = m.desc;
  const int NB = K_in / 32;
  const int nbq = (NB + 31) / 32;
  if (g.max_active <= 0) return cudaSuccess;
  const int pairs = (n_rows_total + 1) / 2;
  dim3 grid((unsigned)((pairs + kWarps - 1) / kWarps), (unsigned)g.max_active);
  const size_t smem = (size_t)TC * 33 * NB * sizeof(float);
  cudaError_t err = cudaSuccess;
#define GB_LAUNCH_NBQ(Q)                                                                         \
  {                                                                                              \
    auto kern = expert_rows_kernel<MODE, TC, Q>;                                                 \
    err = set_smem_limit(kern, smem);                                                            \
    if (err != cudaSuccess) return err;                                                          \
    kern<<<grid, kWarps * 32, smem, st>>>(in, K_in, n_rows_total, g.perm_div, blocks, scales, sp, \
                                          bias, m.w.zero_scale, g.counts, g.offsets, g.active,   \
                                          g.meta, g.perm, m.e_begin, d.act_kind, d.swiglu_limit, \
                                          d.act_clamp, MODE == DOWN ? g.out_rows : nullptr, out,  \
                                          out_stride);                                           \
  }
  switch (nbq) {
    case 1: GB_LAUNCH_NBQ(1) break;
    case 2: GB_LAUNCH_NBQ(2) break;
    case 3: GB_LAUNCH_NBQ(3) break;
    case 4: GB_LAUNCH_NBQ(4) break;
    default: return cudaErrorInvalidValue;
  }
#undef GB_LAUNCH_NBQ
  return cudaGetLastError();
}

// out[t, :] = sum over ranks of w * y, rows scaled then added to a running sum
// from zero (gpt_oss.rs:223).  expert_order: add in ascending expert order
// (gpt_oss_q.rs:252-266, lfm2moe_q.rs:303-311) instead of rank order.
__global__ void combine_kernel(const float* __restrict__ y, const int32_t* __restrict__ inv,
                               const float* __restrict__ wts, const int32_t* __restrict__ idx,
                               int H, int K, int expert_order, const float* __restrict__ escale,
                               const float* __restrict__ add, float* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  const int o4 = blockIdx.y * blockDim.x + threadIdx.x;
  if (o4 * 4 >= H) return;
  // the token's k entries first (K <= 8), then all its y rows at once: one
  // dependent round trip instead of one per rank
  int e[8], order[8];
  int64_t p[8];
  float wv[8];
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    if (r < K) {
      e[r] = idx[(int64_t)t * K + r];
      p[r] = inv ? inv[(int64_t)t * K + r] : (int64_t)t * K + r;
      wv[r] = wts[(int64_t)t * K + r];
      order[r] = r;
    }
  }
  if (expert_order) {
    for (int a = 1; a < K; ++a) {
      const int cur = order[a];
      int b = a - 1;
      while (b >= 0 && e[order[b]] > e[cur]) {
        order[b + 1] = order[b];
        --b;
      }
      order[b + 1] = cur;
    }
  }
  float4 v[8];
#pragma unroll
  for (int r = 0; r < 8; ++r)
    if (r < K) v[r] = reinterpret_cast<const float4*>(y + p[r] * H)[o4];
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int q = 0; q < K; ++q) {
    const int r = order[q];
    float4 vr = v[0];
    float w = wv[0];
    int er = e[0];
#pragma unroll
    for (int i = 1; i < 8; ++i)
      if (i == r) {
        vr = v[i];
        w = wv[i];
        er = e[i];
      }
    if (escale) {  // the expert's output scale, before the routing weight (gemma4_q.rs:308-314)
      const float s = escale[er];
      vr.x = __fmul_rn(vr.x, s);
      vr.y = __fmul_rn(vr.y, s);
      vr.z = __fmul_rn(vr.z, s);
      vr.w = __fmul_rn(vr.w, s);
    }
    acc.x = __fadd_rn(acc.x, __fmul_rn(vr.x, w));
    acc.y = __fadd_rn(acc.y, __fmul_rn(vr.y, w));
    acc.z = __fadd_rn(acc.z, __fmul_rn(vr.z, w));
    acc.w = __fadd_rn(acc.w, __fmul_rn(vr.w, w));
  }
  if (add) {  // the shared expert's row, added after the routed sum (ffn.rs:160-163)
    const float4 a = reinterpret_cast<const float4*>(add + (int64_t)t * H)[o4];
    acc.x = __fadd_rn(acc.x, a.x);
    acc.y = __fadd_rn(acc.y, a.y);
    acc.z = __fadd_rn(acc.z, a.z);
    acc.w = __fadd_rn(acc.w, a.w);
  }
  reinterpret_cast<float4*>(out + (int64_t)t * H)[o4] = acc;
}

// One thread per (row, block): value = code * scale, as gpt_oss.rs:157-159.
__global__ void dequant_kernel(const uint8_t* __restrict__ blocks, const uint8_t* __restrict__ scales,
                               int sp, float zero_scale, int64_t row_base, int row_step, int nrows,
                               int K, float* __restrict__ out) {
  const int NB = K >> 5;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)nrows * NB) return;
  const int r = (int)(i / NB), b = (int)(i % NB);
  const int64_t row = row_base + (int64_t)r * row_step;
  const uint4 q = *reinterpret_cast<const uint4*>(blocks + (row * NB + b) * 16);
  const float s = e8m0_scale(scales[row * sp + b], zero_scale);
  float v[32];
  decode_block_f32(q, v);
  float* dst = out + (int64_t)r * K + b * 32;
#pragma unroll
  for (int el = 0; el < 32; ++el) dst[el] = __fmul_rn(v[el], s);
}

// GGUF 17-byte block [e8m0, 16 bytes; low nibble of byte j = element j, high
// nibble = element j+16] -> split block (byte j = elements 2j, 2j+1) + scale.
__global__ void gguf_to_split_kernel(const uint8_t* __restrict__ raw, int64_t rows, int NB,
                                     uint8_t* __restrict__ blocks, int64_t row_stride_blocks,
                                     uint8_t* __restrict__ scales, int64_t row_stride_scales) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * NB) return;
  const int64_t r = i / NB;
  const int b = (int)(i % NB);
  const uint8_t* src = raw + i * 17;
  // The GGUF table has +0 for code 8 (quantized.rs:370, i8 zero), where E2M1
  // reads it as -0: store code 0 instead so the decode is bit-identical.
  uint8_t el[32];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const uint8_t lo = src[1 + j] & 0xF, hi = src[1 + j] >> 4;
    el[j] = lo == 8 ? 0 : lo;
    el[j + 16] = hi == 8 ? 0 : hi;
  }
  uint8_t* dst = blocks + (r * row_stride_blocks + b) * 16;
#pragma unroll
  for (int j = 0; j < 16; ++j) dst[j] = (uint8_t)(el[2 * j] | (el[2 * j + 1] << 4));
  scales[r * row_stride_scales + b] = src[0];
}

}  // namespace

cudaError_t launch_gate_up(const Moe& m, const Groups& g, const float* x, ExpertBufs& eb,
                           cudaStream_t st) {
  const gb_moe_desc& d = m.desc;
  return launch_rows<GATE_UP, 8>(m, g, x, d.hidden, 2 * d.inter, m.w.gu_blocks, m.w.gu_scales,
                                 m.w.sp_h, m.w.gu_bias, eb.h, d.inter, st);
}

cudaError_t launch_down(const Moe& m, const Groups& g, ExpertBufs& eb, cudaStream_t st) {
  const gb_moe_desc& d = m.desc;
  return launch_rows<DOWN, 8>(m, g, eb.h, d.inter, d.hidden, m.w.dn_blocks, m.w.dn_scales,
                              m.w.sp_i, m.w.dn_bias, eb.y, d.hidden, st);
}

cudaError_t launch_combine(const Moe& m, int64_t T, const Workspace& ws, const float* y, float* out,
                           cudaStream_t st, bool slots) {
  const int H = m.desc.hidden;
  const int threads = 256;
  dim3 grid((unsigned)T, (unsigned)((H / 4 + threads - 1) / threads));
  // rank order for the safetensors GPT-OSS and generic MoEFFN blocks
  // (gpt_oss.rs:223, ffn.rs:153-156), expert order for the GGUF ones
  const int expert_order =
      m.desc.weight_format == GB_FMT_MXFP4_GGUF || m.desc.weight_format == GB_FMT_Q4_K;
  const float* add = m.desc.shared_inter > 0 ? (const float*)ws.sh_y : nullptr;
  return launch_pdl(combine_kernel, grid, dim3(threads), 0, st, y,
                    slots ? (const int32_t*)nullptr : (const int32_t*)ws.inv, ws.wts, ws.idx, H,
                    m.desc.top_k, expert_order, (const float*)m.w.expert_scale, add, out);
}

cudaError_t launch_dequant_expert(const Moe& m, int which, int local_expert, float* out,
                                  cudaStream_t st) {
  const int H = m.desc.hidden, I = m.desc.inter;
  int64_t row_base;
  int row_step, nrows, K, sp;
  const uint8_t *blocks, *scales;
  if (which == 2) {
    blocks = m.w.dn_blocks;
    scales = m.w.dn_scales;
    sp = m.w.sp_i;
    row_base = (int64_t)local_expert * H;
    row_step = 1;
    nrows = H;
    K = I;
  } else {
    blocks = m.w.gu_blocks;
    scales = m.w.gu_scales;
    sp = m.w.sp_h;
    row_base = (int64_t)local_expert * 2 * I + which;
    row_step = 2;
    nrows = I;
    K = H;
  }
  const int64_t n = (int64_t)nrows * (K / 32);
  dequant_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(blocks, scales, sp, m.w.zero_scale,
                                                               row_base, row_step, nrows, K, out);
  return cudaGetLastError();
}

cudaError_t launch_gguf_to_split(const uint8_t* raw_dev, int64_t rows, int k, uint8_t* blocks_dev,
                                 int64_t row_stride_blocks, uint8_t* scales_dev,
                                 int64_t row_stride_scales, cudaStream_t st) {
  const int NB = k / 32;
  const int64_t n = rows * NB;
  gguf_to_split_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(
      raw_dev, rows, NB, blocks_dev, row_stride_blocks, scales_dev, row_stride_scales);
  return cudaGetLastError();
}

}  // namespace gb
