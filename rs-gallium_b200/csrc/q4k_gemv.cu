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
// Kernel: q4k_rows_kernel below.
#include <algorithm>

#include "common.cuh"
#include "moe_internal.h"

namespace gb {
namespace {

constexpr int kQWarps = 8;
constexpr int kQPitch = 68;  // floats per staged 64-element task (+4: lanes 0-7 on distinct banks)

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
  float clamp;  // act_clamp
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

// 1 + q / 16 as an f32 (exact) for the nibble q at bit `lo` of `word`: the
// nibble becomes the top four mantissa bits of 1.0.  Two integer operations,
// where an int-to-float conversion is a quarter-rate instruction.
__device__ __forceinline__ float nibble_float(uint32_t word, int lo) {
  const uint32_t m = lo <= 19 ? (word << (19 - lo)) : (word >> (lo - 19));
  return __uint_as_float((m & (0xFu << 19)) | 0x3F800000u);
}

__device__ __forceinline__ uint32_t word_of(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// One CTA per (active expert, 16 PAIRS rows); warp w owns PAIRS row pairs.
// Lane c takes the 64-element tasks c, c + 32, ... of a row: the sub-block
// pair (2j, 2j+1) of a super-block, whose 32 quant bytes hold sub-block 2j
// in the low nibbles and 2j+1 in the high ones, so each quant byte is loaded
// once.  TT tokens are staged in shared memory with their 32-element sums;
// a task adds d1 * sum(x q) - m1 * sum(x) per sub-block for the two rows of
// a pair and every staged token, each nibble converted once for all tokens;
// a butterfly folds the lanes.  The nibbles enter the products as
// 1 + q / 16 (nibble_float) and the sub-block's x sum takes the offset out:
// sum x q = 16 (sum x (1 + q / 16) - sum x).
template <int MODE, int TT, int PAIRS>
__global__ void __launch_bounds__(kQWarps * 32) q4k_rows_kernel(const QArgs a) {
  extern __shared__ float qsm[];
  const int K = a.K;
  const int NP = K >> 6;  // 64-element tasks per row
  const int NB = K >> 5;  // 32-element sub-blocks per row
  const int nsb = K >> 8;
  const int xstride = NP * kQPitch;
  float* xs = qsm;                   // [TT][NP][kQPitch]
  float* xsum = xs + TT * xstride;   // [TT][NB]

  const int slot = blockIdx.y;
  if (slot >= a.meta[0]) return;
  const int e = a.active[slot];
  const int le = e - a.e_begin;
  const int n = a.counts[e];
  const int p0 = a.offsets[e];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wrow0 = blockIdx.x * (kQWarps * 2 * PAIRS) + warp * 2 * PAIRS;
  const int64_t row_bytes = (int64_t)nsb * 144;
  const uint8_t* ebase = a.q + (int64_t)le * a.rows * row_bytes;

  for (int c0 = 0; c0 < n; c0 += TT) {
    const int nc = min(TT, n - c0);
    __syncthreads();
    // Every (token, float4) is independent, so all the row loads are in
    // flight; eight consecutive threads hold one 32-element sub-block and
    // fold its sum with three shuffles (the trip count is a multiple of the
    // block so that whole warps shuffle).
    const int per = K >> 2;
    const int span = (TT * per + blockDim.x - 1) / blockDim.x * blockDim.x;
#pragma unroll 2
    for (int i = threadIdx.x; i < span; i += blockDim.x) {
      const int j = i / per, k4 = i - j * per, k = k4 << 2;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (j < nc) {
        const int64_t src = MODE == GATE_UP ? a.perm[p0 + c0 + j] / a.top_k : p0 + c0 + j;
        v = reinterpret_cast<const float4*>(a.in + src * K)[k4];
      }
      float sum = __fadd_rn(__fadd_rn(v.x, v.y), __fadd_rn(v.z, v.w));
#pragma unroll
      for (int o = 4; o >= 1; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(kFullMask, sum, o));
      if (j < TT) {
        *reinterpret_cast<float4*>(xs + j * xstride + (k >> 6) * kQPitch + (k & 63)) = v;
        if ((k4 & 7) == 0) xsum[j * NB + (k >> 5)] = sum;
      }
    }
    __syncthreads();

    if (c0 == 0) {
      // pull every row pair's blocks toward L2 at once: the pairs below run
      // one after the other, so without this each waits a full HBM round trip
      for (int p = 1; p < PAIRS; ++p) {
        const int row = wrow0 + 2 * p;
        if (row >= a.rows) break;
        for (int c = lane; c < NP; c += 32) {
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            const uint8_t* blk = ebase + (int64_t)(row + r) * row_bytes + (c >> 2) * 144;
            asm volatile("prefetch.global.L2 [%0];" ::"l"(blk));
            asm volatile("prefetch.global.L2 [%0];" ::"l"(blk + 128));
          }
        }
      }
    }
    for (int p = 0; p < PAIRS; ++p) {
      const int row = wrow0 + 2 * p;
      if (row >= a.rows) break;
      float acc[2][TT];
#pragma unroll
      for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int t = 0; t < TT; ++t) acc[r][t] = 0.0f;
      for (int c = lane; c < NP; c += 32) {
        const int sb = c >> 2, jj = 2 * (c & 3);
        uint4 hdr[2], qa[2], qb[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const uint8_t* blk = ebase + (int64_t)(row + r) * row_bytes + sb * 144;
          hdr[r] = __ldg(reinterpret_cast<const uint4*>(blk));
          qa[r] = __ldg(reinterpret_cast<const uint4*>(blk + 16 + 16 * jj));
          qb[r] = __ldg(reinterpret_cast<const uint4*>(blk + 32 + 16 * jj));
        }
        float d1[2][2], m1[2][2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const uint8_t* hb = reinterpret_cast<const uint8_t*>(&hdr[r]);
          const float d = half_bits_to_f32((uint16_t)(hb[0] | (hb[1] << 8)));
          const float dmin = half_bits_to_f32((uint16_t)(hb[2] | (hb[3] << 8)));
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            int sc, mn;
            q4k_scale_min(jj + h, hb + 4, sc, mn);
            d1[r][h] = __fmul_rn(d, (float)sc);
            m1[r][h] = __fmul_rn(dmin, (float)mn);
          }
        }
        // s[r][h][t]: sum over the sub-block (h = 0 low nibbles, 1 high) of x q
        float s[2][2][TT];
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int t = 0; t < TT; ++t) s[r][h][t] = 0.0f;
        const float* xp = xs + c * kQPitch;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
          float qv[2][2][4];
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            const uint32_t word = w < 4 ? word_of(qa[r], w) : word_of(qb[r], w - 4);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              qv[r][0][i] = nibble_float(word, 8 * i);
              qv[r][1][i] = nibble_float(word, 8 * i + 4);
            }
          }
#pragma unroll
          for (int t = 0; t < TT; ++t) {
            const float4 xl = *reinterpret_cast<const float4*>(xp + t * xstride + 4 * w);
            const float4 xh = *reinterpret_cast<const float4*>(xp + t * xstride + 32 + 4 * w);
#pragma unroll
            for (int r = 0; r < 2; ++r) {
              s[r][0][t] = __fmaf_rn(xl.x, qv[r][0][0], s[r][0][t]);
              s[r][0][t] = __fmaf_rn(xl.y, qv[r][0][1], s[r][0][t]);
              s[r][0][t] = __fmaf_rn(xl.z, qv[r][0][2], s[r][0][t]);
              s[r][0][t] = __fmaf_rn(xl.w, qv[r][0][3], s[r][0][t]);
              s[r][1][t] = __fmaf_rn(xh.x, qv[r][1][0], s[r][1][t]);
              s[r][1][t] = __fmaf_rn(xh.y, qv[r][1][1], s[r][1][t]);
              s[r][1][t] = __fmaf_rn(xh.z, qv[r][1][2], s[r][1][t]);
              s[r][1][t] = __fmaf_rn(xh.w, qv[r][1][3], s[r][1][t]);
            }
          }
        }
#pragma unroll
        for (int t = 0; t < TT; ++t) {
          const float xa = xsum[t * NB + 2 * c], xb = xsum[t * NB + 2 * c + 1];
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            // s = sum x (1 + q / 16) = sum x + (sum x q) / 16
            const float sqa = __fmul_rn(16.0f, __fsub_rn(s[r][0][t], xa));
            const float sqb = __fmul_rn(16.0f, __fsub_rn(s[r][1][t], xb));
            const float pa = __fsub_rn(__fmul_rn(d1[r][0], sqa), __fmul_rn(m1[r][0], xa));
            const float pb = __fsub_rn(__fmul_rn(d1[r][1], sqb), __fmul_rn(m1[r][1], xb));
            acc[r][t] = __fadd_rn(acc[r][t], __fadd_rn(pa, pb));
          }
        }
      }
#pragma unroll
      for (int t = 0; t < TT; ++t) {
        if (t >= nc) break;
        const float s0 = warp_sum_butterfly(acc[0][t]);
        const float s1 = warp_sum_butterfly(acc[1][t]);
        if (lane == 0) {
          const int64_t pos = p0 + c0 + t;
          if (MODE == GATE_UP) {
            a.out[pos * a.out_stride + (row >> 1)] =
                act_apply(a.act_kind, s0, s1, a.limit, a.clamp);
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

template <int MODE, int TT, int PAIRS>
cudaError_t launch_q_shape(const Groups& g, const QArgs& a, cudaStream_t st) {
  constexpr int rows_cta = kQWarps * 2 * PAIRS;
  dim3 grid((unsigned)((a.rows + rows_cta - 1) / rows_cta), (unsigned)g.max_active);
  const size_t smem = (size_t)TT * (a.K / 64) * kQPitch * sizeof(float) +
                      (size_t)TT * (a.K / 32) * sizeof(float);
  auto kern = q4k_rows_kernel<MODE, TT, PAIRS>;
  cudaError_t err = set_smem_limit(kern, smem);
  if (err != cudaSuccess) return err;
  kern<<<grid, kQWarps * 32, smem, st>>>(a);
  return cudaGetLastError();
}

// Tokens staged per pass from the mean rows per local expert (an expert with
// more rows takes several passes over its weights, from L2).  From three rows
// per expert each warp owns four row pairs, so that a staged token serves 64
// rows; at one or two, a warp owns one pair (four times the CTAs, and no warp
// waits for one pair's bytes after another's).
template <int MODE>
cudaError_t launch_q(const Moe& m, const Groups& g, const QArgs& a, cudaStream_t st) {
  if (g.max_active <= 0) return cudaSuccess;
  const int64_t nloc = std::max(1, m.e_end - m.e_begin);
  const int64_t mean = (g.rows + nloc - 1) / nloc;
  if (mean <= 1) return launch_q_shape<MODE, 1, 1>(g, a, st);
  if (mean <= 2) return launch_q_shape<MODE, 2, 1>(g, a, st);
  if (mean <= 4) return launch_q_shape<MODE, 4, 4>(g, a, st);
  return launch_q_shape<MODE, 8, 4>(g, a, st);
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
  a.clamp = m.desc.act_clamp;
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
  return launch_q<GATE_UP>(m, g, a, st);
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
  return launch_q<DOWN>(m, g, a, st);
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
