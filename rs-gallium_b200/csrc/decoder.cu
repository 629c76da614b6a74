// decoder.cu -- the GPT-OSS decode stack around the MoE block (GGUF model,
// crates/gallium-models/src/gpt_oss_q.rs): embeddings, per layer RMSNorm ->
// attention with sinks -> residual -> RMSNorm -> MoE block -> residual, then
// the final RMSNorm, LM head and greedy token.
//
// Data layout in HBM (f32 unless noted):
//   h [rows][H]                      residual stream, rows = B * T (sequence-major)
//   xn [rows][H]                     normed rows (attention and MoE inputs)
//   qkv [rows][(nh + 2 nkv) hd]      q heads, then k heads, then v heads
//   att [rows][nh hd]                attention output (head-major, as the
//                                    reference's transpose + reshape leaves it)
//   kcache, vcache [layer][max_batch][nkv][S][hd]  K (after RoPE) and V per position
//   part [rows][nh][kSlots][hd + 2]  attention partials (max, sum, acc) per slot
//   bf16 hi / lo copies of a linear layer's input for the tensor-core GEMMs.
// Weights: wqkv [(nh + 2 nkv) hd][H] bf16 (q, k, v rows concatenated), wo
// [H][nh hd], embed / lm_head [vocab][H] bf16, norms and biases f32.
//
// The position of the next token lives on the device (d_pos) and every
// kernel that needs it reads it there, so one captured graph serves every
// step of a greedy decode.
#include <math.h>

#include <algorithm>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "exp_f32.h"
#include "umma.cuh"
#include "moe_internal.h"

namespace gb {
namespace dec {

constexpr int kChunk = 64;    // keys per attention chunk (staged in shared memory)
constexpr int kSlots = 8;     // CTAs splitting one query's keys (flash-decoding)
constexpr int kMaxHeadDim = 256;
constexpr int kMaxRep = 16;   // query heads per KV head
constexpr int kGemvWarps = 8;
constexpr int kGemvRows = 4;  // x rows staged per pass of the CUDA-core linear kernel

// ---- embeddings, norms, residuals -----------------------------------------

// h[r] = embed[tokens[r]] (bf16 widened).  One CTA per row.
__global__ void embed_kernel(const int32_t* __restrict__ tokens, const uint16_t* __restrict__ table,
                             int H, int vocab, float* __restrict__ h, int* __restrict__ err) {
  const int r = blockIdx.x;
  int tok = tokens[r];
  if (tok < 0 || tok >= vocab) {
    if (threadIdx.x == 0) atomicOr(err, 1);
    tok = 0;
  }
  const uint16_t* src = table + (int64_t)tok * H;
  for (int i = threadIdx.x; i < H; i += blockDim.x)
    h[(int64_t)r * H + i] = bf16_bits_to_f32(src[i]);
}

// RMSNorm of rows (candle_nn::ops::rms_norm: x / sqrt(mean(x^2) + eps) * w),
// after adding `delta` into the residual stream when delta is set
// (h = h + delta; the reference's `h + h_moe`).  Row r of the input is row
// src_row(r) = r * src_stride + src_off, so the final norm can take each
// sequence's last token.  One CTA of kNormThreads per output row; each
// thread keeps its float4s of the row in registers, so the row is read once
// and every load is issued before the first is used (H <= 4 * 4 * 1024).
constexpr int kNormThreads = 1024;
constexpr int kNormVec = 4;  // float4s per thread
// oh / ol (nullable): the output also as bf16 hi / lo (hi = bf16(v),
// lo = bf16(v - hi)), the input a tensor-core linear layer takes.
__device__ __forceinline__ void split_store(__nv_bfloat16* oh, __nv_bfloat16* ol, int64_t i,
                                            float v) {
  const __nv_bfloat16 hi = __float2bfloat16_rn(v);
  oh[i] = hi;
  ol[i] = __float2bfloat16_rn(__fsub_rn(v, __bfloat162float(hi)));
}

__global__ void __launch_bounds__(kNormThreads)
    add_rmsnorm_kernel(float* __restrict__ h, const float* __restrict__ delta,
                       const float* __restrict__ w, int H, float eps, int src_stride, int src_off,
                       float* __restrict__ out, __nv_bfloat16* __restrict__ oh,
                       __nv_bfloat16* __restrict__ ol) {
  __shared__ float red[32];
  const int r = blockIdx.x;
  const int64_t src = (int64_t)(r * src_stride + src_off) * H;
  float4* x4 = reinterpret_cast<float4*>(h + src);
  const float4* d4 = delta ? reinterpret_cast<const float4*>(delta + src) : nullptr;
  const int n4 = H / 4;
  const float4* w4 = reinterpret_cast<const float4*>(w);
  float4 v[kNormVec], wv[kNormVec];
#pragma unroll
  for (int j = 0; j < kNormVec; ++j) {  // the weights with the row, not after the reduction
    const int i = threadIdx.x + j * kNormThreads;
    wv[j] = i < n4 ? w4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int j = 0; j < kNormVec; ++j) {
    const int i = threadIdx.x + j * kNormThreads;
    v[j] = i < n4 ? x4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (d4) {
#pragma unroll
    for (int j = 0; j < kNormVec; ++j) {
      const int i = threadIdx.x + j * kNormThreads;
      if (i < n4) {
        const float4 dv = d4[i];
        v[j].x = __fadd_rn(v[j].x, dv.x);
        v[j].y = __fadd_rn(v[j].y, dv.y);
        v[j].z = __fadd_rn(v[j].z, dv.z);
        v[j].w = __fadd_rn(v[j].w, dv.w);
        x4[i] = v[j];
      }
    }
  }
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < kNormVec; ++j) {
    ss = __fmaf_rn(v[j].x, v[j].x, ss);
    ss = __fmaf_rn(v[j].y, v[j].y, ss);
    ss = __fmaf_rn(v[j].z, v[j].z, ss);
    ss = __fmaf_rn(v[j].w, v[j].w, ss);
  }
  ss = warp_sum_butterfly(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
    t = warp_sum_butterfly(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float m = sqrtf(__fadd_rn(__fdiv_rn(red[0], (float)H), eps));
  float4* o4 = reinterpret_cast<float4*>(out + (int64_t)r * H);
#pragma unroll
  for (int j = 0; j < kNormVec; ++j) {
    const int i = threadIdx.x + j * kNormThreads;
    if (i < n4) {
      const float4 y = make_float4(__fmul_rn(__fdiv_rn(v[j].x, m), wv[j].x),
                                   __fmul_rn(__fdiv_rn(v[j].y, m), wv[j].y),
                                   __fmul_rn(__fdiv_rn(v[j].z, m), wv[j].z),
                                   __fmul_rn(__fdiv_rn(v[j].w, m), wv[j].w));
      o4[i] = y;
      if (oh) {
        const int64_t b = (int64_t)r * H + 4 * i;
        split_store(oh, ol, b, y.x);
        split_store(oh, ol, b + 1, y.y);
        split_store(oh, ol, b + 2, y.z);
        split_store(oh, ol, b + 3, y.w);
      }
    }
  }
}

// ---- linear layers on the CUDA cores (fewer than 16 rows) ------------------
// Up to four rows: gemv_rows_kernel (and qkv_rope_gemv_kernel for the q/k/v
// projection), a warp per output row with all its weight loads in flight.
// Five to fifteen rows: linear_rows_kernel, a warp per pair of output rows.
// From sixteen rows the projections run on the tensor cores (dense_tc.cu).

// out[p][o] = (add ? out[p][o] : 0) + (x[p] . W[o] + bias[o]), W bf16 [n_out][K].
// A warp owns two output rows; x rows are staged kGemvRows at a time.
__global__ void __launch_bounds__(kGemvWarps * 32)
    linear_rows_kernel(const float* __restrict__ x, int n_x, int K,
                       const uint16_t* __restrict__ W, int n_out,
                       const float* __restrict__ bias, float* __restrict__ out, int out_stride,
                       int add) {
  extern __shared__ float xs[];  // [kGemvRows][K]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int o0 = (blockIdx.x * kGemvWarps + warp) * 2;
  const bool v0 = o0 < n_out, v1 = o0 + 1 < n_out;
  const uint16_t* w0 = W + (int64_t)(v0 ? o0 : 0) * K;
  const uint16_t* w1 = W + (int64_t)(v1 ? o0 + 1 : 0) * K;
  const int npieces = K / 8;  // 16-byte pieces of 8 bf16
  for (int p0 = 0; p0 < n_x; p0 += kGemvRows) {
    const int np = min(kGemvRows, n_x - p0);
    __syncthreads();
    for (int i = threadIdx.x; i < np * K / 4; i += blockDim.x)
      reinterpret_cast<float4*>(xs)[i] = reinterpret_cast<const float4*>(x + (int64_t)p0 * K)[i];
    __syncthreads();
    if (!v0) continue;
    float acc[2][kGemvRows];
#pragma unroll
    for (int j = 0; j < kGemvRows; ++j) acc[0][j] = acc[1][j] = 0.0f;
#pragma unroll 4
    for (int q = lane; q < npieces; q += 32) {
      const uint4 a = __ldg(reinterpret_cast<const uint4*>(w0) + q);
      const uint4 b = __ldg(reinterpret_cast<const uint4*>(w1) + q);
      const uint32_t wa[4] = {a.x, a.y, a.z, a.w}, wb[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int j = 0; j < kGemvRows; ++j) {
        if (j < np) {
          const float* xj = xs + j * K + q * 8;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float xa = xj[2 * e], xb = xj[2 * e + 1];
            acc[0][j] = __fmaf_rn(xa, __uint_as_float(wa[e] << 16), acc[0][j]);
            acc[0][j] = __fmaf_rn(xb, __uint_as_float(wa[e] & 0xffff0000u), acc[0][j]);
            acc[1][j] = __fmaf_rn(xa, __uint_as_float(wb[e] << 16), acc[1][j]);
            acc[1][j] = __fmaf_rn(xb, __uint_as_float(wb[e] & 0xffff0000u), acc[1][j]);
          }
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kGemvRows; ++j) {
      if (j >= np) break;
      const float s0 = warp_sum_butterfly(acc[0][j]);
      const float s1 = warp_sum_butterfly(acc[1][j]);
      if (lane == 0) {
        float* o = out + (int64_t)(p0 + j) * out_stride + o0;
        float r0 = bias ? __fadd_rn(s0, bias[o0]) : s0;
        if (add) r0 = __fadd_rn(__ldcg(o), r0);
        o[0] = r0;
        if (v1) {
          float r1 = bias ? __fadd_rn(s1, bias[o0 + 1]) : s1;
          if (add) r1 = __fadd_rn(__ldcg(o + 1), r1);
          o[1] = r1;
        }
      }
    }
  }
}

// The same product for up to kGemvRows rows of x, a warp per output row:
// each lane requests all its 16-byte pieces of the row (KP per pass of 32 KP
// pieces) before the first multiply, so a warp keeps up to 8 KB of weights
// in flight.  Used when x has at most kGemvRows rows.
template <int KP>
__global__ void __launch_bounds__(kGemvWarps * 32)
    gemv_rows_kernel(const float* __restrict__ x, int n_x, int K,
                     const uint16_t* __restrict__ W, int n_out, const float* __restrict__ bias,
                     float* __restrict__ out, int out_stride, int add) {
  extern __shared__ float xs[];  // [n_x][K]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  {
    const int n4 = n_x * K / 4;
    const float4* src = reinterpret_cast<const float4*>(x);
    float4* dst = reinterpret_cast<float4*>(xs);
#pragma unroll 4
    for (int i = threadIdx.x; i < n4; i += blockDim.x) dst[i] = src[i];
  }
  __syncthreads();
  const int o = blockIdx.x * kGemvWarps + warp;
  if (o >= n_out) return;
  const uint4* wr = reinterpret_cast<const uint4*>(W + (int64_t)o * K);
  const int npieces = K / 8;
  float acc[kGemvRows];
#pragma unroll
  for (int j = 0; j < kGemvRows; ++j) acc[j] = 0.0f;
  for (int base = 0; base < npieces; base += 32 * KP) {
    uint4 wv[KP];
#pragma unroll
    for (int u = 0; u < KP; ++u) {
      const int q = base + lane + 32 * u;
      wv[u] = q < npieces ? __ldg(wr + q) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < KP; ++u) {
      const int q = base + lane + 32 * u;
      if (q < npieces) {
        const uint32_t ww[4] = {wv[u].x, wv[u].y, wv[u].z, wv[u].w};
#pragma unroll
        for (int j = 0; j < kGemvRows; ++j) {
          if (j < n_x) {
            const float* xj = xs + j * K + q * 8;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              acc[j] = __fmaf_rn(xj[2 * e], __uint_as_float(ww[e] << 16), acc[j]);
              acc[j] = __fmaf_rn(xj[2 * e + 1], __uint_as_float(ww[e] & 0xffff0000u), acc[j]);
            }
          }
        }
      }
    }
  }
#pragma unroll
  for (int j = 0; j < kGemvRows; ++j) {
    if (j >= n_x) break;
    const float sum = warp_sum_butterfly(acc[j]);
    if (lane == 0) {
      float* dst = out + (int64_t)j * out_stride + o;
      float r = bias ? __fadd_rn(sum, bias[o]) : sum;
      if (add) r = __fadd_rn(__ldcg(dst), r);
      *dst = r;
    }
  }
}

// q/k/v projection of up to kGemvRows rows with RoPE and the KV-cache store
// folded in: a warp owns output rows j and j + hd / 2 of one head (the pair
// one rotation mixes), requests KP pieces of each row per pass before the
// first multiply, and lane 0 adds the biases, rotates q and k as
// rope_append_kernel does (same roundings) and stores q into qkv, k and v
// into sequence b's cache at position pos + t.
template <int KP>
__global__ void __launch_bounds__(kGemvWarps * 32)
    qkv_rope_gemv_kernel(const float* __restrict__ x, int n_x, int K,
                         const uint16_t* __restrict__ W, const float* __restrict__ bias, int nh,
                         int nkv, int hd, int T, const float* __restrict__ cos_t,
                         const float* __restrict__ sin_t, const int* __restrict__ d_pos, int S,
                         float* __restrict__ qkv, float* __restrict__ kcache,
                         float* __restrict__ vcache) {
  extern __shared__ float xs[];  // [n_x][K]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  {
    const int n4 = n_x * K / 4;
    const float4* src = reinterpret_cast<const float4*>(x);
    float4* dst = reinterpret_cast<float4*>(xs);
#pragma unroll 4
    for (int i = threadIdx.x; i < n4; i += blockDim.x) dst[i] = src[i];
  }
  __syncthreads();
  const int half = hd / 2;
  const int pidx = blockIdx.x * kGemvWarps + warp;
  if (pidx >= (nh + 2 * nkv) * half) return;
  const int hh = pidx / half, j = pidx - hh * half;
  const int r1 = hh * hd + j, r2 = r1 + half;
  const uint4* w1 = reinterpret_cast<const uint4*>(W + (int64_t)r1 * K);
  const uint4* w2 = reinterpret_cast<const uint4*>(W + (int64_t)r2 * K);
  const int npieces = K / 8;
  float a1[kGemvRows], a2[kGemvRows];
#pragma unroll
  for (int t = 0; t < kGemvRows; ++t) a1[t] = a2[t] = 0.0f;
  for (int base = 0; base < npieces; base += 32 * KP) {
    uint4 v1[KP], v2[KP];
#pragma unroll
    for (int u = 0; u < KP; ++u) {
      const int q = base + lane + 32 * u;
      v1[u] = q < npieces ? __ldg(w1 + q) : make_uint4(0u, 0u, 0u, 0u);
      v2[u] = q < npieces ? __ldg(w2 + q) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < KP; ++u) {
      const int q = base + lane + 32 * u;
      if (q < npieces) {
        const uint32_t b1[4] = {v1[u].x, v1[u].y, v1[u].z, v1[u].w};
        const uint32_t b2[4] = {v2[u].x, v2[u].y, v2[u].z, v2[u].w};
#pragma unroll
        for (int t = 0; t < kGemvRows; ++t) {
          if (t < n_x) {
            const float* xt = xs + t * K + q * 8;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float xa = xt[2 * e], xb = xt[2 * e + 1];
              a1[t] = __fmaf_rn(xa, __uint_as_float(b1[e] << 16), a1[t]);
              a1[t] = __fmaf_rn(xb, __uint_as_float(b1[e] & 0xffff0000u), a1[t]);
              a2[t] = __fmaf_rn(xa, __uint_as_float(b2[e] << 16), a2[t]);
              a2[t] = __fmaf_rn(xb, __uint_as_float(b2[e] & 0xffff0000u), a2[t]);
            }
          }
        }
      }
    }
  }
  const int qkv_w = (nh + 2 * nkv) * hd;
#pragma unroll
  for (int t = 0; t < kGemvRows; ++t) {
    if (t >= n_x) break;
    float s1 = warp_sum_butterfly(a1[t]);
    float s2 = warp_sum_butterfly(a2[t]);
    if (lane == 0) {
      if (bias) {
        s1 = __fadd_rn(s1, bias[r1]);
        s2 = __fadd_rn(s2, bias[r2]);
      }
      const int b = t / T, tt = t - b * T;
      const int p = *d_pos + tt;
      if (hh < nh + nkv) {  // q and k heads rotate
        const float c = cos_t[(int64_t)p * half + j], sn = sin_t[(int64_t)p * half + j];
        const float y1 = __fsub_rn(__fmul_rn(s1, c), __fmul_rn(s2, sn));
        const float y2 = __fadd_rn(__fmul_rn(s1, sn), __fmul_rn(s2, c));
        s1 = y1;
        s2 = y2;
      }
      if (hh < nh) {
        qkv[(int64_t)t * qkv_w + r1] = s1;
        qkv[(int64_t)t * qkv_w + r2] = s2;
      } else {
        const bool is_k = hh < nh + nkv;
        const int g = is_k ? hh - nh : hh - nh - nkv;
        float* dst = (is_k ? kcache : vcache) + (((int64_t)b * nkv + g) * S + p) * hd;
        dst[j] = s1;
        dst[j + half] = s2;
      }
    }
  }
}

// ---- RoPE and the KV cache --------------------------------------------------

// Rotates the q and k heads of row (b, t) at position pos + t in place
// (candle_nn::rotary_emb::rope, halves layout: x1' = x1 cos - x2 sin,
// x2' = x1 sin + x2 cos, each product rounded, pos_enc.rs:199-217) and
// stores k and v at that position of sequence b's cache.  Grid (rows,
// heads nh + 2 nkv); one thread per rotated pair (hd / 2 threads).
__global__ void rope_append_kernel(float* __restrict__ qkv, int T, int nh, int nkv, int hd,
                                   const float* __restrict__ cos_t,
                                   const float* __restrict__ sin_t, const int* __restrict__ d_pos,
                                   int S, float* __restrict__ kcache, float* __restrict__ vcache) {
  const int r = blockIdx.x, hh = blockIdx.y, j = threadIdx.x;
  const int b = r / T, t = r - b * T;
  const int p = *d_pos + t;
  const int half = hd / 2;
  float* x = qkv + (int64_t)r * (nh + 2 * nkv) * hd + hh * hd;
  float x1 = x[j], x2 = x[j + half];
  if (hh < nh + nkv) {  // q and k heads rotate
    const float c = cos_t[(int64_t)p * half + j], s = sin_t[(int64_t)p * half + j];
    const float y1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
    const float y2 = __fadd_rn(__fmul_rn(x1, s), __fmul_rn(x2, c));
    x1 = y1;
    x2 = y2;
    if (hh < nh) {
      x[j] = x1;
      x[j + half] = x2;
      return;
    }
  }
  const bool is_k = hh < nh + nkv;
  const int g = is_k ? hh - nh : hh - nh - nkv;
  float* dst = (is_k ? kcache : vcache) + (((int64_t)b * nkv + g) * S + p) * hd;
  dst[j] = x1;
  dst[j + half] = x2;
}

// ---- attention --------------------------------------------------------------

// Partial attention of query row (b, t) against KV head g's keys, for every
// query head of the group (warp w = head g * rep + w): scores (q . k) * scale
// over the visible keys (causal; the last `window` positions on sliding
// layers), a running max and sum, and sum_j p_j v_j.  The visible keys are
// split into kChunk-key chunks; CTA slot c of gridDim.x (at most kSlots)
// takes chunks c, c + gridDim.x, ... and writes (max, sum, acc[hd]) for its
// chunks.  Keys and values of a chunk
// are staged in shared memory once for the group.
// Query rows row0 + blockIdx.z; partials indexed by blockIdx.z.
__global__ void __launch_bounds__(kMaxRep * 32)
    attn_partial_kernel(const float* __restrict__ qkv, int row0, int T, int nh, int nkv, int hd,
                        const int* __restrict__ d_pos, int sliding, int window, float scale,
                        int S, const float* __restrict__ kcache,
                        const float* __restrict__ vcache, float* __restrict__ part) {
  extern __shared__ float sm[];
  const int rep = nh / nkv;
  const int slot = blockIdx.x, g = blockIdx.y, r = row0 + blockIdx.z;
  const int b = r / T, t = r - b * T;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hq = g * rep + warp;
  const int qp = *d_pos + t;                      // the query's position
  const int lo = sliding ? max(0, qp - window + 1) : 0;
  const int nkeys = qp - lo + 1;
  const int nchunks = (nkeys + kChunk - 1) / kChunk;
  const int kpitch = hd + 1;
  float* ks = sm;                                 // [kChunk][hd + 1]
  float* vs = ks + kChunk * kpitch;               // [kChunk][hd]
  float* qs = vs + kChunk * hd;                   // [rep][hd]
  float* ps = qs + rep * hd;                      // [rep][kChunk]
  const int qkv_w = (nh + 2 * nkv) * hd;
  for (int i = threadIdx.x; i < rep * hd; i += blockDim.x)
    qs[i] = qkv[(int64_t)r * qkv_w + (g * rep) * hd + i];
  const float* kbase = kcache + ((int64_t)b * nkv + g) * S * hd;
  const float* vbase = vcache + ((int64_t)b * nkv + g) * S * hd;
  float m_run = -INFINITY, s_run = 0.0f;
  float acc[kMaxHeadDim / 32];
#pragma unroll
  for (int i = 0; i < kMaxHeadDim / 32; ++i) acc[i] = 0.0f;
  const int dpl = hd / 32;  // dims per lane (hd a multiple of 32)
  for (int c = slot; c < nchunks; c += gridDim.x) {
    const int j0 = lo + c * kChunk;
    const int nj = min(kChunk, qp + 1 - j0);
    __syncthreads();
    {
      // float4 loads, all of a thread's issued before any is stored
      const int n4 = nj * hd / 4, hd4 = hd / 4;
      const float4* k4 = reinterpret_cast<const float4*>(kbase + (int64_t)j0 * hd);
      const float4* v4 = reinterpret_cast<const float4*>(vbase + (int64_t)j0 * hd);
      constexpr int kU = kChunk * kMaxHeadDim / 4 / (kMaxRep * 32) > 8
                             ? 8
                             : kChunk * kMaxHeadDim / 4 / (kMaxRep * 32);
      for (int i0 = threadIdx.x; i0 < n4; i0 += kU * blockDim.x) {
        float4 kv[kU], vv[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int i = i0 + u * blockDim.x;
          if (i < n4) {
            kv[u] = k4[i];
            vv[u] = v4[i];
          }
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int i = i0 + u * blockDim.x;
          if (i < n4) {
            const int j = i / hd4, d = (i - j * hd4) * 4;
            float* kd = ks + j * kpitch + d;
            kd[0] = kv[u].x;
            kd[1] = kv[u].y;
            kd[2] = kv[u].z;
            kd[3] = kv[u].w;
            *reinterpret_cast<float4*>(vs + j * hd + d) = vv[u];
          }
        }
      }
    }
    __syncthreads();
    if (warp < rep) {
      const float* q = qs + warp * hd;
      float* p = ps + warp * kChunk;
      float cmax = -INFINITY;
      for (int j = lane; j < nj; j += 32) {
        const float* kj = ks + j * kpitch;
        float dot = 0.0f;
        for (int d = 0; d < hd; ++d) dot = __fmaf_rn(q[d], kj[d], dot);
        const float sc = __fmul_rn(dot, scale);
        p[j] = sc;
        cmax = fmaxf(cmax, sc);
      }
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) cmax = fmaxf(cmax, __shfl_xor_sync(kFullMask, cmax, o));
      const float m_new = fmaxf(m_run, cmax);
      const float corr = m_run == -INFINITY ? 0.0f : exp_f32(__fsub_rn(m_run, m_new));
      float csum = 0.0f;
      for (int j = lane; j < nj; j += 32) {
        const float e = exp_f32(__fsub_rn(p[j], m_new));
        p[j] = e;
        csum = __fadd_rn(csum, e);
      }
      csum = warp_sum_butterfly(csum);
      s_run = __fadd_rn(__fmul_rn(s_run, corr), csum);
      __syncwarp();
#pragma unroll
      for (int i = 0; i < kMaxHeadDim / 32; ++i) {
        if (i < dpl) {
          const int d = lane + 32 * i;
          float a = __fmul_rn(acc[i], corr);
          for (int j = 0; j < nj; ++j) a = __fmaf_rn(p[j], vs[j * hd + d], a);
          acc[i] = a;
        }
      }
      m_run = m_new;
    }
  }
  if (warp < rep) {
    float* o = part + (((int64_t)blockIdx.z * nh + hq) * kSlots + slot) * (hd + 2);
    if (lane == 0) {
      o[0] = m_run;
      o[1] = s_run;
    }
#pragma unroll
    for (int i = 0; i < kMaxHeadDim / 32; ++i)
      if (i < dpl) o[2 + lane + 32 * i] = acc[i];
  }
}

// Merges the slots of each (row, head) with the head's sink logit
// (gpt_oss_q.rs:92-101: softmax over the scores and the sink, the sink's
// column dropped): out = sum_c acc_c e^(m_c - M) / (e^(sink - M) + sum_c s_c
// e^(m_c - M)), M the largest of the sink and the slots' maxima (the first
// nslots slots are used).  One warp per (row, head); partial row i is output
// row row0 + i.
__global__ void attn_combine_kernel(const float* __restrict__ part, int rows, int row0, int nh,
                                    int hd, int nslots, const float* __restrict__ sinks,
                                    float* __restrict__ out, __nv_bfloat16* __restrict__ oh,
                                    __nv_bfloat16* __restrict__ ol) {
  const int wid = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (wid >= rows * nh) return;
  const int r = row0 + wid / nh, hq = wid % nh;
  const float* pp = part + (int64_t)wid * kSlots * (hd + 2);
  const float sink = sinks[hq];
  float M = sink;
  for (int c = 0; c < nslots; ++c) M = fmaxf(M, pp[c * (hd + 2)]);
  float S = exp_f32(__fsub_rn(sink, M));
  float f[kSlots];
  for (int c = 0; c < nslots; ++c) {
    const float mc = pp[c * (hd + 2)];
    f[c] = mc == -INFINITY ? 0.0f : exp_f32(__fsub_rn(mc, M));
    S = __fadd_rn(S, __fmul_rn(pp[c * (hd + 2) + 1], f[c]));
  }
  for (int d = lane; d < hd; d += 32) {
    float a = 0.0f;
    for (int c = 0; c < nslots; ++c)
      if (f[c] != 0.0f) a = __fmaf_rn(pp[c * (hd + 2) + 2 + d], f[c], a);
    const int64_t o = (int64_t)r * nh * hd + hq * hd + d;
    const float y = __fdiv_rn(a, S);
    out[o] = y;
    if (oh) split_store(oh, ol, o, y);
  }
}

// ---- greedy token -----------------------------------------------------------

// next[b] = the index of the largest logit of row b, the highest index among
// equal maxima (Iterator::max_by keeps the last maximum, sampling.rs:85-92);
// a NaN never wins.  Grid (chunks, B): each CTA reduces kArgmaxPerThread x
// blockDim logits to one key (the value's bits made orderable in the high
// half, the index in the low half, so the largest key is the largest value
// and, among equal values, the highest index), atomicMax into slot[b]; the
// CTA that finishes last for row b publishes the token and clears the slot
// and its ticket for the next step.
constexpr int kArgmaxThreads = 1024;
constexpr int kArgmaxPerThread = 8;

__device__ __forceinline__ unsigned long long argmax_key(float v, int i) {
  uint32_t u = __float_as_uint(v == 0.0f ? 0.0f : v);  // -0 and +0 compare equal
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (uint32_t)i;
}

__global__ void __launch_bounds__(kArgmaxThreads)
    argmax_kernel(const float* __restrict__ logits, int vocab,
                  unsigned long long* __restrict__ slot, unsigned* __restrict__ ticket,
                  int32_t* __restrict__ next, int32_t* __restrict__ out_tokens) {
  __shared__ unsigned long long red[32];
  __shared__ bool last;
  const int b = blockIdx.y;
  const float* row = logits + (int64_t)b * vocab;
  const int base = blockIdx.x * kArgmaxThreads * kArgmaxPerThread + threadIdx.x;
  float v[kArgmaxPerThread];
#pragma unroll
  for (int j = 0; j < kArgmaxPerThread; ++j) {
    const int i = base + j * kArgmaxThreads;
    v[j] = i < vocab ? row[i] : __int_as_float(0x7fc00000);  // NaN: skipped
  }
  unsigned long long best = 0;
#pragma unroll
  for (int j = 0; j < kArgmaxPerThread; ++j)
    if (!(v[j] != v[j])) {
      const unsigned long long k = argmax_key(v[j], base + j * kArgmaxThreads);
      best = k > best ? k : best;
    }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(kFullMask, best, o);
    best = other > best ? other : best;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kArgmaxThreads / 32; ++w) best = red[w] > best ? red[w] : best;
    if (best) atomicMax(&slot[b], best);
    __threadfence();
    last = atomicAdd(&ticket[b], 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    __threadfence();
    const unsigned long long k = atomicExch(&slot[b], 0ull);
    ticket[b] = 0;
    const int tok = (int)(uint32_t)(k & 0xffffffffull);  // 0 when every logit was NaN
    next[b] = tok;
    if (out_tokens) out_tokens[b] = tok;
  }
}

__global__ void set_int_kernel(int* __restrict__ p, int v) { *p = v; }

// After a greedy step: the next position.
__global__ void advance_kernel(int* __restrict__ d_pos, int T) { *d_pos += T; }

}  // namespace dec
}  // namespace gb

// ===========================================================================
// Host side
// ===========================================================================
namespace gb {
namespace {

constexpr int kTcMinRows = 16;     // linear layers with this many rows use the tensor cores
constexpr int64_t kLinearPartFloats = int64_t(4) << 20;  // split-K partial sums (16 MB)
constexpr int kAttnRowsPerLaunch = 256;  // query rows per attention launch (partials buffer)

struct DecLayer {
  float* attn_norm = nullptr;
  float* post_norm = nullptr;
  uint16_t* wqkv = nullptr;  // [(nh + 2 nkv) hd][H] bf16 bits
  uint16_t* wo = nullptr;    // [H][nh hd]
  float* bqkv = nullptr;     // [(nh + 2 nkv) hd], absent parts zero; null if none
  float* bo = nullptr;
  float* sinks = nullptr;
  int sliding = 0;
  gb_moe* moe = nullptr;
  alignas(64) unsigned char map_qkv[128] = {};
  alignas(64) unsigned char map_o[128] = {};
};

struct GenGraph {
  int B = 0;
  cudaGraphExec_t exec = nullptr;
};

}  // namespace

struct Decoder {
  gb_decoder_desc d{};
  int device = 0, sm_count = 0;
  int qkv_w = 0, att_w = 0;  // (nh + 2 nkv) hd, nh hd
  int64_t rows_cap = 0;      // max_batch * max_tokens
  bool tc = false;           // linear layers may use the tensor cores
  std::vector<DecLayer> layers;
  uint16_t* embed = nullptr;
  uint16_t* lm_head = nullptr;  // == embed when tied
  float* final_norm = nullptr;
  float* rope_cos = nullptr;    // [S][hd / 2]
  float* rope_sin = nullptr;
  float* kcache = nullptr;      // [L][max_batch][nkv][S][hd]
  float* vcache = nullptr;
  void* act_base = nullptr;     // one allocation for the buffers below
  float *h = nullptr, *xn = nullptr, *qkv = nullptr, *att = nullptr, *moe_out = nullptr;
  float *last = nullptr, *logits = nullptr, *part = nullptr;
  float* lin_part = nullptr;  // [kLinearPartFloats] split-K partials of the linear layers
  __nv_bfloat16 *xh = nullptr, *xl = nullptr;  // [rows_cap][max(H, nh hd)]
  int32_t *next = nullptr, *tok_buf = nullptr, *d_pos = nullptr, *err = nullptr;
  unsigned long long* am_slot = nullptr;  // [max_batch] greedy-token reduction, zero between steps
  unsigned* am_ticket = nullptr;          // [max_batch]
  alignas(64) unsigned char map_xh_h[128] = {};  // split activations, K = H
  alignas(64) unsigned char map_xl_h[128] = {};
  alignas(64) unsigned char map_xh_a[128] = {};  // K = nh hd
  alignas(64) unsigned char map_xl_a[128] = {};
  alignas(64) unsigned char map_lm[128] = {};
  int64_t pos = 0;
  int batch = 0;
  bool profiling = false;
  std::vector<cudaEvent_t> ev;  // per layer: attention start, MoE start; then head start, end
  bool timed = false;
  cudaStream_t cap = nullptr;
  std::vector<GenGraph> gens;
};

namespace {

struct DevScope {
  int prev = -1;
  explicit DevScope(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    cudaSetDevice(dev);
  }
  ~DevScope() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

#define DEC_CUDA(expr, what)                                                           \
  do {                                                                                 \
    cudaError_t e_ = (expr);                                                           \
    if (e_ != cudaSuccess)                                                             \
      return set_error(GB_ERR_CUDA, "%s: %s", (what), cudaGetErrorString(e_));         \
  } while (0)

template <typename Tp>
int dalloc(Tp** p, size_t bytes, const char* what) {
  if (cudaMalloc((void**)p, std::max<size_t>(bytes, 16)) != cudaSuccess) {
    cudaGetLastError();
    return set_error(GB_ERR_NO_MEMORY, "cudaMalloc(%zu bytes) for %s failed", bytes, what);
  }
  return GB_OK;
}

template <typename Tp>
int upload(Tp** dst, const void* src, size_t bytes, const char* what) {
  int rc = dalloc(dst, bytes, what);
  if (rc) return rc;
  DEC_CUDA(cudaMemcpy(*dst, src, bytes, cudaMemcpyHostToDevice), what);
  return GB_OK;
}

// RoPE cos / sin tables [S][hd / 2] as pos_enc.rs:82-176 builds them:
// inverse frequencies in f64 (YaRN-adjusted when the factor is above 1),
// rounded to f32; each angle the f32 product position x frequency; cos and
// sin of that f32 angle in f32.
void rope_tables(const gb_decoder_desc& d, std::vector<float>& c, std::vector<float>& s) {
  const int rot = d.head_dim, half = rot / 2;
  std::vector<double> inv(half);
  const double theta = d.rope_theta;
  for (int i = 0; i < half; ++i) inv[i] = 1.0 / pow(theta, 2.0 * i / (double)rot);
  if (d.rope_scaling_factor > 1.0f) {
    const double factor = d.rope_scaling_factor, orig = d.rope_orig_ctx;
    const double bf = d.rope_beta_fast > 0.0f ? d.rope_beta_fast : 32.0;
    const double bs = d.rope_beta_slow > 0.0f ? d.rope_beta_slow : 1.0;
    const double pi = 3.14159265358979323846;
    const double low = floor(orig / (bf * 2.0 * pi));
    const double high = floor(orig / (bs * 2.0 * pi));
    for (int i = 0; i < half; ++i) {
      const double wavelength = 2.0 * pi / inv[i];
      const double ratio = wavelength / orig;
      if (ratio < low / rot) {
        // high frequency: kept
      } else if (ratio > high / rot) {
        inv[i] /= factor;
      } else {
        const double t = ((double)i - low) / (high - low);
        inv[i] *= 1.0 / (1.0 + (factor - 1.0) * t);
      }
    }
  }
  c.resize((size_t)d.max_seq_len * half);
  s.resize(c.size());
  for (int p = 0; p < d.max_seq_len; ++p) {
    for (int i = 0; i < half; ++i) {
      const float ang = (float)p * (float)inv[i];
      c[(size_t)p * half + i] = cosf(ang);
      s[(size_t)p * half + i] = sinf(ang);
    }
  }
}

int validate(const gb_decoder_desc* d) {
  if (!d) return set_error(GB_ERR_INVALID_ARG, "desc is null");
  if (d->struct_size != sizeof(gb_decoder_desc))
    return set_error(GB_ERR_INVALID_ARG, "gb_decoder_desc.struct_size %u != %zu", d->struct_size,
                     sizeof(gb_decoder_desc));
  if (d->n_layers < 1 || d->hidden < 32 || d->hidden % 32 ||
      d->hidden > 4 * dec::kNormVec * dec::kNormThreads || d->n_heads < 1 ||
      d->n_kv_heads < 1 || d->n_heads % d->n_kv_heads || d->n_heads / d->n_kv_heads > dec::kMaxRep)
    return set_error(GB_ERR_INVALID_ARG,
                     "need n_layers >= 1, hidden a multiple of 32 up to %d, n_heads a multiple "
                     "of n_kv_heads with at most %d query heads per KV head",
                     4 * dec::kNormVec * dec::kNormThreads, dec::kMaxRep);
  if (d->head_dim < 32 || d->head_dim % 32 || d->head_dim > dec::kMaxHeadDim)
    return set_error(GB_ERR_UNSUPPORTED, "head_dim %d: a multiple of 32 up to %d", d->head_dim,
                     dec::kMaxHeadDim);
  if ((d->n_heads * d->head_dim) % 8)
    return set_error(GB_ERR_INVALID_ARG, "n_heads * head_dim must be a multiple of 8");
  if (d->vocab < 1 || d->sliding_window < 1 || d->max_seq_len < 1 || d->max_batch < 1 ||
      d->max_tokens < 1)
    return set_error(GB_ERR_INVALID_ARG,
                     "vocab, sliding_window, max_seq_len, max_batch and max_tokens must be >= 1");
  if ((int64_t)d->max_batch * d->max_tokens > (1 << 20))
    return set_error(GB_ERR_UNSUPPORTED, "max_batch * max_tokens above 2^20");
  if (!(d->rope_theta > 0.0f) || !(d->rms_eps >= 0.0f))
    return set_error(GB_ERR_INVALID_ARG, "rope_theta must be > 0 and rms_eps >= 0");
  if (d->rope_scaling_factor > 1.0f && d->rope_orig_ctx < 1)
    return set_error(GB_ERR_INVALID_ARG, "YaRN scaling needs rope_orig_ctx >= 1");
  if (!d->embed || !d->final_norm || !d->layers)
    return set_error(GB_ERR_INVALID_ARG, "embed, final_norm and layers are required");
  for (int l = 0; l < d->n_layers; ++l) {
    const gb_decoder_layer& L = d->layers[l];
    if (!L.attn_norm || !L.post_attn_norm || !L.wq || !L.wk || !L.wv || !L.wo || !L.sinks ||
        !L.moe)
      return set_error(GB_ERR_INVALID_ARG,
                       "layer %d: attn_norm, post_attn_norm, wq, wk, wv, wo, sinks and moe are "
                       "required",
                       l);
    if (L.moe->hidden != d->hidden)
      return set_error(GB_ERR_INVALID_ARG, "layer %d: the MoE block's hidden %d != %d", l,
                       L.moe->hidden, d->hidden);
    if (L.sliding != 0 && L.sliding != 1)
      return set_error(GB_ERR_INVALID_ARG, "layer %d: sliding must be 0 or 1", l);
  }
  return GB_OK;
}

void release(Decoder* D) {
  if (!D) return;
  DevScope ds(D->device);
  for (auto& g : D->gens)
    if (g.exec) cudaGraphExecDestroy(g.exec);
  for (auto& L : D->layers) {
    for (void* p : {(void*)L.attn_norm, (void*)L.post_norm, (void*)L.wqkv, (void*)L.wo,
                    (void*)L.bqkv, (void*)L.bo, (void*)L.sinks})
      cudaFree(p);
    if (L.moe) gb_moe_destroy(L.moe);
  }
  if (D->lm_head != D->embed) cudaFree(D->lm_head);
  for (void* p : {(void*)D->embed, (void*)D->final_norm, (void*)D->rope_cos, (void*)D->rope_sin,
                  (void*)D->kcache, (void*)D->vcache, D->act_base})
    cudaFree(p);
  for (cudaEvent_t e : D->ev) cudaEventDestroy(e);
  if (D->cap) cudaStreamDestroy(D->cap);
  delete D;
}

int upload_layer(Decoder& D, const gb_decoder_layer& src, DecLayer& L) {
  const gb_decoder_desc& d = D.d;
  const size_t H = d.hidden, hd = d.head_dim;
  const size_t qn = d.n_heads * hd, kn = d.n_kv_heads * hd;
  int rc;
  if ((rc = upload(&L.attn_norm, src.attn_norm, H * 4, "attention norm"))) return rc;
  if ((rc = upload(&L.post_norm, src.post_attn_norm, H * 4, "post-attention norm"))) return rc;
  if ((rc = dalloc(&L.wqkv, (qn + 2 * kn) * H * 2, "q/k/v weights"))) return rc;
  DEC_CUDA(cudaMemcpy(L.wqkv, src.wq, qn * H * 2, cudaMemcpyHostToDevice), "q weights");
  DEC_CUDA(cudaMemcpy(L.wqkv + qn * H, src.wk, kn * H * 2, cudaMemcpyHostToDevice), "k weights");
  DEC_CUDA(cudaMemcpy(L.wqkv + (qn + kn) * H, src.wv, kn * H * 2, cudaMemcpyHostToDevice),
           "v weights");
  if ((rc = upload(&L.wo, src.wo, H * qn * 2, "o weights"))) return rc;
  if (src.bq || src.bk || src.bv) {
    if ((rc = dalloc(&L.bqkv, (qn + 2 * kn) * 4, "q/k/v biases"))) return rc;
    DEC_CUDA(cudaMemset(L.bqkv, 0, (qn + 2 * kn) * 4), "q/k/v biases");
    if (src.bq) DEC_CUDA(cudaMemcpy(L.bqkv, src.bq, qn * 4, cudaMemcpyHostToDevice), "q bias");
    if (src.bk)
      DEC_CUDA(cudaMemcpy(L.bqkv + qn, src.bk, kn * 4, cudaMemcpyHostToDevice), "k bias");
    if (src.bv)
      DEC_CUDA(cudaMemcpy(L.bqkv + qn + kn, src.bv, kn * 4, cudaMemcpyHostToDevice), "v bias");
  }
  if (src.bo && (rc = upload(&L.bo, src.bo, H * 4, "o bias"))) return rc;
  if ((rc = upload(&L.sinks, src.sinks, (size_t)d.n_heads * 4, "sinks"))) return rc;
  L.sliding = src.sliding;
  gb_moe_desc md = *src.moe;
  md.device = d.device;
  md.max_tokens = (int32_t)D.rows_cap;
  md.ep_rank = 0;
  md.ep_size = 1;
  md.nccl_id = nullptr;
  if ((rc = gb_moe_create(&md, &L.moe))) return rc;
  if ((rc = gb_moe_set_graphs(L.moe, 0))) return rc;
  if (D.tc) {
    DEC_CUDA(make_bf16_map(L.map_qkv, L.wqkv, H, qn + 2 * kn, kLinearBoxRows), "q/k/v map");
    DEC_CUDA(make_bf16_map(L.map_o, L.wo, qn, H, kLinearBoxRows), "o map");
  }
  return GB_OK;
}

struct Piece {
  void** dst;
  size_t bytes;
};

int alloc_activations(Decoder& D) {
  const gb_decoder_desc& d = D.d;
  const size_t R = (size_t)D.rows_cap, H = d.hidden, B = d.max_batch;
  const size_t kmax = std::max<size_t>(H, (size_t)D.att_w);
  const size_t attn_rows = std::min<size_t>(R, kAttnRowsPerLaunch);
  Piece pieces[] = {
      {(void**)&D.h, R * H * 4},
      {(void**)&D.xn, R * H * 4},
      {(void**)&D.qkv, R * (size_t)D.qkv_w * 4},
      {(void**)&D.att, R * (size_t)D.att_w * 4},
      {(void**)&D.moe_out, R * H * 4},
      {(void**)&D.last, B * H * 4},
      {(void**)&D.logits, B * (size_t)d.vocab * 4},
      {(void**)&D.part, attn_rows * d.n_heads * dec::kSlots * (d.head_dim + 2) * 4},
      {(void**)&D.xh, D.tc ? R * kmax * 2 : 0},
      {(void**)&D.xl, D.tc ? R * kmax * 2 : 0},
      {(void**)&D.lin_part, D.tc ? (size_t)kLinearPartFloats * 4 : 0},
      {(void**)&D.next, B * 4},
      {(void**)&D.tok_buf, B * 4},
      {(void**)&D.d_pos, 4},
      {(void**)&D.err, 4},
      {(void**)&D.am_slot, B * 8},
      {(void**)&D.am_ticket, B * 4},
  };
  size_t total = 0;
  for (const Piece& p : pieces) total += (p.bytes + 255) & ~(size_t)255;
  int rc = dalloc((char**)&D.act_base, total, "decoder activations");
  if (rc) return rc;
  char* at = static_cast<char*>(D.act_base);
  for (const Piece& p : pieces) {
    *p.dst = p.bytes ? at : nullptr;
    at += (p.bytes + 255) & ~(size_t)255;
  }
  DEC_CUDA(cudaMemset(D.err, 0, 4), "decoder error word");
  DEC_CUDA(cudaMemset(D.am_slot, 0, B * 8), "greedy-token slots");
  DEC_CUDA(cudaMemset(D.am_ticket, 0, B * 4), "greedy-token tickets");
  if (D.tc) {
    DEC_CUDA(make_bf16_map(D.map_xh_h, D.xh, H, R, kLinearBoxRows), "activation map");
    DEC_CUDA(make_bf16_map(D.map_xl_h, D.xl, H, R, kLinearBoxRows), "activation map");
    DEC_CUDA(make_bf16_map(D.map_xh_a, D.xh, D.att_w, R, kLinearBoxRows), "activation map");
    DEC_CUDA(make_bf16_map(D.map_xl_a, D.xl, D.att_w, R, kLinearBoxRows), "activation map");
  }
  return GB_OK;
}

// out[p] (+)= W x[p] + bias for p < n: the tensor cores from kTcMinRows rows,
// else the CUDA-core kernel.
// Whether a linear layer of n rows runs on the tensor cores (its input then
// needs the bf16 hi / lo copies in D.xh / D.xl).
bool linear_tc(const Decoder& D, int n) { return D.tc && n >= kTcMinRows; }

// presplit: the producer of x already wrote its hi / lo copies.
int linear(Decoder& D, const float* x, int n, int K, const uint16_t* W, const void* map_w,
           int n_out, const float* bias, float* out, int out_stride, bool add, cudaStream_t st,
           bool presplit = false) {
  if (n <= 0) return GB_OK;
  if (D.tc && map_w && n >= kTcMinRows) {
    const bool kh = K == D.d.hidden;
    if (!presplit)
      DEC_CUDA(split_rows(x, nullptr, 1, K, n, D.xh, D.xl, st), "split activations");
    DEC_CUDA(launch_linear_tc(D.sm_count, map_w, kh ? D.map_xh_h : D.map_xh_a,
                              kh ? D.map_xl_h : D.map_xl_a, K, n_out, n, bias, out, out_stride,
                              add, D.err, D.lin_part, kLinearPartFloats, st),
             "tensor-core linear launch");
    return GB_OK;
  }
  if (n <= dec::kGemvRows) {
    // a warp per output row, every piece of the row requested up front
    const size_t smem = (size_t)n * K * 4;
    const unsigned grid = (unsigned)((n_out + dec::kGemvWarps - 1) / dec::kGemvWarps);
    const int per_lane = (K / 8 + 31) / 32;
    auto go = [&](auto kern) -> int {
      DEC_CUDA(set_smem_limit(kern, (size_t)dec::kGemvRows * K * 4), "GEMV shared memory");
      kern<<<grid, dec::kGemvWarps * 32, smem, st>>>(x, n, K, W, n_out, bias, out, out_stride,
                                                     add ? 1 : 0);
      DEC_CUDA(cudaGetLastError(), "GEMV launch");
      return GB_OK;
    };
    if (per_lane <= 4) return go(dec::gemv_rows_kernel<4>);
    if (per_lane <= 8) return go(dec::gemv_rows_kernel<8>);
    if (per_lane <= 12) return go(dec::gemv_rows_kernel<12>);
    return go(dec::gemv_rows_kernel<16>);
  }
  // shared memory for the rows staged at once
  const size_t smem = (size_t)std::min(n, dec::kGemvRows) * K * 4;
  DEC_CUDA(set_smem_limit(dec::linear_rows_kernel, (size_t)dec::kGemvRows * K * 4),
           "linear kernel shared memory");
  const unsigned grid = (unsigned)((n_out + 2 * dec::kGemvWarps - 1) / (2 * dec::kGemvWarps));
  dec::linear_rows_kernel<<<grid, dec::kGemvWarps * 32, smem, st>>>(x, n, K, W, n_out, bias, out,
                                                                    out_stride, add ? 1 : 0);
  DEC_CUDA(cudaGetLastError(), "linear kernel launch");
  return GB_OK;
}

int record(Decoder& D, size_t i, cudaStream_t st) {
  if (D.profiling) DEC_CUDA(cudaEventRecord(D.ev[i], st), "stage event");
  return GB_OK;
}

// Enqueues one forward of B x T tokens (positions from d_pos); logits of the
// last tokens into `logits`, greedy tokens into `next` (and out_tokens).
int run_step(Decoder& D, const int32_t* tokens, int B, int T, float* logits, int32_t* next,
             int32_t* out_tokens, cudaStream_t st) {
  const gb_decoder_desc& d = D.d;
  const int H = d.hidden, nh = d.n_heads, nkv = d.n_kv_heads, hd = d.head_dim;
  const int rows = B * T, rep = nh / nkv;
  const int64_t S = d.max_seq_len;
  const size_t layer_kv = (size_t)d.max_batch * nkv * S * hd;
  const float scale = (float)(1.0 / sqrt((double)hd));
  const size_t attn_smem =
      sizeof(float) * ((size_t)dec::kChunk * (hd + 1) + (size_t)dec::kChunk * hd +
                       (size_t)rep * hd + (size_t)rep * dec::kChunk);
  DEC_CUDA(set_smem_limit(dec::attn_partial_kernel, attn_smem), "attention shared memory");
  int rc;
  if ((rc = record(D, 0, st))) return rc;
  dec::embed_kernel<<<rows, 256, 0, st>>>(tokens, D.embed, H, d.vocab, D.h, D.err);
  DEC_CUDA(cudaGetLastError(), "embedding launch");
  for (int l = 0; l < d.n_layers; ++l) {
    DecLayer& L = D.layers[l];
    if (l > 0 && (rc = record(D, 2 * l, st))) return rc;
    // RMSNorm (after the previous layer's MoE residual), q/k/v, RoPE + cache
    const bool split = linear_tc(D, rows);  // producers write the hi / lo copies
    dec::add_rmsnorm_kernel<<<rows, dec::kNormThreads, 0, st>>>(
        D.h, l ? D.moe_out : nullptr, L.attn_norm, H, d.rms_eps, 1, 0, D.xn,
        split ? D.xh : nullptr, split ? D.xl : nullptr);
    DEC_CUDA(cudaGetLastError(), "norm launch");
    float* kc = D.kcache + (size_t)l * layer_kv;
    float* vc = D.vcache + (size_t)l * layer_kv;
    if (!split && rows <= dec::kGemvRows) {
      // q/k/v, RoPE and the cache store in one launch
      const size_t smem = (size_t)rows * H * 4;
      const int pairs = (nh + 2 * nkv) * (hd / 2);
      DEC_CUDA(set_smem_limit(dec::qkv_rope_gemv_kernel<8>, (size_t)dec::kGemvRows * H * 4),
               "q/k/v kernel shared memory");
      dec::qkv_rope_gemv_kernel<8><<<(pairs + dec::kGemvWarps - 1) / dec::kGemvWarps,
                                     dec::kGemvWarps * 32, smem, st>>>(
          D.xn, rows, H, L.wqkv, L.bqkv, nh, nkv, hd, T, D.rope_cos, D.rope_sin, D.d_pos, (int)S,
          D.qkv, kc, vc);
      DEC_CUDA(cudaGetLastError(), "q/k/v launch");
    } else {
      if ((rc = linear(D, D.xn, rows, H, L.wqkv, D.tc ? L.map_qkv : nullptr, D.qkv_w, L.bqkv,
                       D.qkv, D.qkv_w, false, st, split)))
        return rc;
      dec::rope_append_kernel<<<dim3(rows, nh + 2 * nkv), hd / 2, 0, st>>>(
          D.qkv, T, nh, nkv, hd, D.rope_cos, D.rope_sin, D.d_pos, (int)S, kc, vc);
      DEC_CUDA(cudaGetLastError(), "RoPE launch");
    }
    // key slots per query: every slot for a lone row; from 16 rows the rows
    // fill the GPU and two slots keep CTAs busy with several chunks each
    const int slots = rows >= 16 ? 2 : rows >= 4 ? 4 : dec::kSlots;
    for (int r0 = 0; r0 < rows; r0 += kAttnRowsPerLaunch) {
      const int nr = std::min(kAttnRowsPerLaunch, rows - r0);
      dec::attn_partial_kernel<<<dim3(slots, nkv, nr), rep * 32, attn_smem, st>>>(
          D.qkv, r0, T, nh, nkv, hd, D.d_pos, L.sliding, d.sliding_window, scale, (int)S, kc, vc,
          D.part);
      DEC_CUDA(cudaGetLastError(), "attention launch");
      const int warps = nr * nh;
      dec::attn_combine_kernel<<<(warps + 7) / 8, 256, 0, st>>>(
          D.part, nr, r0, nh, hd, slots, L.sinks, D.att, split ? D.xh : nullptr,
          split ? D.xl : nullptr);
      DEC_CUDA(cudaGetLastError(), "attention combine launch");
    }
    // o projection + residual, RMSNorm, MoE block (its residual joins the next norm)
    if ((rc = linear(D, D.att, rows, D.att_w, L.wo, D.tc ? L.map_o : nullptr, H, L.bo, D.h, H,
                     true, st, split)))
      return rc;
    dec::add_rmsnorm_kernel<<<rows, dec::kNormThreads, 0, st>>>(
        D.h, nullptr, L.post_norm, H, d.rms_eps, 1, 0, D.xn, nullptr, nullptr);
    DEC_CUDA(cudaGetLastError(), "norm launch");
    if ((rc = record(D, 2 * l + 1, st))) return rc;
    if ((rc = gb_moe_forward(L.moe, D.xn, rows, D.moe_out, st))) return rc;
  }
  const size_t head_ev = 2 * (size_t)d.n_layers;
  if ((rc = record(D, head_ev, st))) return rc;
  // last layer's MoE residual + final norm on each sequence's last token
  const bool split_head = linear_tc(D, B);
  dec::add_rmsnorm_kernel<<<B, dec::kNormThreads, 0, st>>>(
      D.h, D.moe_out, D.final_norm, H, d.rms_eps, T, T - 1, D.last,
      split_head ? D.xh : nullptr, split_head ? D.xl : nullptr);
  DEC_CUDA(cudaGetLastError(), "final norm launch");
  if ((rc = linear(D, D.last, B, H, D.lm_head, D.tc ? D.map_lm : nullptr, d.vocab, nullptr,
                   logits, d.vocab, false, st, split_head)))
    return rc;
  {
    const int per_cta = dec::kArgmaxThreads * dec::kArgmaxPerThread;
    dec::argmax_kernel<<<dim3((d.vocab + per_cta - 1) / per_cta, B), dec::kArgmaxThreads, 0, st>>>(
        logits, d.vocab, D.am_slot, D.am_ticket, next, out_tokens);
  }
  DEC_CUDA(cudaGetLastError(), "greedy token launch");
  return record(D, head_ev + 1, st);
}

int check_positions(Decoder& D, int B, int T, int64_t pos) {
  const gb_decoder_desc& d = D.d;
  if (B < 1 || B > d.max_batch)
    return set_error(GB_ERR_INVALID_ARG, "B = %d outside [1, %d]", B, d.max_batch);
  if (T < 1 || T > d.max_tokens)
    return set_error(GB_ERR_INVALID_ARG, "T = %d outside [1, %d]", T, d.max_tokens);
  if (pos != D.pos)
    return set_error(GB_ERR_INVALID_ARG, "pos %lld != the %lld positions cached (reset first)",
                     (long long)pos, (long long)D.pos);
  if (D.pos > 0 && B != D.batch)
    return set_error(GB_ERR_INVALID_ARG, "B = %d but the cache holds %d sequences", B, D.batch);
  return GB_OK;
}

}  // namespace
}  // namespace gb

struct gb_decoder {
  gb::Decoder* D;
};

extern "C" {

int gb_decoder_create(const gb_decoder_desc* desc, gb_decoder** out) {
  using namespace gb;
  if (!out) return set_error(GB_ERR_INVALID_ARG, "out is null");
  *out = nullptr;
  int rc = validate(desc);
  if (rc) return rc;
  Decoder* D = new Decoder();
  D->d = *desc;
  D->d.layers = nullptr;  // host pointers are not kept
  D->device = desc->device;
  DevScope ds(D->device);
  const gb_decoder_desc& d = D->d;
  D->qkv_w = (d.n_heads + 2 * d.n_kv_heads) * d.head_dim;
  D->att_w = d.n_heads * d.head_dim;
  D->rows_cap = (int64_t)d.max_batch * d.max_tokens;
  D->tc = d.hidden % 64 == 0 && D->att_w % 64 == 0 && tensor_map_encoder() != nullptr;
  auto fail = [&](int code) {
    const std::string msg = gb_last_error();
    release(D);
    set_error(code, "%s", msg.c_str());
    return code;
  };
  if (cudaDeviceGetAttribute(&D->sm_count, cudaDevAttrMultiProcessorCount, D->device) !=
      cudaSuccess)
    return fail(set_error(GB_ERR_CUDA, "query SM count on device %d", D->device));
  const size_t H = d.hidden, V = d.vocab;
  if ((rc = upload(&D->embed, desc->embed, V * H * 2, "embeddings"))) return fail(rc);
  if (desc->lm_head) {
    if ((rc = upload(&D->lm_head, desc->lm_head, V * H * 2, "LM head"))) return fail(rc);
  } else {
    D->lm_head = D->embed;
  }
  if ((rc = upload(&D->final_norm, desc->final_norm, H * 4, "final norm"))) return fail(rc);
  if (D->tc && make_bf16_map(D->map_lm, D->lm_head, H, V, kLinearBoxRows) != cudaSuccess)
    return fail(set_error(GB_ERR_CUDA, "LM head map"));
  {
    std::vector<float> c, s;
    rope_tables(d, c, s);
    if ((rc = upload(&D->rope_cos, c.data(), c.size() * 4, "RoPE cos"))) return fail(rc);
    if ((rc = upload(&D->rope_sin, s.data(), s.size() * 4, "RoPE sin"))) return fail(rc);
  }
  D->layers.resize(d.n_layers);
  for (int l = 0; l < d.n_layers; ++l)
    if ((rc = upload_layer(*D, desc->layers[l], D->layers[l]))) return fail(rc);
  const size_t kv = (size_t)d.n_layers * d.max_batch * d.n_kv_heads * d.max_seq_len *
                    d.head_dim * sizeof(float);
  if ((rc = dalloc(&D->kcache, kv, "K cache"))) return fail(rc);
  if ((rc = dalloc(&D->vcache, kv, "V cache"))) return fail(rc);
  if ((rc = alloc_activations(*D))) return fail(rc);
  D->ev.resize(2 * (size_t)d.n_layers + 2);
  for (auto& e : D->ev)
    if (cudaEventCreate(&e) != cudaSuccess) return fail(set_error(GB_ERR_CUDA, "create events"));
  if (cudaStreamCreateWithFlags(&D->cap, cudaStreamNonBlocking) != cudaSuccess)
    return fail(set_error(GB_ERR_CUDA, "create capture stream"));
  if (cudaDeviceSynchronize() != cudaSuccess)
    return fail(set_error(GB_ERR_CUDA, "decoder set-up: %s", cudaGetErrorString(cudaGetLastError())));
  *out = new gb_decoder{D};
  return GB_OK;
}

int gb_decoder_forward(gb_decoder* h, const int32_t* tokens_dev, int32_t B, int32_t T,
                       int64_t pos, float* logits_dev, int32_t* next_dev, void* stream) {
  using namespace gb;
  if (!h) return set_error(GB_ERR_INVALID_ARG, "handle is null");
  Decoder& D = *h->D;
  if (!tokens_dev) return set_error(GB_ERR_INVALID_ARG, "tokens_dev is null");
  int rc = check_positions(D, B, T, pos);
  if (rc) return rc;
  if (pos + T > D.d.max_seq_len)
    return set_error(GB_ERR_INVALID_ARG, "pos + T = %lld exceeds max_seq_len %d",
                     (long long)(pos + T), D.d.max_seq_len);
  if (logits_dev && (reinterpret_cast<uintptr_t>(logits_dev) & 15))
    return set_error(GB_ERR_INVALID_ARG, "logits_dev must be 16-byte aligned");
  DevScope ds(D.device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  dec::set_int_kernel<<<1, 1, 0, st>>>(D.d_pos, (int)pos);
  DEC_CUDA(cudaGetLastError(), "position launch");
  if ((rc = run_step(D, tokens_dev, B, T, logits_dev ? logits_dev : D.logits,
                     next_dev ? next_dev : D.next, nullptr, st)))
    return rc;
  D.timed = D.profiling;
  D.pos = pos + T;
  D.batch = B;
  return GB_OK;
}

int gb_decoder_generate(gb_decoder* h, const int32_t* tokens_dev, int32_t B, int64_t pos,
                        int32_t n_steps, int32_t* out_dev, void* stream) {
  using namespace gb;
  if (!h) return set_error(GB_ERR_INVALID_ARG, "handle is null");
  Decoder& D = *h->D;
  if (!tokens_dev || !out_dev) return set_error(GB_ERR_INVALID_ARG, "tokens or out is null");
  if (n_steps < 0) return set_error(GB_ERR_INVALID_ARG, "n_steps < 0");
  int rc = check_positions(D, B, 1, pos);
  if (rc) return rc;
  if (pos + n_steps > D.d.max_seq_len)
    return set_error(GB_ERR_INVALID_ARG, "pos + n_steps = %lld exceeds max_seq_len %d",
                     (long long)(pos + n_steps), D.d.max_seq_len);
  if (n_steps == 0) return GB_OK;
  DevScope ds(D.device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  DEC_CUDA(cudaMemcpyAsync(D.tok_buf, tokens_dev, sizeof(int32_t) * B, cudaMemcpyDeviceToDevice,
                           st),
           "copy tokens");
  dec::set_int_kernel<<<1, 1, 0, st>>>(D.d_pos, (int)pos);
  DEC_CUDA(cudaGetLastError(), "position launch");
  GenGraph* g = nullptr;
  for (auto& x : D.gens)
    if (x.B == B) g = &x;
  int step = 0;
  auto eager_step = [&]() -> int {
    int r = run_step(D, D.tok_buf, B, 1, D.logits, D.tok_buf, nullptr, st);
    if (r) return r;
    dec::advance_kernel<<<1, 1, 0, st>>>(D.d_pos, 1);
    DEC_CUDA(cudaGetLastError(), "advance launch");
    DEC_CUDA(cudaMemcpyAsync(out_dev + (size_t)step * B, D.tok_buf, sizeof(int32_t) * B,
                             cudaMemcpyDeviceToDevice, st),
             "copy tokens out");
    ++step;
    return GB_OK;
  };
  if (D.profiling) {  // eager steps, so the stage events time them
    while (step < n_steps)
      if ((rc = eager_step())) return rc;
    D.timed = true;
  } else {
    if (!g) {
      // the first step runs eagerly (it also sets every kernel's attributes
      // outside the capture), then the step is captured once for this B
      if ((rc = eager_step())) return rc;
      DEC_CUDA(cudaStreamSynchronize(st), "synchronise before capture");
      DEC_CUDA(cudaStreamBeginCapture(D.cap, cudaStreamCaptureModeThreadLocal), "begin capture");
      int r = run_step(D, D.tok_buf, B, 1, D.logits, D.tok_buf, nullptr, D.cap);
      if (!r) {
        dec::advance_kernel<<<1, 1, 0, D.cap>>>(D.d_pos, 1);
        if (cudaGetLastError() != cudaSuccess) r = set_error(GB_ERR_CUDA, "advance launch");
      }
      cudaGraph_t graph = nullptr;
      const cudaError_t ce = cudaStreamEndCapture(D.cap, &graph);
      if (r) {
        if (graph) cudaGraphDestroy(graph);
        return r;
      }
      if (ce != cudaSuccess) return set_error(GB_ERR_CUDA, "end capture: %s", cudaGetErrorString(ce));
      cudaGraphExec_t exec = nullptr;
      const cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
      cudaGraphDestroy(graph);
      if (ie != cudaSuccess)
        return set_error(GB_ERR_CUDA, "instantiate decode graph: %s", cudaGetErrorString(ie));
      D.gens.push_back(GenGraph{B, exec});
      g = &D.gens.back();
    }
    for (; step < n_steps; ++step) {
      DEC_CUDA(cudaGraphLaunch(g->exec, st), "decode graph launch");
      DEC_CUDA(cudaMemcpyAsync(out_dev + (size_t)step * B, D.tok_buf, sizeof(int32_t) * B,
                               cudaMemcpyDeviceToDevice, st),
               "copy tokens out");
    }
  }
  D.pos = pos + n_steps;
  D.batch = B;
  return GB_OK;
}

int gb_decoder_reset(gb_decoder* h) {
  if (!h) return gb::set_error(GB_ERR_INVALID_ARG, "handle is null");
  h->D->pos = 0;
  h->D->batch = 0;
  return GB_OK;
}

int gb_decoder_set_profiling(gb_decoder* h, int32_t enable) {
  if (!h) return gb::set_error(GB_ERR_INVALID_ARG, "handle is null");
  h->D->profiling = enable != 0;
  h->D->timed = false;
  return GB_OK;
}

int gb_decoder_stage_times(gb_decoder* h, float ms_out[3], void* stream) {
  using namespace gb;
  if (!h || !ms_out) return set_error(GB_ERR_INVALID_ARG, "null argument");
  Decoder& D = *h->D;
  if (!D.timed) return set_error(GB_ERR_INVALID_ARG, "no profiled forward since profiling was enabled");
  DevScope ds(D.device);
  DEC_CUDA(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "synchronise");
  const int L = D.d.n_layers;
  float attn = 0.0f, moe = 0.0f, t = 0.0f;
  for (int l = 0; l < L; ++l) {
    DEC_CUDA(cudaEventElapsedTime(&t, D.ev[2 * l], D.ev[2 * l + 1]), "stage time");
    attn += t;
    DEC_CUDA(cudaEventElapsedTime(&t, D.ev[2 * l + 1], D.ev[l + 1 < L ? 2 * (l + 1) : 2 * L]),
             "stage time");
    moe += t;
  }
  DEC_CUDA(cudaEventElapsedTime(&t, D.ev[2 * L], D.ev[2 * L + 1]), "stage time");
  ms_out[0] = attn;
  ms_out[1] = moe;
  ms_out[2] = t;
  return GB_OK;
}

int gb_decoder_device_status(gb_decoder* h, void* stream) {
  using namespace gb;
  if (!h) return set_error(GB_ERR_INVALID_ARG, "handle is null");
  Decoder& D = *h->D;
  DevScope ds(D.device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  DEC_CUDA(cudaStreamSynchronize(st), "synchronise");
  int32_t bits = 0;
  DEC_CUDA(cudaMemcpy(&bits, D.err, 4, cudaMemcpyDeviceToHost), "read decoder error word");
  DEC_CUDA(cudaMemset(D.err, 0, 4), "clear decoder error word");
  for (auto& L : D.layers) {
    const int rc = gb_moe_device_status(L.moe, stream);
    if (rc) return rc;
  }
  if (bits & 2) return set_error(GB_ERR_TIMEOUT, "a tensor-core pipeline wait timed out");
  if (bits & 1) return set_error(GB_ERR_INVALID_ARG, "a token id was outside [0, vocab)");
  return GB_OK;
}

int gb_decoder_destroy(gb_decoder* h) {
  if (!h) return GB_OK;
  gb::release(h->D);
  delete h;
  return GB_OK;
}

}  // extern "C"
