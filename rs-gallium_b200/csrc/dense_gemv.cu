// dense_gemv.cu -- grouped dense expert products on CUDA cores: the generic
// gallium-core MoEFFN (crates/gallium-core/src/ffn.rs:72-166), whose experts
// are GatedFFN blocks (ffn.rs:30-67) with dense gate / up / down weights in the
// model's dtype, and its optional shared expert over all tokens.
//
//   gate_up: h[p, i] = clamp(act(x_p . Wg[i]), -c, c) * (x_p . Wu[i])
//            (clamp only when c > 0; act = SiLU, GELU (erf), GELU (tanh), ReLU)
//   down:    y[p, o] = h_p . Wd[o]
//
// dense_rows_kernel<MODE, TC, W>: one CTA per (active expert, tile of rows); a
// warp owns two weight rows (GATE_UP: gate row i and up row i, stored
// interleaved as rows 2i and 2i + 1; DOWN: rows 2p, 2p + 1).  The expert's rows stream through shared memory TC at a time; lane
// l reads 16-byte pieces l, l + 32, ... of both weight rows (bf16 or f32, as
// stored; exact in f32) and accumulates f32 FMAs, folded by a butterfly.  For
// decode-sized groups (one chunk) each weight byte is read from HBM once; more
// chunks re-read the expert's rows from L2.
#include <math.h>

#include <algorithm>

#include "common.cuh"
#include "moe_internal.h"
#include "ptx.cuh"

namespace gb {
namespace {

constexpr int kWarps = 8;
enum Mode { GATE_UP = 0, DOWN = 1 };

__device__ __forceinline__ void widen(const uint4& q, float (&v)[8], const __nv_bfloat16*) {
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

__device__ __forceinline__ void widen(const uint4& q, float (&v)[8], const float*) {
  v[0] = __uint_as_float(q.x);
  v[1] = __uint_as_float(q.y);
  v[2] = __uint_as_float(q.z);
  v[3] = __uint_as_float(q.w);
}

// identity != 0: the shared expert: `identity` positions, position p = input
// row p, weights at w0 directly (one expert).  GATE_UP: w0 holds 2 n_rows
// interleaved gate / up rows per expert; DOWN: n_rows rows.
template <int MODE, int TC, typename W>
__global__ void __launch_bounds__(kWarps * 32)
    dense_rows_kernel(const float* __restrict__ in, int K_in, int n_rows, int top_k,
                      const W* __restrict__ w0,
                      const int32_t* __restrict__ counts, const int32_t* __restrict__ offsets,
                      const int32_t* __restrict__ active, const int32_t* __restrict__ meta,
                      const int32_t* __restrict__ perm, int e_begin, int act_kind, float clamp,
                      const int32_t* __restrict__ out_rows, float* __restrict__ out,
                      int out_stride, int identity) {
  extern __shared__ float xs[];  // [TC][K_in]
  pdl_trigger();
  pdl_wait();
  int le, n, p0;
  if (identity) {
    if (blockIdx.y > 0) return;
    le = 0;
    n = identity;
    p0 = 0;
  } else {
    const int slot = blockIdx.y;
    if (slot >= meta[0]) return;
    const int e = active[slot];
    le = e - e_begin;
    n = counts[e];
    p0 = offsets[e];
  }
  constexpr int EPQ = 16 / (int)sizeof(W);  // weights per 16-byte piece
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pair = blockIdx.x * kWarps + warp;
  // GATE_UP: gate row `pair` and up row `pair` (stored rows 2 pair, 2 pair + 1
  // of the expert's 2 n_rows); DOWN: rows 2 pair, 2 pair + 1
  const int64_t r0 = MODE == GATE_UP ? pair : 2 * pair;
  const bool valid = MODE == GATE_UP ? pair < n_rows : r0 < n_rows;
  const bool valid1 = MODE == GATE_UP ? valid : r0 + 1 < n_rows;
  const W* row_a;
  const W* row_b;
  if (MODE == GATE_UP) {
    row_a = w0 + ((int64_t)le * 2 * n_rows + (valid ? 2 * r0 : 0)) * K_in;
    row_b = row_a + K_in;
  } else {
    row_a = w0 + ((int64_t)le * n_rows + (valid ? r0 : 0)) * K_in;
    row_b = w0 + ((int64_t)le * n_rows + (valid1 ? r0 + 1 : 0)) * K_in;
  }
  const int npieces = K_in / EPQ;

  for (int c0 = 0; c0 < n; c0 += TC) {
    const int nc = min(TC, n - c0);
    __syncthreads();
    for (int j = 0; j < nc; ++j) {
      int64_t src_row;
      if (identity || MODE == DOWN) src_row = p0 + c0 + j;
      else src_row = perm[p0 + c0 + j] / top_k;
      const float4* src = reinterpret_cast<const float4*>(in + src_row * K_in);
      float4* dst = reinterpret_cast<float4*>(xs + j * K_in);
      for (int k4 = threadIdx.x; k4 < (K_in >> 2); k4 += blockDim.x) dst[k4] = src[k4];
    }
    __syncthreads();
    if (!valid) continue;
    float acc[2][TC];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int j = 0; j < TC; ++j) acc[r][j] = 0.0f;
    for (int q = lane; q < npieces; q += 32) {
      float va[8], vb[8];
      widen(ld_stream_u4(row_a + (int64_t)q * EPQ), va, (const W*)nullptr);
      widen(ld_stream_u4(row_b + (int64_t)q * EPQ), vb, (const W*)nullptr);
#pragma unroll
      for (int j = 0; j < TC; ++j) {
        if (j < nc) {
          const float* xj = xs + j * K_in + q * EPQ;
#pragma unroll
          for (int el = 0; el < EPQ; ++el) {
            acc[0][j] = __fmaf_rn(xj[el], va[el], acc[0][j]);
            acc[1][j] = __fmaf_rn(xj[el], vb[el], acc[1][j]);
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
          out[pos * out_stride + pair] = __fmul_rn(act_generic(act_kind, s0, clamp), s1);
        } else {
          const int64_t orow = out_rows ? out_rows[pos] : pos;
          out[orow * out_stride + r0] = s0;
          if (valid1) out[orow * out_stride + r0 + 1] = s1;
        }
      }
    }
  }
}

template <int MODE, typename W>
cudaError_t launch_dense(const Moe& m, const Groups* g, int identity, const float* in, int K_in,
                         int n_rows, const void* w0, float* out, int out_stride, int max_active,
                         int64_t max_per_expert, cudaStream_t st) {
  const gb_moe_desc& d = m.desc;
  if (max_active <= 0) return cudaSuccess;
  const int units = MODE == GATE_UP ? n_rows : (n_rows + 1) / 2;
  dim3 grid((unsigned)((units + kWarps - 1) / kWarps), (unsigned)max_active);
  const bool big = max_per_expert > 4;
  const size_t smem = (size_t)(big ? 8 : 4) * K_in * sizeof(float);
  auto go = [&](auto kern) -> cudaError_t {
    cudaError_t err = set_smem_limit(kern, smem);
    if (err != cudaSuccess) return err;
    return launch_pdl(kern, grid, dim3(kWarps * 32), smem, st, in, K_in, n_rows,
                      g ? g->perm_div : 1, static_cast<const W*>(w0),
                      g ? g->counts : nullptr, g ? g->offsets : nullptr,
                      g ? g->active : nullptr, g ? (const int32_t*)g->meta : nullptr,
                      g ? g->perm : nullptr, m.e_begin, d.act_kind, d.act_clamp,
                      (MODE == DOWN && g) ? g->out_rows : nullptr, out, out_stride, identity);
  };
  return big ? go(dense_rows_kernel<MODE, 8, W>) : go(dense_rows_kernel<MODE, 4, W>);
}

template <int MODE>
cudaError_t launch_dense_any(const Moe& m, const Groups* g, int identity, const float* in,
                             int K_in, int n_rows, const void* w0, float* out, int out_stride,
                             int max_active, int64_t max_per_expert, cudaStream_t st) {
  if (m.w.dense_bf16)
    return launch_dense<MODE, __nv_bfloat16>(m, g, identity, in, K_in, n_rows, w0, out,
                                             out_stride, max_active, max_per_expert, st);
  return launch_dense<MODE, float>(m, g, identity, in, K_in, n_rows, w0, out, out_stride,
                                   max_active, max_per_expert, st);
}

// Stored rows [row0 + i * step] (i < nrows) of K values -> f32 [nrows][K].
template <typename W>
__global__ void widen_rows_kernel(const W* __restrict__ w, int64_t row0, int step, int nrows,
                                  int K, float* __restrict__ out) {
  const int64_t n = (int64_t)nrows * K;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / K, k = i - r * K;
    const W v = w[(row0 + r * step) * K + k];
    if constexpr (sizeof(W) == 2)
      out[i] = __bfloat162float(v);
    else
      out[i] = v;
  }
}

}  // namespace

cudaError_t launch_dense_gate_up(const Moe& m, const Groups& g, const float* x, ExpertBufs& eb,
                                 cudaStream_t st) {
  const gb_moe_desc& d = m.desc;
  return launch_dense_any<GATE_UP>(m, &g, 0, x, d.hidden, d.inter, m.w.dense_gu, eb.h, d.inter,
                                   g.max_active, g.max_per_expert, st);
}

cudaError_t launch_dense_down(const Moe& m, const Groups& g, ExpertBufs& eb, cudaStream_t st) {
  const gb_moe_desc& d = m.desc;
  return launch_dense_any<DOWN>(m, &g, 0, eb.h, d.inter, d.hidden, m.w.dense_down, eb.y, d.hidden,
                                g.max_active, g.max_per_expert, st);
}

cudaError_t launch_shared_expert(const Moe& m, const float* x, int64_t T, float* h, float* y,
                                 cudaStream_t st) {
  const gb_moe_desc& d = m.desc;
  if (T <= 0) return cudaSuccess;
  cudaError_t e = launch_dense_any<GATE_UP>(m, nullptr, (int)T, x, d.hidden, d.shared_inter,
                                            m.w.sh_gu, h, d.shared_inter, 1, T, st);
  if (e != cudaSuccess) return e;
  return launch_dense_any<DOWN>(m, nullptr, (int)T, h, d.shared_inter, d.hidden, m.w.sh_down, y,
                                d.hidden, 1, T, st);
}

cudaError_t launch_dense_dequant(const Moe& m, int which, int local_expert, float* out,
                                 cudaStream_t st) {
  const gb_moe_desc& d = m.desc;
  const int H = d.hidden, I = d.inter;
  const void* w;
  int64_t row0;
  int step, nrows, K;
  if (which == 2) {
    w = m.w.dense_down;
    row0 = (int64_t)local_expert * H;
    step = 1;
    nrows = H;
    K = I;
  } else {
    w = m.w.dense_gu;
    row0 = (int64_t)local_expert * 2 * I + which;
    step = 2;
    nrows = I;
    K = H;
  }
  const unsigned blocks = (unsigned)std::min<int64_t>(((int64_t)nrows * K + 255) / 256, 4096);
  if (m.w.dense_bf16)
    widen_rows_kernel<<<blocks, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(w), row0, step,
                                              nrows, K, out);
  else
    widen_rows_kernel<<<blocks, 256, 0, st>>>(static_cast<const float*>(w), row0, step, nrows, K,
                                              out);
  return cudaGetLastError();
}

}  // namespace gb
