// decode_gemv.cu -- grouped MXFP4 expert GEMV for decode-sized batches.
//
// Reference math: gpt_oss.rs:189-221 (gate_up + bias, interleaved split,
// clamped SwiGLU, down + bias), gpt_oss_q.rs:194-246.
//
// HBM-bound: every weight byte of an active expert is read once per forward
// and used by only a few tokens, so the kernel is built to keep many bytes in
// flight while keeping the per-element instruction count low.
//
//  * One CTA = 4 warps = 64 weight rows of one active expert; a warp walks 8
//    row pairs (gate/up pairs for gate_up).  Each warp stages its next three
//    row pairs (MXFP4 blocks and E8M0 bytes, ~9 KB) in its own shared-memory
//    ring with 16-byte cp.async copies, lane l taking blocks l, l+32, l+64 of
//    a row, so every copy instruction moves 512 contiguous bytes and nothing
//    in flight occupies registers.
//  * Each block is decoded in registers (hardware E2M1 -> f16x2, then f32) and
//    dotted with up to TC tokens' activations, staged once per CTA in shared
//    memory with a 36-float pitch per 32-element block (conflict-free 128-bit
//    reads); four independent FMA chains per block.  The block sum is scaled
//    by its E8M0 scale, and a butterfly folds the 32 lanes of each row.
#include <algorithm>

#include "common.cuh"
#include "moe_internal.h"

namespace gb {
namespace {

constexpr int kDecWarps = 4;
constexpr int kPairs = 8;                        // row pairs per warp
constexpr int kRowsPerCta = kDecWarps * 2 * kPairs;
constexpr int kLoadsPerRow = 3;                  // 16-byte loads per lane per row (K <= 3072)
constexpr int kBlockPitch = 36;                  // floats per staged 32-element block (+4 pad)
constexpr int kRing = 4;                         // row-pair slots per warp (3 in flight)

enum Mode { GATE_UP = 0, DOWN = 1 };

struct DecArgs {
  const float* in;         // GATE_UP: x [T, K] (rows gathered through perm); DOWN: h [T*k, K]
  int K;
  int rows;                // weight rows per expert (2I or H)
  int top_k;
  const uint8_t* blocks;   // [E_loc][rows][K/32][16]
  const uint8_t* scales;   // [E_loc][rows][sp]
  int sp;
  const float* bias;       // [E_loc][rows] or null
  float zero_scale;
  const int32_t* counts;
  const int32_t* offsets;
  const int32_t* active;
  const int32_t* meta;     // [0] active experts
  const int32_t* perm;
  int e_begin;
  int act_kind;
  float clamp;  // act_clamp
  float limit;
  const int32_t* out_rows;  // DOWN: output row of each position (null: the position)
  float* out;
  int out_stride;
};

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "l"(gmem_src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int MODE, int TC>
__global__ void __launch_bounds__(kDecWarps * 32) decode_rows_kernel(const DecArgs a) {
  extern __shared__ __align__(16) uint8_t smem_b[];
  const int K = a.K;
  const int NB = K >> 5;
  const int row_bytes = NB * 16;
  const int slot_bytes = 2 * (row_bytes + a.sp);  // a row pair: blocks then scales
  const int xstride = NB * kBlockPitch;           // floats per staged token row
  float* xs = reinterpret_cast<float*>(smem_b);   // [TC][NB][kBlockPitch]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* ring = smem_b + (size_t)TC * xstride * sizeof(float) +
                  (size_t)warp * kRing * slot_bytes;  // this warp's [kRing] pair slots

  const int slot = blockIdx.y;
  if (slot >= a.meta[0]) return;
  const int e = a.active[slot];
  const int le = e - a.e_begin;
  const int n = a.counts[e];
  const int p0 = a.offsets[e];
  const int row0 = blockIdx.x * kRowsPerCta + warp * 2 * kPairs;
  const int npairs = max(0, min(kPairs, (a.rows - row0) >> 1));
  const int64_t erow = (int64_t)le * a.rows;

  // Copy row pair p into ring slot (p % kRing); always commits a group so the
  // wait counts stay aligned (an out-of-range pair commits an empty group).
  auto fetch_pair = [&](int p) {
    if (p < npairs) {
      uint8_t* dst = ring + (p % kRing) * slot_bytes;
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int64_t row = erow + row0 + 2 * p + r;
        const uint8_t* rb = a.blocks + row * row_bytes;
        for (int c = lane; c < NB; c += 32) cp_async16(dst + r * row_bytes + c * 16, rb + c * 16);
        const uint8_t* rs = a.scales + row * a.sp;
        for (int c = lane; c < (a.sp >> 4); c += 32)
          cp_async16(dst + 2 * row_bytes + r * a.sp + c * 16, rs + c * 16);
      }
    }
    cp_async_commit();
  };

  for (int c0 = 0; c0 < n; c0 += TC) {
    const int nc = min(TC, n - c0);
    if (c0 > 0) __syncthreads();
#pragma unroll
    for (int p = 0; p < kRing - 1; ++p) fetch_pair(p);
    for (int j = 0; j < nc; ++j) {
      const float* src = MODE == GATE_UP
                             ? a.in + (int64_t)(a.perm[p0 + c0 + j] / a.top_k) * K
                             : a.in + (int64_t)(p0 + c0 + j) * K;
      for (int k4 = threadIdx.x; k4 < (K >> 2); k4 += blockDim.x) {
        const int k = k4 << 2;
        *reinterpret_cast<float4*>(xs + j * xstride + (k >> 5) * kBlockPitch + (k & 31)) =
            reinterpret_cast<const float4*>(src)[k4];
      }
    }
    __syncthreads();

    for (int p = 0; p < npairs; ++p) {
      fetch_pair(p + kRing - 1);
      cp_async_wait<kRing - 1>();  // pair p has landed (this lane's copies)
      __syncwarp();                // ... and every lane's
      const uint8_t* sl = ring + (p % kRing) * slot_bytes;

      float acc[2][TC];
#pragma unroll
      for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int t = 0; t < TC; ++t) acc[r][t] = 0.0f;
#pragma unroll
      for (int r = 0; r < 2; ++r) {
#pragma unroll
        for (int i = 0; i < kLoadsPerRow; ++i) {
          const int b = lane + 32 * i;
          if (b >= NB) continue;
          const uint4 q = *reinterpret_cast<const uint4*>(sl + r * row_bytes + b * 16);
          const float sc = e8m0_scale(sl[2 * row_bytes + r * a.sp + b], a.zero_scale);
          float v[32];
          decode_block_f32(q, v);
#pragma unroll
          for (int t = 0; t < TC; ++t) {
            if (t < nc) {
              const float4* x4 = reinterpret_cast<const float4*>(xs + t * xstride + b * kBlockPitch);
              float f0 = 0.0f, f1 = 0.0f, f2 = 0.0f, f3 = 0.0f;
#pragma unroll
              for (int q4 = 0; q4 < 8; ++q4) {
                const float4 xv = x4[q4];
                f0 = __fmaf_rn(xv.x, v[4 * q4], f0);
                f1 = __fmaf_rn(xv.y, v[4 * q4 + 1], f1);
                f2 = __fmaf_rn(xv.z, v[4 * q4 + 2], f2);
                f3 = __fmaf_rn(xv.w, v[4 * q4 + 3], f3);
              }
              acc[r][t] =
                  __fmaf_rn(__fadd_rn(__fadd_rn(f0, f1), __fadd_rn(f2, f3)), sc, acc[r][t]);
            }
          }
        }
      }
      __syncwarp();  // slot p % kRing is refilled by a later fetch
      const int row = row0 + 2 * p;  // gate (GATE_UP) / first output row (DOWN)
#pragma unroll
      for (int t = 0; t < TC; ++t) {
        if (t >= nc) break;
        const float s0 = warp_sum_butterfly(acc[0][t]);
        const float s1 = warp_sum_butterfly(acc[1][t]);
        if (lane == 0) {
          const int64_t pos = p0 + c0 + t;
          if (MODE == GATE_UP) {
            float g = s0, u = s1;
            if (a.bias) {
              g = __fadd_rn(g, a.bias[erow + row]);
              u = __fadd_rn(u, a.bias[erow + row + 1]);
            }
            a.out[pos * a.out_stride + (row >> 1)] =
                act_apply(a.act_kind, g, u, a.limit, a.clamp);
          } else {
            float y0 = s0, y1 = s1;
            if (a.bias) {
              y0 = __fadd_rn(y0, a.bias[erow + row]);
              y1 = __fadd_rn(y1, a.bias[erow + row + 1]);
            }
            const int64_t orow = a.out_rows ? a.out_rows[pos] : pos;
            a.out[orow * a.out_stride + row] = y0;
            a.out[orow * a.out_stride + row + 1] = y1;
          }
        }
      }
    }
    cp_async_wait<0>();
  }
}

template <int MODE, int TC>
cudaError_t launch_dec(const Moe& m, const Groups& g, const DecArgs& a, cudaStream_t st) {
  (void)m;
  if (g.max_active <= 0) return cudaSuccess;
  dim3 grid((unsigned)((a.rows + kRowsPerCta - 1) / kRowsPerCta), (unsigned)g.max_active);
  const size_t smem = (size_t)TC * (a.K / 32) * kBlockPitch * sizeof(float) +
                      (size_t)kDecWarps * kRing * 2 * ((a.K / 32) * 16 + a.sp);
  auto kern = decode_rows_kernel<MODE, TC>;
  cudaError_t err = set_smem_limit(kern, smem);
  if (err != cudaSuccess) return err;
  kern<<<grid, kDecWarps * 32, smem, st>>>(a);
  return cudaGetLastError();
}

DecArgs base_args(const Moe& m, const Groups& g) {
  const gb_moe_desc& d = m.desc;
  DecArgs a{};
  a.top_k = g.perm_div;
  a.zero_scale = m.w.zero_scale;
  a.counts = g.counts;
  a.offsets = g.offsets;
  a.active = g.active;
  a.meta = g.meta;
  a.perm = g.perm;
  a.e_begin = m.e_begin;
  a.act_kind = d.act_kind;
  a.clamp = d.act_clamp;
  a.limit = d.swiglu_limit;
  return a;
}

}  // namespace

bool decode_supported(const Moe& m) {
  const gb_moe_desc& d = m.desc;
  // whole row pairs; a row is at most 3 x 32 blocks (K <= 3072)
  return d.weight_format != GB_FMT_Q4_K && d.hidden % 64 == 0 && d.inter % 64 == 0 &&
         d.hidden <= 3072 && d.inter <= 3072;
}

// Tokens per expert decide the template: one token shares nothing, so the
// single-token variant keeps its shared-memory footprint minimal.
cudaError_t launch_decode_gate_up(const Moe& m, const Groups& g, const float* x, ExpertBufs& eb,
                                  cudaStream_t st) {
  const gb_moe_desc& d = m.desc;
  DecArgs a = base_args(m, g);
  a.in = x;
  a.K = d.hidden;
  a.rows = 2 * d.inter;
  a.blocks = m.w.gu_blocks;
  a.scales = m.w.gu_scales;
  a.sp = m.w.sp_h;
  a.bias = m.w.gu_bias;
  a.out = eb.h;
  a.out_stride = d.inter;
  return g.max_per_expert <= 1 ? launch_dec<GATE_UP, 1>(m, g, a, st) : launch_dec<GATE_UP, 4>(m, g, a, st);
}

cudaError_t launch_decode_down(const Moe& m, const Groups& g, ExpertBufs& eb, cudaStream_t st) {
  const gb_moe_desc& d = m.desc;
  DecArgs a = base_args(m, g);
  a.in = eb.h;
  a.K = d.inter;
  a.rows = d.hidden;
  a.blocks = m.w.dn_blocks;
  a.scales = m.w.dn_scales;
  a.sp = m.w.sp_i;
  a.bias = m.w.dn_bias;
  a.out_rows = g.out_rows;
  a.out = eb.y;
  a.out_stride = d.hidden;
  return g.max_per_expert <= 1 ? launch_dec<DOWN, 1>(m, g, a, st) : launch_dec<DOWN, 4>(m, g, a, st);
}

}  // namespace gb
