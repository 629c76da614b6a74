// decode_fused.cu -- the whole MoE layer in one cooperative launch for
// decode-sized batches (T <= 8 tokens, T*k <= 32 token-expert entries), MXFP4
// experts in the repacked row layout (safetensors or GGUF), one GPU.
//
// Reference math: gpt_oss.rs:166-231 and gpt_oss_q.rs:165-269 (router,
// top-k, gate_up + bias, clamped SwiGLU, down + bias, weighted sum).
//
// At these sizes the separate kernels of the layer spend most of their time
// starting up and waiting on each other; here one persistent grid (every CTA
// resident, one per SM) runs five phases separated by grid barriers (a
// counter and a generation word in global memory, every wait bounded):
//   1. router logits: the token rows staged in shared memory, one warp per
//      expert with its router row loaded into registers at once, the router
//      kernel's reduction order (lane-strided FMAs, butterfly, bias), so the
//      logits are bit-identical to it;
//   2. (no barrier after) every CTA selects the top-k of every token from the
//      logits with the router's select_topk and builds the same grouping
//      (experts ascending, tokens ascending) in shared memory;
//   3. gate_up: the active experts' 2I rows as row pairs, a contiguous range
//      of pairs per CTA (so a CTA stages the inputs of one or two experts) and
//      a contiguous run per warp; each warp streams its pairs through a
//      shared-memory ring with 16-byte cp.async copies (MXFP4 blocks and E8M0
//      bytes), decodes them in registers and dots them with the expert's
//      staged token rows (the token count a template parameter, 1, 2, 4 or
//      8, so the unrolled body stays small); bias + activation -> h;
//   4. down: the same over the H rows with the staged h rows -> y (+ bias);
//   5. combine: out[t] = sum over ranks of w * y, in the reference's order.
// Phases 3 and 4 read each weight byte from HBM once; the grid barriers cost
// about a microsecond each.
#include <algorithm>

#include "common.cuh"
#include "moe_internal.h"
#include "ptx.cuh"
#include "route_select.cuh"

namespace gb {
namespace {

constexpr int kFWarps = 16;
constexpr int kFThreads = kFWarps * 32;
constexpr int kMaxTok = 8;      // tokens of one forward
constexpr int kStageTok = 4;    // input rows staged at a time per expert
constexpr int kMaxPos = 32;     // token-expert entries
constexpr int kMaxK = 8;        // top-k
constexpr int kRing = 3;        // row-pair slots per warp (2 in flight)
constexpr int kPitch = 36;      // floats per staged 32-element block (+4 pad)
constexpr int kMaxNB = 96;      // 32-element blocks per row (K <= 3072)

struct FusedArgs {
  const float* x;
  int T, H, I, E, K;
  int router_kind;
  const float* rw;        // [E][H] f32
  const float* rb;        // [E] or null
  const float* sel_bias;  // [E] or null
  float* logits;          // [T][E]
  int32_t* idx_out;       // [T][K] (written by CTA 0, for inspection)
  float* w_out;
  const uint8_t* gu_blocks;  // [E][2I][H/32][16]
  const uint8_t* gu_scales;  // [E][2I][sp_h]
  int sp_h;
  const float* gu_bias;      // [E][2I] or null
  const uint8_t* dn_blocks;  // [E][H][I/32][16]
  const uint8_t* dn_scales;  // [E][H][sp_i]
  int sp_i;
  const float* dn_bias;      // [E][H] or null
  float zero_scale;
  int act_kind;
  float limit, clamp;
  float* h;    // [kMaxPos][I]
  float* y;    // [kMaxPos][H]
  float* out;  // [T][H]
  int expert_order;
  unsigned* bar;  // [0] arrivals, [1] generation
  int* err;       // error word (bit 2: a wait ran out)
  uint64_t wait_ns;
};

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "l"(gmem_src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Grid barrier over every CTA of the (cooperative) launch; false when a wait
// ran out or another CTA gave up (then every CTA leaves the kernel).
__device__ bool grid_barrier(const FusedArgs& a, int* s_ok) {
  __syncthreads();
  if (threadIdx.x == 0) {
    volatile unsigned* gen = a.bar + 1;
    const unsigned g = *gen;
    __threadfence();
    if (atomicAdd(a.bar, 1u) == gridDim.x - 1) {
      a.bar[0] = 0;
      __threadfence();
      atomicAdd(a.bar + 1, 1u);
    } else {
      const uint64_t t0 = globaltimer();
      while (*gen == g) {
        if ((*reinterpret_cast<volatile int*>(a.err) & 2) || globaltimer() - t0 > a.wait_ns) {
          atomicOr(a.err, 2);
          *s_ok = 0;
          break;
        }
        __nanosleep(64);
      }
    }
    __threadfence();
  }
  __syncthreads();
  return *s_ok != 0;
}

// The rows of one phase (MODE 0: gate_up, 2I rows, K = H; 1: down, H rows,
// K = I) as this warp sees them.
struct PhaseRows {
  const uint8_t* blocks;
  const uint8_t* scales;
  const float* bias;
  int K, rows, NB, sp, row_bytes, slot_bytes, xstride;
};

// This warp's contiguous run of row pairs [q0, q1) of local expert le,
// streamed through its ring (kRing - 1 pairs in flight), dotted with the TC
// (>= n) staged rows of xs; results to h (MODE 0) or y (MODE 1) at positions
// p0 .. p0 + n - 1.  The token count is a template parameter so that the
// unrolled body stays small (the usual decode expert has one token).
template <int MODE, int TC>
__device__ void stream_pairs(const FusedArgs& a, const PhaseRows& R, const float* xs,
                             uint8_t* ring, int le, int q0, int q1, int p0, int n) {
  const int lane = threadIdx.x & 31;
  const int64_t erow = (int64_t)le * R.rows;
  const int np = q1 - q0;
  auto fetch = [&](int p) {
    if (p < np) {
      uint8_t* dst = ring + (p % kRing) * R.slot_bytes;
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int64_t row = erow + 2 * (q0 + p) + r;
        const uint8_t* rbp = R.blocks + row * R.row_bytes;
        for (int c = lane; c < R.NB; c += 32) cp_async16(dst + r * R.row_bytes + c * 16, rbp + c * 16);
        const uint8_t* rs = R.scales + row * R.sp;
        for (int c = lane; c < (R.sp >> 4); c += 32)
          cp_async16(dst + 2 * R.row_bytes + r * R.sp + c * 16, rs + c * 16);
      }
    }
    cp_async_commit();
  };
#pragma unroll
  for (int p = 0; p < kRing - 1; ++p) fetch(p);
  for (int p = 0; p < np; ++p) {
    fetch(p + kRing - 1);
    cp_async_wait<kRing - 1>();
    __syncwarp();
    const uint8_t* sl = ring + (p % kRing) * R.slot_bytes;
    float acc[2][TC];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int t = 0; t < TC; ++t) acc[r][t] = 0.0f;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
#pragma unroll
      for (int i = 0; i < kMaxNB / 32; ++i) {
        const int b = lane + 32 * i;
        if (b >= R.NB) continue;
        const uint4 q = *reinterpret_cast<const uint4*>(sl + r * R.row_bytes + b * 16);
        const float sc = e8m0_scale(sl[2 * R.row_bytes + r * R.sp + b], a.zero_scale);
        float v[32];
        decode_block_f32(q, v);
#pragma unroll
        for (int t = 0; t < TC; ++t) {
          if (TC == 1 || t < n) {
            const float4* x4 = reinterpret_cast<const float4*>(xs + t * R.xstride + b * kPitch);
            float f0 = 0.0f, f1 = 0.0f, f2 = 0.0f, f3 = 0.0f;
#pragma unroll
            for (int q4 = 0; q4 < 8; ++q4) {
              const float4 xv = x4[q4];
              f0 = __fmaf_rn(xv.x, v[4 * q4], f0);
              f1 = __fmaf_rn(xv.y, v[4 * q4 + 1], f1);
              f2 = __fmaf_rn(xv.z, v[4 * q4 + 2], f2);
              f3 = __fmaf_rn(xv.w, v[4 * q4 + 3], f3);
            }
            acc[r][t] = __fmaf_rn(__fadd_rn(__fadd_rn(f0, f1), __fadd_rn(f2, f3)), sc, acc[r][t]);
          }
        }
      }
    }
    __syncwarp();  // the slot is refilled by a later fetch
    const int row = 2 * (q0 + p);
#pragma unroll
    for (int t = 0; t < TC; ++t) {
      if (TC > 1 && t >= n) break;
      const float s0 = warp_sum_butterfly(acc[0][t]);
      const float s1 = warp_sum_butterfly(acc[1][t]);
      if (lane == 0) {
        const int64_t pos = p0 + t;
        if (MODE == 0) {
          float g = s0, u = s1;
          if (R.bias) {
            g = __fadd_rn(g, R.bias[erow + row]);
            u = __fadd_rn(u, R.bias[erow + row + 1]);
          }
          a.h[pos * a.I + (row >> 1)] = act_apply(a.act_kind, g, u, a.limit, a.clamp);
        } else {
          float y0 = s0, y1 = s1;
          if (R.bias) {
            y0 = __fadd_rn(y0, R.bias[erow + row]);
            y1 = __fadd_rn(y1, R.bias[erow + row + 1]);
          }
          a.y[pos * a.H + row] = y0;
          a.y[pos * a.H + row + 1] = y1;
        }
      }
    }
  }
  cp_async_wait<0>();
}

// One phase over the active experts' row pairs: a contiguous range of pairs
// per CTA (so a CTA stages the inputs of one or two experts), split into a
// contiguous run per warp inside each expert.
template <int MODE>
__device__ void expert_phase(const FusedArgs& a, uint8_t* smem, const int* s_act, const int* s_off,
                             const int* s_tok, int nact) {
  PhaseRows R;
  R.K = MODE == 0 ? a.H : a.I;
  R.rows = MODE == 0 ? 2 * a.I : a.H;
  R.NB = R.K >> 5;
  R.sp = MODE == 0 ? a.sp_h : a.sp_i;
  R.row_bytes = R.NB * 16;
  R.slot_bytes = 2 * (R.row_bytes + R.sp);
  R.xstride = R.NB * kPitch;
  R.blocks = MODE == 0 ? a.gu_blocks : a.dn_blocks;
  R.scales = MODE == 0 ? a.gu_scales : a.dn_scales;
  R.bias = MODE == 0 ? a.gu_bias : a.dn_bias;
  float* xs = reinterpret_cast<float*>(smem);  // [kStageTok][NB][kPitch]
  const int warp = threadIdx.x >> 5;
  uint8_t* ring = smem + (size_t)kStageTok * kMaxNB * kPitch * sizeof(float) +
                  (size_t)warp * kRing * R.slot_bytes;
  const int ppe = R.rows / 2;  // row pairs per expert
  const int total = nact * ppe;
  const int lo = (int)((int64_t)blockIdx.x * total / gridDim.x);
  const int hi = (int)((int64_t)(blockIdx.x + 1) * total / gridDim.x);
  for (int s = lo / ppe; s < nact && s * ppe < hi; ++s) {
    const int a_lo = max(lo, s * ppe) - s * ppe, a_hi = min(hi, (s + 1) * ppe) - s * ppe;
    const int pe = s_off[s], ne = s_off[s + 1] - s_off[s];  // ne <= kMaxTok
    // positions in chunks of kStageTok (an expert with more than 4 of the
    // batch's tokens streams its rows once per chunk)
    for (int c0 = 0; c0 < ne; c0 += kStageTok) {
      const int p0 = pe + c0, n = min(kStageTok, ne - c0);
      __syncthreads();  // the previous rows are no longer read
      for (int j = 0; j < n; ++j) {
        const float* src =
            MODE == 0 ? a.x + (int64_t)s_tok[p0 + j] * R.K : a.h + (int64_t)(p0 + j) * R.K;
        for (int k4 = threadIdx.x; k4 < (R.K >> 2); k4 += blockDim.x) {
          const int k = k4 << 2;
          const float4 v = MODE == 0 ? reinterpret_cast<const float4*>(src)[k4]
                                     : __ldcg(reinterpret_cast<const float4*>(src) + k4);
          *reinterpret_cast<float4*>(xs + j * R.xstride + (k >> 5) * kPitch + (k & 31)) = v;
        }
      }
      __syncthreads();
      const int span = a_hi - a_lo;
      const int q0 = a_lo + span * warp / kFWarps, q1 = a_lo + span * (warp + 1) / kFWarps;
      if (q1 > q0) {
        const int le = s_act[s];
        if (n <= 1) stream_pairs<MODE, 1>(a, R, xs, ring, le, q0, q1, p0, n);
        else if (n <= 2) stream_pairs<MODE, 2>(a, R, xs, ring, le, q0, q1, p0, n);
        else stream_pairs<MODE, 4>(a, R, xs, ring, le, q0, q1, p0, n);
      }
    }
  }
}

__global__ void __launch_bounds__(kFThreads, 1) fused_decode_kernel(const FusedArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float s_exp[kMaxTok][256];  // warps t < T select token t
  __shared__ int s_idx[kMaxTok * kMaxK];
  __shared__ float s_w[kMaxTok * kMaxK];
  __shared__ int s_act[kMaxPos], s_off[kMaxPos + 1], s_tok[kMaxPos], s_inv[kMaxTok * kMaxK];
  __shared__ int s_nact, s_ok;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int T = a.T, H = a.H, E = a.E, K = a.K;
  if (threadIdx.x == 0) s_ok = 1;

  // 1. router logits: the T token rows staged in shared memory; one warp per
  // expert loads its whole router row into registers at once (one memory
  // round trip), then accumulates every token in the router's order
  // (lane-strided FMAs, butterfly, bias)
  if ((int)blockIdx.x * kFWarps < E) {
    float* xs = reinterpret_cast<float*>(smem);  // [T][H]
    for (int i = threadIdx.x; i < T * (H >> 2); i += blockDim.x)
      reinterpret_cast<float4*>(xs)[i] = reinterpret_cast<const float4*>(a.x)[i];
    __syncthreads();
    for (int e = blockIdx.x * kFWarps + warp; e < E; e += gridDim.x * kFWarps) {
      const float* wr = a.rw + (int64_t)e * H;
      const int nb = H >> 5;
      float wv[kMaxNB];
#pragma unroll
      for (int j = 0; j < kMaxNB; ++j)
        if (j < nb) wv[j] = __ldg(wr + lane + (j << 5));
      for (int t = 0; t < T; ++t) {
        float acc = 0.0f;
#pragma unroll
        for (int j = 0; j < kMaxNB; ++j)
          if (j < nb) acc = __fmaf_rn(xs[t * H + lane + (j << 5)], wv[j], acc);
        acc = warp_sum_butterfly(acc);
        if (lane == 0) a.logits[(int64_t)t * E + e] = a.rb ? __fadd_rn(acc, a.rb[e]) : acc;
      }
    }
  }
  if (!grid_barrier(a, &s_ok)) return;

  // 2. every CTA: the same top-k and grouping
  for (int t = warp; t < T; t += kFWarps)
    select_topk(a.logits + (int64_t)t * E, E, K, a.router_kind, a.sel_bias, s_exp[warp],
                s_idx + t * K, s_w + t * K);
  __syncthreads();
  if (threadIdx.x == 0) {
    int n = 0;
    for (int i = 0; i < T * K; ++i) {  // distinct experts, ascending
      const int e = s_idx[i];
      int j = 0;
      while (j < n && s_act[j] < e) ++j;
      if (j < n && s_act[j] == e) continue;
      for (int q = n; q > j; --q) s_act[q] = s_act[q - 1];
      s_act[j] = e;
      ++n;
    }
    int pos = 0;
    for (int s = 0; s < n; ++s) {  // per expert: tokens ascending (gpt_oss_q.rs:175-192)
      s_off[s] = pos;
      for (int t = 0; t < T; ++t)
        for (int r = 0; r < K; ++r)
          if (s_idx[t * K + r] == s_act[s]) {
            s_tok[pos] = t;
            s_inv[t * K + r] = pos;
            ++pos;
          }
    }
    s_off[n] = pos;
    s_nact = n;
    if (blockIdx.x == 0)
      for (int i = 0; i < T * K; ++i) {
        a.idx_out[i] = s_idx[i];
        a.w_out[i] = s_w[i];
      }
  }
  __syncthreads();

  // 3. gate_up -> h
  expert_phase<0>(a, smem, s_act, s_off, s_tok, s_nact);
  if (!grid_barrier(a, &s_ok)) return;
  // 4. down -> y
  expert_phase<1>(a, smem, s_act, s_off, s_tok, s_nact);
  if (!grid_barrier(a, &s_ok)) return;

  // 5. combine: rank order, or expert order (GGUF, gpt_oss_q.rs:252-266)
  const int n4 = H >> 2;
  for (int u = blockIdx.x * kFThreads + threadIdx.x; u < T * n4; u += gridDim.x * kFThreads) {
    const int t = u / n4, c = u - t * n4;
    int order[kMaxK];
    for (int r = 0; r < K; ++r) order[r] = r;
    if (a.expert_order)
      for (int i = 1; i < K; ++i) {
        const int cur = order[i];
        int b = i - 1;
        while (b >= 0 && s_idx[t * K + order[b]] > s_idx[t * K + cur]) {
          order[b + 1] = order[b];
          --b;
        }
        order[b + 1] = cur;
      }
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int q = 0; q < K; ++q) {
      const int r = order[q];
      const float w = s_w[t * K + r];
      const float4 v = __ldcg(reinterpret_cast<const float4*>(a.y + (int64_t)s_inv[t * K + r] * H) + c);
      acc.x = __fadd_rn(acc.x, __fmul_rn(v.x, w));
      acc.y = __fadd_rn(acc.y, __fmul_rn(v.y, w));
      acc.z = __fadd_rn(acc.z, __fmul_rn(v.z, w));
      acc.w = __fadd_rn(acc.w, __fmul_rn(v.w, w));
    }
    reinterpret_cast<float4*>(a.out + (int64_t)t * H)[c] = acc;
  }
}

// One size for every handle (the kernel attribute is shared by all of them):
// the largest rows (K = 3072: 96 blocks, 96 scale bytes).  Phase 1 uses the
// same space for the T token rows (at most 8 x 3072 floats).
constexpr size_t kFusedSmem = (size_t)kStageTok * kMaxNB * kPitch * sizeof(float) +
                              (size_t)kFWarps * kRing * 2 * (kMaxNB * 16 + kMaxNB);
static_assert(kFusedSmem >= (size_t)kMaxTok * kMaxNB * 32 * sizeof(float), "phase 1 rows");

size_t fused_smem(const Moe&) { return kFusedSmem; }

}  // namespace

bool fused_decode_fits(const Moe& m, int64_t T) {
  const gb_moe_desc& d = m.desc;
  return m.fused_ctas > 0 && m.ep_size == 1 && T >= 1 && T <= kMaxTok &&
         T * d.top_k <= kMaxPos && d.top_k <= kMaxK && m.w.gu_blocks != nullptr &&
         (d.weight_format == GB_FMT_MXFP4_SPLIT || d.weight_format == GB_FMT_MXFP4_GGUF) &&
         !d.input_norm && !d.output_norm && !d.expert_scale && d.hidden % 64 == 0 &&
         d.inter % 64 == 0 && d.hidden / 32 <= kMaxNB && d.inter / 32 <= kMaxNB &&
         d.n_experts <= 256;
}

cudaError_t fused_decode_prepare(Moe& m) {
  m.fused_ctas = 0;
  int coop = 0;
  cudaError_t e = cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, m.device);
  if (e != cudaSuccess || !coop) return e;
  const size_t smem = fused_smem(m);
  if ((e = cudaFuncSetAttribute(fused_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)smem)) != cudaSuccess) {
    cudaGetLastError();
    return cudaSuccess;  // no fused path on this device
  }
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fused_decode_kernel, kFThreads, smem);
  if (e != cudaSuccess || per_sm < 1) {
    cudaGetLastError();
    return cudaSuccess;
  }
  m.fused_ctas = m.sm_count;  // one CTA per SM (the kernel needs no more)
  return cudaSuccess;
}

cudaError_t launch_fused_decode(const Moe& m, const float* x, int64_t T, float* out,
                                cudaStream_t st) {
  const gb_moe_desc& d = m.desc;
  FusedArgs a{};
  a.x = x;
  a.T = (int)T;
  a.H = d.hidden;
  a.I = d.inter;
  a.E = d.n_experts;
  a.K = d.top_k;
  a.router_kind = d.router_kind;
  a.rw = m.router_w;
  a.rb = m.router_b;
  a.sel_bias = m.sel_bias;
  a.logits = m.ws.logits;
  a.idx_out = m.ws.idx;
  a.w_out = m.ws.wts;
  a.gu_blocks = m.w.gu_blocks;
  a.gu_scales = m.w.gu_scales;
  a.sp_h = m.w.sp_h;
  a.gu_bias = m.w.gu_bias;
  a.dn_blocks = m.w.dn_blocks;
  a.dn_scales = m.w.dn_scales;
  a.sp_i = m.w.sp_i;
  a.dn_bias = m.w.dn_bias;
  a.zero_scale = m.w.zero_scale;
  a.act_kind = d.act_kind;
  a.limit = d.swiglu_limit;
  a.clamp = d.act_clamp;
  a.h = m.ws.eb.h;
  a.y = m.ws.eb.y;
  a.out = out;
  a.expert_order = d.weight_format == GB_FMT_MXFP4_GGUF;
  a.bar = m.ws.grid_bar;
  a.err = m.ws.meta + 1;
  a.wait_ns = m.test_wait_ns ? m.test_wait_ns : kMbarWaitNs;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)m.fused_ctas);
  cfg.blockDim = dim3(kFThreads);
  cfg.dynamicSmemBytes = fused_smem(m);
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, fused_decode_kernel, a);
}

}  // namespace gb
