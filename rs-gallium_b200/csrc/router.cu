// router.cu -- router projection + top-k selection + combine weights.
//
// Reference: gpt_oss.rs:172-182 (softmax router), lfm2moe_q.rs:241-258
// (sigmoid router with selection bias), docs/gpt-oss.md:83-93.
//
// logits[t, e] = dot(x[t, :], W[e, :]) + b[e], reduced in a fixed order: lane l
// of a warp accumulates k = l, l+32, l+64, ... with FMAs, then a butterfly over
// the 32 lanes (xor 16, 8, 4, 2, 1), then the bias add.  The oracle restates
// the same order, so expert indices compare bit for bit.
//
// Grid: (token tiles of TT, expert groups).  Each warp computes EPW experts'
// logits for the TT tokens of its tile; the last CTA of a tile to finish
// (threadfence + per-tile ticket, no waiting) runs the top-k for that tile.
//
// Selection follows the reference's arithmetic to the last bit: softmax over
// all experts (max, exp, sum in expert order, divide), stable descending
// sort of the probabilities (equal probabilities keep the lower index), the
// first k, weights p / max(sum, 1e-9).  exp is the correctly rounded one of
// exp_f32.h, on the host and on the GPU alike.
#include <math.h>

#include <mutex>

#include "common.cuh"
#include "exp_f32.h"
#include "route_select.cuh"
#include "moe_internal.h"
#include "ptx.cuh"

namespace gb {
namespace {

constexpr int kRouterWarps = 8;
constexpr int kPreloadBlocks = 96;  // H <= 3072 for the preloading variant

// After this CTA stored its logits of token tile blockIdx.x: the last CTA of
// the tile to finish (threadfence + per-tile ticket, no waiting) runs the
// top-k and combine weights of the tile's nt tokens, one warp per token.
__device__ __forceinline__ void route_tail(int t0, int nt, const float* __restrict__ logits,
                                           unsigned* __restrict__ tickets, int E, int K,
                                           int kind, const float* __restrict__ sel_bias,
                                           int32_t* __restrict__ idx_out,
                                           float* __restrict__ w_out) {
  __shared__ unsigned s_ticket;
  __shared__ float s_exp[kRouterWarps][256];  // per warp: exp(l - max) of a token's experts
  const int warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;  // both router kernels run kRouterWarps warps
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_ticket = atomicAdd(&tickets[blockIdx.x], 1u);
  __syncthreads();
  if (s_ticket != gridDim.y - 1) return;
  __threadfence();
  if (threadIdx.x == 0) tickets[blockIdx.x] = 0;  // ready for the next forward

  for (int t = warp; t < nt; t += nwarps)
    select_topk(logits + (int64_t)(t0 + t) * E, E, K, kind, sel_bias, s_exp[warp],
                idx_out + (int64_t)(t0 + t) * K, w_out + (int64_t)(t0 + t) * K);
}

template <int TT, int EPW>
__global__ void __launch_bounds__(kRouterWarps * 32)
    router_kernel(const float* __restrict__ x, int T, int H, const float* __restrict__ rw,
                  const float* __restrict__ rb, int E, int K, int kind,
                  const float* __restrict__ sel_bias, float* __restrict__ logits,
                  unsigned* __restrict__ tickets, int32_t* __restrict__ idx_out,
                  float* __restrict__ w_out) {
  extern __shared__ float xs[];  // [TT][H]
  pdl_trigger();
  pdl_wait();
  const int t0 = blockIdx.x * TT;
  const int nt = min(TT, T - t0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e0 = (blockIdx.y * (int)(blockDim.x >> 5) + warp) * EPW;
  const int nb = H >> 5;
  // Decode-sized batches: few warps read the router weight, so each lane
  // issues all of its weight loads first, then the x loads, and only then
  // waits (one memory round trip for the CTA).
  constexpr bool kPreload = EPW == 1 && TT <= 4;
  const bool preload = kPreload && nb <= kPreloadBlocks && e0 < E;
  float wv[kPreload ? kPreloadBlocks : 1];
  if constexpr (kPreload) {
    if (preload) {
      const float* wr = rw + (int64_t)e0 * H;
#pragma unroll
      for (int j = 0; j < kPreloadBlocks; ++j)
        if (j < nb) wv[j] = __ldg(wr + lane + (j << 5));
    }
  }

  {
    const float4* src = reinterpret_cast<const float4*>(x + (int64_t)t0 * H);
    float4* dst = reinterpret_cast<float4*>(xs);
    const int n4 = nt * H / 4;
#pragma unroll 4
    for (int i = threadIdx.x; i < TT * H / 4; i += blockDim.x)
      dst[i] = i < n4 ? src[i] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  __syncthreads();

  if (e0 < E) {
    float acc[EPW][TT];
#pragma unroll
    for (int q = 0; q < EPW; ++q)
#pragma unroll
      for (int t = 0; t < TT; ++t) acc[q][t] = 0.0f;
    const float* wrow[EPW];
#pragma unroll
    for (int q = 0; q < EPW; ++q) wrow[q] = rw + (int64_t)min(e0 + q, E - 1) * H;
    if (preload) {
#pragma unroll
      for (int j = 0; j < kPreloadBlocks; ++j) {
        if (j < nb) {
#pragma unroll
          for (int t = 0; t < TT; ++t)
            acc[0][t] = __fmaf_rn(xs[t * H + lane + (j << 5)], wv[j], acc[0][t]);
        }
      }
    } else {
#pragma unroll 6
      for (int j = 0; j < nb; ++j) {
        const int kk = lane + (j << 5);
        float wv[EPW];
#pragma unroll
        for (int q = 0; q < EPW; ++q) wv[q] = __ldg(wrow[q] + kk);
#pragma unroll
        for (int t = 0; t < TT; ++t) {
          const float xv = xs[t * H + kk];
#pragma unroll
          for (int q = 0; q < EPW; ++q) acc[q][t] = __fmaf_rn(xv, wv[q], acc[q][t]);
        }
      }
    }
#pragma unroll
    for (int q = 0; q < EPW; ++q) {
#pragma unroll
      for (int t = 0; t < TT; ++t) {
        const float v = warp_sum_butterfly(acc[q][t]);
        const int e = e0 + q;
        if (lane == 0 && e < E && t < nt)
          logits[(int64_t)(t0 + t) * E + e] = rb ? __fadd_rn(v, rb[e]) : v;
      }
    }
  }

  route_tail(t0, nt, logits, tickets, E, K, kind, sel_bias, idx_out, w_out);
}

// Prefill-sized batches: a CTA computes the logits of 32 tokens x 16 experts,
// each warp 8 tokens x 8 experts (64 partial sums per lane), with x and W
// staged through shared memory 256 k at a time (cp.async, two buffers).  Lane l still accumulates
// k = l, l + 32, ... in increasing k with FMAs, and the 64 sums are reduced
// over the lanes in the butterfly's pairing (xor 16, 8, 4, 2, 1; IEEE
// addition commutes, so every lane of the butterfly holds the same value),
// as a reduce-scatter that leaves lane l the sums of (token l / 4, experts
// 2 (l % 4) and 2 (l % 4) + 1).  Logits are bit-identical to router_kernel.
constexpr int kTileTokens = 32, kTileExperts = 16, kTileK = 256;

__global__ void __launch_bounds__(256, 2)
    router_tiled_kernel(const float* __restrict__ x, int T, int H, const float* __restrict__ rw,
                        const float* __restrict__ rb, int E, int K, int kind,
                        const float* __restrict__ sel_bias, float* __restrict__ logits,
                        unsigned* __restrict__ tickets, int32_t* __restrict__ idx_out,
                        float* __restrict__ w_out) {
  extern __shared__ __align__(16) float sm[];  // two buffers of [32 tokens + 16 experts][256]
  pdl_trigger();
  pdl_wait();
  constexpr int kBuf = (kTileTokens + kTileExperts) * kTileK;
  const int t0 = blockIdx.x * kTileTokens, e0 = blockIdx.y * kTileExperts;
  const int nt = min(kTileTokens, T - t0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tw = (warp & 3) * 8, ew = (warp >> 2) * 8;
  const int nchunks = (H + kTileK - 1) / kTileK;
  float acc[8][8];
#pragma unroll
  for (int t = 0; t < 8; ++t)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[t][e] = 0.0f;

  // chunk c of x (rows past T zero-filled) and W into buffer c % 2
  auto stage = [&](int c) {
    float* xs = sm + (c & 1) * kBuf;
    float* ws = xs + kTileTokens * kTileK;
    const int k0 = c * kTileK, q4 = min(kTileK, H - k0) / 4;
    if (q4 == kTileK / 4) {
      // full chunk: thread i copies column 4 (i % 64) of rows i / 64 + 4 n
      // (256 threads, 64 16-byte pieces per row), no per-copy division
      const int col = 4 * (threadIdx.x & 63), r0 = threadIdx.x >> 6;
#pragma unroll
      for (int n = 0; n < kTileTokens / 4; ++n) {
        const int r = r0 + 4 * n;
        const float* src = x + (int64_t)(t0 + (r < nt ? r : 0)) * H + k0 + col;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                         smem_u32(xs + r * kTileK + col)),
                     "l"(src), "r"(r < nt ? 16 : 0)
                     : "memory");
      }
#pragma unroll
      for (int n = 0; n < kTileExperts / 4; ++n) {
        const int r = r0 + 4 * n;
        const float* src = rw + (int64_t)min(e0 + r, E - 1) * H + k0 + col;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                         smem_u32(ws + r * kTileK + col)),
                     "l"(src)
                     : "memory");
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
      return;
    }
    for (int i = threadIdx.x; i < (kTileTokens + kTileExperts) * q4; i += blockDim.x) {
      const int r = i / q4, col = 4 * (i - r * q4);
      const float* src;
      float* dst;
      int bytes = 16;
      if (r < kTileTokens) {
        const int tr = r < nt ? r : 0;
        src = x + (int64_t)(t0 + tr) * H + k0 + col;
        dst = xs + r * kTileK + col;
        if (r >= nt) bytes = 0;
      } else {
        src = rw + (int64_t)min(e0 + r - kTileTokens, E - 1) * H + k0 + col;
        dst = ws + (r - kTileTokens) * kTileK + col;
      }
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
                   "r"(bytes)
                   : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };

  stage(0);
  for (int c = 0; c < nchunks; ++c) {
    if (c + 1 < nchunks) {
      stage(c + 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();  // chunk c has landed for every thread
    const float* xs = sm + (c & 1) * kBuf;
    const float* ws = xs + kTileTokens * kTileK;
    const int kl = min(kTileK, H - c * kTileK);  // a multiple of 32
#pragma unroll 2
    for (int jj = 0; jj < kl / 32; ++jj) {
      const int kk = jj * 32 + lane;
      float xv[8], wv[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) xv[t] = xs[(tw + t) * kTileK + kk];
#pragma unroll
      for (int e = 0; e < 8; ++e) wv[e] = ws[(ew + e) * kTileK + kk];
#pragma unroll
      for (int t = 0; t < 8; ++t)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[t][e] = __fmaf_rn(xv[t], wv[e], acc[t][e]);
    }
    __syncthreads();  // buffer c % 2 may be refilled by the next iteration
  }

  // reduce-scatter of the 64 sums (index 8 t + e) over the 32 lanes
  float r32[32], r16[16], r8[8], r4[4];
#pragma unroll
  for (int q = 0; q < 32; ++q) {
    const bool up = lane & 16;
    const float lo = acc[q >> 3][q & 7], hi = acc[(q + 32) >> 3][(q + 32) & 7];
    r32[q] = __fadd_rn(up ? hi : lo, __shfl_xor_sync(kFullMask, up ? lo : hi, 16));
  }
#pragma unroll
  for (int q = 0; q < 16; ++q) {
    const bool up = lane & 8;
    r16[q] = __fadd_rn(up ? r32[q + 16] : r32[q],
                       __shfl_xor_sync(kFullMask, up ? r32[q] : r32[q + 16], 8));
  }
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const bool up = lane & 4;
    r8[q] = __fadd_rn(up ? r16[q + 8] : r16[q],
                      __shfl_xor_sync(kFullMask, up ? r16[q] : r16[q + 8], 4));
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const bool up = lane & 2;
    r4[q] = __fadd_rn(up ? r8[q + 4] : r8[q], __shfl_xor_sync(kFullMask, up ? r8[q] : r8[q + 4], 2));
  }
  float res[2];
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const bool up = lane & 1;
    res[q] = __fadd_rn(up ? r4[q + 2] : r4[q], __shfl_xor_sync(kFullMask, up ? r4[q] : r4[q + 2], 1));
  }
  const int t = tw + (lane >> 2);
  if (t < nt) {
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int e = e0 + ew + 2 * (lane & 3) + q;
      if (e < E) logits[(int64_t)(t0 + t) * E + e] = rb ? __fadd_rn(res[q], rb[e]) : res[q];
    }
  }
  route_tail(t0, nt, logits, tickets, E, K, kind, sel_bias, idx_out, w_out);
}

// warps: experts per CTA (EPW each); fewer warps spread a small batch's
// router rows over more SMs.  A warp computes its experts' dot products
// whole, so the logits do not depend on it.
template <int TT, int EPW>
cudaError_t launch(const Moe& m, const float* x, int64_t T, int32_t* idx, float* wts,
                   cudaStream_t st, int warps = kRouterWarps) {
  const gb_moe_desc& d = m.desc;
  const int H = d.hidden, E = d.n_experts;
  dim3 grid((unsigned)((T + TT - 1) / TT), (unsigned)((E + warps * EPW - 1) / (warps * EPW)));
  const size_t smem = (size_t)TT * H * sizeof(float);
  auto kern = router_kernel<TT, EPW>;
  cudaError_t err = set_smem_limit(kern, smem);
  if (err != cudaSuccess) return err;
  return launch_pdl(kern, grid, dim3(warps * 32), smem, st, x, (int)T, H, m.router_w,
                    m.router_b, E, d.top_k, d.router_kind, m.sel_bias, m.ws.logits, m.ws.tickets,
                    idx, wts);
}

}  // namespace

cudaError_t launch_router_topk(const Moe& m, const float* x, int64_t T, int32_t* idx, float* wts,
                               cudaStream_t st) {
  if (T <= 0) return cudaSuccess;
  // measured on 128 experts x 2880: one token per CTA is fastest to 16
  // tokens, two to 64 (more tokens per warp lengthen its dependent chains);
  // the tiled kernel needs more than a few hundred tokens to fill the GPU.
  // (Two warps per CTA at one token, E / 2 CTAs, measured slower: 15.1 vs
  // 13.5 us.)
  if (T <= 16) return launch<1, 1>(m, x, T, idx, wts, st);
  if (T <= 256) return launch<2, 1>(m, x, T, idx, wts, st);
  const gb_moe_desc& d = m.desc;
  dim3 grid((unsigned)((T + kTileTokens - 1) / kTileTokens),
            (unsigned)((d.n_experts + kTileExperts - 1) / kTileExperts));
  const size_t smem = 2 * (size_t)(kTileTokens + kTileExperts) * kTileK * sizeof(float);
  cudaError_t err = set_smem_limit(router_tiled_kernel, smem);
  if (err != cudaSuccess) return err;
  return launch_pdl(router_tiled_kernel, grid, dim3(256), smem, st, x, (int)T, d.hidden,
                    m.router_w, m.router_b, d.n_experts, d.top_k, d.router_kind, m.sel_bias,
                    m.ws.logits, m.ws.tickets, idx, wts);
}

}  // namespace gb

// ---------------------------------------------------------------------------
// Routing that allocates nothing (gb_route_noalloc).
//
// For callers that cannot call cudaMalloc when they route: a candle custom op
// whose device buffers must all come from candle's own allocator, or a serving
// process that has reserved the device's memory up front.  The router kernel
// above needs scratch beyond its inputs and outputs (the [T, E] logits and one
// ticket per token tile); here that scratch is a fixed array in this library's
// device image, so the call allocates nothing.  Every GPU that loads the
// library holds the array until the process exits.
// ---------------------------------------------------------------------------
namespace gb {
namespace {

constexpr int64_t kNoAllocMaxLogits = 65536;  // T * n_experts
constexpr int64_t kNoAllocMaxTiles = 4096;    // token tiles (at most T)
constexpr size_t kNoAllocTicketOffset = (size_t)kNoAllocMaxLogits * sizeof(float);
constexpr size_t kNoAllocBytes = kNoAllocTicketOffset + (size_t)kNoAllocMaxTiles * sizeof(unsigned);
constexpr int kNoAllocMaxDevices = 64;

}  // namespace
}  // namespace gb

// The scratch: logits at offset 0, tickets after them.  In host code this
// name is only a stand-in for the symbol, never a device address; host code
// uses the address from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_route_scratch[gb::kNoAllocBytes];

namespace gb {
namespace {

std::mutex g_route_scratch_mu;
void* g_route_scratch_addr[kNoAllocMaxDevices] = {};

// Device address of g_route_scratch on device `dev` (which must be current),
// looked up once per device on its first use and kept for the life of the
// process.  A cudaDeviceReset (or any teardown of the device's primary
// context) invalidates that address; gb_route_noalloc must not be called on a
// device after such a reset.
int route_scratch_address(int dev, void** out) {
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return set_error(GB_ERR_UNSUPPORTED, "device ordinal %d >= %d", dev, kNoAllocMaxDevices);
  std::lock_guard<std::mutex> lock(g_route_scratch_mu);
  if (!g_route_scratch_addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_route_scratch);
    if (e != cudaSuccess || !p)
      return set_error(GB_ERR_CUDA, "cudaGetSymbolAddress(route scratch) on device %d: %s", dev,
                       cudaGetErrorString(e));
    g_route_scratch_addr[dev] = p;
  }
  *out = g_route_scratch_addr[dev];
  return GB_OK;
}

template <int TT, int EPW>
cudaError_t launch_noalloc(const float* x, int64_t T, int H, const float* rw, const float* rb,
                           int E, int K, int kind, const float* sel_bias, float* logits,
                           unsigned* tickets, int32_t* idx, float* wts, cudaStream_t st) {
  const int64_t tiles = (T + TT - 1) / TT;
  cudaError_t err = cudaMemsetAsync(tickets, 0, sizeof(unsigned) * (size_t)tiles, st);
  if (err != cudaSuccess) return err;
  dim3 grid((unsigned)tiles, (unsigned)((E + kRouterWarps * EPW - 1) / (kRouterWarps * EPW)));
  const size_t smem = (size_t)TT * H * sizeof(float);
  auto kern = router_kernel<TT, EPW>;
  err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (err != cudaSuccess) return err;
  kern<<<grid, kRouterWarps * 32, smem, st>>>(x, (int)T, H, rw, rb, E, K, kind, sel_bias, logits,
                                              tickets, idx, wts);
  return cudaGetLastError();
}

}  // namespace
}  // namespace gb

extern "C" int gb_route_noalloc(const float* x_dev, const float* router_weight_dev,
                                const float* router_bias_dev, const float* selection_bias_dev,
                                int64_t T, int32_t hidden, int32_t n_experts, int32_t top_k,
                                int32_t router_kind, int32_t* idx_dev, float* w_dev,
                                void* stream) {
  using namespace gb;
  if (T < 0) return set_error(GB_ERR_INVALID_ARG, "T = %lld < 0", (long long)T);
  // hidden <= 4096 as for gb_moe_create; it also keeps the 8-token tile of x
  // (8 * hidden floats) inside one CTA's shared memory.
  if (hidden <= 0 || hidden % 32 != 0 || hidden > 4096)
    return set_error(GB_ERR_INVALID_ARG, "hidden %d must be a positive multiple of 32, <= 4096",
                     hidden);
  if (n_experts < 1 || n_experts > 256)
    return set_error(GB_ERR_INVALID_ARG, "n_experts %d not in 1..256", n_experts);
  if (top_k < 1 || top_k > 8 || top_k > n_experts)
    return set_error(GB_ERR_INVALID_ARG, "top_k %d must be in 1..min(8, n_experts)", top_k);
  if (router_kind != GB_ROUTER_SOFTMAX_TOPK && router_kind != GB_ROUTER_SIGMOID_TOPK)
    return set_error(GB_ERR_INVALID_ARG, "unknown router_kind %d", router_kind);
  if (T == 0) return GB_OK;
  if (!x_dev || !router_weight_dev || !idx_dev || !w_dev)
    return set_error(GB_ERR_INVALID_ARG, "x, router_weight, idx and w must not be null");
  // the kernel reads x rows as 16-byte vectors
  if (reinterpret_cast<uintptr_t>(x_dev) & 15)
    return set_error(GB_ERR_INVALID_ARG, "x must be 16-byte aligned");
  if (T * (int64_t)n_experts > kNoAllocMaxLogits || T > kNoAllocMaxTiles)
    return set_error(GB_ERR_INVALID_ARG,
                     "T * n_experts = %lld exceeds the fixed routing scratch of %lld logits "
                     "(and T <= %lld); route in smaller batches",
                     (long long)(T * (int64_t)n_experts), (long long)kNoAllocMaxLogits,
                     (long long)kNoAllocMaxTiles);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(GB_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  void* scratch = nullptr;
  const int rc = route_scratch_address(dev, &scratch);
  if (rc) return rc;
  float* logits = static_cast<float*>(scratch);
  unsigned* tickets = reinterpret_cast<unsigned*>(static_cast<char*>(scratch) + kNoAllocTicketOffset);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (T <= 4)
    e = launch_noalloc<1, 1>(x_dev, T, hidden, router_weight_dev, router_bias_dev, n_experts, top_k,
                             router_kind, selection_bias_dev, logits, tickets, idx_dev, w_dev, st);
  else if (T <= 64)
    e = launch_noalloc<4, 1>(x_dev, T, hidden, router_weight_dev, router_bias_dev, n_experts, top_k,
                             router_kind, selection_bias_dev, logits, tickets, idx_dev, w_dev, st);
  else
    e = launch_noalloc<8, 4>(x_dev, T, hidden, router_weight_dev, router_bias_dev, n_experts, top_k,
                             router_kind, selection_bias_dev, logits, tickets, idx_dev, w_dev, st);
  if (e != cudaSuccess)
    return set_error(GB_ERR_CUDA, "no-alloc router launch: %s", cudaGetErrorString(e));
  return GB_OK;
}
