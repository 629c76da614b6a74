// route_select.cuh -- the top-k selection of one token's router logits, as
// the reference computes it, for a whole warp (the router's last CTA and the
// fused decode kernel both call it, so both select identically).
//
// Softmax router (gpt_oss.rs:172-182): softmax over all E experts as candle's
// softmax_last_dim evaluates a row (the maximum, exp(l - max), their sum in
// expert order, each exp divided by the sum), a stable descending sort of the
// probabilities (equal probabilities keep the lower index), the first k,
// weights p / max(sum of the k, 1e-9) summed in rank order.  Sigmoid router
// (lfm2moe_q.rs:241-258): p = 1 / (exp(-l) + 1), selection by p + bias,
// weights p / max(sum, 1e-20).  exp is exp_f32 (exp_f32.h), the correctly
// rounded exp.  Experts whose keys are all NaN go to the lowest free index
// with weight 0.
#pragma once

#include <math.h>

#include "common.cuh"
#include "exp_f32.h"

namespace gb {

// Every lane of the warp calls it; lane 0 writes idx_out[0..K), w_out[0..K).
// s_exp_row: E floats of shared memory owned by this warp.  E <= 256, K <= 8.
__device__ __forceinline__ void select_topk(const float* __restrict__ lg, int E, int K, int kind,
                                            const float* __restrict__ sel_bias,
                                            float* __restrict__ s_exp_row,
                                            int32_t* __restrict__ idx_out,
                                            float* __restrict__ w_out) {
  const int lane = threadIdx.x & 31;
    constexpr int kMaxPerLane = 8;  // E <= 256
    float key[kMaxPerLane];
    float raw[kMaxPerLane];
    unsigned taken = 0;
    if (kind == GB_ROUTER_SIGMOID_TOPK) {
      // p = 1 / (exp(-l) + 1) (candle's sigmoid); selection by p + bias
#pragma unroll
      for (int q = 0; q < kMaxPerLane; ++q) {
        const int e = lane + 32 * q;
        raw[q] = 0.0f;
        key[q] = -INFINITY;
        if (e < E) {
          const float p = __fdiv_rn(1.0f, __fadd_rn(exp_f32(-__ldcg(lg + e)), 1.0f));
          raw[q] = p;
          key[q] = __fadd_rn(p, sel_bias ? sel_bias[e] : 0.0f);
        }
      }
    } else {
      // softmax over all E experts as candle's softmax_last_dim evaluates a
      // row (gpt_oss.rs:174): the row maximum, exp(l - max), their sum in
      // expert order, then each exp divided by the sum.  Experts are ranked
      // by these probabilities, so two logits whose probabilities round to
      // the same f32 tie and go to the lower index, as in the reference.
      float l[kMaxPerLane];
      float mx = -INFINITY;
#pragma unroll
      for (int q = 0; q < kMaxPerLane; ++q) {
        const int e = lane + 32 * q;
        l[q] = e < E ? __ldcg(lg + e) : -INFINITY;
        mx = fmaxf(mx, l[q]);
      }
#pragma unroll
      for (int s = 16; s >= 1; s >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFullMask, mx, s));
      float* ex = s_exp_row;
#pragma unroll
      for (int q = 0; q < kMaxPerLane; ++q) {
        raw[q] = 0.0f;
        if (lane + 32 * q < E) {
          raw[q] = exp_f32(__fsub_rn(l[q], mx));
          ex[lane + 32 * q] = raw[q];
        }
      }
      __syncwarp();
      // every lane adds the E values in expert order (broadcast loads, so
      // only the additions form a chain)
      float sum = 0.0f;
#pragma unroll 8
      for (int e = 0; e < E; ++e) sum = __fadd_rn(sum, ex[e]);
      __syncwarp();  // the next token of this warp rewrites ex
#pragma unroll
      for (int q = 0; q < kMaxPerLane; ++q) {
        const bool in = lane + 32 * q < E;
        raw[q] = in ? __fdiv_rn(raw[q], sum) : 0.0f;
        key[q] = in ? raw[q] : -INFINITY;
      }
    }
    float sel_raw[8];
    int sel_idx[8];
    for (int r = 0; r < K; ++r) {
      float best = -INFINITY, braw = 0.0f;
      int bi = 0x7fffffff;
#pragma unroll
      for (int q = 0; q < kMaxPerLane; ++q) {
        const int e = lane + 32 * q;
        if (e < E && !((taken >> q) & 1u) &&
            (key[q] > best || (key[q] == best && e < bi))) {
          best = key[q];
          bi = e;
          braw = raw[q];
        }
      }
#pragma unroll
      for (int s = 16; s >= 1; s >>= 1) {
        const float ob = __shfl_xor_sync(kFullMask, best, s);
        const int oi = __shfl_xor_sync(kFullMask, bi, s);
        const float orw = __shfl_xor_sync(kFullMask, braw, s);
        if (ob > best || (ob == best && oi < bi)) {
          best = ob;
          bi = oi;
          braw = orw;
        }
      }
      if (bi >= E) {  // only NaN keys left: take the lowest free index, weight 0
        bi = 0;
        for (int e = 0; e < E; ++e) {
          bool used = false;
          for (int rr = 0; rr < r; ++rr) used |= sel_idx[rr] == e;
          if (!used) {
            bi = e;
            break;
          }
        }
        braw = 0.0f;
      }
      if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
      sel_idx[r] = bi;
      sel_raw[r] = braw;
    }
    if (lane == 0) {
      int32_t* io = idx_out;
      float* wo = w_out;
      if (kind == GB_ROUTER_SIGMOID_TOPK) {
        float total = 0.0f;
        for (int r = 0; r < K; ++r) total = __fadd_rn(total, sel_raw[r]);
        total = fmaxf(total, 1e-20f);
        for (int r = 0; r < K; ++r) {
          io[r] = sel_idx[r];
          wo[r] = __fdiv_rn(sel_raw[r], total);
        }
      } else {
        // w = p / max(sum of the k selected p, 1e-9), summed in rank order
        // (gpt_oss.rs:180-182); the reference divides in f64 and rounds to
        // f32, which equals the f32 division
        float total = 0.0f;
        for (int r = 0; r < K; ++r) total = __fadd_rn(total, sel_raw[r]);
        total = fmaxf(total, 1e-9f);
        for (int r = 0; r < K; ++r) {
          io[r] = sel_idx[r];
          wo[r] = __fdiv_rn(sel_raw[r], total);
        }
      }
    }
}

}  // namespace gb
