// permute.cu -- group the (token, rank) routing entries by expert.
//
// Reference: gpt_oss_q.rs:175-192 (and lfm2moe_q.rs:245-264): expert_tokens[e]
// is filled in token order, and the active experts are taken in ascending
// order.  The sorted order here is therefore (expert ascending, token
// ascending), a stable counting sort, and it is bit-identical to the oracle.
//
// One CTA of 1024 threads.  Counts come from shared-memory atomics (order
// free).  Positions come from per-expert bitmaps of each 1024-token chunk:
// bit (t mod 32) of word [e][(t mod 1024) / 32] says token t chose expert e;
// a warp scan of the word popcounts gives each word's offset, and a popcount
// of the lower lanes' bits gives the token's place inside its word.
#include "common.cuh"
#include "moe_internal.h"
#include "ptx.cuh"

namespace gb {
namespace {

constexpr int kPermThreads = 1024;
constexpr int kWords = kPermThreads / 32;

__global__ void __launch_bounds__(kPermThreads)
    permute_kernel(const int32_t* __restrict__ idx, int T, int E, int K, int e_begin, int e_end,
                   int32_t* __restrict__ counts, int32_t* __restrict__ offsets,
                   int32_t* __restrict__ active, int32_t* __restrict__ meta,
                   int32_t* __restrict__ perm, int32_t* __restrict__ inv) {
  extern __shared__ unsigned sm[];
  unsigned* cnt = sm;                  // [E]
  unsigned* base = cnt + E;            // [E]
  unsigned* bits = base + E;           // [E][kWords]
  unsigned* wpre = bits + E * kWords;  // [E][kWords]
  unsigned* chunk = wpre + E * kWords; // [E]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_trigger();
  pdl_wait();

  for (int e = tid; e < E; e += kPermThreads) cnt[e] = 0;
  __syncthreads();
  unsigned bad = 0;
  for (int i = tid; i < T * K; i += kPermThreads) {
    const int e = idx[i];
    if (e < 0 || e >= E) {
      bad = 1;
      continue;
    }
    atomicAdd(&cnt[e], 1u);
  }
  if (bad) atomicOr(reinterpret_cast<unsigned*>(meta + 1), 1u);
  __syncthreads();

  // Exclusive scan of counts (warp 0; E <= 256 -> 8 entries per lane).
  if (warp == 0) {
    const int per = (E + 31) / 32;
    unsigned local = 0, nact = 0;
    for (int q = 0; q < per; ++q) {
      const int e = lane * per + q;
      if (e < E) {
        local += cnt[e];
        nact += (cnt[e] > 0 && e >= e_begin && e < e_end) ? 1u : 0u;
      }
    }
    unsigned incl = local, inact = nact;
#pragma unroll
    for (int s = 1; s < 32; s <<= 1) {
      const unsigned o = __shfl_up_sync(kFullMask, incl, s);
      const unsigned oa = __shfl_up_sync(kFullMask, inact, s);
      if (lane >= s) {
        incl += o;
        inact += oa;
      }
    }
    unsigned run = incl - local, arun = inact - nact;
    for (int q = 0; q < per; ++q) {
      const int e = lane * per + q;
      if (e < E) {
        base[e] = run;
        counts[e] = (int32_t)cnt[e];
        offsets[e] = (int32_t)run;
        if (cnt[e] > 0 && e >= e_begin && e < e_end) active[arun++] = e;
        run += cnt[e];
      }
    }
    if (lane == 31) {
      offsets[E] = (int32_t)incl;
      meta[0] = (int32_t)inact;
    }
  }
  __syncthreads();

  for (int c0 = 0; c0 < T; c0 += kPermThreads) {
    for (int i = tid; i < E * kWords; i += kPermThreads) bits[i] = 0;
    __syncthreads();
    const int t = c0 + tid;
    int my_e[8];
    if (t < T) {
      for (int r = 0; r < K; ++r) {
        const int e = idx[t * K + r];
        my_e[r] = e;
        if (e >= 0 && e < E) atomicOr(&bits[e * kWords + warp], 1u << lane);
      }
    }
    __syncthreads();
    for (int e = warp; e < E; e += kWords) {
      const unsigned v = __popc(bits[e * kWords + lane]);
      unsigned incl = v;
#pragma unroll
      for (int s = 1; s < 32; s <<= 1) {
        const unsigned o = __shfl_up_sync(kFullMask, incl, s);
        if (lane >= s) incl += o;
      }
      wpre[e * kWords + lane] = incl - v;
      if (lane == 31) chunk[e] = incl;
    }
    __syncthreads();
    if (t < T) {
      const unsigned below = (1u << lane) - 1u;
      for (int r = 0; r < K; ++r) {
        const int e = my_e[r];
        if (e < 0 || e >= E) continue;
        const unsigned pos = base[e] + wpre[e * kWords + warp] +
                             __popc(bits[e * kWords + warp] & below);
        perm[pos] = t * K + r;
        inv[t * K + r] = (int32_t)pos;
      }
    }
    __syncthreads();
    for (int e = tid; e < E; e += kPermThreads) base[e] += chunk[e];
    __syncthreads();
  }
}

}  // namespace

cudaError_t launch_permute(const Moe& m, const int32_t* idx, int64_t T, Workspace& ws,
                           cudaStream_t st) {
  const int E = m.desc.n_experts;
  const size_t smem = sizeof(unsigned) * ((size_t)3 * E + (size_t)2 * E * kWords);
  cudaError_t err = set_smem_limit(permute_kernel, smem);
  if (err != cudaSuccess) return err;
  return launch_pdl(permute_kernel, dim3(1), dim3(kPermThreads), smem, st, idx, (int)T, E,
                    m.desc.top_k, m.e_begin, m.e_end, ws.counts, ws.offsets, ws.active, ws.meta,
                    ws.perm, ws.inv);
}

}  // namespace gb
