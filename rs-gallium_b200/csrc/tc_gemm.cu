// tc_gemm.cu -- grouped MXFP4 expert GEMMs on the 5th-generation tensor cores.
//
// Reference math: gpt_oss.rs:189-221 (gate_up + bias, interleaved split,
// clamped SwiGLU, down + bias).  Prefill-sized batches run here.
//
// Precision.  Outputs must stay within 2e-2 of an f32 reference while they are
// O(10^2..10^3), so activations need ~22 significant bits.  Each activation is
// split into two f16 values, hi = f16(v') and lo = f16(v' - hi), where
// v' = v * 2^-s puts the row's largest magnitude in [2^14, 2^15).  Expert
// weights are exact in f16: an E2M1 code times 2^(e - rowmax + 13), where
// rowmax is the largest E8M0 byte of the weight row; the row's power of two
// 2^(rowmax - 140) and the activation's 2^s are applied in the epilogue.
// Two kind::f16 MMAs per K step accumulate the hi and lo products into two
// f32 TMEM accumulators (the small lo sum keeps its own rounding away from the
// large hi sum); the epilogue adds them.
//
// Tiles.  D[m, n] = sum_k W[m, k] * X[n, k]: M = 128 weight rows, N = 128
// grouped token rows of one expert, K stepped by 64 (two MXFP4 blocks).  A
// (weights) arrives as raw MXFP4 bytes by TMA and is decoded by four warps
// into shared memory in the canonical K-major 128-byte-swizzled layout, with
// the row's E8M0 bytes staged once per tile; B (activation hi / lo) arrives by
// TMA with the same swizzle.  Four pipeline stages of 52 KB; two TMEM
// accumulator pairs (512 columns) so the epilogue of one tile overlaps the
// MMAs of the next.  The grid is persistent (one CTA per SM) over work items
// (N tile, M tile), M fastest so concurrent CTAs share an expert's weights
// and token tile in L2.
//
// Warp roles (320 threads): 0-3 epilogue (TMEM lanes 0-127), 4-7 weight
// decode, 8 TMA producer, 9 MMA issuer.  Every mbarrier wait is bounded: on
// timeout the CTA raises an abort flag, records an error bit, lets in-flight
// copies land, frees its TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "moe_internal.h"
#include "ptx.cuh"
#include "umma.cuh"

namespace gb {
namespace tc {

constexpr int BM = 128, BN = 128, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;
constexpr int B_BYTES = BN * BK * 2;
constexpr int STAGE_BYTES = A_BYTES + 2 * B_BYTES;
constexpr int RAW_BYTES = BM * 32;  // one stage of MXFP4 weight bytes (two blocks per row)
constexpr int kScaleRow = 96;       // E8M0 bytes kept per row (K <= 3072)
constexpr int kThreads = 320;
constexpr int kTmemCols = 4 * BN;   // two buffers x (hi, lo) accumulators
constexpr size_t kSmemBytes =
    (size_t)STAGES * (STAGE_BYTES + RAW_BYTES) + BM * kScaleRow + 1024 + 256;

enum Mode { GATE_UP = 0, DOWN = 1 };

struct Args {
  const uint8_t* blocks;     // [E_loc][rows][K/32][16]
  const uint8_t* scales;     // [E_loc][rows][sp]
  const uint8_t* rowmax;     // [E_loc][rows]
  const float* bias;         // [E_loc][rows] or null
  int sp;
  int split_zero;            // 1: E8M0 byte 0 means 0 (safetensors); 0: 2^-127 (GGUF)
  int K;                     // reduction length (H for gate_up, I for down)
  int rows;                  // weight rows per expert (2I or H)
  int m_tiles;               // ceil(rows / BM)
  int e_begin;
  const int32_t* meta;       // [2] = number of N tiles
  const int32_t* tile_expert;
  const int32_t* tile_row0;
  const int32_t* tile_rows;
  const float* xscale;       // [positions] 2^s of the activation rows (GATE_UP), or null
  float limit;               // SwiGLU clamp
  __half* out_hi;            // GATE_UP: h hi [positions][I]
  __half* out_lo;            // GATE_UP: h lo
  float* out_y;              // DOWN: y [rows][H], row = out_rows[position] (or position)
  const int32_t* out_rows;
  int out_stride;            // I or H
  int* err;                  // error flags (bit 1: wait timed out)
};

// Instruction descriptor: kind::f16, A = B = f16, D = f32, both K-major,
// N = BN, M = BM.
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(kIdesc), "r"(accumulate)
      : "memory");
}

// f16 bits of 2^e for e in [-24, 15]; 0 below.
__device__ __forceinline__ uint32_t f16_pow2_bits(int e) {
  if (e >= -14) return (uint32_t)(e + 15) << 10;
  if (e >= -24) return 1u << (e + 24);
  return 0u;
}

// One 16-byte MXFP4 block (32 codes) times an f16 power of two -> 16 f16x2
// words in element order.
__device__ __forceinline__ void decode_block_f16(const uint4& q, uint32_t mult_bits,
                                                 uint32_t (&out)[16]) {
  const uint32_t m2 = mult_bits | (mult_bits << 16);
  const __half2 mh = *reinterpret_cast<const __half2*>(&m2);
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      uint32_t h = e2m1x2_to_f16x2((w[i] >> (8 * b)) & 0xffu);
      __half2 hv = __hmul2(*reinterpret_cast<const __half2*>(&h), mh);
      out[i * 4 + b] = *reinterpret_cast<const uint32_t*>(&hv);
    }
  }
}

// Work item -> (expert-local index, m tile, first position, valid rows).
struct Item {
  int le, m_tile, row0, nrows;
};

__device__ __forceinline__ Item decode_item(const Args& a, int item) {
  Item it;
  const int j = item / a.m_tiles;
  it.m_tile = item - j * a.m_tiles;
  it.le = a.tile_expert[j] - a.e_begin;
  it.row0 = a.tile_row0[j];
  it.nrows = a.tile_rows[j];
  return it;
}

// Epilogue of one tile: thread m owns TMEM lane m (weight row m of the M
// tile); hi_addr / lo_addr are this warp's lane-adjusted addresses of the hi
// and lo accumulators (NT columns each).  GATE_UP: bias, clamped SwiGLU of
// the neighbouring gate/up lanes, h split into f16 hi / lo; DOWN: bias, y.
template <int MODE, int NT>
__device__ __forceinline__ void epilogue_tile(const Args& a, const Item& it, uint32_t hi_addr,
                                              uint32_t lo_addr, int m) {
  const int row = it.m_tile * BM + m;
  const bool valid = row < a.rows;
  const int64_t grow = (int64_t)it.le * a.rows + (valid ? row : 0);
  const float row_f = valid ? pow2f((int)a.rowmax[grow] - 140) : 0.0f;
  const float bias = (valid && a.bias) ? a.bias[grow] : 0.0f;
#pragma unroll 1
  for (int c0 = 0; c0 < NT; c0 += 16) {
    uint32_t vh[16], vl[16];
    tmem_ld16(hi_addr + (uint32_t)c0, vh);
    tmem_ld16(lo_addr + (uint32_t)c0, vl);
    tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int n = c0 + j;
      const int64_t pos = (int64_t)it.row0 + n;
      float val = __fmul_rn(__fadd_rn(__uint_as_float(vh[j]), __uint_as_float(vl[j])), row_f);
      if (MODE == GATE_UP && n < it.nrows) val = __fmul_rn(val, pow2f((int)a.xscale[pos]));
      if (a.bias) val = __fadd_rn(val, bias);
      if (MODE == GATE_UP) {
        // rows 2i (gate) and 2i+1 (up) sit in neighbouring lanes
        const float up = __shfl_down_sync(kFullMask, val, 1);
        if ((m & 1) == 0 && valid && n < it.nrows) {
          const float h = act_gptoss(val, up, a.limit);
          const __half hi = __float2half_rn(h);
          const __half lo = __float2half_rn(__fsub_rn(h, __half2float(hi)));
          const int64_t o = pos * a.out_stride + (row >> 1);
          a.out_hi[o] = hi;
          a.out_lo[o] = lo;
        }
      } else {
        if (valid && n < it.nrows) {
          const int64_t orow = a.out_rows ? a.out_rows[pos] : pos;
          a.out_y[orow * a.out_stride + row] = val;
        }
      }
    }
  }
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    tc_expert_gemm(const __grid_constant__ CUtensorMap tmap_w,
                   const __grid_constant__ CUtensorMap tmap_hi,
                   const __grid_constant__ CUtensorMap tmap_lo, const Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* raw_w = smem + STAGES * STAGE_BYTES;         // [STAGES][128 rows][32 B]
  uint8_t* scale_s = raw_w + STAGES * RAW_BYTES;        // [128 rows][kScaleRow]
  uint64_t* tma_full = reinterpret_cast<uint64_t*>(scale_s + BM * kScaleRow);
  uint64_t* a_full = tma_full + STAGES;
  uint64_t* empty = a_full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total_items = a.meta[2] * a.m_tiles;
  const int nk = a.K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&tma_full[s], 1);  // producer's expect_tx arrival + transaction bytes
      mbar_init(&a_full[s], 128);  // decode threads
      mbar_init(&empty[s], 1);     // MMA commit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);     // MMA commit
      mbar_init(&acc_empty[b], 128);  // epilogue threads
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 8) {
    // ---------------- TMA producer: raw weight bytes, activation hi / lo -----
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < total_items && ok; item += gridDim.x) {
        const Item it = decode_item(a, item);
        const int wrow = it.le * a.rows + it.m_tile * BM;
        for (int kc = 0; kc < nk; ++kc) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, a.err)) {
            ok = false;
            break;
          }
          uint8_t* sb = smem + stage * STAGE_BYTES + A_BYTES;
          mbar_arrive_expect_tx(&tma_full[stage], RAW_BYTES + 2 * B_BYTES);
          tma_load_2d(raw_w + stage * RAW_BYTES, &tmap_w, kc * 32, wrow, &tma_full[stage]);
          tma_load_2d(sb, &tmap_hi, kc * BK, it.row0, &tma_full[stage]);
          tma_load_2d(sb + B_BYTES, &tmap_lo, kc * BK, it.row0, &tma_full[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // Let copies already issued land before the CTA leaves (they finish in
        // microseconds; 2 ms is a generous bound).
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 2000000ull) {
        }
      }
    }
  } else if (warp == 9) {
    // ---------------- MMA issuer ---------------------------------------------
    // Buffer b: hi accumulator at columns [b*2*BN, b*2*BN + BN), lo after it.
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc_iter = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < total_items && ok; item += gridDim.x, ++acc_iter) {
        const int b = acc_iter & 1;
        const uint32_t acc_phase = (acc_iter >> 1) & 1;
        if (!mbar_wait(&acc_empty[b], acc_phase ^ 1, abort_flag, a.err)) break;
        tc_fence_after();
        const uint32_t d_hi = tmem_base + (uint32_t)(b * 2 * BN);
        const uint32_t d_lo = d_hi + (uint32_t)BN;
        for (int kc = 0; kc < nk; ++kc) {
          if (!mbar_wait(&a_full[stage], phase, abort_flag, a.err) ||
              !mbar_wait(&tma_full[stage], phase, abort_flag, a.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t sh = sa + A_BYTES;
          const uint32_t sl = sh + B_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t da = sw128_desc(sa + kk * 32);
            const uint32_t acc = (kc | kk) != 0;
            mma_f16(d_hi, da, sw128_desc(sh + kk * 32), acc);
            mma_f16(d_lo, da, sw128_desc(sl + kk * 32), acc);
          }
          mma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) mma_commit(&acc_full[b]);
      }
      if (!ok || *abort_flag) {
        // MMAs already issued read shared memory and TMEM: let them finish.
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 2000000ull) {
        }
      }
    }
  } else if (warp >= 4) {
    // ---------------- weight decode: thread r owns row r of the M tile -------
    const int r = threadIdx.x - 128;
    uint8_t* my_scales = scale_s + r * kScaleRow;
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < total_items && ok; item += gridDim.x) {
      const Item it = decode_item(a, item);
      const int row = it.m_tile * BM + r;
      const bool valid = row < a.rows;
      const int64_t grow = (int64_t)it.le * a.rows + (valid ? row : 0);
      const int rmax = valid ? (int)a.rowmax[grow] : 0;
      // this row's E8M0 bytes for the whole tile, into this thread's smem slot
      {
        const uint4* src = reinterpret_cast<const uint4*>(a.scales + grow * a.sp);
        uint4* dst = reinterpret_cast<uint4*>(my_scales);
        for (int i = 0; i < a.sp / 16; ++i) dst[i] = valid ? __ldg(src + i) : make_uint4(0, 0, 0, 0);
      }
      for (int kc = 0; kc < nk; ++kc) {
        if (!mbar_wait(&tma_full[stage], phase, abort_flag, a.err)) {
          ok = false;
          break;
        }
        const uint4* rw = reinterpret_cast<const uint4*>(raw_w + stage * RAW_BYTES + r * 32);
        const uint4 q0 = rw[0], q1 = rw[1];
        const uint32_t s01 = *reinterpret_cast<const uint16_t*>(my_scales + 2 * kc);
        uint32_t w0[16], w1[16];
        {
          const int s0 = (int)(s01 & 0xffu), s1 = (int)(s01 >> 8);
          const uint32_t m0 =
              (!valid || (a.split_zero && s0 == 0)) ? 0u : f16_pow2_bits(s0 - rmax + 13);
          const uint32_t m1 =
              (!valid || (a.split_zero && s1 == 0)) ? 0u : f16_pow2_bits(s1 - rmax + 13);
          decode_block_f16(q0, m0, w0);
          decode_block_f16(q1, m1, w1);
        }
        uint8_t* sa = smem + stage * STAGE_BYTES;
        uint8_t* rowbase = sa + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint32_t* src = c < 4 ? &w0[c * 4] : &w1[(c - 4) * 4];
          *reinterpret_cast<uint4*>(rowbase + ((c ^ (r & 7)) << 4)) =
              make_uint4(src[0], src[1], src[2], src[3]);
        }
        fence_proxy_async_smem();
        mbar_arrive(&a_full[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else {
    // ---------------- epilogue: thread = TMEM lane = weight row ---------------
    const int m = threadIdx.x;  // 0..127
    int acc_iter = 0;
    for (int item = blockIdx.x; item < total_items; item += gridDim.x, ++acc_iter) {
      const int b = acc_iter & 1;
      const uint32_t acc_phase = (acc_iter >> 1) & 1;
      if (!mbar_wait(&acc_full[b], acc_phase, abort_flag, a.err)) break;
      tc_fence_after();
      const Item it = decode_item(a, item);
      const uint32_t hi_addr =
          tmem_base + ((uint32_t)(warp * 32) << 16) + (uint32_t)(b * 2 * BN);
      epilogue_tile<MODE, BN>(a, it, hi_addr, hi_addr + (uint32_t)BN, m);
      tc_fence_before();
      mbar_arrive(&acc_empty[b]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(kTmemCols));
  }
}


// x rows (gathered through perm) -> f16 hi / lo with a per-row power of two.
// xscale stores the exponent s as a float: x = 2^s * (hi + lo).
__global__ void split_gather_kernel(const float* __restrict__ x, const int32_t* __restrict__ perm,
                                    int top_k, int H, int positions, __half* __restrict__ xh,
                                    __half* __restrict__ xl, float* __restrict__ xscale) {
  __shared__ float red[32];
  const int p = blockIdx.x;
  if (p >= positions) return;
  const int tok = perm[p] / top_k;
  const float4* src = reinterpret_cast<const float4*>(x + (int64_t)tok * H);
  float mx = 0.0f;
  for (int i = threadIdx.x; i < H / 4; i += blockDim.x) {
    const float4 v = src[i];
    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFullMask, mx, s));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x < 32) {
    mx = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFullMask, mx, s));
    if (threadIdx.x == 0) red[0] = mx;
  }
  __syncthreads();
  mx = red[0];
  // s such that mx * 2^-s lies in [2^14, 2^15)
  int s = 0;
  if (mx > 0.0f && isfinite(mx)) {
    int ex;
    frexpf(mx, &ex);  // mx = f * 2^ex, f in [0.5, 1)
    s = ex - 15;
  }
  if (threadIdx.x == 0) xscale[p] = (float)s;
  __half2* dh = reinterpret_cast<__half2*>(xh + (int64_t)p * H);
  __half2* dl = reinterpret_cast<__half2*>(xl + (int64_t)p * H);
  for (int i = threadIdx.x; i < H / 4; i += blockDim.x) {
    const float4 v = src[i];
    const float a0 = ldexpf(v.x, -s), a1 = ldexpf(v.y, -s), a2 = ldexpf(v.z, -s),
                a3 = ldexpf(v.w, -s);
    const __half h0 = __float2half_rn(a0), h1 = __float2half_rn(a1), h2 = __float2half_rn(a2),
                 h3 = __float2half_rn(a3);
    dh[2 * i] = __halves2half2(h0, h1);
    dh[2 * i + 1] = __halves2half2(h2, h3);
    dl[2 * i] = __halves2half2(__float2half_rn(__fsub_rn(a0, __half2float(h0))),
                               __float2half_rn(__fsub_rn(a1, __half2float(h1))));
    dl[2 * i + 1] = __halves2half2(__float2half_rn(__fsub_rn(a2, __half2float(h2))),
                                   __float2half_rn(__fsub_rn(a3, __half2float(h3))));
  }
}

// N-tile table over the local experts: tile j covers grouped positions
// [row0, row0 + rows) of expert tile_expert[j], experts ascending.
// meta[2] = number of tiles.  One warp: lane l takes expert base + l, an
// exclusive warp scan of the tile counts places its tiles.
__global__ void tile_table_kernel(const int32_t* __restrict__ counts,
                                  const int32_t* __restrict__ offsets, int e_begin, int e_end,
                                  int bn, int32_t* __restrict__ meta,
                                  int32_t* __restrict__ tile_expert,
                                  int32_t* __restrict__ tile_row0, int32_t* __restrict__ tile_rows) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x;
  int base_j = 0;
  for (int e0 = e_begin; e0 < e_end; e0 += 32) {
    const int e = e0 + lane;
    const int c = e < e_end ? counts[e] : 0;
    const int off = e < e_end ? offsets[e] : 0;
    const int nt = (c + bn - 1) / bn;
    int incl = nt;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int v = __shfl_up_sync(kFullMask, incl, d);
      if (lane >= d) incl += v;
    }
    int j = base_j + incl - nt;
    for (int i = 0; i < c; i += bn, ++j) {
      tile_expert[j] = e;
      tile_row0[j] = off + i;
      tile_rows[j] = min(bn, c - i);
    }
    base_j += __shfl_sync(kFullMask, incl, 31);
  }
  if (lane == 0) meta[2] = base_j;
}

// Largest E8M0 byte of each weight row.
__global__ void rowmax_kernel(const uint8_t* __restrict__ scales, int sp, int nb, int64_t rows,
                              uint8_t* __restrict__ out) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  uint8_t mx = 0;
  for (int b = 0; b < nb; ++b) mx = max(mx, scales[r * sp + b]);
  out[r] = mx;
}

}  // namespace tc

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

bool tc_supported(const Moe& m) {
  const gb_moe_desc& d = m.desc;
  return d.act_kind == GB_ACT_GPTOSS_CLAMP && d.hidden % tc::BK == 0 && d.inter % tc::BK == 0 &&
         m.w.sp_h <= tc::kScaleRow && m.w.sp_i <= tc::kScaleRow && m.w.gu_rowmax != nullptr &&
         m.w.dn_rowmax != nullptr;
}

cudaError_t tc_prepare_weights(Moe& m) {
  const gb_moe_desc& d = m.desc;
  const int64_t nloc = m.e_end - m.e_begin;
  const int64_t gu_rows = nloc * 2 * d.inter, dn_rows = nloc * d.hidden;
  cudaError_t e = cudaMalloc(&m.w.gu_rowmax, (size_t)gu_rows);
  if (e != cudaSuccess) return e;
  e = cudaMalloc(&m.w.dn_rowmax, (size_t)dn_rows);
  if (e != cudaSuccess) return e;
  tc::rowmax_kernel<<<(unsigned)((gu_rows + 255) / 256), 256>>>(m.w.gu_scales, m.w.sp_h,
                                                                d.hidden / 32, gu_rows,
                                                                m.w.gu_rowmax);
  tc::rowmax_kernel<<<(unsigned)((dn_rows + 255) / 256), 256>>>(m.w.dn_scales, m.w.sp_i,
                                                                d.inter / 32, dn_rows,
                                                                m.w.dn_rowmax);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  // TMA descriptors of the raw weight bytes: [E_loc * rows][K / 2] u8, one
  // box = 128 rows x 32 bytes (two MXFP4 blocks of each row).
  auto encode = tensor_map_encoder();
  if (!encode) return cudaErrorNotSupported;
  auto make = [&](CUtensorMap* map, void* base, uint64_t row_bytes, uint64_t rows) -> cudaError_t {
    cuuint64_t dims[2] = {row_bytes, rows};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {32, tc::BM};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, base, dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
  };
  if ((e = make(reinterpret_cast<CUtensorMap*>(m.w.map_gu), m.w.gu_blocks, (uint64_t)d.hidden / 2,
                (uint64_t)gu_rows)) != cudaSuccess)
    return e;
  if ((e = make(reinterpret_cast<CUtensorMap*>(m.w.map_dn), m.w.dn_blocks, (uint64_t)d.inter / 2,
                (uint64_t)dn_rows)) != cudaSuccess)
    return e;
  return cudaDeviceSynchronize();
}

cudaError_t tc_make_maps(const Moe& m, ExpertBufs& eb) {
  auto encode = tensor_map_encoder();
  if (!encode) return cudaErrorNotSupported;
  const gb_moe_desc& d = m.desc;
  const uint64_t rows = (uint64_t)eb.rows_cap;
  // f16 [rows][K], one box = box_rows rows x 64 elements, 128-byte swizzle
  // (the canonical K-major layout the MMA descriptors expect).
  auto make = [&](void* map, void* base, uint64_t K, uint32_t box_rows) -> cudaError_t {
    cuuint64_t dims[2] = {K, rows};
    cuuint64_t strides[1] = {K * 2};
    cuuint32_t box[2] = {tc::BK, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode(reinterpret_cast<CUtensorMap*>(map), CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                        base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
  };
  cudaError_t e;
  if ((e = make(eb.map_xh, eb.xh, d.hidden, tc::BN)) != cudaSuccess) return e;
  if ((e = make(eb.map_xl, eb.xl, d.hidden, tc::BN)) != cudaSuccess) return e;
  if ((e = make(eb.map_hh, eb.hh, d.inter, tc::BN)) != cudaSuccess) return e;
  if ((e = make(eb.map_hl, eb.hl, d.inter, tc::BN)) != cudaSuccess) return e;
  if (d.weight_format != GB_FMT_Q4_K) return cudaSuccess;
  if ((e = make(eb.map_xh_s, eb.xh, d.hidden, kQ4SmallBox)) != cudaSuccess) return e;
  if ((e = make(eb.map_xl_s, eb.xl, d.hidden, kQ4SmallBox)) != cudaSuccess) return e;
  if ((e = make(eb.map_hh_s, eb.hh, d.inter, kQ4SmallBox)) != cudaSuccess) return e;
  return make(eb.map_hl_s, eb.hl, d.inter, kQ4SmallBox);
}

namespace {

tc::Args common_args(const Moe& m, const Groups& g, ExpertBufs& eb) {
  const gb_moe_desc& d = m.desc;
  tc::Args a{};
  a.split_zero = d.weight_format == GB_FMT_MXFP4_SPLIT ? 1 : 0;
  a.e_begin = m.e_begin;
  a.meta = g.meta;
  a.tile_expert = eb.tile_expert;
  a.tile_row0 = eb.tile_row0;
  a.tile_rows = eb.tile_rows;
  a.limit = d.swiglu_limit;
  a.err = g.meta + 1;
  return a;
}

template <int MODE>
cudaError_t launch_gemm(const Moe& m, const tc::Args& a, const void* map_w, const void* map_hi,
                        const void* map_lo, cudaStream_t st) {
  auto k = tc::tc_expert_gemm<MODE>;
  cudaError_t e = set_smem_limit(k, tc::kSmemBytes);
  if (e != cudaSuccess) return e;
  k<<<m.sm_count, tc::kThreads, tc::kSmemBytes, st>>>(*reinterpret_cast<const CUtensorMap*>(map_w),
                                                      *reinterpret_cast<const CUtensorMap*>(map_hi),
                                                      *reinterpret_cast<const CUtensorMap*>(map_lo),
                                                      a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_tile_table(const Moe& m, const Groups& g, int bn, ExpertBufs& eb,
                              cudaStream_t st) {
  return launch_pdl(tc::tile_table_kernel, dim3(1), dim3(32), 0, st, g.counts, g.offsets,
                    m.e_begin, m.e_end, bn, g.meta, eb.tile_expert, eb.tile_row0, eb.tile_rows);
}

cudaError_t launch_split_gather(const Moe& m, const Groups& g, const float* x, ExpertBufs& eb,
                                cudaStream_t st) {
  const int positions = (int)g.rows;
  if (positions <= 0) return cudaSuccess;
  tc::split_gather_kernel<<<positions, 256, 0, st>>>(x, g.perm, g.perm_div, m.desc.hidden,
                                                     positions, eb.xh, eb.xl, eb.xscale);
  return cudaGetLastError();
}

cudaError_t launch_tc_gate_up(const Moe& m, const Groups& g, const float* x, ExpertBufs& eb,
                              cudaStream_t st) {
  const gb_moe_desc& d = m.desc;
  cudaError_t e;
  if ((e = launch_tile_table(m, g, tc::BN, eb, st)) != cudaSuccess) return e;
  if ((e = launch_split_gather(m, g, x, eb, st)) != cudaSuccess) return e;
  tc::Args a = common_args(m, g, eb);
  a.blocks = m.w.gu_blocks;
  a.scales = m.w.gu_scales;
  a.rowmax = m.w.gu_rowmax;
  a.bias = m.w.gu_bias;
  a.sp = m.w.sp_h;
  a.K = d.hidden;
  a.rows = 2 * d.inter;
  a.m_tiles = (a.rows + tc::BM - 1) / tc::BM;
  a.xscale = eb.xscale;
  a.out_hi = eb.hh;
  a.out_lo = eb.hl;
  a.out_stride = d.inter;
  return launch_gemm<tc::GATE_UP>(m, a, m.w.map_gu, eb.map_xh, eb.map_xl, st);
}

cudaError_t launch_tc_down(const Moe& m, const Groups& g, ExpertBufs& eb, cudaStream_t st) {
  const gb_moe_desc& d = m.desc;
  tc::Args a = common_args(m, g, eb);
  a.blocks = m.w.dn_blocks;
  a.scales = m.w.dn_scales;
  a.rowmax = m.w.dn_rowmax;
  a.bias = m.w.dn_bias;
  a.sp = m.w.sp_i;
  a.K = d.inter;
  a.rows = d.hidden;
  a.m_tiles = (a.rows + tc::BM - 1) / tc::BM;
  a.out_y = eb.y;
  a.out_rows = g.out_rows;
  a.out_stride = d.hidden;
  return launch_gemm<tc::DOWN>(m, a, m.w.map_dn, eb.map_hh, eb.map_hl, st);
}

}  // namespace gb
