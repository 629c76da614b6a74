// dense_tc.cu -- grouped dense bf16 expert GEMMs on the 5th-generation tensor
// cores: gallium-core's generic MoEFFN (crates/gallium-core/src/ffn.rs:72-166)
// with GatedFFN experts (ffn.rs:30-67) stored in bf16, and its shared expert.
//
//   gate_up: h[p, i] = clamp(act(x_p . Wg[i]), -c, c) * (x_p . Wu[i])
//   down:    y[p, o] = h_p . Wd[o]
//
// Precision.  Weights are bf16 and enter the MMA exactly.  Activations are
// f32; each is split into two bf16 values, hi = bf16(v) and lo = bf16(v - hi)
// (16 significant bits, bf16 keeps f32's exponent range so no row scaling is
// needed), and two kind::f16 MMAs per K step accumulate the hi and lo
// products into two f32 TMEM accumulators that the epilogue adds.
//
// Tiles.  D[m, n] = sum_k W[m, k] * X[n, k]: M = 128 weight rows, N = the
// tile's grouped positions rounded up to 16 (at most 128; the MMA is only as
// wide as the tile), K stepped by 64 (one 128-byte swizzle atom of bf16).
// Weights arrive by TMA from the expert's rows as stored, except that gate
// and up rows are interleaved at load time (row 2i = gate i, row 2i + 1 =
// up i) so the epilogue pairs them in neighbouring TMEM lanes; activations
// (hi, lo) by TMA from the grouped buffers.  Four stages of 48 KB; two TMEM
// accumulator pairs (512 columns) so the epilogue of one tile overlaps the
// MMAs of the next.  Persistent grid (one CTA per SM) over work items (N
// tile, M tile), M fastest, so CTAs running together share an expert's token
// tile and read its weight tiles once from HBM.
//
// Warp roles (192 threads): 0-3 epilogue (TMEM lanes 0-127), 4 TMA producer,
// 5 MMA issuer.  Every mbarrier wait is bounded: on timeout the CTA raises an
// abort flag, records an error bit, lets in-flight copies and MMAs finish,
// frees its TMEM and returns.
#include <cuda.h>
#include <algorithm>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "moe_internal.h"
#include "ptx.cuh"
#include "umma.cuh"

namespace gb {
namespace dtc {

constexpr int BM = 128, BN = 128, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;
constexpr int B_BYTES = BN * BK * 2;
constexpr int STAGE_BYTES = A_BYTES + 2 * B_BYTES;
constexpr int kThreads = 192;
constexpr int kTmemCols = 4 * BN;  // two buffers x (hi, lo) accumulators
constexpr size_t kSmemBytes = (size_t)STAGES * STAGE_BYTES + 1024 + 256;

enum Mode { GATE_UP = 0, DOWN = 1 };

struct Args {
  int K;                     // reduction length (H for gate_up, I or Is for down)
  int rows;                  // weight rows per expert (2I interleaved, or H)
  int m_tiles;               // ceil(rows / BM)
  int e_begin;
  const int32_t* meta;       // [2] = number of N tiles (grouped mode)
  const int32_t* tile_expert;  // null: one expert, positions [0, uniform_rows)
  const int32_t* tile_row0;
  const int32_t* tile_rows;
  int uniform_rows;
  int act_kind;
  float clamp;
  __nv_bfloat16* out_hi;     // GATE_UP: h hi [positions][out_stride]
  __nv_bfloat16* out_lo;     // GATE_UP: h lo
  float* out_y;              // DOWN: y [rows][out_stride], row = out_rows[position] (or position)
  const int32_t* out_rows;
  int out_stride;
  const float* bias;         // DOWN: + bias[row] (nullable)
  int add_out;               // DOWN: y = y + (acc + bias) instead of y = acc + bias
  int ksplit;                // uniform DOWN only: K split into ksplit ranges (1 = none)
  float* part;               // ksplit > 1: raw sums [ksplit][uniform_rows][rows]
  int* err;                  // error flags (bit 1: wait timed out)
  uint64_t wait_ns;          // bound of every mbarrier wait
};

// Instruction descriptor: kind::f16, A = B = bf16, D = f32, both K-major,
// M = 128, N = n (a multiple of 16, 16..256).
__device__ __forceinline__ uint32_t idesc_bf16(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// The gate_up activation, fixed per kernel (SiLU without a clamp, the common
// case, or any gallium-core activation), so the unrolled epilogue holds one
// variant.
enum Act { ACT_SILU = 0, ACT_GENERIC = 1 };
// The down epilogue, fixed per kernel: the grouped expert rows (a plain
// store), or the plain-GEMM form of a linear layer (bias, residual add,
// split-K partials).  The down GEMM's tiles have few K steps, so its
// epilogue is on the critical path and carries no branch it does not need.
enum Epi { EPI_GROUPED = 0, EPI_LINEAR = 1 };

struct Item {
  int le, m_tile, row0, nrows, ks, k0, k1;  // k0 .. k1: the item's K steps
};

__device__ __forceinline__ int n_tiles(const Args& a) {
  return a.tile_expert ? a.meta[2] : (a.uniform_rows + BN - 1) / BN;
}

// SPLIT: the item index also carries a K range (the linear-layer form);
// otherwise every item covers all of K.
template <bool SPLIT>
__device__ __forceinline__ Item decode_item(const Args& a, int item) {
  Item it;
  const int nk = a.K / BK;
  if (SPLIT) {
    it.ks = item % a.ksplit;
    item /= a.ksplit;
    it.k0 = it.ks * nk / a.ksplit;
    it.k1 = (it.ks + 1) * nk / a.ksplit;
  } else {
    it.ks = 0;
    it.k0 = 0;
    it.k1 = nk;
  }
  const int j = item / a.m_tiles;
  it.m_tile = item - j * a.m_tiles;
  if (a.tile_expert) {
    it.le = a.tile_expert[j] - a.e_begin;
    it.row0 = a.tile_row0[j];
    it.nrows = a.tile_rows[j];
  } else {
    it.le = 0;
    it.row0 = j * BN;
    it.nrows = min(BN, a.uniform_rows - it.row0);
  }
  return it;
}

__device__ __forceinline__ int mma_cols(int nrows) { return (nrows + 15) & ~15; }


template <int ACT>
__device__ __forceinline__ float activation(const Args& a, float g) {
  if (ACT == ACT_SILU) return __fdiv_rn(g, __fadd_rn(expf(-g), 1.0f));
  return act_generic(a.act_kind, g, a.clamp);
}

// Epilogue of one tile: thread m owns TMEM lane m (weight row m of the M
// tile); hi_addr / lo_addr are this warp's lane-adjusted accumulator
// addresses.  GATE_UP: gate (even lane) and up (odd lane) -> h as bf16 hi /
// lo; DOWN: y.
template <int MODE, int ACT, int EPI>
__device__ __forceinline__ void epilogue_tile(const Args& a, const Item& it, uint32_t hi_addr,
                                              uint32_t lo_addr, int m) {
  const int row = it.m_tile * BM + m;
  const bool valid = row < a.rows;
  const int ncols = mma_cols(it.nrows);
  const float bias = (EPI == EPI_LINEAR && MODE == DOWN && a.bias && valid) ? a.bias[row] : 0.0f;
#pragma unroll 1
  for (int c0 = 0; c0 < ncols; c0 += 16) {
    uint32_t vh[16], vl[16];
    tmem_ld16(hi_addr + (uint32_t)c0, vh);
    tmem_ld16(lo_addr + (uint32_t)c0, vl);
    tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int n = c0 + j;
      const int64_t pos = (int64_t)it.row0 + n;
      const float val = __fadd_rn(__uint_as_float(vh[j]), __uint_as_float(vl[j]));
      if (MODE == GATE_UP) {
        const float up = __shfl_down_sync(kFullMask, val, 1);
        if ((m & 1) == 0 && valid && n < it.nrows) {
          const float h = __fmul_rn(activation<ACT>(a, val), up);
          const __nv_bfloat16 hi = __float2bfloat16_rn(h);
          const __nv_bfloat16 lo = __float2bfloat16_rn(__fsub_rn(h, __bfloat162float(hi)));
          const int64_t o = pos * a.out_stride + (row >> 1);
          a.out_hi[o] = hi;
          a.out_lo[o] = lo;
        }
      } else if (EPI == EPI_GROUPED) {
        if (valid && n < it.nrows) {
          const int64_t orow = a.out_rows ? a.out_rows[pos] : pos;
          a.out_y[orow * a.out_stride + row] = val;
        }
      } else if (valid && n < it.nrows) {
        if (a.ksplit > 1) {
          a.part[((int64_t)it.ks * a.uniform_rows + pos) * a.rows + row] = val;
        } else {
          float* o = a.out_y + pos * a.out_stride + row;
          float v = a.bias ? __fadd_rn(val, bias) : val;
          // the old value is read only when it is added to
          if (a.add_out) v = __fadd_rn(__ldcg(o), v);
          *o = v;
        }
      }
    }
  }
}

template <int MODE, int ACT, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    dense_tc_gemm(const __grid_constant__ CUtensorMap tmap_w,
                  const __grid_constant__ CUtensorMap tmap_hi,
                  const __grid_constant__ CUtensorMap tmap_lo, const Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total_items = n_tiles(a) * a.m_tiles * (EPI == EPI_LINEAR ? a.ksplit : 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);   // producer's expect_tx arrival + transaction bytes
      mbar_init(&empty[s], 1);  // MMA commit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);     // MMA commit
      mbar_init(&acc_empty[b], 128);  // epilogue threads
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 4) {
    // ---------------- TMA producer: weight rows, activation hi / lo ----------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < total_items && ok; item += gridDim.x) {
        const Item it = decode_item<EPI == EPI_LINEAR>(a, item);
        const int wrow = it.le * a.rows + it.m_tile * BM;
        for (int kc = it.k0; kc < it.k1; ++kc) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, a.err, a.wait_ns)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * STAGE_BYTES;
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          tma_load_2d(sa, &tmap_w, kc * BK, wrow, &full[stage]);
          tma_load_2d(sa + A_BYTES, &tmap_hi, kc * BK, it.row0, &full[stage]);
          tma_load_2d(sa + A_BYTES + B_BYTES, &tmap_lo, kc * BK, it.row0, &full[stage]);
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
  } else if (warp == 5) {
    // ---------------- MMA issuer ---------------------------------------------
    // Buffer b: hi accumulator at columns [b*2*BN, b*2*BN + BN), lo after it.
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc_iter = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < total_items && ok; item += gridDim.x, ++acc_iter) {
        const Item it = decode_item<EPI == EPI_LINEAR>(a, item);
        const uint32_t idesc = idesc_bf16(mma_cols(it.nrows));
        const int b = acc_iter & 1;
        const uint32_t acc_phase = (acc_iter >> 1) & 1;
        if (!mbar_wait(&acc_empty[b], acc_phase ^ 1, abort_flag, a.err, a.wait_ns)) break;
        tc_fence_after();
        const uint32_t d_hi = tmem_base + (uint32_t)(b * 2 * BN);
        const uint32_t d_lo = d_hi + (uint32_t)BN;
        for (int kc = it.k0; kc < it.k1; ++kc) {
          if (!mbar_wait(&full[stage], phase, abort_flag, a.err, a.wait_ns)) {
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
            const uint32_t acc = (kc != it.k0 || kk != 0) ? 1u : 0u;
            mma_bf16(d_hi, da, sw128_desc(sh + kk * 32), idesc, acc);
            mma_bf16(d_lo, da, sw128_desc(sl + kk * 32), idesc, acc);
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
  } else if (warp < 4) {
    // ---------------- epilogue: thread = TMEM lane = weight row ---------------
    const int m = threadIdx.x;  // 0..127
    int acc_iter = 0;
    for (int item = blockIdx.x; item < total_items; item += gridDim.x, ++acc_iter) {
      const int b = acc_iter & 1;
      const uint32_t acc_phase = (acc_iter >> 1) & 1;
      if (!mbar_wait(&acc_full[b], acc_phase, abort_flag, a.err, a.wait_ns)) break;
      tc_fence_after();
      const Item it = decode_item<EPI == EPI_LINEAR>(a, item);
      const uint32_t hi_addr =
          tmem_base + ((uint32_t)(warp * 32) << 16) + (uint32_t)(b * 2 * BN);
      epilogue_tile<MODE, ACT, EPI>(a, it, hi_addr, hi_addr + (uint32_t)BN, m);
      tc_fence_before();
      mbar_arrive(&acc_empty[b]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// Activation rows (gathered through perm, or in order when perm is null) ->
// bf16 hi / lo: x = hi + lo to 16 significant bits.
__global__ void split_bf16_kernel(const float* __restrict__ x, const int32_t* __restrict__ perm,
                                  int perm_div, int H, int positions,
                                  __nv_bfloat16* __restrict__ xh, __nv_bfloat16* __restrict__ xl) {
  const int p = blockIdx.x;
  if (p >= positions) return;
  const int64_t src_row = perm ? perm[p] / perm_div : p;
  const float4* src = reinterpret_cast<const float4*>(x + src_row * H);
  __nv_bfloat162* dh = reinterpret_cast<__nv_bfloat162*>(xh + (int64_t)p * H);
  __nv_bfloat162* dl = reinterpret_cast<__nv_bfloat162*>(xl + (int64_t)p * H);
  for (int i = threadIdx.x; i < H / 4; i += blockDim.x) {
    const float4 v = src[i];
    const float f[4] = {v.x, v.y, v.z, v.w};
    __nv_bfloat16 hi[4], lo[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      hi[j] = __float2bfloat16_rn(f[j]);
      lo[j] = __float2bfloat16_rn(__fsub_rn(f[j], __bfloat162float(hi[j])));
    }
    dh[2 * i] = __halves2bfloat162(hi[0], hi[1]);
    dh[2 * i + 1] = __halves2bfloat162(hi[2], hi[3]);
    dl[2 * i] = __halves2bfloat162(lo[0], lo[1]);
    dl[2 * i + 1] = __halves2bfloat162(lo[2], lo[3]);
  }
}

// out[p][r] = (add_out ? out[p][r] : 0) + ((sum over s of part[s][p][r], s
// ascending) + bias[r]): the split-K sums of the plain-GEMM form, folded in
// one fixed order.
__global__ void split_reduce_kernel(const float* __restrict__ part, int ksplit, int n_pos,
                                    int rows, const float* __restrict__ bias, float* __restrict__ out,
                                    int out_stride, int add_out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)n_pos * rows) return;
  const int p = (int)(i / rows), r = (int)(i - (int64_t)p * rows);
  float v = part[i];
  for (int s = 1; s < ksplit; ++s) v = __fadd_rn(v, part[(int64_t)s * n_pos * rows + i]);
  if (bias) v = __fadd_rn(v, bias[r]);
  float* o = out + (int64_t)p * out_stride + r;
  if (add_out) v = __fadd_rn(__ldcg(o), v);
  *o = v;
}

}  // namespace dtc

// bf16 [rows][K] row-major, one box = box_rows rows x 64 elements, 128-byte
// swizzle (the canonical K-major layout of the MMA descriptors).
cudaError_t make_bf16_map(void* map, const void* base, uint64_t K, uint64_t rows,
                          uint32_t box_rows) {
  auto encode = tensor_map_encoder();
  if (!encode) return cudaErrorNotSupported;
  cuuint64_t dims[2] = {K, rows};
  cuuint64_t strides[1] = {K * 2};
  cuuint32_t box[2] = {dtc::BK, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(reinterpret_cast<CUtensorMap*>(map), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                      const_cast<void*>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

namespace {

template <int MODE, int ACT, int EPI = dtc::EPI_GROUPED>
cudaError_t launch_gemm_act(int sm_count, const dtc::Args& a, const void* map_w,
                            const void* map_hi, const void* map_lo, cudaStream_t st) {
  auto k = dtc::dense_tc_gemm<MODE, ACT, EPI>;
  cudaError_t e = set_smem_limit(k, dtc::kSmemBytes);
  if (e != cudaSuccess) return e;
  k<<<sm_count, dtc::kThreads, dtc::kSmemBytes, st>>>(
      *reinterpret_cast<const CUtensorMap*>(map_w), *reinterpret_cast<const CUtensorMap*>(map_hi),
      *reinterpret_cast<const CUtensorMap*>(map_lo), a);
  return cudaGetLastError();
}

template <int MODE>
cudaError_t launch_gemm(int sm_count, const dtc::Args& a, const void* map_w, const void* map_hi,
                        const void* map_lo, cudaStream_t st) {
  if (MODE == dtc::GATE_UP && !(a.act_kind == GB_ACT_SILU && !(a.clamp > 0.0f)))
    return launch_gemm_act<MODE, dtc::ACT_GENERIC>(sm_count, a, map_w, map_hi, map_lo, st);
  return launch_gemm_act<MODE, dtc::ACT_SILU>(sm_count, a, map_w, map_hi, map_lo, st);
}

dtc::Args base_args(const Moe& m, int* err) {
  dtc::Args a{};
  a.ksplit = 1;
  a.e_begin = m.e_begin;
  a.act_kind = m.desc.act_kind;
  a.clamp = m.desc.act_clamp;
  a.err = err;
  a.wait_ns = m.test_wait_ns ? m.test_wait_ns : kMbarWaitNs;
  return a;
}

}  // namespace

cudaError_t split_rows(const float* x, const int32_t* perm, int perm_div, int H, int64_t positions,
                       __nv_bfloat16* xh, __nv_bfloat16* xl, cudaStream_t st) {
  if (positions <= 0) return cudaSuccess;
  dtc::split_bf16_kernel<<<(unsigned)positions, 256, 0, st>>>(x, perm, perm_div, H,
                                                              (int)positions, xh, xl);
  return cudaGetLastError();
}

cudaError_t launch_linear_tc(int sm_count, const void* map_w, const void* map_xh,
                             const void* map_xl, int K, int rows, int n_pos, const float* bias,
                             float* out, int out_stride, bool add_out, int* err, float* part,
                             int64_t part_floats, cudaStream_t st) {
  if (n_pos <= 0) return cudaSuccess;
  dtc::Args a{};
  a.err = err;
  a.wait_ns = kMbarWaitNs;
  a.uniform_rows = n_pos;
  a.K = K;
  a.rows = rows;
  a.m_tiles = (rows + dtc::BM - 1) / dtc::BM;
  a.out_y = out;
  a.out_stride = out_stride;
  a.bias = bias;
  a.add_out = add_out ? 1 : 0;
  // split K when the tiles alone would leave SMs idle: up to one item per
  // SM, at least four K steps per item, as the partial buffer allows
  const int tiles = a.m_tiles * ((n_pos + dtc::BN - 1) / dtc::BN);
  int ks = std::min((sm_count + tiles - 1) / tiles, std::max(1, (K / dtc::BK) / 4));
  if (part && part_floats > 0)
    ks = (int)std::min<int64_t>(ks, part_floats / ((int64_t)n_pos * rows));
  else
    ks = 1;
  a.ksplit = std::max(1, ks);
  a.part = part;
  cudaError_t e = launch_gemm_act<dtc::DOWN, dtc::ACT_SILU, dtc::EPI_LINEAR>(sm_count, a, map_w,
                                                                             map_xh, map_xl, st);
  if (e != cudaSuccess || a.ksplit == 1) return e;
  const int64_t n = (int64_t)n_pos * rows;
  dtc::split_reduce_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(
      part, a.ksplit, n_pos, rows, bias, out, out_stride, add_out ? 1 : 0);
  return cudaGetLastError();
}

bool dense_tc_supported(const Moe& m) {
  const gb_moe_desc& d = m.desc;
  return d.weight_format == GB_FMT_DENSE && m.w.dense_bf16 && d.hidden % dtc::BK == 0 &&
         d.inter % dtc::BK == 0 && tensor_map_encoder() != nullptr;
}

bool dense_tc_shared_supported(const Moe& m) {
  return dense_tc_supported(m) && m.desc.shared_inter > 0 && m.desc.shared_inter % dtc::BK == 0;
}

cudaError_t dense_tc_prepare(Moe& m) {
  const gb_moe_desc& d = m.desc;
  const uint64_t nloc = (uint64_t)(m.e_end - m.e_begin), H = d.hidden, I = d.inter;
  cudaError_t e;
  if ((e = make_bf16_map(m.w.map_dense_gu, m.w.dense_gu, H, nloc * 2 * I, dtc::BM)) != cudaSuccess)
    return e;
  if ((e = make_bf16_map(m.w.map_dense_dn, m.w.dense_down, I, nloc * H, dtc::BM)) != cudaSuccess)
    return e;
  if (dense_tc_shared_supported(m)) {
    const uint64_t Is = d.shared_inter;
    if ((e = make_bf16_map(m.w.map_sh_gu, m.w.sh_gu, H, 2 * Is, dtc::BM)) != cudaSuccess) return e;
    if ((e = make_bf16_map(m.w.map_sh_dn, m.w.sh_down, Is, H, dtc::BM)) != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t dense_tc_make_maps(const Moe& m, ExpertBufs& eb) {
  const gb_moe_desc& d = m.desc;
  const uint64_t rows = (uint64_t)eb.rows_cap;
  cudaError_t e;
  if ((e = make_bf16_map(eb.map_xh, eb.xh, d.hidden, rows, dtc::BN)) != cudaSuccess) return e;
  if ((e = make_bf16_map(eb.map_xl, eb.xl, d.hidden, rows, dtc::BN)) != cudaSuccess) return e;
  if ((e = make_bf16_map(eb.map_hh, eb.hh, d.inter, rows, dtc::BN)) != cudaSuccess) return e;
  return make_bf16_map(eb.map_hl, eb.hl, d.inter, rows, dtc::BN);
}

cudaError_t dense_tc_make_ws_maps(const Moe& m, Workspace& ws) {
  const gb_moe_desc& d = m.desc;
  const uint64_t T = (uint64_t)ws.tokens;
  cudaError_t e;
  if ((e = make_bf16_map(ws.map_sh_xh, ws.sh_xh, d.hidden, T, dtc::BN)) != cudaSuccess) return e;
  if ((e = make_bf16_map(ws.map_sh_xl, ws.sh_xl, d.hidden, T, dtc::BN)) != cudaSuccess) return e;
  if ((e = make_bf16_map(ws.map_sh_hh, ws.sh_hh, d.shared_inter, T, dtc::BN)) != cudaSuccess)
    return e;
  return make_bf16_map(ws.map_sh_hl, ws.sh_hl, d.shared_inter, T, dtc::BN);
}

cudaError_t launch_dense_tc_gate_up(const Moe& m, const Groups& g, const float* x,
                                    ExpertBufs& eb, cudaStream_t st) {
  const gb_moe_desc& d = m.desc;
  cudaError_t e;
  if ((e = launch_tile_table(m, g, dtc::BN, eb, st)) != cudaSuccess) return e;
  auto* xh = reinterpret_cast<__nv_bfloat16*>(eb.xh);
  auto* xl = reinterpret_cast<__nv_bfloat16*>(eb.xl);
  if ((e = split_rows(x, g.perm, g.perm_div, d.hidden, g.rows, xh, xl, st)) != cudaSuccess)
    return e;
  dtc::Args a = base_args(m, g.meta + 1);
  a.meta = g.meta;
  a.tile_expert = eb.tile_expert;
  a.tile_row0 = eb.tile_row0;
  a.tile_rows = eb.tile_rows;
  a.K = d.hidden;
  a.rows = 2 * d.inter;
  a.m_tiles = (a.rows + dtc::BM - 1) / dtc::BM;
  a.out_hi = reinterpret_cast<__nv_bfloat16*>(eb.hh);
  a.out_lo = reinterpret_cast<__nv_bfloat16*>(eb.hl);
  a.out_stride = d.inter;
  return launch_gemm<dtc::GATE_UP>(m.sm_count, a, m.w.map_dense_gu, eb.map_xh, eb.map_xl, st);
}

cudaError_t launch_dense_tc_down(const Moe& m, const Groups& g, ExpertBufs& eb, cudaStream_t st) {
  const gb_moe_desc& d = m.desc;
  dtc::Args a = base_args(m, g.meta + 1);
  a.meta = g.meta;
  a.tile_expert = eb.tile_expert;
  a.tile_row0 = eb.tile_row0;
  a.tile_rows = eb.tile_rows;
  a.K = d.inter;
  a.rows = d.hidden;
  a.m_tiles = (a.rows + dtc::BM - 1) / dtc::BM;
  a.out_y = eb.y;
  a.out_rows = g.out_rows;
  a.out_stride = d.hidden;
  return launch_gemm<dtc::DOWN>(m.sm_count, a, m.w.map_dense_dn, eb.map_hh, eb.map_hl, st);
}

cudaError_t launch_shared_expert_tc(const Moe& m, const float* x, int64_t T, float* y,
                                    cudaStream_t st) {
  const gb_moe_desc& d = m.desc;
  if (T <= 0) return cudaSuccess;
  const Workspace& ws = m.ws;
  cudaError_t e;
  if ((e = split_rows(x, nullptr, 1, d.hidden, T, ws.sh_xh, ws.sh_xl, st)) != cudaSuccess)
    return e;
  dtc::Args a = base_args(m, ws.meta + 1);
  a.uniform_rows = (int)T;
  a.K = d.hidden;
  a.rows = 2 * d.shared_inter;
  a.m_tiles = (a.rows + dtc::BM - 1) / dtc::BM;
  a.out_hi = ws.sh_hh;
  a.out_lo = ws.sh_hl;
  a.out_stride = d.shared_inter;
  if ((e = launch_gemm<dtc::GATE_UP>(m.sm_count, a, m.w.map_sh_gu, ws.map_sh_xh, ws.map_sh_xl, st)) !=
      cudaSuccess)
    return e;
  dtc::Args b = base_args(m, ws.meta + 1);
  b.uniform_rows = (int)T;
  b.K = d.shared_inter;
  b.rows = d.hidden;
  b.m_tiles = (b.rows + dtc::BM - 1) / dtc::BM;
  b.out_y = y;
  b.out_stride = d.hidden;
  return launch_gemm<dtc::DOWN>(m.sm_count, b, m.w.map_sh_dn, ws.map_sh_hh, ws.map_sh_hl, st);
}

}  // namespace gb
