// q4k_tc.cu -- grouped Q4_K expert GEMMs on the tensor cores (LFM2.5 batches
// of at least 2 rows per expert).
//
// Reference math: lfm2moe_q.rs:279-296 (h = silu(x Wg^T) * (x Wu^T), y =
// h Wd^T, no biases) over candle's Q4_K dequantiser (quantized.rs:162-177):
// element j of sub-block s of a 144-byte super-block is w = d1 * q - m1 with
// d1 = d * sc_s and m1 = dmin * m_s, each product rounded to f32.
//
// Precision.  w carries up to 21 significant bits, so it goes onto the tensor
// cores as two f16 values: w' = w * 2^e (e per expert, so that |w'| <= 2^14),
// hi = f16(w'), lo = f16(w' - hi).  Activations are split the same way as on
// the MXFP4 kind::f16 path (x' = x * 2^-s, hi + lo).  Three kind::f16 MMAs per
// K step: A_hi * B_hi into one TMEM accumulator, A_hi * B_lo and A_lo * B_hi
// into a second (the small terms keep their own rounding); the epilogue adds
// them and applies 2^-e and 2^s.
//
// Tiles and roles follow tc_gemm.cu: D[m, n] = sum_k W[m, k] X[n, k] with
// M = 128 weight rows, N = 128 grouped positions of one expert, K stepped by
// 64 (one Q4_K sub-block pair).  Warps 4-11 decode, as two groups taking
// alternate K steps: thread r of a group loads row r's super-block header
// and 32 quant bytes straight from HBM (its next three steps' bytes in
// flight, six K steps ahead, in a register ring walked with compile-time
// slots) and, once the MMAs have released the stage, decodes both
// sub-blocks into A hi / lo in shared memory in the K-major
// 128-byte-swizzled layout (decoding, not the MMAs, bounds this kernel,
// hence eight warps);
// warp 12 copies B hi / lo by TMA; warp 13 issues the MMAs; warps 0-3 run
// the epilogue (bias-free SiLU or clamped SwiGLU into h hi / lo, or y).  Three 64 KB stages; two TMEM
// accumulator pairs so the epilogue of one tile overlaps the next tile's MMAs.
// Every mbarrier wait is bounded (timeout -> abort flag, error bit 2, TMEM
// freed, return).
#include <cuda.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "moe_internal.h"
#include "ptx.cuh"
#include "umma.cuh"

namespace gb {
namespace q4tc {

constexpr int BM = 128, BN = 128, BK = 64, STAGES = 3;
constexpr int A_BYTES = BM * BK * 2;
constexpr int B_BYTES = BN * BK * 2;
constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;  // A hi, A lo, B hi, B lo
constexpr int kThreads = 448;
constexpr int kDecoders = 256;  // two threads per weight row
constexpr int kTmemCols = 4 * BN;  // two buffers x (hi, lo) accumulators
constexpr size_t kSmemBytes = (size_t)STAGES * STAGE_BYTES + 1024 + 256;

enum Mode { GATE_UP = 0, DOWN = 1 };

struct Args {
  const uint8_t* q;       // tiled copy: [E_loc][m_tiles][K/256][128 * 144] (tiled_row)
  const int32_t* wexp;    // [E_loc] decode scale exponent e
  int K;
  int rows;               // 2I (gate/up interleaved) or H
  int m_tiles;
  int e_begin;
  const int32_t* meta;    // [2] = number of N tiles
  const int32_t* tile_expert;
  const int32_t* tile_row0;
  const int32_t* tile_rows;
  const float* xscale;    // GATE_UP: exponent s of each position's row
  int act_kind;
  float clamp;  // act_clamp
  float limit;
  __half* out_hi;         // GATE_UP: h hi [positions][I]
  __half* out_lo;
  float* out_y;           // DOWN: y [rows][H], row = out_rows[position] (or position)
  const int32_t* out_rows;
  int out_stride;
  int* err;
  const float* xsum;      // small-batch kernel: [positions][K / 32] sub-block sums of B
};

// kind::f16, A = B = f16, D = f32, K-major, M = BM; N (bits 17-22) per tile:
// the tile's positions rounded up to 16 (decode-sized batches fill a tile
// with a few positions, and a full-width MMA would multiply empty ones).
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(BM >> 4) << 24);

__host__ __device__ constexpr uint32_t idesc_for(int rows) {
  return kIdesc | ((uint32_t)(((rows < 1 ? 1 : rows < BN ? rows : BN) + 15) & ~15) >> 3 << 17);
}
static_assert(idesc_for(0) == idesc_for(16) && idesc_for(8) == (kIdesc | (2u << 17)) &&
                  idesc_for(1000) == (kIdesc | ((uint32_t)(BN >> 3) << 17)),
              "MMA width: 16..BN in steps of 16");

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ float f16_bits_to_f32(uint32_t h) {
  const uint16_t b = (uint16_t)h;
  return __half2float(*reinterpret_cast<const __half*>(&b));
}

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

// The decoders read a tile-interleaved copy of each Q4_K matrix, made once at
// load (tile_q4k_kernel): per (local expert, 128-row tile, super-block) one
// block of 128 * 144 bytes holding the 16-byte headers of the tile's rows
// (row r at 16 r), then for each sub-block pair c its first and its second
// 16 quant bytes of every row (at 2048 + 4096 c and 4096 + 4096 c, row r at
// 16 r).  Decoder thread r loads row r, so each warp-wide 16-byte load reads
// 512 consecutive bytes, where rows of the GGUF layout lie a whole row of
// super-blocks apart (32 separate lines per warp load).  Rows past the
// matrix in the last tile are zero.
constexpr int kTileBlock = BM * 144;

// Row r of an item's tile at super-block 0 in the tiled copy.
__device__ __forceinline__ const uint8_t* tiled_row(const Args& a, const Item& it, int r,
                                                    int nsb) {
  return a.q + ((int64_t)it.le * a.m_tiles + it.m_tile) * nsb * kTileBlock + r * 16;
}

// K step kc's bytes of a row: the header of super-block kc / 4 and the 32
// quant bytes of sub-block pair kc % 4.
__device__ __forceinline__ void load_step(const uint8_t* tr, int kc, uint4& hdr, uint4& qa,
                                          uint4& qb) {
  const uint8_t* blk = tr + (int64_t)(kc >> 2) * kTileBlock;
  hdr = __ldg(reinterpret_cast<const uint4*>(blk));
  qa = __ldg(reinterpret_cast<const uint4*>(blk + 2048 + 4096 * (kc & 3)));
  qb = __ldg(reinterpret_cast<const uint4*>(blk + 4096 + 4096 * (kc & 3)));
}

// Scale and min of sub-block j = 2c + h of a super-block (candle's
// get_scale_min_k4), read from the header words by shifts: the twelve scale
// bytes are header bytes 4..15 (words y, z, w), so no byte array is indexed
// at run time (which would put the header in local memory).  c is a
// constant wherever the caller's loop is unrolled.
__device__ __forceinline__ void q4k_scale_min_hdr(const uint4& hdr, int c, int h, int& sc,
                                                  int& mn) {
  const int sh = 8 * ((2 * c + h) & 3);
  if (c < 2) {  // j < 4: sc = s[j] & 63, m = s[j + 4] & 63
    sc = (int)((hdr.y >> sh) & 63u);
    mn = (int)((hdr.z >> sh) & 63u);
  } else {  // j >= 4: from s[j + 4] (word w), s[j - 4] (word y) and s[j] (word z)
    const uint32_t b8 = (hdr.w >> sh) & 0xFFu, b0 = (hdr.y >> sh) & 0xFFu;
    const uint32_t b4 = (hdr.z >> sh) & 0xFFu;
    sc = (int)((b8 & 0xFu) | ((b0 >> 6) << 4));
    mn = (int)((b8 >> 4) | ((b4 >> 6) << 4));
  }
}

// Two f32 lanes in one 64-bit register, and the sm_100 paired f32 ops on
// them (each lane rounded to nearest like its scalar op).
__device__ __forceinline__ uint64_t f2_pack(float x, float y) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(x), "f"(y));
  return r;
}
__device__ __forceinline__ float2 f2_unpack(uint64_t r) {
  float2 v;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(v.x), "=f"(v.y) : "l"(r));
  return v;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t x, uint64_t y) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(x), "l"(y));
  return r;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t x, uint64_t y) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(x), "l"(y));
  return r;
}

// The 32 values of sub-block 2c + h of a super-block (h = 0: the low
// nibbles of the pair's 32 quant bytes, 1: the high nibbles) times 2^e, as
// f16 hi / lo pairs packed two per word in element order.
//
// Each nibble q, sitting at bit 8k of its word (k = 0, 1, 2), becomes the
// float 2^23 + q 2^8k by OR-ing in the exponent of 2^23 (one logic op, no
// int-to-float conversion); subtracting 2^23 leaves q 2^8k exactly, and
// multiplying by d1 2^(e - 8k) gives the correctly rounded d1 q 2^e.  So every
// value is bit-identical to the reference's d1 * q - m1 (each product rounded
// to f32), times 2^e: powers of two are exact and commute with the roundings.
// Two elements go through each paired op.
__device__ __forceinline__ void decode_half(const uint4& hdr, const uint4& qa, const uint4& qb,
                                            int c, int h, float scale, uint32_t (&hi)[16],
                                            uint32_t (&lo)[16]) {
  const float d = f16_bits_to_f32(hdr.x & 0xFFFFu);
  const float dmin = f16_bits_to_f32(hdr.x >> 16);
  int sc, mn;
  q4k_scale_min_hdr(hdr, c, h, sc, mn);
  const float d0 = __fmul_rn(__fmul_rn(d, (float)sc), scale);  // d1 2^e
  const float m1 = __fmul_rn(__fmul_rn(dmin, (float)mn), scale);
  const uint64_t d_lo = f2_pack(d0, __fmul_rn(d0, 0x1p-8f));  // bytes 0, 1 of a word
  const float d16 = __fmul_rn(d0, 0x1p-16f);
  const uint64_t d_hi = f2_pack(d16, d16);  // bytes 2, 3 (byte 3 moved down to bit 16)
  const uint64_t mm = f2_pack(m1, m1);
  const uint64_t two23 = f2_pack(0x1p23f, 0x1p23f);
  const int shift = 4 * h;  // the wanted nibble of each byte moved to its low half
  const uint32_t words[8] = {qa.x >> shift, qa.y >> shift, qa.z >> shift, qa.w >> shift,
                             qb.x >> shift, qb.y >> shift, qb.z >> shift, qb.w >> shift};
#pragma unroll
  for (int i = 0; i < 16; ++i) {  // elements 2i, 2i + 1 of the sub-block: bytes 2i, 2i + 1
    const uint32_t w = words[i >> 1];
    uint32_t b0, b1;
    if ((i & 1) == 0) {
      b0 = (w & 0xFu) | 0x4B000000u;
      b1 = (w & 0xF00u) | 0x4B000000u;
    } else {
      b0 = (w & 0xF0000u) | 0x4B000000u;
      b1 = ((w >> 8) & 0xF0000u) | 0x4B000000u;
    }
    const uint64_t q = f2_sub(f2_pack(__uint_as_float(b0), __uint_as_float(b1)), two23);
    const uint64_t v = f2_sub(f2_mul(q, (i & 1) ? d_hi : d_lo), mm);
    const float2 vf = f2_unpack(v);
    const __half2 vh = __floats2half2_rn(vf.x, vf.y);
    const float2 back = __half22float2(vh);
    const float2 rf = f2_unpack(f2_sub(v, f2_pack(back.x, back.y)));
    const __half2 vl = __floats2half2_rn(rf.x, rf.y);
    hi[i] = *reinterpret_cast<const uint32_t*>(&vh);
    lo[i] = *reinterpret_cast<const uint32_t*>(&vl);
  }
}

// The activation of the gate_up epilogue, fixed per kernel so that the
// unrolled epilogue holds one variant (the code of all of them, unrolled
// sixteen times, crowded the decode warps out of the instruction cache:
// gate_up at 2048 tokens took 910 instead of 770 us).
enum Act { ACT_GPTOSS = 0, ACT_SILU = 1, ACT_GENERIC = 2 };

template <int ACT>
__device__ __forceinline__ float activation(const Args& a, float g, float u) {
  if (ACT == ACT_GPTOSS) return act_gptoss(g, u, a.limit);
  if (ACT == ACT_SILU) return act_silu(g, u);
  return __fmul_rn(act_generic(a.act_kind, g, a.clamp), u);
}

// Thread m holds TMEM lane m (weight row m of the tile) for the tile's
// columns (positions).  The per-column factors (2^s of each position, or its
// output row) are read for sixteen columns at a time before that chunk's
// stores.  For gate_up, rows 2i (gate) and 2i + 1 (up) sit in neighbouring
// lanes; the pair swaps one value per two columns so that the even lane
// finishes column j and the odd lane column j + 1, each lane computing the
// activation of half the columns (the same values and roundings as one lane
// doing them all).
template <int MODE, int ACT>
__device__ __forceinline__ void epilogue_tile(const Args& a, const Item& it, uint32_t hi_addr,
                                              uint32_t lo_addr, int m) {
  const int row = it.m_tile * BM + m;
  const bool valid = row < a.rows;
  const float row_f = pow2f(-a.wexp[it.le]);
  const int odd = m & 1;
#pragma unroll 1
  for (int c0 = 0; c0 < it.nrows; c0 += 16) {  // the columns the MMAs wrote
    uint32_t vh[16], vl[16];
    tmem_ld16(hi_addr + (uint32_t)c0, vh);
    tmem_ld16(lo_addr + (uint32_t)c0, vl);
    float colf[16];
    int64_t orow[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int n = c0 + j;
      const int64_t pos = (int64_t)it.row0 + n;
      if (MODE == GATE_UP) {
        colf[j] = n < it.nrows ? pow2f((int)__ldg(a.xscale + pos)) : 1.0f;
      } else {
        orow[j] = n < it.nrows ? (a.out_rows ? (int64_t)__ldg(a.out_rows + pos) : pos) : 0;
      }
    }
    tmem_wait_ld();
    if (MODE == GATE_UP) {
#pragma unroll
      for (int j = 0; j < 16; j += 2) {
        const float v0 = __fmul_rn(
            __fmul_rn(__fadd_rn(__uint_as_float(vh[j]), __uint_as_float(vl[j])), row_f), colf[j]);
        const float v1 = __fmul_rn(
            __fmul_rn(__fadd_rn(__uint_as_float(vh[j + 1]), __uint_as_float(vl[j + 1])), row_f),
            colf[j + 1]);
        const float recv = __shfl_xor_sync(kFullMask, odd ? v0 : v1, 1);
        const float g = odd ? recv : v0;
        const float u = odd ? v1 : recv;
        const int n = c0 + j + odd;
        if (valid && n < it.nrows) {
          const float h = activation<ACT>(a, g, u);
          const __half hi = __float2half_rn(h);
          const __half lo = __float2half_rn(__fsub_rn(h, __half2float(hi)));
          const int64_t o = ((int64_t)it.row0 + n) * a.out_stride + (row >> 1);
          a.out_hi[o] = hi;
          a.out_lo[o] = lo;
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float val =
            __fmul_rn(__fadd_rn(__uint_as_float(vh[j]), __uint_as_float(vl[j])), row_f);
        if (valid && c0 + j < it.nrows) a.out_y[orow[j] * a.out_stride + row] = val;
      }
    }
  }
}

template <int MODE, int ACT>
__global__ void __launch_bounds__(kThreads, 1)
    q4k_tc_gemm(const __grid_constant__ CUtensorMap tmap_hi,
                const __grid_constant__ CUtensorMap tmap_lo, const Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* tma_full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
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
      mbar_init(&tma_full[s], 1);
      mbar_init(&a_full[s], kDecoders / 2);  // one decoder group per stage
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 12) {
    // ---------------- TMA producer: activation hi / lo -----------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < total_items && ok; item += gridDim.x) {
        const Item it = decode_item(a, item);
        for (int kc = 0; kc < nk; ++kc) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, a.err)) {
            ok = false;
            break;
          }
          uint8_t* sb = smem + stage * STAGE_BYTES + 2 * A_BYTES;
          mbar_arrive_expect_tx(&tma_full[stage], 2 * B_BYTES);
          tma_load_2d(sb, &tmap_hi, kc * BK, it.row0, &tma_full[stage]);
          tma_load_2d(sb + B_BYTES, &tmap_lo, kc * BK, it.row0, &tma_full[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 2000000ull) {
        }
      }
    }
  } else if (warp == 13) {
    // ---------------- MMA issuer ---------------------------------------------
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
        // (B hi and B lo as one 256-row operand, A hi meeting both in one
        // MMA, measured slower: 585 vs 560 us for gate_up at 2048 tokens)
        const uint32_t idesc = idesc_for(decode_item(a, item).nrows);
        for (int kc = 0; kc < nk; ++kc) {
          if (!mbar_wait(&a_full[stage], phase, abort_flag, a.err) ||
              !mbar_wait(&tma_full[stage], phase, abort_flag, a.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sah = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t sal = sah + A_BYTES;
          const uint32_t sbh = sal + A_BYTES;
          const uint32_t sbl = sbh + B_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t dah = sw128_desc(sah + kk * 32), dal = sw128_desc(sal + kk * 32);
            const uint64_t dbh = sw128_desc(sbh + kk * 32), dbl = sw128_desc(sbl + kk * 32);
            const uint32_t acc = (kc | kk) != 0;
            mma_f16(d_hi, dah, dbh, idesc, acc);
            mma_f16(d_lo, dah, dbl, idesc, acc);
            mma_f16(d_lo, dal, dbh, idesc, 1u);
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
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 2000000ull) {
        }
      }
    }
  } else if (warp >= 4) {
    // ---------------- weight decode --------------------------------------------
    // Group g = 0, 1 (warps 4-7, 8-11) takes the K steps of parity g; thread
    // r of a group decodes both sub-blocks of row r in its steps, so its ring
    // of four steps of bytes reaches six K steps ahead of the MMAs.  The ring
    // is walked with compile-time slots, so no register copy waits for a
    // load still in flight.
    const int r = (threadIdx.x - 128) & 127;
    const int grp = (threadIdx.x - 128) >> 7;
    const int nsb = a.K >> 8;  // super-blocks per row
    const int nks = nk / 2;  // K steps per group (nk is a multiple of four)
    int stage = grp;         // global step index gs = grp (mod 2), stage = gs % STAGES
    uint32_t phase = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < total_items && ok; item += gridDim.x) {
      const Item it = decode_item(a, item);
      const int row = it.m_tile * BM + r;
      const bool valid = row < a.rows;
      const uint8_t* tr = tiled_row(a, it, r, nsb);
      const float scale = valid ? pow2f(a.wexp[it.le]) : 0.0f;
      auto load = [&](int kc, uint4& hdr, uint4& qa, uint4& qb) { load_step(tr, kc, hdr, qa, qb); };
      uint4 hdr[4], qa[4], qb[4];
#pragma unroll
      for (int u = 0; u < 3; ++u)
        if (u < nks) load(grp + 2 * u, hdr[u], qa[u], qb[u]);
      for (int j0 = 0; j0 < nks && ok; j0 += 4) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int j = j0 + u;
          if (j < nks) {
            const int kc = grp + 2 * j;
            if (j + 3 < nks) load(kc + 6, hdr[(u + 3) & 3], qa[(u + 3) & 3], qb[(u + 3) & 3]);
            // the slot is free once the MMAs that read it have completed
            if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, a.err)) {
              ok = false;
              break;
            }
            uint8_t* sah = smem + stage * STAGE_BYTES;
            const int rb = (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
            for (int h = 0; h < 2; ++h) {  // sub-block 2c + h: chunks 4h .. 4h + 3 of the row
              uint32_t hi[16], lo[16];
              decode_half(hdr[u], qa[u], qb[u], kc & 3, h, scale, hi, lo);
#pragma unroll
              for (int cc = 0; cc < 4; ++cc) {
                const int off = rb + (((4 * h + cc) ^ (r & 7)) << 4);
                *reinterpret_cast<uint4*>(sah + off) =
                    make_uint4(hi[4 * cc], hi[4 * cc + 1], hi[4 * cc + 2], hi[4 * cc + 3]);
                *reinterpret_cast<uint4*>(sah + A_BYTES + off) =
                    make_uint4(lo[4 * cc], lo[4 * cc + 1], lo[4 * cc + 2], lo[4 * cc + 3]);
              }
            }
            fence_proxy_async_smem();
            mbar_arrive(&a_full[stage]);
            stage += 2;  // STAGES > 2: one wrap at most
            if (stage >= STAGES) {
              stage -= STAGES;
              phase ^= 1;
            }
          }
        }
      }
    }
  } else {
    // ---------------- epilogue: thread = TMEM lane = weight row ---------------
    const int m = threadIdx.x;
    int acc_iter = 0;
    for (int item = blockIdx.x; item < total_items; item += gridDim.x, ++acc_iter) {
      const int b = acc_iter & 1;
      const uint32_t acc_phase = (acc_iter >> 1) & 1;
      if (!mbar_wait(&acc_full[b], acc_phase, abort_flag, a.err)) break;
      tc_fence_after();
      const Item it = decode_item(a, item);
      const uint32_t hi_addr =
          tmem_base + ((uint32_t)(warp * 32) << 16) + (uint32_t)(b * 2 * BN);
      epilogue_tile<MODE, ACT>(a, it, hi_addr, hi_addr + (uint32_t)BN, m);
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

// ---------------------------------------------------------------------------
// Small batches (at most kSmallBN positions per tile): the weights go onto
// the tensor cores as the exact integers sc * q, one f16 each.
//
// Over one super-block (256 K) the weight of row r at k is
// d * (sc_s q_k) - dmin * m_s (s = k's sub-block), so
//   y[r][p] = sum_sb ( d_sb * A_sb[r][p] - dmin_sb * sum_s m_s * S[p][s] )
// with A_sb = sum over the super-block of (sc q) x (tcgen05, kind::f16; the
// tile's x rows as f16 hi and then as f16 lo make one B operand, so each MMA
// fills the hi and the lo columns of the accumulator at once) and S[p][s]
// the sub-block sums of x = hi + lo.  sc q <= 945 is exact in f16, so each weight costs one byte
// permute, one logic op and half a paired f16 FMA, where the f16 hi + lo
// decode of the kernel above costs about four times that; the MMAs read one
// A operand instead of two.  The epilogue warps read each super-block's
// accumulators out of TMEM and fold them into registers (one per position),
// so the tile is at most 32 positions wide.  The sums are the reference's
// dequantise-then-multiply regrouped (exact weights, x as hi + lo as in the
// kernel above); they differ from it by f32 rounding only.
//
// Roles as above: warps 4-11 decode, 12 copies B by TMA, 13 issues the MMAs,
// 0-3 fold the super-blocks and finish the tile.  Six 24 KB stages; two TMEM
// buffers of (hi, lo) accumulators so that one super-block's MMAs run while
// the previous one is folded.
constexpr int kSmallBN = 32;
constexpr int kSmallStages = 6;
// K steps of weight bytes in each decoder thread's register ring (six
// spilled registers and ran slower)
constexpr int kSmallRing = 4;
constexpr int SA_BYTES = BM * BK * 2;
constexpr int SB_BYTES = kSmallBN * BK * 2;
constexpr int SSTAGE_BYTES = SA_BYTES + 2 * SB_BYTES;  // A, B hi, B lo
constexpr int kSmallTmemCols = 4 * kSmallBN;           // 2 buffers x (hi, lo)

// B rows per operand half of a tile: its positions rounded up to 16.
__host__ __device__ constexpr int small_nh(int nrows) {
  return nrows <= kQ4SmallBox ? kQ4SmallBox : kSmallBN;
}

__host__ __device__ constexpr size_t small_smem_bytes(int K) {
  // stages, the tile's sub-block sums [kSmallBN][K / 32], barriers
  return (size_t)kSmallStages * SSTAGE_BYTES + (size_t)kSmallBN * (K / 32) * 4 + 1024 + 256;
}

// The 32 values sc * q of sub-block 2c + h of a super-block as f16, packed
// two per word in element order: byte b's nibble goes to a half of
// 0x6400 | q (the f16 1024 + q) and one paired FMA (1024 + q) sc - 1024 sc
// leaves sc q exactly (every intermediate is an integer below 2^16).
__device__ __forceinline__ void decode_int_half(const uint4& hdr, const uint4& qa, const uint4& qb,
                                                int c, int h, uint32_t (&v)[16]) {
  int sc, mn;
  q4k_scale_min_hdr(hdr, c, h, sc, mn);
  const __half2 s2 = __float2half2_rn((float)sc);
  const __half2 o2 = __float2half2_rn(-1024.0f * (float)sc);
  const int shift = 4 * h;
  const uint32_t words[8] = {qa.x >> shift, qa.y >> shift, qa.z >> shift, qa.w >> shift,
                             qb.x >> shift, qb.y >> shift, qb.z >> shift, qb.w >> shift};
#pragma unroll
  for (int i = 0; i < 16; ++i) {  // elements 2i, 2i + 1: bytes 2i, 2i + 1
    const uint32_t w = words[i >> 1];
    // bytes (0, 1) or (2, 3) of the word to bits 0-7 and 16-23
    const uint32_t r = __byte_perm(w, 0u, (i & 1) ? 0x4342u : 0x4140u);
    const uint32_t f = (r & 0x000F000Fu) | 0x64006400u;
    const __half2 x = __hfma2(*reinterpret_cast<const __half2*>(&f), s2, o2);
    v[i] = *reinterpret_cast<const uint32_t*>(&x);
  }
}

// Columns J0 .. J0 + NJ - 1 of one super-block folded into y: y[j] += d A[j]
// - dmin sum_s m_s S[j][s], A = hi + lo read from TMEM, S from shared memory.
// NJ is fixed at compile time and every column is folded: columns past the
// tile's positions compute values nobody stores (their S entries are stale
// shared memory), which costs less than a test per column.
template <int J0, int NJ>
__device__ __forceinline__ void fold16(uint32_t hi_addr, uint32_t lo_addr, float d, float dmin,
                                       const float (&mf)[8], const float* xs, int nsub, int sb,
                                       float (&y)[kSmallBN]) {
  static_assert(NJ == 8 || NJ == 16, "8 or 16 columns per fold");
  uint32_t vh[16], vl[16];
  tmem_ld16(hi_addr + (uint32_t)J0, vh);
  tmem_ld16(lo_addr + (uint32_t)J0, vl);
  tmem_wait_ld();
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    {
      const float4* sp = reinterpret_cast<const float4*>(xs + (J0 + j) * nsub + sb * 8);
      const float4 s0 = sp[0], s1 = sp[1];
      float t = mf[0] * s0.x;
      t = fmaf(mf[1], s0.y, t);
      t = fmaf(mf[2], s0.z, t);
      t = fmaf(mf[3], s0.w, t);
      t = fmaf(mf[4], s1.x, t);
      t = fmaf(mf[5], s1.y, t);
      t = fmaf(mf[6], s1.z, t);
      t = fmaf(mf[7], s1.w, t);
      const float acc = __uint_as_float(vh[j]) + __uint_as_float(vl[j]);
      y[J0 + j] += fmaf(d, acc, -dmin * t);
    }
  }
}

// The mins m_0 .. m_7 of a super-block from its header (get_scale_min_k4).
__device__ __forceinline__ void q4k_mins(const uint4& hdr, float (&mf)[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int sh = 8 * (j & 3);
    uint32_t mv;
    if (j < 4) {
      mv = (hdr.z >> sh) & 63u;
    } else {
      mv = ((hdr.w >> sh) >> 4 & 0xFu) | (((hdr.z >> sh) >> 6 & 3u) << 4);
    }
    mf[j] = (float)mv;
  }
}

template <int MODE, int ACT>
__global__ void __launch_bounds__(kThreads, 1)
    q4k_tc_small(const __grid_constant__ CUtensorMap tmap_hi,
                 const __grid_constant__ CUtensorMap tmap_lo, const Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int nsub = a.K / 32;
  float* xs = reinterpret_cast<float*>(smem + kSmallStages * SSTAGE_BYTES);  // [kSmallBN][nsub]
  uint64_t* tma_full = reinterpret_cast<uint64_t*>(xs + kSmallBN * nsub);
  uint64_t* a_full = tma_full + kSmallStages;
  uint64_t* empty = a_full + kSmallStages;
  uint64_t* acc_full = empty + kSmallStages;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total_items = a.meta[2] * a.m_tiles;
  const int nk = a.K / BK;
  const int nsb = a.K / 256;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSmallStages; ++s) {
      mbar_init(&tma_full[s], 1);
      mbar_init(&a_full[s], kDecoders / 2);  // one decoder group per stage
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) tmem_alloc(tmem_slot, kSmallTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 12) {
    // ---------------- TMA producer: B hi / lo ---------------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < total_items && ok; item += gridDim.x) {
        const Item it = decode_item(a, item);
        const int nh = small_nh(it.nrows);
        for (int kc = 0; kc < nk; ++kc) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, a.err)) {
            ok = false;
            break;
          }
          // the tile's nh hi rows, then its nh lo rows (16-row boxes)
          uint8_t* sb = smem + stage * SSTAGE_BYTES + SA_BYTES;
          mbar_arrive_expect_tx(&tma_full[stage], 2 * nh * BK * 2);
          for (int q = 0; q < nh; q += kQ4SmallBox) {
            tma_load_2d(sb + q * BK * 2, &tmap_hi, kc * BK, it.row0 + q, &tma_full[stage]);
            tma_load_2d(sb + (nh + q) * BK * 2, &tmap_lo, kc * BK, it.row0 + q, &tma_full[stage]);
          }
          if (++stage == kSmallStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 2000000ull) {
        }
      }
    }
  } else if (warp == 13) {
    // ---------------- MMA issuer: one accumulator pair per super-block --------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int sbi = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < total_items && ok; item += gridDim.x) {
        const int nh = small_nh(decode_item(a, item).nrows);
        const uint32_t idesc = kIdesc | ((uint32_t)(2 * nh) >> 3 << 17);  // N = hi + lo rows
        for (int sb = 0; sb < nsb && ok; ++sb, ++sbi) {
          const int b = sbi & 1;
          if (!mbar_wait(&acc_empty[b], ((sbi >> 1) & 1) ^ 1, abort_flag, a.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem_base + (uint32_t)(b * 2 * kSmallBN);  // hi cols, then lo
          for (int kq = 0; kq < 4; ++kq) {
            if (!mbar_wait(&a_full[stage], phase, abort_flag, a.err) ||
                !mbar_wait(&tma_full[stage], phase, abort_flag, a.err)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t sa = smem_u32(smem + stage * SSTAGE_BYTES);
            const uint32_t sbh = sa + SA_BYTES;
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk)  // one MMA over the hi and lo rows of B
              mma_f16(d, sw128_desc(sa + kk * 32), sw128_desc(sbh + kk * 32), idesc,
                      (kq | kk) != 0);
            mma_commit(&empty[stage]);
            if (++stage == kSmallStages) {
              stage = 0;
              phase ^= 1;
            }
          }
          if (ok) mma_commit(&acc_full[b]);
        }
      }
      if (!ok || *abort_flag) {
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 2000000ull) {
        }
      }
    }
  } else if (warp >= 4) {
    // ---------------- weight decode --------------------------------------------
    // Group g = 0, 1 (warps 4-7, 8-11) takes the K steps of parity g; thread
    // r of a group decodes both sub-blocks of row r in its steps.  Its ring
    // of kSmallRing steps of bytes then reaches 2 (kSmallRing - 1) K steps
    // ahead of the MMAs.
    const int r = (threadIdx.x - 128) & 127;
    const int grp = (threadIdx.x - 128) >> 7;
    const int nks = nk / 2;  // K steps per group (nk is a multiple of four)
    int stage = grp;         // global step index gs = grp (mod 2), stage = gs % 6
    uint32_t phase = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < total_items && ok; item += gridDim.x) {
      const Item it = decode_item(a, item);
      const uint8_t* tr = tiled_row(a, it, r, nsb);
      auto load = [&](int kc, uint4& hdr, uint4& qa, uint4& qb) { load_step(tr, kc, hdr, qa, qb); };
      uint4 hdr[kSmallRing], qa[kSmallRing], qb[kSmallRing];
#pragma unroll
      for (int u = 0; u < kSmallRing - 1; ++u)
        if (u < nks) load(grp + 2 * u, hdr[u], qa[u], qb[u]);
      for (int j0 = 0; j0 < nks && ok; j0 += kSmallRing) {
#pragma unroll
        for (int u = 0; u < kSmallRing; ++u) {
          const int j = j0 + u;
          if (j < nks) {
            const int kc = grp + 2 * j;
            constexpr int n = kSmallRing - 1;  // steps in flight ahead of this one
            if (j + n < nks)
              load(kc + 2 * n, hdr[(u + n) % kSmallRing], qa[(u + n) % kSmallRing],
                   qb[(u + n) % kSmallRing]);
            if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, a.err)) {
              ok = false;
              break;
            }
            uint8_t* sa = smem + stage * SSTAGE_BYTES + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
            for (int h = 0; h < 2; ++h) {  // sub-block 2c + h: chunks 4h .. 4h + 3 of the row
              uint32_t v[16];
              decode_int_half(hdr[u], qa[u], qb[u], kc & 3, h, v);
              // rows past the matrix are zero bytes in the tiled copy, so
              // they decode to zero (sc = 0) without a select here
#pragma unroll
              for (int cc = 0; cc < 4; ++cc)
                *reinterpret_cast<uint4*>(sa + (((4 * h + cc) ^ (r & 7)) << 4)) =
                    make_uint4(v[4 * cc], v[4 * cc + 1], v[4 * cc + 2], v[4 * cc + 3]);
            }
            fence_proxy_async_smem();
            mbar_arrive(&a_full[stage]);
            stage += 2;
            if (stage >= kSmallStages) {
              stage -= kSmallStages;
              phase ^= 1;
            }
          }
        }
      }
    }
  } else {
    // ---------------- epilogue: thread = TMEM lane = weight row ---------------
    const int m = threadIdx.x;
    const int odd = m & 1;
    int sbi = 0;
    bool ok = true;
    // every epilogue thread runs every item (the named barriers below need
    // all 128); after a failed wait a thread only walks the loops
    for (int item = blockIdx.x; item < total_items; item += gridDim.x) {
      const Item it = decode_item(a, item);
      const int row = it.m_tile * BM + m;
      const bool valid = row < a.rows;
      const int ncols = it.nrows < kSmallBN ? it.nrows : kSmallBN;
      // the tile's sub-block sums into shared memory (after every epilogue
      // thread has finished with the previous tile's)
      asm volatile("bar.sync 1, 128;" ::: "memory");
      {
        const float4* src = reinterpret_cast<const float4*>(a.xsum + (int64_t)it.row0 * nsub);
        float4* dst = reinterpret_cast<float4*>(xs);
        const int n4 = ncols * nsub / 4;
        for (int i = m; i < n4; i += 128) dst[i] = __ldg(src + i);
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      const uint8_t* hp = tiled_row(a, it, m, nsb);  // super-block headers, kTileBlock apart
      float y[kSmallBN];
#pragma unroll
      for (int j = 0; j < kSmallBN; ++j) y[j] = 0.0f;
      uint4 hnext = __ldg(reinterpret_cast<const uint4*>(hp));
      for (int sb = 0; sb < nsb; ++sb, ++sbi) {
        const uint4 hdr = hnext;
        if (sb + 1 < nsb)
          hnext = __ldg(reinterpret_cast<const uint4*>(hp + (int64_t)(sb + 1) * kTileBlock));
        const int b = sbi & 1;
        if (ok && !mbar_wait(&acc_full[b], (sbi >> 1) & 1, abort_flag, a.err)) ok = false;
        if (!ok) continue;
        tc_fence_after();
        const float d = f16_bits_to_f32(hdr.x & 0xFFFFu);
        const float dmin = f16_bits_to_f32(hdr.x >> 16);
        float mf[8];
        q4k_mins(hdr, mf);
        const uint32_t hi_addr =
            tmem_base + ((uint32_t)(warp * 32) << 16) + (uint32_t)(b * 2 * kSmallBN);
        const uint32_t lo_addr = hi_addr + (uint32_t)small_nh(it.nrows);
        if (ncols <= 8) {
          fold16<0, 8>(hi_addr, lo_addr, d, dmin, mf, xs, nsub, sb, y);
        } else {
          fold16<0, 16>(hi_addr, lo_addr, d, dmin, mf, xs, nsub, sb, y);
          if (ncols > 16) fold16<16, 16>(hi_addr, lo_addr, d, dmin, mf, xs, nsub, sb, y);
        }
        tc_fence_before();
        mbar_arrive(&acc_empty[b]);
      }
      if (!ok) continue;
      if (MODE == GATE_UP) {
        // rows 2i (gate) and 2i + 1 (up) in neighbouring lanes: the even lane
        // finishes column j, the odd lane column j + 1
#pragma unroll
        for (int j = 0; j < kSmallBN; j += 2) {
          if (j >= ncols) break;
          const int64_t p0 = (int64_t)it.row0 + j;
          const float v0 = j < ncols ? __fmul_rn(y[j], pow2f((int)__ldg(a.xscale + p0))) : 0.0f;
          const float v1 =
              j + 1 < ncols ? __fmul_rn(y[j + 1], pow2f((int)__ldg(a.xscale + p0 + 1))) : 0.0f;
          const float recv = __shfl_xor_sync(kFullMask, odd ? v0 : v1, 1);
          const float g = odd ? recv : v0;
          const float u = odd ? v1 : recv;
          const int n = j + odd;
          if (valid && n < ncols) {
            const float h = activation<ACT>(a, g, u);
            const __half hi = __float2half_rn(h);
            const __half lo = __float2half_rn(__fsub_rn(h, __half2float(hi)));
            const int64_t o = ((int64_t)it.row0 + n) * a.out_stride + (row >> 1);
            a.out_hi[o] = hi;
            a.out_lo[o] = lo;
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < kSmallBN; ++j) {
          if (j >= ncols) break;
          const int64_t pos = (int64_t)it.row0 + j;
          const int64_t orow = a.out_rows ? (int64_t)__ldg(a.out_rows + pos) : pos;
          if (valid) a.out_y[orow * a.out_stride + row] = y[j];
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kSmallTmemCols);
  }
}

// Decode exponent e of one local expert's matrix: the largest |d| * 63 * 15 +
// |dmin| * 63 over its super-blocks bounds |w|; e puts that bound at or below
// 2^14.  One CTA per local expert.
__global__ void wexp_kernel(const uint8_t* __restrict__ q, int64_t blocks_per_expert,
                            int32_t* __restrict__ wexp) {
  __shared__ float red[32];
  const int le = blockIdx.x;
  const uint8_t* base = q + (int64_t)le * blocks_per_expert * 144;
  float mx = 0.0f;
  for (int64_t b = threadIdx.x; b < blocks_per_expert; b += blockDim.x) {
    const uint8_t* blk = base + b * 144;
    const float d = fabsf(f16_bits_to_f32((uint32_t)blk[0] | ((uint32_t)blk[1] << 8)));
    const float dmin = fabsf(f16_bits_to_f32((uint32_t)blk[2] | ((uint32_t)blk[3] << 8)));
    const float bound = d * 945.0f + dmin * 63.0f;
    if (isfinite(bound)) mx = fmaxf(mx, bound);
  }
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFullMask, mx, s));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) mx = fmaxf(mx, red[w]);
    mx = fmaxf(mx, red[0]);
    int e = 0;
    if (mx > 0.0f) {
      int ex;
      frexpf(mx, &ex);  // mx < 2^ex
      e = 14 - ex;
    }
    wexp[le] = max(-60, min(60, e));
  }
}

// The tiled copy of one Q4_K matrix set ([n_exp][rows][nsb][144] in, layout
// at tiled_row out; the output is cleared beforehand for the padding rows):
// one thread per (expert, row, super-block) moves its nine 16-byte pieces.
__global__ void tile_q4k_kernel(const uint8_t* __restrict__ src, int rows, int nsb, int m_tiles,
                                int64_t n, uint8_t* __restrict__ dst) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= n) return;
  const int64_t er = t / nsb;  // expert * rows + row
  const int sb = (int)(t - er * nsb);
  const int64_t le = er / rows;
  const int row = (int)(er - le * rows);
  const uint4* s = reinterpret_cast<const uint4*>(src + t * 144);
  uint8_t* blk = dst + ((le * m_tiles + row / BM) * nsb + sb) * kTileBlock + (row % BM) * 16;
  *reinterpret_cast<uint4*>(blk) = __ldg(s);
#pragma unroll
  for (int j = 0; j < 8; ++j)  // quant bytes 16 j .. 16 j + 15: pair j / 2, half j % 2
    *reinterpret_cast<uint4*>(blk + 2048 + 2048 * j) = __ldg(s + 1 + j);
}

// Sub-block sums of the split rows: out[p][s] = sum over i < 32 of
// (hi + lo)[p][32 s + i], in order, in f32 (hi + lo is exact in f32).
__global__ void sub_sums_kernel(const __half* __restrict__ hi, const __half* __restrict__ lo,
                                int K, int64_t n, float* __restrict__ out) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= n) return;
  const int nsub = K / 32;
  const int64_t p = t / nsub;
  const int sub = (int)(t - p * nsub);
  const uint4* h4 = reinterpret_cast<const uint4*>(hi + p * K + sub * 32);
  const uint4* l4 = reinterpret_cast<const uint4*>(lo + p * K + sub * 32);
  float acc = 0.0f;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint4 hv = __ldg(h4 + c), lv = __ldg(l4 + c);
    const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w}, lw[4] = {lv.x, lv.y, lv.z, lv.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 hf = __half22float2(*reinterpret_cast<const __half2*>(&hw[e]));
      const float2 lf = __half22float2(*reinterpret_cast<const __half2*>(&lw[e]));
      acc = __fadd_rn(acc, __fadd_rn(hf.x, lf.x));
      acc = __fadd_rn(acc, __fadd_rn(hf.y, lf.y));
    }
  }
  out[t] = acc;
}

static_assert(kSmallBN == kQ4SmallBN, "small-batch tile width");
static_assert(kSmallStages % 2 == 0, "each decoder group keeps to its own stages");

}  // namespace q4tc

bool q4k_tc_supported(const Moe& m) {
  const gb_moe_desc& d = m.desc;
  return d.weight_format == GB_FMT_Q4_K && d.hidden % 256 == 0 && d.inter % 256 == 0 &&
         m.w.q4_gu_exp != nullptr && m.w.q4_gu_t != nullptr && m.w.q4_dn_t != nullptr;
}

namespace {

// The tiled copy of one matrix set (q4tc::tile_q4k_kernel), counted in the
// handle's weight bytes.
cudaError_t make_tiled(Moe& m, const uint8_t* src, int nloc, int rows, int K, uint8_t** out) {
  const int nsb = K / 256;
  const int m_tiles = (rows + q4tc::BM - 1) / q4tc::BM;
  const size_t bytes = (size_t)nloc * m_tiles * nsb * q4tc::kTileBlock;
  cudaError_t e = cudaMalloc(out, bytes);
  if (e != cudaSuccess) return e;
  m.weight_bytes += (int64_t)bytes;
  if ((e = cudaMemset(*out, 0, bytes)) != cudaSuccess) return e;
  const int64_t n = (int64_t)nloc * rows * nsb;
  q4tc::tile_q4k_kernel<<<(unsigned)((n + 255) / 256), 256>>>(src, rows, nsb, m_tiles, n, *out);
  return cudaGetLastError();
}

}  // namespace

cudaError_t q4k_tc_prepare(Moe& m) {
  const gb_moe_desc& d = m.desc;
  const int nloc = m.e_end - m.e_begin;
  if (d.weight_format != GB_FMT_Q4_K || nloc <= 0) return cudaSuccess;
  cudaError_t e = cudaMalloc(&m.w.q4_gu_exp, sizeof(int32_t) * 2 * (size_t)nloc);
  if (e != cudaSuccess) return e;
  m.w.q4_dn_exp = m.w.q4_gu_exp + nloc;
  q4tc::wexp_kernel<<<nloc, 256>>>(m.w.q4_gu, (int64_t)2 * d.inter * (d.hidden / 256),
                                   m.w.q4_gu_exp);
  q4tc::wexp_kernel<<<nloc, 256>>>(m.w.q4_dn, (int64_t)d.hidden * (d.inter / 256),
                                   m.w.q4_dn_exp);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  if (d.hidden % 256 == 0 && d.inter % 256 == 0) {
    if ((e = make_tiled(m, m.w.q4_gu, nloc, 2 * d.inter, d.hidden, &m.w.q4_gu_t)) != cudaSuccess)
      return e;
    if ((e = make_tiled(m, m.w.q4_dn, nloc, d.hidden, d.inter, &m.w.q4_dn_t)) != cudaSuccess)
      return e;
  }
  return cudaDeviceSynchronize();
}

namespace {

q4tc::Args q4tc_args(const Moe& m, const Groups& g, ExpertBufs& eb) {
  q4tc::Args a{};
  a.e_begin = m.e_begin;
  a.meta = g.meta;
  a.tile_expert = eb.tile_expert;
  a.tile_row0 = eb.tile_row0;
  a.tile_rows = eb.tile_rows;
  a.act_kind = m.desc.act_kind;
  a.clamp = m.desc.act_clamp;
  a.limit = m.desc.swiglu_limit;
  a.err = g.meta + 1;
  return a;
}

template <int MODE, int ACT>
cudaError_t launch_q4tc_act(const Moe& m, const q4tc::Args& a, const void* map_hi,
                            const void* map_lo, cudaStream_t st) {
  auto k = q4tc::q4k_tc_gemm<MODE, ACT>;
  cudaError_t e = set_smem_limit(k, q4tc::kSmemBytes);
  if (e != cudaSuccess) return e;
  k<<<m.sm_count, q4tc::kThreads, q4tc::kSmemBytes, st>>>(
      *reinterpret_cast<const CUtensorMap*>(map_hi), *reinterpret_cast<const CUtensorMap*>(map_lo),
      a);
  return cudaGetLastError();
}

template <int MODE, int ACT>
cudaError_t launch_q4tc_small_act(const Moe& m, const q4tc::Args& a, const void* map_hi,
                                  const void* map_lo, cudaStream_t st) {
  auto k = q4tc::q4k_tc_small<MODE, ACT>;
  const size_t smem = q4tc::small_smem_bytes(a.K);
  cudaError_t e = set_smem_limit(k, smem);
  if (e != cudaSuccess) return e;
  k<<<m.sm_count, q4tc::kThreads, smem, st>>>(*reinterpret_cast<const CUtensorMap*>(map_hi),
                                              *reinterpret_cast<const CUtensorMap*>(map_lo), a);
  return cudaGetLastError();
}

template <int MODE>
cudaError_t launch_q4tc_small(const Moe& m, const q4tc::Args& a, const void* map_hi,
                              const void* map_lo, cudaStream_t st) {
  if (MODE != q4tc::GATE_UP || a.act_kind == GB_ACT_GPTOSS_CLAMP)
    return launch_q4tc_small_act<MODE, q4tc::ACT_GPTOSS>(m, a, map_hi, map_lo, st);
  if (a.act_kind == GB_ACT_SILU && !(a.clamp > 0.0f))
    return launch_q4tc_small_act<MODE, q4tc::ACT_SILU>(m, a, map_hi, map_lo, st);
  return launch_q4tc_small_act<MODE, q4tc::ACT_GENERIC>(m, a, map_hi, map_lo, st);
}

cudaError_t launch_sub_sums(const __half* hi, const __half* lo, int K, int64_t positions,
                            float* out, cudaStream_t st) {
  const int64_t n = positions * (K / 32);
  if (n <= 0) return cudaSuccess;
  q4tc::sub_sums_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(hi, lo, K, n, out);
  return cudaGetLastError();
}

template <int MODE>
cudaError_t launch_q4tc(const Moe& m, const q4tc::Args& a, const void* map_hi, const void* map_lo,
                        cudaStream_t st) {
  if (MODE != q4tc::GATE_UP || a.act_kind == GB_ACT_GPTOSS_CLAMP)
    return launch_q4tc_act<MODE, q4tc::ACT_GPTOSS>(m, a, map_hi, map_lo, st);
  if (a.act_kind == GB_ACT_SILU && !(a.clamp > 0.0f))
    return launch_q4tc_act<MODE, q4tc::ACT_SILU>(m, a, map_hi, map_lo, st);
  return launch_q4tc_act<MODE, q4tc::ACT_GENERIC>(m, a, map_hi, map_lo, st);
}

}  // namespace

bool use_q4k_small(const Moe& m, const Groups& g) {
  const gb_moe_desc& d = m.desc;
  if (m.expert_path == GB_PATH_TENSOR_CORES_F16) return false;
  if (q4tc::small_smem_bytes(std::max(d.hidden, d.inter)) > (size_t)227 * 1024) return false;
  // up to 24 rows per expert on average: beyond that, folding 32-column
  // accumulators every super-block costs more than the f16 decode saves
  // (LFM2.5 layer: 273 vs 333 us at 20 rows per expert, 292 vs 333 at 24,
  // 365 vs 340 at 32)
  const int64_t nloc = std::max(1, m.e_end - m.e_begin);
  return g.rows <= (int64_t)(q4tc::kSmallBN * 3 / 4) * nloc;
}

cudaError_t launch_q4k_tc_gate_up(const Moe& m, const Groups& g, const float* x, ExpertBufs& eb,
                                  cudaStream_t st) {
  const gb_moe_desc& d = m.desc;
  const bool small = use_q4k_small(m, g);
  cudaError_t e;
  if ((e = launch_tile_table(m, g, small ? q4tc::kSmallBN : q4tc::BN, eb, st)) != cudaSuccess)
    return e;
  if ((e = launch_split_gather(m, g, x, eb, st)) != cudaSuccess) return e;
  q4tc::Args a = q4tc_args(m, g, eb);
  a.q = m.w.q4_gu_t;
  a.wexp = m.w.q4_gu_exp;
  a.K = d.hidden;
  a.rows = 2 * d.inter;
  a.m_tiles = (a.rows + q4tc::BM - 1) / q4tc::BM;
  a.xscale = eb.xscale;
  a.out_hi = eb.hh;
  a.out_lo = eb.hl;
  a.out_stride = d.inter;
  if (small) {
    if ((e = launch_sub_sums(eb.xh, eb.xl, d.hidden, g.rows, eb.xsum, st)) != cudaSuccess)
      return e;
    a.xsum = eb.xsum;
    return launch_q4tc_small<q4tc::GATE_UP>(m, a, eb.map_xh_s, eb.map_xl_s, st);
  }
  return launch_q4tc<q4tc::GATE_UP>(m, a, eb.map_xh, eb.map_xl, st);
}

cudaError_t launch_q4k_tc_down(const Moe& m, const Groups& g, ExpertBufs& eb, cudaStream_t st) {
  const gb_moe_desc& d = m.desc;
  q4tc::Args a = q4tc_args(m, g, eb);
  a.q = m.w.q4_dn_t;
  a.wexp = m.w.q4_dn_exp;
  a.K = d.inter;
  a.rows = d.hidden;
  a.m_tiles = (a.rows + q4tc::BM - 1) / q4tc::BM;
  a.out_y = eb.y;
  a.out_rows = g.out_rows;
  a.out_stride = d.hidden;
  if (use_q4k_small(m, g)) {
    cudaError_t e = launch_sub_sums(eb.hh, eb.hl, d.inter, g.rows, eb.xsum, st);
    if (e != cudaSuccess) return e;
    a.xsum = eb.xsum;
    return launch_q4tc_small<q4tc::DOWN>(m, a, eb.map_hh_s, eb.map_hl_s, st);
  }
  return launch_q4tc<q4tc::DOWN>(m, a, eb.map_hh, eb.map_hl, st);
}

}  // namespace gb
