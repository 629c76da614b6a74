// mx_gemm.cu -- grouped MXFP4 expert GEMMs on the block-scaled tensor cores
// (tcgen05.mma kind::mxf8f6f4.block_scale).
//
// Reference math: gpt_oss.rs:189-221 (gate_up + bias, interleaved split,
// clamped SwiGLU, down + bias).
//
// Weights.  MXFP4 is the block-scaled MMA's own operand format: E2M1 codes
// with one E8M0 scale per 32 elements along K.  TMA expands each 16 packed
// codes into the 16-byte padded form the MMA reads from shared memory
// (CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B), the scales reach tensor memory with
// tcgen05.cp, and no thread touches a weight.  Device layout, built once at
// load time from the caller's tensors (KC = roundup(K, 128) / 128 chunks):
//   nib [E_loc][KC][rows][64 B]  K-chunk major: one chunk of 128 codes of
//                                every row, so a tile of R rows of one chunk is
//                                R x 64 contiguous bytes (one TMA copy; copies
//                                of 16 KB keep HBM busy where 8 KB copies stall
//                                the issuing CTA).  Codes past K are zero, and
//                                so is a block whose safetensors scale byte is
//                                0 (0 there, 2^-127 to the hardware).
//   sfa [E_loc][KC][MT2][512]    scale atoms: atom t of chunk kc holds the
//                                scales of rows 128t..128t+127, byte
//                                16 r + 4 g + b = row 128t + 32g + r, block b
//                                of the chunk (the MMA's scale-factor order);
//                                MT2 = 128-row tiles rounded up to even.
//
// Activations need ~20 significant bits (outputs within 2e-2 at magnitudes of
// 10^2..10^3), E4M3 has 4.  A row x is scaled to x' = x * 2^-s with
// max |x'| in [128, 256) and written as five E4M3 pieces
//   x' = q0 + q1/16 + q2/16^2 + q3/16^3 + q4/16^4 (+ error < 2^-20 max|x'|),
// piece p being the E4M3 rounding of 16^p times the remainder of the earlier
// pieces; the matching block scale 2^-4p comes from a constant scale region
// in tensor memory.  The SwiGLU output h feeds down the same way with one
// fixed exponent: |h| <= max(limit, 1) * (limit + 1) under the clamps.
//
// Two kernels:
//   mx_decode_gemm  few positions per expert.  A = 256 weight rows (two
//     M = 128 halves), B = the pieces of NT positions packed into N = 8 NT
//     rows (row 8n + p = piece p of position n; rows 5-7 of each position are
//     the TMA's zero fill), so one MMA per K = 32 step covers all pieces and
//     D[m, 8n + p] keeps each piece in its own column.
//   mx_expert_gemm  many positions per expert.  A = 128 weight rows, B = 128
//     positions, one MMA per piece (piece 0 into one accumulator, pieces 1-4
//     into another, so small terms are not added into the large sum).
// Both run a persistent grid (one or two CTAs per SM) over work items
// (N tile, M tile), M fastest, with warp roles: 0-3 epilogue (TMEM lanes
// 0-127), TMA producer(s), MMA issuer.  Every mbarrier wait is bounded: on timeout the CTA
// raises an abort flag, records error bit 2, lets in-flight copies land,
// frees its TMEM and returns.
#include <cuda.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "moe_internal.h"
#include "ptx.cuh"
#include "umma.cuh"

namespace gb {
namespace mx {

constexpr int BM = 128, BK = 128, kPieces = 5;
constexpr int SF_BYTES = 512;
constexpr int kSmemLimit = 232448;
constexpr int kPrefillBN = 128;  // positions per prefill tile

// ---- shared device helpers ---------------------------------------------------

__device__ __forceinline__ void mma_mx(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t sfa_tmem, uint32_t sfb_tmem,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(
          d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

// 32 rows x 16 bytes of shared memory -> TMEM lanes 0-31, 4 columns, copied
// to all four lane quarters.
__device__ __forceinline__ void tmem_cp_sf(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc)
               : "memory");
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&v)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]),
                 "=r"(v[6]), "=r"(v[7])
               : "r"(taddr));
}

// E4M3 of one f32 (round to nearest even, saturating) and back.
__device__ __forceinline__ uint32_t e4m3_of(float v) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(0.0f), "f"(v));
  return r & 0xffu;
}

__device__ __forceinline__ uint32_t e4m3x2_of(float hi, float lo) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ float2 e4m3x2_value(uint32_t v) {
  uint32_t h;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"((uint16_t)v));
  const __half2 hv = *reinterpret_cast<const __half2*>(&h);
  return __half22float2(hv);  // .x = low byte, .y = high byte
}

__device__ __forceinline__ float e4m3_value(uint32_t v) { return e4m3x2_value(v).x; }

// Writes the five pieces of hp (|hp| < 256) at dst, dst + step, ...
__device__ __forceinline__ void store_pieces(float hp, uint8_t* dst, int64_t step) {
#pragma unroll
  for (int p = 0; p < kPieces; ++p) {
    const uint32_t q = e4m3_of(hp);
    dst[p * step] = (uint8_t)q;
    hp = __fmul_rn(__fsub_rn(hp, e4m3_value(q)), 16.0f);
  }
}

// Word `word` of the constant scale atom of slot-packed pieces: byte
// 16 r + 4 g + b belongs to B row 32 g + r, whose slot is r % 8; slot p < 5
// carries 2^-4p (E8M0 127 - 4p), the zero-filled slots 1.
__device__ __forceinline__ uint32_t slot_scale_word(int word) {
  const int slot = (word >> 2) & 7;
  const uint32_t b = slot < kPieces ? 127u - 4u * (uint32_t)slot : 127u;
  return b * 0x01010101u;
}

struct Args {
  const uint8_t* sfa;         // [E_loc][KC][mt2][512] scale atoms
  int kchunks;                // KC
  int mt2;                    // atoms per (expert, chunk)
  int rows;                   // weight rows per expert (2I or H)
  int m_tiles;                // M tiles per expert (of the kernel's M)
  int e_begin;
  const int32_t* meta;        // [2] = number of N tiles
  const int32_t* tile_expert;
  const int32_t* tile_row0;
  const int32_t* tile_rows;
  const float* bias;          // [E_loc][rows] f32, or null
  const float* xscale;        // GATE_UP: exponent s of each position's row (x = 2^s x')
  int in_exp;                 // DOWN: h = 2^in_exp h'
  float limit;                // SwiGLU clamp
  int h_exp;                  // GATE_UP: h is written as pieces of h * 2^-h_exp
  uint8_t* out_q;             // GATE_UP: h pieces, piece p of (position, i) at
  int64_t q_pos;              //   out_q + position * q_pos + p * q_piece + i
  int64_t q_piece;
  float* out_y;               // DOWN: y [rows][H], row = out_rows[position] (or position)
  const int32_t* out_rows;
  int out_stride;             // H (DOWN)
  int* err;                   // error bits (2: a wait timed out)
};

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

// Bias + activation + pieces (GATE_UP) or bias + store (DOWN) of the value
// `sum` of weight row `row` for position n of the tile.  All 32 lanes of the
// warp call it (the gate/up pair is a shuffle between neighbouring lanes).
template <int MODE>
__device__ __forceinline__ void finish(const Args& a, const Item& it, int row, bool valid,
                                       float bias, int n, float sum, int lane_parity) {
  const int64_t pos = (int64_t)it.row0 + n;
  const bool live = valid && n < it.nrows;
  if (MODE == 0) {
    float val = n < it.nrows ? __fmul_rn(sum, pow2f((int)a.xscale[pos])) : 0.0f;
    val = __fadd_rn(val, bias);
    // rows 2i (gate) and 2i+1 (up) sit in neighbouring lanes
    const float up = __shfl_down_sync(kFullMask, val, 1);
    if (lane_parity == 0 && live)
      store_pieces(__fmul_rn(act_gptoss(val, up, a.limit), pow2f(-a.h_exp)),
                   a.out_q + pos * a.q_pos + (row >> 1), a.q_piece);
  } else if (live) {
    const int64_t orow = a.out_rows ? a.out_rows[pos] : pos;
    a.out_y[orow * a.out_stride + row] = __fadd_rn(__fmul_rn(sum, pow2f(a.in_exp)), bias);
  }
}

__device__ __forceinline__ void linger_2ms() {
  const uint64_t t0 = globaltimer();
  while (globaltimer() - t0 < 2000000ull) {
  }
}

// ---------------------------------------------------------------------------
// Decode tiles: 256 weight rows x NT positions (N = 8 NT piece rows).
// ---------------------------------------------------------------------------
constexpr int kDecThreads = 224;  // warps 0-3 epilogue, 4 and 6 TMA, 5 MMA
constexpr int DM = 256;           // weight rows per tile

// CPS CTAs share an SM (2 for NT <= 8: each issues its own copies, which
// raises the SM's copy rate; TMEM <= 256 columns and half the shared memory
// each).
template <int NT>
struct Dec {
  static constexpr int CPS = NT <= 8 ? 2 : 1;
  static constexpr int N = 8 * NT;
  static constexpr int W_BYTES = DM * BK;            // 32 KB in shared memory, 16 KB packed
  static constexpr int X_BYTES = N * BK;             // NT positions x 8 slots x 128 bytes
  static constexpr int SFW = 2 * SF_BYTES;           // scale atoms of the two halves
  static constexpr int STAGE = (W_BYTES + X_BYTES + SFW + 1023) / 1024 * 1024;
  static constexpr int STAGES = std::min(6, (kSmemLimit / CPS - 1024 - SF_BYTES - 256) / STAGE);
  static constexpr int ACCS = N <= 16 ? 2 : 1;       // accumulators per half and tile
  static constexpr int NACC = NT <= 4 ? 2 : 1;       // tile buffers
  static constexpr int BUF = 2 * ACCS * N;
  static constexpr int SFB_COL = NACC * BUF;         // constant slot scales, 4 columns
  static constexpr int SFA_COL = SFB_COL + 4;        // 8 columns per stage
  static constexpr int USED = SFA_COL + 8 * STAGES;
  static constexpr int TMEM_COLS = USED <= 128 ? 128 : USED <= 256 ? 256 : 512;
  static constexpr size_t SMEM = (size_t)STAGES * STAGE + SF_BYTES + 1024 + 256;
  static_assert(TMEM_COLS * CPS <= 512, "tensor memory");
  static_assert(SMEM * CPS <= (size_t)kSmemLimit, "shared memory");
  // A = E2M1 (5), B = E4M3 (0), N, M = 128, E8M0 scales; bits 29-30 select
  // the A scale block (the weights' scale byte of the K = 32 step).
  static constexpr uint32_t IDESC = (5u << 7) | (0u << 10) | ((uint32_t)(N >> 3) << 17) |
                                    (1u << 23) | ((uint32_t)(BM >> 4) << 24);
};

template <int MODE, int NT>
__global__ void __launch_bounds__(kDecThreads, Dec<NT>::CPS)
    mx_decode_gemm(const __grid_constant__ CUtensorMap tmap_w,
                   const __grid_constant__ CUtensorMap tmap_x, const Args a) {
  using D = Dec<NT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  // stage s: [weights 32 KB][activation pieces N x 128][two scale atoms]
  uint8_t* sfb_const = smem + D::STAGES * D::STAGE;
  uint64_t* full = reinterpret_cast<uint64_t*>(sfb_const + SF_BYTES);
  uint64_t* empty = full + D::STAGES;
  uint64_t* acc_full = empty + D::STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total_items = a.meta[2] * a.m_tiles;
  const int nk = a.kchunks;

  for (int i = threadIdx.x; i < SF_BYTES / 4; i += kDecThreads)
    reinterpret_cast<uint32_t*>(sfb_const)[i] = slot_scale_word(i);
  fence_proxy_async_smem();
  if (threadIdx.x == 0) {
    for (int s = 0; s < D::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) tmem_alloc(tmem_slot, D::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 4 || warp == 6) {
    // ---------------- TMA producers: warp 4 even steps, warp 6 odd ----------
    if (lane == 0) {
      const uint32_t mine = warp == 4 ? 0u : 1u;
      uint32_t g = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < total_items && ok; item += gridDim.x) {
        const Item it = decode_item(a, item);
        for (int kc = 0; kc < nk; ++kc, ++g) {
          if ((g & 1u) != mine) continue;
          const uint32_t s = g % D::STAGES, ph = (g / D::STAGES) & 1u;
          if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, a.err)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * D::STAGE;
          // weights count their packed bytes; the activation box counts its
          // zero-filled slots too
          mbar_arrive_expect_tx(&full[s], D::W_BYTES / 2 + D::X_BYTES + D::SFW);
          tma_load_3d(st, &tmap_w, 0, it.m_tile * DM, it.le * nk + kc, &full[s]);
          tma_load_3d(st + D::W_BYTES, &tmap_x, kc * BK, 0, it.row0, &full[s]);
          bulk_load(st + D::W_BYTES + D::X_BYTES,
                    a.sfa + (((int64_t)it.le * nk + kc) * a.mt2 + 2 * it.m_tile) * SF_BYTES,
                    D::SFW, &full[s]);
        }
      }
      if (!ok) linger_2ms();
    }
  } else if (warp == 5) {
    // ---------------- MMA issuer ---------------------------------------------
    if (lane == 0) {
      const uint32_t sfb = tmem_base + (uint32_t)D::SFB_COL;
      tmem_cp_sf(sfb, rows16_desc(smem_u32(sfb_const)));
      uint32_t g = 0;
      int acc_iter = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < total_items && ok; item += gridDim.x, ++acc_iter) {
        const int b = acc_iter % D::NACC;
        const uint32_t acc_phase = (uint32_t)(acc_iter / D::NACC) & 1u;
        if (!mbar_wait(&acc_empty[b], acc_phase ^ 1u, abort_flag, a.err)) break;
        tc_fence_after();
        const uint32_t dbase = tmem_base + (uint32_t)(b * D::BUF);
        for (int kc = 0; kc < nk; ++kc, ++g) {
          const uint32_t s = g % D::STAGES, ph = (g / D::STAGES) & 1u;
          if (!mbar_wait(&full[s], ph, abort_flag, a.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sw = smem_u32(smem + s * D::STAGE);
          const uint32_t sx = sw + D::W_BYTES;
          const uint32_t sf = sx + D::X_BYTES;
          const uint32_t sfa = tmem_base + (uint32_t)(D::SFA_COL + 8 * s);
          tmem_cp_sf(sfa, rows16_desc(sf));
          tmem_cp_sf(sfa + 4, rows16_desc(sf + SF_BYTES));
#pragma unroll
          for (int j = 0; j < BK / 32; ++j) {
            const uint64_t bdesc = sw128_desc(sx + 32 * j);
            const uint32_t acc = (uint32_t)(j % D::ACCS);
            const uint32_t on = (kc != 0 || j >= D::ACCS) ? 1u : 0u;
#pragma unroll
            for (int h = 0; h < 2; ++h)
              mma_mx(dbase + (uint32_t)((h * D::ACCS + acc) * D::N),
                     sw128_desc(sw + h * (BM * BK) + 32 * j), bdesc,
                     D::IDESC | ((uint32_t)j << 29), (sfa + 4 * h) | ((uint32_t)j << 30), sfb, on);
          }
          mma_commit(&empty[s]);
        }
        if (ok) mma_commit(&acc_full[b]);
      }
      if (!ok || *abort_flag) linger_2ms();
    }
  } else if (warp < 4) {
    // ---------------- epilogue: thread m owns TMEM lane m -------------------
    const int m = threadIdx.x;
    int acc_iter = 0;
    for (int item = blockIdx.x; item < total_items; item += gridDim.x, ++acc_iter) {
      const int b = acc_iter % D::NACC;
      const uint32_t acc_phase = (uint32_t)(acc_iter / D::NACC) & 1u;
      if (!mbar_wait(&acc_full[b], acc_phase, abort_flag, a.err)) break;
      tc_fence_after();
      const Item it = decode_item(a, item);
      const uint32_t base =
          tmem_base + ((uint32_t)(warp * 32) << 16) + (uint32_t)(b * D::BUF);
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        const int row = it.m_tile * DM + h * BM + m;
        const bool valid = row < a.rows;
        const int64_t grow = (int64_t)it.le * a.rows + (valid ? row : 0);
        const float bias = (valid && a.bias) ? a.bias[grow] : 0.0f;
#pragma unroll 1
        for (int n = 0; n < NT; ++n) {
          uint32_t v[D::ACCS][8];
#pragma unroll
          for (int q = 0; q < D::ACCS; ++q)
            tmem_ld8(base + (uint32_t)((h * D::ACCS + q) * D::N + 8 * n), v[q]);
          tmem_wait_ld();
          float sum = 0.0f;
#pragma unroll
          for (int p = 0; p < kPieces; ++p) {
            float t = __uint_as_float(v[0][p]);
#pragma unroll
            for (int q = 1; q < D::ACCS; ++q) t = __fadd_rn(t, __uint_as_float(v[q][p]));
            sum = p == 0 ? t : __fadd_rn(sum, t);
          }
          finish<MODE>(a, it, row, valid, bias, n, sum, m & 1);
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[b]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, D::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Prefill tiles: 128 weight rows x BN positions, one MMA per piece.
// Piece layout: [5][position][K] bytes (one plane per piece).
// ---------------------------------------------------------------------------
constexpr int kPreThreads = 192;  // warps 0-3 epilogue, 4 TMA, 5 MMA

template <int BN>
struct Pre {
  static constexpr int A_BYTES = BM * BK;  // 16 KB in shared memory, 8 KB packed
  static constexpr int B_BYTES = kPieces * BN * BK;
  static constexpr int STAGE = (A_BYTES + B_BYTES + SF_BYTES + 1023) / 1024 * 1024;
  static constexpr int STAGES =
      std::min(8, (kSmemLimit - 1024 - kPieces * SF_BYTES - 256) / STAGE);
  static constexpr int NACC = BN <= 64 ? 2 : 1;  // accumulator (hi, lo) buffers
  static constexpr int ACC_COLS = NACC * 2 * BN;
  static constexpr int SFB_COL = ACC_COLS;                 // kPieces regions of 4 columns
  static constexpr int SFA_COL = SFB_COL + 4 * kPieces;    // 4 columns per stage
  static constexpr int USED = SFA_COL + 4 * STAGES;
  static constexpr int TMEM_COLS =
      USED <= 32 ? 32 : USED <= 64 ? 64 : USED <= 128 ? 128 : USED <= 256 ? 256 : 512;
  static constexpr size_t SMEM = (size_t)STAGES * STAGE + kPieces * SF_BYTES + 1024 + 256;
  static_assert(USED <= 512, "tensor memory");
  static_assert(SMEM <= (size_t)kSmemLimit, "shared memory");
  static constexpr uint32_t IDESC = (5u << 7) | (0u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                    (1u << 23) | ((uint32_t)(BM >> 4) << 24);
};

template <int MODE, int BN>
__global__ void __launch_bounds__(kPreThreads, 1)
    mx_expert_gemm(const __grid_constant__ CUtensorMap tmap_w,
                   const __grid_constant__ CUtensorMap tmap_x, const Args a) {
  using C = Pre<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  // stage s: [A 16 KB][B kPieces x BN x 128][scale atom 512]
  uint8_t* sfb_const = smem + C::STAGES * C::STAGE;  // kPieces x 512
  uint64_t* full = reinterpret_cast<uint64_t*>(sfb_const + kPieces * SF_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* acc_full = empty + C::STAGES;
  uint64_t* acc_empty = acc_full + C::NACC;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + C::NACC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total_items = a.meta[2] * a.m_tiles;
  const int nk = a.kchunks;

  for (int i = threadIdx.x; i < kPieces * SF_BYTES / 4; i += kPreThreads) {
    const uint32_t b = 127u - 4u * (uint32_t)(i / (SF_BYTES / 4));
    reinterpret_cast<uint32_t*>(sfb_const)[i] = b * 0x01010101u;
  }
  fence_proxy_async_smem();
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < C::NACC; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) tmem_alloc(tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 4) {
    if (lane == 0) {
      uint32_t g = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < total_items && ok; item += gridDim.x) {
        const Item it = decode_item(a, item);
        for (int kc = 0; kc < nk; ++kc, ++g) {
          const uint32_t s = g % C::STAGES, ph = (g / C::STAGES) & 1u;
          if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, a.err)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * C::STAGE;
          mbar_arrive_expect_tx(&full[s], C::A_BYTES / 2 + C::B_BYTES + SF_BYTES);
          tma_load_3d(st, &tmap_w, 0, it.m_tile * BM, it.le * nk + kc, &full[s]);
          tma_load_3d(st + C::A_BYTES, &tmap_x, kc * BK, it.row0, 0, &full[s]);
          bulk_load(st + C::A_BYTES + C::B_BYTES,
                    a.sfa + (((int64_t)it.le * nk + kc) * a.mt2 + it.m_tile) * SF_BYTES, SF_BYTES,
                    &full[s]);
        }
      }
      if (!ok) linger_2ms();
    }
  } else if (warp == 5) {
    if (lane == 0) {
      for (int p = 0; p < kPieces; ++p)
        tmem_cp_sf(tmem_base + (uint32_t)(C::SFB_COL + 4 * p),
                   rows16_desc(smem_u32(sfb_const + p * SF_BYTES)));
      uint32_t g = 0;
      int acc_iter = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < total_items && ok; item += gridDim.x, ++acc_iter) {
        const int b = acc_iter % C::NACC;
        const uint32_t acc_phase = (uint32_t)(acc_iter / C::NACC) & 1u;
        if (!mbar_wait(&acc_empty[b], acc_phase ^ 1u, abort_flag, a.err)) break;
        tc_fence_after();
        const uint32_t d_hi = tmem_base + (uint32_t)(b * 2 * BN);
        const uint32_t d_lo = d_hi + (uint32_t)BN;
        for (int kc = 0; kc < nk; ++kc, ++g) {
          const uint32_t s = g % C::STAGES, ph = (g / C::STAGES) & 1u;
          if (!mbar_wait(&full[s], ph, abort_flag, a.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * C::STAGE);
          const uint32_t sb = sa + C::A_BYTES;
          const uint32_t sfa = tmem_base + (uint32_t)(C::SFA_COL + 4 * s);
          tmem_cp_sf(sfa, rows16_desc(sb + C::B_BYTES));
#pragma unroll
          for (int j = 0; j < BK / 32; ++j) {
            const uint64_t adesc = sw128_desc(sa + 32 * j);
            const uint32_t id = C::IDESC | ((uint32_t)j << 29);
            const uint32_t sfa_j = sfa | ((uint32_t)j << 30);
            const uint32_t first = (kc | j) != 0;
#pragma unroll
            for (int p = 0; p < kPieces; ++p) {
              const uint64_t bdesc = sw128_desc(sb + p * BN * BK + 32 * j);
              const uint32_t sfb = tmem_base + (uint32_t)(C::SFB_COL + 4 * p);
              if (p == 0)
                mma_mx(d_hi, adesc, bdesc, id, sfa_j, sfb, first);
              else
                mma_mx(d_lo, adesc, bdesc, id, sfa_j, sfb, first || p > 1);
            }
          }
          mma_commit(&empty[s]);
        }
        if (ok) mma_commit(&acc_full[b]);
      }
      if (!ok || *abort_flag) linger_2ms();
    }
  } else {
    const int m = threadIdx.x;
    int acc_iter = 0;
    for (int item = blockIdx.x; item < total_items; item += gridDim.x, ++acc_iter) {
      const int b = acc_iter % C::NACC;
      const uint32_t acc_phase = (uint32_t)(acc_iter / C::NACC) & 1u;
      if (!mbar_wait(&acc_full[b], acc_phase, abort_flag, a.err)) break;
      tc_fence_after();
      const Item it = decode_item(a, item);
      const int row = it.m_tile * BM + m;
      const bool valid = row < a.rows;
      const int64_t grow = (int64_t)it.le * a.rows + (valid ? row : 0);
      const float bias = (valid && a.bias) ? a.bias[grow] : 0.0f;
      const uint32_t hi_addr =
          tmem_base + ((uint32_t)(warp * 32) << 16) + (uint32_t)(b * 2 * BN);
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 16) {
        uint32_t vh[16], vl[16];
        tmem_ld16(hi_addr + (uint32_t)c0, vh);
        tmem_ld16(hi_addr + (uint32_t)(BN + c0), vl);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j)
          finish<MODE>(a, it, row, valid, bias, c0 + j,
                       __fadd_rn(__uint_as_float(vh[j]), __uint_as_float(vl[j])), m & 1);
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[b]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Activation rows (gathered through perm) -> exponent s and five E4M3 pieces
// of x * 2^-s, piece p of position pos at q + pos * pos_stride +
// p * piece_stride.  One CTA per position.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) split_pieces_kernel(
    const float* __restrict__ x, const int32_t* __restrict__ perm, int perm_div, int K,
    int positions, uint8_t* __restrict__ q, int64_t pos_stride, int64_t piece_stride,
    float* __restrict__ xscale) {
  const int pos = blockIdx.x;
  if (pos >= positions) return;
  const float4* src = reinterpret_cast<const float4*>(x + (int64_t)(perm[pos] / perm_div) * K);
  const int n4 = K / 4;
  __shared__ float red[4];
  float mx = 0.0f;
  for (int i = threadIdx.x; i < n4; i += blockDim.x) {
    const float4 v = src[i];
    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFullMask, mx, s));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  // max |x'| in [128, 256); exponents kept where 2^-s stays a normal f32
  int s = mx > 0.0f ? ilogbf(mx) - 7 : 0;
  s = max(-120, min(120, s));
  const float inv = pow2f(-s);
  if (threadIdx.x == 0) xscale[pos] = (float)s;
  uint32_t* dst = reinterpret_cast<uint32_t*>(q + (int64_t)pos * pos_stride);
  for (int i = threadIdx.x; i < n4; i += blockDim.x) {
    const float4 v = src[i];
    float r[4] = {__fmul_rn(v.x, inv), __fmul_rn(v.y, inv), __fmul_rn(v.z, inv),
                  __fmul_rn(v.w, inv)};
#pragma unroll
    for (int p = 0; p < kPieces; ++p) {
      const uint32_t lo = e4m3x2_of(r[1], r[0]), hi = e4m3x2_of(r[3], r[2]);
      dst[p * (piece_stride / 4) + i] = lo | (hi << 16);
      const float2 a = e4m3x2_value(lo), b = e4m3x2_value(hi);
      r[0] = __fmul_rn(__fsub_rn(r[0], a.x), 16.0f);
      r[1] = __fmul_rn(__fsub_rn(r[1], a.y), 16.0f);
      r[2] = __fmul_rn(__fsub_rn(r[2], b.x), 16.0f);
      r[3] = __fmul_rn(__fsub_rn(r[3], b.y), 16.0f);
    }
  }
}

// Caller nibbles [E_loc][rows][nb][16] -> [E_loc][KC][rows][4 blocks][16],
// zero codes past K and in blocks whose scale byte means 0 (safetensors).
// One thread per 16-byte block slot of the destination.
__global__ void pack_nibbles_kernel(const uint8_t* __restrict__ blocks,
                                    const uint8_t* __restrict__ scales, int sp, int nb, int rows,
                                    int kchunks, int64_t total, int split_zero,
                                    uint8_t* __restrict__ out) {
  const int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (u >= total) return;
  const int q = (int)(u & 3);
  int64_t t = u >> 2;
  const int r = (int)(t % rows);
  t /= rows;
  const int kc = (int)(t % kchunks);
  const int64_t e = t / kchunks;
  const int b = kc * 4 + q;
  const int64_t grow = e * rows + r;
  uint4 v = make_uint4(0, 0, 0, 0);
  if (b < nb && !(split_zero && scales[grow * sp + b] == 0))
    v = *reinterpret_cast<const uint4*>(blocks + (grow * nb + b) * 16);
  *reinterpret_cast<uint4*>(out + u * 16) = v;
}

// Scale bytes [E_loc][rows][sp] -> atoms [E_loc][KC][mt2][512].
__global__ void pack_sfa_kernel(const uint8_t* __restrict__ scales, int sp, int nb, int rows,
                                int mt2, int kchunks, int64_t total, uint8_t* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int in = (int)(i % SF_BYTES);
  int64_t t = i / SF_BYTES;
  const int mt = (int)(t % mt2);
  t /= mt2;
  const int kc = (int)(t % kchunks);
  const int64_t e = t / kchunks;
  const int row = mt * BM + (in >> 2 & 3) * 32 + (in >> 4);
  const int blk = kc * 4 + (in & 3);
  out[i] = (row < rows && blk < nb) ? scales[(e * rows + row) * sp + blk] : (uint8_t)127;
}

}  // namespace mx

namespace {

int64_t round_up64(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

// 3-D tensor map {x, y, z} with the given y and z strides in bytes.
cudaError_t encode_3d(void* map, CUtensorMapDataType type, const void* base, uint64_t x,
                      uint64_t y, uint64_t z, uint64_t y_bytes, uint64_t z_bytes, uint32_t bx,
                      uint32_t by, uint32_t bz) {
  auto encode = tensor_map_encoder();
  if (!encode) return cudaErrorNotSupported;
  cuuint64_t dims[3] = {x, y, z};
  cuuint64_t strides[2] = {y_bytes, z_bytes};
  cuuint32_t box[3] = {bx, by, bz};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode(reinterpret_cast<CUtensorMap*>(map), type, 3, const_cast<void*>(base), dims,
                      strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace

bool mx_supported(const Moe& m) {
  const gb_moe_desc& d = m.desc;
  return d.weight_format != GB_FMT_Q4_K && d.act_kind == GB_ACT_GPTOSS_CLAMP &&
         d.hidden % 64 == 0 && d.inter % 64 == 0 && std::isfinite(d.swiglu_limit) &&
         d.swiglu_limit >= 0.0f && d.swiglu_limit < 1.0e15f;
}

cudaError_t mx_prepare_weights(Moe& m) {
  const gb_moe_desc& d = m.desc;
  const int64_t nloc = m.e_end - m.e_begin;
  const int H = d.hidden, I = d.inter;
  MxWeights& x = m.mx;
  x.kc_h = (int)(round_up64(H, mx::BK) / mx::BK);
  x.kc_i = (int)(round_up64(I, mx::BK) / mx::BK);
  x.mt2_gu = (int)round_up64((2 * I + mx::BM - 1) / mx::BM, 2);
  x.mt2_dn = (int)round_up64((H + mx::BM - 1) / mx::BM, 2);
  const int64_t gu_rows = 2 * (int64_t)I, dn_rows = H;
  const int64_t gu_units = nloc * x.kc_h * gu_rows * 4, dn_units = nloc * x.kc_i * dn_rows * 4;
  const size_t gu_sf = (size_t)(nloc * x.kc_h * x.mt2_gu * mx::SF_BYTES);
  const size_t dn_sf = (size_t)(nloc * x.kc_i * x.mt2_dn * mx::SF_BYTES);
  cudaError_t e;
  if ((e = cudaMalloc(&x.gu_nib, (size_t)gu_units * 16)) != cudaSuccess) return e;
  if ((e = cudaMalloc(&x.dn_nib, (size_t)dn_units * 16)) != cudaSuccess) return e;
  if ((e = cudaMalloc(&x.gu_sfa, gu_sf)) != cudaSuccess) return e;
  if ((e = cudaMalloc(&x.dn_sfa, dn_sf)) != cudaSuccess) return e;
  const int split_zero = d.weight_format == GB_FMT_MXFP4_SPLIT ? 1 : 0;
  const int nbh = H / 32, nbi = I / 32;
  mx::pack_nibbles_kernel<<<(unsigned)((gu_units + 255) / 256), 256>>>(
      m.w.gu_blocks, m.w.gu_scales, m.w.sp_h, nbh, (int)gu_rows, x.kc_h, gu_units, split_zero,
      x.gu_nib);
  mx::pack_nibbles_kernel<<<(unsigned)((dn_units + 255) / 256), 256>>>(
      m.w.dn_blocks, m.w.dn_scales, m.w.sp_i, nbi, (int)dn_rows, x.kc_i, dn_units, split_zero,
      x.dn_nib);
  mx::pack_sfa_kernel<<<(unsigned)((gu_sf + 255) / 256), 256>>>(
      m.w.gu_scales, m.w.sp_h, nbh, (int)gu_rows, x.mt2_gu, x.kc_h, (int64_t)gu_sf, x.gu_sfa);
  mx::pack_sfa_kernel<<<(unsigned)((dn_sf + 255) / 256), 256>>>(
      m.w.dn_scales, m.w.sp_i, nbi, (int)dn_rows, x.mt2_dn, x.kc_i, (int64_t)dn_sf, x.dn_sfa);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  // weights: {128 codes, rows, E_loc * KC}, boxes of 128 (prefill) or 256
  // (decode) rows of one chunk
  auto wmap = [&](void* map, const uint8_t* nib, int64_t rows, int kc, uint32_t box_rows) {
    return encode_3d(map, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, nib, mx::BK, (uint64_t)rows,
                     (uint64_t)(nloc * kc), 64, (uint64_t)rows * 64, mx::BK, box_rows, 1);
  };
  if ((e = wmap(x.map_gu128, x.gu_nib, gu_rows, x.kc_h, mx::BM)) != cudaSuccess) return e;
  if ((e = wmap(x.map_dn128, x.dn_nib, dn_rows, x.kc_i, mx::BM)) != cudaSuccess) return e;
  if ((e = wmap(x.map_gu256, x.gu_nib, gu_rows, x.kc_h, mx::DM)) != cudaSuccess) return e;
  if ((e = wmap(x.map_dn256, x.dn_nib, dn_rows, x.kc_i, mx::DM)) != cudaSuccess) return e;
  const double bound = std::max(1.0, (double)d.swiglu_limit) * ((double)d.swiglu_limit + 1.0);
  x.h_exp = ilogb(bound) - 7;
  x.weight_bytes = (gu_units + dn_units) * 16 + (int64_t)(gu_sf + dn_sf);
  if ((e = cudaDeviceSynchronize()) != cudaSuccess) return e;
  x.ok = true;
  return cudaSuccess;
}

void mx_release(MxWeights& x) {
  cudaFree(x.gu_nib);
  cudaFree(x.dn_nib);
  cudaFree(x.gu_sfa);
  cudaFree(x.dn_sfa);
  x = MxWeights{};
}

cudaError_t mx_make_maps(const Moe& m, ExpertBufs& eb) {
  const gb_moe_desc& d = m.desc;
  const uint64_t rows = (uint64_t)eb.rows_cap;
  const uint64_t P = mx::kPieces;
  cudaError_t e;
  // prefill tiles: planes [5][rows][K], box 128 x BN rows x 5 planes
  auto planes = [&](void* map, const uint8_t* q, uint64_t K) {
    return encode_3d(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, q, K, rows, P, K, K * rows, mx::BK,
                     mx::kPrefillBN, mx::kPieces);
  };
  // decode tiles: [rows][5][K], box 128 x 8 slots x NT positions (slots 5-7
  // read past the 5 pieces and are zero-filled)
  auto slots = [&](void* map, const uint8_t* q, uint64_t K, uint32_t nt) {
    return encode_3d(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, q, K, P, rows, K, K * P, mx::BK, 8, nt);
  };
  if ((e = planes(eb.map_xq_p, eb.xq, d.hidden)) != cudaSuccess) return e;
  if ((e = planes(eb.map_hq_p, eb.hq, d.inter)) != cudaSuccess) return e;
  for (int i = 0; i < kDecodeTileKinds; ++i) {
    const uint32_t nt = 1u << i;
    if ((e = slots(eb.map_xq_d[i], eb.xq, d.hidden, nt)) != cudaSuccess) return e;
    if ((e = slots(eb.map_hq_d[i], eb.hq, d.inter, nt)) != cudaSuccess) return e;
  }
  return cudaSuccess;
}

size_t mx_piece_bytes(int64_t rows, int k) { return (size_t)(rows * k) * mx::kPieces; }

namespace {

template <int MODE, int NT>
cudaError_t launch_decode(const Moe& m, const mx::Args& a, const void* map_w, const void* map_x,
                          cudaStream_t st) {
  auto k = mx::mx_decode_gemm<MODE, NT>;
  const size_t smem = mx::Dec<NT>::SMEM;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  k<<<m.sm_count * mx::Dec<NT>::CPS, mx::kDecThreads, smem, st>>>(
      *reinterpret_cast<const CUtensorMap*>(map_w),
                                               *reinterpret_cast<const CUtensorMap*>(map_x), a);
  return cudaGetLastError();
}

// nt_log2 < 0: prefill tiles; otherwise decode tiles of 2^nt_log2 positions.
template <int MODE>
cudaError_t launch_mx(const Moe& m, const mx::Args& a, const ExpertBufs& eb, int nt_log2,
                      cudaStream_t st) {
  const MxWeights& x = m.mx;
  const void* w256 = MODE == 0 ? x.map_gu256 : x.map_dn256;
  const unsigned char(*maps)[128] = MODE == 0 ? eb.map_xq_d : eb.map_hq_d;
  switch (nt_log2) {
    case 0: return launch_decode<MODE, 1>(m, a, w256, maps[0], st);
    case 1: return launch_decode<MODE, 2>(m, a, w256, maps[1], st);
    case 2: return launch_decode<MODE, 4>(m, a, w256, maps[2], st);
    case 3: return launch_decode<MODE, 8>(m, a, w256, maps[3], st);
    case 4: return launch_decode<MODE, 16>(m, a, w256, maps[4], st);
    default: break;
  }
  auto k = mx::mx_expert_gemm<MODE, mx::kPrefillBN>;
  const size_t smem = mx::Pre<mx::kPrefillBN>::SMEM;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const void* map_w = MODE == 0 ? x.map_gu128 : x.map_dn128;
  const void* map_x = MODE == 0 ? eb.map_xq_p : eb.map_hq_p;
  k<<<m.sm_count, mx::kPreThreads, smem, st>>>(*reinterpret_cast<const CUtensorMap*>(map_w),
                                               *reinterpret_cast<const CUtensorMap*>(map_x), a);
  return cudaGetLastError();
}

// Positions per decode tile: the power of two at or above twice the mean
// rows per local expert, at most 8 (two CTAs per SM) while the mean is at
// most 8, else 16.
int decode_nt_log2(const Moe& m, const Groups& g) {
  const int64_t nloc = std::max<int64_t>(1, m.e_end - m.e_begin);
  if (g.rows > 8 * nloc) return kDecodeTileKinds - 1;
  const int64_t target = (2 * g.rows + nloc - 1) / nloc;
  int l = 0;
  while (l < kDecodeTileKinds - 2 && (int64_t(1) << l) < target) ++l;
  return l;
}

mx::Args mx_common(const Moe& m, const Groups& g, const ExpertBufs& eb, int rows, int nt_log2) {
  mx::Args a{};
  a.e_begin = m.e_begin;
  a.meta = g.meta;
  a.tile_expert = eb.tile_expert;
  a.tile_row0 = eb.tile_row0;
  a.tile_rows = eb.tile_rows;
  a.limit = m.desc.swiglu_limit;
  a.err = g.meta + 1;
  a.rows = rows;
  const int tile_m = nt_log2 >= 0 ? mx::DM : mx::BM;
  a.m_tiles = (rows + tile_m - 1) / tile_m;
  return a;
}

cudaError_t mx_gate_up(const Moe& m, const Groups& g, const float* x, ExpertBufs& eb, int nt_log2,
                       cudaStream_t st) {
  const gb_moe_desc& d = m.desc;
  const bool decode = nt_log2 >= 0;
  const int positions = (int)g.rows;
  const int64_t H = d.hidden, I = d.inter, P = mx::kPieces, R = eb.rows_cap;
  cudaError_t e;
  if ((e = launch_tile_table(m, g, decode ? 1 << nt_log2 : mx::kPrefillBN, eb, st)) != cudaSuccess)
    return e;
  if (positions > 0) {
    mx::split_pieces_kernel<<<positions, 128, 0, st>>>(x, g.perm, g.perm_div, d.hidden, positions,
                                                      eb.xq, decode ? P * H : H,
                                                      decode ? H : R * H, eb.xscale);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  mx::Args a = mx_common(m, g, eb, 2 * d.inter, nt_log2);
  a.sfa = m.mx.gu_sfa;
  a.kchunks = m.mx.kc_h;
  a.mt2 = m.mx.mt2_gu;
  a.bias = m.w.gu_bias;
  a.xscale = eb.xscale;
  a.h_exp = m.mx.h_exp;
  a.out_q = eb.hq;
  a.q_pos = decode ? P * I : I;
  a.q_piece = decode ? I : R * I;
  return launch_mx<0>(m, a, eb, nt_log2, st);
}

cudaError_t mx_down(const Moe& m, const Groups& g, ExpertBufs& eb, int nt_log2, cudaStream_t st) {
  const gb_moe_desc& d = m.desc;
  mx::Args a = mx_common(m, g, eb, d.hidden, nt_log2);
  a.sfa = m.mx.dn_sfa;
  a.kchunks = m.mx.kc_i;
  a.mt2 = m.mx.mt2_dn;
  a.bias = m.w.dn_bias;
  a.in_exp = m.mx.h_exp;
  a.out_y = eb.y;
  a.out_rows = g.out_rows;
  a.out_stride = d.hidden;
  return launch_mx<1>(m, a, eb, nt_log2, st);
}

}  // namespace

cudaError_t launch_mx_gate_up(const Moe& m, const Groups& g, const float* x, ExpertBufs& eb,
                              bool decode_tiles, cudaStream_t st) {
  return mx_gate_up(m, g, x, eb, decode_tiles ? decode_nt_log2(m, g) : -1, st);
}

cudaError_t launch_mx_down(const Moe& m, const Groups& g, ExpertBufs& eb, bool decode_tiles,
                           cudaStream_t st) {
  return mx_down(m, g, eb, decode_tiles ? decode_nt_log2(m, g) : -1, st);
}

}  // namespace gb
