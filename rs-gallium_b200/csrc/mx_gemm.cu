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
//                                every row, so a tile of 256 rows of one chunk
//                                is 16 contiguous KB, one TMA copy (copies of
//                                16 KB keep HBM busy where 8 KB copies stall
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
// max |x'| in [128, 256) and written as four E4M3 pieces
//   x' = q0 + q1/16 + q2/16^2 + q3/16^3 (+ error < 2^-19 max|x'|),
// piece p being the E4M3 rounding of 16^p times the remainder of the earlier
// pieces.  The SwiGLU output h feeds down the same way with one fixed
// exponent: |h| <= max(limit, 1) * (limit + 1) under the clamps.
// Piece layout: [position][4][K] bytes.
//
// Tiles.  A = 256 weight rows (two M = 128 halves), B = the pieces of NT
// positions packed into N = 4 NT rows (row 4n + p = piece p of position n)
// with the constant B scale 2^-4p for row 4n + p.  One MMA per K = 32 step and
// half covers every piece, and
//   D[m, 4n + p] = 16^-p sum_k w[m, k] q_p[n, k]
// keeps each piece in its own accumulator column (adding the small pieces
// into the large sum inside the tensor core would lose their low bits); the
// epilogue thread of weight row m adds its position's 4 columns.  NT (2..60)
// follows the batch: few positions per expert in decode, 30 or 60 in
// prefill, where 4 pieces at the E4M3 rate cost the same tensor time as two
// f16 passes.  The four K steps of a stage rotate over ACCS accumulators so
// consecutive MMAs do not wait on one another.
//
// Persistent grid (two CTAs per SM; one for 60-position tiles) over work
// items (N tile, M tile, K split), M fastest; when the tiles cannot fill the
// grid, K is split and the last split to finish adds the partial sums in
// split order.  Grouped decode batches run gate_up and down as one launch
// (MODE 2, see the kernel).  Warps: 0-3 epilogue (TMEM lanes 0-127; 8-11 a
// second group for 60-position tiles), 4 and 6 TMA producers (alternate
// stages), 5 MMA issuer.  Every mbarrier wait is bounded: on
// timeout the CTA raises an abort flag, records error bit 2, lets in-flight
// copies land, frees its TMEM and returns.
#include <cuda.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "moe_internal.h"
#include "pieces.cuh"
#include "ptx.cuh"
#include "umma.cuh"

namespace gb {
namespace mx {

constexpr int BM = 128, BK = 128, kPieces = kActPieces;
constexpr int DM = 256;  // weight rows per tile
constexpr int SF_BYTES = 512;
constexpr int kSmemLimit = 232448;
constexpr int kThreads = 224;  // warps 0-3 epilogue, 4 and 6 TMA, 5 MMA
constexpr int kMaxSplit = 8;   // K splits of one tile (choose_ksplit)
constexpr int kSchedRing = 8;  // items handed out ahead (one-launch mode)

// ---- device helpers ----------------------------------------------------------

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

// Writes the pieces of hp (|hp| < 256) at dst, dst + step, ...
__device__ __forceinline__ void store_pieces(float hp, uint8_t* dst, int64_t step) {
#pragma unroll
  for (int p = 0; p < kPieces; ++p) {
    const uint32_t q = e4m3_of(hp);
    dst[p * step] = (uint8_t)q;
    hp = __fmul_rn(__fsub_rn(hp, e4m3_value(q)), 16.0f);
  }
}

// Word `word` of the constant B scale atom: byte 16 r + 4 g + b belongs to B
// row 32 g + r, which holds piece r % 4, scale 2^-4p (E8M0 127 - 4p).
__device__ __forceinline__ uint32_t piece_scale_word(int word) {
  const uint32_t p = (uint32_t)((word >> 2) % kPieces);
  return (127u - 4u * p) * 0x01010101u;
}

struct Args {
  const uint8_t* sfa;         // [E_loc][KC][mt2][512] scale atoms
  int kchunks;                // KC
  int mt2;                    // atoms per (expert, chunk)
  int rows;                   // weight rows per expert (2I or H)
  int m_tiles;                // 256-row tiles per expert
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
  uint8_t* out_q;             // GATE_UP: h pieces [position][4][I]
  int out_stride;             // I (GATE_UP) or H (DOWN)
  float* out_y;               // DOWN: y [rows][H], row = out_rows[position] (or position)
  const int32_t* out_rows;
  // DOWN, expert parallel: position p's row goes to return slot
  // ret_dst[p] & 0xffffffff of rank ret_dst[p] >> 32, at ret_base[rank] +
  // slot * H (peer memory); out_y is then unused
  const int64_t* ret_dst;
  float* ret_base[8];
  int64_t ret_slots;
  int* err;                   // error bits (2: a wait timed out)
  // split K: each (N tile, M tile) runs as ksplit items over consecutive
  // ranges of K chunks; partial sums meet in `partial`, the last to arrive
  // (ticket in `arrivals`, reset by it) adds them in split order
  int ksplit;
  float* partial;             // [tile * m_tiles + m_tile][ksplit][256 rows][NT]
  int* arrivals;              // [tile * m_tiles + m_tile]
  // one-launch gate_up + down: gate_up tile (j, m) sets ready[j * ready_stride
  // + m] once its h pieces are stored (the 128 h columns of down K chunk m)
  int* ready;
  int ready_stride;
  int* next_item;             // one-launch mode: items handed out so far beyond the grid
  // failure-handling tests: every bounded wait gives up after wait_ns (0 =
  // kMbarWaitNs); withhold_ready keeps gate_up tile 0's first ready flag
  // unpublished, so down items that need it wait until the limit
  uint64_t wait_ns;
  int withhold_ready;
};

struct Item {
  int tile;         // N tile
  int le, m_tile, row0, nrows;
  int slot;         // tile * m_tiles + m_tile
  int split;        // which K range
  int kc0, kc1;     // K chunks [kc0, kc1)
};

__device__ __forceinline__ Item decode_item(const Args& a, int item) {
  Item it;
  it.split = item % a.ksplit;
  it.slot = item / a.ksplit;
  const int j = it.slot / a.m_tiles;
  it.tile = j;
  it.m_tile = it.slot - j * a.m_tiles;
  it.le = a.tile_expert[j] - a.e_begin;
  it.row0 = a.tile_row0[j];
  it.nrows = a.tile_rows[j];
  it.kc0 = it.split * a.kchunks / a.ksplit;
  it.kc1 = (it.split + 1) * a.kchunks / a.ksplit;
  return it;
}

// Bias + clamped SwiGLU + pieces of h (GATE_UP) or bias + y (DOWN) for
// positions pg + n and pg + n + 1 of the tile (pg: the epilogue group's first
// position; lane n holds position pg + n's scale or output row), val[u]
// being the sum of weight row `row` for position pg + n + u.  Every lane of
// the warp calls it (the gate/up pair of rows 2i, 2i+1 is exchanged between
// neighbouring lanes: the even lane finishes position pg + n, the odd lane
// pg + n + 1).
template <int MODE>
__device__ __forceinline__ void finish_pair(const Args& a, const Item& it, int row, bool valid,
                                            float bias, int pg, int n, float (&val)[2],
                                            float lane_scale, int64_t lane_orow, int m) {
  if (MODE == 0) {
#pragma unroll
    for (int u = 0; u < 2; ++u)
      val[u] = __fadd_rn(__fmul_rn(val[u], __shfl_sync(kFullMask, lane_scale, n + u)), bias);
    const bool odd = m & 1;
    const float other = __shfl_xor_sync(kFullMask, odd ? val[0] : val[1], 1);
    const float gate = odd ? other : val[0];
    const float up = odd ? val[1] : other;
    const int np = pg + n + (odd ? 1 : 0);
    if (valid && np < it.nrows)
      store_pieces(__fmul_rn(act_gptoss(gate, up, a.limit), pow2f(-a.h_exp)),
                   a.out_q + ((int64_t)it.row0 + np) * (kPieces * a.out_stride) + (row >> 1),
                   a.out_stride);
  } else {
    const float f = pow2f(a.in_exp);
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      // lane_orow carries the address of the position's output row
      float* orow = reinterpret_cast<float*>(__shfl_sync(kFullMask, lane_orow, n + u));
      if (valid && pg + n + u < it.nrows && orow) orow[row] = __fadd_rn(__fmul_rn(val[u], f), bias);
    }
  }
}

__device__ __forceinline__ void linger_2ms() {
  const uint64_t t0 = globaltimer();
  while (globaltimer() - t0 < 2000000ull) {
  }
}

// Tile of 256 weight rows x NT positions (N = 4 NT piece rows).  Two CTAs
// share an SM: each issues its own copies (one CTA's copies stall near
// 40 GB/s), and one CTA's epilogue overlaps the other's MMAs; each has at most
// 256 TMEM columns and half the shared memory.
// NT = 60 (large batches, gate_up or down launched alone): one CTA per SM
// with all 512 TMEM columns, N = 240 per MMA, and two epilogue groups
// (warps 0-3 positions 0-29, warps 8-11 positions 30-59).  Each MMA
// instruction costs a fixed overhead besides its N-proportional time, so the
// 240-column MMAs keep the tensor pipe busier than 120-column ones.
// From NT = 30 a tile's MMAs are only as wide as its positions (N = 8
// ceil(rows / 2)), so an expert's last, partial tile costs its own rows.
// TMEM: NACC tile buffers of (2 halves x ACCS accumulators x N columns), then
// the constant piece scales (4 columns, 8 for N > 128) and one 8-column slot
// of weight scales, rewritten by tcgen05.cp before each stage's MMAs (the
// tcgen05 pipeline runs a thread's copies and MMAs in issue order; a ring of
// slots measured no faster and costs the widest tile 2 positions).
template <int NT>
struct Tile {
  static constexpr int N = kPieces * NT;
  static constexpr int GROUPS = NT > 32 ? 2 : 1;     // epilogue groups of 4 warps
  static constexpr int EPT = NT / GROUPS;            // positions per epilogue group
  static constexpr int THREADS = GROUPS == 1 ? kThreads : 384;
  static constexpr int CPS = GROUPS == 1 ? 2 : 1;
  static constexpr bool VARN = NT >= 30;             // MMA width follows the tile's rows
  static constexpr int SFB_COLS = N > 128 ? 8 : 4;
  static constexpr int W_BYTES = DM * BK;            // 32 KB in shared memory, 16 KB packed
  static constexpr int X_BYTES = N * BK;             // NT positions x 4 pieces x 128 bytes
  static constexpr int SFW = 2 * SF_BYTES;           // scale atoms of the two halves
  static constexpr int STAGE = (W_BYTES + X_BYTES + SFW + 1023) / 1024 * 1024;
  static constexpr int STAGES = std::min(6, (kSmemLimit / CPS - 1024 - SF_BYTES - 256) / STAGE);
  static constexpr int ACCS = N <= 16 ? 2 : 1;       // accumulators per half and tile
  static constexpr int BUF = 2 * ACCS * N;
  static constexpr int COLS_MAX = 512 / CPS;
  static constexpr int NACC = 2 * BUF + SFB_COLS + 8 <= COLS_MAX ? 2 : 1;  // tile buffers
  static constexpr int SFB_COL = NACC * BUF;         // constant piece scales
  static constexpr int SFA_COL = SFB_COL + SFB_COLS;  // weight scales, 8 columns
  static constexpr int USED = SFA_COL + 8;
  static constexpr int TMEM_COLS = USED <= 128 ? 128 : USED <= 256 ? 256 : 512;
  static constexpr int PAIRS = EPT >= 8 ? 4 : EPT / 2;  // position pairs per epilogue batch
  static constexpr size_t SMEM = (size_t)STAGES * STAGE + SF_BYTES + 1024 + 256;
  static_assert(NT % 2 == 0 && EPT % 2 == 0 && EPT <= 32,
                "positions are read in pairs, one lane each per epilogue group");
  static_assert(N <= 256, "MMA width");
  static_assert(STAGES >= 2, "pipeline depth");
  static_assert(TMEM_COLS <= COLS_MAX, "tensor memory");
  static_assert(SMEM * CPS <= (size_t)kSmemLimit, "shared memory");
  // A = E2M1 (5), B = E4M3 (0), N, M = 128, E8M0 scales; bits 29-30 select
  // the A scale block (the weights' scale byte of the K = 32 step).
  static constexpr uint32_t IDESC = (5u << 7) | (0u << 10) | ((uint32_t)(N >> 3) << 17) |
                                    (1u << 23) | ((uint32_t)(BM >> 4) << 24);
};

// Acquire load of a flag another CTA releases.
__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait for a ready flag; false if the CTA is aborting or it ran out.
__device__ __forceinline__ bool wait_ready(const int* p, volatile int* abort_flag, int* err,
                                           uint64_t limit_ns) {
  if (ld_acquire(p)) return true;
  const uint64_t t0 = globaltimer();
  while (!ld_acquire(p)) {
    if (*abort_flag) return false;
    if (globaltimer() - t0 > limit_ns) {
      *abort_flag = 1;
      atomicOr(err, 2);
      return false;
    }
    __nanosleep(32);
  }
  return true;
}

// Orders this thread's generic-proxy view of global memory (a flag just
// acquired, or h just stored) with its later async-proxy (TMA) copies.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// After the 128 epilogue threads stored a gate_up tile's h pieces: publish
// ready[tile * ready_stride + m_tile] for the down copies of that K chunk.
__device__ __forceinline__ void publish_ready(const Args& a, const Item& it, int m) {
  __threadfence();
  fence_proxy_async_global();
  asm volatile("bar.sync 1, 128;" ::: "memory");
  if (m == 0 && !(a.withhold_ready && it.tile == 0 && it.m_tile == 0)) {
    int* f = a.ready + (int64_t)it.tile * a.ready_stride + it.m_tile;
    asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(f), "r"(1) : "memory");
  }
}

// MODE 0: gate_up (a0, maps w0/x0).  MODE 1: down (a1, maps w1/x1).
// MODE 2: both in one launch: the gate_up items come first in every CTA's
// list, then the down items.  A down stage copies its weights and scales at
// once; its h chunk kc waits for ready[tile][kc] (the gate_up tile that
// writes those 128 h columns), the copy parked in a small queue meanwhile so
// that the producer keeps streaming weights.  Gate_up items wait on nothing,
// so with every CTA resident (one grid of 2 CTAs per SM) the waits end.
template <int MODE, int NT>
__global__ void __launch_bounds__(Tile<NT>::THREADS, Tile<NT>::CPS)
    mx_expert_gemm(const __grid_constant__ CUtensorMap tmap_w0,
                   const __grid_constant__ CUtensorMap tmap_x0,
                   const __grid_constant__ CUtensorMap tmap_w1,
                   const __grid_constant__ CUtensorMap tmap_x1, const Args a0, const Args a1) {
  using D = Tile<NT>;
  static_assert(D::GROUPS == 1 || MODE != 2, "the one-launch mode runs tiles of at most 30");
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
  // MODE 2 schedule: producer warp 4 takes items from a0.next_item (the
  // first is blockIdx.x) and hands each to warp 6, the MMA warp and the
  // epilogue through this ring; -1 ends the list
  __shared__ int s_sched[kSchedRing];
  __shared__ __align__(8) uint64_t s_sched_full[kSchedRing], s_sched_empty[kSchedRing];
  pdl_trigger();

  for (int i = threadIdx.x; i < SF_BYTES / 4; i += D::THREADS)
    reinterpret_cast<uint32_t*>(sfb_const)[i] = piece_scale_word(i);
  fence_proxy_async_smem();
  if (threadIdx.x == 0) {
    for (int s = 0; s < D::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128 * D::GROUPS);
    }
    for (int r = 0; r < kSchedRing; ++r) {
      mbar_init(&s_sched_full[r], 1);
      mbar_init(&s_sched_empty[r], 3);  // warp 6, the MMA warp, the epilogue
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 4 && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_w0) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_x0) : "memory");
    if (MODE != 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_w1) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_x1) : "memory");
    }
  }
  if (warp == 0) tmem_alloc(tmem_slot, D::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint64_t wait_ns = a0.wait_ns ? a0.wait_ns : kMbarWaitNs;
  // Everything above touches only this CTA's shared memory and TMEM, so it
  // overlaps the tail of the grid before; global memory is read after the wait.
  pdl_wait();
  const int n0 = MODE == 1 ? 0 : a0.meta[2] * a0.m_tiles * a0.ksplit;
  const int total_items = n0 + (MODE == 0 ? 0 : a1.meta[2] * a1.m_tiles * a1.ksplit);
  // item -> phase (0 gate_up, 1 down) and index within the phase
  auto phase_of = [&](int item) -> int { return MODE == 2 ? (item >= n0 ? 1 : 0) : MODE; };
  auto local_of = [&](int item) -> int { return MODE == 2 && item >= n0 ? item - n0 : item; };
  // i-th item of this CTA, or -1.  MODE 0 / 1: items blockIdx.x + i gridDim.x.
  // MODE 2: `publish` (warp 4) fetches and hands it out, the others read it.
  auto static_item = [&](int i) -> int {
    const int item = blockIdx.x + i * gridDim.x;
    return item < total_items ? item : -1;
  };
  auto publish_item = [&](int i) -> int {
    const int r = i % kSchedRing;
    if (!mbar_wait(&s_sched_empty[r], ((i / kSchedRing) & 1) ^ 1, abort_flag, a0.err, wait_ns)) return -1;
    int item = i == 0 ? (int)blockIdx.x : (int)gridDim.x + atomicAdd(a0.next_item, 1);
    if (item >= total_items) item = -1;
    s_sched[r] = item;
    mbar_arrive(&s_sched_full[r]);
    return item;
  };
  auto read_item = [&](int i) -> int {
    const int r = i % kSchedRing;
    if (!mbar_wait(&s_sched_full[r], (i / kSchedRing) & 1, abort_flag, a0.err, wait_ns)) return -1;
    return *reinterpret_cast<volatile int*>(&s_sched[r]);
  };

  if (warp == 4 || warp == 6) {
    // ---------------- TMA producers: warp 4 even steps, warp 6 odd ----------
    if (lane == 0) {
      const uint32_t mine = warp == 4 ? 0u : 1u;
      uint32_t g = 0;
      bool ok = true;
      // MODE 2: down stages whose h copy waits for its gate_up tile, oldest first
      constexpr int QCAP = 8;
      uint32_t q_g[QCAP] = {};
      int q_kc[QCAP] = {}, q_row0[QCAP] = {}, q_flag[QCAP] = {};
      int qh = 0, qn = 0;
      auto issue_front = [&]() {
        const uint32_t s = q_g[qh] % D::STAGES;
        fence_proxy_async_global();
        tma_load_3d(smem + s * D::STAGE + D::W_BYTES, &tmap_x1, q_kc[qh] * BK, 0, q_row0[qh],
                    &full[s]);
        qh = (qh + 1) % QCAP;
        --qn;
      };
      // Parked h copies are issued before any wait on the schedule ring: the
      // other producer may be waiting (through the MMA's in-order stages) for
      // one of them, and the ring may be waiting for that producer.  Flags
      // depend on gate_up items only, which wait on nothing.
      auto drain = [&]() {
        while (ok && qn > 0) {
          if (!wait_ready(a1.ready + q_flag[qh], abort_flag, a1.err, wait_ns)) ok = false;
          else issue_front();
        }
      };
      for (int i = 0; ok; ++i) {
        int item;
        if (MODE != 2) {
          item = static_item(i);
        } else {
          const int r = i % kSchedRing;
          const uint32_t rph = (uint32_t)(i / kSchedRing) & 1u;
          if (qn > 0 && !mbar_try_wait(warp == 4 ? &s_sched_empty[r] : &s_sched_full[r],
                                       warp == 4 ? rph ^ 1u : rph))
            drain();
          if (!ok) break;
          if (warp == 4) {
            item = publish_item(i);
          } else {
            item = read_item(i);
            mbar_arrive(&s_sched_empty[r]);
          }
        }
        if (item < 0) break;
        const int ph = phase_of(item);
        const Args& A = ph ? a1 : a0;
        const CUtensorMap* tw = ph ? &tmap_w1 : &tmap_w0;
        const CUtensorMap* tx = ph ? &tmap_x1 : &tmap_x0;
        const Item it = decode_item(A, local_of(item));
        for (int kc = it.kc0; kc < it.kc1; ++kc, ++g) {
          if ((g & 1u) != mine) continue;
          const uint32_t s = g % D::STAGES, sph = (g / D::STAGES) & 1u;
          if (MODE == 2) {
            // the stage that last used slot s needs its h copy before slot s frees
            while (ok && qn > 0 && (q_g[qh] + D::STAGES <= g || qn == QCAP)) {
              if (!wait_ready(a1.ready + q_flag[qh], abort_flag, A.err, wait_ns)) ok = false;
              else issue_front();
            }
            if (!ok) break;
          }
          if (!mbar_wait(&empty[s], sph ^ 1u, abort_flag, A.err, wait_ns)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * D::STAGE;
          // the weight box counts its packed bytes
          mbar_arrive_expect_tx(&full[s], D::W_BYTES / 2 + D::X_BYTES + D::SFW);
          tma_load_3d(st, tw, 0, it.m_tile * DM, it.le * A.kchunks + kc, &full[s]);
          bulk_load(st + D::W_BYTES + D::X_BYTES,
                    A.sfa + (((int64_t)it.le * A.kchunks + kc) * A.mt2 + 2 * it.m_tile) * SF_BYTES,
                    D::SFW, &full[s]);
          if (MODE == 2 && ph == 1) {
            const int flag = it.tile * a1.ready_stride + kc;
            const int t = (qh + qn) % QCAP;
            q_g[t] = g;
            q_kc[t] = kc;
            q_row0[t] = it.row0;
            q_flag[t] = flag;
            ++qn;
            while (qn > 0 && ld_acquire(a1.ready + q_flag[qh])) issue_front();
          } else {
            tma_load_3d(st + D::W_BYTES, tx, kc * BK, 0, it.row0, &full[s]);
          }
        }
      }
      if (MODE == 2) drain();
      if (!ok) linger_2ms();
    }
  } else if (warp == 5) {
    // ---------------- MMA issuer ---------------------------------------------
    if (lane == 0) {
      // The issue loop is kept short (one thread issues for the whole tile):
      // stage index and phase advance incrementally, shared-memory
      // descriptors are a constant OR the address (+2 per 32 K bytes).
      const uint32_t sfb = tmem_base + (uint32_t)D::SFB_COL;
      const uint32_t sfa = tmem_base + (uint32_t)D::SFA_COL;
      tmem_cp_sf(sfb, rows16_desc(smem_u32(sfb_const)));
      if (D::SFB_COLS > 4) tmem_cp_sf(sfb + 4, rows16_desc(smem_u32(sfb_const)));  // rows 128-255
      const uint64_t dconst = sw128_desc(0), rconst = rows16_desc(0);
      const uint32_t smem0 = smem_u32(smem);
      uint32_t s = 0, sph = 0, sw = smem0;
      int acc_iter = 0;
      bool ok = true;
      for (int i = 0; ok; ++i, ++acc_iter) {
        int item;
        if (MODE != 2) {
          item = static_item(i);
        } else {
          item = read_item(i);
          mbar_arrive(&s_sched_empty[i % kSchedRing]);
        }
        if (item < 0) break;
        const int ph = phase_of(item);
        const Args& A = ph ? a1 : a0;
        const int b = acc_iter % D::NACC;
        const uint32_t acc_phase = (uint32_t)(acc_iter / D::NACC) & 1u;
        if (!mbar_wait(&acc_empty[b], acc_phase ^ 1u, abort_flag, A.err, wait_ns)) break;
        tc_fence_after();
        const uint32_t dbase = tmem_base + (uint32_t)(b * D::BUF);
        const Item it = decode_item(A, local_of(item));
        // MMA width: the tile's positions rounded up to even (4 piece rows each)
        const uint32_t idesc =
            D::VARN ? (D::IDESC & ~(0x3Fu << 17)) |
                          ((uint32_t)min(D::N, 8 * ((it.nrows + 1) >> 1)) >> 3 << 17)
                    : D::IDESC;
        for (int kc = it.kc0; kc < it.kc1; ++kc) {
          if (!mbar_wait(&full[s], sph, abort_flag, A.err, wait_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = dconst | (sw >> 4);                           // weights
          const uint64_t db = dconst | ((sw + D::W_BYTES) >> 4);            // pieces
          const uint64_t dsf = rconst | ((sw + D::W_BYTES + D::X_BYTES) >> 4);
          tmem_cp_sf(sfa, dsf);
          tmem_cp_sf(sfa + 4, dsf + (SF_BYTES >> 4));
          const bool first = kc == it.kc0;
#pragma unroll
          for (int j = 0; j < BK / 32; ++j) {
            const uint32_t acc = (uint32_t)(j % D::ACCS);
            const uint32_t on = (!first || j >= D::ACCS) ? 1u : 0u;
#pragma unroll
            for (int h = 0; h < 2; ++h)
              mma_mx(dbase + (uint32_t)((h * D::ACCS + acc) * D::N),
                     da + (uint64_t)((h * BM * BK) >> 4) + (uint64_t)(2 * j), db + (uint64_t)(2 * j),
                     idesc | ((uint32_t)j << 29), (sfa + 4 * h) | ((uint32_t)j << 30), sfb, on);
          }
          mma_commit(&empty[s]);
          if (++s == (uint32_t)D::STAGES) {
            s = 0;
            sph ^= 1u;
            sw = smem0;
          } else {
            sw += (uint32_t)D::STAGE;
          }
        }
        if (ok) mma_commit(&acc_full[b]);
      }
      if (!ok || *abort_flag) linger_2ms();
    }
  } else if (warp < 4 || (D::GROUPS > 1 && warp >= 8)) {
    // ---------------- epilogue: thread m owns TMEM lane m -------------------
    // Group grp (warps 0-3; warps 8-11 in 60-position tiles) finishes
    // positions pg .. pg + EPT - 1.  Its thread 0 takes the item and waits
    // for the accumulator, then the group's 128 threads agree on it at named
    // barrier 1 + grp (so that a wait that gave up ends every thread's loop
    // at the same item).
    const int m = threadIdx.x & 127, grp = warp >> 3, pg = grp * D::EPT;
    const uint32_t nbar = 1u + (uint32_t)grp;
    __shared__ int s_epi_item[2][2];
    __shared__ int s_last[2];
    int acc_iter = 0;
    for (int i = 0;; ++i, ++acc_iter) {
      const int b = acc_iter % D::NACC;
      const uint32_t acc_phase = (uint32_t)(acc_iter / D::NACC) & 1u;
      if (m == 0) {
        int item = MODE != 2 ? static_item(i) : read_item(i);
        if (MODE == 2 && item >= 0) mbar_arrive(&s_sched_empty[i % kSchedRing]);
        if (item >= 0 && !mbar_wait(&acc_full[b], acc_phase, abort_flag, a0.err, wait_ns)) item = -1;
        s_epi_item[grp][i & 1] = item;
      }
      asm volatile("bar.sync %0, 128;" ::"r"(nbar) : "memory");
      const int item = *reinterpret_cast<volatile int*>(&s_epi_item[grp][i & 1]);
      if (item < 0) break;
      const int ph = phase_of(item);
      const Args& A = ph ? a1 : a0;
      tc_fence_after();
      const Item it = decode_item(A, local_of(item));
      const bool split = A.ksplit > 1;
      float* part = A.partial + ((int64_t)it.slot * A.ksplit + it.split) * (DM * NT);
      // lane n holds position pg + n's activation scale (gate_up) or the
      // address of its output row (down: local y, or the return slot on the
      // token's own rank)
      float lane_scale = 0.0f;
      int64_t lane_orow = 0;
      if (lane < D::EPT && pg + lane < it.nrows) {
        const int64_t pos = (int64_t)it.row0 + pg + lane;
        if (ph == 0) {
          lane_scale = pow2f((int)A.xscale[pos]);
        } else if (A.ret_dst) {
          const int64_t dst = A.ret_dst[pos];
          const int rk = (int)(dst >> 32);
          const int64_t sl = dst & 0xffffffffll;
          float* base = nullptr;
#pragma unroll
          for (int q = 0; q < 8; ++q)
            if (q == rk) base = A.ret_base[q];
          if (dst >= 0 && base && sl < A.ret_slots)
            lane_orow = reinterpret_cast<int64_t>(base + sl * A.out_stride);
          else
            atomicOr(A.err, 1);  // no valid slot: the row is dropped
        } else {
          lane_orow = reinterpret_cast<int64_t>(
              A.out_y + (A.out_rows ? (int64_t)A.out_rows[pos] : pos) * A.out_stride);
        }
      }
      auto finish = [&](int row, bool valid, float bias, int n, float (&val)[2]) {
        if (MODE != 1 && ph == 0)
          finish_pair<0>(a0, it, row, valid, bias, pg, n, val, lane_scale, lane_orow, m);
        else if (MODE != 0)
          finish_pair<1>(a1, it, row, valid, bias, pg, n, val, lane_scale, lane_orow, m);
      };
      const uint32_t base =
          tmem_base + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)(b * D::BUF);
      // Sums of the pieces (and accumulators) of positions pg + n0p .. pg +
      // n0p + 2 PAIRS - 1 of half h; columns 4n .. 4n + 7 hold positions n,
      // n + 1.
      auto load_sums = [&](int h, int n0p, float (&sums)[D::PAIRS][2]) {
        uint32_t v[D::PAIRS][D::ACCS][8];
#pragma unroll
        for (int pp = 0; pp < D::PAIRS; ++pp)
#pragma unroll
          for (int q = 0; q < D::ACCS; ++q)
            if (n0p + 2 * pp < D::EPT)
              tmem_ld8(base + (uint32_t)((h * D::ACCS + q) * D::N + kPieces * (pg + n0p + 2 * pp)),
                       v[pp][q]);
        tmem_wait_ld();
#pragma unroll
        for (int pp = 0; pp < D::PAIRS; ++pp)
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            float sum = 0.0f;
#pragma unroll
            for (int p = 0; p < kPieces; ++p) {
              float t = __uint_as_float(v[pp][0][u * kPieces + p]);
#pragma unroll
              for (int q = 1; q < D::ACCS; ++q)
                t = __fadd_rn(t, __uint_as_float(v[pp][q][u * kPieces + p]));
              sum = p == 0 ? t : __fadd_rn(sum, t);
            }
            sums[pp][u] = sum;
          }
      };
      auto store_pair = [&](int h, int row, bool valid, float bias, int n, float (&val)[2]) {
        if (split)
          *reinterpret_cast<float2*>(part + (h * BM + m) * NT + pg + n) =
              make_float2(val[0], val[1]);
        else
          finish(row, valid, bias, n, val);
      };
      if constexpr (D::NACC == 1) {
        // One accumulator buffer (the widest tiles): the group's sums
        // (2 x EPT per thread) come out of TMEM first and the buffer is
        // handed back at once, so that the next item's MMAs run while this
        // thread stores h or y.  The arrive is relaxed: the MMA warp reads
        // none of the stores.
        float acc[2][D::EPT];
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int n0p = 0; n0p < D::EPT; n0p += 2 * D::PAIRS) {
            float sums[D::PAIRS][2];
            load_sums(h, n0p, sums);
#pragma unroll
            for (int pp = 0; pp < D::PAIRS; ++pp)
              if (n0p + 2 * pp < D::EPT) {
                acc[h][n0p + 2 * pp] = sums[pp][0];
                acc[h][n0p + 2 * pp + 1] = sums[pp][1];
              }
          }
        tc_fence_before();
        mbar_arrive_relaxed(&acc_empty[b]);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int row = it.m_tile * DM + h * BM + m;
          const bool valid = row < A.rows;
          const int64_t grow = (int64_t)it.le * A.rows + (valid ? row : 0);
          const float bias = (valid && A.bias) ? A.bias[grow] : 0.0f;
#pragma unroll
          for (int n = 0; n < D::EPT; n += 2) {
            float val[2] = {acc[h][n], acc[h][n + 1]};
            store_pair(h, row, valid, bias, n, val);
          }
        }
      } else {
        // Two buffers: the next item's MMAs already run in the other one.
#pragma unroll 1
        for (int h = 0; h < 2; ++h) {
          const int row = it.m_tile * DM + h * BM + m;
          const bool valid = row < A.rows;
          const int64_t grow = (int64_t)it.le * A.rows + (valid ? row : 0);
          const float bias = (valid && A.bias) ? A.bias[grow] : 0.0f;
#pragma unroll 1
          for (int n0p = 0; n0p < D::EPT; n0p += 2 * D::PAIRS) {
            float sums[D::PAIRS][2];
            load_sums(h, n0p, sums);
#pragma unroll
            for (int pp = 0; pp < D::PAIRS; ++pp)
              if (n0p + 2 * pp < D::EPT) store_pair(h, row, valid, bias, n0p + 2 * pp, sums[pp]);
          }
        }
        tc_fence_before();
        mbar_arrive(&acc_empty[b]);
      }
      if (!split) {
        if (MODE == 2 && ph == 0) publish_ready(a0, it, m);
      } else {
        // the last of the tile's ksplit items adds the partial sums in split
        // order and finishes the tile (no waiting: a ticket per tile; tiles of
        // one epilogue group only, the host never splits 60-position tiles)
        __threadfence();
        asm volatile("bar.sync %0, 128;" ::"r"(nbar) : "memory");
        if (m == 0) s_last[grp] = atomicAdd(&A.arrivals[it.slot], 1) == A.ksplit - 1;
        asm volatile("bar.sync %0, 128;" ::"r"(nbar) : "memory");
        if (s_last[grp]) {
          __threadfence();
          if (m == 0) A.arrivals[it.slot] = 0;  // ready for the next forward
          const float* p0 = A.partial + (int64_t)it.slot * A.ksplit * (DM * NT);
          float bias[2];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int row = it.m_tile * DM + h * BM + m;
            const int64_t grow = (int64_t)it.le * A.rows + (row < A.rows ? row : 0);
            bias[h] = (row < A.rows && A.bias) ? A.bias[grow] : 0.0f;
          }
#pragma unroll 1
          for (int n = 0; n < NT; n += 2) {
            // every split's partial sums of both halves in flight at once
            float2 pv[2][kMaxSplit];
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
              for (int sp = 0; sp < kMaxSplit; ++sp)
                if (sp < A.ksplit)
                  pv[h][sp] = __ldcg(reinterpret_cast<const float2*>(
                      p0 + (int64_t)sp * (DM * NT) + (h * BM + m) * NT + n));
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              float val[2] = {pv[h][0].x, pv[h][0].y};
#pragma unroll
              for (int sp = 1; sp < kMaxSplit; ++sp)
                if (sp < A.ksplit) {
                  val[0] = __fadd_rn(val[0], pv[h][sp].x);
                  val[1] = __fadd_rn(val[1], pv[h][sp].y);
                }
              const int row = it.m_tile * DM + h * BM + m;
              finish(row, row < A.rows, bias[h], n, val);
            }
          }
          if (MODE == 2 && ph == 0) publish_ready(a0, it, m);
        }
      }
    }
    // rows stored in peers' return slots are visible system-wide before this
    // kernel ends (the return flags are released after it)
    if (MODE != 0 && a1.ret_dst) __threadfence_system();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, D::TMEM_COLS);
  }
}

// Activation rows (gathered through perm) -> pieces, [position][4][K].  One
// CTA per position.
__global__ void __launch_bounds__(128) split_pieces_kernel(
    const float* __restrict__ x, const int32_t* __restrict__ perm, int perm_div, int K,
    int positions, uint8_t* __restrict__ q, float* __restrict__ xscale) {
  pdl_trigger();
  pdl_wait();
  const int pos = blockIdx.x;
  if (pos >= positions) return;
  row_pieces(x + (int64_t)(perm[pos] / perm_div) * K, K, q, xscale, &pos, 1);
}

// Small batches (T * top_k <= kGroupEntries): grouping, N-tile table and
// pieces in one launch, one CTA per token.  Every CTA counts all T * top_k
// routing entries in shared memory and scans them to the expert offsets
// (a few hundred entries); the entry of token t, rank r goes to position
// offsets[e] + (entries before it with the same expert), the stable
// (expert, token) order of permute_kernel, so perm, inv, counts, offsets,
// active and meta[0] are the same as there.  CTA 0 writes the per-expert
// arrays and the tile table of tile_table_kernel and clears the one-launch
// expert kernel's ready flags of those tiles; CTA t writes perm and inv of
// its entries and the pieces of x[t] at each of its positions.
constexpr int kGroupEntries = kMxGroupEntries;
constexpr int kGroupExperts = 256;
// Threads of the grouping kernel: its pass over the token's row (max, then
// the pieces) takes two float4 per thread at H = 2880 instead of six.
constexpr int kGroupThreads = 512;

__global__ void __launch_bounds__(kGroupThreads) group_pieces_kernel(
    const float* __restrict__ x, const int32_t* __restrict__ idx, int T, int E, int topk,
    int H, int e_begin, int e_end, int bn, int32_t* __restrict__ counts,
    int32_t* __restrict__ offsets, int32_t* __restrict__ active, int32_t* __restrict__ meta,
    int32_t* __restrict__ perm, int32_t* __restrict__ inv, int32_t* __restrict__ tile_expert,
    int32_t* __restrict__ tile_row0, int32_t* __restrict__ tile_rows, uint8_t* __restrict__ q,
    float* __restrict__ xscale, int* __restrict__ ready, int ready_per_tile,
    int* __restrict__ next_item) {
  __shared__ int s_idx[kGroupEntries];
  __shared__ int s_tiles;
  __shared__ int s_cnt[kGroupExperts], s_off[kGroupExperts];
  __shared__ int s_pos[8];
  pdl_trigger();
  pdl_wait();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n = T * topk, t = blockIdx.x;
  for (int e = tid; e < E; e += blockDim.x) s_cnt[e] = 0;
  __syncthreads();
  unsigned bad = 0;
  for (int i = tid; i < n; i += blockDim.x) {
    int e = __ldg(idx + i);
    if (e < 0 || e >= E) {
      bad = 1;
      e = -1;
    } else {
      atomicAdd(&s_cnt[e], 1);
    }
    s_idx[i] = e;
  }
  if (bad && t == 0) atomicOr(reinterpret_cast<unsigned*>(meta + 1), 1u);
  __syncthreads();
  if (warp == 0) {
    // exclusive scan of the counts, 8 experts per lane
    const int per = (E + 31) / 32;
    int local = 0;
    for (int q2 = 0; q2 < per; ++q2) {
      const int e = lane * per + q2;
      if (e < E) local += s_cnt[e];
    }
    int incl = local;
#pragma unroll
    for (int s = 1; s < 32; s <<= 1) {
      const int o = __shfl_up_sync(kFullMask, incl, s);
      if (lane >= s) incl += o;
    }
    const int total = __shfl_sync(kFullMask, incl, 31);
    int run = incl - local;
    for (int q2 = 0; q2 < per; ++q2) {
      const int e = lane * per + q2;
      if (e < E) {
        s_off[e] = run;
        run += s_cnt[e];
      }
    }
    if (t == 0) {
      __syncwarp();
      int arun = 0, tiles = 0;
      for (int e0 = 0; e0 < E; e0 += 32) {
        const int e = e0 + lane;
        const bool local_e = e < E && e >= e_begin && e < e_end;
        const int c = e < E ? s_cnt[e] : 0;
        const int off = e < E ? s_off[e] : 0;
        if (e < E) {
          counts[e] = c;
          offsets[e] = off;
        }
        const int act = local_e && c > 0;
        const unsigned am = __ballot_sync(kFullMask, act);
        if (act) active[arun + __popc(am & ((1u << lane) - 1u))] = e;
        arun += __popc(am);
        const int nt = local_e ? (c + bn - 1) / bn : 0;
        int tin = nt;
#pragma unroll
        for (int s = 1; s < 32; s <<= 1) {
          const int o = __shfl_up_sync(kFullMask, tin, s);
          if (lane >= s) tin += o;
        }
        int j = tiles + tin - nt;
        for (int i = 0; i < c && local_e; i += bn, ++j) {
          tile_expert[j] = e;
          tile_row0[j] = off + i;
          tile_rows[j] = min(bn, c - i);
        }
        tiles += __shfl_sync(kFullMask, tin, 31);
      }
      if (lane == 0) {
        offsets[E] = total;
        meta[0] = arun;
        meta[2] = tiles;
        s_tiles = tiles;
      }
    }
  }
  __syncthreads();
  // the one-launch expert kernel's ready flags of this forward's tiles
  if (t == 0 && ready) {
    for (int i = tid; i < s_tiles * ready_per_tile; i += blockDim.x) ready[i] = 0;
    if (tid == 0) *next_item = 0;
  }
  // positions of this token's entries: warp w takes rank w, w + nwarps, ...
  for (int r = warp; r < topk; r += (int)(blockDim.x >> 5)) {
    const int i = t * topk + r;
    const int e = s_idx[i];
    int before = 0;
    for (int j0 = 0; j0 < i; j0 += 32) {
      const int j = j0 + lane;
      before += __popc(__ballot_sync(kFullMask, j < i && s_idx[j] == e));
    }
    const int pos = e >= 0 ? s_off[e] + before : -1;
    if (lane == 0) {
      s_pos[r] = pos;
      if (pos >= 0) perm[pos] = i;
      inv[i] = max(pos, 0);  // an invalid entry is flagged in meta[1]; keep inv in range
    }
  }
  __syncthreads();
  int nd = 0;
  int dpos[8];
  for (int r = 0; r < topk; ++r)
    if (s_pos[r] >= 0) dpos[nd++] = s_pos[r];
  row_pieces(x + (int64_t)t * H, H, q, xscale, dpos, nd);
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
  m.weight_bytes += (gu_units + dn_units) * 16 + (int64_t)(gu_sf + dn_sf);
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
  // weights: {128 codes, rows, E_loc * KC}, boxes of 256 rows of one chunk
  auto wmap = [&](void* map, const uint8_t* nib, int64_t rows, int kc) {
    return encode_3d(map, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, nib, mx::BK, (uint64_t)rows,
                     (uint64_t)(nloc * kc), 64, (uint64_t)rows * 64, mx::BK, mx::DM, 1);
  };
  if ((e = wmap(x.map_gu, x.gu_nib, gu_rows, x.kc_h)) != cudaSuccess) return e;
  if ((e = wmap(x.map_dn, x.dn_nib, dn_rows, x.kc_i)) != cudaSuccess) return e;
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
  // pieces [rows][4][K], box 128 bytes x 4 pieces x NT positions
  auto pieces = [&](void* map, const uint8_t* q, uint64_t K, uint32_t nt) {
    return encode_3d(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, q, K, P, rows, K, K * P, mx::BK,
                     mx::kPieces, nt);
  };
  for (int i = 0; i < kMxTileKinds; ++i) {
    const uint32_t nt = (uint32_t)mx_tile_positions(i);
    if ((e = pieces(eb.map_xq[i], eb.xq, d.hidden, nt)) != cudaSuccess) return e;
    if ((e = pieces(eb.map_hq[i], eb.hq, d.inter, nt)) != cudaSuccess) return e;
  }
  return cudaSuccess;
}

size_t mx_piece_bytes(int64_t rows, int k) { return (size_t)(rows * k) * mx::kPieces; }

int mx_tile_positions(int kind) {
  return kind < kMxKind30 ? 2 << kind : kind == kMxKind30 ? 30 : 60;
}

int mx_tile_kind(const Moe& m, const Groups& g) {
  const int64_t nloc = std::max<int64_t>(1, m.e_end - m.e_begin);
  // positions per tile: the power of two at or above twice the mean rows per
  // local expert, at least 2; at most 16 (two CTAs per SM) while the mean is
  // at most 8, 30 (the widest tile whose accumulators fit half the TMEM) up
  // to a mean of 30, else 60 (one CTA per SM; the one-launch mode caps the
  // kind at 30)
  if (g.rows > 30 * nloc) return kMxKind60;
  if (g.rows > 8 * nloc) return kMxKind30;
  const int64_t target = (2 * g.rows + nloc - 1) / nloc;
  int i = 0;
  while (i < kMxKind30 - 1 && (int64_t(2) << i) < target) ++i;
  return i;
}

namespace {

// One launch of 2 CTAs per SM (every CTA resident: the one-launch mode's
// waits rely on it).  a0 / maps 0 are gate_up's, a1 / maps 1 down's.
template <int MODE, int NT>
cudaError_t launch_tiles(const Moe& m, const mx::Args& a0, const mx::Args& a1,
                         const ExpertBufs& eb, int kind, cudaStream_t st) {
  using D = mx::Tile<NT>;
  auto k = mx::mx_expert_gemm<MODE, NT>;
  const size_t smem = D::SMEM;
  cudaError_t e = set_smem_limit(k, smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(k, dim3(m.sm_count * D::CPS), dim3(D::THREADS), smem, st,
                    *reinterpret_cast<const CUtensorMap*>(m.mx.map_gu),
                    *reinterpret_cast<const CUtensorMap*>(eb.map_xq[kind]),
                    *reinterpret_cast<const CUtensorMap*>(m.mx.map_dn),
                    *reinterpret_cast<const CUtensorMap*>(eb.map_hq[kind]), a0, a1);
}

template <int MODE>
cudaError_t launch_mx(const Moe& m, const mx::Args& a0, const mx::Args& a1,
                      const ExpertBufs& eb, int kind, cudaStream_t st) {
  switch (kind) {
    case 0: return launch_tiles<MODE, 2>(m, a0, a1, eb, kind, st);
    case 1: return launch_tiles<MODE, 4>(m, a0, a1, eb, kind, st);
    case 2: return launch_tiles<MODE, 8>(m, a0, a1, eb, kind, st);
    case 3: return launch_tiles<MODE, 16>(m, a0, a1, eb, kind, st);
    case 4: return launch_tiles<MODE, 30>(m, a0, a1, eb, kind, st);
    default:
      if constexpr (MODE != 2) return launch_tiles<MODE, 60>(m, a0, a1, eb, kind, st);
      return cudaErrorInvalidValue;
  }
}

// K splits for a launch of at most `items` work items on `slots` CTAs: the
// fewest (1..8, at most the K chunks) that fill at least 80 % of the waves,
// within the partial-sum buffer.
int choose_ksplit(int64_t items, int slots, int kchunks, int nt) {
  int best = 1;
  double best_eff = 0.0;
  for (int s = 1; s <= std::min(mx::kMaxSplit, kchunks); ++s) {
    if (s > 1 && (items * s > kMxSplitSlots ||
                  items * s * mx::DM * nt * (int64_t)sizeof(float) > (int64_t)kMxPartialBytes))
      break;
    const int64_t n = items * s;
    const double eff = (double)n / ((double)((n + slots - 1) / slots) * slots);
    if (eff >= 0.8) return s;
    if (eff > best_eff + 1e-9) {
      best_eff = eff;
      best = s;
    }
  }
  return best;
}

mx::Args mx_common(const Moe& m, const Groups& g, const ExpertBufs& eb, int rows) {
  mx::Args a{};
  a.e_begin = m.e_begin;
  a.meta = g.meta;
  a.tile_expert = eb.tile_expert;
  a.tile_row0 = eb.tile_row0;
  a.tile_rows = eb.tile_rows;
  a.limit = m.desc.swiglu_limit;
  a.err = g.meta + 1;
  a.rows = rows;
  a.m_tiles = (rows + mx::DM - 1) / mx::DM;
  a.ksplit = 1;
  a.partial = eb.mx_partial;
  a.arrivals = eb.mx_arrivals;
  a.wait_ns = m.test_wait_ns;
  a.withhold_ready = m.test_withhold_ready;
  return a;
}

// Split K when the tiles cannot fill the CTAs: bounded by the most N tiles a
// grouping of g.rows rows can make.
void set_ksplit(const Moe& m, const Groups& g, int kind, mx::Args& a) {
  const int nt = mx_tile_positions(kind);
  if (kind == kMxKind60) return;  // two epilogue groups per tile: never split
  const int64_t nloc = std::max<int64_t>(1, m.e_end - m.e_begin);
  const int64_t tiles = std::min<int64_t>(g.rows, nloc + g.rows / nt);
  a.ksplit = choose_ksplit(tiles * a.m_tiles, m.sm_count * 2, a.kchunks, nt);
}

mx::Args gate_up_args(const Moe& m, const Groups& g, ExpertBufs& eb, int kind) {
  const gb_moe_desc& d = m.desc;
  mx::Args a = mx_common(m, g, eb, 2 * d.inter);
  a.sfa = m.mx.gu_sfa;
  a.kchunks = m.mx.kc_h;
  a.mt2 = m.mx.mt2_gu;
  a.bias = m.w.gu_bias;
  a.xscale = eb.xscale;
  a.h_exp = m.mx.h_exp;
  a.out_q = eb.hq;
  a.out_stride = d.inter;
  set_ksplit(m, g, kind, a);
  return a;
}

mx::Args down_args(const Moe& m, const Groups& g, ExpertBufs& eb, int kind) {
  const gb_moe_desc& d = m.desc;
  mx::Args a = mx_common(m, g, eb, d.hidden);
  a.sfa = m.mx.dn_sfa;
  a.kchunks = m.mx.kc_i;
  a.mt2 = m.mx.mt2_dn;
  a.bias = m.w.dn_bias;
  a.in_exp = m.mx.h_exp;
  a.out_y = eb.y;
  a.out_rows = g.out_rows;
  a.ret_dst = g.ret_dst;
  for (int q = 0; q < 8; ++q) a.ret_base[q] = g.ret_base[q];
  a.ret_slots = g.ret_slots;
  a.out_stride = d.hidden;
  set_ksplit(m, g, kind, a);
  return a;
}

}  // namespace

int mx_ready_per_tile(const Moe& m) { return (2 * m.desc.inter + mx::DM - 1) / mx::DM; }

bool mx_group_fits(const Moe& m, int64_t T) {
  const gb_moe_desc& d = m.desc;
  return T > 0 && T * d.top_k <= mx::kGroupEntries && d.n_experts <= mx::kGroupExperts &&
         d.top_k <= 8 && d.hidden % 4 == 0;
}

cudaError_t launch_mx_group(const Moe& m, const float* x, int64_t T, Workspace& ws, int kind,
                            cudaStream_t st) {
  const gb_moe_desc& d = m.desc;
  return launch_pdl(mx::group_pieces_kernel, dim3((unsigned)T), dim3(mx::kGroupThreads), 0, st, x,
                    (const int32_t*)ws.idx, (int)T, d.n_experts, d.top_k, d.hidden, m.e_begin,
                    m.e_end, mx_tile_positions(kind), ws.counts, ws.offsets, ws.active, ws.meta,
                    ws.perm, ws.inv, ws.eb.tile_expert, ws.eb.tile_row0, ws.eb.tile_rows,
                    ws.eb.xq, ws.eb.xscale, ws.eb.mx_ready + 1, mx_ready_per_tile(m),
                    ws.eb.mx_ready);
}

cudaError_t launch_mx_gate_up(const Moe& m, const Groups& g, const float* x, ExpertBufs& eb,
                              int kind, cudaStream_t st) {
  const gb_moe_desc& d = m.desc;
  const int positions = (int)g.rows;
  cudaError_t e;
  if (!g.grouped &&
      (e = launch_tile_table(m, g, mx_tile_positions(kind), eb, st)) != cudaSuccess)
    return e;
  if (!g.grouped && positions > 0) {
    if ((e = launch_pdl(mx::split_pieces_kernel, dim3(positions), dim3(128), 0, st, x, g.perm,
                        g.perm_div, d.hidden, positions, eb.xq, eb.xscale)) != cudaSuccess)
      return e;
  }
  const mx::Args a = gate_up_args(m, g, eb, kind);
  return launch_mx<0>(m, a, a, eb, kind, st);
}

cudaError_t launch_mx_down(const Moe& m, const Groups& g, ExpertBufs& eb, int kind,
                           cudaStream_t st) {
  const mx::Args a = down_args(m, g, eb, kind);
  return launch_mx<1>(m, a, a, eb, kind, st);
}

cudaError_t launch_mx_ffn(const Moe& m, const Groups& g, ExpertBufs& eb, int kind,
                          cudaStream_t st) {
  if (!g.grouped || !eb.mx_ready) return cudaErrorInvalidValue;
  mx::Args a0 = gate_up_args(m, g, eb, kind);
  mx::Args a1 = down_args(m, g, eb, kind);
  // down's split-K sums and tickets live in the second half of each buffer
  a1.partial = eb.mx_partial + kMxPartialBytes / sizeof(float);
  a1.arrivals = eb.mx_arrivals + kMxSplitSlots;
  // mx_ready[0] counts the items handed out, the flags follow
  a0.next_item = a1.next_item = eb.mx_ready;
  a0.ready = a1.ready = eb.mx_ready + 1;
  a0.ready_stride = a1.ready_stride = mx_ready_per_tile(m);
  return launch_mx<2>(m, a0, a1, eb, kind, st);
}

}  // namespace gb
