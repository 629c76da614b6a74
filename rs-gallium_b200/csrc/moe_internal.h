// moe_internal.h -- state of a gb_moe handle and the kernel launchers.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/gallium_b200.h"

namespace gb {

// Launches `kern` with programmatic stream serialization: its blocks may be
// scheduled while the previous kernel on the stream finishes (its own
// pdl_wait() orders its memory accesses after that kernel).
// Raises a kernel's dynamic shared-memory limit to `bytes` on the current
// device; the attribute is set once per kernel and device (moe_api.cu).
cudaError_t set_smem_limit_fn(const void* kern, size_t bytes);
template <typename... KArgs>
cudaError_t set_smem_limit(void (*kern)(KArgs...), size_t bytes) {
  return set_smem_limit_fn(reinterpret_cast<const void*>(kern), bytes);
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

// Repacked expert weights of the local experts (device memory).
//
// Layout (MXFP4, one layout for both caller formats):
//   gu_blocks [E_loc][2I][H/32][16]  fused gate_up, row 2i = gate_i, 2i+1 = up_i;
//                                    byte j of a block = elements 2j (low
//                                    nibble) and 2j+1 (high nibble)
//   gu_scales [E_loc][2I][SP_H]      E8M0 bytes, rows padded to SP_H =
//                                    roundup(H/32, 16) so a row's scales start
//                                    16-byte aligned
//   dn_blocks [E_loc][H][I/32][16], dn_scales [E_loc][H][SP_I]
//   gu_bias [E_loc][2I], dn_bias [E_loc][H] f32 (or null)
// zero_scale is the value of an E8M0 byte 0: 0 for safetensors, 2^-127 for
// GGUF (quantized.rs:375-383).
struct ExpertWeights {
  uint8_t* gu_blocks = nullptr;
  uint8_t* gu_scales = nullptr;
  uint8_t* dn_blocks = nullptr;
  uint8_t* dn_scales = nullptr;
  float* gu_bias = nullptr;
  float* dn_bias = nullptr;
  uint8_t* gu_rowmax = nullptr;  // [E_loc][2I] largest E8M0 byte per row (tensor-core path)
  uint8_t* dn_rowmax = nullptr;  // [E_loc][H]
  alignas(64) unsigned char map_gu[128] = {};  // CUtensorMap of gu_blocks (TMA)
  alignas(64) unsigned char map_dn[128] = {};  // CUtensorMap of dn_blocks
  float zero_scale = 0.0f;
  int sp_h = 0, sp_i = 0;  // padded scale row strides
  // GGML Q4_K experts (144-byte super-blocks), gate/up rows interleaved:
  // q4_gu [E_loc][2I][H/256][144], q4_dn [E_loc][H][I/256][144]
  uint8_t* q4_gu = nullptr;
  uint8_t* q4_dn = nullptr;
  // tensor-core Q4_K path: per local expert, weights decode as w * 2^exp
  int32_t* q4_gu_exp = nullptr;  // [E_loc] (one allocation with q4_dn_exp)
  int32_t* q4_dn_exp = nullptr;  // [E_loc]
  // the same bytes tile-interleaved for the tensor-core decoders (q4k_tc.cu
  // q4tc::tile_q4k_kernel): [E_loc][128-row tile][super-block][18432 B]
  uint8_t* q4_gu_t = nullptr;
  uint8_t* q4_dn_t = nullptr;
  // Dense experts (GB_FMT_DENSE), values as stored (bf16 or f32), gate and
  // up rows interleaved: dense_gu [E_loc][2I][H] (row 2i = gate i, 2i + 1 =
  // up i), dense_down [E_loc][H][I]; the shared expert's sh_gu [2Is][H],
  // sh_down [H][Is]
  void* dense_gu = nullptr;
  void* dense_down = nullptr;
  void* sh_gu = nullptr;
  void* sh_down = nullptr;
  bool dense_bf16 = false;
  // CUtensorMaps of the bf16 dense weights (dense_tc.cu): 128-row boxes
  alignas(64) unsigned char map_dense_gu[128] = {};
  alignas(64) unsigned char map_dense_dn[128] = {};
  alignas(64) unsigned char map_sh_gu[128] = {};
  alignas(64) unsigned char map_sh_dn[128] = {};
  // Gemma-4: per-expert output scale [E] (all experts: the combine reads it),
  // input / output norm vectors [H]
  float* expert_scale = nullptr;
  float* router_in_scale = nullptr;
  float* expert_in_norm = nullptr;
  float* out_norm = nullptr;
};

// Weights in the block-scaled tensor-core layout (mx_gemm.cu), built from
// ExpertWeights at load time (KC = roundup(K, 128) / 128):
//   gu_nib [E_loc][KC_H][2I][64 B], dn_nib [E_loc][KC_I][H][64 B]  nibbles,
//     K-chunk major, codes past K zero
//   gu_sfa [E_loc][KC_H][MT2_GU][512], dn_sfa likewise: E8M0 bytes of each
//     128-row x 4-block tile in the MMA's scale-factor order
struct MxWeights {
  bool ok = false;
  uint8_t* gu_nib = nullptr;
  uint8_t* dn_nib = nullptr;
  uint8_t* gu_sfa = nullptr;
  uint8_t* dn_sfa = nullptr;
  int kc_h = 0, kc_i = 0;      // 128-code chunks of gate_up (H) and down (I)
  int mt2_gu = 0, mt2_dn = 0;  // scale atoms per chunk (128-row tiles, even)
  int h_exp = 0;               // h enters down as pieces of h * 2^-h_exp
  int64_t weight_bytes = 0;
  alignas(64) unsigned char map_gu[128] = {};  // CUtensorMaps, 256-row boxes of one chunk
  alignas(64) unsigned char map_dn[128] = {};
};

// The grouped view the expert kernels work on: rows grouped by expert
// (expert ascending), each group a contiguous range of positions.
struct Groups {
  const int32_t* counts = nullptr;    // [E] rows per (global) expert id
  const int32_t* offsets = nullptr;   // [E+1] first position of each expert
  const int32_t* active = nullptr;    // local experts with rows (global ids), ascending
  int32_t* meta = nullptr;            // [0] active count, [1] error bits, [2] N tiles
  const int32_t* perm = nullptr;      // position -> input row * perm_div (+ slot)
  int perm_div = 1;
  int64_t rows = 0;                   // positions in use this forward (upper bound)
  int max_active = 0;                 // bound on the active count (grid size)
  int64_t max_per_expert = 0;         // bound on the rows of one expert
  const int32_t* out_rows = nullptr;  // output row of position p for DOWN (null: p)
  bool grouped = false;  // tile table and activation pieces already written (mx_group)
  // Expert parallel: the output row of position p belongs in return slot
  // (ret_dst[p] & 0xffffffff) of rank ret_dst[p] >> 32, at ret_base[rank] +
  // slot * H (peer addresses).  A down kernel that stores there itself
  // reports it through run_experts; otherwise rows stay in ExpertBufs::y.
  const int64_t* ret_dst = nullptr;
  float* ret_base[8] = {};
  int64_t ret_slots = 0;  // slots per rank (bounds every store)
};

// Positions per tile of the small-batch Q4_K tensor-core kernel (q4k_tc.cu).
constexpr int kQ4SmallBN = 32;
// Rows per TMA box of that kernel's activation maps (a tile's f16 hi and lo
// rows are loaded back to back, 16 rows at a time).
constexpr int kQ4SmallBox = 16;

// Buffers indexed by grouped position, sized for rows_cap positions.
struct ExpertBufs {
  int64_t rows_cap = 0;
  size_t bytes = 0;
  void* base = nullptr;
  float* h = nullptr;          // [rows, I] SwiGLU output (CUDA-core paths)
  float* y = nullptr;          // [rows, H] expert outputs (row = out_rows[p] or p)
  __half* xh = nullptr;        // [rows, H] grouped activation rows, f16 hi (tensor cores)
  __half* xl = nullptr;        // [rows, H] f16 lo
  float* xscale = nullptr;     // [rows] exponent s of each row (x = 2^s (hi + lo))
  __half* hh = nullptr;        // [rows, I] SwiGLU output, f16 hi
  __half* hl = nullptr;        // [rows, I] f16 lo
  int32_t* tile_expert = nullptr;  // [rows + E + 1] N-tile table (tiles of >= 1 row)
  int32_t* tile_row0 = nullptr;
  int32_t* tile_rows = nullptr;
  alignas(64) unsigned char map_xh[128] = {};  // CUtensorMap of xh (TMA)
  alignas(64) unsigned char map_xl[128] = {};
  alignas(64) unsigned char map_hh[128] = {};
  alignas(64) unsigned char map_hl[128] = {};
  // the same four in boxes of kQ4SmallBox rows (small-batch Q4_K kernel)
  alignas(64) unsigned char map_xh_s[128] = {};
  alignas(64) unsigned char map_xl_s[128] = {};
  alignas(64) unsigned char map_hh_s[128] = {};
  alignas(64) unsigned char map_hl_s[128] = {};
  float* xsum = nullptr;       // [rows][max(H, I) / 32] sub-block sums of x or h (Q4_K)
  uint8_t* xq = nullptr;       // [rows][4][H] E4M3 pieces of the grouped activations
  uint8_t* hq = nullptr;       // [rows][4][I] E4M3 pieces of the SwiGLU output
  alignas(64) unsigned char map_xq[6][128] = {};  // CUtensorMaps, tiles of 2, 4, 8, 16, 30,
  alignas(64) unsigned char map_hq[6][128] = {};  // 60 positions (index: kind)
  float* mx_partial = nullptr;  // split-K partial sums (2 x kMxPartialBytes: gate_up, down)
  int* mx_arrivals = nullptr;   // split-K tickets [2 x kMxSplitSlots], zero between forwards
  int* mx_ready = nullptr;      // one-launch expert kernel: [0] item counter, then
                                //   [tile][gate_up M tile] ready flags
  bool maps_ok = false;
  bool mx_maps_ok = false;
};

// Per-forward routing scratch, sized for `tokens` local tokens.
struct Workspace {
  int64_t tokens = 0;
  size_t bytes = 0;
  void* base = nullptr;
  float* logits = nullptr;     // [T, E] router logits
  unsigned* tickets = nullptr; // [T] per token tile, zero between forwards
  unsigned* grid_bar = nullptr;  // [2] fused decode kernel's grid barrier (arrivals, generation)
  int32_t* idx = nullptr;      // [T*k]
  float* wts = nullptr;        // [T*k]
  int32_t* counts = nullptr;   // [E]
  int32_t* offsets = nullptr;  // [E+1]
  int32_t* active = nullptr;   // [E] active local expert ids, ascending
  int32_t* meta = nullptr;     // [0] active count, [1] error flags, [2] N tiles
  int32_t* perm = nullptr;     // [T*k]
  int32_t* inv = nullptr;      // [T*k]
  float* x_route = nullptr;    // [T, H] the router's input (input_norm 1)
  float* x_expert = nullptr;   // [T, H] the experts' input (input_norm 1)
  float* sh_h = nullptr;       // [T, Is] shared expert's activation (GB_FMT_DENSE)
  float* sh_y = nullptr;       // [T, H] shared expert's output
  // shared expert on the tensor cores (bf16 dense weights): x and h as bf16
  // hi / lo, [T, H] and [T, Is], with their CUtensorMaps
  __nv_bfloat16* sh_xh = nullptr;
  __nv_bfloat16* sh_xl = nullptr;
  __nv_bfloat16* sh_hh = nullptr;
  __nv_bfloat16* sh_hl = nullptr;
  alignas(64) unsigned char map_sh_xh[128] = {};
  alignas(64) unsigned char map_sh_xl[128] = {};
  alignas(64) unsigned char map_sh_hh[128] = {};
  alignas(64) unsigned char map_sh_hl[128] = {};
  float* x_stage = nullptr;    // [T, H] host-path staging
  float* out_stage = nullptr;  // [T, H]
  ExpertBufs eb;               // single GPU: T*k positions
};

constexpr int kHostChunksMax = 8;  // host-buffer forward: chunks per call

struct Moe {
  gb_moe_desc desc{};  // copy; host pointers inside are not kept valid
  int device = 0;
  int sm_count = 0;
  int e_begin = 0, e_end = 0;  // local experts
  int ep_rank = 0, ep_size = 1;
  // router, replicated on every rank
  float* router_w = nullptr;  // [E][H] f32 (bf16 widened exactly)
  float* router_b = nullptr;  // [E] or null
  float* sel_bias = nullptr;  // [E] or null
  ExpertWeights w;
  MxWeights mx;
  int64_t weight_bytes = 0;
  Workspace ws;
  struct Ep* ep = nullptr;  // expert-parallel state (ep_size > 1), ep.cu
  // profiling: events at the stage boundaries of the last forward
  static constexpr int kStages = 5;  // router, permute, gate_up, down, combine
  bool profiling = false;
  bool profiled_once = false;
  cudaEvent_t ev[kStages + 1] = {};
  int64_t launches = 0;
  int expert_path = 0;  // gb_expert_path
  // gb_moe_set_test_hooks: bounded-wait limit of the block-scaled kernels
  // (0 = default) and the withheld ready flag of the one-launch kernel
  uint64_t test_wait_ns = 0;
  int test_withhold_ready = 0;
  int fused_ctas = 0;  // CTAs of the fused decode kernel's cooperative grid (0: unavailable)
  // gb_moe_forward_host pipelining: copy streams and chunk events (lazily made)
  cudaStream_t h2d = nullptr, d2h = nullptr;
  cudaEvent_t host_ev[2 + 2 * kHostChunksMax] = {};
  // Replayed forwards: one CUDA graph per (x, out, T), captured on `cap` the
  // second time a single-GPU forward of at most kGraphMaxTokens tokens meets
  // that triple (a triple seen once sits in `seen`); least recently used
  // replaced.  Cleared whenever the workspace, the expert path or the graph
  // count changes.
  struct Graph {
    const float* x = nullptr;
    float* out = nullptr;
    int64_t T = 0;
    cudaGraphExec_t exec = nullptr;
    int64_t launches = 0;  // kernels in the graph
    uint64_t used = 0;
  };
  static constexpr int kGraphSlots = 16;
  static constexpr int64_t kGraphMaxTokens = 512;
  Graph graphs[kGraphSlots];
  Graph seen[kGraphSlots];  // exec unused
  int graph_slots = kGraphSlots;  // gb_moe_set_graphs; 0 = launch kernels directly
  uint64_t graph_clock = 0;
  int64_t graph_captures = 0;
  cudaStream_t cap = nullptr;
};

// Records an error message for gb_last_error() and returns `code`.
int set_error(int code, const char* fmt, ...);

// Records stage boundary event i on `st` when profiling is on.
int mark_stage(Moe& m, int i, cudaStream_t st);

// Launchers.  All asynchronous on `st`.
cudaError_t launch_router_topk(const Moe& m, const float* x, int64_t T, int32_t* idx, float* wts,
                               cudaStream_t st);
cudaError_t launch_permute(const Moe& m, const int32_t* idx, int64_t T, Workspace& ws,
                           cudaStream_t st);

// CUDA-core expert kernels, any shape (expert_gemv.cu).
cudaError_t launch_gate_up(const Moe& m, const Groups& g, const float* x, ExpertBufs& eb,
                           cudaStream_t st);
cudaError_t launch_down(const Moe& m, const Groups& g, ExpertBufs& eb, cudaStream_t st);
// Decode-sized expert GEMV (decode_gemv.cu); needs H, I multiples of 64.
bool decode_supported(const Moe& m);
cudaError_t launch_decode_gate_up(const Moe& m, const Groups& g, const float* x, ExpertBufs& eb,
                                  cudaStream_t st);
cudaError_t launch_decode_down(const Moe& m, const Groups& g, ExpertBufs& eb, cudaStream_t st);

// Q4_K expert kernels on the tensor cores (q4k_tc.cu): kind::f16 with the
// weights split into f16 hi + lo while they are decoded.
bool q4k_tc_supported(const Moe& m);
cudaError_t q4k_tc_prepare(Moe& m);
cudaError_t launch_q4k_tc_gate_up(const Moe& m, const Groups& g, const float* x, ExpertBufs& eb,
                                  cudaStream_t st);
cudaError_t launch_q4k_tc_down(const Moe& m, const Groups& g, ExpertBufs& eb, cudaStream_t st);
// Whether this batch runs the small-batch Q4_K kernel (weights as exact
// integers, at most kQ4SmallBN positions per tile) rather than the f16 hi + lo one.
bool use_q4k_small(const Moe& m, const Groups& g);
// Activation rows (through perm) -> f16 hi / lo with a per-row power of two
// (tc_gemm.cu), the B operand of the kind::f16 kernels.
cudaError_t launch_split_gather(const Moe& m, const Groups& g, const float* x, ExpertBufs& eb,
                                cudaStream_t st);

// Q4_K expert kernels (q4k_gemv.cu).
cudaError_t launch_q4k_gate_up(const Moe& m, const Groups& g, const float* x, ExpertBufs& eb,
                               cudaStream_t st);
cudaError_t launch_q4k_down(const Moe& m, const Groups& g, ExpertBufs& eb, cudaStream_t st);
cudaError_t launch_q4k_dequant(const Moe& m, int which, int local_expert, float* out,
                               cudaStream_t st);

// Block-scaled tensor-core expert path (mx_gemm.cu).
constexpr int kMxTileKinds = 6;  // tiles of 2, 4, 8, 16, 30, 60 positions
constexpr int kMxKind30 = 4;     // the widest tile of the one-launch mode
constexpr int kMxKind60 = 5;     // gate_up / down launched alone, one CTA per SM
constexpr size_t kMxPartialBytes = size_t(8) << 20;  // split-K partial sums
constexpr int kMxSplitSlots = 4096;                  // split-K tiles x splits
constexpr int kMxGroupEntries = 512;  // routing entries of the one-launch grouping
// Grouped forwards of at least this many positions run gate_up and down as
// one launch; below it the two launches measured faster (the wait for h
// chunks costs more than the second launch when each CTA has one item).
constexpr int64_t kMxOneLaunchRows = 24;
bool mx_supported(const Moe& m);
cudaError_t mx_prepare_weights(Moe& m);
void mx_release(MxWeights& x);
cudaError_t mx_make_maps(const Moe& m, ExpertBufs& eb);
size_t mx_piece_bytes(int64_t rows, int k);
// Tile kind for a grouping of this size, and the positions per tile of a kind.
int mx_tile_kind(const Moe& m, const Groups& g);
int mx_tile_positions(int kind);
// Small single-GPU batches: grouping, tile table and pieces in one launch
// (replaces launch_permute, the tile table and the pieces of launch_mx_gate_up).
bool mx_group_fits(const Moe& m, int64_t T);
cudaError_t launch_mx_group(const Moe& m, const float* x, int64_t T, Workspace& ws, int kind,
                            cudaStream_t st);
// gate_up and down in one launch (needs g.grouped): the down copies of h wait
// per K chunk for the gate_up tile that writes it.
cudaError_t launch_mx_ffn(const Moe& m, const Groups& g, ExpertBufs& eb, int kind,
                          cudaStream_t st);
int mx_ready_per_tile(const Moe& m);  // gate_up M tiles = down K chunks
cudaError_t launch_mx_gate_up(const Moe& m, const Groups& g, const float* x, ExpertBufs& eb,
                              int kind, cudaStream_t st);
cudaError_t launch_mx_down(const Moe& m, const Groups& g, ExpertBufs& eb, int kind,
                           cudaStream_t st);

// N-tile table of the local experts' grouped rows, tiles of bn rows (tc_gemm.cu).
cudaError_t launch_tile_table(const Moe& m, const Groups& g, int bn, ExpertBufs& eb,
                              cudaStream_t st);

// Tensor-core expert path (tc_gemm.cu).
bool tc_supported(const Moe& m);
cudaError_t tc_prepare_weights(Moe& m);
cudaError_t tc_make_maps(const Moe& m, ExpertBufs& eb);
cudaError_t launch_tc_gate_up(const Moe& m, const Groups& g, const float* x, ExpertBufs& eb,
                              cudaStream_t st);
cudaError_t launch_tc_down(const Moe& m, const Groups& g, ExpertBufs& eb, cudaStream_t st);

// out[t] = sum_r w[t, r] * y[inv[t*k + r]] in the fixed order (expert_gemv.cu);
// with `slots`, y is indexed by t*k + r directly (expert-parallel return slots).
cudaError_t launch_combine(const Moe& m, int64_t T, const Workspace& ws, const float* y, float* out,
                           cudaStream_t st, bool slots = false);

// Gemma-4 norms (norm.cu): the router's and the experts' inputs from x, and
// the output norm in place.
cudaError_t launch_input_norms(const Moe& m, const float* x, int64_t T, float* x_route,
                               float* x_expert, cudaStream_t st);
cudaError_t launch_output_norm(const Moe& m, float* out, int64_t T, cudaStream_t st);

// The whole layer in one cooperative launch for decode-sized single-GPU
// batches of MXFP4 experts (decode_fused.cu).
bool fused_decode_fits(const Moe& m, int64_t T);
cudaError_t fused_decode_prepare(Moe& m);
cudaError_t launch_fused_decode(const Moe& m, const float* x, int64_t T, float* out,
                                cudaStream_t st);

// Dense experts on CUDA cores (dense_gemv.cu): the generic MoEFFN.
cudaError_t launch_dense_gate_up(const Moe& m, const Groups& g, const float* x, ExpertBufs& eb,
                                 cudaStream_t st);
cudaError_t launch_dense_down(const Moe& m, const Groups& g, ExpertBufs& eb, cudaStream_t st);
// The shared expert over all T tokens: h [T, Is], y [T, H] (ws.sh_h / sh_y).
cudaError_t launch_shared_expert(const Moe& m, const float* x, int64_t T, float* h, float* y,
                                 cudaStream_t st);
// Stored dense weights of one local expert widened to f32 (which: 0 gate,
// 1 up, 2 down), for gb_moe_dequant_expert.
cudaError_t launch_dense_dequant(const Moe& m, int which, int local_expert, float* out,
                                 cudaStream_t st);

// Dense bf16 experts on the tensor cores (dense_tc.cu): kind::f16 with the
// activations split into bf16 hi + lo.  The routed experts use the grouped
// buffers of ExpertBufs (xh / xl / hh / hl hold bf16 there) and the tile
// table; the shared expert the workspace's sh_x* / sh_h* buffers.
bool dense_tc_supported(const Moe& m);
bool dense_tc_shared_supported(const Moe& m);
cudaError_t dense_tc_prepare(Moe& m);
cudaError_t dense_tc_make_maps(const Moe& m, ExpertBufs& eb);
cudaError_t dense_tc_make_ws_maps(const Moe& m, Workspace& ws);
cudaError_t launch_dense_tc_gate_up(const Moe& m, const Groups& g, const float* x,
                                    ExpertBufs& eb, cudaStream_t st);
cudaError_t launch_dense_tc_down(const Moe& m, const Groups& g, ExpertBufs& eb, cudaStream_t st);
cudaError_t launch_shared_expert_tc(const Moe& m, const float* x, int64_t T, float* y,
                                    cudaStream_t st);
// Whether the shared expert of a T-token forward runs on the tensor cores.
bool use_dense_tc_shared(const Moe& m, int64_t T);

// Plain bf16-weight linear layers on the same tensor-core kernel (the GPT-OSS
// decode stack's projections and LM head, decoder.cu).
// make_bf16_map: CUtensorMap of a bf16 [rows][K] matrix, boxes of box_rows
// rows x 64 columns, 128-byte swizzle (K a multiple of 64).
cudaError_t make_bf16_map(void* map, const void* base, uint64_t K, uint64_t rows,
                          uint32_t box_rows);
constexpr int kLinearBoxRows = 128;  // weight rows and activation rows per tile
// f32 rows (through perm / perm_div when perm is set) -> bf16 hi / lo [positions][H].
cudaError_t split_rows(const float* x, const int32_t* perm, int perm_div, int H, int64_t positions,
                       __nv_bfloat16* xh, __nv_bfloat16* xl, cudaStream_t st);
// out[p][r] = (add_out ? out[p][r] : 0) + (W[r] . x[p] + bias[r]) for p < n_pos,
// r < rows: map_w of W [rows][K], map_xh / map_xl of the split activations.
// When the tiles would leave SMs idle, K is split and the partial sums (in
// `part`, up to part_floats floats) are folded in a fixed order by a second
// kernel.
cudaError_t launch_linear_tc(int sm_count, const void* map_w, const void* map_xh,
                             const void* map_xl, int K, int rows, int n_pos, const float* bias,
                             float* out, int out_stride, bool add_out, int* err, float* part,
                             int64_t part_floats, cudaStream_t st);
cudaError_t launch_dequant_expert(const Moe& m, int which, int local_expert, float* out,
                                  cudaStream_t st);
cudaError_t launch_gguf_to_split(const uint8_t* raw_dev, int64_t rows, int k, uint8_t* blocks_dev,
                                 int64_t row_stride_blocks, uint8_t* scales_dev,
                                 int64_t row_stride_scales, cudaStream_t st);

// Expert parallelism (ep.cu).
struct Ep;
int nccl_unique_id(uint8_t out[128]);
// The EP grouping's meta array ([1] holds error bits), or null without EP.
int32_t* ep_meta(Moe& m);
int ep_init(Moe& m, const uint8_t* nccl_id);
void ep_destroy(Moe& m);
int ep_forward(Moe& m, const float* x, int64_t T, float* out, cudaStream_t st);
// Tokens per rank an expert-parallel forward may hold (0 without EP).
int64_t ep_capacity(const Moe& m);
// Split-K tickets of the expert-parallel expert buffers (null without EP).
int* ep_arrivals(Moe& m);
// Largest v over the ranks (a collective: every rank calls it).
int ep_agree_max(Moe& m, int64_t v, int64_t* out, cudaStream_t st);

// Allocates the grouped-position buffers for `rows` positions (and their TMA
// descriptors when the tensor-core path applies); frees the previous ones.
int alloc_expert_bufs(const Moe& m, ExpertBufs& eb, int64_t rows);
void free_expert_bufs(ExpertBufs& eb);

// Runs the expert products for a grouped view, choosing the kernels for T
// (local tokens) and the handle's expert path.  Returns a gb_status.  With
// g.ret_dst set, *stored_return tells whether the down kernel stored the
// output rows in their return slots itself.
int run_experts(Moe& m, const Groups& g, const float* x, int64_t T, ExpertBufs& eb,
                cudaStream_t st, bool* stored_return = nullptr);

}  // namespace gb
