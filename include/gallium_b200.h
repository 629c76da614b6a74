/*
 * gallium_b200.h -- C ABI of the B200 (sm_100a) mixture-of-experts FFN block.
 *
 * This library replaces the MoE FFN blocks of rs-gallium:
 *   - OssMoEFFN::forward  (crates/gallium-models/src/gpt_oss.rs:166-231, safetensors GPT-OSS)
 *   - QMoEFFN::forward    (crates/gallium-models/src/gpt_oss_q.rs:165-269, GGUF GPT-OSS)
 *   - QMoEFFN::forward    (crates/gallium-models/src/lfm2moe_q.rs:234-313, LFM2.5)
 * whose common shape is `fn forward(&self, x: &Tensor) -> Result<Tensor>` with
 * x of shape (batch, seq, hidden) (gallium-core FfnImpl::forward,
 * crates/gallium-core/src/ffn.rs:175-181).  The weights those structs load in
 * `load` (gpt_oss.rs:115-142, gpt_oss_q.rs:135-163, lfm2moe_q.rs:214-232) are
 * handed to gb_moe_create as host buffers; the library copies and repacks them
 * into its own device layout once.
 *
 * Conventions:
 *   - Every function returns a gb_status; on failure gb_last_error() (per
 *     thread) holds a message.  Nothing aborts and no kernel traps.
 *   - Pointers named *_dev are device pointers on the handle's device; all
 *     other buffer pointers are host pointers.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *   - A handle is not re-entrant: one forward at a time per handle, like the
 *     reference, where the model is borrowed mutably per generation
 *     (crates/gallium-agent/src/llm_candle.rs:199).
 */
#ifndef GALLIUM_B200_H
#define GALLIUM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GB_ABI_VERSION 4

typedef enum gb_status {
  GB_OK = 0,
  GB_ERR_INVALID_ARG = 1, /* null pointer, bad enum, top_k > experts, ...   */
  GB_ERR_SHAPE = 2,       /* ragged quant blocks (quantized.rs:417-425), ... */
  GB_ERR_CUDA = 3,        /* a CUDA runtime call failed                       */
  GB_ERR_NCCL = 4,        /* an NCCL call failed (expert parallel only)       */
  GB_ERR_TIMEOUT = 5,     /* a bounded device or host wait ran out            */
  GB_ERR_UNSUPPORTED = 6, /* valid request this build does not implement      */
  GB_ERR_NO_MEMORY = 7    /* host or device allocation failed                 */
} gb_status;

/* Router: GPT-OSS softmax over all experts, the k largest probabilities
 * (equal ones by lower index) renormalised to sum 1 (gpt_oss.rs:172-182), or
 * the LFM2.5 sigmoid router whose selection bias steers selection only
 * (lfm2moe_q.rs:241-258). */
typedef enum { GB_ROUTER_SOFTMAX_TOPK = 0, GB_ROUTER_SIGMOID_TOPK = 1 } gb_router_kind;

/* Expert activation: GPT-OSS clamped SwiGLU (gpt_oss.rs:202-212), or a gated
 * h = act(gate) * up with act one of gallium-core's Activation
 * (ffn.rs:4-24): SiLU (also the LFM2.5 experts, lfm2moe_q.rs:287-290), GELU
 * (erf), GELU (tanh), ReLU.  The gated kinds clamp act(gate) to
 * [-act_clamp, act_clamp] when act_clamp > 0 (ffn.rs:56-66).  GELU, GELU_TANH
 * and RELU apply to GB_FMT_DENSE experts. */
typedef enum {
  GB_ACT_GPTOSS_CLAMP = 0,
  GB_ACT_SILU = 1,
  GB_ACT_GELU = 2,
  GB_ACT_GELU_TANH = 3,
  GB_ACT_RELU = 4
} gb_act_kind;

/* Expert weight format as the caller holds it. */
typedef enum {
  /* Safetensors MXFP4 (gpt_oss.rs:96-164): fused gate_up with interleaved
   * rows (row 2i = gate_i, 2i+1 = up_i).  *_blocks [E, rows, K/32, 16] u8,
   * byte j holding elements 2j (low nibble) and 2j+1 (high nibble);
   * *_scales [E, rows, K/32] u8, value 2^(s-127), s == 0 -> 0. */
  GB_FMT_MXFP4_SPLIT = 0,
  /* GGUF type 39 (quantized.rs:361-449): separate gate/up [E, I, H] and down
   * [E, H, I] tensors of 17-byte blocks [e8m0, 16 bytes]; low nibble of byte
   * j -> element j, high nibble -> j+16. */
  GB_FMT_MXFP4_GGUF = 1,
  /* GGML Q4_K (144-byte, 256-element super-blocks), separate gate/up/down
   * like GGUF (quantized.rs:139-178, the LFM2.5 experts of
   * lfm2moe_q.rs:203-232).  H and I multiples of 256. */
  GB_FMT_Q4_K = 2,
  /* Dense expert weights in weight_dtype (gallium-core MoEFFN's GatedFFN
   * experts, ffn.rs:30-67, 72-166): gate_raw, up_raw [E, I, H], down_raw
   * [E, H, I], no biases; router_weight [E, H], no bias; combine in rank
   * order; optional shared expert.  bf16 weights run on the tensor cores
   * (from one grouped position per two local experts, and H, I multiples of
   * 64), f32 weights on the CUDA cores. */
  GB_FMT_DENSE = 3
} gb_weight_format;

typedef enum { GB_DTYPE_F32 = 0, GB_DTYPE_BF16 = 1 } gb_dtype;

/* Everything gb_moe_create needs.  Zero-initialise, set struct_size =
 * sizeof(gb_moe_desc), then fill in.  Host pointers; the library copies what
 * it needs and keeps no reference after create returns. */
typedef struct gb_moe_desc {
  uint32_t struct_size;
  int32_t hidden;        /* H (multiple of 32; 256 for Q4_K)               */
  int32_t inter;         /* I, expert intermediate size (same rule)         */
  int32_t n_experts;     /* E (<= 256)                                       */
  int32_t top_k;         /* k (1..8, <= E)                                   */
  int32_t router_kind;   /* gb_router_kind                                   */
  int32_t act_kind;      /* gb_act_kind                                      */
  int32_t weight_format; /* gb_weight_format                                 */
  float swiglu_limit;    /* GPT-OSS clamp limit (config swiglu_limit, 7.0)   */
  int32_t device;        /* CUDA device ordinal                              */
  int32_t max_tokens;    /* workspace is sized for this many tokens; a
                            forward with more tokens grows it (synchronously) */

  /* Router: weight [E, H], bias [E] (NULL = none), in router_dtype. */
  const void* router_weight;
  const void* router_bias;
  int32_t router_dtype; /* gb_dtype */
  /* Sigmoid router selection bias [E] f32 (exp_probs_b, lfm2moe_q.rs:216-221);
   * NULL = zeros. */
  const float* selection_bias;

  /* GB_FMT_MXFP4_SPLIT */
  const uint8_t* gate_up_blocks; /* [E, 2I, H/32, 16] */
  const uint8_t* gate_up_scales; /* [E, 2I, H/32]     */
  const uint8_t* down_blocks;    /* [E, H, I/32, 16]  */
  const uint8_t* down_scales;    /* [E, H, I/32]      */

  /* GB_FMT_MXFP4_GGUF / GB_FMT_Q4_K: raw block bytes */
  const uint8_t* gate_raw; /* [E, I, H] */
  const uint8_t* up_raw;   /* [E, I, H] */
  const uint8_t* down_raw; /* [E, H, I] */

  /* Biases in bias_dtype, NULL = none.  SPLIT: gate_up_bias [E, 2I]
   * (interleaved like the rows).  GGUF: gate_bias, up_bias [E, I].
   * down_bias [E, H] for both. */
  const void* gate_up_bias;
  const void* gate_bias;
  const void* up_bias;
  const void* down_bias;
  int32_t bias_dtype; /* gb_dtype */

  /* Expert parallelism (one process per GPU).  ep_size 1 = single GPU.
   * For ep_size > 1 every rank passes the same full [E, ...] weight arrays
   * (or at least valid pointers covering its own experts); rank r keeps
   * experts [r*E/ep_size, (r+1)*E/ep_size).  nccl_id is the 128-byte
   * ncclUniqueId from gb_nccl_unique_id() on rank 0, shared out of band. */
  int32_t ep_rank;
  int32_t ep_size;
  const uint8_t* nccl_id;
  /* Expert parallel: how long a host or device wait for the other ranks may
   * last, in milliseconds (0 = 60000).  A wait that runs out aborts the
   * communicator and the call returns GB_ERR_TIMEOUT (host) or the device
   * status reports it; the handle then refuses further forwards and must be
   * destroyed on every rank. */
  int32_t ep_timeout_ms;

  /* GB_FMT_DENSE: dtype of gate_raw / up_raw / down_raw and of the shared
   * expert's weights (gb_dtype). */
  int32_t weight_dtype;
  /* Gated activations: clamp of act(gate) to [-act_clamp, act_clamp]; 0 = none. */
  float act_clamp;
  /* GB_FMT_DENSE: shared expert over all tokens, added after the routed
   * combine (ffn.rs:160-163); shared_inter 0 = none.  shared_gate,
   * shared_up [shared_inter, H], shared_down [H, shared_inter], weight_dtype. */
  int32_t shared_inter;
  const void* shared_gate;
  const void* shared_up;
  const void* shared_down;

  /* Gemma-4's routed experts (QGemmaMoe, gemma4_q.rs:187-330):
   * gate_up_merged != 0 (GGUF MXFP4 / Q4_K): gate_raw holds the merged
   *   [E, 2I, H] tensor, gate rows [0, I) then up rows [I, 2I); up_raw unused.
   * expert_scale [E] f32: each expert's output row is multiplied by it
   *   before the routing weight (ffn_down_exps.scale); NULL = none.
   * input_norm 1: the router reads rms(x) * H^-0.5 * router_input_scale and
   *   the experts read rms_norm(x) * expert_input_norm (both [H] f32), where
   *   rms(x) = x / sqrt(mean(x^2) + rms_eps); 0 = both read x.
   * output_norm [H] f32: the result is rms_norm(result) * output_norm
   *   (post_ffw_norm_2); NULL = none. */
  int32_t gate_up_merged;
  const float* expert_scale;
  int32_t input_norm;
  const float* router_input_scale;
  const float* expert_input_norm;
  const float* output_norm;
  float rms_eps;
} gb_moe_desc;

typedef struct gb_moe gb_moe;

/* Information about a created handle. */
typedef struct gb_moe_info {
  uint32_t struct_size;
  int32_t local_expert_begin, local_expert_end;
  int64_t weight_bytes;    /* device bytes of the expert weights in every
                              layout the kernels read (row layout, plus the
                              block-scaled MXFP4 or tiled Q4_K copy)        */
  int64_t workspace_bytes; /* device bytes of the current workspace        */
  int32_t workspace_tokens;
  int32_t sm_count;
  int64_t kernel_launches;  /* kernels this handle has launched so far */
  int64_t graph_captures;   /* forward graphs captured so far (gb_moe_set_graphs) */
} gb_moe_info;

/* Create: validates the descriptor, uploads and repacks the weights.
 * Replaces OssMoEFFN::load (gpt_oss.rs:115-142), QMoEFFN::load
 * (gpt_oss_q.rs:135-163) and QMoEFFN::load (lfm2moe_q.rs:214-232). */
int gb_moe_create(const gb_moe_desc* desc, gb_moe** out);

/* Forward: x_dev [T, H] f32 row-major -> out_dev [T, H] f32, both 16-byte
 * aligned (GB_ERR_INVALID_ARG otherwise).  Asynchronous on `stream`.  Replaces the forward methods listed at the top of this file;
 * the caller flattens (batch, seq) into T and adds the residual itself, as
 * gpt_oss.rs:385 and gpt_oss_q.rs:296 do.  T == 0 is a no-op.
 * Expert parallel (ep_size > 1): every rank calls the forward the same
 * number of times (T may differ, 0 included); the call waits on the host
 * for the other ranks' expert counts, then returns with the rest queued;
 * T may not exceed the largest max_tokens the ranks gave at create. */
int gb_moe_forward(gb_moe* m, const float* x_dev, int64_t T, float* out_dev, void* stream);

/* Same with host buffers: copies x in, runs, copies out, and synchronises
 * the stream before returning (the path a candle CPU tensor takes). */
int gb_moe_forward_host(gb_moe* m, const float* x_host, int64_t T, float* out_host,
                        void* stream);

/* Routing only, for parity checks (gpt_oss.rs:172-182 / lfm2moe_q.rs:241-264
 * and the grouping of gpt_oss_q.rs:175-192).  Device outputs, any may be NULL:
 *   idx_dev [T, k] i32, expert per rank, ranks in descending router order;
 *   w_dev [T, k] f32, combine weights;
 *   counts_dev [E] i32, offsets_dev [E+1] i32 (exclusive prefix);
 *   perm_dev [T*k] i32, entry t*k+r at each sorted position (expert
 *   ascending, then token ascending).
 * x_dev is 16-byte aligned (GB_ERR_INVALID_ARG otherwise).  Synchronises the
 * stream. */
int gb_moe_route(gb_moe* m, const float* x_dev, int64_t T, int32_t* idx_dev, float* w_dev,
                 int32_t* counts_dev, int32_t* offsets_dev, int32_t* perm_dev, void* stream);

/* Dequantise one local expert's matrix from the repacked device layout to
 * f32, for parity checks of the repack and the in-kernel decoder.
 * which: 0 = gate (gate rows of the fused gate_up), 1 = up, 2 = down.
 * out_dev [rows, K] f32 (gate/up: [I, H]; down: [H, I]). Synchronises. */
int gb_moe_dequant_expert(gb_moe* m, int32_t which, int32_t expert, float* out_dev,
                          void* stream);

int gb_moe_get_info(const gb_moe* m, gb_moe_info* info);

/* Error bits the forward kernels recorded on the device since the last call:
 * synchronises `stream`, reads and clears them.  Returns GB_OK, or
 * GB_ERR_TIMEOUT when a tensor-core pipeline wait ran out (that forward's
 * output is invalid), or GB_ERR_INVALID_ARG when routing produced an expert
 * index out of range.  gb_moe_forward_host checks them itself; callers of
 * the asynchronous gb_moe_forward call this when they consume the output.
 * No counterpart in the reference, whose CPU path has no asynchronous
 * failure. */
int gb_moe_device_status(gb_moe* m, void* stream);

/* Which kernels run the expert products.  AUTO and TENSOR_CORES pick the
 * block-scaled tcgen05 GEMM (MXFP4 weights as stored, activations as four
 * E4M3 pieces, tiles of 256 weight rows x 2-32 positions chosen from the
 * batch); CUDA_CORES forces the streaming MXFP4 rows with f32 FMA;
 * TENSOR_CORES_F16 the kind::f16 GEMM that decodes the weights to f16 in
 * shared memory (activations as f16 hi + lo, 128-position tiles).  The
 * tensor-core kernels need the GPT-OSS activation and H, I multiples of 64;
 * without them every path uses the CUDA cores.  Q4_K experts: AUTO runs the
 * CUDA cores below 2 grouped rows per local expert on average and kind::f16
 * tcgen05 from there (weights as the exact integers sc * q up to 24 rows per
 * expert, as f16 hi + lo above); TENSOR_CORES takes the tensor cores at any
 * size, TENSOR_CORES_F16 the hi + lo kernel.  Dense bf16 experts: AUTO runs
 * kind::f16 tcgen05 from one grouped row per two local experts, the CUDA
 * cores below that and for f32 weights.  No counterpart in the reference,
 * which has one CPU path. */
typedef enum {
  GB_PATH_AUTO = 0,
  GB_PATH_CUDA_CORES = 1,
  GB_PATH_TENSOR_CORES = 2,
  GB_PATH_TENSOR_CORES_F16 = 3,
  /* A single-GPU MXFP4 batch of at most 8 tokens (32 token-expert entries)
   * as one cooperative launch: router, grouping, expert rows streamed on the
   * CUDA cores, combine, with bounded grid barriers between them; larger
   * batches as TENSOR_CORES.  Measured slower than TENSOR_CORES at every
   * size it takes (1 token: 77 vs 52 us at 128 experts), so AUTO does not
   * choose it. */
  GB_PATH_FUSED_DECODE = 4
} gb_expert_path;
int gb_moe_set_expert_path(gb_moe* m, int32_t path);

/* Forward graphs.  A single-GPU gb_moe_forward (and gb_moe_forward_host) of
 * at most 512 tokens (except the batches that GB_PATH_FUSED_DECODE runs
 * as one launch) is captured once per (x, out, T) into a CUDA graph and
 * replayed on later calls with the same triple, which removes the host launch
 * cost of its kernels; the graph reads x and writes out at replay time, so
 * new contents of the same buffers are used.  Up to `max_graphs` (0..16,
 * default 16) graphs are kept, least recently used replaced; 0 launches
 * every kernel directly.  Changing the expert path, growing the workspace
 * or calling this clears the cache.  No counterpart in the reference, which
 * has one CPU path. */
int gb_moe_set_graphs(gb_moe* m, int32_t max_graphs);

/* Failure-handling test hooks (no counterpart in the reference; its CPU path
 * has no asynchronous waits).  wait_limit_us: how long each bounded wait of
 * the block-scaled expert kernel may last before it gives up (0 = the
 * default, 2 s).  withhold_ready != 0: the one-launch expert kernel (grouped
 * batches of 16-512 positions) leaves the first gate_up tile's ready flag
 * unset, so the down work that needs it waits until the limit; that forward's
 * output is invalid and gb_moe_device_status reports GB_ERR_TIMEOUT.  Both
 * apply to later forwards until reset with (0, 0); the next forward after a
 * reset is complete again.  Clears the forward graph cache. */
int gb_moe_set_test_hooks(gb_moe* m, int64_t wait_limit_us, int32_t withhold_ready);

/* Stage timing for profiling (no counterpart in the reference, whose timing
 * is per generated token, crates/gallium-agent/src/llm_candle.rs:302-345).
 * When enabled, each forward records a CUDA event at every stage boundary on
 * its stream.  gb_moe_stage_times synchronises on the last forward's final
 * event and writes up to `capacity` per-stage durations in milliseconds
 * (stage names from gb_moe_stage_name) and the stage count. */
int gb_moe_set_profiling(gb_moe* m, int enable);
int gb_moe_stage_times(gb_moe* m, float* ms_out, int32_t capacity, int32_t* n_stages);
const char* gb_moe_stage_name(int32_t stage);

/* Releases device memory, streams and (expert parallel) the communicator. */
int gb_moe_destroy(gb_moe* m);

/* Routing that allocates nothing.  No counterpart in the reference: it is
 * the router projection, top-k and combine weights of gb_moe_route (the
 * routing of gpt_oss.rs:172-182 / lfm2moe_q.rs:241-258), for callers that
 * cannot call cudaMalloc when they route -- a candle custom op whose device
 * buffers must all come from candle's allocator, or a serving process that
 * has reserved the device's memory up front.  The caller passes every input
 * and output as device pointers on the current device: x_dev [T, hidden] f32,
 * 16-byte aligned (GB_ERR_INVALID_ARG otherwise; hidden a multiple of 32, at
 * most 4096, as for gb_moe_create),
 * router_weight_dev [n_experts, hidden] f32, router_bias_dev [n_experts] f32
 * (NULL = none), selection_bias_dev [n_experts] f32 (sigmoid router only,
 * NULL = zeros), idx_dev [T, top_k] i32, w_dev [T, top_k] f32.  Results equal
 * gb_moe_route's idx / w for the same inputs.
 * Scratch (router logits and per-tile tickets) is a fixed 272 KiB array inside
 * the library, held on every GPU that loads the library until the process
 * exits; requests with T * n_experts > 65536 or T > 4096 are rejected with
 * GB_ERR_INVALID_ARG.  The first call on each device looks up that array's
 * device address (cudaGetSymbolAddress); make that first call before any
 * stream capture.  The address is kept for the life of the process: after a
 * cudaDeviceReset of a device, do not call this on that device again.
 * Every call shares the one array and each call overwrites
 * it: calls that overlap on the GPU (other streams, other threads) race, so
 * serialise them.  Asynchronous on `stream`; calls no cudaMalloc or cudaFree. */
int gb_route_noalloc(const float* x_dev, const float* router_weight_dev,
                     const float* router_bias_dev, const float* selection_bias_dev, int64_t T,
                     int32_t hidden, int32_t n_experts, int32_t top_k, int32_t router_kind,
                     int32_t* idx_dev, float* w_dev, void* stream);

/* ---- GPT-OSS decode stack ------------------------------------------------
 * The GGUF GPT-OSS model around the MoE block (crates/gallium-models/src/
 * gpt_oss_q.rs:15-107 attention, :270-297 block, :437-472 forward): per
 * layer, RMSNorm -> attention (q/k/v projections with biases, RoPE, grouped
 * queries, learned per-head sink logits, a sliding window on the layers
 * marked so) -> residual add -> RMSNorm -> the MoE block -> residual add;
 * then the final RMSNorm, the LM head on each sequence's last token and the
 * greedy token (the largest logit, ties to the highest token id, as
 * sampling.rs:85-92 takes Iterator::max_by's last maximum).  Activations,
 * the KV cache and all arithmetic are f32; attention and LM-head weights
 * are bf16 (widened exactly).  B sequences run in lockstep: every forward
 * gives each of them T tokens at the same positions pos .. pos + T - 1, as
 * the reference's (batch, seq_len) token tensor does. */

typedef struct gb_decoder gb_decoder;

typedef struct gb_decoder_layer {
  const float* attn_norm;        /* [hidden] RMSNorm weight before attention */
  const float* post_attn_norm;   /* [hidden] RMSNorm weight before the MoE block */
  const uint16_t* wq;            /* [n_heads * head_dim][hidden] bf16 bits */
  const uint16_t* wk;            /* [n_kv_heads * head_dim][hidden] */
  const uint16_t* wv;            /* [n_kv_heads * head_dim][hidden] */
  const uint16_t* wo;            /* [hidden][n_heads * head_dim] */
  const float* bq;               /* biases, each nullable: [n_heads * head_dim] */
  const float* bk;               /* [n_kv_heads * head_dim] */
  const float* bv;               /* [n_kv_heads * head_dim] */
  const float* bo;               /* [hidden] */
  const float* sinks;            /* [n_heads] sink logits */
  int32_t sliding;               /* 1: sliding-window attention, 0: full causal */
  const gb_moe_desc* moe;        /* the layer's MoE block (device, max_tokens and the
                                    expert-parallel fields are set by the decoder) */
} gb_decoder_layer;

typedef struct gb_decoder_desc {
  uint32_t struct_size;          /* sizeof(gb_decoder_desc) */
  int32_t n_layers;
  int32_t hidden;
  int32_t n_heads;               /* query heads, a multiple of n_kv_heads */
  int32_t n_kv_heads;
  int32_t head_dim;              /* even, <= 256 */
  int32_t vocab;
  int32_t sliding_window;        /* keys visible to a sliding layer, the query's own included */
  int32_t max_seq_len;           /* KV cache positions per sequence */
  int32_t max_batch;             /* sequences per forward */
  int32_t max_tokens;            /* tokens per sequence per forward */
  float rope_theta;
  float rope_scaling_factor;     /* > 1: YaRN frequencies (pos_enc.rs:113-137) */
  int32_t rope_orig_ctx;         /* YaRN original context length */
  float rope_beta_fast;          /* YaRN betas (0: 32 and 1) */
  float rope_beta_slow;
  float rms_eps;
  int32_t device;
  const uint16_t* embed;         /* [vocab][hidden] bf16 token embeddings */
  const uint16_t* lm_head;       /* [vocab][hidden] bf16, NULL: tied to embed */
  const float* final_norm;       /* [hidden] */
  const gb_decoder_layer* layers; /* [n_layers] */
} gb_decoder_desc;

/* Uploads every weight (the MoE blocks through gb_moe_create) and sizes the
 * KV cache for max_batch x max_seq_len positions.  Host pointers are read
 * during the call only. */
int gb_decoder_create(const gb_decoder_desc* desc, gb_decoder** out);

/* One forward of B sequences x T tokens at positions pos .. pos + T - 1
 * (tokens_dev: device int32 [B][T]).  pos must equal the positions already
 * cached (0 after create or reset) and B the batch of the cached positions;
 * pos + T <= max_seq_len.  logits_dev (nullable): device f32 [B][vocab], the
 * logits of each sequence's last token; next_dev (nullable): device int32
 * [B], its greedy token.  Asynchronous on `stream`. */
int gb_decoder_forward(gb_decoder* d, const int32_t* tokens_dev, int32_t B, int32_t T,
                       int64_t pos, float* logits_dev, int32_t* next_dev, void* stream);

/* n_steps greedy decode steps of B sequences, each feeding the previous
 * step's greedy token: step 0 feeds tokens_dev [B] at position pos.  Writes
 * the n_steps x B tokens produced to out_dev (device int32 [n_steps][B]).
 * Each step replays one CUDA graph (captured on the first call for each B).
 * Asynchronous on `stream`. */
int gb_decoder_generate(gb_decoder* d, const int32_t* tokens_dev, int32_t B, int64_t pos,
                        int32_t n_steps, int32_t* out_dev, void* stream);

/* Forget the cached positions (the next forward starts at pos 0). */
int gb_decoder_reset(gb_decoder* d);

/* Stage timing of the following forwards (CUDA events): when enabled,
 * gb_decoder_stage_times returns the milliseconds of the last eager forward
 * spent in attention (norms, projections, RoPE, attention, residual), in
 * the MoE blocks (norms, MoE, residual) and in the head (final norm, LM head,
 * greedy token).  Synchronises `stream`. */
int gb_decoder_set_profiling(gb_decoder* d, int32_t enable);
int gb_decoder_stage_times(gb_decoder* d, float ms_out[3], void* stream);

/* Device error words of every layer's MoE block (gb_moe_device_status). */
int gb_decoder_device_status(gb_decoder* d, void* stream);

int gb_decoder_destroy(gb_decoder* d);

/* Expert parallel: a fresh 128-byte ncclUniqueId (rank 0 calls this and
 * shares the bytes with the other ranks). */
int gb_nccl_unique_id(uint8_t out[128]);

/* Last error message of the calling thread ("" if none). */
const char* gb_last_error(void);

/* ABI version this library was built with (GB_ABI_VERSION). */
int gb_abi_version(void);

#ifdef __cplusplus
}
#endif
#endif /* GALLIUM_B200_H */
