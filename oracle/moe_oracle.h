/*
 * moe_oracle.h -- CPU restatement of rs-gallium's mixture-of-experts FFN path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA path in
 * rs-gallium_b200/csrc: only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / reference arm load it.  The product never links or calls it.
 *
 * Parity status: the MXFP4 GGUF decoder is pinned by the reference's own unit
 * tests (crates/gallium-core/src/quantized.rs:917-1010, ported in
 * tests/test_oracle_goldens.py).  Everything else (safetensors nibble order,
 * router/top-k, clamped SwiGLU, GEMMs, combine, Q4_K) has no golden vector in
 * the reference; those functions restate the reference code line by line (file
 * and line cited at each function) and are cross-checked in tests against an
 * independent numpy restatement -- "parity unpinned" for those parts.
 *
 * Arithmetic that lives in the third-party dependency candle 0.10.2
 * (git rev 097655a2, Cargo.lock:159-212) -- f32 matmul, softmax_last_dim,
 * tanh/clamp, sigmoid/silu and the Q4_K dequantiser -- is restated from its
 * published algorithm (the GGML k-quant block format for Q4_K).
 *
 * All pointers are host pointers.  Functions return 0 on success and a
 * non-zero code with a message in or_last_error() on failure.
 */
#ifndef GALLIUM_MOE_ORACLE_H
#define GALLIUM_MOE_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- quant decoders ---------------------------------------------------- */

/* E2M1 code -> value, MXFP4_TABLE at crates/gallium-models/src/gpt_oss.rs:21-24. */
float or_e2m1_value(int code);

/* Safetensors MXFP4 (gpt_oss.rs:145-164): blocks [rows, k/32, 16] u8,
 * scales [rows, k/32] u8 -> out [rows, k] f32.  Byte j of a block holds
 * element 2j in its low nibble and 2j+1 in its high nibble; scale byte e gives
 * 2^(e-127), and e == 0 gives 0. */
int or_mxfp4_split_dequant(const uint8_t* blocks, const uint8_t* scales,
                           int64_t rows, int64_t k, float* out);

/* GGUF type-39 MXFP4 (quantized.rs:361-449). */
float or_e8m0_to_f32(uint8_t b);                       /* quantized.rs:375-383 */
int or_mxfp4_blocks_per_expert(int64_t n_elems, int64_t* n_blocks); /* :417-425 */
int or_mxfp4_gguf_dequant(const uint8_t* raw, int64_t n_elems, float* out); /* :393-449 */

/* GGML Q4_K (256-element super-blocks, 144 bytes each), restating the public
 * block layout that candle's k_quants dequantiser implements. */
int or_q4k_dequant(const uint8_t* raw, int64_t n_elems, float* out);

/* ---- routing ----------------------------------------------------------- */

/* Router logits[t,e] = dot(x[t,:], w[e,:]) + b[e].  The reference leaves the
 * summation order to candle's gemm; this restatement fixes one: 32 partial
 * sums, partial l accumulating k = l, l+32, l+64, ... with fused
 * multiply-adds, then a butterfly over the 32 partials (xor 16, 8, 4, 2, 1),
 * then the bias add.  The CUDA router reduces in exactly this order, which is
 * what makes expert indices comparable bit for bit.  h % 32 == 0.
 * w is f32 [e, h]; b may be NULL. */
int or_router_logits(const float* x, const float* w, const float* b,
                     int64_t t, int64_t h, int64_t e, float* logits);

/* GPT-OSS routing, gpt_oss.rs:174-182: softmax over all experts, stable
 * descending sort by probability (ties: lower index first), keep k, weight =
 * p / max(sum p, 1e-9) computed in f64 and rounded to f32 (gpt_oss.rs:223).
 * idx, w are [t, k]; rank r = position in the sorted order. */
int or_route_softmax_topk(const float* logits, int64_t t, int64_t e, int64_t k,
                          int32_t* idx, float* w);

/* LFM2.5 routing, lfm2moe_q.rs:241-258: p = sigmoid(logit); select by
 * p + sel_bias (stable descending); weight = p / max(sum_topk p, 1e-20). */
int or_route_sigmoid_topk(const float* logits, const float* sel_bias, int64_t t,
                          int64_t e, int64_t k, int32_t* idx, float* w);

/* Grouping, gpt_oss_q.rs:175-192: expert lists filled in token order.
 * counts[e], offsets[e+1] (exclusive prefix, offsets[e] = start of expert e),
 * perm[pos] = t*k + r for the entry at sorted position pos (expert ascending,
 * token ascending), inv[t*k + r] = pos. */
int or_permute(const int32_t* idx, int64_t t, int64_t e, int64_t k,
               int32_t* counts, int32_t* offsets, int32_t* perm, int32_t* inv);

/* ---- expert FFN and the whole block ------------------------------------ */

enum { OR_ROUTER_SOFTMAX_TOPK = 0, OR_ROUTER_SIGMOID_TOPK = 1 };
/* Activations: GPT-OSS clamped SwiGLU, or a gated act(gate) * up with act one
 * of gallium-core's Activation (ffn.rs:4-24), act(gate) clamped to
 * [-act_clamp, act_clamp] when act_clamp > 0 (ffn.rs:56-66). */
enum { OR_ACT_GPTOSS_CLAMP = 0, OR_ACT_SILU = 1, OR_ACT_GELU = 2, OR_ACT_GELU_TANH = 3,
       OR_ACT_RELU = 4 };
/* OR_FMT_DENSE: gallium-core MoEFFN (ffn.rs:72-166), dense f32 experts. */
enum { OR_FMT_MXFP4_SPLIT = 0, OR_FMT_MXFP4_GGUF = 1, OR_FMT_Q4_K = 2, OR_FMT_DENSE = 3 };

typedef struct {
  int64_t hidden, inter, n_experts, top_k;
  int32_t router_kind, act_kind, weight_format;
  float swiglu_limit;             /* GPT-OSS clamp (7.0) */
  const float* router_w;          /* [E, H] f32 (bf16 values widened exactly) */
  const float* router_b;          /* [E] or NULL */
  const float* sel_bias;          /* [E] or NULL (sigmoid router selection bias) */
  /* MXFP4_SPLIT: fused, interleaved gate_up (row 2i = gate_i, 2i+1 = up_i) */
  const uint8_t* gu_blocks;       /* [E, 2I, H/32, 16] */
  const uint8_t* gu_scales;       /* [E, 2I, H/32] */
  const uint8_t* dn_blocks;       /* [E, H, I/32, 16] */
  const uint8_t* dn_scales;       /* [E, H, I/32] */
  /* MXFP4_GGUF / Q4_K: separate gate, up [E, I, H] and down [E, H, I] raw
   * block bytes (17-byte MXFP4 blocks or 144-byte Q4_K super-blocks). */
  const uint8_t* gate_raw;
  const uint8_t* up_raw;
  const uint8_t* down_raw;
  /* biases (f32, NULL = none): gate_up [E, 2I] interleaved for SPLIT;
   * gate [E, I], up [E, I] for GGUF; down [E, H]. */
  const float* gu_bias;
  const float* gate_bias;
  const float* up_bias;
  const float* dn_bias;
  /* DENSE: gate, up [E, I, H], down [E, H, I] f32; the shared expert
   * (shared_inter > 0) sh_gate, sh_up [Is, H], sh_down [H, Is] f32. */
  const float* dense_gate;
  const float* dense_up;
  const float* dense_down;
  int64_t shared_inter;
  const float* sh_gate;
  const float* sh_up;
  const float* sh_down;
  float act_clamp;
  /* Gemma-4 routed experts (gemma4_q.rs:187-330): merged gate_up (gate_raw
   * [E, 2I, H], gate rows first); per-expert output scale [E]; input_norm 1:
   * router on rms(x) * H^-0.5 * router_input_scale, experts on rms_norm(x) *
   * expert_input_norm; output_norm [H] on the result. */
  int32_t gate_up_merged;
  const float* expert_scale;
  int32_t input_norm;
  const float* router_input_scale;
  const float* expert_input_norm;
  const float* output_norm;
  float rms_eps;
} or_moe_desc;

/* Full block forward.  x [t, H] f32 -> out [t, H] f32.  Per active expert the
 * weights are dequantised once and applied to every token routed to it
 * (gpt_oss_q.rs:194-246, lfm2moe_q.rs:268-297); experts run in parallel over
 * n_threads OpenMP threads like par_map_on_cpu (device.rs:91-108).  Each token's
 * output sums its k weighted expert rows in rank order starting from zero
 * (gpt_oss.rs:223).  idx/w (may be NULL) receive the routing. */
int or_moe_forward(const or_moe_desc* d, const float* x, int64_t t, float* out,
                   int32_t* idx, float* w, int n_threads);

/* One expert's FFN (the per-expert closure of gpt_oss_q.rs:194-246) on n
 * rows xs [n, H] -> ys [n, H]. */
int or_expert_ffn(const or_moe_desc* d, int64_t expert, const float* xs, int64_t n, float* ys);

/* Bounded CPU baseline: run the expert FFN of or_moe_forward for the given
 * (expert, token-count) work list only (routing excluded), returning the
 * number of token-expert rows processed.  Used to time a sample. */
int64_t or_moe_expert_sample(const or_moe_desc* d, const float* x,
                             const int32_t* experts, const int32_t* ntok,
                             int64_t n_items, float* y_scratch, int n_threads);

/* One expert's weight matrix dequantised to f32 row-major [rows, K] with
 * n_threads OpenMP threads: which 0 = gate_up [2I, H] (interleaved rows,
 * MXFP4_SPLIT) or gate [I, H] (GGUF / Q4_K), 1 = up [I, H] (GGUF / Q4_K),
 * 2 = down [H, I].  The dequantise-once step of gpt_oss_q.rs:203-209. */
int or_dequant_expert_matrix(const or_moe_desc* d, int which, int64_t expert, float* out,
                             int n_threads);

/* The expert activation over n rows: h[t, i] = act(gate[t*stride + i*s],
 * up[t*stride + i*s]) with s = 2 when stride == 2I (the interleaved gate_up
 * product of MXFP4_SPLIT, gate and up pointing at its columns 0 and 1), else
 * s = 1 (separate gate and up products, stride I).  h is [n, I].  act is the
 * descriptor's activation as the experts apply it (clamped SwiGLU, SiLU, or
 * gallium-core's gated kinds with their clamp). */
void or_act_rows(const or_moe_desc* d, const float* gate, const float* up, int64_t n,
                 int64_t stride, float* h, int n_threads);

/* exp(x) correctly rounded to f32 (the router's exp), for known-answer and
 * cross-checks. */
float or_exp_rn(float x);

/* The two expert activations, exposed for known-answer tests. */
float or_act_gptoss(float gate, float up, float limit);
float or_act_silu(float gate, float up);

const char* or_last_error(void);

#ifdef __cplusplus
}
#endif
#endif
