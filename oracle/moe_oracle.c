/*
 * moe_oracle.c -- CPU restatement of rs-gallium's MoE FFN path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA path, never part of it.
 * Built with -ffp-contract=off so that every multiply and add rounds the way
 * the reference's Rust code (which never contracts) rounds them; the only
 * fused multiply-adds are the explicit fmaf() calls, which stand for the FMA
 * instructions of candle's SIMD gemm kernels.  See moe_oracle.h for the
 * pinned / unpinned status of each function.
 */
#include "moe_oracle.h"

#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static __thread char g_err[512];

static int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof g_err, fmt, ap);
  va_end(ap);
  return code;
}

const char* or_last_error(void) { return g_err; }

/* ---- quant decoders ---------------------------------------------------- */

/* gpt_oss.rs:21-24 */
static const float kMxfp4Table[16] = {0.0f,  0.5f,  1.0f,  1.5f,  2.0f,  3.0f,  4.0f,  6.0f,
                                      -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};

float or_e2m1_value(int code) { return kMxfp4Table[code & 15]; }

/* gpt_oss.rs:145-164: scale 2^(e-127) (2f32.powi), e == 0 -> 0.  For e >= 1 the
 * f32 with exponent field e and a zero mantissa is that power of two (e = 255
 * gives +inf, as 2f32.powi(128) overflows to). */
static float split_scale(uint8_t e) {
  const uint32_t bits = (uint32_t)e << 23;
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

int or_mxfp4_split_dequant(const uint8_t* blocks, const uint8_t* scales, int64_t rows, int64_t k,
                           float* out) {
  if (k % 32 != 0) return fail(2, "MXFP4 row length %lld is not a multiple of 32", (long long)k);
  const int64_t nb = k / 32;
  for (int64_t o = 0; o < rows; ++o) {
    for (int64_t b = 0; b < nb; ++b) {
      const float sc = split_scale(scales[o * nb + b]);
      const uint8_t* src = blocks + (o * nb + b) * 16;
      float* dst = out + o * k + b * 32;
      for (int j = 0; j < 16; ++j) {
        const uint8_t byte = src[j];
        dst[2 * j] = kMxfp4Table[byte & 0xF] * sc;
        dst[2 * j + 1] = kMxfp4Table[byte >> 4] * sc;
      }
    }
  }
  return 0;
}

/* quantized.rs:370: the GGUF LUT is the E2M1 table times two. */
static const int8_t kE2m1Lut2[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};

/* quantized.rs:375-383: bytes >= 2 build an f32 with exponent field b-1 and a
 * zero mantissa (2^(b-128)); bytes 0 and 1 give the subnormals 2^-128, 2^-127. */
float or_e8m0_to_f32(uint8_t b) {
  uint32_t bits = b < 2 ? (0x00200000u << b) : ((uint32_t)(b - 1) << 23);
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

/* quantized.rs:417-425 */
int or_mxfp4_blocks_per_expert(int64_t n_elems, int64_t* n_blocks) {
  if (n_elems % 32 != 0)
    return fail(2, "MXFP4 expert of %lld elements is not a whole number of 32-element blocks",
                (long long)n_elems);
  *n_blocks = n_elems / 32;
  return 0;
}

/* quantized.rs:393-449 (scalar path; the AVX2 path at :459-518 computes the
 * same products). */
int or_mxfp4_gguf_dequant(const uint8_t* raw, int64_t n_elems, float* out) {
  int64_t nb;
  int rc = or_mxfp4_blocks_per_expert(n_elems, &nb);
  if (rc) return rc;
  for (int64_t b = 0; b < nb; ++b) {
    const uint8_t* blk = raw + b * 17;
    const float sc = or_e8m0_to_f32(blk[0]);
    float* dst = out + b * 32;
    for (int j = 0; j < 16; ++j) {
      const uint8_t byte = blk[1 + j];
      dst[j] = (float)kE2m1Lut2[byte & 0xF] * sc;
      dst[j + 16] = (float)kE2m1Lut2[byte >> 4] * sc;
    }
  }
  return 0;
}

/* IEEE half -> float (exact). */
static float half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  const uint32_t exp = (h >> 10) & 0x1F;
  const uint32_t man = h & 0x3FF;
  float f;
  if (exp == 0) {
    f = ldexpf((float)man, -24);
    if (sign) f = -f;
    return f;
  }
  uint32_t bits;
  if (exp == 31)
    bits = sign | 0x7F800000u | (man << 13);
  else
    bits = sign | ((exp + 112) << 23) | (man << 13);
  memcpy(&f, &bits, 4);
  return f;
}

/* Q4_K super-block: f16 d, f16 dmin, 12 bytes of packed 6-bit sub-block
 * scales and mins, 128 bytes of 4-bit quants.  Sub-block j (32 elements) has
 * scale sc_j and min m_j; element value = d*sc_j*q - dmin*m_j.  The 6-bit
 * unpacking: for j < 4, sc = s[j] & 63, m = s[j+4] & 63; otherwise
 * sc = (s[j+4] & 15) | ((s[j-4] >> 6) << 4), m = (s[j+4] >> 4) | ((s[j] >> 6) << 4).
 * Quant bytes are consumed 32 at a time: the low nibbles give sub-block 2c,
 * the high nibbles sub-block 2c+1, for chunk c = 0..3. */
static void q4k_scale_min(int j, const uint8_t* s, uint8_t* sc, uint8_t* m) {
  if (j < 4) {
    *sc = s[j] & 63;
    *m = s[j + 4] & 63;
  } else {
    *sc = (uint8_t)((s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4));
    *m = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
  }
}

int or_q4k_dequant(const uint8_t* raw, int64_t n_elems, float* out) {
  if (n_elems % 256 != 0)
    return fail(2, "Q4_K tensor of %lld elements is not a whole number of 256-element blocks",
                (long long)n_elems);
  const int64_t nb = n_elems / 256;
  for (int64_t b = 0; b < nb; ++b) {
    const uint8_t* blk = raw + b * 144;
    const float d = half_to_float((uint16_t)(blk[0] | (blk[1] << 8)));
    const float dmin = half_to_float((uint16_t)(blk[2] | (blk[3] << 8)));
    const uint8_t* s = blk + 4;
    const uint8_t* q = blk + 16;
    float* y = out + b * 256;
    for (int c = 0; c < 4; ++c) {
      uint8_t sc, m;
      q4k_scale_min(2 * c, s, &sc, &m);
      const float d1 = d * (float)sc, m1 = dmin * (float)m;
      q4k_scale_min(2 * c + 1, s, &sc, &m);
      const float d2 = d * (float)sc, m2 = dmin * (float)m;
      for (int l = 0; l < 32; ++l) y[l] = d1 * (float)(q[l] & 0xF) - m1;
      for (int l = 0; l < 32; ++l) y[32 + l] = d2 * (float)(q[l] >> 4) - m2;
      y += 64;
      q += 32;
    }
  }
  return 0;
}

/* ---- routing ----------------------------------------------------------- */

int or_router_logits(const float* x, const float* w, const float* b, int64_t t, int64_t h,
                     int64_t e, float* logits) {
  if (h % 32 != 0) return fail(2, "hidden %lld is not a multiple of 32", (long long)h);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < t; ++i) {
    for (int64_t j = 0; j < e; ++j) {
      float part[32];
      for (int l = 0; l < 32; ++l) {
        float acc = 0.0f;
        for (int64_t kk = l; kk < h; kk += 32) acc = fmaf(x[i * h + kk], w[j * h + kk], acc);
        part[l] = acc;
      }
      for (int s = 16; s >= 1; s >>= 1) {
        float nxt[32];
        for (int l = 0; l < 32; ++l) nxt[l] = part[l] + part[l ^ s];
        memcpy(part, nxt, sizeof part);
      }
      logits[i * e + j] = b ? part[0] + b[j] : part[0];
    }
  }
  return 0;
}

typedef struct {
  int32_t idx;
  float key;
} keyed;

/* Stable descending insertion sort: equal keys keep ascending index order,
 * which is what Rust's stable sort_by with a reversed comparison gives. */
static void stable_sort_desc(keyed* v, int64_t n) {
  for (int64_t i = 1; i < n; ++i) {
    keyed cur = v[i];
    int64_t j = i - 1;
    while (j >= 0 && v[j].key < cur.key) {
      v[j + 1] = v[j];
      --j;
    }
    v[j + 1] = cur;
  }
}

/* exp(x) rounded once to f32.  The reference calls the platform's expf (Rust's
 * f32::exp); glibc's expf is not always the nearest f32 to exp(x) (on this
 * machine's glibc it differs from it by one unit in the last place on 170,648
 * of the 2,240,020,482 f32 arguments in [-104, 90]), so the oracle takes the
 * correctly rounded value, from the x87 extended-precision expl: the
 * platform-independent definition of the same arithmetic. */
static float exp_rn(float x) { return (float)expl((long double)x); }

float or_exp_rn(float x) { return exp_rn(x); }

/* gpt_oss.rs:174-182 with candle's softmax_last_dim (max, exp(v - max), sum,
 * divide), then the weight w / max(total, 1e-9) evaluated in f64 and rounded
 * to f32 by the tensor scale at gpt_oss.rs:223. */
int or_route_softmax_topk(const float* logits, int64_t t, int64_t e, int64_t k, int32_t* idx,
                          float* w) {
  if (k < 1 || k > e) return fail(1, "top_k %lld out of range for %lld experts", (long long)k,
                                  (long long)e);
  keyed* v = (keyed*)malloc(sizeof(keyed) * (size_t)e);
  float* p = (float*)malloc(sizeof(float) * (size_t)e);
  for (int64_t i = 0; i < t; ++i) {
    const float* l = logits + i * e;
    float mx = l[0];
    for (int64_t j = 1; j < e; ++j) mx = l[j] > mx ? l[j] : mx;
    float sum = 0.0f;
    for (int64_t j = 0; j < e; ++j) {
      p[j] = exp_rn(l[j] - mx);
      sum += p[j];
    }
    for (int64_t j = 0; j < e; ++j) {
      v[j].idx = (int32_t)j;
      v[j].key = p[j] / sum;
    }
    stable_sort_desc(v, e);
    float total = 0.0f;
    for (int64_t r = 0; r < k; ++r) total += v[r].key;
    if (total < 1e-9f) total = 1e-9f;
    for (int64_t r = 0; r < k; ++r) {
      idx[i * k + r] = v[r].idx;
      w[i * k + r] = (float)((double)v[r].key / (double)total);
    }
  }
  free(v);
  free(p);
  return 0;
}

/* lfm2moe_q.rs:241-258 (sigmoid = 1 / (1 + exp(-x)), candle_nn::ops::sigmoid). */
int or_route_sigmoid_topk(const float* logits, const float* sel_bias, int64_t t, int64_t e,
                          int64_t k, int32_t* idx, float* w) {
  if (k < 1 || k > e) return fail(1, "top_k %lld out of range for %lld experts", (long long)k,
                                  (long long)e);
  keyed* v = (keyed*)malloc(sizeof(keyed) * (size_t)e);
  float* p = (float*)malloc(sizeof(float) * (size_t)e);
  for (int64_t i = 0; i < t; ++i) {
    for (int64_t j = 0; j < e; ++j) {
      p[j] = 1.0f / (exp_rn(-logits[i * e + j]) + 1.0f);
      v[j].idx = (int32_t)j;
      v[j].key = p[j] + (sel_bias ? sel_bias[j] : 0.0f);
    }
    stable_sort_desc(v, e);
    float total = 0.0f;
    for (int64_t r = 0; r < k; ++r) total += p[v[r].idx];
    if (total < 1e-20f) total = 1e-20f;
    for (int64_t r = 0; r < k; ++r) {
      idx[i * k + r] = v[r].idx;
      w[i * k + r] = p[v[r].idx] / total;
    }
  }
  free(v);
  free(p);
  return 0;
}

/* gpt_oss_q.rs:175-192: expert_tokens[e] is pushed in token order. */
int or_permute(const int32_t* idx, int64_t t, int64_t e, int64_t k, int32_t* counts,
               int32_t* offsets, int32_t* perm, int32_t* inv) {
  memset(counts, 0, sizeof(int32_t) * (size_t)e);
  for (int64_t i = 0; i < t * k; ++i) {
    if (idx[i] < 0 || idx[i] >= e) return fail(1, "expert index %d out of range", idx[i]);
    counts[idx[i]]++;
  }
  offsets[0] = 0;
  for (int64_t j = 0; j < e; ++j) offsets[j + 1] = offsets[j] + counts[j];
  int32_t* fill = (int32_t*)malloc(sizeof(int32_t) * (size_t)e);
  memcpy(fill, offsets, sizeof(int32_t) * (size_t)e);
  for (int64_t i = 0; i < t; ++i)
    for (int64_t r = 0; r < k; ++r) {
      const int32_t ex = idx[i * k + r];
      const int32_t pos = fill[ex]++;
      perm[pos] = (int32_t)(i * k + r);
      if (inv) inv[i * k + r] = pos;
    }
  free(fill);
  return 0;
}

/* ---- expert FFN -------------------------------------------------------- */

/* f32 dot product in the shape of a SIMD gemm micro-kernel: 16 running sums
 * advanced with fused multiply-adds, folded pairwise at the end. */
__attribute__((target_clones("avx512f", "avx2", "default")))
static float dot_f32(const float* a, const float* b, int64_t n) {
  float acc[16] = {0};
  int64_t i = 0;
  for (; i + 16 <= n; i += 16)
    for (int j = 0; j < 16; ++j) acc[j] = fmaf(a[i + j], b[i + j], acc[j]);
  for (; i < n; ++i) acc[i & 15] = fmaf(a[i], b[i], acc[i & 15]);
  for (int s = 8; s >= 1; s >>= 1)
    for (int j = 0; j < s; ++j) acc[j] += acc[j + s];
  return acc[0];
}

/* gpt_oss.rs:202-212 (also gpt_oss_q.rs:224-239): gate clamped above at limit
 * (candle clamp = maximum(-1e38) then minimum(limit)), sigmoid(1.702 g) as
 * (tanh(0.851 g) + 1) * 0.5 through candle's affine ops, up clamped to
 * [-limit, limit] and shifted by one. */
static float act_gptoss(float g, float u, float limit) {
  g = fmaxf(g, -1e38f);
  g = fminf(g, limit);
  float s = tanhf(g * 0.851f + 0.0f);
  s = s * 1.0f + 1.0f;
  s = s * 0.5f + 0.0f;
  const float glu = g * s;
  u = fminf(fmaxf(u, -limit), limit);
  const float u1 = u * 1.0f + 1.0f;
  return glu * u1;
}

/* lfm2moe_q.rs:288-290: silu(g) * u with candle's silu v / (1 + exp(-v)). */
static float act_silu(float g, float u) { return (g / (1.0f + expf(-g))) * u; }

/* gallium-core's gated activations (ffn.rs:16-24, 56-66): act(gate), clamped
 * to [-clamp, clamp] when clamp > 0 (candle clamp: maximum, then minimum),
 * times up.  GELU (erf) with erf evaluated in f64 as candle's gelu_erf does;
 * GELU (tanh) as candle's gelu, 0.5 v (1 + tanh(sqrt(2/pi) v (1 + 0.044715 v^2))). */
static float act_gated(int kind, float g, float u, float clamp) {
  float a;
  switch (kind) {
    case OR_ACT_GELU:
      a = (float)(0.5 * (double)g * (1.0 + erf((double)g / sqrt(2.0))));
      break;
    case OR_ACT_GELU_TANH:
      a = 0.5f * g * (1.0f + tanhf(0.7978845608028654f * g * (1.0f + 0.044715f * g * g)));
      break;
    case OR_ACT_RELU:
      a = g > 0.0f ? g : 0.0f;
      break;
    default:
      a = g / (1.0f + expf(-g));
  }
  if (clamp > 0.0f) a = fminf(fmaxf(a, -clamp), clamp);
  return a * u;
}

static float act_apply(const or_moe_desc* d, float g, float u) {
  if (d->act_kind == OR_ACT_GPTOSS_CLAMP) return act_gptoss(g, u, d->swiglu_limit);
  if (d->act_kind == OR_ACT_SILU && !(d->act_clamp > 0.0f)) return act_silu(g, u);
  return act_gated(d->act_kind, g, u, d->act_clamp);
}

float or_act_gptoss(float g, float u, float limit) { return act_gptoss(g, u, limit); }
float or_act_silu(float g, float u) { return act_silu(g, u); }

/* Dequantise one row of a weight matrix into dst. */
typedef struct {
  const or_moe_desc* d;
  int which; /* 0 = gate (or fused gate_up), 1 = up, 2 = down */
} rowsrc;

static void dequant_row(const or_moe_desc* d, int which, int64_t ex, int64_t row, float* dst) {
  const int64_t H = d->hidden, I = d->inter;
  const int64_t rows = which == 2 ? H : (d->weight_format == OR_FMT_MXFP4_SPLIT ? 2 * I : I);
  const int64_t kdim = which == 2 ? I : H;
  if (d->weight_format == OR_FMT_DENSE) {
    const float* w = which == 0 ? d->dense_gate : which == 1 ? d->dense_up : d->dense_down;
    memcpy(dst, w + (ex * rows + row) * kdim, sizeof(float) * (size_t)kdim);
    return;
  }
  if (d->weight_format == OR_FMT_MXFP4_SPLIT) {
    const uint8_t* blocks = which == 2 ? d->dn_blocks : d->gu_blocks;
    const uint8_t* scales = which == 2 ? d->dn_scales : d->gu_scales;
    const int64_t nb = kdim / 32;
    or_mxfp4_split_dequant(blocks + ((ex * rows + row) * nb) * 16, scales + (ex * rows + row) * nb,
                           1, kdim, dst);
  } else {
    const uint8_t* raw = which == 0 ? d->gate_raw : which == 1 ? d->up_raw : d->down_raw;
    /* merged gate_up [E, 2I, H]: gate rows [0, I), up rows [I, 2I) (gemma4_q.rs:297-303) */
    int64_t r = ex * rows + row;
    if (which < 2 && d->gate_up_merged) {
      raw = d->gate_raw;
      r = ex * 2 * rows + (which == 1 ? rows : 0) + row;
    }
    if (d->weight_format == OR_FMT_MXFP4_GGUF) {
      const int64_t rb = kdim / 32 * 17;
      or_mxfp4_gguf_dequant(raw + r * rb, kdim, dst);
    } else {
      const int64_t rb = kdim / 256 * 144;
      or_q4k_dequant(raw + r * rb, kdim, dst);
    }
  }
}

/* Expert FFN for n tokens (rows of xs, [n, H]) through expert ex -> ys [n, H].
 * Dequantises row by row; the dequantised values and every dot product are
 * the same as dequantising the whole matrix first. */
static void expert_ffn(const or_moe_desc* d, int64_t ex, const float* xs, int64_t n, float* ys,
                       float* hbuf, float* rowbuf) {
  const int64_t H = d->hidden, I = d->inter;
  float* r0 = rowbuf;
  float* r1 = rowbuf + (H > I ? H : I);
  for (int64_t i = 0; i < I; ++i) {
    float bg = 0.0f, bu = 0.0f;
    if (d->weight_format == OR_FMT_MXFP4_SPLIT) {
      dequant_row(d, 0, ex, 2 * i, r0);
      dequant_row(d, 0, ex, 2 * i + 1, r1);
      if (d->gu_bias) {
        bg = d->gu_bias[ex * 2 * I + 2 * i];
        bu = d->gu_bias[ex * 2 * I + 2 * i + 1];
      }
    } else {
      dequant_row(d, 0, ex, i, r0);
      dequant_row(d, 1, ex, i, r1);
      if (d->gate_bias) bg = d->gate_bias[ex * I + i];
      if (d->up_bias) bu = d->up_bias[ex * I + i];
    }
    const int has_gb = d->weight_format == OR_FMT_MXFP4_SPLIT ? d->gu_bias != NULL
                                                               : d->gate_bias != NULL;
    const int has_ub = d->weight_format == OR_FMT_MXFP4_SPLIT ? d->gu_bias != NULL
                                                               : d->up_bias != NULL;
    for (int64_t t = 0; t < n; ++t) {
      float g = dot_f32(xs + t * H, r0, H);
      float u = dot_f32(xs + t * H, r1, H);
      if (has_gb) g = g + bg;
      if (has_ub) u = u + bu;
      hbuf[t * I + i] = act_apply(d, g, u);
    }
  }
  for (int64_t o = 0; o < H; ++o) {
    dequant_row(d, 2, ex, o, r0);
    const float bd = d->dn_bias ? d->dn_bias[ex * H + o] : 0.0f;
    for (int64_t t = 0; t < n; ++t) {
      float y = dot_f32(hbuf + t * I, r0, I);
      if (d->dn_bias) y = y + bd;
      ys[t * H + o] = y;
    }
  }
}

static int check_desc(const or_moe_desc* d) {
  if (!d) return fail(1, "null descriptor");
  if (d->hidden <= 0 || d->inter <= 0 || d->n_experts <= 0 || d->top_k <= 0 ||
      d->top_k > d->n_experts)
    return fail(1, "bad shape H=%lld I=%lld E=%lld k=%lld", (long long)d->hidden,
                (long long)d->inter, (long long)d->n_experts, (long long)d->top_k);
  const int64_t blk = d->weight_format == OR_FMT_Q4_K ? 256 : 32;
  if (d->weight_format == OR_FMT_DENSE && (!d->dense_gate || !d->dense_up || !d->dense_down))
    return fail(1, "dense weights missing");
  if (d->shared_inter > 0 && (!d->sh_gate || !d->sh_up || !d->sh_down))
    return fail(1, "shared expert weights missing");
  if (d->hidden % blk || d->inter % blk)
    return fail(2, "H=%lld / I=%lld not multiples of the %lld-element block",
                (long long)d->hidden, (long long)d->inter, (long long)blk);
  if (!d->router_w) return fail(1, "router weight missing");
  return 0;
}

/* v / sqrt(mean(v^2) + eps), candle_nn::ops::rms_norm's arithmetic (the sum
 * of squares in order). */
static float rms_of(const float* v, int64_t n, float eps) {
  float ss = 0.0f;
  for (int64_t k = 0; k < n; ++k) ss += v[k] * v[k];
  return sqrtf(ss / (float)n + eps);
}

/* The block from router logits to the combined output: the router reads
 * x_route, the experts x. */
static int moe_forward_core(const or_moe_desc* d, const float* x_route, const float* x, int64_t t,
                            float* out, int32_t* idx_out, float* w_out, int n_threads) {
  int rc = check_desc(d);
  if (rc) return rc;
  const int64_t H = d->hidden, I = d->inter, E = d->n_experts, K = d->top_k;
  if (t == 0) return 0;
  float* logits = (float*)malloc(sizeof(float) * (size_t)(t * E));
  int32_t* idx = (int32_t*)malloc(sizeof(int32_t) * (size_t)(t * K));
  float* w = (float*)malloc(sizeof(float) * (size_t)(t * K));
  int32_t* counts = (int32_t*)malloc(sizeof(int32_t) * (size_t)E);
  int32_t* offsets = (int32_t*)malloc(sizeof(int32_t) * (size_t)(E + 1));
  int32_t* perm = (int32_t*)malloc(sizeof(int32_t) * (size_t)(t * K));
  int32_t* inv = (int32_t*)malloc(sizeof(int32_t) * (size_t)(t * K));
  float* y = (float*)malloc(sizeof(float) * (size_t)(t * K * H));
  if (!logits || !idx || !w || !counts || !offsets || !perm || !inv || !y) {
    rc = fail(7, "out of host memory");
    goto done;
  }
  rc = or_router_logits(x_route, d->router_w, d->router_b, t, H, E, logits);
  if (rc) goto done;
  rc = d->router_kind == OR_ROUTER_SOFTMAX_TOPK
           ? or_route_softmax_topk(logits, t, E, K, idx, w)
           : or_route_sigmoid_topk(logits, d->sel_bias, t, E, K, idx, w);
  if (rc) goto done;
  rc = or_permute(idx, t, E, K, counts, offsets, perm, inv);
  if (rc) goto done;

#ifdef _OPENMP
  if (n_threads <= 0) n_threads = omp_get_max_threads();
#else
  n_threads = 1;
#endif
  /* par_map_on_cpu over the active experts (device.rs:91-108). */
#pragma omp parallel num_threads(n_threads)
  {
    const int64_t cap = (H > I ? H : I);
    float* rowbuf = (float*)malloc(sizeof(float) * (size_t)(2 * cap));
    float* xs = NULL;
    float* hbuf = NULL;
    float* ys = NULL;
    int64_t have = 0;
#pragma omp for schedule(dynamic, 1)
    for (int64_t ex = 0; ex < E; ++ex) {
      const int64_t n = counts[ex];
      if (n == 0) continue;
      if (n > have) {
        free(xs);
        free(hbuf);
        free(ys);
        xs = (float*)malloc(sizeof(float) * (size_t)(n * H));
        hbuf = (float*)malloc(sizeof(float) * (size_t)(n * I));
        ys = (float*)malloc(sizeof(float) * (size_t)(n * H));
        have = n;
      }
      for (int64_t j = 0; j < n; ++j) {
        const int64_t tok = perm[offsets[ex] + j] / K;
        memcpy(xs + j * H, x + tok * H, sizeof(float) * (size_t)H);
      }
      expert_ffn(d, ex, xs, n, ys, hbuf, rowbuf);
      memcpy(y + (int64_t)offsets[ex] * H, ys, sizeof(float) * (size_t)(n * H));
    }
    free(rowbuf);
    free(xs);
    free(hbuf);
    free(ys);
  }

  /* Combine.  Safetensors GPT-OSS (gpt_oss.rs:223): ranks in order, each
   * row scaled then added to a running sum from zero.  GGUF GPT-OSS
   * (gpt_oss_q.rs:252-266) and LFM2 (lfm2moe_q.rs:303-311): rows added in
   * ascending expert order. */
  for (int64_t i = 0; i < t; ++i) {
    int order[64];
    for (int r = 0; r < K; ++r) order[r] = r;
    if (d->weight_format == OR_FMT_MXFP4_GGUF || d->weight_format == OR_FMT_Q4_K) {
      for (int a = 1; a < K; ++a) {
        int cur = order[a], b = a - 1;
        while (b >= 0 && idx[i * K + order[b]] > idx[i * K + cur]) {
          order[b + 1] = order[b];
          --b;
        }
        order[b + 1] = cur;
      }
    }
    for (int64_t o = 0; o < H; ++o) {
      float acc = 0.0f;
      for (int q = 0; q < K; ++q) {
        const int r = order[q];
        float yv = y[(int64_t)inv[i * K + r] * H + o];
        /* an expert's output scale comes before the routing weight (gemma4_q.rs:308-314) */
        if (d->expert_scale) yv = yv * d->expert_scale[idx[i * K + r]];
        const float term = yv * w[i * K + r];
        acc = acc + term;
      }
      out[i * H + o] = acc;
    }
  }
  /* The shared expert over all tokens, added after the routed sum
   * (ffn.rs:160-163): a GatedFFN with the experts' activation. */
  if (d->shared_inter > 0) {
    or_moe_desc sd = *d;
    sd.weight_format = OR_FMT_DENSE;
    sd.inter = d->shared_inter;
    sd.n_experts = 1;
    sd.dense_gate = d->sh_gate;
    sd.dense_up = d->sh_up;
    sd.dense_down = d->sh_down;
    sd.gu_bias = sd.gate_bias = sd.up_bias = sd.dn_bias = NULL;
    float* sy = (float*)malloc(sizeof(float) * (size_t)(t * H));
    if (!sy) {
      rc = fail(7, "out of host memory");
      goto done;
    }
#pragma omp parallel num_threads(n_threads)
    {
      const int64_t Is = sd.inter, cap = (H > Is ? H : Is);
      float* rowbuf = (float*)malloc(sizeof(float) * (size_t)(2 * cap));
      float* hbuf = (float*)malloc(sizeof(float) * (size_t)Is);
#pragma omp for schedule(dynamic, 1)
      for (int64_t i = 0; i < t; ++i) expert_ffn(&sd, 0, x + i * H, 1, sy + i * H, hbuf, rowbuf);
      free(rowbuf);
      free(hbuf);
    }
    for (int64_t i = 0; i < t * H; ++i) out[i] = out[i] + sy[i];
    free(sy);
  }
  if (idx_out) memcpy(idx_out, idx, sizeof(int32_t) * (size_t)(t * K));
  if (w_out) memcpy(w_out, w, sizeof(float) * (size_t)(t * K));
done:
  free(logits);
  free(idx);
  free(w);
  free(counts);
  free(offsets);
  free(perm);
  free(inv);
  free(y);
  return rc;
}

int or_moe_forward(const or_moe_desc* d, const float* x, int64_t t, float* out, int32_t* idx_out,
                   float* w_out, int n_threads) {
  int rc = check_desc(d);
  if (rc) return rc;
  if (d->input_norm != 1) {
    rc = moe_forward_core(d, x, x, t, out, idx_out, w_out, n_threads);
  } else {
    /* Gemma-4: the router reads rms(x) * H^-0.5 * scale, the experts
     * rms(x) * norm weight (gemma4_q.rs:267-276) */
    const int64_t H = d->hidden;
    float* xr = (float*)malloc(sizeof(float) * (size_t)(t * H) + 4);
    float* xe = (float*)malloc(sizeof(float) * (size_t)(t * H) + 4);
    if (!xr || !xe) {
      free(xr);
      free(xe);
      return fail(7, "out of host memory");
    }
    const float inv_sqrt_h = (float)(1.0 / sqrt((double)H));
    for (int64_t i = 0; i < t; ++i) {
      const float m = rms_of(x + i * H, H, d->rms_eps);
      for (int64_t k = 0; k < H; ++k) {
        const float nv = x[i * H + k] / m;
        xr[i * H + k] = nv * inv_sqrt_h * d->router_input_scale[k];
        xe[i * H + k] = nv * d->expert_input_norm[k];
      }
    }
    rc = moe_forward_core(d, xr, xe, t, out, idx_out, w_out, n_threads);
    free(xr);
    free(xe);
  }
  if (!rc && d->output_norm) { /* post_ffw_norm_2 (gemma4_q.rs:327) */
    const int64_t H = d->hidden;
    for (int64_t i = 0; i < t; ++i) {
      const float m = rms_of(out + i * H, H, d->rms_eps);
      for (int64_t k = 0; k < H; ++k) out[i * H + k] = out[i * H + k] / m * d->output_norm[k];
    }
  }
  return rc;
}

int or_dequant_expert_matrix(const or_moe_desc* d, int which, int64_t expert, float* out,
                             int n_threads) {
  int rc = check_desc(d);
  if (rc) return rc;
  if (expert < 0 || expert >= d->n_experts) return fail(1, "expert %lld out of range", (long long)expert);
  if (which < 0 || which > 2 || (which == 1 && d->weight_format == OR_FMT_MXFP4_SPLIT))
    return fail(1, "which = %d not valid for this format", which);
  const int64_t H = d->hidden, I = d->inter;
  const int64_t rows = which == 2 ? H : (d->weight_format == OR_FMT_MXFP4_SPLIT ? 2 * I : I);
  const int64_t kdim = which == 2 ? I : H;
#ifdef _OPENMP
  if (n_threads <= 0) n_threads = omp_get_max_threads();
#else
  (void)n_threads;
#endif
#pragma omp parallel for schedule(static) num_threads(n_threads)
  for (int64_t o = 0; o < rows; ++o) dequant_row(d, which, expert, o, out + o * kdim);
  return 0;
}

void or_act_rows(const or_moe_desc* d, const float* gate, const float* up, int64_t n,
                 int64_t stride, float* h, int n_threads) {
  const int64_t I = d->inter;
#ifdef _OPENMP
  if (n_threads <= 0) n_threads = omp_get_max_threads();
#else
  (void)n_threads;
#endif
#pragma omp parallel for schedule(static) num_threads(n_threads)
  for (int64_t t = 0; t < n; ++t)
    for (int64_t i = 0; i < I; ++i) {
      const float g = gate[t * stride + i * (stride == 2 * I ? 2 : 1)];
      const float u = up[t * stride + i * (stride == 2 * I ? 2 : 1)];
      h[t * I + i] = act_apply(d, g, u);
    }
}

int or_expert_ffn(const or_moe_desc* d, int64_t expert, const float* xs, int64_t n, float* ys) {
  int rc = check_desc(d);
  if (rc) return rc;
  if (expert < 0 || expert >= d->n_experts) return fail(1, "expert %lld out of range", (long long)expert);
  const int64_t H = d->hidden, I = d->inter;
  const int64_t cap = (H > I ? H : I);
  float* rowbuf = (float*)malloc(sizeof(float) * (size_t)(2 * cap));
  float* hbuf = (float*)malloc(sizeof(float) * (size_t)((n > 0 ? n : 1) * I));
  if (!rowbuf || !hbuf) {
    free(rowbuf);
    free(hbuf);
    return fail(7, "out of host memory");
  }
  if (n > 0) expert_ffn(d, expert, xs, n, ys, hbuf, rowbuf);
  free(rowbuf);
  free(hbuf);
  return 0;
}

int64_t or_moe_expert_sample(const or_moe_desc* d, const float* x, const int32_t* experts,
                             const int32_t* ntok, int64_t n_items, float* y_scratch,
                             int n_threads) {
  if (check_desc(d)) return -1;
  const int64_t H = d->hidden, I = d->inter;
  int64_t rows = 0;
  for (int64_t i = 0; i < n_items; ++i) rows += ntok[i];
  (void)y_scratch;
#ifdef _OPENMP
  if (n_threads <= 0) n_threads = omp_get_max_threads();
#else
  n_threads = 1;
#endif
#pragma omp parallel num_threads(n_threads)
  {
    const int64_t cap = (H > I ? H : I);
    float* rowbuf = (float*)malloc(sizeof(float) * (size_t)(2 * cap));
#pragma omp for schedule(dynamic, 1)
    for (int64_t i = 0; i < n_items; ++i) {
      const int64_t n = ntok[i];
      float* hbuf = (float*)malloc(sizeof(float) * (size_t)(n * I));
      float* ys = (float*)malloc(sizeof(float) * (size_t)(n * H));
      expert_ffn(d, experts[i], x, n, ys, hbuf, rowbuf);
      free(hbuf);
      free(ys);
    }
    free(rowbuf);
  }
  return rows;
}
