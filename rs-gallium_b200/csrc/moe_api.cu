// moe_api.cu -- the C ABI (include/gallium_b200.h): handle lifetime, weight
// upload and repack, workspace, and the forward pipeline
//   router + top-k -> grouping -> expert products -> combine.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <new>
#include <string>
#include <tuple>
#include <vector>

#include "moe_internal.h"

namespace {

thread_local char g_err[1024] = "";

int set_err(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof g_err, fmt, ap);
  va_end(ap);
  return code;
}

int cuda_err(cudaError_t e, const char* what) {
  return set_err(GB_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

#define GB_CUDA(call, what)                    \
  do {                                         \
    cudaError_t _e = (call);                   \
    if (_e != cudaSuccess) return cuda_err(_e, what); \
  } while (0)

// Makes `dev` current for the scope and restores the caller's device.
struct DeviceScope {
  int prev = -1;
  bool ok = false;
  explicit DeviceScope(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    ok = cudaSetDevice(dev) == cudaSuccess;
  }
  ~DeviceScope() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

float bf16_to_f32(uint16_t b) {
  uint32_t bits = (uint32_t)b << 16;
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

// Widen a [n] vector of f32 or bf16 host values to f32.
std::vector<float> widen(const void* src, int64_t n, int dtype) {
  std::vector<float> out((size_t)n);
  if (dtype == GB_DTYPE_BF16) {
    const uint16_t* s = static_cast<const uint16_t*>(src);
    for (int64_t i = 0; i < n; ++i) out[(size_t)i] = bf16_to_f32(s[i]);
  } else {
    memcpy(out.data(), src, sizeof(float) * (size_t)n);
  }
  return out;
}

int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

int validate(const gb_moe_desc* d) {
  if (!d) return set_err(GB_ERR_INVALID_ARG, "descriptor is null");
  if (d->struct_size < sizeof(gb_moe_desc))
    return set_err(GB_ERR_INVALID_ARG, "descriptor struct_size %u < %zu (header mismatch)",
                   d->struct_size, sizeof(gb_moe_desc));
  if (d->hidden <= 0 || d->inter <= 0 || d->n_experts <= 0 || d->top_k <= 0)
    return set_err(GB_ERR_INVALID_ARG, "non-positive shape H=%d I=%d E=%d k=%d", d->hidden,
                   d->inter, d->n_experts, d->top_k);
  if (d->n_experts > 256)
    return set_err(GB_ERR_UNSUPPORTED, "n_experts %d > 256", d->n_experts);
  if (d->top_k > d->n_experts || d->top_k > 8)
    return set_err(GB_ERR_INVALID_ARG, "top_k %d must be <= n_experts (%d) and <= 8", d->top_k,
                   d->n_experts);
  if (d->router_kind != GB_ROUTER_SOFTMAX_TOPK && d->router_kind != GB_ROUTER_SIGMOID_TOPK)
    return set_err(GB_ERR_INVALID_ARG, "unknown router_kind %d", d->router_kind);
  if (d->act_kind < GB_ACT_GPTOSS_CLAMP || d->act_kind > GB_ACT_RELU)
    return set_err(GB_ERR_INVALID_ARG, "unknown act_kind %d", d->act_kind);
  if (d->act_kind > GB_ACT_SILU && d->weight_format == GB_FMT_MXFP4_SPLIT)
    return set_err(GB_ERR_UNSUPPORTED, "act_kind %d does not apply to MXFP4_SPLIT experts",
                   d->act_kind);
  if (!(d->act_clamp >= 0.0f) || (d->act_clamp > 0.0f && d->act_kind == GB_ACT_GPTOSS_CLAMP))
    return set_err(GB_ERR_INVALID_ARG,
                   "act_clamp must be >= 0 (and 0 for the GPT-OSS activation, which uses "
                   "swiglu_limit)");
  if (d->gate_up_merged && d->weight_format != GB_FMT_MXFP4_GGUF && d->weight_format != GB_FMT_Q4_K)
    return set_err(GB_ERR_INVALID_ARG, "gate_up_merged applies to GGUF MXFP4 and Q4_K experts");
  if (d->input_norm != 0 && d->input_norm != 1)
    return set_err(GB_ERR_INVALID_ARG, "unknown input_norm %d", d->input_norm);
  if (d->input_norm == 1 && (!d->router_input_scale || !d->expert_input_norm))
    return set_err(GB_ERR_INVALID_ARG,
                   "input_norm 1 needs router_input_scale and expert_input_norm");
  if ((d->input_norm || d->output_norm) && !(d->rms_eps >= 0.0f))
    return set_err(GB_ERR_INVALID_ARG, "rms_eps must be >= 0");
  if (d->shared_inter < 0 || (d->shared_inter > 0 && d->weight_format != GB_FMT_DENSE))
    return set_err(GB_ERR_UNSUPPORTED, "a shared expert needs GB_FMT_DENSE experts");
  if (d->shared_inter > 0 &&
      (d->shared_inter % 32 != 0 || d->shared_inter > 4096 || !d->shared_gate ||
       !d->shared_up || !d->shared_down))
    return set_err(GB_ERR_INVALID_ARG,
                   "shared expert: shared_inter %d must be a multiple of 32, <= 4096, with "
                   "shared_gate, shared_up and shared_down",
                   d->shared_inter);
  if (d->router_dtype != GB_DTYPE_F32 && d->router_dtype != GB_DTYPE_BF16)
    return set_err(GB_ERR_INVALID_ARG, "unknown router_dtype %d", d->router_dtype);
  if (d->bias_dtype != GB_DTYPE_F32 && d->bias_dtype != GB_DTYPE_BF16)
    return set_err(GB_ERR_INVALID_ARG, "unknown bias_dtype %d", d->bias_dtype);
  if (!d->router_weight) return set_err(GB_ERR_INVALID_ARG, "router_weight is null");
  switch (d->weight_format) {
    case GB_FMT_MXFP4_SPLIT:
      if (!d->gate_up_blocks || !d->gate_up_scales || !d->down_blocks || !d->down_scales)
        return set_err(GB_ERR_INVALID_ARG, "MXFP4_SPLIT needs gate_up/down blocks and scales");
      break;
    case GB_FMT_MXFP4_GGUF:
      if (!d->gate_raw || (!d->up_raw && !d->gate_up_merged) || !d->down_raw)
        return set_err(GB_ERR_INVALID_ARG, "MXFP4_GGUF needs gate_raw, up_raw and down_raw");
      break;
    case GB_FMT_DENSE:
      if (!d->gate_raw || !d->up_raw || !d->down_raw)
        return set_err(GB_ERR_INVALID_ARG, "DENSE needs gate_raw, up_raw and down_raw");
      if (d->weight_dtype != GB_DTYPE_F32 && d->weight_dtype != GB_DTYPE_BF16)
        return set_err(GB_ERR_INVALID_ARG, "unknown weight_dtype %d", d->weight_dtype);
      if (d->act_kind == GB_ACT_GPTOSS_CLAMP)
        return set_err(GB_ERR_UNSUPPORTED, "DENSE experts take a gated activation");
      break;
    case GB_FMT_Q4_K:
      if (!d->gate_raw || (!d->up_raw && !d->gate_up_merged) || !d->down_raw)
        return set_err(GB_ERR_INVALID_ARG, "Q4_K needs gate_raw, up_raw and down_raw");
      // QExperts::dequantize_expert (quantized.rs:162-177) refuses a ragged expert
      if (d->hidden % 256 != 0 || d->inter % 256 != 0)
        return set_err(GB_ERR_SHAPE,
                       "Q4_K expert rows of %d (hidden) / %d (inter) elements are not a whole "
                       "number of 256-element super-blocks",
                       d->hidden, d->inter);
      break;
    default:
      return set_err(GB_ERR_INVALID_ARG, "unknown weight_format %d", d->weight_format);
  }
  // quantized.rs:417-425: a ragged expert is an error naming the count and block size.
  const int64_t elems_gu = (int64_t)d->hidden, elems_dn = (int64_t)d->inter;
  if (elems_gu % 32 != 0 || elems_dn % 32 != 0)
    return set_err(GB_ERR_SHAPE,
                   "MXFP4 expert rows of %lld (hidden) / %lld (inter) elements are not a whole "
                   "number of 32-element blocks",
                   (long long)elems_gu, (long long)elems_dn);
  if (d->hidden / 32 > 128 || d->inter / 32 > 128)
    return set_err(GB_ERR_UNSUPPORTED, "hidden/inter above 4096 are not supported");
  if (d->ep_size < 0 || (d->ep_size > 1 && (d->ep_rank < 0 || d->ep_rank >= d->ep_size)))
    return set_err(GB_ERR_INVALID_ARG, "bad ep_rank %d / ep_size %d", d->ep_rank, d->ep_size);
  if (d->ep_size > 1) {
    if (d->n_experts % d->ep_size != 0)
      return set_err(GB_ERR_INVALID_ARG, "n_experts %d not divisible by ep_size %d", d->n_experts,
                     d->ep_size);
    if (!d->nccl_id) return set_err(GB_ERR_INVALID_ARG, "ep_size > 1 needs nccl_id");
  }
  if (d->max_tokens < 0) return set_err(GB_ERR_INVALID_ARG, "max_tokens %d < 0", d->max_tokens);
  return GB_OK;
}

void free_ws(gb::Workspace& ws) {
  gb::free_expert_bufs(ws.eb);
  if (ws.base) cudaFree(ws.base);
  ws = gb::Workspace{};
}

// Destroys the cached forward graphs once the device has finished them.
// The handle's device is current.
void clear_graphs(gb::Moe& m) {
  bool any = false;
  for (const auto& g : m.graphs) any |= g.exec != nullptr;
  if (!any) return;
  cudaDeviceSynchronize();
  for (auto& g : m.graphs) {
    if (g.exec) cudaGraphExecDestroy(g.exec);
    g = gb::Moe::Graph{};
  }
  for (auto& g : m.seen) g = gb::Moe::Graph{};
}

struct Piece {
  void** ptr;
  size_t bytes;
};

// One allocation carved into 256-byte aligned pieces, zero-filled.
template <size_t N>
int carve(Piece (&pieces)[N], void** base_out, size_t* bytes_out, const char* what) {
  size_t total = 0;
  for (auto& p : pieces) total += (size_t)round_up((int64_t)p.bytes, 256);
  void* base = nullptr;
  cudaError_t e = cudaMalloc(&base, total);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_err(GB_ERR_NO_MEMORY, "%s: %zu bytes: %s", what, total, cudaGetErrorString(e));
  }
  e = cudaMemset(base, 0, total);
  if (e != cudaSuccess) {
    cudaFree(base);
    return cuda_err(e, what);
  }
  size_t off = 0;
  for (auto& p : pieces) {
    *p.ptr = p.bytes ? static_cast<char*>(base) + off : nullptr;
    off += (size_t)round_up((int64_t)p.bytes, 256);
  }
  *base_out = base;
  *bytes_out = total;
  return GB_OK;
}

// Routing workspace for T local tokens, plus the single-GPU expert buffers.
int alloc_ws(gb::Moe& m, int64_t T) {
  const gb_moe_desc& d = m.desc;
  const int64_t E = d.n_experts, K = d.top_k, H = d.hidden;
  T = std::max<int64_t>(T, 1);
  const bool ep = m.ep_size > 1;
  const bool sh_tc = gb::dense_tc_shared_supported(m);
  gb::Workspace ws;
  ws.tokens = T;
  Piece pieces[] = {
      {(void**)&ws.logits, sizeof(float) * (size_t)(T * E)},
      {(void**)&ws.tickets, sizeof(unsigned) * (size_t)T},
      {(void**)&ws.grid_bar, sizeof(unsigned) * 2},
      {(void**)&ws.idx, sizeof(int32_t) * (size_t)(T * K)},
      {(void**)&ws.wts, sizeof(float) * (size_t)(T * K)},
      {(void**)&ws.counts, sizeof(int32_t) * (size_t)E},
      {(void**)&ws.offsets, sizeof(int32_t) * (size_t)(E + 1)},
      {(void**)&ws.active, sizeof(int32_t) * (size_t)E},
      {(void**)&ws.meta, sizeof(int32_t) * 4},
      {(void**)&ws.perm, sizeof(int32_t) * (size_t)(T * K)},
      {(void**)&ws.inv, sizeof(int32_t) * (size_t)(T * K)},
      {(void**)&ws.x_route, d.input_norm ? sizeof(float) * (size_t)(T * H) : 0},
      {(void**)&ws.x_expert, d.input_norm ? sizeof(float) * (size_t)(T * H) : 0},
      {(void**)&ws.sh_h, sizeof(float) * (size_t)(T * std::max(d.shared_inter, 0))},
      {(void**)&ws.sh_y, d.shared_inter > 0 ? sizeof(float) * (size_t)(T * H) : 0},
      {(void**)&ws.sh_xh, sh_tc ? 2 * (size_t)(T * H) : 0},
      {(void**)&ws.sh_xl, sh_tc ? 2 * (size_t)(T * H) : 0},
      {(void**)&ws.sh_hh, sh_tc ? 2 * (size_t)(T * d.shared_inter) : 0},
      {(void**)&ws.sh_hl, sh_tc ? 2 * (size_t)(T * d.shared_inter) : 0},
      {(void**)&ws.x_stage, sizeof(float) * (size_t)(T * H)},
      {(void**)&ws.out_stage, sizeof(float) * (size_t)(T * H)},
  };
  void* base = nullptr;
  size_t bytes = 0;
  int rc = carve(pieces, &base, &bytes, "routing workspace");
  if (rc) return rc;
  ws.base = base;
  ws.bytes = bytes;
  if (sh_tc) {
    const cudaError_t e = gb::dense_tc_make_ws_maps(m, ws);
    if (e != cudaSuccess) {
      cudaFree(base);
      return cuda_err(e, "TMA descriptors of the shared expert");
    }
  }
  if (!ep && (rc = gb::alloc_expert_bufs(m, ws.eb, T * K))) {
    cudaFree(base);
    return rc;
  }
  clear_graphs(m);
  free_ws(m.ws);
  m.ws = ws;
  return GB_OK;
}

int ensure_ws(gb::Moe& m, int64_t T, cudaStream_t st) {
  if (T <= m.ws.tokens) return GB_OK;
  GB_CUDA(cudaStreamSynchronize(st), "synchronise before workspace growth");
  return alloc_ws(m, T);
}

template <typename Tp>
int dev_alloc(Tp** p, size_t bytes, const char* what) {
  cudaError_t e = cudaMalloc((void**)p, bytes);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_err(GB_ERR_NO_MEMORY, "cudaMalloc %s (%zu bytes): %s", what, bytes,
                   cudaGetErrorString(e));
  }
  return GB_OK;
}

// Frees the device memory of a handle (the handle object itself stays).
void release_moe(gb::Moe& m) {
  DeviceScope ds(m.device);
  for (auto& e : m.ev)
    if (e) cudaEventDestroy(e);
  for (auto& e : m.host_ev)
    if (e) cudaEventDestroy(e);
  clear_graphs(m);
  if (m.cap) cudaStreamDestroy(m.cap);
  if (m.h2d) cudaStreamDestroy(m.h2d);
  if (m.d2h) cudaStreamDestroy(m.d2h);
  cudaFree(m.router_w);
  cudaFree(m.router_b);
  cudaFree(m.sel_bias);
  cudaFree(m.w.gu_blocks);
  cudaFree(m.w.gu_scales);
  cudaFree(m.w.dn_blocks);
  cudaFree(m.w.dn_scales);
  cudaFree(m.w.gu_bias);
  cudaFree(m.w.dn_bias);
  cudaFree(m.w.gu_rowmax);
  cudaFree(m.w.dn_rowmax);
  cudaFree(m.w.q4_gu);
  cudaFree(m.w.q4_dn);
  cudaFree(m.w.q4_gu_exp);
  cudaFree(m.w.q4_gu_t);
  cudaFree(m.w.q4_dn_t);
  for (void* p : {m.w.dense_gu, m.w.dense_down, m.w.sh_gu, m.w.sh_down,
                  (void*)m.w.expert_scale, (void*)m.w.router_in_scale,
                  (void*)m.w.expert_in_norm, (void*)m.w.out_norm})
    cudaFree(p);
  gb::mx_release(m.mx);
  free_ws(m.ws);
  gb::ep_destroy(m);
  m = gb::Moe{};
}

int upload_router(gb::Moe& m);

// Q4_K: the caller's blocks as they are, gate and up rows interleaved.
int upload_q4k(gb::Moe& m) {
  const gb_moe_desc& d = m.desc;
  const int64_t H = d.hidden, I = d.inter;
  const int64_t nloc = m.e_end - m.e_begin;
  const size_t rb_h = (size_t)(H / 256) * 144, rb_i = (size_t)(I / 256) * 144;
  const size_t gu_bytes = (size_t)(nloc * 2 * I) * rb_h, dn_bytes = (size_t)(nloc * H) * rb_i;
  int rc;
  if ((rc = dev_alloc(&m.w.q4_gu, gu_bytes, "Q4_K gate_up"))) return rc;
  if ((rc = dev_alloc(&m.w.q4_dn, dn_bytes, "Q4_K down"))) return rc;
  m.weight_bytes = (int64_t)(gu_bytes + dn_bytes);
  for (int64_t le = 0; le < nloc; ++le) {
    const int64_t e = m.e_begin + le;
    uint8_t* dst = m.w.q4_gu + (size_t)(le * 2 * I) * rb_h;
    // separate gate / up [E, I, H], or merged [E, 2I, H] with gate rows first
    const uint8_t* gsrc = d.gate_up_merged ? d.gate_raw + (size_t)(e * 2 * I) * rb_h
                                           : d.gate_raw + (size_t)(e * I) * rb_h;
    const uint8_t* usrc = d.gate_up_merged ? gsrc + (size_t)I * rb_h
                                           : d.up_raw + (size_t)(e * I) * rb_h;
    GB_CUDA(cudaMemcpy2D(dst, 2 * rb_h, gsrc, rb_h, rb_h, (size_t)I, cudaMemcpyHostToDevice),
            "upload Q4_K gate");
    GB_CUDA(cudaMemcpy2D(dst + rb_h, 2 * rb_h, usrc, rb_h, rb_h, (size_t)I, cudaMemcpyHostToDevice),
            "upload Q4_K up");
  }
  GB_CUDA(cudaMemcpy(m.w.q4_dn, d.down_raw + (size_t)(m.e_begin * H) * rb_i, dn_bytes,
                     cudaMemcpyHostToDevice),
          "upload Q4_K down");
  return upload_router(m);
}

// Dense experts: the caller's rows as they are (bf16 or f32), local experts
// only; the shared expert whole.
int upload_dense(gb::Moe& m) {
  const gb_moe_desc& d = m.desc;
  const size_t es = d.weight_dtype == GB_DTYPE_BF16 ? 2 : 4;
  const int64_t H = d.hidden, I = d.inter, nloc = m.e_end - m.e_begin;
  m.w.dense_bf16 = d.weight_dtype == GB_DTYPE_BF16;
  const size_t mat = (size_t)(I * H) * es;
  int rc;
  struct Part {
    void** dst;
    const void* src;
    size_t bytes;
    const char* what;
  };
  const size_t sh = (size_t)d.shared_inter * (size_t)H * es;
  const size_t row = (size_t)H * es;
  m.weight_bytes = 0;
  // gate and up rows interleaved on the device: row 2i = gate i, 2i + 1 = up i
  auto interleave = [&](void** dst, const void* gate, const void* up, size_t rows,
                        const char* what) -> int {
    int r = dev_alloc((char**)dst, 2 * rows * row, what);
    if (r) return r;
    GB_CUDA(cudaMemcpy2D(*dst, 2 * row, gate, row, row, rows, cudaMemcpyHostToDevice), what);
    GB_CUDA(cudaMemcpy2D(static_cast<char*>(*dst) + row, 2 * row, up, row, row, rows,
                         cudaMemcpyHostToDevice),
            what);
    m.weight_bytes += (int64_t)(2 * rows * row);
    return GB_OK;
  };
  if ((rc = interleave(&m.w.dense_gu,
                       static_cast<const char*>((const void*)d.gate_raw) + m.e_begin * mat,
                       static_cast<const char*>((const void*)d.up_raw) + m.e_begin * mat,
                       (size_t)(nloc * I), "dense gate_up")))
    return rc;
  if ((rc = dev_alloc((char**)&m.w.dense_down, nloc * mat, "dense down"))) return rc;
  GB_CUDA(cudaMemcpy(m.w.dense_down,
                     static_cast<const char*>((const void*)d.down_raw) + m.e_begin * mat,
                     nloc * mat, cudaMemcpyHostToDevice),
          "dense down");
  m.weight_bytes += (int64_t)(nloc * mat);
  if (sh) {
    if ((rc = interleave(&m.w.sh_gu, d.shared_gate, d.shared_up, (size_t)d.shared_inter,
                         "shared gate_up")))
      return rc;
    if ((rc = dev_alloc((char**)&m.w.sh_down, sh, "shared down"))) return rc;
    GB_CUDA(cudaMemcpy(m.w.sh_down, d.shared_down, sh, cudaMemcpyHostToDevice), "shared down");
    m.weight_bytes += (int64_t)sh;
  }
  return upload_router(m);
}

int upload_weights(gb::Moe& m) {
  const gb_moe_desc& d = m.desc;
  if (d.weight_format == GB_FMT_Q4_K) return upload_q4k(m);
  if (d.weight_format == GB_FMT_DENSE) return upload_dense(m);
  const int64_t H = d.hidden, I = d.inter;
  const int64_t nloc = m.e_end - m.e_begin;
  const int64_t nbh = H / 32, nbi = I / 32;
  m.w.sp_h = (int)round_up(nbh, 16);
  m.w.sp_i = (int)round_up(nbi, 16);
  m.w.zero_scale = d.weight_format == GB_FMT_MXFP4_GGUF ? 0x1p-127f : 0.0f;

  const size_t gu_blocks = (size_t)(nloc * 2 * I * nbh * 16);
  const size_t gu_scales = (size_t)(nloc * 2 * I * m.w.sp_h);
  const size_t dn_blocks = (size_t)(nloc * H * nbi * 16);
  const size_t dn_scales = (size_t)(nloc * H * m.w.sp_i);
  int rc;
  if ((rc = dev_alloc(&m.w.gu_blocks, gu_blocks, "gate_up blocks"))) return rc;
  if ((rc = dev_alloc(&m.w.gu_scales, gu_scales, "gate_up scales"))) return rc;
  if ((rc = dev_alloc(&m.w.dn_blocks, dn_blocks, "down blocks"))) return rc;
  if ((rc = dev_alloc(&m.w.dn_scales, dn_scales, "down scales"))) return rc;
  GB_CUDA(cudaMemset(m.w.gu_scales, 0, gu_scales), "memset scales");
  GB_CUDA(cudaMemset(m.w.dn_scales, 0, dn_scales), "memset scales");
  m.weight_bytes = (int64_t)(gu_blocks + gu_scales + dn_blocks + dn_scales);

  if (d.weight_format == GB_FMT_MXFP4_SPLIT) {
    const int64_t e0 = m.e_begin;
    GB_CUDA(cudaMemcpy(m.w.gu_blocks, d.gate_up_blocks + e0 * 2 * I * nbh * 16, gu_blocks,
                       cudaMemcpyHostToDevice),
            "upload gate_up blocks");
    GB_CUDA(cudaMemcpy2D(m.w.gu_scales, (size_t)m.w.sp_h, d.gate_up_scales + e0 * 2 * I * nbh,
                         (size_t)nbh, (size_t)nbh, (size_t)(nloc * 2 * I), cudaMemcpyHostToDevice),
            "upload gate_up scales");
    GB_CUDA(cudaMemcpy(m.w.dn_blocks, d.down_blocks + e0 * H * nbi * 16, dn_blocks,
                       cudaMemcpyHostToDevice),
            "upload down blocks");
    GB_CUDA(cudaMemcpy2D(m.w.dn_scales, (size_t)m.w.sp_i, d.down_scales + e0 * H * nbi,
                         (size_t)nbi, (size_t)nbi, (size_t)(nloc * H), cudaMemcpyHostToDevice),
            "upload down scales");
  } else {
    // GGUF: per expert, upload the raw 17-byte blocks and convert on the device.
    const size_t raw_gate = (size_t)(I * nbh * 17), raw_down = (size_t)(H * nbi * 17);
    uint8_t* tmp = nullptr;
    if ((rc = dev_alloc(&tmp, std::max(raw_gate, raw_down), "GGUF staging"))) return rc;
    for (int64_t le = 0; le < nloc && rc == GB_OK; ++le) {
      const int64_t e = m.e_begin + le;
      for (int which = 0; which < 3 && rc == GB_OK; ++which) {
        const size_t bytes = which == 2 ? raw_down : raw_gate;
        const uint8_t* src;
        if (which == 2)
          src = d.down_raw + (size_t)e * bytes;
        else if (d.gate_up_merged)  // [E, 2I, H]: gate rows, then up rows
          src = d.gate_raw + (size_t)e * 2 * bytes + (size_t)which * bytes;
        else
          src = (which == 0 ? d.gate_raw : d.up_raw) + (size_t)e * bytes;
        cudaError_t ce = cudaMemcpy(tmp, src, bytes, cudaMemcpyHostToDevice);
        if (ce == cudaSuccess) {
          if (which < 2) {
            // gate row i -> fused row 2i, up row i -> 2i+1
            ce = gb::launch_gguf_to_split(
                tmp, I, (int)H, m.w.gu_blocks + ((le * 2 * I + which) * nbh) * 16, 2 * nbh,
                m.w.gu_scales + (le * 2 * I + which) * m.w.sp_h, 2 * (int64_t)m.w.sp_h, 0);
          } else {
            ce = gb::launch_gguf_to_split(tmp, H, (int)I, m.w.dn_blocks + (le * H * nbi) * 16, nbi,
                                          m.w.dn_scales + le * H * m.w.sp_i, m.w.sp_i, 0);
          }
        }
        if (ce == cudaSuccess) ce = cudaDeviceSynchronize();
        if (ce != cudaSuccess) rc = cuda_err(ce, "GGUF expert upload");
      }
    }
    cudaFree(tmp);
    if (rc) return rc;
  }

  // Biases -> f32, fused gate_up order.
  if (d.weight_format == GB_FMT_MXFP4_SPLIT ? d.gate_up_bias != nullptr
                                            : (d.gate_bias != nullptr || d.up_bias != nullptr)) {
    std::vector<float> gub((size_t)(nloc * 2 * I), 0.0f);
    if (d.weight_format == GB_FMT_MXFP4_SPLIT) {
      const size_t esz = d.bias_dtype == GB_DTYPE_BF16 ? 2 : 4;
      gub = widen(static_cast<const char*>(d.gate_up_bias) + (size_t)(m.e_begin * 2 * I) * esz,
                  nloc * 2 * I, d.bias_dtype);
    } else {
      const size_t esz = d.bias_dtype == GB_DTYPE_BF16 ? 2 : 4;
      std::vector<float> g, u;
      if (d.gate_bias)
        g = widen(static_cast<const char*>(d.gate_bias) + (size_t)(m.e_begin * I) * esz, nloc * I,
                  d.bias_dtype);
      if (d.up_bias)
        u = widen(static_cast<const char*>(d.up_bias) + (size_t)(m.e_begin * I) * esz, nloc * I,
                  d.bias_dtype);
      for (int64_t le = 0; le < nloc; ++le)
        for (int64_t i = 0; i < I; ++i) {
          gub[(size_t)(le * 2 * I + 2 * i)] = g.empty() ? 0.0f : g[(size_t)(le * I + i)];
          gub[(size_t)(le * 2 * I + 2 * i + 1)] = u.empty() ? 0.0f : u[(size_t)(le * I + i)];
        }
    }
    if ((rc = dev_alloc(&m.w.gu_bias, gub.size() * 4, "gate_up bias"))) return rc;
    GB_CUDA(cudaMemcpy(m.w.gu_bias, gub.data(), gub.size() * 4, cudaMemcpyHostToDevice),
            "upload gate_up bias");
  }
  if (d.down_bias) {
    const size_t esz = d.bias_dtype == GB_DTYPE_BF16 ? 2 : 4;
    std::vector<float> db = widen(
        static_cast<const char*>(d.down_bias) + (size_t)(m.e_begin * H) * esz, nloc * H, d.bias_dtype);
    if ((rc = dev_alloc(&m.w.dn_bias, db.size() * 4, "down bias"))) return rc;
    GB_CUDA(cudaMemcpy(m.w.dn_bias, db.data(), db.size() * 4, cudaMemcpyHostToDevice),
            "upload down bias");
  }

  return upload_router(m);
}

int upload_router(gb::Moe& m) {
  const gb_moe_desc& d = m.desc;
  const int64_t H = d.hidden, E = d.n_experts;
  int rc;
  // Router (replicated).
  std::vector<float> rw = widen(d.router_weight, E * H, d.router_dtype);
  if ((rc = dev_alloc(&m.router_w, rw.size() * 4, "router weight"))) return rc;
  GB_CUDA(cudaMemcpy(m.router_w, rw.data(), rw.size() * 4, cudaMemcpyHostToDevice),
          "upload router weight");
  if (d.router_bias) {
    std::vector<float> rb = widen(d.router_bias, E, d.router_dtype);
    if ((rc = dev_alloc(&m.router_b, rb.size() * 4, "router bias"))) return rc;
    GB_CUDA(cudaMemcpy(m.router_b, rb.data(), rb.size() * 4, cudaMemcpyHostToDevice),
            "upload router bias");
  }
  if (d.selection_bias) {
    if ((rc = dev_alloc(&m.sel_bias, (size_t)E * 4, "selection bias"))) return rc;
    GB_CUDA(cudaMemcpy(m.sel_bias, d.selection_bias, (size_t)E * 4, cudaMemcpyHostToDevice),
            "upload selection bias");
  }
  // Gemma-4: expert output scales (all E: the combine reads them by global
  // id) and the norm vectors
  const struct {
    float** dst;
    const float* src;
    int64_t n;
  } vecs[] = {{&m.w.expert_scale, d.expert_scale, E},
              {&m.w.router_in_scale, d.input_norm ? d.router_input_scale : nullptr, H},
              {&m.w.expert_in_norm, d.input_norm ? d.expert_input_norm : nullptr, H},
              {&m.w.out_norm, d.output_norm, H}};
  for (const auto& v : vecs) {
    if (!v.src) continue;
    if ((rc = dev_alloc(v.dst, (size_t)v.n * 4, "Gemma-4 vector"))) return rc;
    GB_CUDA(cudaMemcpy(*v.dst, v.src, (size_t)v.n * 4, cudaMemcpyHostToDevice),
            "upload Gemma-4 vector");
  }
  return GB_OK;
}

// Stage boundary: record event i when profiling.
int mark(gb::Moe& m, int i, cudaStream_t st) { return gb::mark_stage(m, i, st); }

int run_route(gb::Moe& m, const float* x, int64_t T, cudaStream_t st) {
  int rc;
  if ((rc = mark(m, 0, st))) return rc;
  GB_CUDA(gb::launch_router_topk(m, x, T, m.ws.idx, m.ws.wts, st), "router kernel launch");
  if ((rc = mark(m, 1, st))) return rc;
  GB_CUDA(gb::launch_permute(m, m.ws.idx, T, m.ws, st), "permute kernel launch");
  m.launches += 2;
  return mark(m, 2, st);
}

enum class ExpertKernel { kCudaCores, kF16, kMx };

ExpertKernel pick_expert_kernel(const gb::Moe& m, const gb::ExpertBufs& eb) {
  const bool mx = m.mx.ok && eb.mx_maps_ok;
  const bool f16 = gb::tc_supported(m) && eb.maps_ok;
  switch (m.expert_path) {
    case GB_PATH_CUDA_CORES:
      return ExpertKernel::kCudaCores;
    case GB_PATH_TENSOR_CORES_F16:
      return f16 ? ExpertKernel::kF16 : ExpertKernel::kCudaCores;
    default:  // AUTO, TENSOR_CORES
      return mx ? ExpertKernel::kMx : f16 ? ExpertKernel::kF16 : ExpertKernel::kCudaCores;
  }
}

gb::Groups local_groups(const gb::Moe& m, int64_t T) {
  gb::Groups g;
  g.counts = m.ws.counts;
  g.offsets = m.ws.offsets;
  g.active = m.ws.active;
  g.meta = m.ws.meta;
  g.perm = m.ws.perm;
  g.perm_div = m.desc.top_k;
  g.rows = T * m.desc.top_k;
  g.max_active = (int)std::min<int64_t>(m.e_end - m.e_begin, T * m.desc.top_k);
  g.max_per_expert = T;
  g.out_rows = nullptr;
  return g;
}

// Reads and clears the error bits the kernels OR into meta[1] (bit 0: an
// expert index out of range in routing; bit 1: a pipeline wait timed out).
int read_device_status(gb::Moe& m, cudaStream_t st) {
  int32_t bits = 0, b2 = 0;
  const int32_t zero = 0;
  GB_CUDA(cudaMemcpyAsync(&bits, m.ws.meta + 1, sizeof bits, cudaMemcpyDeviceToHost, st),
          "read device status");
  GB_CUDA(cudaMemcpyAsync(m.ws.meta + 1, &zero, sizeof zero, cudaMemcpyHostToDevice, st),
          "clear device status");
  if (int32_t* em = gb::ep_meta(m)) {
    GB_CUDA(cudaMemcpyAsync(&b2, em + 1, sizeof b2, cudaMemcpyDeviceToHost, st),
            "read device status");
    GB_CUDA(cudaMemcpyAsync(em + 1, &zero, sizeof zero, cudaMemcpyHostToDevice, st),
            "clear device status");
  }
  GB_CUDA(cudaStreamSynchronize(st), "synchronise device status");
  bits |= b2;
  if (bits) {
    // a kernel that gave up may have left split-K tickets counted: clear them
    // so that the next forward starts from zero
    if (m.ws.eb.mx_arrivals)
      GB_CUDA(cudaMemsetAsync(m.ws.eb.mx_arrivals, 0, 2 * sizeof(int) * (size_t)gb::kMxSplitSlots, st),
              "clear split-K tickets");
    if (int* a = gb::ep_arrivals(m))
      GB_CUDA(cudaMemsetAsync(a, 0, 2 * sizeof(int) * (size_t)gb::kMxSplitSlots, st),
              "clear split-K tickets");
    if (m.ws.grid_bar)  // a grid barrier left mid-count
      GB_CUDA(cudaMemsetAsync(m.ws.grid_bar, 0, sizeof(unsigned), st), "clear grid barrier");
    GB_CUDA(cudaStreamSynchronize(st), "clear split-K tickets");
  }
  if (bits & 2) return set_err(GB_ERR_TIMEOUT, "a tensor-core pipeline wait timed out on the device");
  if (bits & 1) return set_err(GB_ERR_INVALID_ARG, "routing produced an expert index out of range");
  return GB_OK;
}

// Router, then grouping, tile table and pieces in one launch (small
// single-GPU batches on the block-scaled path); g.grouped set.
int run_route_grouped(gb::Moe& m, const float* x, int64_t T, gb::Groups& g, int kind,
                      cudaStream_t st) {
  int rc;
  if ((rc = mark(m, 0, st))) return rc;
  GB_CUDA(gb::launch_router_topk(m, x, T, m.ws.idx, m.ws.wts, st), "router kernel launch");
  if ((rc = mark(m, 1, st))) return rc;
  GB_CUDA(gb::launch_mx_group(m, x, T, m.ws, kind, st), "grouping kernel launch");
  m.launches += 2;
  g.grouped = true;
  return mark(m, 2, st);
}

int run_forward(gb::Moe& m, const float* x, int64_t T, float* out, cudaStream_t st) {
  int rc;
  if (m.expert_path == GB_PATH_FUSED_DECODE && gb::fused_decode_fits(m, T)) {
    // one launch: the router, grouping, expert and combine stages of the
    // profile are empty except the expert stage, which holds the kernel
    for (int i = 0; i < 3; ++i)
      if ((rc = mark(m, i, st))) return rc;
    GB_CUDA(gb::launch_fused_decode(m, x, T, out, st), "fused decode launch");
    m.launches += 1;
    for (int i = 3; i < 6; ++i)
      if ((rc = mark(m, i, st))) return rc;
    m.profiled_once = m.profiling;
    return GB_OK;
  }
  if (m.ep_size == 1 && m.desc.weight_format != GB_FMT_Q4_K && !m.desc.input_norm &&
      !m.w.out_norm && gb::mx_group_fits(m, T) &&
      pick_expert_kernel(m, m.ws.eb) == ExpertKernel::kMx) {
    gb::Groups g = local_groups(m, T);
    const int kind = std::min(gb::mx_tile_kind(m, g), gb::kMxKind30);
    if ((rc = run_route_grouped(m, x, T, g, kind, st))) return rc;
    if (g.rows >= gb::kMxOneLaunchRows) {
      // gate_up and down in one launch: the "down" stage is empty
      GB_CUDA(gb::launch_mx_ffn(m, g, m.ws.eb, kind, st), "block-scaled expert launch");
      m.launches += 1;
      if ((rc = mark(m, 3, st))) return rc;
    } else {
      GB_CUDA(gb::launch_mx_gate_up(m, g, x, m.ws.eb, kind, st), "block-scaled gate_up launch");
      if ((rc = mark(m, 3, st))) return rc;
      GB_CUDA(gb::launch_mx_down(m, g, m.ws.eb, kind, st), "block-scaled down launch");
      m.launches += 2;
    }
    if ((rc = mark(m, 4, st))) return rc;
    GB_CUDA(gb::launch_combine(m, T, m.ws, m.ws.eb.y, out, st), "combine kernel launch");
    m.launches += 1;
    if ((rc = mark(m, 5, st))) return rc;
    m.profiled_once = m.profiling;
    return GB_OK;
  }
  // Gemma-4: the router and the experts read differently normed copies of x
  const float* x_route = x;
  const float* x_expert = x;
  if (m.desc.input_norm && T > 0) {
    GB_CUDA(gb::launch_input_norms(m, x, T, m.ws.x_route, m.ws.x_expert, st), "input norm launch");
    x_route = m.ws.x_route;
    x_expert = m.ws.x_expert;
    m.launches += 1;
  }
  if (T > 0) {
    if ((rc = run_route(m, x_route, T, st))) return rc;
  } else {
    GB_CUDA(cudaMemsetAsync(m.ws.counts, 0, sizeof(int32_t) * m.desc.n_experts, st),
            "clear counts");
  }
  if (m.desc.shared_inter > 0 && T > 0) {  // shared expert over all tokens, added by combine
    if (gb::use_dense_tc_shared(m, T)) {
      GB_CUDA(gb::launch_shared_expert_tc(m, x_expert, T, m.ws.sh_y, st),
              "shared expert launch");
      m.launches += 3;
    } else {
      GB_CUDA(gb::launch_shared_expert(m, x_expert, T, m.ws.sh_h, m.ws.sh_y, st),
              "shared expert launch");
      m.launches += 2;
    }
  }
  if (m.ep_size > 1) {
    if ((rc = gb::ep_forward(m, x_expert, T, out, st))) return rc;
  } else {
    gb::Groups g = local_groups(m, T);
    if ((rc = gb::run_experts(m, g, x_expert, T, m.ws.eb, st))) return rc;
    if ((rc = mark(m, 4, st))) return rc;
    GB_CUDA(gb::launch_combine(m, T, m.ws, m.ws.eb.y, out, st), "combine kernel launch");
    m.launches += 1;
  }
  if (m.w.out_norm && T > 0) {  // post_ffw_norm_2 on the result
    GB_CUDA(gb::launch_output_norm(m, out, T, st), "output norm launch");
    m.launches += 1;
  }
  if ((rc = mark(m, 5, st))) return rc;
  m.profiled_once = m.profiling;
  return GB_OK;
}

// Captures the forward of (x, T, out) into `slot` (replacing what it held).
int capture_forward(gb::Moe& m, const float* x, int64_t T, float* out, gb::Moe::Graph* slot) {
  if (!m.cap) GB_CUDA(cudaStreamCreateWithFlags(&m.cap, cudaStreamNonBlocking), "capture stream");
  if (slot->exec) {
    // the replaced graph may still be running on any stream
    GB_CUDA(cudaDeviceSynchronize(), "synchronise before replacing a forward graph");
    cudaGraphExecDestroy(slot->exec);
    *slot = gb::Moe::Graph{};
  }
  const int64_t before = m.launches;
  GB_CUDA(cudaStreamBeginCapture(m.cap, cudaStreamCaptureModeThreadLocal), "begin forward capture");
  const int rc = run_forward(m, x, T, out, m.cap);
  cudaGraph_t graph = nullptr;
  const cudaError_t ce = cudaStreamEndCapture(m.cap, &graph);
  const int64_t n = m.launches - before;
  m.launches = before;
  if (rc || ce != cudaSuccess) {
    if (graph) cudaGraphDestroy(graph);
    return rc ? rc : cuda_err(ce, "capture forward");
  }
  cudaGraphExec_t exec = nullptr;
  const cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  if (ie != cudaSuccess) return cuda_err(ie, "instantiate forward graph");
  slot->x = x;
  slot->out = out;
  slot->T = T;
  slot->exec = exec;
  slot->launches = n;
  ++m.graph_captures;
  return GB_OK;
}

// Slot of `slots[0..n)` holding (x, out, T), or null; `victim` gets the
// empty or least recently used slot.
gb::Moe::Graph* find_slot(gb::Moe::Graph* slots, int n, const float* x, int64_t T,
                          const float* out, gb::Moe::Graph** victim) {
  *victim = &slots[0];
  for (int i = 0; i < n; ++i) {
    gb::Moe::Graph& g = slots[i];
    if (g.used && g.x == x && g.out == out && g.T == T) return &g;
    if ((*victim)->used && (!g.used || g.used < (*victim)->used)) *victim = &g;
  }
  return nullptr;
}

// The forward as gb_moe_forward runs it.  A single-GPU batch of at most
// kGraphMaxTokens tokens whose (x, out, T) came before replays a cached CUDA
// graph (its kernels last a few microseconds each, so launching them one by
// one from the host would dominate); other forwards launch their kernels
// directly.
int forward_dispatch(gb::Moe& m, const float* x, int64_t T, float* out, cudaStream_t st) {
  // the fused decode forward is one (cooperative) launch: nothing to replay
  if (m.ep_size > 1 || m.profiling || m.graph_slots <= 0 || T <= 0 ||
      T > gb::Moe::kGraphMaxTokens ||
      (m.expert_path == GB_PATH_FUSED_DECODE && gb::fused_decode_fits(m, T)))
    return run_forward(m, x, T, out, st);
  gb::Moe::Graph* victim = nullptr;
  gb::Moe::Graph* hit = find_slot(m.graphs, m.graph_slots, x, T, out, &victim);
  if (!hit) {
    gb::Moe::Graph* seen_victim = nullptr;
    gb::Moe::Graph* seen = find_slot(m.seen, m.graph_slots, x, T, out, &seen_victim);
    if (!seen) {
      // first sighting: remember it and launch directly
      *seen_victim = gb::Moe::Graph{x, out, T, nullptr, 0, ++m.graph_clock};
      return run_forward(m, x, T, out, st);
    }
    *seen = gb::Moe::Graph{};
    int rc = capture_forward(m, x, T, out, victim);
    if (rc) return rc;
    hit = victim;
  }
  hit->used = ++m.graph_clock;
  GB_CUDA(cudaGraphLaunch(hit->exec, st), "forward graph launch");
  m.launches += hit->launches;
  return GB_OK;
}

}  // namespace

namespace gb {

// Q4_K experts: the tensor-core kernels for groups averaging at least 2 rows
// per local expert (or when the tensor cores are forced); the CUDA-core
// kernel streams smaller groups faster (LFM2.5 layer, 32 experts: 16 tokens
// 192 us on the tensor cores against 221 on the CUDA cores, 24 tokens 209
// against 287; the two about even near 1.5 rows per expert).
// Dense bf16 experts: the tensor cores from one grouped position per two
// local experts (measured on 128 experts x 2048 x 768, top-8: T = 8 took
// 178 us on the tensor cores against 249 on the CUDA cores, T = 4 142
// against 123); the shared expert from 16 tokens.
constexpr int64_t kDenseTcShared = 16;

bool use_dense_tc(const Moe& m, const Groups& g, const ExpertBufs& eb) {
  if (!dense_tc_supported(m) || !eb.maps_ok || m.expert_path == GB_PATH_CUDA_CORES) return false;
  if (m.expert_path == GB_PATH_TENSOR_CORES || m.expert_path == GB_PATH_TENSOR_CORES_F16)
    return true;
  const int64_t nloc = std::max(1, m.e_end - m.e_begin);
  return 2 * g.rows >= nloc;
}

bool use_dense_tc_shared(const Moe& m, int64_t T) {
  if (!dense_tc_shared_supported(m) || m.expert_path == GB_PATH_CUDA_CORES) return false;
  if (m.expert_path == GB_PATH_TENSOR_CORES || m.expert_path == GB_PATH_TENSOR_CORES_F16)
    return true;
  return T >= kDenseTcShared;
}

bool use_q4k_tc(const Moe& m, const Groups& g, const ExpertBufs& eb) {
  if (!q4k_tc_supported(m) || !eb.maps_ok || m.expert_path == GB_PATH_CUDA_CORES) return false;
  if (m.expert_path == GB_PATH_TENSOR_CORES || m.expert_path == GB_PATH_TENSOR_CORES_F16)
    return true;
  const int64_t nloc = std::max(1, m.e_end - m.e_begin);
  return g.rows >= 2 * nloc;
}

cudaError_t set_smem_limit_fn(const void* kern, size_t bytes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  static std::mutex mu;
  static std::vector<std::tuple<const void*, int, size_t>> done;
  std::lock_guard<std::mutex> lock(mu);
  for (const auto& [k, d, b] : done)
    if (k == kern && d == dev && b >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e == cudaSuccess) done.emplace_back(kern, dev, bytes);
  return e;
}

int run_experts(Moe& m, const Groups& g, const float* x, int64_t T, ExpertBufs& eb,
                cudaStream_t st, bool* stored_return) {
  int rc;
  (void)T;
  if (stored_return) *stored_return = false;
  if (m.desc.weight_format == GB_FMT_DENSE && use_dense_tc(m, g, eb)) {
    GB_CUDA(launch_dense_tc_gate_up(m, g, x, eb, st), "dense tensor-core gate_up launch");
    if ((rc = mark(m, 3, st))) return rc;
    GB_CUDA(launch_dense_tc_down(m, g, eb, st), "dense tensor-core down launch");
    m.launches += 4;  // tile table, split, two GEMMs
  } else if (m.desc.weight_format == GB_FMT_DENSE) {
    GB_CUDA(launch_dense_gate_up(m, g, x, eb, st), "dense gate_up launch");
    if ((rc = mark(m, 3, st))) return rc;
    GB_CUDA(launch_dense_down(m, g, eb, st), "dense down launch");
    m.launches += 2;
  } else if (m.desc.weight_format == GB_FMT_Q4_K && use_q4k_tc(m, g, eb)) {
    GB_CUDA(launch_q4k_tc_gate_up(m, g, x, eb, st), "Q4_K tensor-core gate_up launch");
    if ((rc = mark(m, 3, st))) return rc;
    GB_CUDA(launch_q4k_tc_down(m, g, eb, st), "Q4_K tensor-core down launch");
    m.launches += 4;  // tile table, split, two GEMMs
  } else if (m.desc.weight_format == GB_FMT_Q4_K) {
    GB_CUDA(launch_q4k_gate_up(m, g, x, eb, st), "Q4_K gate_up launch");
    if ((rc = mark(m, 3, st))) return rc;
    GB_CUDA(launch_q4k_down(m, g, eb, st), "Q4_K down launch");
    m.launches += 2;
  } else if (const ExpertKernel k = pick_expert_kernel(m, eb); k != ExpertKernel::kCudaCores) {
    if (k == ExpertKernel::kMx) {
      const int kind = gb::mx_tile_kind(m, g);
      GB_CUDA(launch_mx_gate_up(m, g, x, eb, kind, st), "block-scaled gate_up launch");
      if ((rc = mark(m, 3, st))) return rc;
      GB_CUDA(launch_mx_down(m, g, eb, kind, st), "block-scaled down launch");
      // the block-scaled down epilogue stores rows in their return slots
      if (stored_return && g.ret_dst) *stored_return = true;
    } else {
      GB_CUDA(launch_tc_gate_up(m, g, x, eb, st), "tensor-core gate_up launch");
      if ((rc = mark(m, 3, st))) return rc;
      GB_CUDA(launch_tc_down(m, g, eb, st), "tensor-core down launch");
    }
    m.launches += 4;  // tile table, split, two GEMMs
  } else if (decode_supported(m)) {
    GB_CUDA(launch_decode_gate_up(m, g, x, eb, st), "decode gate_up launch");
    if ((rc = mark(m, 3, st))) return rc;
    GB_CUDA(launch_decode_down(m, g, eb, st), "decode down launch");
    m.launches += 2;
  } else {
    GB_CUDA(launch_gate_up(m, g, x, eb, st), "gate_up kernel launch");
    if ((rc = mark(m, 3, st))) return rc;
    GB_CUDA(launch_down(m, g, eb, st), "down kernel launch");
    m.launches += 2;
  }
  return GB_OK;
}

}  // namespace gb

namespace {

int check_handle(gb_moe* h) {
  if (!h) return set_err(GB_ERR_INVALID_ARG, "handle is null");
  return GB_OK;
}

}  // namespace

namespace gb {
int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof g_err, fmt, ap);
  va_end(ap);
  return code;
}
}  // namespace gb

namespace gb {

int mark_stage(Moe& m, int i, cudaStream_t st) {
  if (m.profiling) GB_CUDA(cudaEventRecord(m.ev[i], st), "record stage event");
  return GB_OK;
}

void free_expert_bufs(ExpertBufs& eb) {
  if (eb.base) cudaFree(eb.base);
  eb = ExpertBufs{};
}

int alloc_expert_bufs(const Moe& m, ExpertBufs& eb, int64_t rows) {
  const gb_moe_desc& d = m.desc;
  const int64_t E = d.n_experts, H = d.hidden, I = d.inter;
  rows = std::max<int64_t>(rows, 1);
  const bool dense_tc = dense_tc_supported(m);
  const bool tc = tc_supported(m) || q4k_tc_supported(m) || dense_tc;
  ExpertBufs nb;
  nb.rows_cap = rows;
  Piece pieces[] = {
      {(void**)&nb.h, sizeof(float) * (size_t)(rows * I)},
      {(void**)&nb.y, sizeof(float) * (size_t)(rows * H)},
      {(void**)&nb.xh, tc ? sizeof(__half) * (size_t)(rows * H) : 0},
      {(void**)&nb.xl, tc ? sizeof(__half) * (size_t)(rows * H) : 0},
      {(void**)&nb.xscale, (tc || m.mx.ok) ? sizeof(float) * (size_t)rows : 0},
      {(void**)&nb.hh, tc ? sizeof(__half) * (size_t)(rows * I) : 0},
      {(void**)&nb.hl, tc ? sizeof(__half) * (size_t)(rows * I) : 0},
      {(void**)&nb.xsum, q4k_tc_supported(m) ? sizeof(float) * (size_t)(rows * (std::max(H, I) / 32)) : 0},
      {(void**)&nb.xq, m.mx.ok ? mx_piece_bytes(rows, (int)H) : 0},
      {(void**)&nb.hq, m.mx.ok ? mx_piece_bytes(rows, (int)I) : 0},
      {(void**)&nb.mx_partial, m.mx.ok ? 2 * kMxPartialBytes : 0},
      {(void**)&nb.mx_arrivals, m.mx.ok ? 2 * sizeof(int) * (size_t)kMxSplitSlots : 0},
      {(void**)&nb.mx_ready,
       m.mx.ok ? sizeof(int) * (size_t)(1 + std::min<int64_t>(rows, kMxGroupEntries) *
                                               mx_ready_per_tile(m))
               : 0},
      {(void**)&nb.tile_expert, sizeof(int32_t) * (size_t)(rows + E + 1)},
      {(void**)&nb.tile_row0, sizeof(int32_t) * (size_t)(rows + E + 1)},
      {(void**)&nb.tile_rows, sizeof(int32_t) * (size_t)(rows + E + 1)},
  };
  int rc = carve(pieces, &nb.base, &nb.bytes, "expert buffers");
  if (rc) return rc;
  if (tc) {
    cudaError_t e = dense_tc ? dense_tc_make_maps(m, nb) : tc_make_maps(m, nb);
    if (e != cudaSuccess) {
      cudaFree(nb.base);
      return cuda_err(e, "TMA descriptors for the tensor-core path");
    }
    nb.maps_ok = true;
  }
  if (m.mx.ok) {
    cudaError_t e = cudaMemset(nb.mx_arrivals, 0, 2 * sizeof(int) * (size_t)kMxSplitSlots);
    if (e == cudaSuccess) e = mx_make_maps(m, nb);
    if (e != cudaSuccess) {
      cudaFree(nb.base);
      return cuda_err(e, "TMA descriptors for the block-scaled path");
    }
    nb.mx_maps_ok = true;
  }
  free_expert_bufs(eb);
  eb = nb;
  return GB_OK;
}

}  // namespace gb

struct gb_moe {
  gb::Moe m;
};

extern "C" {

int gb_abi_version(void) { return GB_ABI_VERSION; }

const char* gb_last_error(void) { return g_err; }

int gb_moe_create(const gb_moe_desc* desc, gb_moe** out) {
  g_err[0] = 0;
  if (!out) return set_err(GB_ERR_INVALID_ARG, "out is null");
  *out = nullptr;
  // A descriptor from an older header (shorter struct_size) reads as zeros in
  // the fields it lacks.
  gb_moe_desc dcopy;
  memset(&dcopy, 0, sizeof dcopy);
  if (desc && desc->struct_size >= offsetof(gb_moe_desc, ep_timeout_ms))
    memcpy(&dcopy, desc, std::min<size_t>(desc->struct_size, sizeof dcopy));
  else if (desc)
    return set_err(GB_ERR_INVALID_ARG, "descriptor struct_size %u is too small (header mismatch)",
                   desc->struct_size);
  if (desc) {
    dcopy.struct_size = sizeof dcopy;
    desc = &dcopy;
  }
  int rc = validate(desc);
  if (rc) return rc;
  int ndev = 0;
  GB_CUDA(cudaGetDeviceCount(&ndev), "cudaGetDeviceCount");
  if (desc->device < 0 || desc->device >= ndev)
    return set_err(GB_ERR_INVALID_ARG, "device %d does not exist (%d visible)", desc->device, ndev);
  DeviceScope ds(desc->device);
  if (!ds.ok) return set_err(GB_ERR_CUDA, "cannot make device %d current", desc->device);
  gb_moe* h = new (std::nothrow) gb_moe();
  if (!h) return set_err(GB_ERR_NO_MEMORY, "host allocation failed");
  gb::Moe& m = h->m;
  m.desc = *desc;
  m.device = desc->device;
  m.ep_size = std::max(1, desc->ep_size);
  m.ep_rank = m.ep_size > 1 ? desc->ep_rank : 0;
  const int per = desc->n_experts / m.ep_size;
  m.e_begin = m.ep_rank * per;
  m.e_end = m.e_begin + per;
  cudaError_t ce = cudaDeviceGetAttribute(&m.sm_count, cudaDevAttrMultiProcessorCount, m.device);
  if (ce != cudaSuccess) {
    delete h;
    return cuda_err(ce, "query SM count");
  }
  if (m.ep_size > 1) rc = gb::ep_init(m, desc->nccl_id);
  if (!rc) rc = upload_weights(m);
  if (!rc && desc->act_kind == GB_ACT_GPTOSS_CLAMP && desc->hidden % 64 == 0 &&
      desc->inter % 64 == 0 && desc->hidden <= 3072 && desc->inter <= 3072) {
    ce = gb::tc_prepare_weights(m);
    if (ce != cudaSuccess) rc = cuda_err(ce, "row exponents for the tensor-core path");
  }
  if (!rc && gb::dense_tc_supported(m)) {
    ce = gb::dense_tc_prepare(m);
    if (ce != cudaSuccess) rc = cuda_err(ce, "TMA descriptors of the dense expert weights");
  }
  if (!rc && desc->weight_format == GB_FMT_Q4_K) {
    ce = gb::q4k_tc_prepare(m);
    if (ce != cudaSuccess) rc = cuda_err(ce, "decode exponents for the tensor-core Q4_K path");
  }
  if (!rc && gb::mx_supported(m)) {
    ce = gb::mx_prepare_weights(m);
    if (ce != cudaSuccess) rc = cuda_err(ce, "block-scaled weight layout");
  }
  if (!rc && (desc->weight_format == GB_FMT_MXFP4_SPLIT || desc->weight_format == GB_FMT_MXFP4_GGUF)) {
    ce = gb::fused_decode_prepare(m);
    if (ce != cudaSuccess) rc = cuda_err(ce, "fused decode kernel set-up");
  }
  if (!rc) rc = alloc_ws(m, std::max(1, desc->max_tokens));
  if (rc) {
    const std::string msg = g_err;  // release must not overwrite the cause
    release_moe(h->m);
    delete h;
    snprintf(g_err, sizeof g_err, "%s", msg.c_str());
    return rc;
  }
  *out = h;
  return GB_OK;
}

int gb_moe_forward(gb_moe* h, const float* x_dev, int64_t T, float* out_dev, void* stream) {
  int rc = check_handle(h);
  if (rc) return rc;
  if (T < 0) return set_err(GB_ERR_INVALID_ARG, "T = %lld < 0", (long long)T);
  // With expert parallelism every rank joins the exchanges, even with no tokens.
  if (T == 0 && h->m.ep_size == 1) return GB_OK;
  if (T > 0 && (!x_dev || !out_dev)) return set_err(GB_ERR_INVALID_ARG, "x or out is null");
  if (T > 0 && ((reinterpret_cast<uintptr_t>(x_dev) | reinterpret_cast<uintptr_t>(out_dev)) & 15))
    return set_err(GB_ERR_INVALID_ARG, "x and out must be 16-byte aligned");
  if (T > (int64_t)1 << 24) return set_err(GB_ERR_UNSUPPORTED, "T = %lld too large", (long long)T);
  gb::Moe& m = h->m;
  DeviceScope ds(m.device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((rc = ensure_ws(m, T, st))) return rc;
  return forward_dispatch(m, x_dev, T, out_dev, st);
}

}  // extern "C"

namespace {

// Host buffers of at least 2 kHostChunkMin tokens go through in chunks:
// chunk i's copy in (h2d stream) overlaps the forward of chunk i - 1 and its
// copy out (d2h stream) the forward of chunk i + 1.  The first and last
// chunks hold kHostChunkMin tokens (their copies are the ones nothing
// hides); the rest is split into up to kHostChunks - 2 equal middle chunks
// of about kHostChunkMid tokens, whose copies in take about as long as the
// forward before them.  Every chunk holds at least kHostChunkMin tokens.
// The forward of a chunk is the forward of those tokens (routing and
// experts are per token; the expert tiles follow the chunk's rows per
// expert, which at GPT-OSS shapes keeps the one accumulation order of the
// 30- and 60-position tiles).  Expert-parallel ranks chunk by the largest
// batch of any rank, so that all make the same number of forwards.
constexpr int64_t kHostChunkMin = 1024;
constexpr int64_t kHostChunkMid = 3072;
constexpr int kHostChunks = gb::kHostChunksMax;

// Chunk boundaries of a batch of T >= 2 kHostChunkMin tokens; returns the
// chunk count.
int host_chunks(int64_t T, int64_t (&bound)[kHostChunks + 1]) {
  const int64_t rest = T - 2 * kHostChunkMin;
  if (rest < kHostChunkMin) {  // two halves
    bound[0] = 0;
    bound[1] = T / 2;
    bound[2] = T;
    return 2;
  }
  const int nmid = (int)std::min<int64_t>(kHostChunks - 2,
                                          (rest + kHostChunkMid - 1) / kHostChunkMid);
  bound[0] = 0;
  for (int i = 0; i <= nmid; ++i) bound[1 + i] = kHostChunkMin + rest * i / nmid;
  bound[nmid + 2] = T;
  return nmid + 2;
}

// The chunked host-buffer forward over chunks [bound[i], bound[i + 1]).
int forward_host_pipelined(gb::Moe& m, const float* x_host, float* out_host, cudaStream_t st,
                           const int64_t* bound, int n) {
  const int64_t H = m.desc.hidden;
  if (!m.h2d) GB_CUDA(cudaStreamCreateWithFlags(&m.h2d, cudaStreamNonBlocking), "copy stream");
  if (!m.d2h) GB_CUDA(cudaStreamCreateWithFlags(&m.d2h, cudaStreamNonBlocking), "copy stream");
  for (auto& e : m.host_ev)
    if (!e) GB_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "chunk event");
  cudaEvent_t start = m.host_ev[0], done = m.host_ev[1];
  cudaEvent_t* in = m.host_ev + 2;                 // [kHostChunks]
  cudaEvent_t* fwd = m.host_ev + 2 + kHostChunks;  // [kHostChunks]
  // the staging buffers may still be in use by work queued earlier on st
  GB_CUDA(cudaEventRecord(start, st), "record chunk event");
  GB_CUDA(cudaStreamWaitEvent(m.h2d, start, 0), "order copy stream");
  GB_CUDA(cudaStreamWaitEvent(m.d2h, start, 0), "order copy stream");
  for (int i = 0; i < n; ++i) {
    const int64_t t0 = bound[i], tn = bound[i + 1] - bound[i];
    GB_CUDA(cudaMemcpyAsync(m.ws.x_stage + t0 * H, x_host + t0 * H, sizeof(float) * tn * H,
                            cudaMemcpyHostToDevice, m.h2d),
            "copy x in");
    GB_CUDA(cudaEventRecord(in[i], m.h2d), "record chunk event");
  }
  int rc;
  for (int i = 0; i < n; ++i) {
    const int64_t t0 = bound[i], tn = bound[i + 1] - bound[i];
    GB_CUDA(cudaStreamWaitEvent(st, in[i], 0), "wait for chunk in");
    if ((rc = run_forward(m, m.ws.x_stage + t0 * H, tn, m.ws.out_stage + t0 * H, st))) return rc;
    GB_CUDA(cudaEventRecord(fwd[i], st), "record chunk event");
    GB_CUDA(cudaStreamWaitEvent(m.d2h, fwd[i], 0), "wait for chunk forward");
    GB_CUDA(cudaMemcpyAsync(out_host + t0 * H, m.ws.out_stage + t0 * H, sizeof(float) * tn * H,
                            cudaMemcpyDeviceToHost, m.d2h),
            "copy out");
  }
  GB_CUDA(cudaEventRecord(done, m.d2h), "record chunk event");
  GB_CUDA(cudaStreamWaitEvent(st, done, 0), "wait for copies out");
  return GB_OK;
}

}  // namespace

extern "C" {

int gb_moe_forward_host(gb_moe* h, const float* x_host, int64_t T, float* out_host,
                        void* stream) {
  int rc = check_handle(h);
  if (rc) return rc;
  if (T < 0) return set_err(GB_ERR_INVALID_ARG, "T = %lld < 0", (long long)T);
  if (T == 0 && h->m.ep_size == 1) return GB_OK;
  if (T > 0 && (!x_host || !out_host)) return set_err(GB_ERR_INVALID_ARG, "x or out is null");
  gb::Moe& m = h->m;
  DeviceScope ds(m.device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((rc = ensure_ws(m, T, st))) return rc;
  // Expert parallel: every rank must run the same number of forwards, so
  // the ranks first agree on the largest batch and all chunk like it (each
  // rank's chunks in proportion to its own T).
  int64_t t_chunks = T;
  if (m.ep_size > 1 && (rc = gb::ep_agree_max(m, T, &t_chunks, st))) return rc;
  if (t_chunks >= 2 * kHostChunkMin) {
    int64_t bound[kHostChunks + 1];
    const int n = host_chunks(t_chunks, bound);
    for (int i = 0; i <= n; ++i) bound[i] = bound[i] * T / t_chunks;
    if ((rc = forward_host_pipelined(m, x_host, out_host, st, bound, n))) return rc;
  } else {
    const size_t bytes = sizeof(float) * (size_t)(T * m.desc.hidden);
    if (bytes)
      GB_CUDA(cudaMemcpyAsync(m.ws.x_stage, x_host, bytes, cudaMemcpyHostToDevice, st),
              "copy x in");
    if ((rc = forward_dispatch(m, m.ws.x_stage, T, m.ws.out_stage, st))) return rc;
    if (bytes)
      GB_CUDA(cudaMemcpyAsync(out_host, m.ws.out_stage, bytes, cudaMemcpyDeviceToHost, st),
              "copy out");
  }
  GB_CUDA(cudaStreamSynchronize(st), "synchronise forward");
  return read_device_status(m, st);
}

int gb_moe_route(gb_moe* h, const float* x_dev, int64_t T, int32_t* idx_dev, float* w_dev,
                 int32_t* counts_dev, int32_t* offsets_dev, int32_t* perm_dev, void* stream) {
  int rc = check_handle(h);
  if (rc) return rc;
  if (T < 0) return set_err(GB_ERR_INVALID_ARG, "T = %lld < 0", (long long)T);
  if (T > 0 && !x_dev) return set_err(GB_ERR_INVALID_ARG, "x is null");
  if (T > 0 && (reinterpret_cast<uintptr_t>(x_dev) & 15))
    return set_err(GB_ERR_INVALID_ARG, "x must be 16-byte aligned");
  gb::Moe& m = h->m;
  DeviceScope ds(m.device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((rc = ensure_ws(m, T, st))) return rc;
  const int64_t E = m.desc.n_experts, K = m.desc.top_k;
  if (T > 0 && (rc = run_route(m, x_dev, T, st))) return rc;
  if (T == 0) {
    GB_CUDA(cudaMemsetAsync(m.ws.counts, 0, sizeof(int32_t) * E, st), "clear counts");
    GB_CUDA(cudaMemsetAsync(m.ws.offsets, 0, sizeof(int32_t) * (E + 1), st), "clear offsets");
  }
  auto cp = [&](void* dst, const void* src, size_t bytes) -> int {
    if (!dst || bytes == 0) return GB_OK;
    GB_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, st), "copy routing out");
    return GB_OK;
  };
  if ((rc = cp(idx_dev, m.ws.idx, sizeof(int32_t) * (size_t)(T * K)))) return rc;
  if ((rc = cp(w_dev, m.ws.wts, sizeof(float) * (size_t)(T * K)))) return rc;
  if ((rc = cp(counts_dev, m.ws.counts, sizeof(int32_t) * (size_t)E))) return rc;
  if ((rc = cp(offsets_dev, m.ws.offsets, sizeof(int32_t) * (size_t)(E + 1)))) return rc;
  if ((rc = cp(perm_dev, m.ws.perm, sizeof(int32_t) * (size_t)(T * K)))) return rc;
  GB_CUDA(cudaStreamSynchronize(st), "synchronise route");
  return GB_OK;
}

int gb_moe_dequant_expert(gb_moe* h, int32_t which, int32_t expert, float* out_dev,
                          void* stream) {
  int rc = check_handle(h);
  if (rc) return rc;
  gb::Moe& m = h->m;
  if (which < 0 || which > 2) return set_err(GB_ERR_INVALID_ARG, "which = %d not in 0..2", which);
  if (expert < m.e_begin || expert >= m.e_end)
    return set_err(GB_ERR_INVALID_ARG, "expert %d is not local ([%d, %d))", expert, m.e_begin,
                   m.e_end);
  if (!out_dev) return set_err(GB_ERR_INVALID_ARG, "out is null");
  DeviceScope ds(m.device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (m.desc.weight_format == GB_FMT_Q4_K)
    GB_CUDA(gb::launch_q4k_dequant(m, which, expert - m.e_begin, out_dev, st), "dequant launch");
  else if (m.desc.weight_format == GB_FMT_DENSE)
    GB_CUDA(gb::launch_dense_dequant(m, which, expert - m.e_begin, out_dev, st), "dequant launch");
  else
    GB_CUDA(gb::launch_dequant_expert(m, which, expert - m.e_begin, out_dev, st), "dequant launch");
  GB_CUDA(cudaStreamSynchronize(st), "synchronise dequant");
  return GB_OK;
}

int gb_moe_device_status(gb_moe* h, void* stream) {
  int rc = check_handle(h);
  if (rc) return rc;
  DeviceScope ds(h->m.device);
  return read_device_status(h->m, static_cast<cudaStream_t>(stream));
}

int gb_moe_get_info(const gb_moe* h, gb_moe_info* info) {
  if (!h || !info) return set_err(GB_ERR_INVALID_ARG, "null argument");
  if (info->struct_size < sizeof(gb_moe_info))
    return set_err(GB_ERR_INVALID_ARG, "info struct_size %u < %zu", info->struct_size,
                   sizeof(gb_moe_info));
  const gb::Moe& m = h->m;
  info->local_expert_begin = m.e_begin;
  info->local_expert_end = m.e_end;
  info->weight_bytes = m.weight_bytes;
  info->workspace_bytes = (int64_t)m.ws.bytes;
  info->workspace_tokens = (int32_t)m.ws.tokens;
  info->sm_count = m.sm_count;
  info->kernel_launches = m.launches;
  info->graph_captures = m.graph_captures;
  return GB_OK;
}

static const char* kStageNames[gb::Moe::kStages] = {"router", "permute", "gate_up", "down",
                                                     "combine"};

const char* gb_moe_stage_name(int32_t stage) {
  return stage >= 0 && stage < gb::Moe::kStages ? kStageNames[stage] : "";
}

int gb_moe_set_profiling(gb_moe* h, int enable) {
  int rc = check_handle(h);
  if (rc) return rc;
  gb::Moe& m = h->m;
  DeviceScope ds(m.device);
  if (enable && !m.ev[0])
    for (auto& e : m.ev) GB_CUDA(cudaEventCreate(&e), "create stage event");
  m.profiling = enable != 0;
  m.profiled_once = false;
  return GB_OK;
}

int gb_moe_stage_times(gb_moe* h, float* ms_out, int32_t capacity, int32_t* n_stages) {
  int rc = check_handle(h);
  if (rc) return rc;
  gb::Moe& m = h->m;
  if (!m.profiled_once)
    return set_err(GB_ERR_INVALID_ARG, "no profiled forward yet (call gb_moe_set_profiling)");
  DeviceScope ds(m.device);
  GB_CUDA(cudaEventSynchronize(m.ev[gb::Moe::kStages]), "wait for the profiled forward");
  const int n = std::min<int>(gb::Moe::kStages, std::max<int32_t>(capacity, 0));
  for (int i = 0; i < n && ms_out; ++i)
    GB_CUDA(cudaEventElapsedTime(&ms_out[i], m.ev[i], m.ev[i + 1]), "stage elapsed time");
  if (n_stages) *n_stages = gb::Moe::kStages;
  return GB_OK;
}

int gb_moe_destroy(gb_moe* h) {
  if (!h) return GB_OK;
  release_moe(h->m);
  delete h;
  return GB_OK;
}

int gb_moe_set_expert_path(gb_moe* h, int32_t path) {
  int rc = check_handle(h);
  if (rc) return rc;
  if (path < GB_PATH_AUTO || path > GB_PATH_FUSED_DECODE)
    return set_err(GB_ERR_INVALID_ARG, "unknown expert path %d", path);
  if ((path == GB_PATH_TENSOR_CORES || path == GB_PATH_TENSOR_CORES_F16) &&
      !gb::tc_supported(h->m) && !h->m.mx.ok && !gb::q4k_tc_supported(h->m) &&
      !gb::dense_tc_supported(h->m))
    return set_err(GB_ERR_UNSUPPORTED,
                   "tensor-core expert path needs H, I multiples of 64 (and bf16 weights for "
                   "dense experts)");
  DeviceScope ds(h->m.device);
  clear_graphs(h->m);
  h->m.expert_path = path;
  return GB_OK;
}

int gb_moe_set_test_hooks(gb_moe* h, int64_t wait_limit_us, int32_t withhold_ready) {
  int rc = check_handle(h);
  if (rc) return rc;
  if (wait_limit_us < 0 || wait_limit_us > 10000000)
    return set_err(GB_ERR_INVALID_ARG, "wait_limit_us %lld outside [0, 1e7]",
                   (long long)wait_limit_us);
  DeviceScope ds(h->m.device);
  clear_graphs(h->m);
  h->m.test_wait_ns = (uint64_t)wait_limit_us * 1000ull;
  h->m.test_withhold_ready = withhold_ready != 0;
  return GB_OK;
}

int gb_moe_set_graphs(gb_moe* h, int32_t max_graphs) {
  int rc = check_handle(h);
  if (rc) return rc;
  if (max_graphs < 0 || max_graphs > gb::Moe::kGraphSlots)
    return set_err(GB_ERR_INVALID_ARG, "max_graphs %d outside [0, %d]", max_graphs,
                   gb::Moe::kGraphSlots);
  DeviceScope ds(h->m.device);
  clear_graphs(h->m);
  h->m.graph_slots = max_graphs;
  return GB_OK;
}

int gb_nccl_unique_id(uint8_t out[128]) {
  if (!out) return set_err(GB_ERR_INVALID_ARG, "out is null");
  return gb::nccl_unique_id(out);
}

}  // extern "C"
