"""Seeded synthetic MoE layers and inputs (no checkpoints are available).

Shapes and value distributions follow the workloads this path is measured on:

* GPT-OSS-shaped block: hidden 2880, intermediate 2880, top-4, E = 32 (20B
  shape) or 128 (120B shape).  Router weight bf16 ~ N(0, 0.02), bias 0.
  Expert weights MXFP4 in the safetensors layout: E2M1 nibbles uniform over
  the 16 codes, one E8M0 scale per 32 elements uniform over exponents
  -8..-2 (bytes 119..125).  Expert biases bf16 ~ N(0, 0.01).
  Activation: clamped SwiGLU, limit 7.
* Skewed routing: router bias_e = 2 * ln(p_e), p_e proportional to
  (e + 1)^-1.2 (Zipf, s = 1.2), so a few experts take most tokens.
* x ~ N(0, 1) f32.

Everything is generated with numpy's PCG64 from an explicit seed, so the
same call gives the same bytes on every machine.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import numpy as np


def f32_to_bf16_bits(a) -> np.ndarray:
    """Round f32 to bf16 (nearest, ties to even); returns the uint16 bits."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u >> 16) & 1) + 0x7FFF
    return ((u + r) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


@dataclass
class GptOssLayer:
    """One GPT-OSS MoE block in the safetensors MXFP4 layout (gpt_oss.rs:96-142)."""
    hidden: int
    inter: int
    n_experts: int
    top_k: int
    swiglu_limit: float
    router_w: np.ndarray        # [E, H] bf16 bits (uint16)
    router_b: np.ndarray        # [E] bf16 bits
    gu_blocks: np.ndarray       # [E, 2I, H/32, 16] uint8
    gu_scales: np.ndarray       # [E, 2I, H/32] uint8
    gu_bias: np.ndarray         # [E, 2I] bf16 bits
    dn_blocks: np.ndarray       # [E, H, I/32, 16] uint8
    dn_scales: np.ndarray       # [E, H, I/32] uint8
    dn_bias: np.ndarray         # [E, H] bf16 bits
    meta: dict = field(default_factory=dict)

    @property
    def expert_bytes(self) -> int:
        """MXFP4 bytes of one expert (nibbles + scales), 13,219,200 at 2880/2880."""
        H, I = self.hidden, self.inter
        return (2 * I * H + H * I) // 2 + (2 * I * H + H * I) // 32

    @property
    def expert_bias_bytes(self) -> int:
        return 2 * (2 * self.inter + self.hidden)  # bf16


def zipf_router_bias(n_experts: int, s: float = 1.2) -> np.ndarray:
    p = (np.arange(n_experts, dtype=np.float64) + 1.0) ** (-s)
    p /= p.sum()
    return (2.0 * np.log(p)).astype(np.float32)


def _uniform_bytes(rng, shape) -> np.ndarray:
    """Bytes uniform over 0..255 (so both nibbles are uniform over the 16
    E2M1 codes), writable, in the given shape."""
    n = int(np.prod(shape))
    words = rng.bit_generator.random_raw((n + 7) // 8)  # uint64, fresh and writable
    return words.view(np.uint8)[:n].reshape(shape)


def gptoss_layer(n_experts: int = 32, hidden: int = 2880, inter: int = 2880, top_k: int = 4,
                 seed: int = 0, skewed: bool = False, scale_lo: int = 119,
                 scale_hi: int = 125) -> GptOssLayer:
    rng = np.random.default_rng(seed)
    E, H, I = n_experts, hidden, inter
    router_w = f32_to_bf16_bits(rng.normal(0.0, 0.02, (E, H)).astype(np.float32))
    rb = zipf_router_bias(E) if skewed else np.zeros(E, np.float32)
    router_b = f32_to_bf16_bits(rb)
    gu_blocks = _uniform_bytes(rng, (E, 2 * I, H // 32, 16))
    gu_scales = rng.integers(scale_lo, scale_hi + 1, (E, 2 * I, H // 32), dtype=np.uint8)
    gu_bias = f32_to_bf16_bits(rng.normal(0.0, 0.01, (E, 2 * I)).astype(np.float32))
    dn_blocks = _uniform_bytes(rng, (E, H, I // 32, 16))
    dn_scales = rng.integers(scale_lo, scale_hi + 1, (E, H, I // 32), dtype=np.uint8)
    dn_bias = f32_to_bf16_bits(rng.normal(0.0, 0.01, (E, H)).astype(np.float32))
    return GptOssLayer(H, I, E, top_k, 7.0, router_w, router_b, gu_blocks, gu_scales, gu_bias,
                       dn_blocks, dn_scales, dn_bias,
                       meta={"seed": seed, "skewed": skewed})


def tokens(T: int, hidden: int, seed: int = 0) -> np.ndarray:
    """x ~ N(0, 1), f32 [T, hidden]; seed 0 stream is independent of the weights'."""
    rng = np.random.default_rng([seed, 0x5EED])
    return rng.standard_normal((T, hidden), dtype=np.float32)


# ---- GGUF MXFP4 (type 39) views of a safetensors layer ---------------------

def split_to_gguf_blocks(blocks: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """Safetensors blocks [..., nb, 16] + scales [..., nb] -> GGUF 17-byte
    blocks [..., nb * 17] holding the same values (quantized.rs:386-392: low
    nibble of byte j = element j, high nibble = element j + 16; the E8M0 byte
    means the same power of two for bytes >= 1 because the GGUF LUT is the
    E2M1 table doubled and its scale is halved)."""
    lo = blocks & 0x0F
    hi = blocks >> 4
    el = np.empty(blocks.shape[:-1] + (32,), np.uint8)
    el[..., 0::2] = lo
    el[..., 1::2] = hi
    qs = (el[..., :16] | (el[..., 16:] << 4)).astype(np.uint8)
    out = np.concatenate([scales[..., None].astype(np.uint8), qs], axis=-1)
    return np.ascontiguousarray(out.reshape(blocks.shape[:-2] + (blocks.shape[-2] * 17,)))


@dataclass
class GptOssGgufLayer:
    """The same layer as GGUF tensors: separate gate/up [E, I, H] and down
    [E, H, I] (gpt_oss_q.rs:110-163)."""
    base: GptOssLayer
    gate_raw: np.ndarray
    up_raw: np.ndarray
    down_raw: np.ndarray
    gate_bias: np.ndarray  # bf16 bits [E, I]
    up_bias: np.ndarray
    down_bias: np.ndarray


def gptoss_gguf_from_split(layer: GptOssLayer) -> GptOssGgufLayer:
    g = split_to_gguf_blocks(layer.gu_blocks[:, 0::2], layer.gu_scales[:, 0::2])
    u = split_to_gguf_blocks(layer.gu_blocks[:, 1::2], layer.gu_scales[:, 1::2])
    d = split_to_gguf_blocks(layer.dn_blocks, layer.dn_scales)
    return GptOssGgufLayer(layer, g, u, d, np.ascontiguousarray(layer.gu_bias[:, 0::2]),
                           np.ascontiguousarray(layer.gu_bias[:, 1::2]), layer.dn_bias)


def algorithmic_bytes(layer: GptOssLayer, T: int, n_touched: int) -> int:
    """Bytes one forward must move at minimum: touched experts' MXFP4 weights
    and biases, the router weight and bias, x in and out (f32), and the
    routing indices and weights."""
    E, H = layer.n_experts, layer.hidden
    return (n_touched * (layer.expert_bytes + layer.expert_bias_bytes) + E * H * 2 + E * 2
            + 2 * T * H * 4 + T * layer.top_k * 8)


def algorithmic_flops(layer: GptOssLayer, T: int) -> int:
    """Expert GEMM FLOPs (2 * (2I*H + H*I) per token-expert) plus the router."""
    H, I, E, k = layer.hidden, layer.inter, layer.n_experts, layer.top_k
    return T * k * 6 * H * I + 2 * T * H * E


# ---- LFM2.5 MoE block with GGML Q4_K experts ---------------------------------

@dataclass
class Lfm2Layer:
    """LFM2.5-shaped MoE block (lfm2moe_q.rs:203-313): sigmoid router with a
    selection-only bias, SiLU-gated experts without biases, Q4_K weights as
    GGUF tensors gate/up [E, I, H] and down [E, H, I] (144-byte super-blocks)."""
    hidden: int
    inter: int
    n_experts: int
    top_k: int
    router_w: np.ndarray   # [E, H] f32
    sel_bias: np.ndarray   # [E] f32 (exp_probs_b)
    gate_raw: np.ndarray   # [E, I, H/256 * 144] uint8
    up_raw: np.ndarray
    down_raw: np.ndarray   # [E, H, I/256 * 144] uint8
    meta: dict = field(default_factory=dict)

    @property
    def expert_bytes(self) -> int:
        """Q4_K bytes of one expert: 0.5625 bytes per element, 6,193,152 at 2048/1792."""
        return (2 * self.inter * self.hidden + self.hidden * self.inter) // 256 * 144


def q4k_blocks(rng, rows: int, k: int, d: float, dmin: float) -> np.ndarray:
    """rows x (k/256) Q4_K super-blocks: the given f16 d and dmin, uniform 6-bit
    scales and mins (every bit of the 12 packed bytes is used once, so uniform
    bytes give uniform 6-bit values) and uniform 4-bit codes."""
    nb = k // 256
    blk = rng.integers(0, 256, (rows, nb, 144), dtype=np.uint8)
    blk[..., 0:2] = np.frombuffer(np.float16(d).tobytes(), np.uint8)
    blk[..., 2:4] = np.frombuffer(np.float16(dmin).tobytes(), np.uint8)
    return np.ascontiguousarray(blk.reshape(rows, nb * 144))


def lfm2_layer(n_experts: int = 32, hidden: int = 2048, inter: int = 1792, top_k: int = 4,
               seed: int = 0, d: float = 2.0 ** -11, dmin: float = 15 * 2.0 ** -12) -> Lfm2Layer:
    """Default d = 2^-11 and dmin = 7.5 d.  With scales, mins and codes uniform,
    E[d*sc*q - dmin*m] = 31.5 (7.5 d - dmin) = 0, so the weights are centred
    like a trained Q4_K tensor, with a standard deviation near 0.13 (the
    GPT-OSS blocks' is 0.32).  d = dmin would give every weight a positive
    mean and outputs near 1e5, where no two f32 evaluations agree to 2e-2."""
    rng = np.random.default_rng(seed)
    E, H, I = n_experts, hidden, inter
    router_w = rng.normal(0.0, 0.02, (E, H)).astype(np.float32)
    gate = np.stack([q4k_blocks(rng, I, H, d, dmin) for _ in range(E)])
    up = np.stack([q4k_blocks(rng, I, H, d, dmin) for _ in range(E)])
    down = np.stack([q4k_blocks(rng, H, I, d, dmin) for _ in range(E)])
    return Lfm2Layer(H, I, E, top_k, router_w, np.zeros(E, np.float32), gate, up, down,
                     meta={"seed": seed, "d": d, "dmin": dmin})


# ---- gallium-core MoEFFN (dense experts, ffn.rs:72-166) --------------------

@dataclass
class DenseMoeLayer:
    hidden: int
    inter: int
    n_experts: int
    top_k: int
    router_w: np.ndarray   # [E, H] bf16 bits (uint16) or f32
    gate: np.ndarray       # [E, I, H]
    up: np.ndarray         # [E, I, H]
    down: np.ndarray       # [E, H, I]
    act_kind: int = 1      # gb_act_kind: 1 SiLU, 2 GELU, 3 GELU (tanh), 4 ReLU
    act_clamp: float = 0.0
    shared_inter: int = 0
    sh_gate: Optional[np.ndarray] = None  # [Is, H]
    sh_up: Optional[np.ndarray] = None    # [Is, H]
    sh_down: Optional[np.ndarray] = None  # [H, Is]
    meta: dict = field(default_factory=dict)


def dense_layer(n_experts: int = 128, hidden: int = 2048, inter: int = 768, top_k: int = 8,
                shared_inter: int = 512, act_kind: int = 1, act_clamp: float = 0.0,
                seed: int = 0, bf16: bool = True) -> DenseMoeLayer:
    """A generic MoEFFN layer with random weights: router ~ N(0, 0.02), expert
    and shared weights ~ N(0, 1/sqrt(fan_in)) so gate and up products are
    O(1) for x ~ N(0, 1); bf16 bits (uint16) by default, as a bf16 checkpoint
    holds them, else f32."""
    rng = np.random.default_rng(seed)
    E, H, I = n_experts, hidden, inter
    cast = f32_to_bf16_bits if bf16 else (lambda a: a.astype(np.float32))

    def normal(shape, std):
        return cast(rng.standard_normal(shape, dtype=np.float32) * np.float32(std))

    layer = DenseMoeLayer(H, I, E, top_k, normal((E, H), 0.02), normal((E, I, H), H ** -0.5),
                          normal((E, I, H), H ** -0.5), normal((E, H, I), I ** -0.5),
                          act_kind=act_kind, act_clamp=act_clamp, shared_inter=shared_inter,
                          meta={"seed": seed})
    if shared_inter:
        layer.sh_gate = normal((shared_inter, H), H ** -0.5)
        layer.sh_up = normal((shared_inter, H), H ** -0.5)
        layer.sh_down = normal((H, shared_inter), shared_inter ** -0.5)
    return layer


# ---- Gemma-4 routed experts (gemma4_q.rs:187-330) ---------------------------

@dataclass
class Gemma4MoeLayer:
    hidden: int
    inter: int               # n_ff_exp
    n_experts: int
    top_k: int
    fmt: int                 # gb_weight_format: 1 GGUF MXFP4 or 2 Q4_K
    router_w: np.ndarray     # [E, H] f32 (ffn_gate_inp, dequantised)
    router_scale: np.ndarray  # [H] f32 (ffn_gate_inp.scale)
    expert_norm: np.ndarray  # [H] f32 (pre_ffw_norm_2)
    gate_up_raw: np.ndarray  # [E, 2I, row bytes]: gate rows, then up rows
    down_raw: np.ndarray     # [E, H, row bytes]
    expert_scale: Optional[np.ndarray]  # [E] f32 (ffn_down_exps.scale) or None
    output_norm: np.ndarray  # [H] f32 (post_ffw_norm_2)
    rms_eps: float = 1e-6
    meta: dict = field(default_factory=dict)


def gemma4_layer(n_experts: int = 128, hidden: int = 2816, inter: int = 704, top_k: int = 8,
                 fmt: int = 1, seed: int = 0, expert_scale: bool = True) -> Gemma4MoeLayer:
    """A Gemma-4-26B-A4B-like routed-experts block with random weights (the
    default shape is the 26B-A4B one: hidden 2816, 128 experts, top-8, expert
    intermediate 704).  Experts in GGUF MXFP4 (fmt 1: codes uniform, E8M0
    exponents uniform in [-8, -2]) or Q4_K (fmt 2: H and I multiples of 256).
    Router ~ N(0, 1) (its input is normed to ~ N(0, 1/H)); norm weights and
    the router scale uniform in [0.5, 1.5]; expert scales uniform in
    [0.5, 2]."""
    rng = np.random.default_rng(seed)
    E, H, I = n_experts, hidden, inter
    if fmt == 1:
        def mx(rows, k):
            b = _uniform_bytes(rng, (E, rows, k // 32, 16))
            sc = rng.integers(119, 126, (E, rows, k // 32), dtype=np.uint8)
            return split_to_gguf_blocks(b, sc)
        gu, dn = mx(2 * I, H), mx(H, I)
    else:
        d, dmin = 2.0 ** -11, 15 * 2.0 ** -12
        gu = np.stack([q4k_blocks(rng, 2 * I, H, d, dmin) for _ in range(E)])
        dn = np.stack([q4k_blocks(rng, H, I, d, dmin) for _ in range(E)])
    u = lambda n: rng.uniform(0.5, 1.5, n).astype(np.float32)
    return Gemma4MoeLayer(H, I, E, top_k, fmt, rng.standard_normal((E, H), dtype=np.float32),
                          u(H), u(H), gu, dn,
                          rng.uniform(0.5, 2.0, E).astype(np.float32) if expert_scale else None,
                          u(H), meta={"seed": seed})


# ---- GPT-OSS decode stack (gpt_oss_q.rs:15-107, 270-472) --------------------

@dataclass
class DecoderLayerWeights:
    attn_norm: np.ndarray        # [H] f32
    post_attn_norm: np.ndarray   # [H] f32
    wq: np.ndarray               # [nh * hd, H] bf16 bits
    wk: np.ndarray               # [nkv * hd, H]
    wv: np.ndarray               # [nkv * hd, H]
    wo: np.ndarray               # [H, nh * hd]
    bq: Optional[np.ndarray]     # f32 biases or None
    bk: Optional[np.ndarray]
    bv: Optional[np.ndarray]
    bo: Optional[np.ndarray]
    sinks: np.ndarray            # [nh] f32
    sliding: int                 # 1: sliding-window attention
    moe: GptOssGgufLayer         # the layer's MoE block (GGUF MXFP4, gpt_oss_q.rs:119-269)


@dataclass
class GptOssDecoderWeights:
    hidden: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    vocab: int
    sliding_window: int
    rope_theta: float
    rope_scaling_factor: float
    rope_orig_ctx: int
    rms_eps: float
    embed: np.ndarray            # [vocab, H] bf16 bits
    lm_head: Optional[np.ndarray]  # [vocab, H] bf16 bits, None: tied
    final_norm: np.ndarray       # [H] f32
    layers: list
    meta: dict = field(default_factory=dict)

    @property
    def n_layers(self) -> int:
        return len(self.layers)


def gptoss_decoder(n_layers: int = 24, hidden: int = 2880, n_heads: int = 64,
                   n_kv_heads: int = 8, head_dim: int = 64, vocab: int = 201088,
                   n_experts: int = 32, inter: int = 2880, top_k: int = 4,
                   sliding_window: int = 128, rope_theta: float = 150000.0,
                   rope_scaling_factor: float = 32.0, rope_orig_ctx: int = 4096,
                   rms_eps: float = 1e-5, seed: int = 0,
                   share_experts: bool = False) -> GptOssDecoderWeights:
    """A GPT-OSS-shaped decode stack with random weights (defaults: the
    20B shape).  Attention and LM-head weights bf16 ~ N(0, 1/sqrt(fan_in)),
    biases ~ N(0, 0.01), norm weights 1 + N(0, 0.02), sink logits ~ N(0, 1),
    embeddings ~ N(0, 1); even layers sliding-window, odd layers full
    (gpt_oss_q.rs:360-375).  Each layer's MoE block is the GGUF view of
    gptoss_layer(n_experts, hidden, inter, top_k); share_experts reuses one
    block's host arrays for every layer (each layer still gets its own copy on
    the device)."""
    rng = np.random.default_rng([seed, 0xDEC0])
    H, qn, kn = hidden, n_heads * head_dim, n_kv_heads * head_dim

    def w(shape, fan_in, std=None):
        # in chunks of rows, so the f32 and bf16 temporaries stay small
        out = np.empty(shape, np.uint16)
        scale = np.float32(fan_in ** -0.5 if std is None else std)
        step = max(1, (1 << 22) // shape[1])
        for r0 in range(0, shape[0], step):
            r1 = min(shape[0], r0 + step)
            u = (rng.standard_normal((r1 - r0, shape[1]), dtype=np.float32) * scale).view(
                np.uint32)
            # round to nearest even in 32-bit arithmetic (finite values only)
            out[r0:r1] = ((u + (((u >> 16) & 1) + 0x7FFF)) >> 16).astype(np.uint16)
        return out

    def vec(n, std, mean=0.0):
        return (np.float32(mean) + rng.standard_normal(n, dtype=np.float32) *
                np.float32(std)).astype(np.float32)

    shared = None
    layers = []
    for i in range(n_layers):
        if share_experts and shared is not None:
            moe = shared
        else:
            moe = gptoss_gguf_from_split(gptoss_layer(n_experts=n_experts, hidden=hidden,
                                                      inter=inter, top_k=top_k,
                                                      seed=seed * 1000 + i))
            shared = moe
        layers.append(DecoderLayerWeights(
            attn_norm=vec(H, 0.02, 1.0), post_attn_norm=vec(H, 0.02, 1.0),
            wq=w((qn, H), H), wk=w((kn, H), H), wv=w((kn, H), H), wo=w((H, qn), qn),
            bq=vec(qn, 0.01), bk=vec(kn, 0.01), bv=vec(kn, 0.01), bo=vec(H, 0.01),
            sinks=vec(n_heads, 1.0), sliding=1 if i % 2 == 0 else 0, moe=moe))
    embed = w((vocab, H), H, std=1.0)
    lm_head = w((vocab, H), H)
    return GptOssDecoderWeights(H, n_heads, n_kv_heads, head_dim, vocab, sliding_window,
                                rope_theta, rope_scaling_factor, rope_orig_ctx, rms_eps, embed,
                                lm_head, vec(H, 0.02, 1.0), layers,
                                meta={"seed": seed, "share_experts": share_experts})
