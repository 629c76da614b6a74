"""The GPT-OSS decode stack around the MoE block, restated in numpy f32.

TEST INFRASTRUCTURE ONLY: imported by tests/ as the checker of the library's
decoder (gb_decoder_*).  The product path never imports it.

It follows the GGUF model of crates/gallium-models/src/gpt_oss_q.rs:
  forward (:437-472): embeddings, per layer the block (:270-297), final
    RMSNorm, LM head on each sequence's last token;
  block: RMSNorm -> attention (:57-107) -> + x -> RMSNorm -> MoE (the C
    oracle's GGUF QMoEFFN, :165-269) -> + residual;
  attention: q/k/v projections with biases (QLinear, quantized.rs:849-882:
    x W^T, then + bias), RoPE on q and k (pos_enc.rs), K/V appended to the
    cache (kv_cache.rs:21-47), scores (q k^T) * (1/sqrt(hd)) by query-head
    groups (gqa.rs:40-72), the causal or sliding-window mask (mask.rs:5-48),
    the head's sink logit appended as one more column, softmax, the sink
    column dropped, the weighted sum of V, the o projection;
  RMSNorm: candle_nn::ops::rms_norm, x / sqrt(sum(x^2) / n + eps) * w with
    the sum taken in order in f32;
  greedy token: the largest logit, ties to the highest id (sampling.rs:85-92
    takes Iterator::max_by, which keeps the last of equal maxima).
RoPE tables as pos_enc.rs:82-176 builds them: inverse frequencies in f64
(YaRN-adjusted when the factor is above 1, :113-137), rounded to f32; each
angle the f32 product position x frequency; its cos and sin in f32 through
the C library's cosf / sinf, as Rust's f32::cos calls them on Linux.  RoPE
itself is candle's halves layout (candle_nn::rotary_emb::rope): x1' = x1 cos
- x2 sin, x2' = x1 sin + x2 cos, each product rounded to f32.
"""
from __future__ import annotations

import ctypes
import ctypes.util
import math

import numpy as np

from . import OracleMoe

_libm = ctypes.CDLL(ctypes.util.find_library("m") or "libm.so.6")
_libm.cosf.restype = ctypes.c_float
_libm.cosf.argtypes = [ctypes.c_float]
_libm.sinf.restype = ctypes.c_float
_libm.sinf.argtypes = [ctypes.c_float]


def bf16(a: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(a, np.uint16).astype(np.uint32) << 16).view(np.float32)


def rope_inv_freq(head_dim: int, theta: float, factor: float = 1.0, orig_ctx: int = 4096,
                  beta_fast: float = 32.0, beta_slow: float = 1.0) -> np.ndarray:
    """Inverse frequencies of pos_enc.rs:82-137 (f64, YaRN when factor > 1)."""
    rot, half = head_dim, head_dim // 2
    inv = [1.0 / theta ** (2.0 * i / rot) for i in range(half)]
    if factor > 1.0:
        low = math.floor(orig_ctx / (beta_fast * 2.0 * math.pi))
        high = math.floor(orig_ctx / (beta_slow * 2.0 * math.pi))
        for i in range(half):
            ratio = (2.0 * math.pi / inv[i]) / orig_ctx
            if ratio < low / rot:
                pass
            elif ratio > high / rot:
                inv[i] /= factor
            else:
                t = (i - low) / (high - low)
                inv[i] *= 1.0 / (1.0 + (factor - 1.0) * t)
    return np.array(inv, np.float64)


def rope_tables(head_dim: int, n_pos: int, theta: float, factor: float = 1.0,
                orig_ctx: int = 4096):
    inv32 = rope_inv_freq(head_dim, theta, factor, orig_ctx).astype(np.float32)
    pos = np.arange(n_pos, dtype=np.float32)
    ang = (pos[:, None] * inv32[None, :]).astype(np.float32)  # one f32 product each
    cos = np.array([_libm.cosf(float(a)) for a in ang.ravel()], np.float32).reshape(ang.shape)
    sin = np.array([_libm.sinf(float(a)) for a in ang.ravel()], np.float32).reshape(ang.shape)
    return cos, sin


def rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """x (..., T, hd) rotated by cos / sin (T, hd/2), halves layout."""
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    return np.concatenate([x1 * cos - x2 * sin, x1 * sin + x2 * cos], axis=-1).astype(np.float32)


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """Rows of x: x / sqrt(sum(x^2) / n + eps) * w, the sum in order in f32."""
    x = np.asarray(x, np.float32)
    ss = np.cumsum(x * x, axis=-1, dtype=np.float32)[..., -1:]
    m = np.sqrt(ss / np.float32(x.shape[-1]) + np.float32(eps)).astype(np.float32)
    return ((x / m) * w).astype(np.float32)


def visible(q_pos: int, n_keys: int, sliding: bool, window: int) -> np.ndarray:
    """Keys 0 .. n_keys - 1 a query at q_pos may attend to (mask.rs:5-48):
    not in the future, and on sliding layers not more than window - 1
    positions back."""
    j = np.arange(n_keys)
    ok = j <= q_pos
    if sliding and q_pos >= window:
        ok &= j >= q_pos - window + 1
    return ok


def greedy(logits: np.ndarray) -> np.ndarray:
    """Per row: the index of the largest logit, the last of equal maxima."""
    logits = np.asarray(logits, np.float32)
    rev = logits[:, ::-1]
    return (logits.shape[1] - 1 - np.argmax(rev, axis=1)).astype(np.int32)


class OracleDecoder:
    """The decode stack of a synth.GptOssDecoderWeights, with its KV cache."""

    def __init__(self, weights, max_seq_len: int = 512):
        self.w = weights
        self.moe = [OracleMoe(L.moe.base, gguf=L.moe) for L in weights.layers]
        self.cos, self.sin = rope_tables(weights.head_dim, max_seq_len, weights.rope_theta,
                                         weights.rope_scaling_factor, weights.rope_orig_ctx)
        self.embed = bf16(weights.embed)
        self.lm_head = bf16(weights.lm_head if weights.lm_head is not None else weights.embed)
        self.lw = [dict(wq=bf16(L.wq), wk=bf16(L.wk), wv=bf16(L.wv), wo=bf16(L.wo))
                   for L in weights.layers]
        self.reset()

    def reset(self) -> None:
        self.k = [None] * self.w.n_layers  # (B, nkv, S, hd)
        self.v = [None] * self.w.n_layers
        self.pos = 0

    @staticmethod
    def _linear(x, W, b):
        y = (x @ W.T).astype(np.float32)
        return y if b is None else (y + b).astype(np.float32)

    def _attention(self, l, x, pos):
        w, L, P = self.w, self.w.layers[l], self.lw[l]
        B, T, _ = x.shape
        nh, nkv, hd = w.n_heads, w.n_kv_heads, w.head_dim
        q = self._linear(x, P["wq"], L.bq).reshape(B, T, nh, hd).transpose(0, 2, 1, 3)
        k = self._linear(x, P["wk"], L.bk).reshape(B, T, nkv, hd).transpose(0, 2, 1, 3)
        v = self._linear(x, P["wv"], L.bv).reshape(B, T, nkv, hd).transpose(0, 2, 1, 3)
        cos, sin = self.cos[pos:pos + T], self.sin[pos:pos + T]
        q, k = rope(q, cos, sin), rope(k, cos, sin)
        self.k[l] = k if self.k[l] is None else np.concatenate([self.k[l], k], axis=2)
        self.v[l] = v if self.v[l] is None else np.concatenate([self.v[l], v], axis=2)
        K, V = self.k[l], self.v[l]
        n = K.shape[2]
        rep = nh // nkv
        scale = np.float32(1.0 / math.sqrt(hd))
        out = np.empty((B, T, nh * hd), np.float32)
        for b in range(B):
            for h in range(nh):
                g = h // rep
                s = ((q[b, h] @ K[b, g].T).astype(np.float32) * scale).astype(np.float32)
                for t in range(T):
                    ok = visible(pos + t, n, bool(L.sliding), w.sliding_window)
                    row = np.where(ok, s[t], np.float32(-np.inf)).astype(np.float32)
                    row = np.concatenate([row, np.float32([L.sinks[h]])])
                    e = np.exp(row - row.max()).astype(np.float32)
                    p = (e / e.sum(dtype=np.float32)).astype(np.float32)[:n]
                    out[b, t, h * hd:(h + 1) * hd] = (p @ V[b, g]).astype(np.float32)
        return self._linear(out, P["wo"], L.bo)

    def forward(self, tokens: np.ndarray, pos: int) -> np.ndarray:
        """tokens (B, T) at positions pos ..; returns the (B, vocab) logits
        of each sequence's last token."""
        assert pos == self.pos
        w = self.w
        tokens = np.asarray(tokens, np.int64)
        B, T = tokens.shape
        h = self.embed[tokens]
        for l, L in enumerate(w.layers):
            a = self._attention(l, rms_norm(h, L.attn_norm, w.rms_eps), pos)
            h = (a + h).astype(np.float32)
            xn = rms_norm(h, L.post_attn_norm, w.rms_eps)
            y, _, _ = self.moe[l].forward(xn.reshape(B * T, -1))
            h = (y.reshape(B, T, -1) + h).astype(np.float32)
        last = rms_norm(h[:, -1], w.final_norm, w.rms_eps)
        self.pos = pos + T
        return (last @ self.lm_head.T).astype(np.float32)

    def generate(self, tokens: np.ndarray, pos: int, n_steps: int):
        """n_steps greedy steps from tokens (B,) at pos; returns the (n_steps, B)
        tokens and the (n_steps, B, vocab) logits each step produced."""
        toks, logits = [], []
        cur = np.asarray(tokens, np.int64).reshape(-1, 1)
        for i in range(n_steps):
            lg = self.forward(cur, pos + i)
            nxt = greedy(lg)
            toks.append(nxt)
            logits.append(lg)
            cur = nxt.reshape(-1, 1).astype(np.int64)
        return np.stack(toks), np.stack(logits)
