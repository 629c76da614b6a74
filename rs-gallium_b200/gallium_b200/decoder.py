"""Host-side mirror of rs-gallium's GGUF GPT-OSS model over the C ABI.

``GptOssQ`` mirrors crates/gallium-models/src/gpt_oss_q.rs:299-489: ``load``
takes the model's weights (a synth.GptOssDecoderWeights, or the same arrays
read from a checkpoint), ``forward(token_ids, pos)`` returns each sequence's
last-token logits like CausalLM::forward (:437-472), ``reset`` forgets the
cache (:474-476).  ``generate`` runs greedy decode steps on the device (one
replayed CUDA graph per step).  The MoE block of every layer is this
library's gb_moe handle.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np

from . import _lib
from ._lib import DecoderDesc, DecoderLayer, check, load_library
from .moe import _as_f32, _ptr


def _gguf_moe_desc(layer, device: int, max_tokens: int):
    """gb_moe_desc of a GGUF GPT-OSS MoE block (synth.GptOssGgufLayer)."""
    b = layer.base
    d = _lib.MoeDesc()
    d.struct_size = ctypes.sizeof(_lib.MoeDesc)
    d.hidden, d.inter, d.n_experts, d.top_k = b.hidden, b.inter, b.n_experts, b.top_k
    d.router_kind = _lib.GB_ROUTER_SOFTMAX_TOPK
    d.act_kind = _lib.GB_ACT_GPTOSS_CLAMP
    d.weight_format = _lib.GB_FMT_MXFP4_GGUF
    d.swiglu_limit = b.swiglu_limit
    d.device = device
    d.max_tokens = max_tokens
    d.ep_size = 1
    arrs = [None if a is None else np.ascontiguousarray(a) for a in (
        _as_f32(b.router_w), _as_f32(b.router_b), layer.gate_raw, layer.up_raw, layer.down_raw,
        _as_f32(layer.gate_bias), _as_f32(layer.up_bias), _as_f32(layer.down_bias))]
    (d.router_weight, d.router_bias, d.gate_raw, d.up_raw, d.down_raw, d.gate_bias, d.up_bias,
     d.down_bias) = [_ptr(a) for a in arrs]
    d.router_dtype = _lib.GB_DTYPE_F32
    d.bias_dtype = _lib.GB_DTYPE_F32
    return d, arrs


def _f32(a):
    return None if a is None else np.ascontiguousarray(a, np.float32)


def _u16(a):
    return None if a is None else np.ascontiguousarray(a, np.uint16)


class GptOssQ:
    """Owns one gb_decoder handle.  Not re-entrant."""

    def __init__(self, h: ctypes.c_void_p, weights, device: int, max_batch: int,
                 max_tokens: int, max_seq_len: int):
        self._lib = load_library()
        self._h = h
        self.vocab = weights.vocab
        self.hidden = weights.hidden
        self.n_layers = weights.n_layers
        self.device = device
        self.max_batch, self.max_tokens, self.max_seq_len = max_batch, max_tokens, max_seq_len
        self.pos = 0

    @classmethod
    def load(cls, weights, device: int = 0, max_batch: int = 1, max_tokens: int = 128,
             max_seq_len: int = 4096) -> "GptOssQ":
        w = weights
        keep = []
        layers = (DecoderLayer * w.n_layers)()
        moe_descs = []
        for i, L in enumerate(w.layers):
            md, arrs = _gguf_moe_desc(L.moe, device, max_batch * max_tokens)
            keep.append(arrs)
            moe_descs.append(md)
            a = [_f32(L.attn_norm), _f32(L.post_attn_norm), _u16(L.wq), _u16(L.wk), _u16(L.wv),
                 _u16(L.wo), _f32(L.bq), _f32(L.bk), _f32(L.bv), _f32(L.bo), _f32(L.sinks)]
            keep.append(a)
            x = layers[i]
            (x.attn_norm, x.post_attn_norm, x.wq, x.wk, x.wv, x.wo, x.bq, x.bk, x.bv, x.bo,
             x.sinks) = [_ptr(v) for v in a]
            x.sliding = int(L.sliding)
            x.moe = ctypes.pointer(md)
        d = DecoderDesc()
        d.struct_size = ctypes.sizeof(DecoderDesc)
        d.n_layers, d.hidden = w.n_layers, w.hidden
        d.n_heads, d.n_kv_heads, d.head_dim = w.n_heads, w.n_kv_heads, w.head_dim
        d.vocab, d.sliding_window = w.vocab, w.sliding_window
        d.max_seq_len, d.max_batch, d.max_tokens = max_seq_len, max_batch, max_tokens
        d.rope_theta, d.rope_scaling_factor = w.rope_theta, w.rope_scaling_factor
        d.rope_orig_ctx = w.rope_orig_ctx
        d.rms_eps = w.rms_eps
        d.device = device
        top = [_u16(w.embed), _u16(w.lm_head), _f32(w.final_norm)]
        keep.append(top)
        d.embed, d.lm_head, d.final_norm = [_ptr(v) for v in top]
        d.layers = layers
        lib = load_library()
        h = ctypes.c_void_p()
        check(lib.gb_decoder_create(ctypes.byref(d), ctypes.byref(h)))
        del keep, moe_descs
        return cls(h, w, device, max_batch, max_tokens, max_seq_len)

    # -- lifetime ------------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "_h", None) and self._h.value:
            check(self._lib.gb_decoder_destroy(self._h))
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # -- the reference's CausalLM surface --------------------------------------
    def _stream(self):
        import torch

        return torch.cuda.current_stream(torch.device("cuda", self.device)).cuda_stream

    def forward(self, token_ids, pos: int, check_status: bool = True):
        """token_ids (B, T) int32 (torch CUDA tensor or array); returns the
        (B, vocab) f32 logits of each sequence's last token and leaves the
        greedy tokens in self.last_next (B,)."""
        import torch

        dev = torch.device("cuda", self.device)
        t = torch.as_tensor(np.asarray(token_ids) if not torch.is_tensor(token_ids) else token_ids)
        t = t.to(device=dev, dtype=torch.int32).contiguous()
        B, T = t.shape
        logits = torch.empty((B, self.vocab), dtype=torch.float32, device=dev)
        nxt = torch.empty((B,), dtype=torch.int32, device=dev)
        check(self._lib.gb_decoder_forward(self._h, t.data_ptr(), B, T, pos, logits.data_ptr(),
                                           nxt.data_ptr(), self._stream()))
        if check_status:
            check(self._lib.gb_decoder_device_status(self._h, self._stream()))
        self.pos = pos + T
        self.last_next = nxt
        return logits

    def generate(self, tokens, pos: int, n_steps: int, check_status: bool = True):
        """n_steps greedy steps of B sequences from tokens (B,) at pos;
        returns the (n_steps, B) int32 tokens on the device."""
        import torch

        dev = torch.device("cuda", self.device)
        t = torch.as_tensor(np.asarray(tokens) if not torch.is_tensor(tokens) else tokens)
        t = t.to(device=dev, dtype=torch.int32).contiguous().reshape(-1)
        B = t.shape[0]
        out = torch.empty((n_steps, B), dtype=torch.int32, device=dev)
        check(self._lib.gb_decoder_generate(self._h, t.data_ptr(), B, pos, n_steps,
                                            out.data_ptr(), self._stream()))
        if check_status:
            check(self._lib.gb_decoder_device_status(self._h, self._stream()))
        self.pos = pos + n_steps
        return out

    def reset(self) -> None:
        check(self._lib.gb_decoder_reset(self._h))
        self.pos = 0

    def set_profiling(self, enable: bool = True) -> None:
        check(self._lib.gb_decoder_set_profiling(self._h, 1 if enable else 0))

    def stage_times(self) -> dict:
        """Milliseconds of the last profiled step: attention, MoE, head."""
        ms = (ctypes.c_float * 3)()
        check(self._lib.gb_decoder_stage_times(self._h, ms, self._stream()))
        return {"attention": ms[0], "moe": ms[1], "head": ms[2]}
