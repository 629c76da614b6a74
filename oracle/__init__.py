"""ctypes binding of the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference arm, as the checker.  The product path
(rs-gallium_b200) never imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_int64, c_uint8, c_void_p

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "liboracle.so")

OR_ROUTER_SOFTMAX_TOPK, OR_ROUTER_SIGMOID_TOPK = 0, 1
OR_ACT_GPTOSS_CLAMP, OR_ACT_SILU, OR_ACT_GELU, OR_ACT_GELU_TANH, OR_ACT_RELU = 0, 1, 2, 3, 4
OR_FMT_MXFP4_SPLIT, OR_FMT_MXFP4_GGUF, OR_FMT_Q4_K, OR_FMT_DENSE = 0, 1, 2, 3


class OrDesc(ctypes.Structure):
    _fields_ = [
        ("hidden", c_int64), ("inter", c_int64), ("n_experts", c_int64), ("top_k", c_int64),
        ("router_kind", c_int32), ("act_kind", c_int32), ("weight_format", c_int32),
        ("swiglu_limit", c_float),
        ("router_w", c_void_p), ("router_b", c_void_p), ("sel_bias", c_void_p),
        ("gu_blocks", c_void_p), ("gu_scales", c_void_p), ("dn_blocks", c_void_p),
        ("dn_scales", c_void_p),
        ("gate_raw", c_void_p), ("up_raw", c_void_p), ("down_raw", c_void_p),
        ("gu_bias", c_void_p), ("gate_bias", c_void_p), ("up_bias", c_void_p),
        ("dn_bias", c_void_p),
        ("dense_gate", c_void_p), ("dense_up", c_void_p), ("dense_down", c_void_p),
        ("shared_inter", c_int64), ("sh_gate", c_void_p), ("sh_up", c_void_p),
        ("sh_down", c_void_p), ("act_clamp", c_float),
        ("gate_up_merged", c_int32), ("expert_scale", c_void_p), ("input_norm", c_int32),
        ("router_input_scale", c_void_p), ("expert_input_norm", c_void_p),
        ("output_norm", c_void_p), ("rms_eps", c_float),
    ]


_lib = None


def build() -> None:
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P = c_void_p
        sig = {
            "or_e2m1_value": (c_float, [c_int]),
            "or_mxfp4_split_dequant": (c_int, [P, P, c_int64, c_int64, P]),
            "or_e8m0_to_f32": (c_float, [c_uint8]),
            "or_mxfp4_blocks_per_expert": (c_int, [c_int64, POINTER(c_int64)]),
            "or_mxfp4_gguf_dequant": (c_int, [P, c_int64, P]),
            "or_q4k_dequant": (c_int, [P, c_int64, P]),
            "or_router_logits": (c_int, [P, P, P, c_int64, c_int64, c_int64, P]),
            "or_route_softmax_topk": (c_int, [P, c_int64, c_int64, c_int64, P, P]),
            "or_route_sigmoid_topk": (c_int, [P, P, c_int64, c_int64, c_int64, P, P]),
            "or_permute": (c_int, [P, c_int64, c_int64, c_int64, P, P, P, P]),
            "or_moe_forward": (c_int, [POINTER(OrDesc), P, c_int64, P, P, P, c_int]),
            "or_moe_expert_sample": (c_int64, [POINTER(OrDesc), P, P, P, c_int64, P, c_int]),
            "or_expert_ffn": (c_int, [POINTER(OrDesc), c_int64, P, c_int64, P]),
            "or_act_gptoss": (c_float, [c_float, c_float, c_float]),
            "or_act_silu": (c_float, [c_float, c_float]),
            "or_exp_rn": (c_float, [c_float]),
            "or_dequant_expert_matrix": (c_int, [POINTER(OrDesc), c_int, c_int64, P, c_int]),
            "or_act_rows": (None, [POINTER(OrDesc), P, P, c_int64, c_int64, P, c_int]),
            "or_last_error": (c_char_p, []),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype, fn.argtypes = res, args
        _lib = L
    return _lib


class OracleError(RuntimeError):
    pass


def _check(rc: int) -> None:
    if rc != 0:
        raise OracleError(f"oracle error {rc}: {lib().or_last_error().decode()}")


def _p(a):
    return None if a is None else a.ctypes.data


# ---- decoders -------------------------------------------------------------

def e8m0_to_f32(b: int) -> float:
    return lib().or_e8m0_to_f32(b)


def mxfp4_blocks_per_expert(n_elems: int) -> int:
    nb = c_int64()
    _check(lib().or_mxfp4_blocks_per_expert(n_elems, ctypes.byref(nb)))
    return nb.value


def mxfp4_gguf_dequant(raw: np.ndarray, n_elems: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw, np.uint8)
    out = np.empty(n_elems, np.float32)
    _check(lib().or_mxfp4_gguf_dequant(_p(raw), n_elems, _p(out)))
    return out


def mxfp4_split_dequant(blocks: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """blocks [rows, k/32, 16], scales [rows, k/32] -> [rows, k] f32."""
    blocks = np.ascontiguousarray(blocks, np.uint8)
    scales = np.ascontiguousarray(scales, np.uint8)
    rows, nb = scales.shape
    out = np.empty((rows, nb * 32), np.float32)
    _check(lib().or_mxfp4_split_dequant(_p(blocks), _p(scales), rows, nb * 32, _p(out)))
    return out


def q4k_dequant(raw: np.ndarray, n_elems: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw, np.uint8)
    out = np.empty(n_elems, np.float32)
    _check(lib().or_q4k_dequant(_p(raw), n_elems, _p(out)))
    return out


def act_gptoss(g: float, u: float, limit: float = 7.0) -> float:
    return lib().or_act_gptoss(g, u, limit)


def act_silu(g: float, u: float) -> float:
    return lib().or_act_silu(g, u)


def exp_rn(x: float) -> float:
    """exp(x) correctly rounded to f32 (the exp of the router's softmax and
    sigmoid)."""
    return lib().or_exp_rn(x)


# ---- routing --------------------------------------------------------------

def router_logits(x: np.ndarray, w: np.ndarray, b=None) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    b = None if b is None else np.ascontiguousarray(b, np.float32)
    T, H = x.shape
    E = w.shape[0]
    out = np.empty((T, E), np.float32)
    _check(lib().or_router_logits(_p(x), _p(w), _p(b), T, H, E, _p(out)))
    return out


def route_softmax_topk(logits: np.ndarray, k: int):
    logits = np.ascontiguousarray(logits, np.float32)
    T, E = logits.shape
    idx = np.empty((T, k), np.int32)
    w = np.empty((T, k), np.float32)
    _check(lib().or_route_softmax_topk(_p(logits), T, E, k, _p(idx), _p(w)))
    return idx, w


def route_sigmoid_topk(logits: np.ndarray, sel_bias, k: int):
    logits = np.ascontiguousarray(logits, np.float32)
    T, E = logits.shape
    sb = None if sel_bias is None else np.ascontiguousarray(sel_bias, np.float32)
    idx = np.empty((T, k), np.int32)
    w = np.empty((T, k), np.float32)
    _check(lib().or_route_sigmoid_topk(_p(logits), _p(sb), T, E, k, _p(idx), _p(w)))
    return idx, w


def permute(idx: np.ndarray, n_experts: int):
    idx = np.ascontiguousarray(idx, np.int32)
    T, k = idx.shape
    counts = np.empty(n_experts, np.int32)
    offsets = np.empty(n_experts + 1, np.int32)
    perm = np.empty(T * k, np.int32)
    inv = np.empty(T * k, np.int32)
    _check(lib().or_permute(_p(idx), T, n_experts, k, _p(counts), _p(offsets), _p(perm),
                            _p(inv)))
    return counts, offsets, perm, inv


# ---- whole block ----------------------------------------------------------

def _bf(a):
    """A router or bias array as float32: uint16 arrays are bf16 bits; float
    arrays (as read from F32 / F16 checkpoint tensors) widen exactly."""
    if a is None:
        return None
    if a.dtype == np.uint16:
        return (np.ascontiguousarray(a).astype(np.uint32) << 16).view(np.float32)
    return np.ascontiguousarray(a, np.float32)


class OracleMoe:
    """The oracle for one GPT-OSS layer (safetensors layout, or its GGUF view)."""

    def __init__(self, layer, gguf=None):
        self.layer = layer
        d = OrDesc()
        d.hidden, d.inter, d.n_experts, d.top_k = (layer.hidden, layer.inter, layer.n_experts,
                                                   layer.top_k)
        d.router_kind = OR_ROUTER_SOFTMAX_TOPK
        d.act_kind = OR_ACT_GPTOSS_CLAMP
        d.swiglu_limit = layer.swiglu_limit
        keep = {}
        keep["rw"] = _bf(layer.router_w)
        keep["rb"] = _bf(layer.router_b)
        d.router_w, d.router_b = _p(keep["rw"]), _p(keep["rb"])
        if gguf is None:
            d.weight_format = OR_FMT_MXFP4_SPLIT
            for name in ("gu_blocks", "gu_scales", "dn_blocks", "dn_scales"):
                keep[name] = np.ascontiguousarray(getattr(layer, name))
            d.gu_blocks, d.gu_scales = _p(keep["gu_blocks"]), _p(keep["gu_scales"])
            d.dn_blocks, d.dn_scales = _p(keep["dn_blocks"]), _p(keep["dn_scales"])
            keep["gub"] = _bf(layer.gu_bias)
            d.gu_bias = _p(keep["gub"])
        else:
            d.weight_format = OR_FMT_MXFP4_GGUF
            keep["g"], keep["u"], keep["d"] = gguf.gate_raw, gguf.up_raw, gguf.down_raw
            d.gate_raw, d.up_raw, d.down_raw = _p(keep["g"]), _p(keep["u"]), _p(keep["d"])
            keep["gb"] = _bf(gguf.gate_bias)
            keep["ub"] = _bf(gguf.up_bias)
            d.gate_bias, d.up_bias = _p(keep["gb"]), _p(keep["ub"])
        keep["db"] = _bf(layer.dn_bias if gguf is None else gguf.down_bias)
        d.dn_bias = _p(keep["db"])
        self.desc = d
        self._keep = keep

    def forward(self, x: np.ndarray, n_threads: int = 0):
        x = np.ascontiguousarray(x, np.float32)
        T = x.shape[0]
        k = self.layer.top_k
        out = np.empty_like(x)
        idx = np.empty((T, k), np.int32)
        w = np.empty((T, k), np.float32)
        _check(lib().or_moe_forward(ctypes.byref(self.desc), _p(x), T, _p(out), _p(idx), _p(w),
                                    n_threads))
        return out, idx, w

    def expert_ffn(self, expert: int, xs: np.ndarray) -> np.ndarray:
        xs = np.ascontiguousarray(xs, np.float32)
        ys = np.empty_like(xs)
        _check(lib().or_expert_ffn(ctypes.byref(self.desc), expert, _p(xs), xs.shape[0], _p(ys)))
        return ys

    def expert_sample(self, x: np.ndarray, experts, ntok, n_threads: int = 0) -> int:
        x = np.ascontiguousarray(x, np.float32)
        ex = np.ascontiguousarray(experts, np.int32)
        nt = np.ascontiguousarray(ntok, np.int32)
        assert x.shape[0] >= int(nt.max())
        return lib().or_moe_expert_sample(ctypes.byref(self.desc), _p(x), _p(ex), _p(nt),
                                          len(ex), None, n_threads)


class OracleLfm2:
    """The oracle for one LFM2.5 layer (Q4_K experts, sigmoid router, SiLU)."""

    def __init__(self, layer):
        self.layer = layer
        d = OrDesc()
        d.hidden, d.inter, d.n_experts, d.top_k = (layer.hidden, layer.inter, layer.n_experts,
                                                   layer.top_k)
        d.router_kind = OR_ROUTER_SIGMOID_TOPK
        d.act_kind = OR_ACT_SILU
        d.weight_format = OR_FMT_Q4_K
        keep = {k: np.ascontiguousarray(getattr(layer, k))
                for k in ("router_w", "sel_bias", "gate_raw", "up_raw", "down_raw")}
        d.router_w, d.sel_bias = _p(keep["router_w"]), _p(keep["sel_bias"])
        d.gate_raw, d.up_raw, d.down_raw = _p(keep["gate_raw"]), _p(keep["up_raw"]), _p(keep["down_raw"])
        self.desc = d
        self._keep = keep

    forward = OracleMoe.forward
    expert_ffn = OracleMoe.expert_ffn
    expert_sample = OracleMoe.expert_sample


class OracleDense:
    """The oracle for one gallium-core MoEFFN layer (ffn.rs:72-166): dense
    experts (bf16 bits widened exactly, or f32), generic activation with an
    optional clamp, optional shared expert."""

    def __init__(self, layer):
        self.layer = layer
        d = OrDesc()
        d.hidden, d.inter, d.n_experts, d.top_k = (layer.hidden, layer.inter, layer.n_experts,
                                                   layer.top_k)
        d.router_kind = OR_ROUTER_SOFTMAX_TOPK
        d.act_kind = layer.act_kind
        d.act_clamp = layer.act_clamp
        d.weight_format = OR_FMT_DENSE
        keep = {k: _bf(getattr(layer, k)) for k in ("router_w", "gate", "up", "down")}
        d.router_w = _p(keep["router_w"])
        d.dense_gate, d.dense_up, d.dense_down = _p(keep["gate"]), _p(keep["up"]), _p(keep["down"])
        d.shared_inter = layer.shared_inter
        if layer.shared_inter:
            for k in ("sh_gate", "sh_up", "sh_down"):
                keep[k] = _bf(getattr(layer, k))
            d.sh_gate, d.sh_up, d.sh_down = _p(keep["sh_gate"]), _p(keep["sh_up"]), _p(keep["sh_down"])
        self.desc = d
        self._keep = keep

    forward = OracleMoe.forward
    expert_ffn = OracleMoe.expert_ffn
    expert_sample = OracleMoe.expert_sample


class OracleGemma4:
    """The oracle for Gemma-4's routed-experts block (QGemmaMoe::forward,
    gemma4_q.rs:262-328): normed router input, normed expert input, merged
    gate_up, GELU (tanh) gating, per-expert output scale, expert-order sum,
    output norm."""

    def __init__(self, layer):
        self.layer = layer
        d = OrDesc()
        d.hidden, d.inter, d.n_experts, d.top_k = (layer.hidden, layer.inter, layer.n_experts,
                                                   layer.top_k)
        d.router_kind = OR_ROUTER_SOFTMAX_TOPK
        d.act_kind = OR_ACT_GELU_TANH
        d.weight_format = layer.fmt
        d.gate_up_merged = 1
        keep = {k: np.ascontiguousarray(getattr(layer, k)) for k in (
            "router_w", "router_scale", "expert_norm", "gate_up_raw", "down_raw", "output_norm")}
        d.router_w = _p(keep["router_w"])
        d.gate_raw, d.down_raw = _p(keep["gate_up_raw"]), _p(keep["down_raw"])
        if layer.expert_scale is not None:
            keep["expert_scale"] = np.ascontiguousarray(layer.expert_scale, np.float32)
            d.expert_scale = _p(keep["expert_scale"])
        d.input_norm = 1
        d.router_input_scale, d.expert_input_norm = _p(keep["router_scale"]), _p(keep["expert_norm"])
        d.output_norm = _p(keep["output_norm"])
        d.rms_eps = layer.rms_eps
        self.desc = d
        self._keep = keep

    forward = OracleMoe.forward
