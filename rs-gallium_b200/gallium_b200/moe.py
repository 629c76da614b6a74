"""Host-side mirror of rs-gallium's MoE FFN blocks over the C ABI.

The reference's blocks all expose ``forward(&self, x: &Tensor) -> Result<Tensor>``
with x of shape (batch, seq, hidden):

* ``OssMoEFFN``      crates/gallium-models/src/gpt_oss.rs:97-231 (safetensors MXFP4)
* ``GptOssQMoEFFN``  the ``QMoEFFN`` of crates/gallium-models/src/gpt_oss_q.rs:119-269
                     (GGUF MXFP4, separate gate/up tensors)

``load`` mirrors the reference's ``load`` (weights handed over once, repacked
on the device); ``forward`` keeps the reference's shape and dtype contract
(f32 compute, result in x's dtype, gpt_oss.rs:169 and :230).  Errors raise
GalliumError carrying the library's status, where the reference returns a
candle error.  A CUDA tensor runs through gb_moe_forward on torch's current
stream; a CPU tensor goes through gb_moe_forward_host (copies in and out).
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np

from . import _lib
from ._lib import MoeDesc, MoeInfo, check, load_library
from .synth import (DenseMoeLayer, Gemma4MoeLayer, GptOssGgufLayer, GptOssLayer, Lfm2Layer,
                    bf16_bits_to_f32)


def _as_f32(a: Optional[np.ndarray]) -> Optional[np.ndarray]:
    """A router or bias array as float32: uint16 arrays are bf16 bits, float16
    and float32 widen exactly."""
    if a is None:
        return None
    if a.dtype == np.uint16:
        return bf16_bits_to_f32(a)
    return np.ascontiguousarray(a, dtype=np.float32)


def _float_pair(a: Optional[np.ndarray], b: Optional[np.ndarray]):
    """(a, b, gb_dtype): kept as bf16 bits when every given array is bf16
    bits (uint16), else both widened to float32."""
    given = [x for x in (a, b) if x is not None]
    if given and all(x.dtype == np.uint16 for x in given):
        return a, b, _lib.GB_DTYPE_BF16
    return _as_f32(a), _as_f32(b), _lib.GB_DTYPE_F32


def _ptr(a: Optional[np.ndarray]) -> Optional[int]:
    if a is None:
        return None
    if not a.flags["C_CONTIGUOUS"]:
        raise _lib.GalliumError(_lib.GB_ERR_INVALID_ARG, "weight array is not C-contiguous")
    return a.ctypes.data


class MoEBlock:
    """Owns one gb_moe handle.  Not re-entrant (one forward at a time)."""

    def __init__(self, desc: MoeDesc, keepalive: list):
        self._lib = load_library()
        self._keepalive = keepalive  # host arrays stay alive until create returns
        h = ctypes.c_void_p()
        check(self._lib.gb_moe_create(ctypes.byref(desc), ctypes.byref(h)))
        self._h = h
        self._keepalive = None
        self.hidden = desc.hidden
        self.inter = desc.inter
        self.n_experts = desc.n_experts
        self.top_k = desc.top_k
        self.device = desc.device

    # -- lifetime ------------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "_h", None) and self._h.value:
            check(self._lib.gb_moe_destroy(self._h))
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

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._h

    def info(self) -> dict:
        inf = MoeInfo()
        inf.struct_size = ctypes.sizeof(MoeInfo)
        check(self._lib.gb_moe_get_info(self._h, ctypes.byref(inf)))
        return {f: getattr(inf, f) for f, _ in MoeInfo._fields_ if f != "struct_size"}

    # -- forward -------------------------------------------------------------
    def forward(self, x, check_status: bool = True):
        """x: torch.Tensor (batch, seq, hidden) or (tokens, hidden).

        With check_status (the default) a device input waits for the forward
        and raises if a kernel recorded an error; pass False to keep the call
        asynchronous and call device_status() when the output is consumed."""
        import torch

        shape = x.shape
        if shape[-1] != self.hidden:
            raise _lib.GalliumError(_lib.GB_ERR_SHAPE,
                                    f"last dim {shape[-1]} != hidden {self.hidden}")
        self._check_device(x)
        xf = x.reshape(-1, self.hidden).to(torch.float32).contiguous()
        T = xf.shape[0]
        if x.is_cuda:
            out = torch.empty_like(xf)
            stream = torch.cuda.current_stream(xf.device).cuda_stream
            check(self._lib.gb_moe_forward(self._h, xf.data_ptr(), T, out.data_ptr(), stream))
            if check_status:
                check(self._lib.gb_moe_device_status(self._h, stream))
        else:
            out = torch.empty_like(xf)
            check(self._lib.gb_moe_forward_host(self._h, xf.data_ptr(), T, out.data_ptr(), None))
        return out.reshape(shape).to(x.dtype)

    __call__ = forward

    def _check_device(self, x) -> None:
        """A CUDA input must live on the handle's device: the kernels would
        otherwise be handed another GPU's addresses."""
        if x.is_cuda and x.device.index != self.device:
            raise _lib.GalliumError(
                _lib.GB_ERR_INVALID_ARG,
                f"x is on cuda:{x.device.index}, the block on cuda:{self.device}")

    def device_status(self, stream: int = 0) -> None:
        """Waits for `stream` and raises if a forward kernel recorded an error."""
        check(self._lib.gb_moe_device_status(self._h, stream))

    def forward_raw(self, x_ptr: int, T: int, out_ptr: int, stream: int = 0) -> None:
        """Device pointers straight through to gb_moe_forward (no checks)."""
        check(self._lib.gb_moe_forward(self._h, x_ptr, T, out_ptr, stream))

    def set_expert_path(self, path: str) -> None:
        """'auto', 'cuda_cores', 'tensor_cores', 'tensor_cores_f16' or
        'fused_decode' (gb_moe_set_expert_path)."""
        code = {"auto": _lib.GB_PATH_AUTO, "cuda_cores": _lib.GB_PATH_CUDA_CORES,
                "tensor_cores": _lib.GB_PATH_TENSOR_CORES,
                "tensor_cores_f16": _lib.GB_PATH_TENSOR_CORES_F16,
                "fused_decode": _lib.GB_PATH_FUSED_DECODE}[path]
        check(self._lib.gb_moe_set_expert_path(self._h, code))

    def set_graphs(self, max_graphs: int) -> None:
        """Forward graphs kept for replay, 0..16; 0 launches every kernel
        directly (gb_moe_set_graphs)."""
        check(self._lib.gb_moe_set_graphs(self._h, int(max_graphs)))

    def set_test_hooks(self, wait_limit_us: int = 0, withhold_ready: bool = False) -> None:
        """Failure-handling test hooks (gb_moe_set_test_hooks): a shorter
        bounded-wait limit and a withheld ready flag in the one-launch expert
        kernel; (0, False) restores normal operation."""
        check(self._lib.gb_moe_set_test_hooks(self._h, int(wait_limit_us),
                                               1 if withhold_ready else 0))

    def set_profiling(self, enable: bool = True) -> None:
        check(self._lib.gb_moe_set_profiling(self._h, 1 if enable else 0))

    def stage_times(self) -> dict:
        """Per-stage milliseconds of the last profiled forward."""
        buf = (ctypes.c_float * 16)()
        n = ctypes.c_int32()
        check(self._lib.gb_moe_stage_times(self._h, buf, 16, ctypes.byref(n)))
        return {self._lib.gb_moe_stage_name(i).decode(): buf[i] for i in range(n.value)}

    def route(self, x) -> dict:
        """Routing of x (CUDA tensor [T, H] f32) as torch tensors on its device."""
        import torch

        self._check_device(x)
        if not x.is_cuda:
            raise _lib.GalliumError(_lib.GB_ERR_INVALID_ARG, "route takes a CUDA tensor")
        xf = x.reshape(-1, self.hidden).to(torch.float32).contiguous()
        T = xf.shape[0]
        dev = xf.device
        k, E = self.top_k, self.n_experts
        idx = torch.empty((T, k), dtype=torch.int32, device=dev)
        w = torch.empty((T, k), dtype=torch.float32, device=dev)
        counts = torch.empty((E,), dtype=torch.int32, device=dev)
        offsets = torch.empty((E + 1,), dtype=torch.int32, device=dev)
        perm = torch.empty((T * k,), dtype=torch.int32, device=dev)
        stream = torch.cuda.current_stream(dev).cuda_stream
        check(self._lib.gb_moe_route(self._h, xf.data_ptr(), T, idx.data_ptr(), w.data_ptr(),
                                     counts.data_ptr(), offsets.data_ptr(), perm.data_ptr(),
                                     stream))
        return {"idx": idx, "w": w, "counts": counts, "offsets": offsets, "perm": perm}

    def dequant_expert(self, which: int, expert: int):
        """f32 matrix of a local expert from the repacked device layout:
        which 0 = gate [I, H], 1 = up [I, H], 2 = down [H, I]."""
        import torch

        rows, cols = (self.hidden, self.inter) if which == 2 else (self.inter, self.hidden)
        out = torch.empty((rows, cols), dtype=torch.float32, device=f"cuda:{self.device}")
        stream = torch.cuda.current_stream(out.device).cuda_stream
        check(self._lib.gb_moe_dequant_expert(self._h, which, expert, out.data_ptr(), stream))
        return out


def nccl_unique_id() -> bytes:
    """A fresh 128-byte NCCL unique id (rank 0 creates it and shares it)."""
    lib = load_library()
    buf = (ctypes.c_uint8 * 128)()
    check(lib.gb_nccl_unique_id(buf))
    return bytes(buf)


def _base_desc(hidden, inter, n_experts, top_k, device, max_tokens, ep=None) -> MoeDesc:
    """ep: None (one GPU) or (rank, size, nccl_id bytes[, timeout_ms]) for expert
    parallelism; timeout_ms bounds every wait for the other ranks (default
    60000)."""
    d = MoeDesc()
    d.struct_size = ctypes.sizeof(MoeDesc)
    d.hidden, d.inter, d.n_experts, d.top_k = hidden, inter, n_experts, top_k
    d.device = device
    d.max_tokens = max_tokens
    d.ep_size = 1
    if ep is not None:
        rank, size, nid = ep[:3]
        d.ep_rank, d.ep_size = rank, size
        d.ep_timeout_ms = int(ep[3]) if len(ep) > 3 else 0
        d._nccl_id_buf = (ctypes.c_uint8 * 128).from_buffer_copy(nid)
        d.nccl_id = ctypes.addressof(d._nccl_id_buf)
    return d


class OssMoEFFN(MoEBlock):
    """Safetensors GPT-OSS MoE block (gpt_oss.rs:97-231)."""

    @classmethod
    def load(cls, layer: GptOssLayer, device: int = 0, max_tokens: int = 64,
             ep=None) -> "OssMoEFFN":
        """ep = (rank, size, nccl_id) shards the experts over `size` GPUs."""
        d = _base_desc(layer.hidden, layer.inter, layer.n_experts, layer.top_k, device, max_tokens,
                       ep)
        d.router_kind = _lib.GB_ROUTER_SOFTMAX_TOPK
        d.act_kind = _lib.GB_ACT_GPTOSS_CLAMP
        d.weight_format = _lib.GB_FMT_MXFP4_SPLIT
        d.swiglu_limit = layer.swiglu_limit
        # Router and biases go over in their stored dtype: bf16 bits (uint16)
        # as BF16, float32 / float16 as F32.
        rw, rb, d.router_dtype = _float_pair(layer.router_w, layer.router_b)
        gub, dnb, d.bias_dtype = _float_pair(layer.gu_bias, layer.dn_bias)
        arrs = [None if a is None else np.ascontiguousarray(a) for a in (
            rw, rb, layer.gu_blocks, layer.gu_scales, layer.dn_blocks, layer.dn_scales, gub, dnb)]
        (d.router_weight, d.router_bias, d.gate_up_blocks, d.gate_up_scales, d.down_blocks,
         d.down_scales, d.gate_up_bias, d.down_bias) = [_ptr(a) for a in arrs]
        return cls(d, arrs + [getattr(d, "_nccl_id_buf", None)])


class GptOssQMoEFFN(MoEBlock):
    """GGUF GPT-OSS MoE block (QMoEFFN, gpt_oss_q.rs:119-269)."""

    @classmethod
    def load(cls, layer: GptOssGgufLayer, device: int = 0, max_tokens: int = 64,
             ep=None) -> "GptOssQMoEFFN":
        b = layer.base
        d = _base_desc(b.hidden, b.inter, b.n_experts, b.top_k, device, max_tokens, ep)
        d.router_kind = _lib.GB_ROUTER_SOFTMAX_TOPK
        d.act_kind = _lib.GB_ACT_GPTOSS_CLAMP
        d.weight_format = _lib.GB_FMT_MXFP4_GGUF
        d.swiglu_limit = b.swiglu_limit
        # Router and biases as float32 (GGUF F32 tensors, or bf16 bits widened).
        rw, rb = _as_f32(b.router_w), _as_f32(b.router_b)
        gb_, ub, db = _as_f32(layer.gate_bias), _as_f32(layer.up_bias), _as_f32(layer.down_bias)
        arrs = [None if a is None else np.ascontiguousarray(a) for a in (
            rw, rb, layer.gate_raw, layer.up_raw, layer.down_raw, gb_, ub, db)]
        (d.router_weight, d.router_bias, d.gate_raw, d.up_raw, d.down_raw, d.gate_bias,
         d.up_bias, d.down_bias) = [_ptr(a) for a in arrs]
        d.router_dtype = _lib.GB_DTYPE_F32
        d.bias_dtype = _lib.GB_DTYPE_F32
        return cls(d, arrs)


class Lfm2QMoEFFN(MoEBlock):
    """LFM2.5 MoE block with Q4_K experts (QMoEFFN, lfm2moe_q.rs:203-313)."""

    @classmethod
    def load(cls, layer: Lfm2Layer, device: int = 0, max_tokens: int = 64,
             ep=None) -> "Lfm2QMoEFFN":
        d = _base_desc(layer.hidden, layer.inter, layer.n_experts, layer.top_k, device,
                       max_tokens, ep)
        d.router_kind = _lib.GB_ROUTER_SIGMOID_TOPK
        d.act_kind = _lib.GB_ACT_SILU
        d.weight_format = _lib.GB_FMT_Q4_K
        arrs = [None if a is None else np.ascontiguousarray(a) for a in (
            _as_f32(layer.router_w), _as_f32(layer.sel_bias), layer.gate_raw, layer.up_raw,
            layer.down_raw)]
        (d.router_weight, d.selection_bias, d.gate_raw, d.up_raw, d.down_raw) = [
            _ptr(a) for a in arrs]
        d.router_dtype = _lib.GB_DTYPE_F32
        d.bias_dtype = _lib.GB_DTYPE_F32
        return cls(d, arrs + [getattr(d, "_nccl_id_buf", None)])


class MoEFFN(MoEBlock):
    """gallium-core's generic MoE FFN (MoEFFN, crates/gallium-core/src/ffn.rs:72-166):
    dense GatedFFN experts with a configurable activation and optional clamp,
    softmax top-k routing, and an optional shared expert over all tokens
    (the Qwen3.5 MoE layers, crates/gallium-models/src/qwen35.rs:222-233)."""

    @classmethod
    def load(cls, layer: DenseMoeLayer, device: int = 0, max_tokens: int = 64,
             ep=None) -> "MoEFFN":
        d = _base_desc(layer.hidden, layer.inter, layer.n_experts, layer.top_k, device,
                       max_tokens, ep)
        d.router_kind = _lib.GB_ROUTER_SOFTMAX_TOPK
        d.act_kind = layer.act_kind
        d.act_clamp = layer.act_clamp
        d.weight_format = _lib.GB_FMT_DENSE
        mats = [layer.gate, layer.up, layer.down]
        if layer.shared_inter:
            mats += [layer.sh_gate, layer.sh_up, layer.sh_down]
        # weights go over as stored when they are all bf16 bits, else as f32
        bf16 = all(a.dtype == np.uint16 for a in mats)
        mats = [np.ascontiguousarray(a) if bf16 else np.ascontiguousarray(_as_f32(a))
                for a in mats]
        d.weight_dtype = _lib.GB_DTYPE_BF16 if bf16 else _lib.GB_DTYPE_F32
        rw, _, d.router_dtype = _float_pair(layer.router_w, None)
        rw = np.ascontiguousarray(rw)
        d.router_weight = _ptr(rw)
        d.gate_raw, d.up_raw, d.down_raw = [_ptr(a) for a in mats[:3]]
        d.shared_inter = layer.shared_inter
        if layer.shared_inter:
            d.shared_gate, d.shared_up, d.shared_down = [_ptr(a) for a in mats[3:]]
        return cls(d, mats + [rw, getattr(d, "_nccl_id_buf", None)])


class QGemmaMoe(MoEBlock):
    """Gemma-4's routed experts (QGemmaMoe, crates/gallium-models/src/gemma4_q.rs:187-330):
    forward(attn_out) = post_ffw_norm_2(sum of the top-k experts' scaled
    outputs), the router reading rms(x) / sqrt(H) * ffn_gate_inp.scale, the
    experts reading pre_ffw_norm_2(x), merged gate_up (gate rows first), GELU
    (tanh) gating, GGUF MXFP4 or Q4_K experts."""

    @classmethod
    def load(cls, layer: Gemma4MoeLayer, device: int = 0, max_tokens: int = 64,
             ep=None) -> "QGemmaMoe":
        d = _base_desc(layer.hidden, layer.inter, layer.n_experts, layer.top_k, device,
                       max_tokens, ep)
        d.router_kind = _lib.GB_ROUTER_SOFTMAX_TOPK
        d.act_kind = _lib.GB_ACT_GELU_TANH
        d.weight_format = layer.fmt
        d.gate_up_merged = 1
        arrs = [np.ascontiguousarray(a) for a in (
            layer.router_w.astype(np.float32), layer.gate_up_raw, layer.down_raw,
            layer.router_scale.astype(np.float32), layer.expert_norm.astype(np.float32),
            layer.output_norm.astype(np.float32))]
        (d.router_weight, d.gate_raw, d.down_raw, d.router_input_scale, d.expert_input_norm,
         d.output_norm) = [_ptr(a) for a in arrs]
        d.router_dtype = _lib.GB_DTYPE_F32
        d.bias_dtype = _lib.GB_DTYPE_F32
        d.input_norm = 1
        d.rms_eps = layer.rms_eps
        if layer.expert_scale is not None:
            es = np.ascontiguousarray(layer.expert_scale, np.float32)
            arrs.append(es)
            d.expert_scale = _ptr(es)
        return cls(d, arrs + [getattr(d, "_nccl_id_buf", None)])
