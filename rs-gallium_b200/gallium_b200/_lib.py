"""ctypes binding of libgallium_b200.so (the C ABI in include/gallium_b200.h).

The library is built in-tree (``make -C rs-gallium_b200``).  Loading fails
loudly when it is missing: there is no CPU fallback for the MoE path.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_int64, c_uint8, c_uint32, c_void_p

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(_HERE), "libgallium_b200.so")
HEADER_PATH = os.path.join(os.path.dirname(os.path.dirname(_HERE)), "include", "gallium_b200.h")

# gb_status
GB_OK = 0
GB_ERR_INVALID_ARG = 1
GB_ERR_SHAPE = 2
GB_ERR_CUDA = 3
GB_ERR_NCCL = 4
GB_ERR_TIMEOUT = 5
GB_ERR_UNSUPPORTED = 6
GB_ERR_NO_MEMORY = 7
STATUS_NAMES = {
    0: "OK", 1: "INVALID_ARG", 2: "SHAPE", 3: "CUDA", 4: "NCCL", 5: "TIMEOUT",
    6: "UNSUPPORTED", 7: "NO_MEMORY",
}

GB_ROUTER_SOFTMAX_TOPK = 0
GB_ROUTER_SIGMOID_TOPK = 1
GB_ACT_GPTOSS_CLAMP = 0
GB_ACT_SILU = 1
GB_ACT_GELU = 2
GB_ACT_GELU_TANH = 3
GB_ACT_RELU = 4
GB_FMT_MXFP4_SPLIT = 0
GB_FMT_MXFP4_GGUF = 1
GB_FMT_Q4_K = 2
GB_FMT_DENSE = 3
GB_PATH_AUTO = 0
GB_PATH_CUDA_CORES = 1
GB_PATH_TENSOR_CORES = 2
GB_PATH_TENSOR_CORES_F16 = 3
GB_PATH_FUSED_DECODE = 4
GB_DTYPE_F32 = 0
GB_DTYPE_BF16 = 1


class GalliumError(RuntimeError):
    """A non-zero gb_status, with the library's gb_last_error() message."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status
        self.message = message


class MoeDesc(ctypes.Structure):
    _fields_ = [
        ("struct_size", c_uint32),
        ("hidden", c_int32),
        ("inter", c_int32),
        ("n_experts", c_int32),
        ("top_k", c_int32),
        ("router_kind", c_int32),
        ("act_kind", c_int32),
        ("weight_format", c_int32),
        ("swiglu_limit", c_float),
        ("device", c_int32),
        ("max_tokens", c_int32),
        ("router_weight", c_void_p),
        ("router_bias", c_void_p),
        ("router_dtype", c_int32),
        ("selection_bias", c_void_p),
        ("gate_up_blocks", c_void_p),
        ("gate_up_scales", c_void_p),
        ("down_blocks", c_void_p),
        ("down_scales", c_void_p),
        ("gate_raw", c_void_p),
        ("up_raw", c_void_p),
        ("down_raw", c_void_p),
        ("gate_up_bias", c_void_p),
        ("gate_bias", c_void_p),
        ("up_bias", c_void_p),
        ("down_bias", c_void_p),
        ("bias_dtype", c_int32),
        ("ep_rank", c_int32),
        ("ep_size", c_int32),
        ("nccl_id", c_void_p),
        ("ep_timeout_ms", c_int32),
        ("weight_dtype", c_int32),
        ("act_clamp", c_float),
        ("shared_inter", c_int32),
        ("shared_gate", c_void_p),
        ("shared_up", c_void_p),
        ("shared_down", c_void_p),
        ("gate_up_merged", c_int32),
        ("expert_scale", c_void_p),
        ("input_norm", c_int32),
        ("router_input_scale", c_void_p),
        ("expert_input_norm", c_void_p),
        ("output_norm", c_void_p),
        ("rms_eps", c_float),
    ]


class MoeInfo(ctypes.Structure):
    _fields_ = [
        ("struct_size", c_uint32),
        ("local_expert_begin", c_int32),
        ("local_expert_end", c_int32),
        ("weight_bytes", c_int64),
        ("workspace_bytes", c_int64),
        ("workspace_tokens", c_int32),
        ("sm_count", c_int32),
        ("kernel_launches", c_int64),
        ("graph_captures", c_int64),
    ]


class DecoderLayer(ctypes.Structure):
    _fields_ = [
        ("attn_norm", c_void_p),
        ("post_attn_norm", c_void_p),
        ("wq", c_void_p),
        ("wk", c_void_p),
        ("wv", c_void_p),
        ("wo", c_void_p),
        ("bq", c_void_p),
        ("bk", c_void_p),
        ("bv", c_void_p),
        ("bo", c_void_p),
        ("sinks", c_void_p),
        ("sliding", c_int32),
        ("moe", POINTER(MoeDesc)),
    ]


class DecoderDesc(ctypes.Structure):
    _fields_ = [
        ("struct_size", c_uint32),
        ("n_layers", c_int32),
        ("hidden", c_int32),
        ("n_heads", c_int32),
        ("n_kv_heads", c_int32),
        ("head_dim", c_int32),
        ("vocab", c_int32),
        ("sliding_window", c_int32),
        ("max_seq_len", c_int32),
        ("max_batch", c_int32),
        ("max_tokens", c_int32),
        ("rope_theta", c_float),
        ("rope_scaling_factor", c_float),
        ("rope_orig_ctx", c_int32),
        ("rope_beta_fast", c_float),
        ("rope_beta_slow", c_float),
        ("rms_eps", c_float),
        ("device", c_int32),
        ("embed", c_void_p),
        ("lm_head", c_void_p),
        ("final_norm", c_void_p),
        ("layers", POINTER(DecoderLayer)),
    ]


# name -> (restype, argtypes); every symbol the header declares.
SIGNATURES = {
    "gb_moe_create": (c_int, [POINTER(MoeDesc), POINTER(c_void_p)]),
    "gb_moe_forward": (c_int, [c_void_p, c_void_p, c_int64, c_void_p, c_void_p]),
    "gb_moe_forward_host": (c_int, [c_void_p, c_void_p, c_int64, c_void_p, c_void_p]),
    "gb_moe_route": (c_int, [c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p,
                             c_void_p, c_void_p, c_void_p]),
    "gb_moe_dequant_expert": (c_int, [c_void_p, c_int32, c_int32, c_void_p, c_void_p]),
    "gb_moe_get_info": (c_int, [c_void_p, POINTER(MoeInfo)]),
    "gb_moe_device_status": (c_int, [c_void_p, c_void_p]),
    "gb_moe_destroy": (c_int, [c_void_p]),
    "gb_moe_set_expert_path": (c_int, [c_void_p, c_int32]),
    "gb_moe_set_graphs": (c_int, [c_void_p, c_int32]),
    "gb_moe_set_test_hooks": (c_int, [c_void_p, c_int64, c_int32]),
    "gb_moe_set_profiling": (c_int, [c_void_p, c_int]),
    "gb_moe_stage_times": (c_int, [c_void_p, POINTER(c_float), c_int32, POINTER(c_int32)]),
    "gb_moe_stage_name": (c_char_p, [c_int32]),
    "gb_route_noalloc": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int32,
                                 c_int32, c_int32, c_int32, c_void_p, c_void_p, c_void_p]),
    "gb_decoder_create": (c_int, [POINTER(DecoderDesc), POINTER(c_void_p)]),
    "gb_decoder_forward": (c_int, [c_void_p, c_void_p, c_int32, c_int32, c_int64, c_void_p,
                                   c_void_p, c_void_p]),
    "gb_decoder_generate": (c_int, [c_void_p, c_void_p, c_int32, c_int64, c_int32, c_void_p,
                                    c_void_p]),
    "gb_decoder_reset": (c_int, [c_void_p]),
    "gb_decoder_set_profiling": (c_int, [c_void_p, c_int32]),
    "gb_decoder_stage_times": (c_int, [c_void_p, POINTER(c_float), c_void_p]),
    "gb_decoder_device_status": (c_int, [c_void_p, c_void_p]),
    "gb_decoder_destroy": (c_int, [c_void_p]),
    "gb_nccl_unique_id": (c_int, [POINTER(c_uint8)]),
    "gb_last_error": (c_char_p, []),
    "gb_abi_version": (c_int, []),
}

_lib = None


def load_library(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load (once) and bind libgallium_b200.so; raise if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(
            f"{path} is missing: build it with `make -C rs-gallium_b200` "
            "(the MoE path has no CPU fallback)")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status: int) -> None:
    if status != GB_OK:
        msg = load_library().gb_last_error()
        raise GalliumError(status, msg.decode() if msg else "")
