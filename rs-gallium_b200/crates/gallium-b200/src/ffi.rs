//! Raw bindings of include/gallium_b200.h (ABI version 4).  Field order and
//! types follow the header exactly; tests/test_rust_binding.py checks them.
#![allow(non_camel_case_types)]

use std::os::raw::{c_char, c_int, c_void};

pub const GB_ABI_VERSION: c_int = 4;

// gb_status
pub const GB_OK: c_int = 0;
pub const GB_ERR_INVALID_ARG: c_int = 1;
pub const GB_ERR_SHAPE: c_int = 2;
pub const GB_ERR_CUDA: c_int = 3;
pub const GB_ERR_NCCL: c_int = 4;
pub const GB_ERR_TIMEOUT: c_int = 5;
pub const GB_ERR_UNSUPPORTED: c_int = 6;
pub const GB_ERR_NO_MEMORY: c_int = 7;

// gb_router_kind
pub const GB_ROUTER_SOFTMAX_TOPK: i32 = 0;
pub const GB_ROUTER_SIGMOID_TOPK: i32 = 1;

// gb_act_kind
pub const GB_ACT_GPTOSS_CLAMP: i32 = 0;
pub const GB_ACT_SILU: i32 = 1;
pub const GB_ACT_GELU: i32 = 2;
pub const GB_ACT_GELU_TANH: i32 = 3;
pub const GB_ACT_RELU: i32 = 4;

// gb_weight_format
pub const GB_FMT_MXFP4_SPLIT: i32 = 0;
pub const GB_FMT_MXFP4_GGUF: i32 = 1;
pub const GB_FMT_Q4_K: i32 = 2;
pub const GB_FMT_DENSE: i32 = 3;

// gb_dtype
pub const GB_DTYPE_F32: i32 = 0;
pub const GB_DTYPE_BF16: i32 = 1;

// gb_expert_path
pub const GB_PATH_AUTO: i32 = 0;
pub const GB_PATH_CUDA_CORES: i32 = 1;
pub const GB_PATH_TENSOR_CORES: i32 = 2;
pub const GB_PATH_TENSOR_CORES_F16: i32 = 3;
pub const GB_PATH_FUSED_DECODE: i32 = 4;

#[repr(C)]
#[derive(Clone, Copy)]
pub struct gb_moe_desc {
    pub struct_size: u32,
    pub hidden: i32,
    pub inter: i32,
    pub n_experts: i32,
    pub top_k: i32,
    pub router_kind: i32,
    pub act_kind: i32,
    pub weight_format: i32,
    pub swiglu_limit: f32,
    pub device: i32,
    pub max_tokens: i32,
    pub router_weight: *const c_void,
    pub router_bias: *const c_void,
    pub router_dtype: i32,
    pub selection_bias: *const f32,
    pub gate_up_blocks: *const u8,
    pub gate_up_scales: *const u8,
    pub down_blocks: *const u8,
    pub down_scales: *const u8,
    pub gate_raw: *const u8,
    pub up_raw: *const u8,
    pub down_raw: *const u8,
    pub gate_up_bias: *const c_void,
    pub gate_bias: *const c_void,
    pub up_bias: *const c_void,
    pub down_bias: *const c_void,
    pub bias_dtype: i32,
    pub ep_rank: i32,
    pub ep_size: i32,
    pub nccl_id: *const u8,
    pub ep_timeout_ms: i32,
    pub weight_dtype: i32,
    pub act_clamp: f32,
    pub shared_inter: i32,
    pub shared_gate: *const c_void,
    pub shared_up: *const c_void,
    pub shared_down: *const c_void,
    pub gate_up_merged: i32,
    pub expert_scale: *const f32,
    pub input_norm: i32,
    pub router_input_scale: *const f32,
    pub expert_input_norm: *const f32,
    pub output_norm: *const f32,
    pub rms_eps: f32,
}

impl Default for gb_moe_desc {
    /// Zeroed, with struct_size set, as the header asks.
    fn default() -> Self {
        // SAFETY: every field is an integer, a float or a raw pointer, for
        // which all-zero bytes are valid (null pointers).
        let mut d: Self = unsafe { std::mem::zeroed() };
        d.struct_size = std::mem::size_of::<Self>() as u32;
        d
    }
}

#[repr(C)]
#[derive(Clone, Copy, Default)]
pub struct gb_moe_info {
    pub struct_size: u32,
    pub local_expert_begin: i32,
    pub local_expert_end: i32,
    pub weight_bytes: i64,
    pub workspace_bytes: i64,
    pub workspace_tokens: i32,
    pub sm_count: i32,
    pub kernel_launches: i64,
    pub graph_captures: i64,
}

/// Opaque handle.
#[repr(C)]
pub struct gb_moe {
    _private: [u8; 0],
}

#[repr(C)]
#[derive(Clone, Copy)]
pub struct gb_decoder_layer {
    pub attn_norm: *const f32,
    pub post_attn_norm: *const f32,
    pub wq: *const u16,
    pub wk: *const u16,
    pub wv: *const u16,
    pub wo: *const u16,
    pub bq: *const f32,
    pub bk: *const f32,
    pub bv: *const f32,
    pub bo: *const f32,
    pub sinks: *const f32,
    pub sliding: i32,
    pub moe: *const gb_moe_desc,
}

#[repr(C)]
#[derive(Clone, Copy)]
pub struct gb_decoder_desc {
    pub struct_size: u32,
    pub n_layers: i32,
    pub hidden: i32,
    pub n_heads: i32,
    pub n_kv_heads: i32,
    pub head_dim: i32,
    pub vocab: i32,
    pub sliding_window: i32,
    pub max_seq_len: i32,
    pub max_batch: i32,
    pub max_tokens: i32,
    pub rope_theta: f32,
    pub rope_scaling_factor: f32,
    pub rope_orig_ctx: i32,
    pub rope_beta_fast: f32,
    pub rope_beta_slow: f32,
    pub rms_eps: f32,
    pub device: i32,
    pub embed: *const u16,
    pub lm_head: *const u16,
    pub final_norm: *const f32,
    pub layers: *const gb_decoder_layer,
}

impl Default for gb_decoder_desc {
    /// Zeroed, with struct_size set, as the header asks.
    fn default() -> Self {
        // SAFETY: every field is an integer, a float or a raw pointer, for
        // which all-zero bytes are valid (null pointers).
        let mut d: Self = unsafe { std::mem::zeroed() };
        d.struct_size = std::mem::size_of::<Self>() as u32;
        d
    }
}

/// Opaque decoder handle.
#[repr(C)]
pub struct gb_decoder {
    _private: [u8; 0],
}

extern "C" {
    pub fn gb_moe_create(desc: *const gb_moe_desc, out: *mut *mut gb_moe) -> c_int;
    pub fn gb_moe_forward(m: *mut gb_moe, x_dev: *const f32, t: i64, out_dev: *mut f32,
                          stream: *mut c_void) -> c_int;
    pub fn gb_moe_forward_host(m: *mut gb_moe, x_host: *const f32, t: i64, out_host: *mut f32,
                               stream: *mut c_void) -> c_int;
    pub fn gb_moe_route(m: *mut gb_moe, x_dev: *const f32, t: i64, idx_dev: *mut i32,
                        w_dev: *mut f32, counts_dev: *mut i32, offsets_dev: *mut i32,
                        perm_dev: *mut i32, stream: *mut c_void) -> c_int;
    pub fn gb_moe_dequant_expert(m: *mut gb_moe, which: i32, expert: i32, out_dev: *mut f32,
                                 stream: *mut c_void) -> c_int;
    pub fn gb_moe_get_info(m: *const gb_moe, info: *mut gb_moe_info) -> c_int;
    pub fn gb_moe_device_status(m: *mut gb_moe, stream: *mut c_void) -> c_int;
    pub fn gb_moe_set_expert_path(m: *mut gb_moe, path: i32) -> c_int;
    pub fn gb_moe_set_graphs(m: *mut gb_moe, max_graphs: i32) -> c_int;
    pub fn gb_moe_set_test_hooks(m: *mut gb_moe, wait_limit_us: i64, withhold_ready: i32)
        -> c_int;
    pub fn gb_moe_set_profiling(m: *mut gb_moe, enable: c_int) -> c_int;
    pub fn gb_moe_stage_times(m: *mut gb_moe, ms_out: *mut f32, capacity: i32,
                              n_stages: *mut i32) -> c_int;
    pub fn gb_moe_stage_name(stage: i32) -> *const c_char;
    pub fn gb_moe_destroy(m: *mut gb_moe) -> c_int;
    pub fn gb_route_noalloc(x_dev: *const f32, router_weight_dev: *const f32,
                            router_bias_dev: *const f32, selection_bias_dev: *const f32, t: i64,
                            hidden: i32, n_experts: i32, top_k: i32, router_kind: i32,
                            idx_dev: *mut i32, w_dev: *mut f32, stream: *mut c_void) -> c_int;
    pub fn gb_decoder_create(desc: *const gb_decoder_desc, out: *mut *mut gb_decoder) -> c_int;
    pub fn gb_decoder_forward(d: *mut gb_decoder, tokens_dev: *const i32, b: i32, t: i32,
                              pos: i64, logits_dev: *mut f32, next_dev: *mut i32,
                              stream: *mut c_void) -> c_int;
    pub fn gb_decoder_generate(d: *mut gb_decoder, tokens_dev: *const i32, b: i32, pos: i64,
                               n_steps: i32, out_dev: *mut i32, stream: *mut c_void) -> c_int;
    pub fn gb_decoder_reset(d: *mut gb_decoder) -> c_int;
    pub fn gb_decoder_set_profiling(d: *mut gb_decoder, enable: i32) -> c_int;
    pub fn gb_decoder_stage_times(d: *mut gb_decoder, ms_out: *mut f32, stream: *mut c_void)
        -> c_int;
    pub fn gb_decoder_device_status(d: *mut gb_decoder, stream: *mut c_void) -> c_int;
    pub fn gb_decoder_destroy(d: *mut gb_decoder) -> c_int;
    pub fn gb_nccl_unique_id(out: *mut u8) -> c_int;
    pub fn gb_last_error() -> *const c_char;
    pub fn gb_abi_version() -> c_int;
}
