//! Raw bindings of include/gallium_b200.h (ABI version 3).  Field order and
//! types follow the header exactly; tests/test_rust_binding.py checks them.
#![allow(non_camel_case_types)]

use std::os::raw::{c_char, c_int, c_void};

pub const GB_ABI_VERSION: c_int = 3;

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
    pub fn gb_nccl_unique_id(out: *mut u8) -> c_int;
    pub fn gb_last_error() -> *const c_char;
    pub fn gb_abi_version() -> c_int;
}
