//! The candle-facing blocks: drop-in replacements for the structs the models
//! call.  Each `load` takes the tensors the reference's `load` reads (as
//! candle tensors on the CPU, e.g. from its VarBuilder or GGUF reader) and
//! `forward` keeps the reference's contract: (batch, seq, hidden) in, the
//! same shape out in x's dtype, f32 compute, the residual add left to the
//! caller (gpt_oss.rs:169, :230, :385).

use candle_core::{DType, Device, Result, Storage, Tensor};

use crate::{ffi, GalliumError, MoeBlock};

fn cerr(e: GalliumError) -> candle_core::Error {
    candle_core::Error::Msg(e.to_string())
}

/// Host bytes of a CPU tensor (weights handed to gb_moe_create).
fn host_u8(t: &Tensor) -> Result<Vec<u8>> {
    t.flatten_all()?.to_vec1::<u8>()
}

fn host_f32(t: &Tensor) -> Result<Vec<f32>> {
    t.to_dtype(DType::F32)?.flatten_all()?.to_vec1::<f32>()
}

/// The forward every block shares: flatten (batch, seq) into tokens, f32,
/// run on the tensor's device, reshape and cast back.
fn run(block: &MoeBlock, x: &Tensor) -> Result<Tensor> {
    let (b, seq, hidden) = x.dims3()?;
    let t = b * seq;
    let xf = x.reshape((t, hidden))?.to_dtype(DType::F32)?.contiguous()?;
    let out = match x.device() {
        Device::Cpu => {
            let xv = xf.flatten_all()?.to_vec1::<f32>()?;
            let mut ov = vec![0f32; xv.len()];
            block.forward_host(&xv, &mut ov).map_err(cerr)?;
            Tensor::from_vec(ov, (t, hidden), &Device::Cpu)?
        }
        Device::Cuda(dev) => {
            let out = Tensor::zeros((t, hidden), DType::F32, x.device())?;
            {
                let (xs, xl) = xf.storage_and_layout();
                let (os, _) = out.storage_and_layout();
                let (Storage::Cuda(xs), Storage::Cuda(os)) = (&*xs, &*os) else {
                    candle_core::bail!("expected CUDA storage");
                };
                use candle_core::cuda_backend::cudarc::driver::DevicePtr;
                let xp = (*xs.as_cuda_slice::<f32>()?.device_ptr() as usize
                    + xl.start_offset() * 4) as *const f32;
                let op = *os.as_cuda_slice::<f32>()?.device_ptr() as *mut f32;
                let stream = *dev.cu_stream() as *mut std::os::raw::c_void;
                // SAFETY: xp / op address t * hidden floats of live CUDA storage
                // on the block's device; candle's stream orders the work.
                unsafe { block.forward_device(xp, t as i64, op, stream) }.map_err(cerr)?;
                block.device_status(stream).map_err(cerr)?;
            }
            out
        }
        _ => candle_core::bail!("gallium-b200 runs on CUDA (or host buffers from the CPU)"),
    };
    out.reshape((b, seq, hidden))?.to_dtype(x.dtype())
}

/// Safetensors GPT-OSS MoE block (gpt_oss.rs:97-231).
pub struct OssMoEFFN {
    block: MoeBlock,
}

impl OssMoEFFN {
    /// The tensors OssMoEFFN::load reads (gpt_oss.rs:115-142), on the CPU:
    /// router weight [E, H] and bias [E], gate_up_proj_blocks [E, 2I, H/32, 16],
    /// _scales [E, 2I, H/32], _bias [E, 2I], down_proj_* likewise.
    #[allow(clippy::too_many_arguments)]
    pub fn load(hidden: usize, inter: usize, n_experts: usize, top_k: usize, swiglu_limit: f32,
                router_w: &Tensor, router_b: &Tensor, gu_blocks: &Tensor, gu_scales: &Tensor,
                gu_bias: &Tensor, dn_blocks: &Tensor, dn_scales: &Tensor, dn_bias: &Tensor,
                device: i32, max_tokens: i32) -> Result<Self> {
        let (rw, rb) = (host_f32(router_w)?, host_f32(router_b)?);
        let (gub, dnb) = (host_f32(gu_bias)?, host_f32(dn_bias)?);
        let (gbk, gsc, dbk, dsc) =
            (host_u8(gu_blocks)?, host_u8(gu_scales)?, host_u8(dn_blocks)?, host_u8(dn_scales)?);
        let mut d = ffi::gb_moe_desc::default();
        d.hidden = hidden as i32;
        d.inter = inter as i32;
        d.n_experts = n_experts as i32;
        d.top_k = top_k as i32;
        d.router_kind = ffi::GB_ROUTER_SOFTMAX_TOPK;
        d.act_kind = ffi::GB_ACT_GPTOSS_CLAMP;
        d.weight_format = ffi::GB_FMT_MXFP4_SPLIT;
        d.swiglu_limit = swiglu_limit;
        d.device = device;
        d.max_tokens = max_tokens;
        d.ep_size = 1;
        d.router_weight = rw.as_ptr().cast();
        d.router_bias = rb.as_ptr().cast();
        d.router_dtype = ffi::GB_DTYPE_F32;
        d.gate_up_blocks = gbk.as_ptr();
        d.gate_up_scales = gsc.as_ptr();
        d.down_blocks = dbk.as_ptr();
        d.down_scales = dsc.as_ptr();
        d.gate_up_bias = gub.as_ptr().cast();
        d.down_bias = dnb.as_ptr().cast();
        d.bias_dtype = ffi::GB_DTYPE_F32;
        Ok(Self { block: MoeBlock::create(&d).map_err(cerr)? })
    }

    pub fn forward(&self, x: &Tensor) -> Result<Tensor> {
        run(&self.block, x)
    }
}

/// GGUF MoE block with quantised expert tensors: GPT-OSS (QMoEFFN,
/// gpt_oss_q.rs:119-269, MXFP4 type 39, biases, clamped SwiGLU) or LFM2.5
/// (QMoEFFN, lfm2moe_q.rs:203-313, Q4_K, sigmoid router with selection bias,
/// SiLU).
pub struct QMoEFFN {
    block: MoeBlock,
}

impl QMoEFFN {
    /// desc: a descriptor filled by the caller from the GGUF tensors (raw
    /// block bytes in gate_raw / up_raw / down_raw, f32 router and biases);
    /// see include/gallium_b200.h for each field.
    pub fn load(desc: &ffi::gb_moe_desc) -> Result<Self> {
        Ok(Self { block: MoeBlock::create(desc).map_err(cerr)? })
    }

    pub fn forward(&self, x: &Tensor) -> Result<Tensor> {
        run(&self.block, x)
    }
}

/// gallium-core's generic MoEFFN (ffn.rs:72-166) and Gemma-4's routed experts
/// (gemma4_q.rs:187-330) load the same way from a filled descriptor
/// (GB_FMT_DENSE with the shared expert; gate_up_merged, expert_scale and the
/// norms for Gemma-4).
pub type MoEFFN = QMoEFFN;
pub type QGemmaMoe = QMoEFFN;
