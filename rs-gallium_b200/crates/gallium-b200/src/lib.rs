//! gallium-b200: rs-gallium's mixture-of-experts FFN blocks on B200 (sm_100a).
//!
//! The blocks keep the signature their callers use, `fn forward(&self, x:
//! &Tensor) -> Result<Tensor>` with x of shape (batch, seq, hidden):
//!   gpt_oss.rs:384 (`layer.moe.forward(&h_norm)`), gpt_oss_q.rs:295,
//!   lfm2moe_q.rs:364, block.rs:76 through FfnImpl::forward (ffn.rs:175),
//!   and gemma4_q.rs's routed experts.
//! `load` hands the same host tensors the reference's `load` reads to
//! gb_moe_create, which copies and repacks them on the device once.
//!
//! A CUDA tensor runs through gb_moe_forward on candle's stream (device
//! pointers, asynchronous; the device status is read before returning); a CPU
//! tensor through gb_moe_forward_host.  There is no CPU fallback: errors come
//! back as candle errors carrying the library's status and message.

pub mod ffi;

use std::ffi::CStr;
use std::os::raw::c_void;
use std::ptr::NonNull;

/// A non-OK gb_status with gb_last_error()'s message.
#[derive(Debug, Clone)]
pub struct GalliumError {
    pub status: i32,
    pub message: String,
}

impl std::fmt::Display for GalliumError {
    fn fmt(&self, f: &mut std::fmt::Formatter<'_>) -> std::fmt::Result {
        write!(f, "gallium-b200 status {}: {}", self.status, self.message)
    }
}

impl std::error::Error for GalliumError {}

pub fn check(status: i32) -> Result<(), GalliumError> {
    if status == ffi::GB_OK {
        return Ok(());
    }
    // SAFETY: gb_last_error returns a NUL-terminated, thread-local string.
    let message = unsafe { CStr::from_ptr(ffi::gb_last_error()) }.to_string_lossy().into_owned();
    Err(GalliumError { status, message })
}

/// One created block (gb_moe handle).  Not re-entrant, like the reference's
/// blocks, which are borrowed mutably per generation.
pub struct MoeBlock {
    h: NonNull<ffi::gb_moe>,
    hidden: usize,
}

// The handle may move between threads; it is used by one at a time.
unsafe impl Send for MoeBlock {}

impl MoeBlock {
    /// gb_moe_create.  Every pointer in `desc` must stay valid for the call.
    pub fn create(desc: &ffi::gb_moe_desc) -> Result<Self, GalliumError> {
        let mut h = std::ptr::null_mut();
        // SAFETY: desc points at a fully initialised descriptor; h receives the handle.
        check(unsafe { ffi::gb_moe_create(desc, &mut h) })?;
        let h = NonNull::new(h).ok_or(GalliumError { status: -1, message: "null handle".into() })?;
        Ok(Self { h, hidden: desc.hidden as usize })
    }

    pub fn hidden(&self) -> usize {
        self.hidden
    }

    /// Host buffers: x [t, hidden] -> out [t, hidden], synchronous.
    pub fn forward_host(&self, x: &[f32], out: &mut [f32]) -> Result<(), GalliumError> {
        assert_eq!(x.len(), out.len());
        assert_eq!(x.len() % self.hidden, 0);
        let t = (x.len() / self.hidden) as i64;
        // SAFETY: both slices hold t * hidden floats.
        check(unsafe {
            ffi::gb_moe_forward_host(self.h.as_ptr(), x.as_ptr(), t, out.as_mut_ptr(),
                                     std::ptr::null_mut())
        })
    }

    /// Device buffers on the handle's device, asynchronous on `stream`.
    ///
    /// # Safety
    /// x_dev and out_dev must be device pointers to t * hidden floats, 16-byte
    /// aligned, valid until the stream has run the forward.
    pub unsafe fn forward_device(&self, x_dev: *const f32, t: i64, out_dev: *mut f32,
                                 stream: *mut c_void) -> Result<(), GalliumError> {
        check(ffi::gb_moe_forward(self.h.as_ptr(), x_dev, t, out_dev, stream))
    }

    /// Waits for `stream` and reports an error a kernel recorded.
    pub fn device_status(&self, stream: *mut c_void) -> Result<(), GalliumError> {
        // SAFETY: the handle is live.
        check(unsafe { ffi::gb_moe_device_status(self.h.as_ptr(), stream) })
    }

    pub fn info(&self) -> Result<ffi::gb_moe_info, GalliumError> {
        let mut info = ffi::gb_moe_info {
            struct_size: std::mem::size_of::<ffi::gb_moe_info>() as u32,
            ..Default::default()
        };
        // SAFETY: info is a writable, correctly sized struct.
        check(unsafe { ffi::gb_moe_get_info(self.h.as_ptr(), &mut info) })?;
        Ok(info)
    }
}

impl Drop for MoeBlock {
    fn drop(&mut self) {
        // SAFETY: the handle came from gb_moe_create and is destroyed once.
        unsafe { ffi::gb_moe_destroy(self.h.as_ptr()) };
    }
}

/// A fresh NCCL unique id for expert parallelism (rank 0 creates it and
/// shares the 128 bytes with the other ranks).
pub fn nccl_unique_id() -> Result<[u8; 128], GalliumError> {
    let mut id = [0u8; 128];
    // SAFETY: id has the 128 bytes the call writes.
    check(unsafe { ffi::gb_nccl_unique_id(id.as_mut_ptr()) })?;
    Ok(id)
}

#[cfg(feature = "candle")]
pub mod blocks;
