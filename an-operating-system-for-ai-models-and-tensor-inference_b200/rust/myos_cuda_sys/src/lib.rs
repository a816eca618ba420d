//! Bindings to libmyos_cuda, the B200 (sm_100a) Qwen2.5 BF16 token loop, for
//! the MyOS workspace.
//!
//! `ffi` mirrors `include/myos_cuda.h` one to one (same names, argument
//! order and types; plain pointers and sizes). The rest of the crate is the
//! safe layer a `model_core` / `weight_loader` caller switches to: the same
//! operations as `model_core::prefill` / `forward_token` / `greedy_decode` and
//! `KvCache::len` / `clear` (crates/model_core/src/qwen25_block.rs:220,323,765,
//! kv_cache.rs:140-142,234-237) and `SafeTensorsMmap::open`
//! (crates/weight_loader/src/mmap.rs:82-100), with the status codes mapped to
//! one error enum whose variants carry the reference enums' names. As in the
//! reference, a failed call leaves the KV cursor and the logits unchanged.

#![allow(non_camel_case_types)]

use std::ffi::{CStr, CString};
use std::os::raw::{c_char, c_int, c_void};
use std::path::Path;

pub mod ffi {
    use super::*;

    pub const MYOS_OK: c_int = 0;
    pub const MYOS_ERR_SHAPE: c_int = 1;
    pub const MYOS_ERR_TOKEN: c_int = 2;
    pub const MYOS_ERR_ROW_OOB: c_int = 3;
    pub const MYOS_ERR_POSITION: c_int = 4;
    pub const MYOS_ERR_CACHE_FULL: c_int = 5;
    pub const MYOS_ERR_CACHE_RANGE: c_int = 6;
    pub const MYOS_ERR_WEIGHT_MISSING: c_int = 7;
    pub const MYOS_ERR_WEIGHT_DTYPE: c_int = 8;
    pub const MYOS_ERR_WEIGHT_SHAPE: c_int = 9;
    pub const MYOS_ERR_WEIGHT_LENGTH: c_int = 10;
    pub const MYOS_ERR_DUPLICATE: c_int = 11;
    pub const MYOS_ERR_EMPTY_NAME: c_int = 12;
    pub const MYOS_ERR_PARSE: c_int = 13;
    pub const MYOS_ERR_UNSUPPORTED: c_int = 14;
    pub const MYOS_ERR_IO: c_int = 15;
    pub const MYOS_ERR_CUDA: c_int = 16;
    pub const MYOS_ERR_NCCL: c_int = 17;
    pub const MYOS_ERR_TIMEOUT: c_int = 18;
    pub const MYOS_ERR_ARG: c_int = 19;
    pub const MYOS_ERR_SCRATCH_LIMIT: c_int = 20;

    pub const MYOS_F32: i32 = 0;
    pub const MYOS_F16: i32 = 1;
    pub const MYOS_BF16: i32 = 2;
    pub const MYOS_KV_F32: i32 = 0;
    pub const MYOS_KV_BF16: i32 = 1;
    pub const MYOS_NOALLOC_SCRATCH_BYTES: usize = 2 << 20;

    #[repr(C)]
    #[derive(Clone, Copy, Debug, Default, PartialEq)]
    pub struct myos_shape {
        pub hidden: u32,
        pub num_q_heads: u32,
        pub num_kv_heads: u32,
        pub head_dim: u32,
        pub rope_theta: f32,
        pub intermediate: u32,
        pub vocab: u32,
        pub num_layers: u32,
        pub rms_eps: f32,
        pub tied_head: u32,
    }

    #[repr(C)]
    #[derive(Clone, Copy, Debug, Default, PartialEq)]
    pub struct myos_opts {
        pub device: i32,
        pub max_seq: u32,
        pub kv_dtype: i32,
        pub use_graphs: i32,
    }

    #[repr(C)]
    #[derive(Clone, Copy)]
    pub struct myos_tp {
        pub size: i32,
        pub rank: i32,
        pub unique_id: [u8; 128],
    }

    #[repr(C)]
    #[derive(Clone, Copy, Debug, Default, PartialEq)]
    pub struct myos_tp_part {
        pub rows: u64,
        pub cols: u64,
        pub row0: u64,
        pub nrows: u64,
        pub col0: u64,
        pub ncols: u64,
        pub store_rows: u64,
        pub store_cols: u64,
        pub matrix: i32,
        pub kept: i32,
    }

    #[repr(C)]
    pub struct myos_ctx {
        _private: [u8; 0],
    }

    #[link(name = "myos_cuda")]
    extern "C" {
        pub fn myos_shape_qwen25_1_5b() -> myos_shape;
        pub fn myos_shape_qwen25_14b() -> myos_shape;
        pub fn myos_ctx_create(shape: *const myos_shape, opts: *const myos_opts, out: *mut *mut myos_ctx) -> c_int;
        pub fn myos_ctx_destroy(ctx: *mut myos_ctx);
        pub fn myos_tp_unique_id(out: *mut u8) -> c_int;
        pub fn myos_tp_slice(shape: *const myos_shape, size: i32, rank: i32, name: *const c_char, out: *mut myos_tp_part) -> c_int;
        pub fn myos_tp_reduce_selftest(device: i32, n: u32, h: u32, fill: i32, timeout_ms: u32, out: *mut f32) -> c_int;
        pub fn myos_ctx_create_tp(shape: *const myos_shape, opts: *const myos_opts, tp: *const myos_tp, out: *mut *mut myos_ctx) -> c_int;
        pub fn myos_last_error(ctx: *const myos_ctx) -> *const c_char;
        pub fn myos_load_tensor(ctx: *mut myos_ctx, name: *const c_char, dtype: i32, shape: *const i64, rank: i32, bytes: *const c_void, nbytes: usize) -> c_int;
        pub fn myos_load_safetensors(ctx: *mut myos_ctx, path: *const c_char) -> c_int;
        pub fn myos_check_safetensors(path: *const c_char, n_tensors: *mut usize, err: *mut c_char, err_len: usize) -> c_int;
        pub fn myos_weights_ready(ctx: *mut myos_ctx) -> c_int;
        pub fn myos_prefill(ctx: *mut myos_ctx, ids: *const u32, n: usize, logits: *mut f32) -> c_int;
        pub fn myos_forward_token(ctx: *mut myos_ctx, token: u32, pos: usize, logits: *mut f32) -> c_int;
        pub fn myos_greedy_decode(ctx: *mut myos_ctx, steps: usize, out_ids: *mut u32) -> c_int;
        pub fn myos_forced_decode(ctx: *mut myos_ctx, ids: *const u32, steps: usize, argmax_out: *mut u32) -> c_int;
        pub fn myos_kv_len(ctx: *const myos_ctx, len: *mut usize) -> c_int;
        pub fn myos_reset(ctx: *mut myos_ctx) -> c_int;
        pub fn myos_kv_head(ctx: *mut myos_ctx, layer: u32, head: u32, pos: usize, k: *mut f32, v: *mut f32) -> c_int;
        pub fn myos_logits(ctx: *mut myos_ctx, out: *mut f32) -> c_int;
        pub fn myos_profile_kernels(ctx: *mut myos_ctx, iters: c_int, ms_out: *mut f32, bytes_out: *mut f64) -> c_int;
        pub fn myos_last_timing(ctx: *const myos_ctx, prefill_ms: *mut f32, decode_ms: *mut f32) -> c_int;
        pub fn myos_launch_count(out: *mut u64) -> c_int;
        pub fn myos_gemv_bf16(y: *mut f32, y_len: usize, w: *const u8, w_len: usize, x: *const f32, x_len: usize, m: usize, k: usize) -> c_int;
        pub fn myos_rmsnorm_bf16_weight(y: *mut f32, y_len: usize, w: *const u8, w_len: usize, x: *const f32, x_len: usize, eps: f32) -> c_int;
        pub fn myos_gqa_attn_f32(y: *mut f32, y_len: usize, q: *const f32, q_len: usize, k: *const f32, k_len: usize, v: *const f32, v_len: usize, num_q_heads: usize, num_kv_heads: usize, head_dim: usize, seq_len: usize, mask_kind: i32, query_pos: usize) -> c_int;
        pub fn myos_swiglu_mul_f32(h: *mut f32, h_len: usize, gate: *const f32, gate_len: usize, up: *const f32, up_len: usize) -> c_int;
        pub fn myos_rope_f32(y: *mut f32, y_len: usize, x: *const f32, x_len: usize, position: u32, head_dim: usize, theta: f32) -> c_int;
        pub fn myos_greedy_token(logits: *const f32, n: usize, out: *mut u32) -> c_int;
        pub fn myos_dev_gemv_bf16(d_y: *mut f32, d_w: *const c_void, d_x: *const f32, m: usize, k: usize, stream: *mut c_void) -> c_int;
        pub fn myos_batch_generate(ctx: *mut myos_ctx, nseq: usize, ids: *const u32, lens: *const u32, steps: usize, out_ids: *mut u32) -> c_int;
        pub fn myos_batch_forced_decode(ctx: *mut myos_ctx, nseq: usize, ids: *const u32, lens: *const u32, steps: usize, feed: *const u32, argmax_out: *mut u32, logits: *mut f32) -> c_int;
        pub fn myos_dev_gqa_attn_f32_noalloc(d_y: *mut f32, d_q: *const f32, d_k: *const f32, d_v: *const f32, hq: usize, hkv: usize, d: usize, seq: usize, mask_kind: i32, query_pos: usize, stream: *mut c_void) -> c_int;
        pub fn myos_version() -> *const c_char;
    }
}

/// Errors of the reference crates on this path (model_core::BlockError,
/// KvError, QwenBf16Error, weight_loader::WeightError / WeightFileError,
/// tensor_core::Bf16OpError), plus the device-side failures.
#[derive(Debug, Clone, PartialEq, Eq)]
pub enum Error {
    Shape(String),
    Token(String),
    RowOutOfBounds(String),
    Position(String),
    CacheFull(String),
    CacheRange(String),
    WeightMissing(String),
    WeightDType(String),
    WeightShape(String),
    WeightLength(String),
    Duplicate(String),
    EmptyName(String),
    Parse(String),
    UnsupportedDType(String),
    Io(String),
    Cuda(String),
    Nccl(String),
    Timeout(String),
    Arg(String),
    ScratchLimit(String),
}

fn status(code: c_int, msg: String) -> Result<(), Error> {
    use ffi::*;
    match code {
        MYOS_OK => Ok(()),
        MYOS_ERR_SHAPE => Err(Error::Shape(msg)),
        MYOS_ERR_TOKEN => Err(Error::Token(msg)),
        MYOS_ERR_ROW_OOB => Err(Error::RowOutOfBounds(msg)),
        MYOS_ERR_POSITION => Err(Error::Position(msg)),
        MYOS_ERR_CACHE_FULL => Err(Error::CacheFull(msg)),
        MYOS_ERR_CACHE_RANGE => Err(Error::CacheRange(msg)),
        MYOS_ERR_WEIGHT_MISSING => Err(Error::WeightMissing(msg)),
        MYOS_ERR_WEIGHT_DTYPE => Err(Error::WeightDType(msg)),
        MYOS_ERR_WEIGHT_SHAPE => Err(Error::WeightShape(msg)),
        MYOS_ERR_WEIGHT_LENGTH => Err(Error::WeightLength(msg)),
        MYOS_ERR_DUPLICATE => Err(Error::Duplicate(msg)),
        MYOS_ERR_EMPTY_NAME => Err(Error::EmptyName(msg)),
        MYOS_ERR_PARSE => Err(Error::Parse(msg)),
        MYOS_ERR_UNSUPPORTED => Err(Error::UnsupportedDType(msg)),
        MYOS_ERR_IO => Err(Error::Io(msg)),
        MYOS_ERR_NCCL => Err(Error::Nccl(msg)),
        MYOS_ERR_TIMEOUT => Err(Error::Timeout(msg)),
        MYOS_ERR_ARG => Err(Error::Arg(msg)),
        MYOS_ERR_SCRATCH_LIMIT => Err(Error::ScratchLimit(msg)),
        _ => Err(Error::Cuda(msg)),
    }
}

pub use ffi::{myos_opts as Opts, myos_shape as BlockShape};

impl BlockShape {
    /// `BlockShape::qwen25_1_5b()` (qwen25_block.rs:63-74).
    pub fn qwen25_1_5b() -> Self {
        unsafe { ffi::myos_shape_qwen25_1_5b() }
    }
    pub fn qwen25_14b() -> Self {
        unsafe { ffi::myos_shape_qwen25_14b() }
    }
}

/// Weights, KV cache and workspace of one model on one GPU (the reference's
/// `KvCache` + `BlockWorkspace` + borrowed `WeightMap`, held in HBM).
pub struct Engine {
    ctx: *mut ffi::myos_ctx,
    vocab: usize,
}

unsafe impl Send for Engine {}

impl Engine {
    /// `KvCache::new` + `BlockWorkspace::new` on `opts.device`.
    pub fn new(shape: &BlockShape, opts: &Opts) -> Result<Self, Error> {
        let mut ctx = std::ptr::null_mut();
        let rc = unsafe { ffi::myos_ctx_create(shape, opts, &mut ctx) };
        status(rc, "context creation failed".into())?;
        Ok(Engine { ctx, vocab: shape.vocab as usize })
    }

    fn check(&self, rc: c_int) -> Result<(), Error> {
        if rc == ffi::MYOS_OK {
            return Ok(());
        }
        let msg = unsafe { CStr::from_ptr(ffi::myos_last_error(self.ctx)) }.to_string_lossy().into_owned();
        status(rc, msg)
    }

    /// `SafeTensorsMmap::open` + `MmapWeights`: stages every known tensor.
    pub fn load_safetensors(&mut self, path: &Path) -> Result<(), Error> {
        let c = CString::new(path.to_string_lossy().as_bytes()).map_err(|e| Error::Arg(e.to_string()))?;
        self.check(unsafe { ffi::myos_load_safetensors(self.ctx, c.as_ptr()) })
    }

    /// One named tensor from any `WeightMap` (bf16 bytes, little-endian).
    pub fn load_tensor(&mut self, name: &str, shape: &[i64], bytes: &[u8]) -> Result<(), Error> {
        let c = CString::new(name).map_err(|e| Error::Arg(e.to_string()))?;
        self.check(unsafe {
            ffi::myos_load_tensor(self.ctx, c.as_ptr(), ffi::MYOS_BF16, shape.as_ptr(), shape.len() as i32,
                                  bytes.as_ptr() as *const c_void, bytes.len())
        })
    }

    /// `model_core::prefill`: the prompt's logits at its last position.
    pub fn prefill(&mut self, tokens: &[u32]) -> Result<Vec<f32>, Error> {
        let mut logits = vec![0f32; self.vocab];
        self.check(unsafe { ffi::myos_prefill(self.ctx, tokens.as_ptr(), tokens.len(), logits.as_mut_ptr()) })?;
        Ok(logits)
    }

    /// `model_core::forward_token` at `pos` (must equal the cache length).
    pub fn forward_token(&mut self, token: u32, pos: usize) -> Result<Vec<f32>, Error> {
        let mut logits = vec![0f32; self.vocab];
        self.check(unsafe { ffi::myos_forward_token(self.ctx, token, pos, logits.as_mut_ptr()) })?;
        Ok(logits)
    }

    /// `model_core::greedy_decode`: `steps` ids, each the first maximum of
    /// the current logits, fed back on the device.
    pub fn greedy_decode(&mut self, steps: usize) -> Result<Vec<u32>, Error> {
        let mut out = vec![0u32; steps];
        self.check(unsafe { ffi::myos_greedy_decode(self.ctx, steps, out.as_mut_ptr()) })?;
        Ok(out)
    }

    /// `KvCache::len`.
    pub fn kv_len(&self) -> Result<usize, Error> {
        let mut n = 0usize;
        self.check(unsafe { ffi::myos_kv_len(self.ctx, &mut n) })?;
        Ok(n)
    }

    /// `KvCache::clear`.
    pub fn reset(&mut self) -> Result<(), Error> {
        self.check(unsafe { ffi::myos_reset(self.ctx) })
    }

    /// `BlockWorkspace::logits` of the last call.
    pub fn logits(&mut self) -> Result<Vec<f32>, Error> {
        let mut out = vec![0f32; self.vocab];
        self.check(unsafe { ffi::myos_logits(self.ctx, out.as_mut_ptr()) })?;
        Ok(out)
    }
}

impl Drop for Engine {
    fn drop(&mut self) {
        unsafe { ffi::myos_ctx_destroy(self.ctx) }
    }
}

/// `model_core::greedy_token` (lib.rs:157-167) on the device.
pub fn greedy_token(logits: &[f32]) -> Result<u32, Error> {
    let mut out = 0u32;
    status(unsafe { ffi::myos_greedy_token(logits.as_ptr(), logits.len(), &mut out) }, "greedy_token".into())?;
    Ok(out)
}

/// The library version string.
pub fn version() -> String {
    unsafe { CStr::from_ptr(ffi::myos_version()) }.to_string_lossy().into_owned()
}
