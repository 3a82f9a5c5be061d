//! Safe bindings to libgguf_cuda for the gguf crate's `infer/` module.
//!
//! The gguf crate keeps its public API (`quant::dequantize`, `quant::quant_matvec`,
//! `LlamaModel::{new, forward, forward_cached, cache_len, reset_cache}`,
//! `Engine::generate`, `Sampler::sample`) and swaps the bodies for these calls; it
//! maps `Error::status` onto its `GgufError` variants (`src/error.rs:5-58`) one to
//! one.  No CPU fallback: a missing GPU or library is an error.

pub mod ffi;

use std::ffi::CStr;
use std::os::raw::{c_int, c_void};

/// The `GgufError` variant a failing call stands for (status codes of include/gguf_cuda.h).
#[derive(Debug, Clone, Copy, PartialEq, Eq)]
pub enum Status {
    DequantError,
    InvalidTensorShape,
    MissingTensor,
    UnsupportedArchitecture,
    InferenceError,
    KvCacheOverflow,
    InvalidArgument,
    Cuda,
    Nccl,
    DeviceTimeout,
}

impl Status {
    fn from_code(code: c_int) -> Status {
        match code {
            1 => Status::DequantError,
            2 => Status::InvalidTensorShape,
            3 => Status::MissingTensor,
            4 => Status::UnsupportedArchitecture,
            6 => Status::KvCacheOverflow,
            7 => Status::InvalidArgument,
            8 => Status::Cuda,
            9 => Status::Nccl,
            10 => Status::DeviceTimeout,
            _ => Status::InferenceError,
        }
    }
}

/// A failed call: the status and the payload fields of the matching `GgufError` variant.
#[derive(Debug, Clone)]
pub struct Error {
    pub status: Status,
    pub dtype: String,
    pub expected: u64,
    pub actual: u64,
    pub elements: u64,
    pub block: u64,
    pub message: String,
}

impl std::fmt::Display for Error {
    fn fmt(&self, f: &mut std::fmt::Formatter<'_>) -> std::fmt::Result {
        write!(f, "{:?}: {}", self.status, self.message)
    }
}

impl std::error::Error for Error {}

pub type Result<T> = std::result::Result<T, Error>;

fn check(code: c_int) -> Result<()> {
    if code == 0 {
        return Ok(());
    }
    let mut e: ffi::ggc_error_info = unsafe { std::mem::zeroed() };
    unsafe { ffi::ggc_last_error(&mut e) };
    let text = |s: &[std::os::raw::c_char]| unsafe { CStr::from_ptr(s.as_ptr()) }.to_string_lossy().into_owned();
    Err(Error {
        status: Status::from_code(code),
        dtype: text(&e.dtype),
        expected: e.expected,
        actual: e.actual,
        elements: e.elements,
        block: e.block,
        message: text(&e.message),
    })
}

/// One GPU (and, under tensor parallelism, one rank of the group).
pub struct Context {
    raw: *mut ffi::ggc_ctx,
}

impl Context {
    pub fn new(device: i32) -> Result<Context> {
        let mut raw = std::ptr::null_mut();
        check(unsafe { ffi::ggc_ctx_create(device, &mut raw) })?;
        Ok(Context { raw })
    }

    /// Rank `rank` of `world` (one process per GPU); `nccl_id` is rank 0's `nccl_unique_id()`.
    pub fn new_tp(device: i32, rank: i32, world: i32, nccl_id: &[u8; 128]) -> Result<Context> {
        let mut raw = std::ptr::null_mut();
        check(unsafe { ffi::ggc_ctx_create_tp(device, rank, world, nccl_id.as_ptr().cast(), &mut raw) })?;
        Ok(Context { raw })
    }

    pub fn nccl_unique_id() -> Result<[u8; 128]> {
        let mut id = [0u8; 128];
        check(unsafe { ffi::ggc_nccl_unique_id(id.as_mut_ptr().cast()) })?;
        Ok(id)
    }

    pub fn synchronize(&self) -> Result<()> {
        check(unsafe { ffi::ggc_ctx_synchronize(self.raw) })
    }
}

impl Drop for Context {
    fn drop(&mut self) {
        unsafe { ffi::ggc_ctx_destroy(self.raw) };
    }
}

/// quant::dequantize (src/infer/quant.rs:403-448): bit-exact f32 of `n` elements.
pub fn dequantize(ctx: &Context, data: &[u8], dtype: i32, n: usize) -> Result<Vec<f32>> {
    let mut out = vec![0f32; n];
    check(unsafe {
        ffi::ggc_dequantize(ctx.raw, dtype, data.as_ptr().cast(), data.len() as u64, n as u64, out.as_mut_ptr())
    })?;
    Ok(out)
}

/// quant::quant_matvec (src/infer/quant.rs:526-570): y = W x over raw GGUF rows.
pub fn quant_matvec(ctx: &Context, w: &[u8], dtype: i32, rows: usize, cols: usize, x: &[f32], y: &mut [f32]) -> Result<()> {
    check(unsafe {
        ffi::ggc_quant_matvec(ctx.raw, dtype, w.as_ptr().cast(), w.len() as u64, rows as u64, cols as u64,
                              x.as_ptr(), x.len() as u64, y.as_mut_ptr(), y.len() as u64)
    })
}

/// Model shape (HParams, src/infer/model/hparams.rs:15-142) plus the KV cache capacity.
pub type HParams = ffi::ggc_hparams;

/// One role's tensor bytes as `GgufFile::tensor_data` returns them (`None`: an absent bias).
pub struct TensorRef<'a> {
    pub data: Option<&'a [u8]>,
    pub dtype: i32,
    pub n_elements: u64,
}

/// Sampler settings (src/infer/sampler.rs:19-37).
pub type SamplerConfig = ffi::ggc_sampler_config;

/// LlamaModel (src/infer/model/llama.rs) with its weights and KV cache in HBM.
pub struct Model<'c> {
    raw: *mut ffi::ggc_model,
    vocab: usize,
    _ctx: std::marker::PhantomData<&'c Context>,
}

impl<'c> Model<'c> {
    /// `tensors` in the role order token_embd, output_norm, output, then per layer
    /// attn_norm, attn_q, attn_q.bias, attn_k, attn_k.bias, attn_v, attn_v.bias,
    /// attn_output, ffn_norm, ffn_up, ffn_gate, ffn_down.
    pub fn new(ctx: &'c Context, hp: &HParams, tensors: &[TensorRef<'_>]) -> Result<Model<'c>> {
        let descs: Vec<ffi::ggc_tensor_desc> = tensors
            .iter()
            .map(|t| ffi::ggc_tensor_desc {
                data: t.data.map_or(std::ptr::null(), |d| d.as_ptr() as *const c_void),
                nbytes: t.data.map_or(0, |d| d.len() as u64),
                dtype: t.dtype,
                n_elements: t.n_elements,
            })
            .collect();
        let mut raw = std::ptr::null_mut();
        check(unsafe { ffi::ggc_model_create(ctx.raw, hp, descs.as_ptr(), descs.len() as u64, &mut raw) })?;
        Ok(Model { raw, vocab: hp.vocab_size as usize, _ctx: std::marker::PhantomData })
    }

    /// LlamaModel::forward / forward_cached (llama.rs:214-224): last token's logits.
    pub fn forward(&mut self, tokens: &[u32], positions: &[i64]) -> Result<Vec<f32>> {
        if tokens.len() != positions.len() {
            return Err(Error { status: Status::InferenceError, dtype: String::new(), expected: tokens.len() as u64,
                               actual: positions.len() as u64, elements: 0, block: 0,
                               message: "tokens and positions differ in length".into() });
        }
        let mut logits = vec![0f32; self.vocab];
        check(unsafe {
            ffi::ggc_model_forward(self.raw, tokens.as_ptr(), positions.as_ptr(), tokens.len() as u64,
                                   logits.as_mut_ptr(), std::ptr::null_mut())
        })?;
        Ok(logits)
    }

    /// Forward without copying the logits back (for a device-side sample).
    pub fn forward_no_logits(&mut self, tokens: &[u32], positions: &[i64]) -> Result<u32> {
        let mut argmax = 0u32;
        check(unsafe {
            ffi::ggc_model_forward(self.raw, tokens.as_ptr(), positions.as_ptr(), tokens.len() as u64,
                                   std::ptr::null_mut(), &mut argmax)
        })?;
        Ok(argmax)
    }

    pub fn cache_len(&self) -> usize {
        unsafe { ffi::ggc_model_cache_len(self.raw) as usize }
    }

    pub fn reset_cache(&mut self) -> Result<()> {
        check(unsafe { ffi::ggc_model_reset_cache(self.raw) })
    }

    pub fn truncate(&mut self, len: usize) -> Result<()> {
        check(unsafe { ffi::ggc_model_truncate(self.raw, len as u64) })
    }

    /// Engine::generate with the greedy sampler (engine.rs:83-138), the loop on the device.
    pub fn generate_greedy(&mut self, prompt: &[u32], max_tokens: usize, eos: Option<u32>) -> Result<Vec<u32>> {
        let mut out = vec![0u32; max_tokens.max(1)];
        let mut n = 0u64;
        check(unsafe {
            ffi::ggc_model_generate_greedy(self.raw, prompt.as_ptr(), prompt.len() as u64, 0, max_tokens as u64,
                                           eos.map_or(-1, |e| e as i64), out.as_mut_ptr(), &mut n)
        })?;
        out.truncate(n as usize);
        Ok(out)
    }

    /// Sampler::sample (sampler.rs:86-186) on the last forward's logits; `u` is the
    /// caller's `rng.gen_range(0.0..1.0)` draw, `seen` the ids with a count > 0.
    pub fn sample(&mut self, cfg: &SamplerConfig, seen: &[u32], u: f32) -> Result<u32> {
        let mut id = 0u32;
        check(unsafe {
            ffi::ggc_model_sample(self.raw, cfg, seen.as_ptr(), seen.len() as u64, u, &mut id)
        })?;
        Ok(id)
    }
}

impl Drop for Model<'_> {
    fn drop(&mut self) {
        unsafe { ffi::ggc_model_destroy(self.raw) };
    }
}
