//! Raw declarations of the C ABI in include/gguf_cuda.h (one per exported symbol).
//! Every function returns a status (0 = ok, else a GgufError variant code, see
//! `crate::Status`) unless it returns a count or a handle.
#![allow(non_camel_case_types)]

use std::os::raw::{c_char, c_int, c_void};

#[repr(C)]
pub struct ggc_ctx {
    _p: [u8; 0],
}
#[repr(C)]
pub struct ggc_model {
    _p: [u8; 0],
}
#[repr(C)]
pub struct ggc_tensor {
    _p: [u8; 0],
}

#[repr(C)]
#[derive(Clone, Copy)]
pub struct ggc_error_info {
    pub status: c_int,
    pub dtype: [c_char; 16],
    pub expected: u64,
    pub actual: u64,
    pub elements: u64,
    pub block: u64,
    pub message: [c_char; 256],
}

#[repr(C)]
#[derive(Clone, Copy, Default)]
pub struct ggc_hparams {
    pub vocab_size: u32,
    pub embed_dim: u32,
    pub n_heads: u32,
    pub n_kv_heads: u32,
    pub ffn_dim: u32,
    pub n_layers: u32,
    pub rope_freq_base: f64,
    pub max_ctx: u32,
    pub kv_f16: u32,
}

#[repr(C)]
#[derive(Clone, Copy)]
pub struct ggc_tensor_desc {
    pub data: *const c_void,
    pub nbytes: u64,
    pub dtype: c_int,
    pub n_elements: u64,
}

#[repr(C)]
#[derive(Clone, Copy, Default)]
pub struct ggc_tp_shard {
    pub head0: u32,
    pub heads: u32,
    pub kv_head0: u32,
    pub kv_heads: u32,
    pub ffn0: u64,
    pub ffn_len: u64,
}

#[repr(C)]
#[derive(Clone, Copy)]
pub struct ggc_sampler_config {
    pub temperature: f32,
    pub top_k: u32,
    pub top_p: f32,
    pub min_p: f32,
    pub repeat_penalty: f32,
}

extern "C" {
    pub fn ggc_last_error(out: *mut ggc_error_info) -> c_int;
    pub fn ggc_block_size(dtype: c_int) -> i64;
    pub fn ggc_block_bytes(dtype: c_int) -> i64;

    pub fn ggc_ctx_create(device: c_int, out: *mut *mut ggc_ctx) -> c_int;
    pub fn ggc_ctx_create_tp(device: c_int, rank: c_int, world: c_int, nccl_id: *const c_void,
                             out: *mut *mut ggc_ctx) -> c_int;
    pub fn ggc_nccl_unique_id(out128: *mut c_void) -> c_int;
    pub fn ggc_ctx_destroy(ctx: *mut ggc_ctx) -> c_int;
    pub fn ggc_ctx_stream(ctx: *mut ggc_ctx) -> *mut c_void;
    pub fn ggc_ctx_synchronize(ctx: *mut ggc_ctx) -> c_int;
    pub fn ggc_ctx_kernel_launches(ctx: *mut ggc_ctx) -> u64;

    // quant.rs
    pub fn ggc_dequantize(ctx: *mut ggc_ctx, dtype: c_int, raw: *const c_void, raw_len: u64, n: u64,
                          out: *mut f32) -> c_int;
    pub fn ggc_quant_matvec(ctx: *mut ggc_ctx, dtype: c_int, w: *const c_void, w_len: u64, rows: u64,
                            cols: u64, x: *const f32, x_len: u64, y: *mut f32, y_len: u64) -> c_int;
    pub fn ggc_quant_matvec_static(dtype: c_int, w: *const c_void, w_len: u64, rows: u64, cols: u64,
                                   x: *const f32, x_len: u64, y: *mut f32, y_len: u64,
                                   stream: *mut c_void) -> c_int;

    // uploaded tensors
    pub fn ggc_tensor_upload(ctx: *mut ggc_ctx, raw: *const c_void, bytes: u64, dtype: c_int, ne: *const u64,
                             ndim: c_int, repack: c_int, out: *mut *mut ggc_tensor) -> c_int;
    pub fn ggc_tensor_free(t: *mut ggc_tensor) -> c_int;
    pub fn ggc_tensor_matvec(ctx: *mut ggc_ctx, t: *const ggc_tensor, x: *const f32, y: *mut f32) -> c_int;
    pub fn ggc_tensor_matvec_batch(ctx: *mut ggc_ctx, ts: *const *const ggc_tensor, n: u64, x: *const f32,
                                   y: *mut f32) -> c_int;
    pub fn ggc_tensor_dequantize(ctx: *mut ggc_ctx, t: *const ggc_tensor, out: *mut f32) -> c_int;
    pub fn ggc_tensor_matmul(ctx: *mut ggc_ctx, t: *const ggc_tensor, x: *const f32, m: u64, y: *mut f32) -> c_int;
    pub fn ggc_infer_k_quant_dtype(span: u64, n: u64, marked: c_int) -> c_int;

    // ops.rs standalone functions
    pub fn ggc_ops_matvec(ctx: *mut ggc_ctx, a: *const f32, a_len: u64, rows: u64, cols: u64, x: *const f32,
                          x_len: u64, y: *mut f32, y_len: u64, b: *const f32) -> c_int;
    pub fn ggc_ops_matvec_colmajor(ctx: *mut ggc_ctx, a: *const f32, a_len: u64, rows: u64, cols: u64,
                                   x: *const f32, x_len: u64, y: *mut f32, y_len: u64, b: *const f32) -> c_int;
    pub fn ggc_ops_matvec_colmajor_trans(ctx: *mut ggc_ctx, a: *const f32, a_len: u64, dim0: u64, dim1: u64,
                                         x: *const f32, x_len: u64, y: *mut f32, y_len: u64,
                                         b: *const f32) -> c_int;
    pub fn ggc_ops_matmul(ctx: *mut ggc_ctx, a: *const f32, a_len: u64, ra: u64, ca: u64, b: *const f32,
                          b_len: u64, cb: u64, c: *mut f32, c_len: u64) -> c_int;
    pub fn ggc_ops_silu(ctx: *mut ggc_ctx, x: *mut f32, n: u64) -> c_int;
    pub fn ggc_ops_gelu(ctx: *mut ggc_ctx, x: *mut f32, n: u64) -> c_int;
    pub fn ggc_ops_rmsnorm(ctx: *mut ggc_ctx, x: *mut f32, n: u64, w: *const f32, w_len: u64, eps: f32) -> c_int;
    pub fn ggc_ops_layernorm(ctx: *mut ggc_ctx, x: *mut f32, n: u64, w: *const f32, w_len: u64, b: *const f32,
                             b_len: u64, eps: f32) -> c_int;
    pub fn ggc_ops_softmax(ctx: *mut ggc_ctx, x: *mut f32, n: u64) -> c_int;
    pub fn ggc_ops_rope(ctx: *mut ggc_ctx, x: *mut f32, n_x: u64, positions: *const i64, n_pos: u64,
                        freqs: *const f32, n_freqs: u64) -> c_int;

    // model/llama.rs, cache.rs, engine.rs
    pub fn ggc_tp_plan(hp: *const ggc_hparams, attn_output_dtype: c_int, ffn_down_dtype: c_int, rank: c_int,
                       world: c_int, out: *mut ggc_tp_shard) -> c_int;
    pub fn ggc_model_create(ctx: *mut ggc_ctx, hp: *const ggc_hparams, tensors: *const ggc_tensor_desc,
                            n_tensors: u64, out: *mut *mut ggc_model) -> c_int;
    pub fn ggc_model_destroy(m: *mut ggc_model) -> c_int;
    pub fn ggc_model_forward(m: *mut ggc_model, tokens: *const u32, positions: *const i64, n: u64,
                             logits: *mut f32, argmax: *mut u32) -> c_int;
    pub fn ggc_model_cache_len(m: *const ggc_model) -> u64;
    pub fn ggc_model_reset_cache(m: *mut ggc_model) -> c_int;
    pub fn ggc_model_truncate(m: *mut ggc_model, new_len: u64) -> c_int;
    pub fn ggc_model_cache_append(m: *mut ggc_model, layer: u32, k: *const f32, v: *const f32, seq: u64) -> c_int;
    pub fn ggc_model_cache_read(m: *mut ggc_model, layer: u32, k: *mut f32, v: *mut f32) -> c_int;
    pub fn ggc_model_generate_greedy(m: *mut ggc_model, prompt: *const u32, n_prompt: u64, start_pos: i64,
                                     max_tokens: u64, eos: i64, out_ids: *mut u32, n_out: *mut u64) -> c_int;
    pub fn ggc_model_decode(m: *mut ggc_model, steps: u64, eos: i64, sync: c_int, out_ids: *mut u32,
                            n_out: *mut u64) -> c_int;
    pub fn ggc_model_wait(m: *mut ggc_model, out_ids: *mut u32, n_out: *mut u64) -> c_int;
    pub fn ggc_model_allreduce_kind(m: *const ggc_model) -> c_int;

    // sampler.rs
    pub fn ggc_sample(ctx: *mut ggc_ctx, logits: *const f32, vocab: u64, cfg: *const ggc_sampler_config,
                      seen: *const u32, n_seen: u64, u: f32, out_id: *mut u32) -> c_int;
    pub fn ggc_model_sample(m: *mut ggc_model, cfg: *const ggc_sampler_config, seen: *const u32, n_seen: u64,
                            u: f32, out_id: *mut u32) -> c_int;

    // the fused all-reduce's bounded wait, on one GPU
    pub fn ggc_allreduce_probe(ctx: *mut ggc_ctx, rows: u32, peer_writes: c_int, part0: *const f32,
                               part1: *const f32, out: *mut f32) -> c_int;
}
