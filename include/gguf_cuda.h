/*
 * gguf_cuda.h -- C ABI of libgguf_cuda.so, the B200 (sm_100a) implementation of
 * gguf-reader's quantized inference hot path.
 *
 * Every entry point is plain C: pointers, sizes and status codes, no C++ or torch
 * types.  A status code maps one-to-one onto a variant of the reference's
 * GgufError (src/error.rs:5-58); the fields of the last error are kept in
 * thread-local storage and read back with ggc_last_error().
 *
 * Threading: one CUDA stream per context.  A context (and every tensor/model made
 * from it) must not be used from two threads at the same time, like the
 * reference's `&mut self` LlamaModel (src/infer/model/llama.rs:72).
 *
 * Pointers: unless stated otherwise an array argument may be host memory or device
 * memory of the context's GPU; the library detects which (cudaPointerGetAttributes)
 * and stages host buffers through its own device buffers.
 */
#ifndef GGUF_CUDA_H
#define GGUF_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- dtype ids: GGUF on-disk ids (src/types.rs:122-160) ------------------ */
enum ggc_dtype {
    GGC_F32 = 0, GGC_F16 = 1, GGC_Q4_0 = 2, GGC_Q4_1 = 3, GGC_Q5_0 = 6, GGC_Q5_1 = 7,
    GGC_Q8_0 = 8, GGC_Q2_K = 10,
    GGC_Q3_K_S = 11,            /* GGUF "Q3_K" (id 11) maps to Q3_K_S (types.rs:134-136) */
    GGC_Q4_K = 12, GGC_Q5_K = 13, GGC_Q6_K = 14, GGC_Q8_K = 15, GGC_BF16 = 30,
    /* reachable only through the API or span re-inference (no GGUF id):        */
    GGC_Q3_K_L = 111,           /* 110-byte layout, same as Q3_K_S (quant.rs:252-255) */
    GGC_Q3_K_M = 112            /* 114-byte layout, d at byte 112 (quant.rs:247-250) */
};

/* ---- status codes = GgufError variants (src/error.rs) -------------------- */
enum ggc_status {
    GGC_OK = 0,
    GGC_ERR_DEQUANT = 1,                /* DequantError { dtype, expected, actual } */
    GGC_ERR_INVALID_TENSOR_SHAPE = 2,   /* InvalidTensorShape { name, elements, block } */
    GGC_ERR_MISSING_TENSOR = 3,         /* MissingTensor { name, kind } */
    GGC_ERR_UNSUPPORTED_ARCH = 4,       /* UnsupportedArchitecture */
    GGC_ERR_INFERENCE = 5,              /* InferenceError(String): empty input, NaN, ... */
    GGC_ERR_KV_CACHE_OVERFLOW = 6,      /* KvCacheOverflow { layer, seq_len, max_seq } */
    GGC_ERR_INVALID_ARG = 7,            /* null pointer / bad handle (no reference variant) */
    GGC_ERR_CUDA = 8,                   /* CUDA runtime failure (no reference variant) */
    GGC_ERR_NCCL = 9,                   /* NCCL failure or abort (no reference variant) */
    GGC_ERR_TIMEOUT = 10                /* a bounded device-side wait expired */
};

typedef struct ggc_error_info {
    int status;
    char dtype[16];                     /* DequantError.dtype, e.g. "Q4_K" */
    uint64_t expected, actual;          /* DequantError fields */
    uint64_t elements, block;           /* InvalidTensorShape fields */
    char message[256];
} ggc_error_info;

/* Copies the calling thread's last error; returns its status. */
int ggc_last_error(ggc_error_info* out);

/* Block geometry (src/types.rs:182-220, GgmlType::block_size / block_bytes); -1 = None. */
int64_t ggc_block_size(int dtype);
int64_t ggc_block_bytes(int dtype);

/* ---- context ------------------------------------------------------------- */
typedef struct ggc_ctx ggc_ctx;

/* One context per GPU.  `device` is the CUDA ordinal. */
int ggc_ctx_create(int device, ggc_ctx** out);
/* Tensor-parallel member: rank `rank` of `world` over NCCL.  `nccl_id` points to
 * the 128-byte ncclUniqueId made by rank 0 and shared by the caller. */
int ggc_ctx_create_tp(int device, int rank, int world, const void* nccl_id, ggc_ctx** out);
/* Fills 128 bytes with a fresh ncclUniqueId (call on rank 0 only). */
int ggc_nccl_unique_id(void* out128);
int ggc_ctx_destroy(ggc_ctx* ctx);
/* The context's CUDA stream (cudaStream_t as void*), for callers that order work. */
void* ggc_ctx_stream(ggc_ctx* ctx);
int ggc_ctx_synchronize(ggc_ctx* ctx);

/* ---- quant.rs ------------------------------------------------------------ */
/* Replaces quant::dequantize (src/infer/quant.rs:403-448): `n` elements of `dtype`
 * from `raw` (raw_len bytes) into f32 `out` (n floats).  Bit-exact with the
 * reference.  Errors: DequantError (unsupported dtype / short data),
 * InvalidTensorShape (n not a multiple of the block size). */
int ggc_dequantize(ggc_ctx* ctx, int dtype, const void* raw, uint64_t raw_len, uint64_t n, float* out);

/* Replaces quant::quant_matvec (src/infer/quant.rs:526-570): y[r] = sum_c W[r,c] x[c],
 * W raw GGUF rows (row r starts at r * row_bytes), f32 accumulation.
 * Errors follow quant.rs:534-555 in the same order. */
int ggc_quant_matvec(ggc_ctx* ctx, int dtype, const void* w, uint64_t w_len, uint64_t rows,
                     uint64_t cols, const float* x, uint64_t x_len, float* y, uint64_t y_len);

/* No counterpart in the reference (it has no allocation-free entry point).
 * The ggc_quant_matvec product for callers that must not allocate device
 * memory: w, x, y are the caller's DEVICE buffers on the current device, the
 * work is queued on `stream` (cudaStream_t as void*; NULL = legacy default
 * stream) and the call returns without synchronising.  The columns are split
 * across CTAs; partial sums and per-row-group tickets live in a 4 MiB + 32 KiB
 * file-scope device array of the library, so the call runs no cudaMalloc,
 * cudaFree or other allocating routine and needs no ggc_ctx.
 *   - rows <= 65536, else GGC_ERR_INVALID_ARG (message names the limit); the
 *     other errors are those of ggc_quant_matvec, in the same order.
 *   - The first call on each device does a one-time set-up
 *     (cudaGetSymbolAddress of the scratch, with that device current); make
 *     that first call before any stream capture on the device.  The address is
 *     cached per device for the life of the process: after a cudaDeviceReset
 *     it is stale, so do not call this entry again in that process.
 *   - Each call clears the tickets it uses (cudaMemsetAsync on `stream`).
 *   - One scratch per device: calls that overlap on a device (several streams
 *     or host threads at once) race on it; the caller serialises them.
 * Results agree with ggc_quant_matvec within f32 summation-order differences. */
int ggc_quant_matvec_static(int dtype, const void* w, uint64_t w_len, uint64_t rows, uint64_t cols,
                            const float* x, uint64_t x_len, float* y, uint64_t y_len, void* stream);

/* ---- device-resident tensors (the loader side of LlamaModel::materialize,
 *      src/infer/model/llama.rs:183-204; weights stay quantized in HBM) ------- */
typedef struct ggc_tensor ggc_tensor;

/* Uploads one GGUF tensor (ne[0] contiguous; raw in host or device memory).
 * repack != 0 stores it in the tiled layout the decode GEMVs read (a lossless
 * byte permutation, done on the GPU; with GGC_REPACK=host on host threads, which
 * needs raw in host memory). */
int ggc_tensor_upload(ggc_ctx* ctx, const void* raw, uint64_t bytes, int dtype, const uint64_t* ne,
                      int ndim, int repack, ggc_tensor** out);
int ggc_tensor_free(ggc_tensor* t);
/* y = W x for an uploaded 2-D tensor (rows = ne[1], cols = ne[0]); x, y device or host. */
int ggc_tensor_matvec(ggc_ctx* ctx, const ggc_tensor* t, const float* x, float* y);
/* y_i = W_i x for n uploaded tensors of one shape, queued back to back on the
 * context stream without synchronising (x, y device buffers; y shared).  The
 * matvec stream a decode step issues, without the host call per matrix. */
int ggc_tensor_matvec_batch(ggc_ctx* ctx, const ggc_tensor* const* ts, uint64_t n, const float* x, float* y);
/* Dequantises an uploaded tensor to f32 (n = all elements). */
int ggc_tensor_dequantize(ggc_ctx* ctx, const ggc_tensor* t, float* out);
/* ops::matmul (src/infer/ops.rs:74) with a quantized weight used transposed, as
 * every model projection uses it: y[m][rows] = x[m][cols] . W^T, W uploaded with
 * repack = 0.  Runs on the tensor cores (tcgen05, bf16 hi+lo split operands,
 * f32 accumulation; ~1e-5 relative per product).  x / y host or device. */
int ggc_tensor_matmul(ggc_ctx* ctx, const ggc_tensor* t, const float* x, uint64_t m, float* y);

/* Replaces infer_k_quant_dtype (src/infer/model/llama.rs:656-710): the real
 * storage dtype of a tensor whose physical span disagrees with its marked dtype;
 * -1 = None. */
int ggc_infer_k_quant_dtype(uint64_t span, uint64_t n, int marked);

/* ---- ops.rs standalone functions (API surface; the model fuses its own) ----
 * Host or device pointers; lengths as the reference's slices; size errors are
 * DequantError { F32, expected, actual } as in ops.rs.  Products and sums keep
 * the reference's serial order per output (its bits); silu / gelu / softmax /
 * rope use CUDA's expf / tanhf / sincosf (within a few ulp of libm). */
int ggc_ops_matvec(ggc_ctx* ctx, const float* a, uint64_t a_len, uint64_t rows, uint64_t cols, const float* x,
                   uint64_t x_len, float* y, uint64_t y_len, const float* b);            /* ops.rs:14, b: rows or NULL */
int ggc_ops_matvec_colmajor(ggc_ctx* ctx, const float* a, uint64_t a_len, uint64_t rows, uint64_t cols,
                            const float* x, uint64_t x_len, float* y, uint64_t y_len, const float* b);   /* ops.rs:121 */
int ggc_ops_matvec_colmajor_trans(ggc_ctx* ctx, const float* a, uint64_t a_len, uint64_t dim0, uint64_t dim1,
                                  const float* x, uint64_t x_len, float* y, uint64_t y_len, const float* b); /* :172 */
int ggc_ops_matmul(ggc_ctx* ctx, const float* a, uint64_t a_len, uint64_t ra, uint64_t ca, const float* b,
                   uint64_t b_len, uint64_t cb, float* c, uint64_t c_len);                   /* ops.rs:74 */
int ggc_ops_silu(ggc_ctx* ctx, float* x, uint64_t n);                                        /* ops.rs:237 */
int ggc_ops_gelu(ggc_ctx* ctx, float* x, uint64_t n);                                        /* ops.rs:250 */
int ggc_ops_rmsnorm(ggc_ctx* ctx, float* x, uint64_t n, const float* w, uint64_t w_len, float eps);   /* :262 */
int ggc_ops_layernorm(ggc_ctx* ctx, float* x, uint64_t n, const float* w, uint64_t w_len, const float* b,
                      uint64_t b_len, float eps);                                             /* ops.rs:279 */
int ggc_ops_softmax(ggc_ctx* ctx, float* x, uint64_t n);                                     /* ops.rs:295 */
int ggc_ops_rope(ggc_ctx* ctx, float* x, uint64_t n_x, const int64_t* positions, uint64_t n_pos, const float* freqs,
                 uint64_t n_freqs);                                                           /* ops.rs:318 */

/* ---- model/llama.rs ------------------------------------------------------ */
typedef struct ggc_model ggc_model;

/* HParams (src/infer/model/hparams.rs:15-37) plus the device-side limits. */
typedef struct ggc_hparams {
    uint32_t vocab_size, embed_dim, n_heads, n_kv_heads, ffn_dim, n_layers;
    double rope_freq_base;
    uint32_t max_ctx;        /* KV cache capacity in tokens (positions 0..max_ctx-1) */
    uint32_t kv_f16;         /* 0 = f32 KV cache (the reference's), 1 = f16 */
} ggc_hparams;

/* One tensor as the host parsed it (GgufFile::tensor_data, src/file.rs:205). */
typedef struct ggc_tensor_desc {
    const void* data;        /* host bytes; NULL = absent (only for the optional biases) */
    uint64_t nbytes;
    int dtype;
    uint64_t n_elements;
} ggc_tensor_desc;

/* Tensor parallelism: the shard a rank keeps of one layer (Megatron split).
 *   q heads [head0, head0 + heads): rows of attn_q (+ bias), columns of attn_output;
 *   kv heads [kv_head0, kv_head0 + kv_heads): rows of attn_k / attn_v (+ biases) and
 *     the rank's KV cache;
 *   ffn rows [ffn0, ffn0 + ffn_len) of ffn_up / ffn_gate = columns of ffn_down, split
 *     on ffn_down's block boundaries, the remainder going to the lowest ranks
 *     (Llama-2's 43 super-blocks over 2 ranks: 22 + 21).
 * token_embd, the norms and output are replicated; each rank's attn_output and
 * ffn_down products are partial sums that an NCCL all-reduce adds up.  Errors:
 * InvalidArg when world does not divide n_heads and n_kv_heads, when a rank's
 * attn_output columns are not whole blocks, or when there are fewer ffn blocks
 * than ranks. */
typedef struct ggc_tp_shard {
    uint32_t head0, heads;
    uint32_t kv_head0, kv_heads;
    uint64_t ffn0, ffn_len;
} ggc_tp_shard;
int ggc_tp_plan(const ggc_hparams* hp, int attn_output_dtype, int ffn_down_dtype, int rank, int world,
                ggc_tp_shard* out);

/* Tensors in role order: token_embd, output_norm, output, then per layer
 * attn_norm, attn_q, attn_q.bias, attn_k, attn_k.bias, attn_v, attn_v.bias,
 * attn_output, ffn_norm, ffn_up, ffn_gate, ffn_down  (3 + 12 * n_layers entries;
 * the names resolved by LlamaModel::new, src/infer/model/llama.rs:135-157).
 * Under tensor parallelism every rank passes the full tensors and keeps its shard. */
int ggc_model_create(ggc_ctx* ctx, const ggc_hparams* hp, const ggc_tensor_desc* tensors,
                     uint64_t n_tensors, ggc_model** out);
int ggc_model_destroy(ggc_model* m);

/* Replaces LlamaModel::forward / forward_cached (src/infer/model/llama.rs:214-224):
 * runs n tokens at the given positions, appending their K/V to the cache, and
 * returns the last token's logits (vocab floats) in `logits` and/or its greedy
 * argmax (last maximum wins, sampler.rs:113-123) in `argmax`; either may be NULL.
 * tokens/positions/logits/argmax may be host or device pointers. */
int ggc_model_forward(ggc_model* m, const uint32_t* tokens, const int64_t* positions, uint64_t n,
                      float* logits, uint32_t* argmax);
/* LlamaModel::cache_len (llama.rs:227-232) */
uint64_t ggc_model_cache_len(const ggc_model* m);
/* LlamaModel::reset_cache (llama.rs:235-239) */
int ggc_model_reset_cache(ggc_model* m);
/* Cache::truncate_all (src/infer/cache.rs:135-139) */
int ggc_model_truncate(ggc_model* m, uint64_t new_len);
/* KvCache::append / get_k / get_v for one layer (cache.rs:46-63); f32 rows of
 * n_kv_heads*head_dim (this rank's heads under tensor parallelism). */
int ggc_model_cache_append(ggc_model* m, uint32_t layer, const float* k, const float* v, uint64_t seq);
int ggc_model_cache_read(ggc_model* m, uint32_t layer, float* k, float* v);

/* Engine::generate's token loop (src/infer/engine.rs:83-138) with the greedy
 * sampler: forward(prompt) then up to max_tokens steps of argmax -> forward(1),
 * stopping before an `eos` id (eos < 0: none).  The loop runs on the device as
 * one CUDA graph per step without host round trips.  out_ids: host array of
 * max_tokens; *n_out = number generated. */
int ggc_model_generate_greedy(ggc_model* m, const uint32_t* prompt, uint64_t n_prompt,
                              int64_t start_pos, uint64_t max_tokens, int64_t eos,
                              uint32_t* out_ids, uint64_t* n_out);

/* Continues Engine::generate's loop from the logits of the last forward: `steps`
 * iterations of greedy sample -> forward(1 token) on the device, stopping before
 * `eos` (< 0: none).  sync = 0 only enqueues the work on the context stream;
 * ggc_model_wait then synchronises, validates and returns the ids (out_ids: host
 * array of `steps`, may be NULL). */
int ggc_model_decode(ggc_model* m, uint64_t steps, int64_t eos, int sync, uint32_t* out_ids, uint64_t* n_out);
int ggc_model_wait(ggc_model* m, uint32_t* out_ids, uint64_t* n_out);

/* Sampler::sample (src/infer/sampler.rs:86-186) on the device over `vocab`
 * logits (host or device pointer; ggc_model_sample: the logits of the model's last
 * forward / decode step, already on the device): repeat penalty on `seen` (host array of
 * token ids; duplicates count once, as the reference's HashMap keys), temperature
 * (<= 1e-6: greedy, the last maximum), softmax, top-k, top-p, min-p, and the pick
 * with `u` in [0, 1) standing for the reference's rng.gen_range(0.0..1.0) draw --
 * the caller keeps the RNG, so a host holding the reference's StdRng gets its
 * stream.  Only the token id comes back (no logits copy).  Limit: at most 1024
 * candidates after top-k (top_k in 1..1024, or a vocabulary of <= 1024), else
 * InvalidArg.  The softmax sum is a parallel reduction, so a pick can differ from
 * the reference's only when u*total lands within a few ulp of a cumulative
 * boundary.  NaN logits: InferenceError (the reference panics). */
typedef struct ggc_sampler_config {
    float temperature;
    uint32_t top_k;          /* 0 = off */
    float top_p;             /* 1.0 = off */
    float min_p;             /* 0.0 = off */
    float repeat_penalty;    /* 1.0 = off */
} ggc_sampler_config;
int ggc_sample(ggc_ctx* ctx, const float* logits, uint64_t vocab, const ggc_sampler_config* cfg, const uint32_t* seen,
               uint64_t n_seen, float u, uint32_t* out_id);
int ggc_model_sample(ggc_model* m, const ggc_sampler_config* cfg, const uint32_t* seen, uint64_t n_seen, float u,
                     uint32_t* out_id);

/* How a tensor-parallel model sums its row-parallel partials: 0 = single GPU
 * (none), 1 = NCCL all-reduce, 2 = fused into the GEMVs over peer memory. */
int ggc_model_allreduce_kind(const ggc_model* m);

/* No counterpart in the reference (a diagnostic of the fused tensor-parallel
 * all-reduce's bounded wait, allreduce.cuh): one all-reduce step of a world-2
 * group run on this GPU alone.  With peer_writes != 0 the peer's partials are
 * stored too and out[r] = part0[r] + part1[r] (rank order); with 0 they never
 * arrive, the bounded poll gives up and the call returns GGC_ERR_TIMEOUT after
 * about a second, the context staying usable.  Host or device part0/part1/out. */
int ggc_allreduce_probe(ggc_ctx* ctx, uint32_t rows, int peer_writes, const float* part0, const float* part1,
                        float* out);

/* Number of kernels this context launched so far (for launch accounting). */
uint64_t ggc_ctx_kernel_launches(ggc_ctx* ctx);

#ifdef __cplusplus
}
#endif
#endif /* GGUF_CUDA_H */
