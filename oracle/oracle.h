/*
 * oracle.h -- CPU restatement of gguf-reader's quantized inference path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker and the timed
 * CPU baseline ("port" of the reference's rayon CPU path).  It is never linked
 * into, loaded by or called from the product library (libgguf_cuda.so); only the
 * test-suite, the smoke check and the CPU-baseline leg of bench.py load it.
 *
 * Every function restates the Rust reference (chaos-asimo/gguf-reader) with the
 * same f32 operation order and no FMA contraction (built with -ffp-contract=off),
 * so dequantised values are bit-identical to the reference's.
 *
 * Dtype ids are the GGUF on-disk ids (src/types.rs:122-160) plus two ids that are
 * reachable only through the API (Q3_K_M, Q3_K_L), matching include/gguf_cuda.h.
 */
#pragma once
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    ORC_F32 = 0, ORC_F16 = 1, ORC_Q4_0 = 2, ORC_Q4_1 = 3, ORC_Q5_0 = 6, ORC_Q5_1 = 7,
    ORC_Q8_0 = 8, ORC_Q2_K = 10, ORC_Q3_K_S = 11, ORC_Q4_K = 12, ORC_Q5_K = 13,
    ORC_Q6_K = 14, ORC_Q8_K = 15, ORC_BF16 = 30, ORC_Q3_K_L = 111, ORC_Q3_K_M = 112
};

/* status codes: same numbering as the product's GGC_* codes */
enum {
    ORC_OK = 0, ORC_ERR_DEQUANT = 1, ORC_ERR_INVALID_TENSOR_SHAPE = 2,
    ORC_ERR_MISSING_TENSOR = 3, ORC_ERR_UNSUPPORTED_ARCH = 4, ORC_ERR_INFERENCE = 5,
    ORC_ERR_KV_CACHE_OVERFLOW = 6, ORC_ERR_INVALID_ARG = 7
};

typedef struct {
    int status;
    uint64_t expected, actual;   /* DequantError fields */
    uint64_t elements, block;    /* InvalidTensorShape fields */
    char message[256];
} orc_error;

void orc_last_error(orc_error* out);
void orc_set_threads(int n);
int orc_get_threads(void);

/* quant.rs */
float orc_f16_to_f32(uint16_t bits);
float orc_bf16_to_f32(uint16_t bits);
uint16_t orc_f32_to_f16(float v);
int64_t orc_block_size(int dtype);   /* -1 = None */
int64_t orc_block_bytes(int dtype);  /* -1 = None */
int orc_dequantize_block(const uint8_t* data, uint64_t len, int dtype, float* out);
int orc_dequantize(const uint8_t* data, uint64_t len, int dtype, uint64_t n, float* out);
int orc_quant_matvec(const uint8_t* w, uint64_t w_len, int dtype, uint64_t rows, uint64_t cols,
                     const float* x, uint64_t x_len, float* y, uint64_t y_len);

/* ops.rs */
int orc_matvec(const float* a, uint64_t a_len, uint64_t rows, uint64_t cols, const float* x,
               uint64_t x_len, float* y, uint64_t y_len, const float* b);
int orc_matmul(const float* a, uint64_t a_len, uint64_t rows_a, uint64_t cols_a, const float* b,
               uint64_t b_len, uint64_t cols_b, float* c, uint64_t c_len);
int orc_matvec_colmajor(const float* a, uint64_t a_len, uint64_t rows, uint64_t cols, const float* x, uint64_t x_len,
                        float* y, uint64_t y_len, const float* b);
int orc_matvec_colmajor_trans(const float* a, uint64_t a_len, uint64_t dim0, uint64_t dim1,
                              const float* x, uint64_t x_len, float* y, uint64_t y_len,
                              const float* b);
void orc_silu(float* x, uint64_t n);
void orc_gelu(float* x, uint64_t n);
void orc_rmsnorm(float* x, uint64_t n, const float* w, uint64_t w_len, float eps);
void orc_layernorm(float* x, uint64_t n, const float* w, uint64_t w_len, const float* b,
                   uint64_t b_len, float eps);
void orc_softmax(float* x, uint64_t n);
void orc_rope(float* x, uint64_t n, const int64_t* positions, uint64_t n_pos, const float* freqs,
              uint64_t n_freqs);
void orc_build_inv_freq(uint64_t head_dim, double base, float* out);
void orc_rope_freqs(uint64_t dim, float base, uint64_t max_seq_len, float* out);

/* model/llama.rs: physical-span dtype re-inference (-1 = None) */
int orc_infer_k_quant_dtype(uint64_t span, uint64_t n, int marked);

/* model/llama.rs + cache.rs + engine.rs greedy loop */
typedef struct {
    const void* data;      /* raw GGUF bytes of the tensor (NULL = absent, for biases) */
    uint64_t nbytes;
    int dtype;
    uint64_t n_elements;
} orc_tensor_desc;

typedef struct {
    uint32_t vocab_size, embed_dim, n_heads, n_kv_heads, ffn_dim, n_layers;
    double rope_freq_base;
} orc_hparams;

/* Tensors, in order: token_embd, output_norm, output, then per layer
 * attn_norm, wq, bq, wk, bk, wv, bv, wo, ffn_norm, ffn_up, ffn_gate, ffn_down
 * (3 + 12 * n_layers descriptors). */
typedef struct orc_model orc_model;
int orc_model_create(const orc_hparams* hp, const orc_tensor_desc* tensors, uint64_t n_tensors,
                     orc_model** out);
void orc_model_destroy(orc_model* m);
int orc_model_forward(orc_model* m, const uint32_t* tokens, const int64_t* positions, uint64_t n,
                      float* logits);
uint64_t orc_model_cache_len(const orc_model* m);
void orc_model_reset_cache(orc_model* m);
void orc_model_truncate(orc_model* m, uint64_t new_len);
/* appends `seq` rows of K/V ([seq][n_kv*hd] f32) to one layer's cache (test hook) */
int orc_model_cache_append(orc_model* m, uint32_t layer, const float* k, const float* v, uint64_t seq);
int orc_model_cache_read(const orc_model* m, uint32_t layer, float* k, float* v);
/* Engine::generate token loop with greedy sampling (temperature 0, repeat penalty 1):
 * prefill prompt at positions 0..n-1 (relative to start_pos), then up to max_tokens greedy steps.
 * eos < 0 = none. Returns number of generated ids in *n_out. */
int orc_generate_greedy(orc_model* m, const uint32_t* prompt, uint64_t n_prompt, int64_t start_pos,
                        uint64_t max_tokens, int64_t eos, uint32_t* out_ids, uint64_t* n_out);
uint32_t orc_greedy(const float* logits, uint64_t n);
/* Sampler::sample (sampler.rs:86-186) with `u` standing for the one
 * rng.gen_range(0.0..1.0) draw it makes; seen: the distinct token ids with a
 * positive repeat count.  Returns ORC status (NaN logits: the reference panics). */
typedef struct {
    float temperature;
    uint32_t top_k;
    float top_p;
    float min_p;
    float repeat_penalty;
} orc_sampler_cfg;
int orc_sample(const float* logits, uint64_t vocab, const orc_sampler_cfg* cfg, const uint32_t* seen, uint64_t n_seen,
               float u, uint32_t* out);

#ifdef __cplusplus
}
#endif
