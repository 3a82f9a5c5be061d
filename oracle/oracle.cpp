// oracle.cpp -- CPU restatement of gguf-reader's quantized inference path.
//
// TEST INFRASTRUCTURE ONLY: the parity checker and the timed CPU baseline.  The
// product library never links or calls this file.  Build with -O2
// -ffp-contract=off (no fast-math): Rust does not contract a*b+c into an FMA, and
// the f32 operation order below follows the Rust source line by line, so every
// dequantised value is bit-identical to the reference's.
//
// Reference files (chaos-asimo/gguf-reader):
//   src/infer/quant.rs      f16/bf16 codecs, per-format block dequant, quant_matvec
//   src/infer/ops.rs        matvec_colmajor_trans, silu, rmsnorm, softmax, rope, ...
//   src/infer/cache.rs      KvCache / Cache
//   src/infer/model/llama.rs forward_internal, attention_block, attend, ffn_block, lm_head
//   src/infer/engine.rs     generate loop; src/infer/sampler.rs greedy argmax
//
// Threading mirrors rayon: output rows are split across threads, each row is
// reduced serially, so results do not depend on the thread count.
#include "oracle.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <cstdio>
#include <limits>
#include <memory>
#include <string>
#include <thread>
#include <vector>

namespace {

thread_local orc_error g_err;
int g_threads = 0;

int set_err(int status, uint64_t expected, uint64_t actual, const char* msg) {
    g_err.status = status;
    g_err.expected = expected;
    g_err.actual = actual;
    g_err.elements = 0;
    g_err.block = 0;
    std::snprintf(g_err.message, sizeof(g_err.message), "%s", msg ? msg : "");
    return status;
}

int set_shape_err(uint64_t elements, uint64_t block) {
    g_err.status = ORC_ERR_INVALID_TENSOR_SHAPE;
    g_err.expected = g_err.actual = 0;
    g_err.elements = elements;
    g_err.block = block;
    std::snprintf(g_err.message, sizeof(g_err.message),
                  "invalid tensor shape: %llu elements not a multiple of block %llu",
                  (unsigned long long)elements, (unsigned long long)block);
    return ORC_ERR_INVALID_TENSOR_SHAPE;
}

int nthreads() {
    if (g_threads > 0) return g_threads;
    unsigned h = std::thread::hardware_concurrency();
    return h ? (int)h : 1;
}

// Contiguous chunks of [0, n) over the worker threads (rayon-equivalent result).
template <class F>
void parallel_for(uint64_t n, F fn) {
    int t = nthreads();
    if (t <= 1 || n < 2) {
        for (uint64_t i = 0; i < n; ++i) fn(i);
        return;
    }
    if ((uint64_t)t > n) t = (int)n;
    std::vector<std::thread> pool;
    pool.reserve(t);
    for (int k = 0; k < t; ++k) {
        uint64_t lo = n * k / t, hi = n * (k + 1) / t;
        pool.emplace_back([lo, hi, &fn] {
            for (uint64_t i = lo; i < hi; ++i) fn(i);
        });
    }
    for (auto& th : pool) th.join();
}

inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
inline uint32_t rd32(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
inline float bits_f32(uint32_t b) { float f; std::memcpy(&f, &b, 4); return f; }
inline uint32_t f32_bits(float f) { uint32_t b; std::memcpy(&b, &f, 4); return b; }

// quant.rs:12-37 f16_to_f32 (exact; NaN -> canonical f32::NAN, sign dropped)
float f16_to_f32(uint16_t h) {
    uint32_t bits = h;
    bool sign = (bits & 0x8000) != 0;
    uint32_t exp = (bits >> 10) & 0x1F;
    uint32_t mant = bits & 0x3FF;
    float v;
    if (exp == 0) {
        if (mant == 0) v = 0.0f;
        else v = ((float)mant / 1024.0f) * std::ldexp(1.0f, -14);
    } else if (exp == 31) {
        if (mant == 0) v = std::numeric_limits<float>::infinity();
        else return bits_f32(0x7FC00000u);
    } else {
        v = (1.0f + (float)mant / 1024.0f) * std::ldexp(1.0f, (int)exp - 15);
    }
    return sign ? -v : v;
}

inline float f16_at(const uint8_t* b, size_t off) { return f16_to_f32(rd16(b + off)); }
inline float bf16_at(const uint8_t* b, size_t off) { return bits_f32((uint32_t)rd16(b + off) << 16); }

// quant.rs:101-108 k_scale4: 4-bit scales stored in reverse byte order
inline uint32_t k_scale4(const uint8_t* s, int j) {
    int byte = 15 - j / 2;
    return (j % 2 == 0) ? (uint32_t)(s[byte] & 0xF) : (uint32_t)((s[byte] >> 4) & 0xF);
}

// quant.rs:116-124 k_scale_min_6bit
inline void k_scale_min_6bit(const uint8_t* q, int j, uint32_t* sc, uint32_t* mn) {
    if (j < 4) {
        *sc = q[j] & 0x3F;
        *mn = q[j + 4] & 0x3F;
    } else {
        *sc = (uint32_t)(q[j + 4] & 0x0F) | ((uint32_t)(q[j - 4] >> 6) << 4);
        *mn = (uint32_t)(q[j + 4] >> 4) | ((uint32_t)(q[j] >> 6) << 4);
    }
}

// quant.rs:128-135
void deq_q4_0(const uint8_t* b, float* out) {
    float d = f16_at(b, 0);
    for (int i = 0; i < 16; ++i) {
        uint8_t byte = b[2 + i];
        out[2 * i] = d * (float)((int8_t)(byte & 0xF) - 8);
        out[2 * i + 1] = d * (float)((int8_t)(byte >> 4) - 8);
    }
}

// quant.rs:137-145
void deq_q4_1(const uint8_t* b, float* out) {
    float d = f16_at(b, 0), m = f16_at(b, 2);
    for (int i = 0; i < 16; ++i) {
        uint8_t byte = b[4 + i];
        out[2 * i] = d * (float)(byte & 0xF) + m;
        out[2 * i + 1] = d * (float)(byte >> 4) + m;
    }
}

// quant.rs:147-165
void deq_q5_0(const uint8_t* b, float* out) {
    float d = f16_at(b, 0);
    uint32_t qh = rd32(b + 2);
    for (int i = 0; i < 16; ++i) {
        uint8_t byte = b[6 + i];
        uint32_t xh0 = ((qh >> i) << 4) & 0x10;
        uint32_t xh1 = (qh >> (i + 12)) & 0x10;
        int32_t lo = (int32_t)(((uint32_t)(byte & 0xF)) | xh0) - 16;
        int32_t hi = (int32_t)(((uint32_t)(byte >> 4)) | xh1) - 16;
        out[i] = d * (float)lo;
        out[16 + i] = d * (float)hi;
    }
}

// quant.rs:167-182
void deq_q5_1(const uint8_t* b, float* out) {
    float d = f16_at(b, 0), m = f16_at(b, 2);
    uint32_t qh = rd32(b + 4);
    for (int i = 0; i < 16; ++i) {
        uint8_t byte = b[8 + i];
        uint32_t xh0 = ((qh >> i) << 4) & 0x10;
        uint32_t xh1 = (qh >> (i + 12)) & 0x10;
        uint32_t lo = ((uint32_t)(byte & 0xF)) | xh0;
        uint32_t hi = ((uint32_t)(byte >> 4)) | xh1;
        out[i] = d * (float)lo + m;
        out[16 + i] = d * (float)hi + m;
    }
}

// quant.rs:184-189
void deq_q8_0(const uint8_t* b, float* out) {
    float d = f16_at(b, 0);
    for (int i = 0; i < 32; ++i) out[i] = d * (float)(int8_t)b[2 + i];
}

// quant.rs:193-207
void deq_q2_k(const uint8_t* b, float* out) {
    float d = f16_at(b, 80), dmin = f16_at(b, 82);
    for (int j = 0; j < 16; ++j) {
        float s = (float)k_scale4(b, j);
        float m = (s - 8.0f) * dmin;
        float s0 = (s < 8.0f) ? s * d : s * dmin + m;
        for (int i = 0; i < 16; ++i) {
            int k = 16 * j + i;
            float q = (float)((b[16 + k / 4] >> ((k % 4) * 2)) & 0x3);
            out[k] = s0 * q + ((s < 8.0f) ? 0.0f : m);
        }
    }
}

// quant.rs:223-240 (d_off = 108 for Q3_K_S/Q3_K_L, 112 for Q3_K_M)
void deq_q3_k(const uint8_t* b, size_t d_off, float* out) {
    float d = f16_at(b, d_off);
    int32_t sc[16];
    for (int i = 0; i < 16; ++i) {
        uint8_t lo = (b[96 + i / 2] >> ((i % 2) * 4)) & 0xF;
        uint8_t hi = (b[96 + 8 + i / 4] >> ((i % 4) * 2)) & 0x3;
        sc[i] = (int32_t)(uint8_t)(lo | (hi << 4)) - 32;
    }
    for (int i = 0; i < 256; ++i) {
        int32_t ql = (b[32 + i / 4] >> ((i % 4) * 2)) & 3;
        int32_t qh = (b[i / 8] >> (i % 8)) & 1;
        int32_t q = (qh ^ 1) * 4 - ql;
        out[i] = d * (float)sc[i / 16] * (float)q;
    }
}

// quant.rs:257-281
void deq_q4_k(const uint8_t* b, float* out) {
    float d = f16_at(b, 0), dmin = f16_at(b, 2);
    for (int e = 0; e < 256; ++e) {
        int group = e >> 6, in_grp = e & 63, is_high = in_grp >> 5;
        int byte_in_qs = group * 32 + (in_grp & 31);
        int sub_block = group * 2 + is_high;
        uint32_t sc, mn;
        k_scale_min_6bit(b + 4, sub_block, &sc, &mn);
        float s1 = (float)sc * d;
        float s2 = (float)mn * dmin;
        uint8_t byte = b[16 + byte_in_qs];
        uint8_t val = is_high ? (byte >> 4) : (byte & 0x0F);
        out[e] = s1 * (float)val - s2;
    }
}

// quant.rs:283-306
void deq_q5_k(const uint8_t* b, float* out) {
    float d = f16_at(b, 0), dmin = f16_at(b, 2);
    for (int j = 0; j < 8; ++j) {
        uint32_t sc, mn;
        k_scale_min_6bit(b + 4, j, &sc, &mn);
        float s1 = (float)sc * d;
        float s2 = (float)mn * dmin;
        for (int i = 0; i < 32; ++i) {
            int k = 32 * j + i;
            uint8_t byte = b[48 + k / 2];
            int byte_idx = k >> 1;
            uint32_t qh_bit = (b[16 + byte_idx / 8] >> (byte_idx % 8)) & 1;
            uint32_t q = ((k & 1) == 0) ? (((uint32_t)(byte & 0xF)) | (qh_bit << 4))
                                        : (((uint32_t)(byte >> 4)) | (qh_bit << 4));
            out[k] = s1 * (float)q - s2;
        }
    }
}

// quant.rs:308-337
void deq_q6_k(const uint8_t* b, float* out) {
    float d = f16_at(b, 208);
    for (int n = 0; n < 2; ++n) {
        for (int l = 0; l < 32; ++l) {
            int is = l / 16;
            uint8_t ql0 = b[n * 64 + l];
            uint8_t ql1 = b[n * 64 + 32 + l];
            uint8_t qh = b[128 + n * 32 + l];
            const uint8_t* sc = b + 192 + n * 8;
            uint8_t q1 = (ql0 & 0xF) | (((qh >> 0) & 3) << 4);
            uint8_t q2 = (ql1 & 0xF) | (((qh >> 2) & 3) << 4);
            uint8_t q3 = (ql0 >> 4) | (((qh >> 4) & 3) << 4);
            uint8_t q4 = (ql1 >> 4) | (((qh >> 6) & 3) << 4);
            int base = n * 128;
            out[base + l] = d * (float)(int8_t)sc[is] * (float)((int32_t)q1 - 32);
            out[base + l + 32] = d * (float)(int8_t)sc[is + 2] * (float)((int32_t)q2 - 32);
            out[base + l + 64] = d * (float)(int8_t)sc[is + 4] * (float)((int32_t)q3 - 32);
            out[base + l + 96] = d * (float)(int8_t)sc[is + 6] * (float)((int32_t)q4 - 32);
        }
    }
}

// quant.rs:339-345
void deq_q8_k(const uint8_t* b, float* out) {
    float d = bits_f32(rd32(b));
    for (int i = 0; i < 256; ++i) out[i] = d * (float)(int8_t)b[4 + i];
}

// types.rs:182-220
int64_t block_size(int dt) {
    switch (dt) {
        case ORC_F32: case ORC_F16: case ORC_BF16: return 1;
        case ORC_Q4_0: case ORC_Q4_1: case ORC_Q5_0: case ORC_Q5_1: case ORC_Q8_0: return 32;
        case ORC_Q2_K: case ORC_Q3_K_S: case ORC_Q3_K_M: case ORC_Q3_K_L: case ORC_Q4_K:
        case ORC_Q5_K: case ORC_Q6_K: case ORC_Q8_K: return 256;
        default: return -1;
    }
}
int64_t block_bytes(int dt) {
    switch (dt) {
        case ORC_F32: return 4;
        case ORC_F16: case ORC_BF16: return 2;
        case ORC_Q4_0: return 18; case ORC_Q4_1: return 20; case ORC_Q5_0: return 22;
        case ORC_Q5_1: return 24; case ORC_Q8_0: return 34; case ORC_Q2_K: return 84;
        case ORC_Q3_K_S: case ORC_Q3_K_L: return 110; case ORC_Q3_K_M: return 114;
        case ORC_Q4_K: return 144; case ORC_Q5_K: return 176; case ORC_Q6_K: return 210;
        case ORC_Q8_K: return 292;
        default: return -1;
    }
}

// quant.rs:357-398 dequantize_block (out must hold block_size elements)
int dequantize_block(const uint8_t* data, uint64_t len, int dt, float* out) {
    int64_t bb = block_bytes(dt);
    if (bb < 0) return set_err(ORC_ERR_DEQUANT, 0, len, "unsupported dtype");
    if (len < (uint64_t)bb) return set_err(ORC_ERR_DEQUANT, (uint64_t)bb, len, "block too short");
    switch (dt) {
        case ORC_F32: out[0] = bits_f32(rd32(data)); break;
        case ORC_F16: out[0] = f16_at(data, 0); break;
        case ORC_BF16: out[0] = bf16_at(data, 0); break;
        case ORC_Q4_0: deq_q4_0(data, out); break;
        case ORC_Q4_1: deq_q4_1(data, out); break;
        case ORC_Q5_0: deq_q5_0(data, out); break;
        case ORC_Q5_1: deq_q5_1(data, out); break;
        case ORC_Q8_0: deq_q8_0(data, out); break;
        case ORC_Q2_K: deq_q2_k(data, out); break;
        case ORC_Q3_K_S: deq_q3_k(data, 108, out); break;
        case ORC_Q3_K_M: deq_q3_k(data, 112, out); break;
        case ORC_Q3_K_L: deq_q3_k(data, 108, out); break;
        case ORC_Q4_K: deq_q4_k(data, out); break;
        case ORC_Q5_K: deq_q5_k(data, out); break;
        case ORC_Q6_K: deq_q6_k(data, out); break;
        case ORC_Q8_K: deq_q8_k(data, out); break;
        default: return set_err(ORC_ERR_DEQUANT, 0, 0, "unsupported dtype");
    }
    return ORC_OK;
}

// quant.rs:403-448 dequantize
int dequantize(const uint8_t* data, uint64_t len, int dt, uint64_t n, float* out) {
    int64_t bs = block_size(dt);
    if (bs < 0) return set_err(ORC_ERR_DEQUANT, 0, 0, "unsupported dtype");
    if (n % (uint64_t)bs != 0) return set_shape_err(n, (uint64_t)bs);
    uint64_t bb = (uint64_t)block_bytes(dt);
    uint64_t blocks = n / (uint64_t)bs;
    uint64_t need = blocks * bb;
    if (len < need) return set_err(ORC_ERR_DEQUANT, need, len, "data shorter than tensor");
    parallel_for(blocks, [&](uint64_t b) { dequantize_block(data + b * bb, bb, dt, out + b * bs); });
    return ORC_OK;
}

// quant.rs:473-520 dot_row
float dot_row(const uint8_t* w, int dt, uint64_t row_start, uint64_t cols, const float* x) {
    float acc = 0.0f;
    if (dt == ORC_F32) {
        for (uint64_t c = 0; c < cols; ++c) acc += bits_f32(rd32(w + row_start + c * 4)) * x[c];
        return acc;
    }
    if (dt == ORC_F16) {
        for (uint64_t c = 0; c < cols; ++c) acc += f16_at(w, row_start + c * 2) * x[c];
        return acc;
    }
    if (dt == ORC_BF16) {
        for (uint64_t c = 0; c < cols; ++c) acc += bf16_at(w, row_start + c * 2) * x[c];
        return acc;
    }
    uint64_t bs = (uint64_t)block_size(dt), bb = (uint64_t)block_bytes(dt);
    float block[256];
    for (uint64_t b = 0; b < cols / bs; ++b) {
        dequantize_block(w + row_start + b * bb, bb, dt, block);
        for (uint64_t c = 0; c < bs; ++c) acc += block[c] * x[b * bs + c];
    }
    return acc;
}

// ops.rs:172-227 (one output row)
inline float dot_f32(const float* a, const float* x, uint64_t n) {
    float acc = 0.0f;
    for (uint64_t j = 0; j < n; ++j) acc += a[j] * x[j];
    return acc;
}

// n matvec_colmajor_trans products over the same matrix, y[t][i] = dot(a row i,
// x[t]) + 0.0 (ops.rs:204-215 with no bias), each element the same serial f32
// dot as the one-token call.  Blocks of rows x tokens keep both in cache, so the
// matrix is read once per call instead of once per token; only the loop order
// over (row, token) pairs changes, not any element's arithmetic.
void matvec_trans_batch(const float* a, uint64_t dim0, uint64_t dim1, const float* x, uint64_t n, float* y) {
    constexpr uint64_t RB = 16, TB = 16;
    parallel_for((dim1 + RB - 1) / RB, [&](uint64_t rb) {
        const uint64_t r0 = rb * RB, r1 = std::min(dim1, r0 + RB);
        for (uint64_t t0 = 0; t0 < n; t0 += TB) {
            const uint64_t t1 = std::min(n, t0 + TB);
            for (uint64_t i = r0; i < r1; ++i)
                for (uint64_t t = t0; t < t1; ++t) y[t * dim1 + i] = dot_f32(a + i * dim0, x + t * dim0, dim0) + 0.0f;
        }
    });
}

}  // namespace

extern "C" {

void orc_last_error(orc_error* out) { if (out) *out = g_err; }
void orc_set_threads(int n) { g_threads = n; }
int orc_get_threads(void) { return nthreads(); }

float orc_f16_to_f32(uint16_t bits) { return f16_to_f32(bits); }
float orc_bf16_to_f32(uint16_t bits) { return bits_f32((uint32_t)bits << 16); }

// quant.rs:45-84 f32_to_f16 (truncating exponent map, round on the dropped bit)
uint16_t orc_f32_to_f16(float v) {
    uint32_t bits = f32_bits(v);
    uint16_t sign = (uint16_t)((bits & 0x80000000u) >> 16);
    uint32_t exp = (bits >> 23) & 0xFF;
    uint32_t mant = bits & 0x7FFFFF;
    if (exp == 0xFF) return mant != 0 ? (uint16_t)(sign | 0x7E00) : (uint16_t)(sign | 0x7C00);
    if (exp > 0x8E) return (uint16_t)(sign | 0x7C00);
    if (exp > 0x70) {
        uint16_t e = (uint16_t)(exp - 0x70);
        uint16_t m10 = (uint16_t)(mant >> 13);
        return (uint16_t)(sign | (e << 10) | m10);
    }
    if (exp == 0) return sign;
    uint32_t raw = mant | 0x800000u;
    uint32_t shift = 126 - exp;                       // 14..=125
    uint32_t val = shift < 32 ? raw >> shift : 0;
    uint32_t rounding_bit = (shift - 1) < 32 ? (raw >> (shift - 1)) & 1 : 0;
    uint16_t m16 = (uint16_t)(val + rounding_bit);
    return m16 == 0 ? sign : (uint16_t)(m16 | sign);
}

int64_t orc_block_size(int dtype) { return block_size(dtype); }
int64_t orc_block_bytes(int dtype) { return block_bytes(dtype); }

int orc_dequantize_block(const uint8_t* data, uint64_t len, int dtype, float* out) {
    return dequantize_block(data, len, dtype, out);
}

int orc_dequantize(const uint8_t* data, uint64_t len, int dtype, uint64_t n, float* out) {
    return dequantize(data, len, dtype, n, out);
}

// quant.rs:526-570 quant_matvec (+ row_bytes :452-471)
int orc_quant_matvec(const uint8_t* w, uint64_t w_len, int dt, uint64_t rows, uint64_t cols,
                     const float* x, uint64_t x_len, float* y, uint64_t y_len) {
    int64_t bs = block_size(dt), bb = block_bytes(dt);
    if (bs < 0 || bb < 0) return set_err(ORC_ERR_DEQUANT, 0, 0, "unsupported dtype");
    if (cols % (uint64_t)bs != 0) return set_shape_err(cols, (uint64_t)bs);
    uint64_t rb = cols / (uint64_t)bs * (uint64_t)bb;
    if (x_len != cols) return set_err(ORC_ERR_DEQUANT, cols, x_len, "x length != cols");
    if (y_len != rows) return set_err(ORC_ERR_DEQUANT, rows, y_len, "y length != rows");
    if (rows * rb > w_len) return set_err(ORC_ERR_DEQUANT, rows * rb, w_len, "w shorter than rows*row_bytes");
    parallel_for(rows, [&](uint64_t r) { y[r] = dot_row(w, dt, r * rb, cols, x); });
    return ORC_OK;
}

// ops.rs:14-69
int orc_matvec(const float* a, uint64_t a_len, uint64_t rows, uint64_t cols, const float* x,
               uint64_t x_len, float* y, uint64_t y_len, const float* b) {
    if (a_len < rows * cols) return set_err(ORC_ERR_DEQUANT, rows * cols, a_len, "F32");
    if (x_len != cols) return set_err(ORC_ERR_DEQUANT, cols, x_len, "F32");
    if (y_len != rows) return set_err(ORC_ERR_DEQUANT, rows, y_len, "F32");
    parallel_for(rows, [&](uint64_t i) { y[i] = dot_f32(a + i * cols, x, cols) + (b ? b[i] : 0.0f); });
    return ORC_OK;
}

// ops.rs:74-114
int orc_matmul(const float* a, uint64_t a_len, uint64_t ra, uint64_t ca, const float* b,
               uint64_t b_len, uint64_t cb, float* c, uint64_t c_len) {
    if (a_len < ra * ca) return set_err(ORC_ERR_DEQUANT, ra * ca, a_len, "F32");
    if (b_len < ca * cb) return set_err(ORC_ERR_DEQUANT, ca * cb, b_len, "F32");
    if (c_len < ra * cb) return set_err(ORC_ERR_DEQUANT, ra * cb, c_len, "F32");
    for (uint64_t i = 0; i < ra; ++i)
        for (uint64_t j = 0; j < cb; ++j) {
            float acc = 0.0f;
            for (uint64_t k = 0; k < ca; ++k) acc += a[i * ca + k] * b[k * cb + j];
            c[i * cb + j] = acc;
        }
    return ORC_OK;
}

// ops.rs:172-227
// ops.rs:121-170: y[i] = sum_j a[j * rows + i] x[j] (+ b[i])
int orc_matvec_colmajor(const float* a, uint64_t a_len, uint64_t rows, uint64_t cols, const float* x, uint64_t x_len,
                        float* y, uint64_t y_len, const float* b) {
    if (a_len < rows * cols) return set_err(ORC_ERR_DEQUANT, rows * cols, a_len, "F32");
    if (x_len != cols) return set_err(ORC_ERR_DEQUANT, cols, x_len, "F32");
    if (y_len != rows) return set_err(ORC_ERR_DEQUANT, rows, y_len, "F32");
    for (uint64_t i = 0; i < rows; ++i) {
        float acc = 0.0f;
        for (uint64_t j = 0; j < cols; ++j) acc += a[j * rows + i] * x[j];
        y[i] = acc + (b ? b[i] : 0.0f);
    }
    return ORC_OK;
}

int orc_matvec_colmajor_trans(const float* a, uint64_t a_len, uint64_t dim0, uint64_t dim1,
                              const float* x, uint64_t x_len, float* y, uint64_t y_len,
                              const float* b) {
    if (a_len < dim0 * dim1) return set_err(ORC_ERR_DEQUANT, dim0 * dim1, a_len, "F32");
    if (x_len != dim0) return set_err(ORC_ERR_DEQUANT, dim0, x_len, "F32");
    if (y_len != dim1) return set_err(ORC_ERR_DEQUANT, dim1, y_len, "F32");
    parallel_for(dim1, [&](uint64_t i) { y[i] = dot_f32(a + i * dim0, x, dim0) + (b ? b[i] : 0.0f); });
    return ORC_OK;
}

// ops.rs:237-247
void orc_silu(float* x, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i) {
        float v = x[i];
        float sig;
        if (v >= 0.0f) {
            sig = 1.0f / (1.0f + std::exp(-v));
        } else {
            float e = std::exp(v);
            sig = e / (1.0f + e);
        }
        x[i] = v * sig;
    }
}

// ops.rs:250-255
void orc_gelu(float* x, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i) {
        float v = x[i];
        float t = 0.7978846f * (v + 0.044715f * (v * v * v));
        x[i] = 0.5f * v * (1.0f + std::tanh(t));
    }
}

// ops.rs:262-274 (f64 sum of squares)
void orc_rmsnorm(float* x, uint64_t n, const float* w, uint64_t w_len, float eps) {
    if (n != w_len) return;
    double nn = (double)n;
    double ss = 0.0;
    for (uint64_t i = 0; i < n; ++i) ss += (double)x[i] * (double)x[i];
    float scale = (float)std::sqrt(1.0 / (ss / nn + (double)eps));
    for (uint64_t i = 0; i < n; ++i) x[i] = x[i] * scale * w[i];
}

// ops.rs:279-290
void orc_layernorm(float* x, uint64_t n, const float* w, uint64_t w_len, const float* b,
                   uint64_t b_len, float eps) {
    if (n == 0 || n != w_len || n != b_len) return;
    float nf = (float)n;
    float sum = 0.0f;
    for (uint64_t i = 0; i < n; ++i) sum += x[i];
    float mean = sum / nf;
    float vs = 0.0f;
    for (uint64_t i = 0; i < n; ++i) vs += (x[i] - mean) * (x[i] - mean);
    float var = vs / nf;
    float inv_std = std::sqrt(1.0f / (var + eps));
    for (uint64_t i = 0; i < n; ++i) x[i] = (x[i] - mean) * inv_std * w[i] + b[i];
}

// ops.rs:295-308
void orc_softmax(float* x, uint64_t n) {
    if (n == 0) return;
    float mx = -std::numeric_limits<float>::infinity();
    for (uint64_t i = 0; i < n; ++i) mx = std::fmax(mx, x[i]);
    float sum = 0.0f;
    for (uint64_t i = 0; i < n; ++i) sum += std::exp(x[i] - mx);
    float inv_sum = 1.0f / sum;
    for (uint64_t i = 0; i < n; ++i) x[i] = std::exp(x[i] - mx) * inv_sum;
}

// ops.rs:318-337 (NeoX half-split pairs (i, i + hd/2))
void orc_rope(float* x, uint64_t n_x, const int64_t* positions, uint64_t n_pos, const float* freqs,
              uint64_t n_freqs) {
    if (n_x == 0 || n_pos == 0 || n_freqs == 0) return;
    uint64_t half = n_freqs, hd = half * 2, n = n_x / hd;
    for (uint64_t tok = 0; tok < n; ++tok) {
        float pos = (float)(tok < n_pos ? positions[tok] : 0);
        uint64_t base = tok * hd;
        for (uint64_t i = 0; i < half; ++i) {
            float angle = pos * freqs[i];
            float s = std::sin(angle), c = std::cos(angle);
            float a = x[base + i], b = x[base + i + half];
            x[base + i] = a * c - b * s;
            x[base + i + half] = b * c + a * s;
        }
    }
}

// model/llama.rs:778-782
void orc_build_inv_freq(uint64_t head_dim, double base, float* out) {
    for (uint64_t i = 0; i < head_dim / 2; ++i)
        out[i] = (float)std::pow(base, -2.0 * (double)i / (double)head_dim);
}

// ops.rs:340-351
void orc_rope_freqs(uint64_t dim, float base, uint64_t max_seq_len, float* out) {
    float dim_f = (float)dim;
    std::vector<float> inv(dim / 2);
    for (uint64_t i = 0; i < dim / 2; ++i) inv[i] = 1.0f / std::pow(base, (2.0f * (float)i) / dim_f);
    for (uint64_t p = 0; p < max_seq_len; ++p)
        for (uint64_t i = 0; i < dim / 2; ++i) out[p * (dim / 2) + i] = (float)p * inv[i];
}

// model/llama.rs:656-710 infer_k_quant_dtype
int orc_infer_k_quant_dtype(uint64_t span, uint64_t n, int marked) {
    switch (marked) {
        case ORC_Q4_0: case ORC_Q4_1: case ORC_Q5_0: case ORC_Q5_1: case ORC_Q8_0: case ORC_Q2_K:
        case ORC_Q3_K_S: case ORC_Q3_K_M: case ORC_Q3_K_L: case ORC_Q4_K: case ORC_Q5_K:
        case ORC_Q6_K: case ORC_Q8_K: break;
        default: return -1;
    }
    if (n == 0) return -1;
    int64_t bs = block_size(marked);
    uint64_t blocks = bs == 32 ? n / 32 : n / 256;
    if (blocks == 0) return -1;
    uint64_t per256 = bs == 32 ? span * 8 / blocks : span / blocks;
    if (span % blocks > 256) return -1;
    static const struct { uint64_t b; int dt; } table[] = {
        {84, ORC_Q2_K}, {110, ORC_Q3_K_S}, {114, ORC_Q3_K_M}, {144, ORC_Q4_K},
        {176, ORC_Q5_K}, {210, ORC_Q6_K}, {292, ORC_Q8_K}};
    for (auto& e : table)
        if (e.b == per256) return e.dt;
    return -1;
}

uint32_t orc_greedy(const float* logits, uint64_t n) {
    // sampler.rs:189-196 max_by(partial_cmp): the LAST maximum wins
    uint64_t best = 0;
    for (uint64_t i = 1; i < n; ++i)
        if (!(logits[i] < logits[best])) best = i;
    return (uint32_t)best;
}

// sampler.rs:86-186, step by step in the reference's f32 order
int orc_sample(const float* logits, uint64_t vocab, const orc_sampler_cfg* cfg, const uint32_t* seen, uint64_t n_seen,
               float u, uint32_t* out) {
    if (vocab == 0) return set_err(ORC_ERR_INFERENCE, 0, 0, "logits empty");
    std::vector<float> v(logits, logits + vocab);
    for (uint64_t i = 0; i < vocab; ++i)
        if (std::isnan(v[i])) return set_err(ORC_ERR_INFERENCE, 0, 0, "NaN logit");
    // step 1: repeat penalty (sampler.rs:95-110)
    if (cfg->repeat_penalty != 1.0f)
        for (uint64_t k = 0; k < n_seen; ++k) {
            const uint64_t idx = seen[k];
            if (idx < vocab) v[idx] = v[idx] > 0.0f ? v[idx] / cfg->repeat_penalty : v[idx] * cfg->repeat_penalty;
        }
    // step 2: temperature, or greedy (:112-124; max_by keeps the last maximum)
    const float temp = cfg->temperature;
    if (!(temp > 1e-6f)) { *out = orc_greedy(v.data(), vocab); return ORC_OK; }
    for (auto& x : v) x = x / temp;
    // step 3: softmax (:127-130)
    float max_v = -std::numeric_limits<float>::max();
    for (float x : v) max_v = std::fmax(max_v, x);
    std::vector<float> pr(vocab);
    float sum = 0.0f;
    for (uint64_t i = 0; i < vocab; ++i) { pr[i] = expf(v[i] - max_v); sum += pr[i]; }
    for (auto& p : pr) p = p / sum;
    // step 4: top-k (:133-139), stable sort by probability, descending
    std::vector<std::pair<uint32_t, float>> c(vocab);
    for (uint64_t i = 0; i < vocab; ++i) c[i] = {(uint32_t)i, pr[i]};
    auto desc = [](const std::pair<uint32_t, float>& a, const std::pair<uint32_t, float>& b) { return a.second > b.second; };
    if (cfg->top_k > 0 && cfg->top_k < c.size()) {
        std::stable_sort(c.begin(), c.end(), desc);
        c.resize(cfg->top_k);
    }
    // step 5: top-p (:142-156)
    if (cfg->top_p < 1.0f) {
        std::stable_sort(c.begin(), c.end(), desc);
        float total = 0.0f;
        for (auto& e : c) total += e.second;
        const float threshold = total * cfg->top_p;
        float cum = 0.0f;
        size_t cut = c.size();
        for (size_t i = 0; i < c.size(); ++i) {
            cum += c[i].second;
            if (cum >= threshold) { cut = i + 1; break; }
        }
        c.resize(cut);
    }
    // step 6: min-p (:159-163)
    if (cfg->min_p > 0.0f) {
        float mp = 0.0f;
        for (auto& e : c) mp = std::fmax(mp, e.second);
        const float thr = mp * cfg->min_p;
        std::vector<std::pair<uint32_t, float>> kept;
        for (auto& e : c)
            if (e.second >= thr) kept.push_back(e);
        c.swap(kept);
    }
    // step 7: renormalise and pick (:166-184)
    if (c.empty()) { *out = orc_greedy(v.data(), vocab); return ORC_OK; }
    float total = 0.0f;
    for (auto& e : c) total += e.second;
    float r = u * total;
    for (auto& e : c) {
        r -= e.second;
        if (r <= 0.0f) { *out = e.first; return ORC_OK; }
    }
    *out = c.back().first;
    return ORC_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// model/llama.rs forward path with the lazily materialised f32 weights
// (materialize :183-204 caches the dequantised tensor; here it is done at create).
// ---------------------------------------------------------------------------
struct orc_model {
    orc_hparams hp;
    std::vector<float> token_embd, output_norm, output;
    struct Layer {
        std::vector<float> attn_norm, wq, bq, wk, bk, wv, bv, wo, ffn_norm, up, gate, down;
    };
    std::vector<Layer> layers;
    std::vector<float> inv_freq;
    // cache.rs KvCache per layer: [seq][n_kv][hd]
    std::vector<std::vector<float>> kc, vc;
};

namespace {

int materialize(const orc_tensor_desc& t, std::vector<float>& out) {
    if (!t.data) { out.clear(); return ORC_OK; }
    int64_t bs = block_size(t.dtype);
    int64_t bb = block_bytes(t.dtype);
    if (bs < 0 || bb < 0) return set_err(ORC_ERR_DEQUANT, 0, 0, "unsupported dtype");
    // llama.rs:765-767: element count from the number of whole blocks in the data
    uint64_t blocks = t.nbytes / (uint64_t)bb;
    uint64_t elements = blocks * (uint64_t)bs;
    out.resize(elements);
    int st = dequantize((const uint8_t*)t.data, t.nbytes, t.dtype, elements, out.data());
    if (st) return st;
    if (elements != t.n_elements)   // llama.rs:194-200
        return set_err(ORC_ERR_INFERENCE, t.n_elements, elements, "materialize: length != num_elements");
    return ORC_OK;
}

void apply_rmsnorm(const std::vector<float>& w, std::vector<float>& x, uint64_t n) {
    uint64_t d = w.size();
    for (uint64_t i = 0; i < n; ++i) orc_rmsnorm(x.data() + i * d, d, w.data(), d, 1e-6f);
}

// llama.rs:499-545 attend
void attend(const float* q, const float* k, const float* v, uint64_t seq, uint64_t qn, uint64_t kvn,
            uint64_t hd, float inv, int64_t pos, float* o) {
    uint64_t qpk = qn / kvn;
    std::vector<float> scores(seq), oh(hd);
    for (uint64_t h = 0; h < qn; ++h) {
        uint64_t khead = h / qpk;
        const float* qh = q + h * hd;
        for (uint64_t s = 0; s < seq; ++s) {
            const float* kb = k + (s * kvn + khead) * hd;
            float dot = 0.0f;
            for (uint64_t i = 0; i < hd; ++i) dot += qh[i] * kb[i];
            scores[s] = ((int64_t)s <= pos) ? dot * inv : -std::numeric_limits<float>::infinity();
        }
        orc_softmax(scores.data(), seq);
        std::fill(oh.begin(), oh.end(), 0.0f);
        for (uint64_t s = 0; s < seq; ++s) {
            const float* vb = v + (s * kvn + khead) * hd;
            float w = scores[s];
            if (std::fabs(w) > 1e-9f)
                for (uint64_t i = 0; i < hd; ++i) oh[i] += w * vb[i];
        }
        std::memcpy(o + h * hd, oh.data(), hd * sizeof(float));
    }
}

bool any_nan(const std::vector<float>& v) {
    for (float f : v) if (std::isnan(f)) return true;
    return false;
}

}  // namespace

extern "C" {

int orc_model_create(const orc_hparams* hp, const orc_tensor_desc* t, uint64_t n_tensors,
                     orc_model** out) {
    if (!hp || !t || !out) return set_err(ORC_ERR_INVALID_ARG, 0, 0, "null argument");
    if (n_tensors != 3 + 12ull * hp->n_layers)
        return set_err(ORC_ERR_MISSING_TENSOR, 3 + 12ull * hp->n_layers, n_tensors, "tensor count");
    std::unique_ptr<orc_model> m(new orc_model());
    m->hp = *hp;
    int st;
    if ((st = materialize(t[0], m->token_embd))) return st;
    if ((st = materialize(t[1], m->output_norm))) return st;
    if ((st = materialize(t[2], m->output))) return st;
    m->layers.resize(hp->n_layers);
    for (uint32_t l = 0; l < hp->n_layers; ++l) {
        const orc_tensor_desc* d = t + 3 + 12 * l;
        auto& L = m->layers[l];
        std::vector<float>* dst[12] = {&L.attn_norm, &L.wq, &L.bq, &L.wk, &L.bk, &L.wv,
                                       &L.bv, &L.wo, &L.ffn_norm, &L.up, &L.gate, &L.down};
        for (int k = 0; k < 12; ++k) {
            bool optional = (k == 2 || k == 4 || k == 6);
            if (!d[k].data && !optional) return set_err(ORC_ERR_MISSING_TENSOR, 0, 0, "missing tensor");
            if ((st = materialize(d[k], *dst[k]))) return st;
        }
    }
    uint32_t hd = hp->embed_dim / (hp->n_heads ? hp->n_heads : 1);
    m->inv_freq.resize(hd / 2);
    orc_build_inv_freq(hd, hp->rope_freq_base, m->inv_freq.data());
    m->kc.resize(hp->n_layers);
    m->vc.resize(hp->n_layers);
    *out = m.release();
    return ORC_OK;
}

void orc_model_destroy(orc_model* m) { delete m; }

uint64_t orc_model_cache_len(const orc_model* m) {
    if (!m || m->kc.empty()) return 0;
    uint64_t n = (uint64_t)m->hp.n_kv_heads * (m->hp.embed_dim / m->hp.n_heads);
    return m->kc[0].size() / (n ? n : 1);
}

void orc_model_reset_cache(orc_model* m) {
    for (auto& k : m->kc) k.clear();
    for (auto& v : m->vc) v.clear();
}

void orc_model_truncate(orc_model* m, uint64_t new_len) {
    uint64_t n = (uint64_t)m->hp.n_kv_heads * (m->hp.embed_dim / m->hp.n_heads);
    uint64_t keep = new_len * n;
    for (uint32_t l = 0; l < m->hp.n_layers; ++l)
        if (keep < m->kc[l].size()) { m->kc[l].resize(keep); m->vc[l].resize(keep); }
}

int orc_model_cache_append(orc_model* m, uint32_t layer, const float* k, const float* v, uint64_t seq) {
    if (layer >= m->hp.n_layers) return set_err(ORC_ERR_INVALID_ARG, 0, 0, "layer");
    uint64_t n = (uint64_t)m->hp.n_kv_heads * (m->hp.embed_dim / m->hp.n_heads);
    m->kc[layer].insert(m->kc[layer].end(), k, k + seq * n);
    m->vc[layer].insert(m->vc[layer].end(), v, v + seq * n);
    return ORC_OK;
}

int orc_model_cache_read(const orc_model* m, uint32_t layer, float* k, float* v) {
    if (layer >= m->hp.n_layers) return set_err(ORC_ERR_INVALID_ARG, 0, 0, "layer");
    std::memcpy(k, m->kc[layer].data(), m->kc[layer].size() * sizeof(float));
    std::memcpy(v, m->vc[layer].data(), m->vc[layer].size() * sizeof(float));
    return ORC_OK;
}

// llama.rs:266-350 forward_internal; logits of the last token (vocab floats)
int orc_model_forward(orc_model* m, const uint32_t* tokens, const int64_t* positions, uint64_t n,
                      float* logits) {
    if (n == 0) return set_err(ORC_ERR_INFERENCE, 0, 0, "empty input");
    const orc_hparams& hp = m->hp;
    uint64_t d = hp.embed_dim, q = hp.n_heads, kv = hp.n_kv_heads, hd = d / q, f = hp.ffn_dim;
    // embed :367-383
    std::vector<float> hidden(n * d);
    for (uint64_t i = 0; i < n; ++i) {
        uint64_t base = (uint64_t)tokens[i] * d;
        if (base + d > m->token_embd.size()) return set_err(ORC_ERR_INFERENCE, 0, 0, "embed out of bounds");
        std::memcpy(hidden.data() + i * d, m->token_embd.data() + base, d * sizeof(float));
    }
    float inv = 1.0f / std::sqrt((float)hd);
    std::vector<float> qv(q * hd), kbuf(kv * hd), vbuf(kv * hd);
    std::vector<int64_t> qpos(q), kpos(kv);
    for (uint32_t l = 0; l < hp.n_layers; ++l) {
        auto& L = m->layers[l];
        std::vector<float> residual = hidden;
        std::vector<float> attn_in = residual;
        apply_rmsnorm(L.attn_norm, attn_in, n);
        // attention_block :417-495 -- the q/k/v and output products of all n tokens
        // are batched (matvec_trans_batch: each element as in the per-token call);
        // bias, RoPE, cache append and attend run token by token in order
        std::vector<float> attn_out(n * d, 0.0f), qa(n * q * hd), ka(n * kv * hd), va(n * kv * hd), oa(n * q * hd);
        matvec_trans_batch(L.wq.data(), d, q * hd, attn_in.data(), n, qa.data());
        matvec_trans_batch(L.wk.data(), d, kv * hd, attn_in.data(), n, ka.data());
        matvec_trans_batch(L.wv.data(), d, kv * hd, attn_in.data(), n, va.data());
        for (uint64_t tok = 0; tok < n; ++tok) {
            int64_t pos = positions[tok];
            std::memcpy(qv.data(), qa.data() + tok * q * hd, q * hd * sizeof(float));
            for (uint64_t i = 0; i < L.bq.size() && i < q * hd; ++i) qv[i] += L.bq[i];
            std::fill(qpos.begin(), qpos.end(), pos);
            orc_rope(qv.data(), q * hd, qpos.data(), q, m->inv_freq.data(), m->inv_freq.size());
            std::memcpy(kbuf.data(), ka.data() + tok * kv * hd, kv * hd * sizeof(float));
            for (uint64_t i = 0; i < L.bk.size() && i < kv * hd; ++i) kbuf[i] += L.bk[i];
            std::memcpy(vbuf.data(), va.data() + tok * kv * hd, kv * hd * sizeof(float));
            for (uint64_t i = 0; i < L.bv.size() && i < kv * hd; ++i) vbuf[i] += L.bv[i];
            std::fill(kpos.begin(), kpos.end(), pos);
            orc_rope(kbuf.data(), kv * hd, kpos.data(), kv, m->inv_freq.data(), m->inv_freq.size());
            m->kc[l].insert(m->kc[l].end(), kbuf.begin(), kbuf.end());   // cache.rs:46-54
            m->vc[l].insert(m->vc[l].end(), vbuf.begin(), vbuf.end());
            // llama.rs:479 reads a copy of the whole cache prefix; the values are the cache's own
            uint64_t seq = m->kc[l].size() / (kv * hd);
            attend(qv.data(), m->kc[l].data(), m->vc[l].data(), seq, q, kv, hd, inv, pos, oa.data() + tok * q * hd);
        }
        matvec_trans_batch(L.wo.data(), q * hd, d, oa.data(), n, attn_out.data());
        if (any_nan(attn_out)) return set_err(ORC_ERR_INFERENCE, l, 0, "NaN after attention");
        for (uint64_t i = 0; i < n * d; ++i) residual[i] += attn_out[i];
        hidden = residual;
        std::vector<float> ffn_in = hidden;
        apply_rmsnorm(L.ffn_norm, ffn_in, n);
        // ffn_block :547-580 (products batched over the tokens as above)
        std::vector<float> ffn_out(n * d, 0.0f), upa(n * f), gatea(n * f);
        matvec_trans_batch(L.up.data(), d, f, ffn_in.data(), n, upa.data());
        matvec_trans_batch(L.gate.data(), d, f, ffn_in.data(), n, gatea.data());
        for (uint64_t tok = 0; tok < n; ++tok) {
            float* g = gatea.data() + tok * f;
            const float* u = upa.data() + tok * f;
            orc_silu(g, f);
            for (uint64_t i = 0; i < f; ++i) g[i] *= u[i];
        }
        matvec_trans_batch(L.down.data(), f, d, gatea.data(), n, ffn_out.data());
        if (any_nan(ffn_out)) return set_err(ORC_ERR_INFERENCE, l, 0, "NaN after ffn");
        for (uint64_t i = 0; i < n * d; ++i) hidden[i] += ffn_out[i];
    }
    apply_rmsnorm(m->output_norm, hidden, n);
    // lm_head :582-616: logits[v] = sum_i w[v*d + i] * last[i]
    const float* last = hidden.data() + (n - 1) * d;
    const float* w = m->output.data();
    uint64_t vocab = hp.vocab_size;
    parallel_for(vocab, [&](uint64_t v) { logits[v] = dot_f32(w + v * d, last, d); });
    return ORC_OK;
}

// engine.rs:83-138 generate loop, greedy sampler (sampler.rs:113-123)
int orc_generate_greedy(orc_model* m, const uint32_t* prompt, uint64_t n_prompt, int64_t start_pos,
                        uint64_t max_tokens, int64_t eos, uint32_t* out_ids, uint64_t* n_out) {
    *n_out = 0;
    if (n_prompt == 0) return set_err(ORC_ERR_INFERENCE, 0, 0, "prompt tokenize empty");
    std::vector<int64_t> positions(n_prompt);
    for (uint64_t i = 0; i < n_prompt; ++i) positions[i] = start_pos + (int64_t)i;
    std::vector<float> logits(m->hp.vocab_size);
    int st = orc_model_forward(m, prompt, positions.data(), n_prompt, logits.data());
    if (st) return st;
    int64_t pos = start_pos + (int64_t)n_prompt;
    for (uint64_t t = 0; t < max_tokens; ++t) {
        for (uint64_t i = 0; i < logits.size(); ++i)
            if (std::isnan(logits[i])) return set_err(ORC_ERR_INFERENCE, 0, 0, "NaN logits");
        uint32_t id = orc_greedy(logits.data(), logits.size());
        if (eos >= 0 && (int64_t)id == eos) break;
        out_ids[(*n_out)++] = id;
        st = orc_model_forward(m, &id, &pos, 1, logits.data());
        if (st) return st;
        pos += 1;
    }
    return ORC_OK;
}

}  // extern "C"
