// dequant.cuh -- bit-exact GGUF block dequantisation on the device.
//
// Each function returns element `e` of one raw block exactly as the reference's
// deq_* (src/infer/quant.rs:128-345) computes it: the same f32 operations in the
// same association order, rounded with explicit __fmul_rn/__fadd_rn/__fsub_rn so
// that no multiply-add is contracted into an FMA (the translation unit is also
// built with -fmad=false).
#pragma once
#include "common.cuh"

namespace ggc {

// quant.rs:101-108 (4-bit scales stored in reverse byte order)
__device__ __forceinline__ uint32_t k_scale4(const uint8_t* s, int j) {
    int byte = 15 - j / 2;
    return (j % 2 == 0) ? (uint32_t)(s[byte] & 0xF) : (uint32_t)((s[byte] >> 4) & 0xF);
}

// quant.rs:116-124
__device__ __forceinline__ void k_scale_min_6bit(const uint8_t* q, int j, uint32_t& sc, uint32_t& mn) {
    if (j < 4) {
        sc = q[j] & 0x3F;
        mn = q[j + 4] & 0x3F;
    } else {
        sc = (uint32_t)(q[j + 4] & 0x0F) | ((uint32_t)(q[j - 4] >> 6) << 4);
        mn = (uint32_t)(q[j + 4] >> 4) | ((uint32_t)(q[j] >> 6) << 4);
    }
}

template <int DT>
__device__ __forceinline__ float deq_elem(const uint8_t* b, int e);

// quant.rs:371-375
template <> __device__ __forceinline__ float deq_elem<GGC_F32>(const uint8_t* b, int) {
    return __uint_as_float(ld_u32_unaligned(b));
}
template <> __device__ __forceinline__ float deq_elem<GGC_F16>(const uint8_t* b, int) { return f16_ref(ld_u16(b)); }
template <> __device__ __forceinline__ float deq_elem<GGC_BF16>(const uint8_t* b, int) { return bf16_ref(ld_u16(b)); }

// quant.rs:128-135: out[2i] low nibble, out[2i+1] high nibble (interleaved)
template <> __device__ __forceinline__ float deq_elem<GGC_Q4_0>(const uint8_t* b, int e) {
    float d = f16_ref(ld_u16(b));
    uint8_t byte = b[2 + (e >> 1)];
    int q = (e & 1) ? (byte >> 4) : (byte & 0xF);
    return __fmul_rn(d, (float)(q - 8));
}
// quant.rs:137-145
template <> __device__ __forceinline__ float deq_elem<GGC_Q4_1>(const uint8_t* b, int e) {
    float d = f16_ref(ld_u16(b)), m = f16_ref(ld_u16(b + 2));
    uint8_t byte = b[4 + (e >> 1)];
    int q = (e & 1) ? (byte >> 4) : (byte & 0xF);
    return __fadd_rn(__fmul_rn(d, (float)q), m);
}
// quant.rs:147-165
template <> __device__ __forceinline__ float deq_elem<GGC_Q5_0>(const uint8_t* b, int e) {
    float d = f16_ref(ld_u16(b));
    uint32_t qh = ld_u32_unaligned(b + 2);
    int i = e & 15;
    uint8_t byte = b[6 + i];
    int32_t q;
    if (e < 16) q = (int32_t)(((uint32_t)(byte & 0xF)) | (((qh >> i) << 4) & 0x10)) - 16;
    else q = (int32_t)(((uint32_t)(byte >> 4)) | ((qh >> (i + 12)) & 0x10)) - 16;
    return __fmul_rn(d, (float)q);
}
// quant.rs:167-182
template <> __device__ __forceinline__ float deq_elem<GGC_Q5_1>(const uint8_t* b, int e) {
    float d = f16_ref(ld_u16(b)), m = f16_ref(ld_u16(b + 2));
    uint32_t qh = ld_u32_unaligned(b + 4);
    int i = e & 15;
    uint8_t byte = b[8 + i];
    uint32_t q;
    if (e < 16) q = ((uint32_t)(byte & 0xF)) | (((qh >> i) << 4) & 0x10);
    else q = ((uint32_t)(byte >> 4)) | ((qh >> (i + 12)) & 0x10);
    return __fadd_rn(__fmul_rn(d, (float)q), m);
}
// quant.rs:184-189
template <> __device__ __forceinline__ float deq_elem<GGC_Q8_0>(const uint8_t* b, int e) {
    return __fmul_rn(f16_ref(ld_u16(b)), (float)(int8_t)b[2 + e]);
}
// quant.rs:193-207
template <> __device__ __forceinline__ float deq_elem<GGC_Q2_K>(const uint8_t* b, int e) {
    float d = f16_ref(ld_u16(b + 80)), dmin = f16_ref(ld_u16(b + 82));
    int j = e >> 4;
    float s = (float)k_scale4(b, j);
    float m = __fmul_rn(__fsub_rn(s, 8.0f), dmin);
    float s0 = (s < 8.0f) ? __fmul_rn(s, d) : __fadd_rn(__fmul_rn(s, dmin), m);
    float q = (float)((b[16 + e / 4] >> ((e % 4) * 2)) & 0x3);
    return __fadd_rn(__fmul_rn(s0, q), (s < 8.0f) ? 0.0f : m);
}
// quant.rs:223-240
template <int DOFF>
__device__ __forceinline__ float deq_q3_elem(const uint8_t* b, int i) {
    float d = f16_ref(ld_u16(b + DOFF));
    int si = i >> 4;
    uint8_t lo = (b[96 + si / 2] >> ((si % 2) * 4)) & 0xF;
    uint8_t hi = (b[96 + 8 + si / 4] >> ((si % 4) * 2)) & 0x3;
    int32_t sc = (int32_t)(uint8_t)(lo | (hi << 4)) - 32;
    int32_t ql = (b[32 + i / 4] >> ((i % 4) * 2)) & 3;
    int32_t qh = (b[i / 8] >> (i % 8)) & 1;
    int32_t q = (qh ^ 1) * 4 - ql;
    return __fmul_rn(__fmul_rn(d, (float)sc), (float)q);
}
template <> __device__ __forceinline__ float deq_elem<GGC_Q3_K_S>(const uint8_t* b, int e) { return deq_q3_elem<108>(b, e); }
template <> __device__ __forceinline__ float deq_elem<GGC_Q3_K_L>(const uint8_t* b, int e) { return deq_q3_elem<108>(b, e); }
template <> __device__ __forceinline__ float deq_elem<GGC_Q3_K_M>(const uint8_t* b, int e) { return deq_q3_elem<112>(b, e); }
// quant.rs:257-281
template <> __device__ __forceinline__ float deq_elem<GGC_Q4_K>(const uint8_t* b, int e) {
    float d = f16_ref(ld_u16(b)), dmin = f16_ref(ld_u16(b + 2));
    int group = e >> 6, in_grp = e & 63, is_high = in_grp >> 5;
    int byte_in_qs = group * 32 + (in_grp & 31);
    uint32_t sc, mn;
    k_scale_min_6bit(b + 4, group * 2 + is_high, sc, mn);
    float s1 = __fmul_rn((float)sc, d);
    float s2 = __fmul_rn((float)mn, dmin);
    uint8_t byte = b[16 + byte_in_qs];
    uint32_t val = is_high ? (byte >> 4) : (byte & 0x0F);
    return __fsub_rn(__fmul_rn(s1, (float)val), s2);
}
// quant.rs:283-306
template <> __device__ __forceinline__ float deq_elem<GGC_Q5_K>(const uint8_t* b, int k) {
    float d = f16_ref(ld_u16(b)), dmin = f16_ref(ld_u16(b + 2));
    uint32_t sc, mn;
    k_scale_min_6bit(b + 4, k >> 5, sc, mn);
    float s1 = __fmul_rn((float)sc, d);
    float s2 = __fmul_rn((float)mn, dmin);
    uint8_t byte = b[48 + k / 2];
    int byte_idx = k >> 1;
    uint32_t qh_bit = (b[16 + byte_idx / 8] >> (byte_idx % 8)) & 1;
    uint32_t q = ((k & 1) == 0) ? (((uint32_t)(byte & 0xF)) | (qh_bit << 4))
                                : (((uint32_t)(byte >> 4)) | (qh_bit << 4));
    return __fsub_rn(__fmul_rn(s1, (float)q), s2);
}
// quant.rs:308-337
template <> __device__ __forceinline__ float deq_elem<GGC_Q6_K>(const uint8_t* b, int e) {
    float d = f16_ref(ld_u16(b + 208));
    int n = e >> 7, r = e & 127, t = r >> 5, l = r & 31, is = l / 16;
    uint8_t ql = b[n * 64 + ((t & 1) ? 32 : 0) + l];
    uint8_t qh = b[128 + n * 32 + l];
    uint32_t q = ((t < 2) ? (ql & 0xF) : (ql >> 4)) | (((qh >> (2 * t)) & 3) << 4);
    int8_t sc = (int8_t)b[192 + n * 8 + is + 2 * t];
    return __fmul_rn(__fmul_rn(d, (float)sc), (float)((int32_t)q - 32));
}
// quant.rs:339-345
template <> __device__ __forceinline__ float deq_elem<GGC_Q8_K>(const uint8_t* b, int e) {
    return __fmul_rn(__uint_as_float(ld_u32_unaligned(b)), (float)(int8_t)b[4 + e]);
}

// Whole-tensor dequantisation (quant::dequantize): one thread per output
// element; consecutive threads write consecutive floats (coalesced stores), the
// few bytes each reads come from L1.
template <int DT>
__global__ void __launch_bounds__(256) k_dequantize(const uint8_t* __restrict__ raw, uint64_t n,
                                                    float* __restrict__ out) {
    constexpr int BS = block_size_of(DT), BB = block_bytes_of(DT);
    pdl_trigger();
    pdl_wait();
    uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        uint64_t blk = i / BS;
        int e = (int)(i - blk * BS);
        const uint8_t* b = raw + blk * BB + (BS == 1 ? 0 : 0);
        out[i] = deq_elem<DT>(b, e);
    }
}

// Embedding gather (llama.rs:367-383): dequantise row `tok` of token_embd (raw
// GGUF rows of `d` elements) into hidden[d]; an out-of-range id sets an error flag.
template <int DT>
__global__ void __launch_bounds__(256) k_embed_row(const uint8_t* __restrict__ raw, uint64_t n_rows,
                                                   uint32_t d, const uint32_t* __restrict__ tok_ptr,
                                                   float* __restrict__ hidden, int* __restrict__ errf) {
    constexpr int BS = block_size_of(DT), BB = block_bytes_of(DT);
    pdl_trigger();
    pdl_wait();
    uint32_t tok = *tok_ptr;
    if ((uint64_t)tok >= n_rows) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicExch(&errf[ERRF_EMBED_OOB], (int)tok + 1);
        return;
    }
    uint64_t row_bytes = (uint64_t)(d / BS) * BB;
    const uint8_t* row = raw + (uint64_t)tok * row_bytes;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < d; i += gridDim.x * blockDim.x) {
        uint32_t blk = i / BS;
        hidden[i] = deq_elem<DT>(row + (uint64_t)blk * BB, (int)(i - blk * BS));
    }
}

// quant_matvec on raw GGUF rows (quant.rs:526-570): one warp per row, lanes
// stride over the row's blocks, each dequantising its block exactly and
// accumulating in f32; the warp's partial sums are reduced with shuffles.
template <int DT>
__global__ void __launch_bounds__(256) k_matvec_raw(const uint8_t* __restrict__ w, uint64_t rows,
                                                    uint64_t cols, const float* __restrict__ x,
                                                    float* __restrict__ y) {
    constexpr int BS = block_size_of(DT), BB = block_bytes_of(DT);
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const uint64_t warps = (uint64_t)gridDim.x * (blockDim.x >> 5);
    const uint64_t row_bytes = cols / BS * BB;
    const uint64_t nblk = cols / BS;
    for (uint64_t r = (uint64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
        const uint8_t* row = w + r * row_bytes;
        float acc = 0.0f;
        if (BS == 1) {
            for (uint64_t c = lane; c < cols; c += 32) acc = __fadd_rn(acc, __fmul_rn(deq_elem<DT>(row + c * BB, 0), x[c]));
        } else {
            for (uint64_t b = lane; b < nblk; b += 32) {
                const uint8_t* blk = row + b * BB;
                const float* xb = x + b * BS;
#pragma unroll 4
                for (int e = 0; e < BS; ++e) acc = __fadd_rn(acc, __fmul_rn(deq_elem<DT>(blk, e), xb[e]));
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) y[r] = acc;
    }
}

// Runs F<DT> for the runtime dtype.  Returns false for an unsupported dtype.
template <template <int> class F, class... A>
bool dispatch_dtype(int dt, A&&... a) {
    switch (dt) {
        case GGC_F32: F<GGC_F32>::run(a...); return true;
        case GGC_F16: F<GGC_F16>::run(a...); return true;
        case GGC_BF16: F<GGC_BF16>::run(a...); return true;
        case GGC_Q4_0: F<GGC_Q4_0>::run(a...); return true;
        case GGC_Q4_1: F<GGC_Q4_1>::run(a...); return true;
        case GGC_Q5_0: F<GGC_Q5_0>::run(a...); return true;
        case GGC_Q5_1: F<GGC_Q5_1>::run(a...); return true;
        case GGC_Q8_0: F<GGC_Q8_0>::run(a...); return true;
        case GGC_Q2_K: F<GGC_Q2_K>::run(a...); return true;
        case GGC_Q3_K_S: F<GGC_Q3_K_S>::run(a...); return true;
        case GGC_Q3_K_M: F<GGC_Q3_K_M>::run(a...); return true;
        case GGC_Q3_K_L: F<GGC_Q3_K_L>::run(a...); return true;
        case GGC_Q4_K: F<GGC_Q4_K>::run(a...); return true;
        case GGC_Q5_K: F<GGC_Q5_K>::run(a...); return true;
        case GGC_Q6_K: F<GGC_Q6_K>::run(a...); return true;
        case GGC_Q8_K: F<GGC_Q8_K>::run(a...); return true;
        default: return false;
    }
}

}  // namespace ggc
