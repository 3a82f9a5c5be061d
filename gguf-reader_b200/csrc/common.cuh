// common.cuh -- shared definitions of libgguf_cuda (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "../../include/gguf_cuda.h"

namespace ggc {

// ---------------------------------------------------------------------------
// dtype geometry (src/types.rs:182-220)
// ---------------------------------------------------------------------------
__host__ __device__ constexpr int block_size_of(int dt) {
    return (dt == GGC_F32 || dt == GGC_F16 || dt == GGC_BF16) ? 1
         : (dt == GGC_Q4_0 || dt == GGC_Q4_1 || dt == GGC_Q5_0 || dt == GGC_Q5_1 || dt == GGC_Q8_0) ? 32
         : (dt == GGC_Q2_K || dt == GGC_Q3_K_S || dt == GGC_Q3_K_M || dt == GGC_Q3_K_L ||
            dt == GGC_Q4_K || dt == GGC_Q5_K || dt == GGC_Q6_K || dt == GGC_Q8_K) ? 256
         : -1;
}
__host__ __device__ constexpr int block_bytes_of(int dt) {
    return dt == GGC_F32 ? 4 : (dt == GGC_F16 || dt == GGC_BF16) ? 2
         : dt == GGC_Q4_0 ? 18 : dt == GGC_Q4_1 ? 20 : dt == GGC_Q5_0 ? 22 : dt == GGC_Q5_1 ? 24
         : dt == GGC_Q8_0 ? 34 : dt == GGC_Q2_K ? 84
         : (dt == GGC_Q3_K_S || dt == GGC_Q3_K_L) ? 110 : dt == GGC_Q3_K_M ? 114
         : dt == GGC_Q4_K ? 144 : dt == GGC_Q5_K ? 176 : dt == GGC_Q6_K ? 210 : dt == GGC_Q8_K ? 292
         : -1;
}

inline const char* dtype_name(int dt) {
    switch (dt) {
        case GGC_F32: return "F32"; case GGC_F16: return "F16"; case GGC_BF16: return "BF16";
        case GGC_Q4_0: return "Q4_0"; case GGC_Q4_1: return "Q4_1"; case GGC_Q5_0: return "Q5_0";
        case GGC_Q5_1: return "Q5_1"; case GGC_Q8_0: return "Q8_0"; case GGC_Q2_K: return "Q2_K";
        case GGC_Q3_K_S: return "Q3_K_S"; case GGC_Q3_K_M: return "Q3_K_M"; case GGC_Q3_K_L: return "Q3_K_L";
        case GGC_Q4_K: return "Q4_K"; case GGC_Q5_K: return "Q5_K"; case GGC_Q6_K: return "Q6_K";
        case GGC_Q8_K: return "Q8_K";
        default: return "Unknown";
    }
}

// ---------------------------------------------------------------------------
// thread-local last error (GgufError payload)
// ---------------------------------------------------------------------------
ggc_error_info& tls_error();
int set_error(int status, const char* fmt, ...);
int set_dequant_error(int dtype, uint64_t expected, uint64_t actual, const char* what);
int set_shape_error(uint64_t elements, uint64_t block, const char* what);

#define GGC_CUDA_TRY(expr)                                                                   \
    do {                                                                                     \
        cudaError_t e__ = (expr);                                                            \
        if (e__ != cudaSuccess)                                                              \
            return ::ggc::set_error(GGC_ERR_CUDA, "%s:%d %s: %s", __FILE__, __LINE__, #expr, \
                                    cudaGetErrorString(e__));                                \
    } while (0)

#define GGC_TRY(expr)                 \
    do {                              \
        int s__ = (expr);             \
        if (s__ != GGC_OK) return s__; \
    } while (0)

// ---------------------------------------------------------------------------
// number formats with the reference's semantics
// ---------------------------------------------------------------------------
// quant.rs:12-37: exact half -> f32, except NaN becomes the canonical f32 NaN
// (0x7FC00000, sign dropped).  __half2float is exact for every non-NaN half.
__device__ __forceinline__ float f16_ref(uint16_t h) {
    if ((h & 0x7C00u) == 0x7C00u && (h & 0x03FFu)) return __uint_as_float(0x7FC00000u);
    return __half2float(__ushort_as_half(h));
}
// quant.rs:40-42
__device__ __forceinline__ float bf16_ref(uint16_t h) { return __uint_as_float((uint32_t)h << 16); }

__device__ __forceinline__ uint16_t ld_u16(const uint8_t* p) {
    return (uint16_t)(p[0] | (p[1] << 8));
}
__device__ __forceinline__ uint32_t ld_u32_unaligned(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

// byte permute: result byte i = byte sel[i] of {b:a} (PTX prmt.b32)
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

// ---------------------------------------------------------------------------
// programmatic dependent launch (PDL): every kernel waits on its predecessor
// before it reads a predecessor's output or exits, so completion stays transitive.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;"); }

// error-flag slots in the context's device status block
enum : int {
    ERRF_NAN_ATTN = 0,      // NaN in attention output (value = layer + 1)
    ERRF_NAN_FFN = 1,       // NaN in ffn output (value = layer + 1)
    ERRF_EMBED_OOB = 2,     // token id >= rows of token_embd
    ERRF_NAN_LOGITS = 3,    // NaN logit (greedy sampling undefined)
    ERRF_TIMEOUT = 4,       // bounded wait expired
    ERRF_KV_OVERFLOW = 5,   // cache slot >= capacity
    ERRF_BAD_POS = 6,       // negative position (all keys masked)
    ERRF_COUNT = 8
};

template <class T>
__host__ __device__ constexpr T cdiv(T a, T b) { return (a + b - 1) / b; }

}  // namespace ggc
