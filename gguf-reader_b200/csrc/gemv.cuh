// gemv.cuh -- decode matvec over plane-layout weights (the hot path of a token).
//
// Replaces ops::matvec_colmajor_trans over materialised f32 weights
// (src/infer/ops.rs:172-227, called from src/infer/model/llama.rs:452-570) and
// quant::quant_matvec (src/infer/quant.rs:526-570): y[r] = sum_c W[r,c] * x[c]
// with W read once from HBM in its quantized form.
//
// Work mapping.  A warp owns R consecutive rows ("row group") and walks their
// 16-byte chunks of plane 0; lane l takes chunks l, l+32, ... so each load
// instruction of the warp reads 512 contiguous bytes.  The activation x is
// stored once per CTA in shared memory in chunk order (xs[t][c] = float4 of the
// 4 elements chunk c consumes at step t), so the float4 reads of a warp are
// consecutive and bank-conflict free.
//
// Arithmetic.  An unsigned code u < 128 is turned into the float 1 + u/128 with
// a single byte permute (0x3F | 0x80+u as the two top bytes); a chunk then costs
// one PRMT + one FFMA per element.  With S = sum (1 + u_i/128) x_i and
// X = sum x_i over the same scale group, sum u_i x_i = 128 (S - X).  The group
// sums X are computed once per CTA.  8-bit codes use 2^23 + u and an exact FADD.
#pragma once
#include "common.cuh"
#include "planes.cuh"
#include "mbarrier.cuh"
#include "allreduce.cuh"

namespace ggc {

// ---------------------------------------------------------------------------
// loads
// ---------------------------------------------------------------------------
// shared-memory loads of the tile staged by the bulk copies
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ uint4 ld_v4(const uint8_t* p) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(smem_u32(p)));
    return v;
}
__device__ __forceinline__ uint2 ld_v2(const uint8_t* p) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(smem_u32(p)));
    return v;
}
__device__ __forceinline__ uint32_t ld_u32(const uint8_t* p) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)));
    return v;
}
__device__ __forceinline__ uint32_t ld_u16g(const uint8_t* p) {
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(smem_u32(p)));
    return v;
}
__device__ __forceinline__ uint32_t ld_u8g(const uint8_t* p) {
    unsigned short v;
    asm volatile("ld.shared.u8 %0, [%1];" : "=h"(v) : "r"(smem_u32(p)));
    return v & 0xFFu;
}
#define ld_stream_v4 ld_v4

__device__ __forceinline__ float h2f(uint32_t h) { return f16_ref((uint16_t)h); }

// S += sum_k (1 + byte_k(ub)/128 with byte_k = 0x80|u_k) * x_k
__device__ __forceinline__ float fma_b4(uint32_t ub, float4 x, float acc) {
    acc = fmaf(__uint_as_float(prmt(ub, 0x3F000000u, 0x7044u)), x.x, acc);
    acc = fmaf(__uint_as_float(prmt(ub, 0x3F000000u, 0x7144u)), x.y, acc);
    acc = fmaf(__uint_as_float(prmt(ub, 0x3F000000u, 0x7244u)), x.z, acc);
    acc = fmaf(__uint_as_float(prmt(ub, 0x3F000000u, 0x7344u)), x.w, acc);
    return acc;
}
// acc += sum_k int8(byte_k(w)) * x_k
__device__ __forceinline__ float fma_q8(uint32_t w, float4 x, float acc) {
    const uint32_t u = w ^ 0x80808080u;
    acc = fmaf(__uint_as_float(prmt(u, 0x4B000000u, 0x7650u)) - 8388736.0f, x.x, acc);
    acc = fmaf(__uint_as_float(prmt(u, 0x4B000000u, 0x7651u)) - 8388736.0f, x.y, acc);
    acc = fmaf(__uint_as_float(prmt(u, 0x4B000000u, 0x7652u)) - 8388736.0f, x.z, acc);
    acc = fmaf(__uint_as_float(prmt(u, 0x4B000000u, 0x7653u)) - 8388736.0f, x.w, acc);
    return acc;
}
__device__ __forceinline__ uint32_t nib_lo(uint32_t w) { return (w & 0x0F0F0F0Fu) | 0x80808080u; }
__device__ __forceinline__ uint32_t nib_hi(uint32_t w) { return ((w >> 4) & 0x0F0F0F0Fu) | 0x80808080u; }

// 6-bit (scale, min) j of the 12 K-quant scale bytes held in three words (quant.rs:116-124)
__device__ __forceinline__ void kq_scale_min(uint32_t s0, uint32_t s1, uint32_t s2, int j, float& sc, float& mn) {
    auto byte = [&](int i) -> uint32_t {
        uint32_t w = i < 4 ? s0 : (i < 8 ? s1 : s2);
        return (w >> (8 * (i & 3))) & 0xFFu;
    };
    if (j < 4) {
        sc = (float)(byte(j) & 0x3F);
        mn = (float)(byte(j + 4) & 0x3F);
    } else {
        sc = (float)((byte(j + 4) & 0x0F) | ((byte(j - 4) >> 6) << 4));
        mn = (float)((byte(j + 4) >> 4) | ((byte(j) >> 6) << 4));
    }
}

// ---------------------------------------------------------------------------
// per-format chunk decoders
//   E elements per chunk, T = E/4 float4 steps, G scale groups per chunk.
//   elem(c, t, j): column of the j-th float of step t of chunk c.
//   group(t): scale group of step t.
// ---------------------------------------------------------------------------
template <int DT> struct Dec;

template <> struct Dec<GGC_Q4_0> {
    static constexpr int E = 32, T = 8, G = 1;
    struct Ch { uint4 q; uint32_t d; };
    __device__ static int elem(int c, int t, int j) { return c * 32 + 2 * (4 * (t >> 1) + j) + (t & 1); }
    __device__ static int group(int) { return 0; }
    __device__ static Ch load(const TileView& m, uint32_t r, uint32_t c) {
        return Ch{ld_stream_v4(m.p[0] + r * m.pitch[0] + c * 16u), ld_u16g(m.p[1] + r * m.pitch[1] + c * 2u)};
    }
    __device__ static float dot(const Ch& ch, const float4* xs, int n, const float* sx) {
        const uint32_t w[4] = {ch.q.x, ch.q.y, ch.q.z, ch.q.w};
        float S = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) { S = fma_b4(nib_lo(w[i]), xs[(2 * i) * n], S); S = fma_b4(nib_hi(w[i]), xs[(2 * i + 1) * n], S); }
        // value = d * (q - 8):  sum (q-8) x = 128 (S - X) - 8 X
        return h2f(ch.d) * fmaf(128.f, S - sx[0], -8.f * sx[0]);
    }
};

template <> struct Dec<GGC_Q4_1> {
    static constexpr int E = 32, T = 8, G = 1;
    struct Ch { uint4 q; uint32_t dm; };
    __device__ static int elem(int c, int t, int j) { return c * 32 + 2 * (4 * (t >> 1) + j) + (t & 1); }
    __device__ static int group(int) { return 0; }
    __device__ static Ch load(const TileView& m, uint32_t r, uint32_t c) {
        return Ch{ld_stream_v4(m.p[0] + r * m.pitch[0] + c * 16u), ld_u32(m.p[1] + r * m.pitch[1] + c * 4u)};
    }
    __device__ static float dot(const Ch& ch, const float4* xs, int n, const float* sx) {
        const uint32_t w[4] = {ch.q.x, ch.q.y, ch.q.z, ch.q.w};
        float S = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) { S = fma_b4(nib_lo(w[i]), xs[(2 * i) * n], S); S = fma_b4(nib_hi(w[i]), xs[(2 * i + 1) * n], S); }
        // value = d q + m
        return fmaf(h2f(ch.dm & 0xFFFF) * 128.f, S - sx[0], h2f(ch.dm >> 16) * sx[0]);
    }
};

template <int DT_> struct DecQ5_01 {
    static constexpr int E = 32, T = 8, G = 1;
    static constexpr bool HAS_M = DT_ == GGC_Q5_1;
    struct Ch { uint4 q; uint32_t qh; uint32_t d; };
    __device__ static int elem(int c, int t, int j) { return c * 32 + (4 * (t >> 1) + j) + 16 * (t & 1); }
    __device__ static int group(int) { return 0; }
    __device__ static Ch load(const TileView& m, uint32_t r, uint32_t c) {
        Ch ch;
        ch.q = ld_stream_v4(m.p[0] + r * m.pitch[0] + c * 16u);
        ch.qh = ld_u32(m.p[1] + r * m.pitch[1] + c * 4u);
        ch.d = HAS_M ? ld_u32(m.p[2] + r * m.pitch[2] + c * 4u) : ld_u16g(m.p[2] + r * m.pitch[2] + c * 2u);
        return ch;
    }
    __device__ static float dot(const Ch& ch, const float4* xs, int n, const float* sx) {
        const uint32_t w[4] = {ch.q.x, ch.q.y, ch.q.z, ch.q.w};
        float S = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t hl = ((ch.qh << (4 - i)) & 0x10101010u) | 0x80808080u;
            const uint32_t hh = ((ch.qh >> i) & 0x10101010u) | 0x80808080u;
            S = fma_b4((w[i] & 0x0F0F0F0Fu) | hl, xs[(2 * i) * n], S);
            S = fma_b4(((w[i] >> 4) & 0x0F0F0F0Fu) | hh, xs[(2 * i + 1) * n], S);
        }
        const float d = h2f(ch.d & 0xFFFF);
        if (HAS_M) return fmaf(d * 128.f, S - sx[0], h2f(ch.d >> 16) * sx[0]);   // d u + m
        return d * fmaf(128.f, S - sx[0], -16.f * sx[0]);                         // d (u - 16)
    }
};
template <> struct Dec<GGC_Q5_0> : DecQ5_01<GGC_Q5_0> {};
template <> struct Dec<GGC_Q5_1> : DecQ5_01<GGC_Q5_1> {};

template <> struct Dec<GGC_Q8_0> {
    static constexpr int E = 16, T = 4, G = 0;
    struct Ch { uint4 q; uint32_t d; };
    __device__ static int elem(int c, int t, int j) { return c * 16 + 4 * t + j; }
    __device__ static int group(int) { return 0; }
    __device__ static Ch load(const TileView& m, uint32_t r, uint32_t c) {
        return Ch{ld_stream_v4(m.p[0] + r * m.pitch[0] + c * 16u), ld_u16g(m.p[1] + r * m.pitch[1] + (c >> 1) * 2u)};
    }
    __device__ static float dot(const Ch& ch, const float4* xs, int n, const float*) {
        float a = fma_q8(ch.q.x, xs[0], 0.f);
        a = fma_q8(ch.q.y, xs[n], a);
        a = fma_q8(ch.q.z, xs[2 * n], a);
        a = fma_q8(ch.q.w, xs[3 * n], a);
        return h2f(ch.d) * a;
    }
};

template <> struct Dec<GGC_Q8_K> {
    static constexpr int E = 16, T = 4, G = 0;
    struct Ch { uint4 q; uint32_t d; };
    __device__ static int elem(int c, int t, int j) { return c * 16 + 4 * t + j; }
    __device__ static int group(int) { return 0; }
    __device__ static Ch load(const TileView& m, uint32_t r, uint32_t c) {
        return Ch{ld_stream_v4(m.p[0] + r * m.pitch[0] + c * 16u), ld_u32(m.p[1] + r * m.pitch[1] + (c >> 4) * 4u)};
    }
    __device__ static float dot(const Ch& ch, const float4* xs, int n, const float*) {
        float a = fma_q8(ch.q.x, xs[0], 0.f);
        a = fma_q8(ch.q.y, xs[n], a);
        a = fma_q8(ch.q.z, xs[2 * n], a);
        a = fma_q8(ch.q.w, xs[3 * n], a);
        return __uint_as_float(ch.d) * a;
    }
};

template <> struct Dec<GGC_Q2_K> {
    static constexpr int E = 64, T = 16, G = 4;
    struct Ch { uint4 q; uint32_t sc; uint32_t dd; };
    __device__ static int elem(int c, int t, int j) { return c * 64 + 16 * (t >> 2) + 4 * j + (t & 3); }
    __device__ static int group(int t) { return t >> 2; }
    __device__ static Ch load(const TileView& m, uint32_t r, uint32_t c) {
        const uint32_t b = c >> 2, p = c & 3;
        Ch ch;
        ch.q = ld_stream_v4(m.p[0] + r * m.pitch[0] + c * 16u);
        ch.sc = ld_u16g(m.p[1] + r * m.pitch[1] + b * 16u + 14u - 2u * p);   // bytes 14-2p, 15-2p
        ch.dd = ld_u32(m.p[2] + r * m.pitch[2] + b * 4u);
        return ch;
    }
    __device__ static float dot(const Ch& ch, const float4* xs, int n, const float* sx) {
        const uint32_t w[4] = {ch.q.x, ch.q.y, ch.q.z, ch.q.w};
        const float d = h2f(ch.dd & 0xFFFF), dmin = h2f(ch.dd >> 16);
        float out = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float S = 0.f;
#pragma unroll
            for (int s = 0; s < 4; ++s) S = fma_b4(((w[i] >> (2 * s)) & 0x03030303u) | 0x80808080u, xs[(4 * i + s) * n], S);
            // sub-block j = 4p + i; k_scale4(j) (quant.rs:101-108)
            const uint32_t byte = (i < 2) ? (ch.sc >> 8) : ch.sc;
            const float sv = (float)((byte >> (4 * (i & 1))) & 0xF);
            const float mm = (sv - 8.0f) * dmin;
            const float s0 = (sv < 8.0f) ? sv * d : fmaf(sv, dmin, mm);
            const float add = (sv < 8.0f) ? 0.0f : mm;
            out += fmaf(s0 * 128.f, S - sx[i], add * sx[i]);
        }
        return out;
    }
};

template <int DT_> struct DecQ3K {
    static constexpr int E = 64, T = 16, G = 4;
    struct Ch { uint4 q; uint2 hm; uint32_t lo; uint32_t hi; uint32_t d; };
    __device__ static int elem(int c, int t, int j) { return c * 64 + 16 * (t >> 2) + 4 * j + (t & 3); }
    __device__ static int group(int t) { return t >> 2; }
    __device__ static Ch load(const TileView& m, uint32_t r, uint32_t c) {
        const uint32_t b = c >> 2, p = c & 3;
        Ch ch;
        ch.q = ld_stream_v4(m.p[0] + r * m.pitch[0] + c * 16u);
        ch.hm = ld_v2(m.p[1] + r * m.pitch[1] + c * 8u);
        const uint8_t* sb = m.p[2] + r * m.pitch[2] + b * 12u;
        ch.lo = ld_u16g(sb + 2u * p);
        ch.hi = ld_u8g(sb + 8u + p);
        ch.d = ld_u16g(m.p[3] + r * m.pitch[3] + b * 2u);
        return ch;
    }
    __device__ static float dot(const Ch& ch, const float4* xs, int n, const float* sx) {
        const uint32_t w[4] = {ch.q.x, ch.q.y, ch.q.z, ch.q.w};
        const float d = h2f(ch.d);
        float out = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t hw = (i < 2) ? ch.hm.x : ch.hm.y;
            float S = 0.f;
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                const int sh = s + 4 * (i & 1);
                const uint32_t ql = (w[i] >> (2 * s)) & 0x03030303u;
                const uint32_t h4 = (sh >= 2 ? (hw >> (sh - 2)) : (hw << (2 - sh))) & 0x04040404u;
                // u = q + 3 = (ql ^ 3) | ((h ^ 1) << 2), q = (h^1)*4 - ql (quant.rs:237)
                S = fma_b4((ql | h4) ^ 0x87878787u, xs[(4 * i + s) * n], S);
            }
            const int sc = (int)(((ch.lo >> (4 * i)) & 0xF) | (((ch.hi >> (2 * i)) & 3) << 4)) - 32;
            out += (d * (float)sc) * fmaf(128.f, S - sx[i], -3.f * sx[i]);
        }
        return out;
    }
};
template <> struct Dec<GGC_Q3_K_S> : DecQ3K<GGC_Q3_K_S> {};
template <> struct Dec<GGC_Q3_K_M> : DecQ3K<GGC_Q3_K_M> {};
template <> struct Dec<GGC_Q3_K_L> : DecQ3K<GGC_Q3_K_L> {};

template <> struct Dec<GGC_Q4_K> {
    static constexpr int E = 32, T = 8, G = 2;
    // dd = d | dmin << 16; sc / mn = bytes of sub-blocks (2g, 2g+1) of the unpacked scale plane
    struct Ch { uint4 q; uint32_t dd; uint32_t sc; uint32_t mn; };
    // chunk c: block c/8, part p = c%8 -> qs bytes 32g + l0 .. +15 (g = p/2, l0 = 16(p%2)):
    // low nibbles are elements 64g + l0 + i (sub-block 2g), high nibbles 64g + 32 + l0 + i (2g+1)
    __device__ static int elem(int c, int t, int j) {
        const int b = c >> 3, p = c & 7;
        return b * 256 + 64 * (p >> 1) + 32 * (t & 1) + 16 * (p & 1) + 4 * (t >> 1) + j;
    }
    __device__ static int group(int t) { return t & 1; }
    __device__ static Ch load(const TileView& m, uint32_t r, uint32_t c) {
        const uint32_t b = c >> 3, g = (c & 7) >> 1;
        const uint8_t* scm = m.p[2] + r * m.pitch[2] + b * 16u;
        return Ch{ld_v4(m.p[0] + r * m.pitch[0] + c * 16u), ld_u32(m.p[1] + r * m.pitch[1] + b * 4u),
                  ld_u16g(scm + 2u * g), ld_u16g(scm + 8u + 2u * g)};
    }
    __device__ static float dot(const Ch& ch, const float4* xs, int n, const float* sx, int) {
        const uint32_t w[4] = {ch.q.x, ch.q.y, ch.q.z, ch.q.w};
        float SA = 0.f, SB = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) { SA = fma_b4(nib_lo(w[i]), xs[(2 * i) * n], SA); SB = fma_b4(nib_hi(w[i]), xs[(2 * i + 1) * n], SB); }
        const float d = h2f(ch.dd & 0xFFFF), dmin = h2f(ch.dd >> 16);
        // value = (sc d) q - (mn dmin)  (quant.rs:275-279)
        float r = fmaf(((float)(ch.sc & 0xFF) * d) * 128.f, SA - sx[0], -((float)(ch.mn & 0xFF) * dmin) * sx[0]);
        return r + fmaf(((float)(ch.sc >> 8) * d) * 128.f, SB - sx[1], -((float)(ch.mn >> 8) * dmin) * sx[1]);
    }
};

template <> struct Dec<GGC_Q5_K> {
    static constexpr int E = 32, T = 8, G = 1;
    struct Ch { uint4 q; uint32_t qh; uint32_t dd; uint32_t sc; uint32_t mn; };
    // chunk c: block c/8, sub-block p = c%8; qs byte i of the chunk holds elements 32p + 2i (low) and +1 (high)
    __device__ static int elem(int c, int t, int j) {
        const int b = c >> 3, p = c & 7;
        return b * 256 + 32 * p + 2 * (4 * (t >> 1) + j) + (t & 1);
    }
    __device__ static int group(int) { return 0; }
    __device__ static Ch load(const TileView& m, uint32_t r, uint32_t c) {
        const uint32_t b = c >> 3, p = c & 7;
        const uint8_t* scm = m.p[3] + r * m.pitch[3] + b * 16u;
        Ch ch;
        ch.q = ld_v4(m.p[0] + r * m.pitch[0] + c * 16u);
        ch.qh = ld_u32(m.p[1] + r * m.pitch[1] + b * 16u + (p >> 1) * 4u);
        ch.dd = ld_u32(m.p[2] + r * m.pitch[2] + b * 4u);
        ch.sc = ld_u8g(scm + p);
        ch.mn = ld_u8g(scm + 8u + p);
        return ch;
    }
    __device__ static float dot(const Ch& ch, const float4* xs, int n, const float* sx, int c) {
        const uint32_t w[4] = {ch.q.x, ch.q.y, ch.q.z, ch.q.w};
        const int p = c & 7;
        float S = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t hb = (((p & 1) ? (ch.qh >> i) : (ch.qh << (4 - i))) & 0x10101010u) | 0x80808080u;
            S = fma_b4((w[i] & 0x0F0F0F0Fu) | hb, xs[(2 * i) * n], S);
            S = fma_b4(((w[i] >> 4) & 0x0F0F0F0Fu) | hb, xs[(2 * i + 1) * n], S);
        }
        const float d = h2f(ch.dd & 0xFFFF), dmin = h2f(ch.dd >> 16);
        return fmaf(((float)ch.sc * d) * 128.f, S - sx[0], -((float)ch.mn * dmin) * sx[0]);
    }
};

template <> struct Dec<GGC_Q6_K> {
    static constexpr int E = 32, T = 8, G = 2;
    struct Ch { uint4 q; uint4 qh; uint2 sc; uint32_t d; };
    // chunk c: block c/8, p = c%8, half n = p/4, part = p%4.  part 0,1: ql bytes l = 16 part + i
    // give q1 (element 128n + l, low) and q3 (+64, high); part 2,3: ql bytes 32 + l give q2 (+32) and q4 (+96)
    __device__ static int elem(int c, int t, int j) {
        const int b = c >> 3, p = c & 7, n = p >> 2, part = p & 3;
        const int l = 16 * (part & 1) + 4 * (t >> 1) + j;
        return b * 256 + 128 * n + l + (part < 2 ? 0 : 32) + 64 * (t & 1);
    }
    __device__ static int group(int t) { return t & 1; }
    __device__ static Ch load(const TileView& m, uint32_t r, uint32_t c) {
        const uint32_t b = c >> 3, p = c & 7, n = p >> 2, part = p & 3;
        Ch ch;
        ch.q = ld_stream_v4(m.p[0] + r * m.pitch[0] + c * 16u);
        ch.qh = ld_v4(m.p[1] + r * m.pitch[1] + b * 64u + n * 32u + 16u * (part & 1));
        ch.sc = ld_v2(m.p[2] + r * m.pitch[2] + b * 16u + n * 8u);
        ch.d = ld_u16g(m.p[3] + r * m.pitch[3] + b * 2u);
        return ch;
    }
    __device__ static float dot(const Ch& ch, const float4* xs, int n, const float* sx, int c) {
        const uint32_t w[4] = {ch.q.x, ch.q.y, ch.q.z, ch.q.w};
        const uint32_t h[4] = {ch.qh.x, ch.qh.y, ch.qh.z, ch.qh.w};
        const int part = c & 3;
        float SA = 0.f, SB = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            uint32_t hl, hh;
            if (part < 2) { hl = (h[i] << 4) & 0x30303030u; hh = h[i] & 0x30303030u; }
            else { hl = (h[i] << 2) & 0x30303030u; hh = (h[i] >> 2) & 0x30303030u; }
            SA = fma_b4((w[i] & 0x0F0F0F0Fu) | hl | 0x80808080u, xs[(2 * i) * n], SA);
            SB = fma_b4(((w[i] >> 4) & 0x0F0F0F0Fu) | hh | 0x80808080u, xs[(2 * i + 1) * n], SB);
        }
        // scales: is = part%2; q1 -> sc[is], q3 -> sc[is+4]; q2 -> sc[is+2], q4 -> sc[is+6]
        const int ia = (part & 1) + (part < 2 ? 0 : 2), ib = ia + 4;
        const uint32_t wa = ia < 4 ? ch.sc.x : ch.sc.y, wb = ch.sc.y;
        const float sca = (float)(int8_t)((wa >> (8 * (ia & 3))) & 0xFF);
        const float scb = (float)(int8_t)((wb >> (8 * (ib & 3))) & 0xFF);
        const float d = h2f(ch.d);
        // value = (d sc) (u - 32)
        float r = (d * sca) * fmaf(128.f, SA - sx[0], -32.f * sx[0]);
        return r + (d * scb) * fmaf(128.f, SB - sx[1], -32.f * sx[1]);
    }
};

template <> struct Dec<GGC_F16> {
    static constexpr int E = 8, T = 2, G = 0;
    struct Ch { uint4 q; };
    __device__ static int elem(int c, int t, int j) { return c * 8 + 4 * t + j; }
    __device__ static int group(int) { return 0; }
    __device__ static Ch load(const TileView& m, uint32_t r, uint32_t c) { return Ch{ld_stream_v4(m.p[0] + r * m.pitch[0] + c * 16u)}; }
    __device__ static float dot(const Ch& ch, const float4* xs, int n, const float*) {
        const uint32_t w[4] = {ch.q.x, ch.q.y, ch.q.z, ch.q.w};
        float a = 0.f;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            const float4 x = xs[t * n];
            float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&w[2 * t]));
            float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&w[2 * t + 1]));
            a = fmaf(f0.x, x.x, a); a = fmaf(f0.y, x.y, a); a = fmaf(f1.x, x.z, a); a = fmaf(f1.y, x.w, a);
        }
        return a;
    }
};

template <> struct Dec<GGC_BF16> {
    static constexpr int E = 8, T = 2, G = 0;
    struct Ch { uint4 q; };
    __device__ static int elem(int c, int t, int j) { return c * 8 + 4 * t + j; }
    __device__ static int group(int) { return 0; }
    __device__ static Ch load(const TileView& m, uint32_t r, uint32_t c) { return Ch{ld_stream_v4(m.p[0] + r * m.pitch[0] + c * 16u)}; }
    __device__ static float dot(const Ch& ch, const float4* xs, int n, const float*) {
        const uint32_t w[4] = {ch.q.x, ch.q.y, ch.q.z, ch.q.w};
        float a = 0.f;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            const float4 x = xs[t * n];
            a = fmaf(__uint_as_float(w[2 * t] << 16), x.x, a);
            a = fmaf(__uint_as_float(w[2 * t] & 0xFFFF0000u), x.y, a);
            a = fmaf(__uint_as_float(w[2 * t + 1] << 16), x.z, a);
            a = fmaf(__uint_as_float(w[2 * t + 1] & 0xFFFF0000u), x.w, a);
        }
        return a;
    }
};

template <> struct Dec<GGC_F32> {
    static constexpr int E = 4, T = 1, G = 0;
    struct Ch { uint4 q; };
    __device__ static int elem(int c, int, int j) { return c * 4 + j; }
    __device__ static int group(int) { return 0; }
    __device__ static Ch load(const TileView& m, uint32_t r, uint32_t c) { return Ch{ld_stream_v4(m.p[0] + r * m.pitch[0] + c * 16u)}; }
    __device__ static float dot(const Ch& ch, const float4* xs, int, const float*) {
        const float4 x = xs[0];
        float a = __uint_as_float(ch.q.x) * x.x;
        a = fmaf(__uint_as_float(ch.q.y), x.y, a);
        a = fmaf(__uint_as_float(ch.q.z), x.z, a);
        return fmaf(__uint_as_float(ch.q.w), x.w, a);
    }
};

template <int DT>
__device__ __forceinline__ float chunk_dot(const typename Dec<DT>::Ch& ch, const float4* xs, int n, const float* sx, int c) {
    if constexpr (DT == GGC_Q4_K || DT == GGC_Q5_K || DT == GGC_Q6_K) return Dec<DT>::dot(ch, xs, n, sx, c);
    else return Dec<DT>::dot(ch, xs, n, sx);
}


// ---------------------------------------------------------------------------
// integer decoders (dp4a).  x is quantised per (chunk, scale group) to a 22-bit
// fixed-point integer with a power-of-two scale gs (|x| / gs < 2^22, exact
// scaling), split into three 8-bit limbs (two unsigned, the top one signed).  One
// dp4a multiplies four weight codes by four limbs exactly in int32; the three
// limb sums recombine in f32.  L[3 t + k] is limb k of the four x values the
// chunk consumes at step t.  This keeps the per-element work on the half-rate
// integer pipes to ~0.75 dp4a + ~0.4 logic op (the float path needs a byte
// permute + FFMA per element and is bound by the integer ALU pipe).
// ---------------------------------------------------------------------------
__device__ __forceinline__ int dp4a_uu(uint32_t a, uint32_t b, int c) {
    int r; asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c)); return r;
}
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int r; asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c)); return r;
}
__device__ __forceinline__ int dp4a_su(uint32_t a, uint32_t b, int c) {
    int r; asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c)); return r;
}
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
    int r; asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c)); return r;
}
struct Acc3 { int a0 = 0, a1 = 0, a2 = 0; };
// unsigned codes (four per word) times the limbs of one step
__device__ __forceinline__ void dp3u(uint32_t q, const uint32_t* L, Acc3& a) {
    a.a0 = dp4a_uu(q, L[0], a.a0); a.a1 = dp4a_uu(q, L[1], a.a1); a.a2 = dp4a_us(q, L[2], a.a2);
}
// signed (int8) codes
__device__ __forceinline__ void dp3s(uint32_t q, const uint32_t* L, Acc3& a) {
    a.a0 = dp4a_su(q, L[0], a.a0); a.a1 = dp4a_su(q, L[1], a.a1); a.a2 = dp4a_ss(q, L[2], a.a2);
}
__device__ __forceinline__ float comb(const Acc3& a) {
    return fmaf(65536.f, (float)a.a2, fmaf(256.f, (float)a.a1, (float)a.a0));
}
__device__ __forceinline__ float2 h2f2(uint32_t dd) { return __half22float2(*reinterpret_cast<const __half2*>(&dd)); }

template <int DT> struct DecI { static constexpr bool ok = false; };

// Each INT decoder also names the contiguous x range of a (chunk, scale group):
// GL elements from grp_base(c, g); step t's four values sit at off(t, j) in it.
template <> struct DecI<GGC_Q4_K> {
    static constexpr bool ok = true;
    static constexpr int GL = 16;
    __device__ static int grp_base(int c, int g) { const int b = c >> 3, p = c & 7; return b * 256 + 64 * (p >> 1) + 32 * g + 16 * (p & 1); }
    __device__ static constexpr int off(int t, int j) { return 4 * (t >> 1) + j; }
    __device__ static float dot(const Dec<GGC_Q4_K>::Ch& ch, const uint32_t* L, const float* gs, const float* sx, int) {
        const uint32_t w[4] = {ch.q.x, ch.q.y, ch.q.z, ch.q.w};
        Acc3 A, B;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            dp3u(w[i] & 0x0F0F0F0Fu, L + 3 * (2 * i), A);
            dp3u((w[i] >> 4) & 0x0F0F0F0Fu, L + 3 * (2 * i + 1), B);
        }
        const float2 dm = h2f2(ch.dd);
        // value = (sc d) q - (mn dmin)  (quant.rs:275-279)
        float r = fmaf((float)(ch.sc & 0xFF) * dm.x, gs[0] * comb(A), -((float)(ch.mn & 0xFF) * dm.y) * sx[0]);
        return r + fmaf((float)(ch.sc >> 8) * dm.x, gs[1] * comb(B), -((float)(ch.mn >> 8) * dm.y) * sx[1]);
    }
};

template <> struct DecI<GGC_Q6_K> {
    static constexpr bool ok = true;
    static constexpr int GL = 16;
    __device__ static int grp_base(int c, int g) {
        const int b = c >> 3, p = c & 7, n = p >> 2, part = p & 3;
        return b * 256 + 128 * n + 16 * (part & 1) + (part < 2 ? 0 : 32) + 64 * g;
    }
    __device__ static constexpr int off(int t, int j) { return 4 * (t >> 1) + j; }
    __device__ static float dot(const Dec<GGC_Q6_K>::Ch& ch, const uint32_t* L, const float* gs, const float* sx, int c) {
        const uint32_t w[4] = {ch.q.x, ch.q.y, ch.q.z, ch.q.w};
        const uint32_t h[4] = {ch.qh.x, ch.qh.y, ch.qh.z, ch.qh.w};
        const int part = c & 3;
        Acc3 A, B;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            uint32_t hl, hh;
            if (part < 2) { hl = (h[i] << 4) & 0x30303030u; hh = h[i] & 0x30303030u; }
            else { hl = (h[i] << 2) & 0x30303030u; hh = (h[i] >> 2) & 0x30303030u; }
            dp3u((w[i] & 0x0F0F0F0Fu) | hl, L + 3 * (2 * i), A);
            dp3u(((w[i] >> 4) & 0x0F0F0F0Fu) | hh, L + 3 * (2 * i + 1), B);
        }
        const int ia = (part & 1) + (part < 2 ? 0 : 2), ib = ia + 4;
        const uint32_t wa = ia < 4 ? ch.sc.x : ch.sc.y, wb = ch.sc.y;
        const float sca = (float)(int8_t)((wa >> (8 * (ia & 3))) & 0xFF);
        const float scb = (float)(int8_t)((wb >> (8 * (ib & 3))) & 0xFF);
        const float d = h2f(ch.d);
        // value = (d sc) (u - 32)  (quant.rs:331-334)
        float r = (d * sca) * fmaf(-32.f, sx[0], gs[0] * comb(A));
        return r + (d * scb) * fmaf(-32.f, sx[1], gs[1] * comb(B));
    }
};

template <> struct DecI<GGC_Q4_0> {
    static constexpr bool ok = true;
    static constexpr int GL = 32;
    __device__ static int grp_base(int c, int) { return 32 * c; }
    __device__ static constexpr int off(int t, int j) { return 2 * (4 * (t >> 1) + j) + (t & 1); }
    __device__ static float dot(const Dec<GGC_Q4_0>::Ch& ch, const uint32_t* L, const float* gs, const float* sx, int) {
        const uint32_t w[4] = {ch.q.x, ch.q.y, ch.q.z, ch.q.w};
        Acc3 A;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            dp3u(w[i] & 0x0F0F0F0Fu, L + 3 * (2 * i), A);
            dp3u((w[i] >> 4) & 0x0F0F0F0Fu, L + 3 * (2 * i + 1), A);
        }
        // value = d (q - 8)  (quant.rs:132-133)
        return h2f(ch.d) * fmaf(-8.f, sx[0], gs[0] * comb(A));
    }
};

template <> struct DecI<GGC_Q8_0> {
    static constexpr bool ok = true;
    static constexpr int GL = 16;
    __device__ static int grp_base(int c, int) { return 16 * c; }
    __device__ static constexpr int off(int t, int j) { return 4 * t + j; }
    __device__ static float dot(const Dec<GGC_Q8_0>::Ch& ch, const uint32_t* L, const float* gs, const float*, int) {
        Acc3 A;
        dp3s(ch.q.x, L + 0, A);
        dp3s(ch.q.y, L + 3, A);
        dp3s(ch.q.z, L + 6, A);
        dp3s(ch.q.w, L + 9, A);
        return h2f(ch.d) * (gs[0] * comb(A));   // value = d q  (quant.rs:187)
    }
};

// ---------------------------------------------------------------------------
// GEMV launch description
// ---------------------------------------------------------------------------
enum ProKind : int { PRO_PLAIN = 0, PRO_RMSNORM = 1, PRO_SWIGLU = 2 };
enum EpiKind : int {
    EPI_STORE = 0,      // out[r] = acc (+ bias[r])
    EPI_ROPE_Q = 1,     // rows stored in RoPE-pair order; out[lr] = rope(acc + bias)
    EPI_ROPE_KC = 2,    // same, written into the K cache row of this step's slot
    EPI_VC = 3,         // out = acc + bias written into the V cache row
    EPI_RESID = 4,      // out[r] += acc, NaN -> error flag
    EPI_LOGITS = 5,     // out[r] = acc and greedy argmax into a 64-bit key
    EPI_SWIGLU = 6,     // rows (2i, 2i+1) = (ffn_up_i, ffn_gate_i): out[i] = silu(gate_i) * up_i
    EPI_AR = 7          // tensor parallel: partial rows to every rank, summed into out (allreduce.cuh)
};

// silu(g) * u as the reference computes it (ops.rs:237-247, llama.rs:564-567).
// Not inlined: one copy of its expf and two divisions serves every call site.
static __device__ __noinline__ float ffn_silu_mul(float g, float u) {
    float sig;
    if (g >= 0.0f) sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g)));
    else { const float ex = expf(g); sig = __fdiv_rn(ex, __fadd_rn(1.0f, ex)); }
    return __fmul_rn(__fmul_rn(g, sig), u);
}

struct Seg {
    QMat m;
    int epi;
    float* out;             // destination (EPI_STORE/EPI_ROPE_Q/EPI_RESID/EPI_LOGITS)
    void* cache;            // K or V cache of this layer (EPI_ROPE_KC / EPI_VC), [kv head][kv_ctx][hd]
    const float* bias;      // indexed by logical row; may be null
};

struct GemvArgs {
    Seg seg[3];
    int nseg;
    int pro;
    const float* x;         // PRO_PLAIN: x; PRO_RMSNORM: hidden; PRO_SWIGLU: gate
    const float* x2;        // PRO_RMSNORM: norm weight; PRO_SWIGLU: up
    uint32_t cols;          // padded row length of the weights (multiple of the chunk width)
    uint32_t xcols;         // logical length of x (elements >= xcols read as 0)
    const int* st_done;     // skip the launch when *st_done != 0 (may be null)
    const int* st_skip;     // skip when st_skip[0] < st_skip[1] (a prompt token that is not the last)
    const uint32_t* slot;   // cache slot of this step (EPI_ROPE_KC / EPI_VC)
    const int64_t* pos;     // position of this step (RoPE)
    const float2* rope;     // [max_ctx][hd/2] (cos, sin)
    uint32_t hd;
    uint32_t kv_ctx;        // cache rows per kv head (the cache is [kv head][kv_ctx][hd])
    int kv_f16;
    int* errf;
    int err_slot;           // error-flag slot for EPI_RESID NaN
    int err_val;            // value written (layer + 1); 0: no NaN guard in the epilogue
    int pro_err_slot;       // PRO_RMSNORM: flag slot for a NaN in x (tensor parallel: the
    int pro_err_val;        //   reduced hidden state), value written; 0: no check
    const ArGroup* ar;      // EPI_AR: the rank group (one segment only)
    uint32_t ar_k;          // EPI_AR: 1-based index of this all-reduce inside a step
    unsigned long long* argmax_key;
};

// Per-launch stage geometry (computed on the host).
struct TileCfg {
    uint32_t poff[4];        // offset of plane p inside a stage
    uint32_t stage_bytes;
    uint32_t stages;
    uint32_t x_bytes;        // shared bytes of the x region (128-aligned)
};

constexpr int GEMV_WARPS = 16;             // consumer warps: 4 column slices x 4 row groups
constexpr int GEMV_THREADS = GEMV_WARPS * 32 + 32;
constexpr int GEMV_NCS = 4;                // column slices of 32 chunks per tile
constexpr int GEMV_NRG = GEMV_WARPS / GEMV_NCS;
constexpr int GEMV_R = TILE_ROWS / GEMV_NRG;   // rows per warp per tile
constexpr int GEMV_MAX_STAGES = 4;
constexpr uint32_t GEMV_WAIT_LIMIT = BULK_WAIT_LIMIT;

__device__ __forceinline__ unsigned long long argmax_key_of(float v, uint32_t idx) {
    uint32_t b = __float_as_uint(v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);   // order-preserving map
    return ((unsigned long long)b << 32) | idx;         // ties: larger index wins (last maximum)
}

// Epilogue for `nvalid` (1 or 2) consecutive rows starting at r0 of segment `sg`.
__device__ __forceinline__ void gemv_epilogue(const GemvArgs& a, const Seg& sg, uint32_t r0, uint32_t nvalid,
                                              const float* acc) {
    switch (sg.epi) {
        case EPI_STORE:
            for (uint32_t r = 0; r < nvalid; ++r) sg.out[r0 + r] = sg.bias ? __fadd_rn(acc[r], sg.bias[r0 + r]) : acc[r];
            break;
        case EPI_AR:
            ar_store_rows(*a.ar, a.ar_k, sg.out, r0, nvalid, acc);
            break;
        case EPI_SWIGLU:   // r0 even, both rows valid (the fused matrix has 2 f rows)
            if (nvalid == 2) sg.out[r0 >> 1] = ffn_silu_mul(acc[1], acc[0]);
            break;
        case EPI_RESID: {
            bool nan = false;
            for (uint32_t r = 0; r < nvalid; ++r) {
                nan |= isnan(acc[r]);
                sg.out[r0 + r] = __fadd_rn(sg.out[r0 + r], acc[r]);
            }
            if (nan && a.err_val) atomicCAS(&a.errf[a.err_slot], 0, a.err_val);   // layers run in order: the first NaN layer stays
            break;
        }
        case EPI_LOGITS: {
            unsigned long long best = 0ull;
            bool nan = false;
            for (uint32_t r = 0; r < nvalid; ++r) {
                sg.out[r0 + r] = acc[r];
                nan |= isnan(acc[r]);
                const unsigned long long k = argmax_key_of(acc[r], r0 + r);
                best = k > best ? k : best;
            }
            if (nan) atomicMax(&a.errf[ERRF_NAN_LOGITS], 1);
            atomicMax(a.argmax_key, best);
            break;
        }
        case EPI_VC: {   // llama.rs:466-469 then cache.rs:46-54 (rows not permuted)
            const uint32_t slot = *a.slot;
            for (uint32_t r = 0; r < nvalid; ++r) {
                const uint32_t lr = r0 + r, head = lr / a.hd;
                const uint64_t idx = ((uint64_t)head * a.kv_ctx + slot) * a.hd + (lr - head * a.hd);
                const float v = sg.bias ? __fadd_rn(acc[r], sg.bias[lr]) : acc[r];
                if (a.kv_f16) reinterpret_cast<__half*>(sg.cache)[idx] = __float2half_rn(v);
                else reinterpret_cast<float*>(sg.cache)[idx] = v;
            }
            break;
        }
        default: {   // RoPE: rows (2m, 2m+1) = logical rows (h hd + j, h hd + j + hd/2)
            if (nvalid < 2) break;
            const uint32_t half = a.hd / 2;
            const int64_t pos = *a.pos;
            const uint32_t pm = r0 >> 1, head = pm / half, j = pm % half;
            const uint32_t l0 = head * a.hd + j, l1 = l0 + half;
            float v0 = acc[0], v1 = acc[1];
            if (sg.bias) { v0 = __fadd_rn(v0, sg.bias[l0]); v1 = __fadd_rn(v1, sg.bias[l1]); }
            // ops::rope (ops.rs:329-334): a cos - b sin, b cos + a sin
            const float2 cs = a.rope[(uint64_t)pos * half + j];
            const float n0 = __fsub_rn(__fmul_rn(v0, cs.x), __fmul_rn(v1, cs.y));
            const float n1 = __fadd_rn(__fmul_rn(v1, cs.x), __fmul_rn(v0, cs.y));
            if (sg.epi == EPI_ROPE_Q) {
                sg.out[l0] = n0; sg.out[l1] = n1;
            } else {
                const uint64_t base = ((uint64_t)head * a.kv_ctx + *a.slot) * a.hd;
                if (a.kv_f16) {
                    __half* c = reinterpret_cast<__half*>(sg.cache);
                    c[base + j] = __float2half_rn(n0); c[base + j + half] = __float2half_rn(n1);
                } else {
                    float* c = reinterpret_cast<float*>(sg.cache);
                    c[base + j] = n0; c[base + j + half] = n1;
                }
            }
            break;
        }
    }
}

// x[e] of the GEMV input: plain, ops::rmsnorm (ops.rs:262-274, with the CTA's
// f64 scale) or silu(gate)*up (ops.rs:237-247, llama.rs:564-567).
__device__ __forceinline__ float gemv_xval(const GemvArgs& a, uint32_t e, float scale) {
    if (e >= a.xcols) return 0.f;
    if (a.pro == PRO_RMSNORM) return __fmul_rn(__fmul_rn(a.x[e], scale), a.x2[e]);
    if (a.pro == PRO_SWIGLU) {
        const float g = a.x[e];
        float sig;
        if (g >= 0.0f) sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g)));
        else { const float ex = expf(g); sig = __fdiv_rn(ex, __fadd_rn(1.0f, ex)); }
        return __fmul_rn(__fmul_rn(g, sig), a.x2[e]);
    }
    return a.x[e];
}

// ---------------------------------------------------------------------------
// The kernel.  One CTA per SM.  A producer warp streams tiles (16 rows x one
// column tile, every plane) into a ring of shared-memory stages with one bulk
// copy per plane (tiles are contiguous in HBM), completion on an mbarrier; the
// first stages are issued before griddepcontrol.wait, so a GEMV streams its
// weights while its predecessor is still finishing.  16 consumer warps build x
// (overlapping the first copies), then compute x-stationary: warp (rg, cs) keeps
// x of its 32-chunk column slice in registers and walks rows rg, rg+4, ... of
// each tile; the column slices' partial row sums meet in shared memory in fixed
// order (deterministic), and the last warp to finish a row block runs its
// epilogue.  Every wait is bounded; on expiry ERRF_TIMEOUT is raised.
// ---------------------------------------------------------------------------
template <int DT>
__global__ void __launch_bounds__(GEMV_THREADS, 1) k_gemv(const GemvArgs a, const TileCfg tc) {
    using D = Dec<DT>;
    constexpr PlaneSpec PS = plane_spec(DT);
    constexpr int R = GEMV_R;
    constexpr bool INT = DecI<DT>::ok;
    constexpr int NG = D::G > 0 ? D::G : 1;
    constexpr int NSLOT = GEMV_MAX_STAGES + 1;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ Seg sseg[3];
    __shared__ double red[GEMV_WARPS];
    __shared__ float s_scale;
    __shared__ float part[NSLOT][GEMV_NCS][TILE_ROWS];
    __shared__ unsigned pcnt[NSLOT];

    const uint32_t nch = a.cols / D::E;
    float4* xs = reinterpret_cast<float4*>(smem);                                  // FP: [T][nch]
    float* sx = reinterpret_cast<float*>(smem + (size_t)D::T * nch * 16);           // FP: [nch][G]
    uint32_t* xl = reinterpret_cast<uint32_t*>(smem);                               // INT: [3T][nch] limbs
    float2* gsx = reinterpret_cast<float2*>(smem + (size_t)nch * 3 * D::T * 4);      // INT: [nch][NG] (gs, sum x)
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + tc.x_bytes);
    uint64_t* empty = full + GEMV_MAX_STAGES;
    uint8_t* stages = smem + tc.x_bytes + 128;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid < a.nseg) sseg[tid] = a.seg[tid];
    if (tid == 0) {
        for (uint32_t s = 0; s < tc.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], GEMV_WARPS);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    pdl_trigger();

    // balanced contiguous range of row blocks (over all segments) for this CTA
    const uint32_t nct = sseg[0].m.L.nct;
    uint32_t total_rb = 0;
    for (int i = 0; i < a.nseg; ++i) total_rb += sseg[i].m.L.nrb;
    const uint32_t rb0 = (uint32_t)((uint64_t)total_rb * blockIdx.x / gridDim.x);
    const uint32_t rb1 = (uint32_t)((uint64_t)total_rb * (blockIdx.x + 1) / gridDim.x);
    const uint32_t ntiles = (rb1 - rb0) * nct;
    // global row block -> (segment, local row block)
    auto locate = [&](uint32_t g, int& si, uint32_t& rb) {
        si = 0;
        rb = g;
        while (si + 1 < a.nseg && rb >= sseg[si].m.L.nrb) { rb -= sseg[si].m.L.nrb; ++si; }
    };

    if (warp == GEMV_WARPS) {
        // ---------------- producer warp ----------------
        const uint32_t prefetch = ntiles < tc.stages ? ntiles : tc.stages;
        bool waited = false;
        for (uint32_t i = 0; i < ntiles; ++i) {
            if (i == prefetch) {   // the first stages are in flight; now wait for the predecessor
                pdl_wait();
                waited = true;
                if ((a.st_done && *a.st_done) || (a.st_skip && a.st_skip[0] < a.st_skip[1])) break;
            }
            const uint32_t s = i % tc.stages;
            if (i >= tc.stages && !mbar_wait(&empty[s], ((i / tc.stages) - 1) & 1, a.errf)) break;
            if (lane == 0) {
                int si; uint32_t rb;
                locate(rb0 + i / nct, si, rb);
                const uint32_t ct = i % nct;
                const QMat& m = sseg[si].m;
                uint32_t bytes = 0;
#pragma unroll
                for (int p = 0; p < PS.n; ++p) bytes += TILE_ROWS * tile_pitch(m.L, p, ct);
                mbar_arrive_expect_tx(&full[s], bytes);
                uint8_t* st = stages + (size_t)s * tc.stage_bytes;
#pragma unroll
                for (int p = 0; p < PS.n; ++p)
                    bulk_g2s(st + tc.poff[p], m.p[p] + tile_offset(m.L, p, rb, ct), TILE_ROWS * tile_pitch(m.L, p, ct),
                             &full[s]);
            }
            __syncwarp();
        }
        if (!waited) pdl_wait();   // every kernel waits on its predecessor before it completes
        return;
    }

    // ---------------- consumer warps ----------------
    pdl_wait();
    if ((a.st_done && *a.st_done) || (a.st_skip && a.st_skip[0] < a.st_skip[1])) {
        // drain the copies the producer issued before it saw the flag, then leave
        const uint32_t n = ntiles < tc.stages ? ntiles : tc.stages;
        for (uint32_t i = 0; i < n; ++i) mbar_wait(&full[i], 0, a.errf);
        return;
    }
    const uint32_t ctid = tid, cthreads = GEMV_WARPS * 32;
    if (a.pro == PRO_RMSNORM) {
        double ss = 0.0;
        if ((a.xcols & 3) == 0) {
            const float4* x4 = reinterpret_cast<const float4*>(a.x);
            for (uint32_t i = ctid; i < a.xcols / 4; i += cthreads) {
                const float4 v = x4[i];
                ss += (double)v.x * (double)v.x + (double)v.y * (double)v.y + (double)v.z * (double)v.z +
                      (double)v.w * (double)v.w;
            }
        } else {
            for (uint32_t i = ctid; i < a.xcols; i += cthreads) { const double v = (double)a.x[i]; ss += v * v; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) red[warp] = ss;
        asm volatile("bar.sync 1, %0;" ::"r"(cthreads) : "memory");
        if (ctid == 0) {
            double t = 0.0;
            for (int w = 0; w < GEMV_WARPS; ++w) t += red[w];
            s_scale = (float)sqrt(1.0 / (t / (double)a.xcols + (double)1e-6f));
            if (a.pro_err_val && isnan(t)) atomicCAS(&a.errf[a.pro_err_slot], 0, a.pro_err_val);   // NaN in x <=> NaN sum
        }
        asm volatile("bar.sync 1, %0;" ::"r"(cthreads) : "memory");
    }
    const float scale = (a.pro == PRO_RMSNORM) ? s_scale : 0.f;
    if constexpr (INT) {
        // one thread per (chunk, scale group): its GL contiguous x values with float4
        // loads issued back to back -> power-of-two scale -> limbs
        using DI = DecI<DT>;
        constexpr int GL = DI::GL;
        for (uint32_t q = ctid; q < nch * NG; q += cthreads) {
            const uint32_t c = q / NG, g = q % NG;
            const int base = DI::grp_base((int)c, (int)g);
            float v[GL];
            {
                const float4* x4 = reinterpret_cast<const float4*>(a.x + base);
                float4 xa[GL / 4], xb[GL / 4];
#pragma unroll
                for (int k = 0; k < GL / 4; ++k) xa[k] = x4[k];
                if (a.pro != PRO_PLAIN) {
                    const float4* y4 = reinterpret_cast<const float4*>(a.x2 + base);
#pragma unroll
                    for (int k = 0; k < GL / 4; ++k) xb[k] = y4[k];
                }
#pragma unroll
                for (int k = 0; k < GL / 4; ++k) {
                    const float xx[4] = {xa[k].x, xa[k].y, xa[k].z, xa[k].w};
                    const float yy[4] = {xb[k].x, xb[k].y, xb[k].z, xb[k].w};
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        float r = xx[j];
                        if (a.pro == PRO_RMSNORM) {
                            r = __fmul_rn(__fmul_rn(xx[j], scale), yy[j]);   // ops.rs:272
                        } else if (a.pro == PRO_SWIGLU) {                 // ops.rs:237-247, llama.rs:564-567
                            const float gg = xx[j];
                            float sig;
                            if (gg >= 0.0f) sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gg)));
                            else { const float ex = expf(gg); sig = __fdiv_rn(ex, __fadd_rn(1.0f, ex)); }
                            r = __fmul_rn(__fmul_rn(gg, sig), yy[j]);
                        }
                        v[4 * k + j] = r;
                    }
                }
            }
            float mx = 0.f, sum = 0.f;
#pragma unroll
            for (int k = 0; k < GL; ++k) { mx = fmaxf(mx, fabsf(v[k])); sum += v[k]; }
            int ex = 0;
            frexpf(mx, &ex);
            const bool finite = isfinite(mx) && isfinite(sum);
            const float mul = (mx > 0.f && finite) ? ldexpf(1.f, 22 - ex) : 0.f;
            const float gs = !finite ? __int_as_float(0x7FC00000) : (mx > 0.f ? ldexpf(1.f, ex - 22) : 0.f);
#pragma unroll
            for (int t = 0; t < D::T; ++t) {
                if (NG > 1 && D::group(t) != (int)g) continue;
                uint32_t w0 = 0, w1 = 0, w2 = 0;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int xi = __float2int_rn(v[DI::off(t, j)] * mul);
                    w0 |= (uint32_t)(xi & 0xFF) << (8 * j);
                    w1 |= (uint32_t)((xi >> 8) & 0xFF) << (8 * j);
                    w2 |= (uint32_t)((xi >> 16) & 0xFF) << (8 * j);
                }
                xl[(3 * t + 0) * nch + c] = w0;
                xl[(3 * t + 1) * nch + c] = w1;
                xl[(3 * t + 2) * nch + c] = w2;
            }
            gsx[c * NG + g] = make_float2(gs, sum);
        }
    } else {
#pragma unroll 1
        for (int t = 0; t < D::T; ++t) {
            for (uint32_t c = ctid; c < nch; c += cthreads) {
                float v[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) v[j] = gemv_xval(a, (uint32_t)D::elem((int)c, t, j), scale);
                xs[t * nch + c] = make_float4(v[0], v[1], v[2], v[3]);
            }
        }
        asm volatile("bar.sync 1, %0;" ::"r"(cthreads) : "memory");
        if constexpr (D::G > 0) {
            for (uint32_t q = ctid; q < nch * D::G; q += cthreads) {
                const uint32_t c = q / D::G, g = q % D::G;
                float acc = 0.f;
                for (int t = 0; t < D::T; ++t)
                    if (D::group(t) == (int)g) {
                        const float4 v = xs[t * nch + c];
                        acc += (v.x + v.y) + (v.z + v.w);
                    }
                sx[q] = acc;
            }
        }
    }
    for (uint32_t q = ctid; q < NSLOT * GEMV_NCS * TILE_ROWS; q += cthreads) (&part[0][0][0])[q] = 0.f;
    if (ctid < NSLOT) pcnt[ctid] = 0;
    asm volatile("bar.sync 1, %0;" ::"r"(cthreads) : "memory");

    const int cs = warp % GEMV_NCS, rg = warp / GEMV_NCS;
    float4 xr[INT ? 1 : D::T];
    float sxr[NG];
    uint32_t Lr[INT ? 3 * D::T : 1];
    float gsr[NG];
    uint32_t cur_ct = 0xFFFFFFFFu;
    for (uint32_t i = 0; i < ntiles; ++i) {
        const uint32_t s = i % tc.stages;
        if (!mbar_wait(&full[s], (i / tc.stages) & 1, a.errf)) return;
        int si; uint32_t rb;
        locate(rb0 + i / nct, si, rb);
        const uint32_t ct = i % nct;
        const TileLayout& L = sseg[si].m.L;
        const uint32_t tcols = ct + 1 == L.nct ? L.pcols - ct * L.kc : L.kc;
        const uint32_t nrows = min((uint32_t)TILE_ROWS, L.rows - rb * TILE_ROWS);
        const int nchk = (int)(tcols / D::E), cg0 = (int)(ct * L.kc / D::E);
        const int c = cs * 32 + lane;   // chunk of this lane inside the tile
        const bool valid = c < nchk;
        if (ct != cur_ct) {   // x of this lane's column slice into registers
            cur_ct = ct;
            if (valid) {
                if constexpr (INT) {
#pragma unroll
                    for (int q = 0; q < 3 * D::T; ++q) Lr[q] = xl[q * nch + cg0 + c];
#pragma unroll
                    for (int g = 0; g < NG; ++g) { const float2 v2 = gsx[(cg0 + c) * NG + g]; gsr[g] = v2.x; sxr[g] = v2.y; }
                } else {
#pragma unroll
                    for (int q = 0; q < D::T; ++q) xr[q] = xs[q * nch + cg0 + c];
#pragma unroll
                    for (int g = 0; g < NG; ++g) sxr[g] = D::G > 0 ? sx[(cg0 + c) * D::G + g] : 0.f;
                }
            }
        }
        const uint8_t* st = stages + (size_t)s * tc.stage_bytes;
        TileView v;
#pragma unroll
        for (int p = 0; p < 4; ++p) { v.p[p] = st + tc.poff[p]; v.pitch[p] = tile_pitch(L, p, ct); }
        // the R rows are computed branch-free (clamped row / chunk, masked result) so
        // their dependent integer chains interleave
        float accr[R];
        {
            const uint32_t cc = (uint32_t)(valid ? c : 0);
            typename D::Ch ch[R];
#pragma unroll
            for (int k = 0; k < R; ++k) ch[k] = D::load(v, min((uint32_t)(rg + GEMV_NRG * k), nrows - 1), cc);
#pragma unroll
            for (int k = 0; k < R; ++k) {
                float d;
                if constexpr (INT) d = DecI<DT>::dot(ch[k], Lr, gsr, sxr, (int)cc);
                else d = chunk_dot<DT>(ch[k], xr, 1, sxr, (int)cc);
                accr[k] = (valid && (uint32_t)(rg + GEMV_NRG * k) < nrows) ? d : 0.f;
            }
        }
#pragma unroll
        for (int k = 0; k < R; ++k) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) accr[k] += __shfl_xor_sync(0xffffffffu, accr[k], o);
        }
        // partial sums per row block live in NSLOT rotating slots: a warp runs at most
        // `stages` tiles ahead of the slowest one, so a slot is never reused too early
        const uint32_t slot = (i / nct) % NSLOT;
        if (lane == 0) {
#pragma unroll
            for (int k = 0; k < R; ++k) part[slot][cs][rg + GEMV_NRG * k] += accr[k];
        }
        bool last_warp = false;
        if (ct + 1 == nct) {   // this warp finished the row block
            unsigned prev = 0;
            if (lane == 0) {
                __threadfence_block();
                prev = atomicAdd(&pcnt[slot], 1u);
            }
            last_warp = __shfl_sync(0xffffffffu, prev, 0) == (unsigned)(GEMV_WARPS - 1);
        }
        if (last_warp) {
            __threadfence_block();
            if (lane < TILE_ROWS / 2) {
                const uint32_t lr = 2 * lane;
                if (lr < nrows) {
                    float y[2];
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        float sum = 0.f;
#pragma unroll
                        for (int k = 0; k < GEMV_NCS; ++k) sum += part[slot][k][lr + q];
                        y[q] = sum;
                    }
                    gemv_epilogue(a, sseg[si], rb * TILE_ROWS + lr, min(2u, nrows - lr), y);
                }
            }
            __syncwarp();
            for (int q = lane; q < GEMV_NCS * TILE_ROWS; q += 32) (&part[slot][0][0])[q] = 0.f;
            if (lane == 0) pcnt[slot] = 0;
            __threadfence_block();
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (a.ar_k)   // tensor parallel: row `warp` of each of the CTA's row blocks, summed over the ranks
        ar_reduce_rows(
            a.ar, a.ar_k, rb1 - rb0, [&](uint32_t j) { return (rb0 + j) * TILE_ROWS + (uint32_t)warp; },
            sseg[0].m.L.rows, sseg[0].out, a.errf, a.err_slot, a.err_val);
}

// Host: stage layout of a launch over weights of `pcols` columns.
template <int DT>
TileCfg make_tile_cfg(uint32_t pcols, size_t smem_limit) {
    using D = Dec<DT>;
    constexpr PlaneSpec PS = plane_spec(DT);
    const TileLayout L = make_layout(DT, TILE_ROWS, pcols);
    const uint32_t nch = pcols / D::E;
    TileCfg tc{};
    const size_t xb = DecI<DT>::ok ? (size_t)nch * 3 * D::T * 4 + (size_t)nch * (D::G > 0 ? D::G : 1) * 8
                                   : (size_t)nch * D::T * 16 + (size_t)nch * (D::G > 0 ? D::G : 1) * 4;
    tc.x_bytes = (uint32_t)((xb + 127) / 128 * 128);
    uint32_t off = 0;
    for (int p = 0; p < 4; ++p) {
        tc.poff[p] = off;
        off += p < PS.n ? (TILE_ROWS * L.tp_full[p] + 127u) / 128u * 128u : 0u;
    }
    tc.stage_bytes = off;
    const size_t fixed = tc.x_bytes + 128;
    const size_t st = smem_limit > fixed ? (smem_limit - fixed) / tc.stage_bytes : 0;
    tc.stages = (uint32_t)(st > (size_t)GEMV_MAX_STAGES ? GEMV_MAX_STAGES : st);
    return tc;
}

inline size_t gemv_smem_bytes(const TileCfg& tc) { return (size_t)tc.x_bytes + 128 + (size_t)tc.stages * tc.stage_bytes; }

}  // namespace ggc
