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

namespace ggc {

// ---------------------------------------------------------------------------
// loads
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint4 ld_stream_v4(const uint8_t* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ uint4 ld_v4(const uint8_t* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
__device__ __forceinline__ uint2 ld_v2(const uint8_t* p) { return __ldg(reinterpret_cast<const uint2*>(p)); }
__device__ __forceinline__ uint32_t ld_u32(const uint8_t* p) { return __ldg(reinterpret_cast<const uint32_t*>(p)); }
__device__ __forceinline__ uint32_t ld_u16g(const uint8_t* p) { return __ldg(reinterpret_cast<const unsigned short*>(p)); }
__device__ __forceinline__ uint32_t ld_u8g(const uint8_t* p) { return __ldg(p); }

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
    __device__ static Ch load(const QMat& m, uint32_t r, uint32_t c) {
        return Ch{ld_stream_v4(m.p[0] + (uint64_t)r * m.pitch[0] + c * 16u), ld_u16g(m.p[1] + (uint64_t)r * m.pitch[1] + c * 2u)};
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
    __device__ static Ch load(const QMat& m, uint32_t r, uint32_t c) {
        return Ch{ld_stream_v4(m.p[0] + (uint64_t)r * m.pitch[0] + c * 16u), ld_u32(m.p[1] + (uint64_t)r * m.pitch[1] + c * 4u)};
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
    __device__ static Ch load(const QMat& m, uint32_t r, uint32_t c) {
        Ch ch;
        ch.q = ld_stream_v4(m.p[0] + (uint64_t)r * m.pitch[0] + c * 16u);
        ch.qh = ld_u32(m.p[1] + (uint64_t)r * m.pitch[1] + c * 4u);
        ch.d = HAS_M ? ld_u32(m.p[2] + (uint64_t)r * m.pitch[2] + c * 4u) : ld_u16g(m.p[2] + (uint64_t)r * m.pitch[2] + c * 2u);
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
    __device__ static Ch load(const QMat& m, uint32_t r, uint32_t c) {
        return Ch{ld_stream_v4(m.p[0] + (uint64_t)r * m.pitch[0] + c * 16u), ld_u16g(m.p[1] + (uint64_t)r * m.pitch[1] + (c >> 1) * 2u)};
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
    __device__ static Ch load(const QMat& m, uint32_t r, uint32_t c) {
        return Ch{ld_stream_v4(m.p[0] + (uint64_t)r * m.pitch[0] + c * 16u), ld_u32(m.p[1] + (uint64_t)r * m.pitch[1] + (c >> 4) * 4u)};
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
    __device__ static Ch load(const QMat& m, uint32_t r, uint32_t c) {
        const uint32_t b = c >> 2, p = c & 3;
        Ch ch;
        ch.q = ld_stream_v4(m.p[0] + (uint64_t)r * m.pitch[0] + c * 16u);
        ch.sc = ld_u16g(m.p[1] + (uint64_t)r * m.pitch[1] + b * 16u + 14u - 2u * p);   // bytes 14-2p, 15-2p
        ch.dd = ld_u32(m.p[2] + (uint64_t)r * m.pitch[2] + b * 4u);
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
    __device__ static Ch load(const QMat& m, uint32_t r, uint32_t c) {
        const uint32_t b = c >> 2, p = c & 3;
        Ch ch;
        ch.q = ld_stream_v4(m.p[0] + (uint64_t)r * m.pitch[0] + c * 16u);
        ch.hm = ld_v2(m.p[1] + (uint64_t)r * m.pitch[1] + c * 8u);
        const uint8_t* sb = m.p[2] + (uint64_t)r * m.pitch[2] + b * 12u;
        ch.lo = ld_u16g(sb + 2u * p);
        ch.hi = ld_u8g(sb + 8u + p);
        ch.d = ld_u16g(m.p[3] + (uint64_t)r * m.pitch[3] + b * 2u);
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
    struct Ch { uint4 q; uint4 meta; };
    // chunk c: block c/8, part p = c%8 -> qs bytes 32g + l0 .. +15 (g = p/2, l0 = 16(p%2)):
    // low nibbles are elements 64g + l0 + i (sub-block 2g), high nibbles 64g + 32 + l0 + i (2g+1)
    __device__ static int elem(int c, int t, int j) {
        const int b = c >> 3, p = c & 7;
        return b * 256 + 64 * (p >> 1) + 32 * (t & 1) + 16 * (p & 1) + 4 * (t >> 1) + j;
    }
    __device__ static int group(int t) { return t & 1; }
    __device__ static Ch load(const QMat& m, uint32_t r, uint32_t c) {
        return Ch{ld_stream_v4(m.p[0] + (uint64_t)r * m.pitch[0] + c * 16u), ld_v4(m.p[1] + (uint64_t)r * m.pitch[1] + (c >> 3) * 16u)};
    }
    __device__ static float dot(const Ch& ch, const float4* xs, int n, const float* sx, int c) {
        const uint32_t w[4] = {ch.q.x, ch.q.y, ch.q.z, ch.q.w};
        float SA = 0.f, SB = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) { SA = fma_b4(nib_lo(w[i]), xs[(2 * i) * n], SA); SB = fma_b4(nib_hi(w[i]), xs[(2 * i + 1) * n], SB); }
        const float d = h2f(ch.meta.x & 0xFFFF), dmin = h2f(ch.meta.x >> 16);
        const int g = (c & 7) >> 1;
        float scA, mnA, scB, mnB;
        kq_scale_min(ch.meta.y, ch.meta.z, ch.meta.w, 2 * g, scA, mnA);
        kq_scale_min(ch.meta.y, ch.meta.z, ch.meta.w, 2 * g + 1, scB, mnB);
        // value = (sc d) q - (mn dmin)  (quant.rs:275-279)
        float r = fmaf((scA * d) * 128.f, SA - sx[0], -(mnA * dmin) * sx[0]);
        return r + fmaf((scB * d) * 128.f, SB - sx[1], -(mnB * dmin) * sx[1]);
    }
};

template <> struct Dec<GGC_Q5_K> {
    static constexpr int E = 32, T = 8, G = 1;
    struct Ch { uint4 q; uint32_t qh; uint4 meta; };
    // chunk c: block c/8, sub-block p = c%8; qs byte i of the chunk holds elements 32p + 2i (low) and +1 (high)
    __device__ static int elem(int c, int t, int j) {
        const int b = c >> 3, p = c & 7;
        return b * 256 + 32 * p + 2 * (4 * (t >> 1) + j) + (t & 1);
    }
    __device__ static int group(int) { return 0; }
    __device__ static Ch load(const QMat& m, uint32_t r, uint32_t c) {
        const uint32_t b = c >> 3, p = c & 7;
        Ch ch;
        ch.q = ld_stream_v4(m.p[0] + (uint64_t)r * m.pitch[0] + c * 16u);
        ch.qh = ld_u32(m.p[1] + (uint64_t)r * m.pitch[1] + b * 16u + (p >> 1) * 4u);
        ch.meta = ld_v4(m.p[2] + (uint64_t)r * m.pitch[2] + b * 16u);
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
        const float d = h2f(ch.meta.x & 0xFFFF), dmin = h2f(ch.meta.x >> 16);
        float sc, mn;
        kq_scale_min(ch.meta.y, ch.meta.z, ch.meta.w, p, sc, mn);
        return fmaf((sc * d) * 128.f, S - sx[0], -(mn * dmin) * sx[0]);
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
    __device__ static Ch load(const QMat& m, uint32_t r, uint32_t c) {
        const uint32_t b = c >> 3, p = c & 7, n = p >> 2, part = p & 3;
        Ch ch;
        ch.q = ld_stream_v4(m.p[0] + (uint64_t)r * m.pitch[0] + c * 16u);
        ch.qh = ld_v4(m.p[1] + (uint64_t)r * m.pitch[1] + b * 64u + n * 32u + 16u * (part & 1));
        ch.sc = ld_v2(m.p[2] + (uint64_t)r * m.pitch[2] + b * 16u + n * 8u);
        ch.d = ld_u16g(m.p[3] + (uint64_t)r * m.pitch[3] + b * 2u);
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
    __device__ static Ch load(const QMat& m, uint32_t r, uint32_t c) { return Ch{ld_stream_v4(m.p[0] + (uint64_t)r * m.pitch[0] + c * 16u)}; }
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
    __device__ static Ch load(const QMat& m, uint32_t r, uint32_t c) { return Ch{ld_stream_v4(m.p[0] + (uint64_t)r * m.pitch[0] + c * 16u)}; }
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
    __device__ static Ch load(const QMat& m, uint32_t r, uint32_t c) { return Ch{ld_stream_v4(m.p[0] + (uint64_t)r * m.pitch[0] + c * 16u)}; }
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
// GEMV launch description
// ---------------------------------------------------------------------------
enum ProKind : int { PRO_PLAIN = 0, PRO_RMSNORM = 1, PRO_SWIGLU = 2 };
enum EpiKind : int {
    EPI_STORE = 0,      // out[r] = acc (+ bias[r])
    EPI_ROPE_Q = 1,     // rows permuted into RoPE pairs; out[lr] = rope(acc + bias)
    EPI_ROPE_KC = 2,    // same, written into the K cache row of this step's slot
    EPI_VC = 3,         // out = acc + bias written into the V cache row
    EPI_RESID = 4,      // out[r] += acc, NaN -> error flag
    EPI_LOGITS = 5      // out[r] = acc and greedy argmax into a 64-bit key
};

struct StepState;   // model.cu

struct Seg {
    QMat m;
    int epi;
    float* out;             // destination (EPI_STORE/EPI_ROPE_Q/EPI_RESID/EPI_LOGITS)
    void* cache;            // K or V cache of this layer (EPI_ROPE_KC / EPI_VC), [slot][rows]
    const float* bias;      // indexed by logical row; may be null
    uint32_t groups;        // row groups of this segment
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
    const int* st_skip;     // skip when st_skip[0] < st_skip[1] (prompt token that is not the last)
    const uint32_t* slot;   // cache slot of this step (EPI_ROPE_KC / EPI_VC)
    const int64_t* pos;     // position of this step (RoPE)
    const float2* rope;     // [max_ctx][hd/2] (cos, sin)
    uint32_t hd;
    int kv_f16;
    int* errf;
    int err_slot;           // error-flag slot for EPI_RESID NaN
    int err_val;            // value written (layer + 1)
    unsigned long long* argmax_key;
};

constexpr int GEMV_R = 4;          // rows per warp
constexpr int GEMV_WARPS = 8;      // warps per CTA

__device__ __forceinline__ unsigned long long argmax_key_of(float v, uint32_t idx) {
    uint32_t b = __float_as_uint(v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);   // order-preserving map
    return ((unsigned long long)b << 32) | idx;         // ties: larger index wins (last maximum)
}

template <int DT>
__global__ void __launch_bounds__(GEMV_WARPS * 32, 2) k_gemv(const GemvArgs a) {
    using D = Dec<DT>;
    constexpr int R = GEMV_R;
    extern __shared__ float4 smem4[];
    pdl_trigger();
    pdl_wait();
    if (a.st_done && *a.st_done) return;
    if (a.st_skip && a.st_skip[0] < a.st_skip[1]) return;

    const uint32_t cols = a.cols;
    const int nch = (int)(cols / D::E);
    float4* xs = smem4;                                       // [T][nch] float4
    float* sx = reinterpret_cast<float*>(smem4 + (size_t)D::T * nch);   // [nch][G]
    __shared__ double red[GEMV_WARPS];
    __shared__ float s_scale;

    // ---- prologue: x in chunk order -------------------------------------
    const int tid = threadIdx.x, nthr = blockDim.x;
    if (a.pro == PRO_RMSNORM) {
        // ops::rmsnorm (ops.rs:262-274): f64 sum of squares, scale = sqrt(1/(ss/n + eps)) as f32
        double ss = 0.0;
        for (uint32_t i = tid; i < a.xcols; i += nthr) { double v = (double)a.x[i]; ss += v * v; }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if ((tid & 31) == 0) red[tid >> 5] = ss;
        __syncthreads();
        if (tid == 0) {
            double t = 0.0;
            for (int w = 0; w < (nthr >> 5); ++w) t += red[w];
            s_scale = (float)sqrt(1.0 / (t / (double)a.xcols + (double)1e-6f));
        }
        __syncthreads();
    }
    const float scale = (a.pro == PRO_RMSNORM) ? s_scale : 0.f;
#pragma unroll 1
    for (int t = 0; t < D::T; ++t) {
        for (int c = tid; c < nch; c += nthr) {
            float v[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int e = D::elem(c, t, j);
                if ((uint32_t)e >= a.xcols) {
                    v[j] = 0.f;
                } else if (a.pro == PRO_RMSNORM) {
                    v[j] = __fmul_rn(__fmul_rn(a.x[e], scale), a.x2[e]);
                } else if (a.pro == PRO_SWIGLU) {
                    // ops::silu (ops.rs:237-247) then gate *= up (llama.rs:564-567)
                    const float g = a.x[e];
                    float sig;
                    if (g >= 0.0f) sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g)));
                    else { const float ex = expf(g); sig = __fdiv_rn(ex, __fadd_rn(1.0f, ex)); }
                    v[j] = __fmul_rn(__fmul_rn(g, sig), a.x2[e]);
                } else {
                    v[j] = a.x[e];
                }
            }
            xs[t * nch + c] = make_float4(v[0], v[1], v[2], v[3]);
        }
    }
    __syncthreads();
    if constexpr (D::G > 0) {
        for (int q = tid; q < nch * D::G; q += nthr) {
            const int c = q / D::G, g = q % D::G;
            float acc = 0.f;
            for (int t = 0; t < D::T; ++t)
                if (D::group(t) == g) {
                    const float4 v = xs[t * nch + c];
                    acc += (v.x + v.y) + (v.z + v.w);
                }
            sx[q] = acc;
        }
        __syncthreads();
    }

    // ---- main loop over row groups ----------------------------------------
    const int lane = tid & 31;
    const uint32_t total_groups = a.seg[0].groups + (a.nseg > 1 ? a.seg[1].groups : 0) + (a.nseg > 2 ? a.seg[2].groups : 0);
    // balanced contiguous ranges of row groups per warp (they differ by at most one group)
    const uint32_t gwarps = gridDim.x * GEMV_WARPS, wid = blockIdx.x * GEMV_WARPS + (tid >> 5);
    const uint32_t g_begin = (uint32_t)((uint64_t)total_groups * wid / gwarps);
    const uint32_t g_end = (uint32_t)((uint64_t)total_groups * (wid + 1) / gwarps);
    for (uint32_t g = g_begin; g < g_end; ++g) {
        int si = 0;
        uint32_t lg = g;
        while (si + 1 < a.nseg && lg >= a.seg[si].groups) { lg -= a.seg[si].groups; ++si; }
        const Seg& sg = si == 0 ? a.seg[0] : (si == 1 ? a.seg[1] : a.seg[2]);
        const QMat& m = sg.m;
        const uint32_t r0 = lg * R;
        uint32_t rr[R];
#pragma unroll
        for (int r = 0; r < R; ++r) rr[r] = min(r0 + r, m.rows - 1);
        float acc[R];
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r] = 0.f;
        constexpr int U = 2;
        for (int c0 = lane; c0 < nch; c0 += 32 * U) {
            typename D::Ch ch[U][R];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int c = c0 + 32 * u;
                if (c < nch) {
#pragma unroll
                    for (int r = 0; r < R; ++r) ch[u][r] = D::load(m, rr[r], (uint32_t)c);
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int c = c0 + 32 * u;
                if (c < nch) {
                    const float* sxc = sx + (D::G > 0 ? c * D::G : 0);
#pragma unroll
                    for (int r = 0; r < R; ++r) acc[r] += chunk_dot<DT>(ch[u][r], xs + c, nch, sxc, c);
                }
            }
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
        }
        if (lane != 0) continue;
        // ---- epilogue (lane 0) ----
        const uint32_t nvalid = min((uint32_t)R, m.rows - r0);
        switch (sg.epi) {
            case EPI_STORE:
                for (uint32_t r = 0; r < nvalid; ++r) sg.out[r0 + r] = sg.bias ? __fadd_rn(acc[r], sg.bias[r0 + r]) : acc[r];
                break;
            case EPI_RESID: {
                bool nan = false;
                for (uint32_t r = 0; r < nvalid; ++r) {
                    nan |= isnan(acc[r]);
                    sg.out[r0 + r] = __fadd_rn(sg.out[r0 + r], acc[r]);
                }
                if (nan) atomicMax(&a.errf[a.err_slot], a.err_val);
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
                const uint64_t base = (uint64_t)(*a.slot) * m.rows;
                for (uint32_t r = 0; r < nvalid; ++r) {
                    const float v = sg.bias ? __fadd_rn(acc[r], sg.bias[r0 + r]) : acc[r];
                    if (a.kv_f16) reinterpret_cast<__half*>(sg.cache)[base + r0 + r] = __float2half_rn(v);
                    else reinterpret_cast<float*>(sg.cache)[base + r0 + r] = v;
                }
                break;
            }
            default: {   // RoPE: physical rows (2m, 2m+1) = logical rows (h hd + j, h hd + j + hd/2)
                const uint32_t half = a.hd / 2;
                const int64_t pos = *a.pos;
                for (uint32_t r = 0; r + 1 < nvalid; r += 2) {
                    const uint32_t pm = (r0 + r) >> 1, head = pm / half, j = pm % half;
                    const uint32_t l0 = head * a.hd + j, l1 = l0 + half;
                    float v0 = acc[r], v1 = acc[r + 1];
                    if (sg.bias) { v0 = __fadd_rn(v0, sg.bias[l0]); v1 = __fadd_rn(v1, sg.bias[l1]); }
                    // ops::rope (ops.rs:329-334): a cos - b sin, b cos + a sin
                    const float2 cs = a.rope[(uint64_t)pos * half + j];
                    const float n0 = __fsub_rn(__fmul_rn(v0, cs.x), __fmul_rn(v1, cs.y));
                    const float n1 = __fadd_rn(__fmul_rn(v1, cs.x), __fmul_rn(v0, cs.y));
                    if (sg.epi == EPI_ROPE_Q) {
                        sg.out[l0] = n0; sg.out[l1] = n1;
                    } else {
                        const uint64_t base = (uint64_t)(*a.slot) * m.rows;
                        if (a.kv_f16) {
                            __half* c = reinterpret_cast<__half*>(sg.cache);
                            c[base + l0] = __float2half_rn(n0); c[base + l1] = __float2half_rn(n1);
                        } else {
                            float* c = reinterpret_cast<float*>(sg.cache);
                            c[base + l0] = n0; c[base + l1] = n1;
                        }
                    }
                }
                break;
            }
        }
    }
}

// shared-memory bytes of one k_gemv launch
template <int DT>
size_t gemv_smem_bytes(uint32_t cols) {
    using D = Dec<DT>;
    size_t nch = cols / D::E;
    return nch * D::T * sizeof(float4) + nch * (D::G > 0 ? D::G : 1) * sizeof(float);
}

}  // namespace ggc
