// gemv_span.cuh -- decode GEMV y = W x for the block formats (Q4_0, Q4_1, Q5_0,
// Q5_1, Q8_0, Q2_K, Q3_K_*, Q4_K, Q5_K, Q6_K, Q8_K) over the span layout
// (planes.cuh).
//
// Work split.  One CTA per SM over a contiguous range of 16-row blocks; a
// producer warp streams tiles (16 rows x 4096 columns, every plane: one bulk copy
// per plane) into a ring of shared-memory stages, column tile by column tile.  8
// consumer warps each own an adjacent row pair of every tile (RoPE pairs stay in
// one warp); lane l owns the 128-element span l of the column tile, so a row is
// one pass of 32 lanes over their spans and one warp reduction.
//
// x arithmetic.  Before the first tile the CTA turns x (plain, RMS-normalised or
// silu(gate) * up) into, per span, a 22-bit fixed-point integer with one
// power-of-two scale gs (|x| / gs < 2^22: exact scaling), split into three 8-bit
// limbs (two unsigned, the top one signed), stored per (column tile, word, lane)
// in shared memory.  A lane loads the 96 limb words of its span into registers
// once per column tile.  One dp4a multiplies four weight codes by four limbs in
// int32; per-sub-block scales (6-bit / int8) fold into the int32 limb sums; the
// three limb sums recombine in f32 once per row and lane.  High nibbles are used
// as 16 * q (mask, no shift), the factor 16 folded into the scale.  The relative
// error of a row is ~2^-22 * max|x| / rms|x| (f32 reference: ~1e-6).
//
// Every wait is bounded (ERRF_TIMEOUT); the first stages are issued before
// griddepcontrol.wait, so the weights stream while the predecessor finishes.
#pragma once
#include "common.cuh"
#include "planes.cuh"
#include "mbarrier.cuh"
#include "gemv.cuh"

namespace ggc {

constexpr int GS_WARPS = 8;
constexpr int GS_THREADS = GS_WARPS * 32 + 32;
constexpr int GS_MAX_STAGES = 4;
constexpr int GS_WORDS = 96;    // limb words per span: 32 steps x 3 limbs
constexpr int GS_XF = 13;       // floats per span and column tile: gs, then 3 float4 of x sums (see xq_load)

// ---- per-format span decoders --------------------------------------------
// step s (0..31) of a span multiplies four weight codes by x elements
// elem(s, 0..3) of the span; quarter q (0..7) holds the steps of span elements
// [16q, 16q + 16): step_of(q, t), t = 0..3, whose element j is 16q + qoff(t, j).
template <int DT> struct SpanFmt;

__device__ __forceinline__ uint4 lds128(const uint8_t* p) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(smem_addr(p)));
    return v;
}
__device__ __forceinline__ uint2 lds64(const uint8_t* p) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(smem_addr(p)));
    return v;
}
__device__ __forceinline__ uint32_t lds32(const uint8_t* p) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(smem_addr(p)));
    return v;
}
__device__ __forceinline__ uint32_t lds16(const uint8_t* p) {
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(smem_addr(p)));
    return v;
}
// x sums of a lane's span (shared memory, [k][lane] float4): k = 0, 1: the sums over
// its eight 16-element quarters, k = 2: the sums over its four 32-element halves
__device__ __forceinline__ float4 xq_load(const float* xq, int k) {
    const uint4 v = lds128(reinterpret_cast<const uint8_t*>(xq + 128 * k));
    return make_float4(__uint_as_float(v.x), __uint_as_float(v.y), __uint_as_float(v.z), __uint_as_float(v.w));
}
__device__ __forceinline__ float f4sel(const float4& v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }
__device__ __forceinline__ uint32_t wsel(const uint4& u, int i) { return i == 0 ? u.x : i == 1 ? u.y : i == 2 ? u.z : u.w; }
__device__ __forceinline__ float comb3(int t0, int t1, int t2) {
    return fmaf(65536.f, (float)t2, fmaf(256.f, (float)t1, (float)t0));
}

// Plane rows of one tile row (shared memory) and the lane count of the tile.
struct SpanRow {
    const uint8_t* p[4];
    int nl;
};

// Q4_K: span = half n of a block; qs unit k = bytes 64n + 16k .. +16; byte i of
// a 32-byte segment j: low nibble -> element 64j + i (sub-block 2j), high ->
// 64j + 32 + i (quant.rs:262-283).  Local sub-blocks 0..3 of the span.
template <> struct SpanFmt<GGC_Q4_K> {
    __device__ static constexpr int elem(int s, int j) {
        const int w = s >> 1, hi = s & 1, k = w >> 2, i = w & 3;
        return 64 * (k >> 1) + 32 * hi + 16 * (k & 1) + 4 * i + j;
    }
    __device__ static constexpr int step_of(int q, int t) {   // quarter q: sub-block q/2, half q%2
        const int g = q >> 1, k = 2 * (g >> 1) + (q & 1), hi = g & 1;
        return 2 * (4 * k + t) + hi;
    }
    __device__ static constexpr int qoff(int t, int j) { return 4 * t + j; }   // elem(step_of(q, t), j) - 16 q
    __device__ static float dot(const SpanRow& R, int lane, const uint32_t* L, float gs, const float* xq) {
        uint4 u[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) u[k] = lds128(R.p[0] + (k * R.nl + lane) * 16);
        const uint32_t dd = lds32(R.p[1] + (lane >> 1) * 4);
        const uint2 scm = lds64(R.p[2] + lane * 8);
        Acc3 A[4];
#pragma unroll
        for (int w = 0; w < 16; ++w) {
            const uint32_t q = wsel(u[w >> 2], w & 3);
            const int sb = 2 * ((w >> 2) >> 1);
            dp3u(q & 0x0F0F0F0Fu, L + 6 * w, A[sb]);
            dp3u(q & 0xF0F0F0F0u, L + 6 * w + 3, A[sb + 1]);   // 16 q
        }
        // 16 * sum_q sc_q (codes . x_int): low sub-blocks take 16 sc, high ones sc
        int T0 = 0, T1 = 0, T2 = 0;
#pragma unroll
        for (int sb = 0; sb < 4; ++sb) {
            const int c = (int)((scm.x >> (8 * sb)) & 0xFFu) << ((sb & 1) ? 0 : 4);
            T0 += c * A[sb].a0; T1 += c * A[sb].a1; T2 += c * A[sb].a2;
        }
        const float4 xs = xq_load(xq, 2);
        float mn = 0.f;
#pragma unroll
        for (int sb = 0; sb < 4; ++sb) mn = fmaf((float)((scm.y >> (8 * sb)) & 0xFFu), f4sel(xs, sb), mn);
        const float2 dm = h2f2(dd);
        // value = d sc q - dmin mn  (quant.rs:275-279)
        return fmaf(dm.x * (gs * 0.0625f), comb3(T0, T1, T2), -dm.y * mn);
    }
};

// Q6_K: span = half n of a block: ql[64n ..] (4 units), qh[32n ..] (2 units),
// scales[8n ..], d.  For l < 32: q1 = ql[l] lo | qh[l] bits 0-1 (element l), q2 =
// ql[32 + l] lo | bits 2-3 (32 + l), q3 = ql[l] hi | bits 4-5 (64 + l), q4 =
// ql[32 + l] hi | bits 6-7 (96 + l); element e uses scale e / 16 (quant.rs:312-336).
template <> struct SpanFmt<GGC_Q6_K> {
    __device__ static constexpr int elem(int s, int j) {
        const int w = s >> 1, hi = s & 1, l0 = 4 * w;
        return l0 < 32 ? (hi ? 64 : 0) + l0 + j : (hi ? 96 : 32) + (l0 - 32) + j;
    }
    __device__ static constexpr int step_of(int q, int t) {   // 16-element group q
        const int part = q >> 1, l = 16 * (q & 1) + 4 * t;
        const int l0 = (part & 1) ? 32 + l : l, hi = part >> 1;
        return 2 * (l0 >> 2) + hi;
    }
    __device__ static constexpr int qoff(int t, int j) { return 4 * t + j; }
    __device__ static float dot(const SpanRow& R, int lane, const uint32_t* L, float gs, const float* xq) {
        uint4 h[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) h[k] = lds128(R.p[1] + (k * R.nl + lane) * 16);
        const uint2 sc = lds64(R.p[2] + lane * 8);
        const uint32_t d16 = lds16(R.p[3] + (lane >> 1) * 2);
        // value = d sc (u - 32): sum_g sc_g (u . x_int) - 32 sum_g sc_g X_g; two passes
        // of eight ql words (groups {0,1,4,5}, then {2,3,6,7}) fold as they finish
        int T0 = 0, T1 = 0, T2 = 0;
        float off = 0.f;
        const float4 xa = xq_load(xq, 0), xb = xq_load(xq, 1);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            uint4 u[2];
#pragma unroll
            for (int k = 0; k < 2; ++k) u[k] = lds128(R.p[0] + ((2 * half + k) * R.nl + lane) * 16);
            Acc3 A[4];   // groups 2 half + {0, 1} (low nibbles), 4 + 2 half + {0, 1} (high)
#pragma unroll
            for (int v = 0; v < 8; ++v) {
                const int w = 8 * half + v;
                const uint32_t q = wsel(u[v >> 2], v & 3);
                const uint32_t hb = wsel(h[v >> 2], v & 3);
                uint32_t lo, hi;
                if (half == 0) {
                    lo = (q & 0x0F0F0F0Fu) | ((hb << 4) & 0x30303030u);
                    hi = ((q >> 4) & 0x0F0F0F0Fu) | (hb & 0x30303030u);
                } else {
                    lo = (q & 0x0F0F0F0Fu) | ((hb << 2) & 0x30303030u);
                    hi = ((q >> 4) & 0x0F0F0F0Fu) | ((hb >> 2) & 0x30303030u);
                }
                dp3u(lo, L + 6 * w, A[v >> 2]);
                dp3u(hi, L + 6 * w + 3, A[2 + (v >> 2)]);
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int g = (j < 2 ? 0 : 4) + 2 * half + (j & 1);
                const int c = (int)(int8_t)(((g < 4 ? sc.x : sc.y) >> (8 * (g & 3))) & 0xFFu);
                T0 += c * A[j].a0; T1 += c * A[j].a1; T2 += c * A[j].a2;
                off = fmaf((float)c, f4sel(g < 4 ? xa : xb, g & 3), off);
            }
        }
        const float d = h2f(d16);
        return d * fmaf(gs, comb3(T0, T1, T2), -32.f * off);
    }
};

// Q4_0 (the reference's interleaved nibbles: byte m of qs holds element 2m in
// its low and 2m + 1 in its high nibble, quant.rs:139-150): span = 4 blocks.
template <> struct SpanFmt<GGC_Q4_0> {
    __device__ static constexpr int elem(int s, int j) {
        const int k = s >> 3, i = (s >> 1) & 3, hi = s & 1;
        return 32 * k + 8 * i + 2 * j + hi;
    }
    __device__ static constexpr int step_of(int q, int t) {   // elements 16q .. +16: block q/2, words 2(q%2) + t/2
        return 8 * (q >> 1) + 2 * (2 * (q & 1) + (t >> 1)) + (t & 1);
    }
    __device__ static constexpr int qoff(int t, int j) { return 8 * (t >> 1) + 2 * j + (t & 1); }
    __device__ static float dot(const SpanRow& R, int lane, const uint32_t* L, float gs, const float* xq) {
        uint4 u[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) u[k] = lds128(R.p[0] + (k * R.nl + lane) * 16);
        const uint2 dd = lds64(R.p[1] + lane * 8);
        const float4 xs = xq_load(xq, 2);
        float r = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            Acc3 lo, hi;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t q = wsel(u[k], i);
                dp3u(q & 0x0F0F0F0Fu, L + 3 * (8 * k + 2 * i), lo);
                dp3u(q & 0xF0F0F0F0u, L + 3 * (8 * k + 2 * i + 1), hi);   // 16 q
            }
            const float s16 = comb3(16 * lo.a0 + hi.a0, 16 * lo.a1 + hi.a1, 16 * lo.a2 + hi.a2);
            const float d = h2f(((k < 2 ? dd.x : dd.y) >> (16 * (k & 1))) & 0xFFFFu);
            // value = d (q - 8)  (quant.rs:139-150)
            r = fmaf(d, fmaf(gs * 0.0625f, s16, -8.f * f4sel(xs, k)), r);
        }
        return r;
    }
};

// Q8_0: span = 4 blocks of 32 int8; unit k = bytes 16 (k % 2) .. of block k / 2.
template <> struct SpanFmt<GGC_Q8_0> {
    __device__ static constexpr int elem(int s, int j) {
        const int k = s >> 2, i = s & 3;
        return 32 * (k >> 1) + 16 * (k & 1) + 4 * i + j;
    }
    __device__ static constexpr int step_of(int q, int t) { return 4 * q + t; }
    __device__ static constexpr int qoff(int t, int j) { return 4 * t + j; }
    __device__ static float dot(const SpanRow& R, int lane, const uint32_t* L, float gs, const float* xq) {
        uint4 u[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) u[k] = lds128(R.p[0] + (k * R.nl + lane) * 16);
        const uint2 dd = lds64(R.p[1] + lane * 8);
        float r = 0.f;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            Acc3 A;
#pragma unroll
            for (int k = 2 * b; k < 2 * b + 2; ++k)
#pragma unroll
                for (int i = 0; i < 4; ++i) dp3s(wsel(u[k], i), L + 3 * (4 * k + i), A);
            const float d = h2f(((b < 2 ? dd.x : dd.y) >> (16 * (b & 1))) & 0xFFFFu);
            r = fmaf(d, comb(A), r);   // value = d q  (quant.rs:173-180)
        }
        return r * gs;
    }
};

// Q4_1 (interleaved nibbles as Q4_0, value = d q + m, quant.rs:137-145): span = 4 blocks.
template <> struct SpanFmt<GGC_Q4_1> {
    __device__ static constexpr int elem(int s, int j) { return SpanFmt<GGC_Q4_0>::elem(s, j); }
    __device__ static constexpr int step_of(int q, int t) { return SpanFmt<GGC_Q4_0>::step_of(q, t); }
    __device__ static constexpr int qoff(int t, int j) { return SpanFmt<GGC_Q4_0>::qoff(t, j); }
    __device__ static float dot(const SpanRow& R, int lane, const uint32_t* L, float gs, const float* xq) {
        uint4 u[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) u[k] = lds128(R.p[0] + (k * R.nl + lane) * 16);
        const uint4 dm = lds128(R.p[1] + lane * 16);   // d[4], m[4]
        const float4 xs = xq_load(xq, 2);
        float r = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            Acc3 lo, hi;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t q = wsel(u[k], i);
                dp3u(q & 0x0F0F0F0Fu, L + 3 * (8 * k + 2 * i), lo);
                dp3u(q & 0xF0F0F0F0u, L + 3 * (8 * k + 2 * i + 1), hi);   // 16 q
            }
            const float s16 = comb3(16 * lo.a0 + hi.a0, 16 * lo.a1 + hi.a1, 16 * lo.a2 + hi.a2);
            const float d = h2f(((k < 2 ? dm.x : dm.y) >> (16 * (k & 1))) & 0xFFFFu);
            const float m = h2f(((k < 2 ? dm.z : dm.w) >> (16 * (k & 1))) & 0xFFFFu);
            r = fmaf(d, (gs * 0.0625f) * s16, fmaf(m, f4sel(xs, k), r));
        }
        return r;
    }
};

// Q5_0 / Q5_1 (quant.rs:147-186: qs[i] low nibble = element i, high = element 16 + i,
// the 5th bits from qh bits i and 16 + i): span = 4 blocks; block k's qh word is
// permuted so bit 8 j + i / 8 j + 4 + i is the 5th bit of byte j's low / high
// nibble in qs word i.  Value d (q - 16) (Q5_0) or d q + m (Q5_1).
template <int DT> struct SpanQ5 {
    __device__ static constexpr int elem(int s, int j) { return 32 * (s >> 3) + 16 * (s & 1) + 4 * ((s >> 1) & 3) + j; }
    __device__ static constexpr int step_of(int q, int t) { return 8 * (q >> 1) + 2 * t + (q & 1); }
    __device__ static constexpr int qoff(int t, int j) { return 4 * t + j; }
    __device__ static float dot(const SpanRow& R, int lane, const uint32_t* L, float gs, const float* xq) {
        uint4 u[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) u[k] = lds128(R.p[0] + (k * R.nl + lane) * 16);
        const uint4 hq = lds128(R.p[1] + lane * 16);
        uint4 dm;
        if (DT == GGC_Q5_1) {
            dm = lds128(R.p[2] + lane * 16);   // d[4], m[4]
        } else {
            const uint2 d2 = lds64(R.p[2] + lane * 8);
            dm = make_uint4(d2.x, d2.y, 0u, 0u);
        }
        const float4 xs = xq_load(xq, 2);
        float r = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t H = wsel(hq, k);
            Acc3 A;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t q = wsel(u[k], i);
                const uint32_t lo = (q & 0x0F0F0F0Fu) | (((H >> i) << 4) & 0x10101010u);
                const uint32_t hi = ((q >> 4) & 0x0F0F0F0Fu) | ((H >> i) & 0x10101010u);
                dp3u(lo, L + 3 * (8 * k + 2 * i), A);
                dp3u(hi, L + 3 * (8 * k + 2 * i + 1), A);
            }
            const float d = h2f(((k < 2 ? dm.x : dm.y) >> (16 * (k & 1))) & 0xFFFFu);
            if (DT == GGC_Q5_1) {
                const float m = h2f(((k < 2 ? dm.z : dm.w) >> (16 * (k & 1))) & 0xFFFFu);
                r = fmaf(d, gs * comb(A), fmaf(m, f4sel(xs, k), r));
            } else {
                r = fmaf(d, fmaf(gs, comb(A), -16.f * f4sel(xs, k)), r);
            }
        }
        return r;
    }
};
template <> struct SpanFmt<GGC_Q5_0> : SpanQ5<GGC_Q5_0> {};
template <> struct SpanFmt<GGC_Q5_1> : SpanQ5<GGC_Q5_1> {};

// Q2_K (quant.rs:190-205): span = half n of a block; qs byte m of the span holds
// elements 4 m + t at bits 2 t, so qs word w gives, per shift t, the four elements
// 16 w + 4 j + t of local sub-block w (16 elements, scale k_scale4(8 n + w)).
// s < 8: value = d s q; else value = dmin ((2 s - 8) q + (s - 8)).
template <> struct SpanFmt<GGC_Q2_K> {
    __device__ static constexpr int elem(int s, int j) { return 16 * (s >> 2) + 4 * j + (s & 3); }
    __device__ static constexpr int step_of(int q, int t) { return 4 * q + t; }
    __device__ static constexpr int qoff(int t, int j) { return 4 * j + t; }
    __device__ static float dot(const SpanRow& R, int lane, const uint32_t* L, float gs, const float* xq) {
        uint4 u[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) u[k] = lds128(R.p[0] + (k * R.nl + lane) * 16);
        const uint32_t sc4 = lds32(R.p[1] + lane * 4);
        const uint32_t dd = lds32(R.p[2] + (lane >> 1) * 4);
        int D0 = 0, D1 = 0, D2 = 0, M0 = 0, M1 = 0, M2 = 0;
        float offm = 0.f;
#pragma unroll
        for (int p = 0; p < 2; ++p) {
            const float4 xs = xq_load(xq, p);   // sums of sub-blocks 4p .. 4p + 3
            Acc3 A[4];
#pragma unroll
            for (int v = 0; v < 4; ++v) {
                const int w = 4 * p + v;
                const uint32_t W = wsel(u[p], v);
#pragma unroll
                for (int t = 0; t < 4; ++t) dp3u((W >> (2 * t)) & 0x03030303u, L + 3 * (4 * w + t), A[v]);
            }
#pragma unroll
            for (int v = 0; v < 4; ++v) {
                const int sv = (int)((sc4 >> (4 * (4 * p + v))) & 0xFu);
                const int cd = sv < 8 ? sv : 0, cm = sv < 8 ? 0 : 2 * sv - 8;
                D0 += cd * A[v].a0; D1 += cd * A[v].a1; D2 += cd * A[v].a2;
                M0 += cm * A[v].a0; M1 += cm * A[v].a1; M2 += cm * A[v].a2;
                offm = fmaf((float)(sv < 8 ? 0 : sv - 8), f4sel(xs, v), offm);
            }
        }
        const float2 dm = h2f2(dd);
        return fmaf(dm.x * gs, comb3(D0, D1, D2), dm.y * fmaf(gs, comb3(M0, M1, M2), offm));
    }
};

// Q3_K (quant.rs:209-245): element layout as Q2_K; the span's qs and hmask are
// stored inverted, so u = q + 3 = (ql ^ 3) | (h ^ 1) << 2 takes a shift and a mask
// (the h bits of qs word w, shift t at bit t + 4 (w % 2) of hmask word w / 2);
// value = d sc q with the int8 scale of local sub-block w.
template <int DT> struct SpanQ3K {
    __device__ static constexpr int elem(int s, int j) { return 16 * (s >> 2) + 4 * j + (s & 3); }
    __device__ static constexpr int step_of(int q, int t) { return 4 * q + t; }
    __device__ static constexpr int qoff(int t, int j) { return 4 * j + t; }
    __device__ static float dot(const SpanRow& R, int lane, const uint32_t* L, float gs, const float* xq) {
        uint4 u[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) u[k] = lds128(R.p[0] + (k * R.nl + lane) * 16);
        const uint4 hm = lds128(R.p[1] + lane * 16);
        const uint2 sc = lds64(R.p[2] + lane * 8);
        const uint32_t d16 = lds16(R.p[3] + (lane >> 1) * 2);
        int T0 = 0, T1 = 0, T2 = 0;
        float off = 0.f;
#pragma unroll
        for (int p = 0; p < 2; ++p) {
            const float4 xs = xq_load(xq, p);
            Acc3 A[4];
#pragma unroll
            for (int v = 0; v < 4; ++v) {
                const int w = 4 * p + v;
                const uint32_t W = wsel(u[p], v), H = wsel(hm, w >> 1);
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const int sh = t + 4 * (w & 1);
                    const uint32_t h4 = (sh >= 2 ? (H >> (sh - 2)) : (H << (2 - sh))) & 0x04040404u;
                    dp3u(((W >> (2 * t)) & 0x03030303u) | h4, L + 3 * (4 * w + t), A[v]);
                }
            }
#pragma unroll
            for (int v = 0; v < 4; ++v) {
                const int c = (int)(int8_t)(((p == 0 ? sc.x : sc.y) >> (8 * v)) & 0xFFu);
                T0 += c * A[v].a0; T1 += c * A[v].a1; T2 += c * A[v].a2;
                off = fmaf((float)c, f4sel(xs, v), off);
            }
        }
        return h2f(d16) * fmaf(gs, comb3(T0, T1, T2), -3.f * off);
    }
};
template <> struct SpanFmt<GGC_Q3_K_S> : SpanQ3K<GGC_Q3_K_S> {};
template <> struct SpanFmt<GGC_Q3_K_M> : SpanQ3K<GGC_Q3_K_M> {};
template <> struct SpanFmt<GGC_Q3_K_L> : SpanQ3K<GGC_Q3_K_L> {};

// Q5_K as the reference reads it (quant.rs:287-307): element k = nibble k % 2 of
// qs[k / 2] with the 5th bit from qh bit k / 2 (both nibbles of a byte share it),
// sub-blocks of 32 with the 6-bit (scale, min) pairs: span = half n of a block,
// qs unit k = local sub-block k, element layout as Q4_0; the 5th bits of qs word w
// at bit 8 j + w % 8 of qh word w / 8.  Value d sc q - dmin mn.
template <> struct SpanFmt<GGC_Q5_K> {
    __device__ static constexpr int elem(int s, int j) { return SpanFmt<GGC_Q4_0>::elem(s, j); }
    __device__ static constexpr int step_of(int q, int t) { return SpanFmt<GGC_Q4_0>::step_of(q, t); }
    __device__ static constexpr int qoff(int t, int j) { return SpanFmt<GGC_Q4_0>::qoff(t, j); }
    __device__ static float dot(const SpanRow& R, int lane, const uint32_t* L, float gs, const float* xq) {
        uint4 u[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) u[k] = lds128(R.p[0] + (k * R.nl + lane) * 16);
        const uint32_t dd = lds32(R.p[1] + (lane >> 1) * 4);
        const uint2 scm = lds64(R.p[2] + lane * 8);
        const uint2 hw = lds64(R.p[3] + lane * 8);
        int T0 = 0, T1 = 0, T2 = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            Acc3 A;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int w = 4 * k + i, b = w & 7;
                const uint32_t q = wsel(u[k], i), H = w < 8 ? hw.x : hw.y;
                const uint32_t h5 = (b <= 4 ? (H << (4 - b)) : (H >> (b - 4))) & 0x10101010u;
                dp3u((q & 0x0F0F0F0Fu) | h5, L + 3 * (8 * k + 2 * i), A);
                dp3u(((q >> 4) & 0x0F0F0F0Fu) | h5, L + 3 * (8 * k + 2 * i + 1), A);
            }
            const int c = (int)((scm.x >> (8 * k)) & 0xFFu);
            T0 += c * A.a0; T1 += c * A.a1; T2 += c * A.a2;
        }
        const float4 xs = xq_load(xq, 2);
        float mn = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) mn = fmaf((float)((scm.y >> (8 * k)) & 0xFFu), f4sel(xs, k), mn);
        const float2 dm = h2f2(dd);
        return fmaf(dm.x * gs, comb3(T0, T1, T2), -dm.y * mn);
    }
};

// Q8_K (quant.rs:338-344): span = half a block of int8, one f32 d; element layout as Q8_0.
template <> struct SpanFmt<GGC_Q8_K> {
    __device__ static constexpr int elem(int s, int j) { return 4 * s + j; }
    __device__ static constexpr int step_of(int q, int t) { return 4 * q + t; }
    __device__ static constexpr int qoff(int t, int j) { return 4 * t + j; }
    __device__ static float dot(const SpanRow& R, int lane, const uint32_t* L, float gs, const float* xq) {
        uint4 u[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) u[k] = lds128(R.p[0] + (k * R.nl + lane) * 16);
        const uint32_t dd = lds32(R.p[1] + (lane >> 1) * 4);
        Acc3 A;
#pragma unroll
        for (int k = 0; k < 8; ++k)
#pragma unroll
            for (int i = 0; i < 4; ++i) dp3s(wsel(u[k], i), L + 3 * (4 * k + i), A);
        return __uint_as_float(dd) * (comb(A) * gs);
    }
};

// ---- launch geometry (host) ------------------------------------------------
struct SpanCfg {
    uint32_t poff[4];       // plane offsets inside a stage
    uint32_t stage_bytes, stages;
    uint32_t xl_bytes;      // limb words + per-span floats of every column tile
    uint32_t part_rows;     // row sums kept per CTA (its rows, added over the column tiles)
    uint32_t smem;          // dynamic shared memory
};

template <int DT>
SpanCfg make_span_cfg(uint32_t pcols, uint32_t total_rb, uint32_t ctas, size_t smem_limit) {
    const TileLayout L = make_layout(DT, TILE_ROWS, pcols);
    const SpanSpec sp = span_spec(DT);
    SpanCfg c{};
    uint32_t off = 0;
    for (int p = 0; p < 4; ++p) {
        c.poff[p] = off;
        off += p < sp.n ? (TILE_ROWS * L.tp_full[p] + 127u) / 128u * 128u : 0u;
    }
    c.stage_bytes = off;
    const uint32_t nsp_full = L.nct * SPAN_LANES;
    c.xl_bytes = (nsp_full * (GS_WORDS + GS_XF) * 4u + 127u) / 128u * 128u;
    c.part_rows = ((total_rb + ctas - 1) / ctas) * TILE_ROWS;   // every row's sum, gathered for the epilogues
    const size_t fixed = (size_t)c.xl_bytes + c.part_rows * 4u + 128;
    const size_t st = smem_limit > fixed ? (smem_limit - fixed) / c.stage_bytes : 0;
    c.stages = (uint32_t)(st > (size_t)GS_MAX_STAGES ? GS_MAX_STAGES : st);
    c.smem = (uint32_t)(fixed + (size_t)c.stages * c.stage_bytes);
    return c;
}

// x of one GEMV into the span limb layout for every column tile: xl[ct][24][lane][4]
// limb words and xfs[ct] (gs per lane, then [3][lane] float4 of x sums).  Run by the 256 consumer
// threads (named barrier 1); activations are read through L2 (written by other
// CTAs of a persistent grid).  `red`: NWARPS doubles, `s_scale`: one float.  Run by
// the NWARPS consumer warps (named barrier 1).
// The prologue's input by value (kernel parameters cannot alias the stores the
// prologue makes; fields read through a reference to global memory would be
// re-loaded after each of them).
struct SpanX {
    const float* x;
    const float* x2;
    uint32_t xcols;
    int pro;
    int* errf;
    int pro_err_slot, pro_err_val;
};
__device__ __forceinline__ SpanX span_x_of(const GemvArgs& a) {
    return SpanX{a.x, a.x2, a.xcols, a.pro, a.errf, a.pro_err_slot, a.pro_err_val};
}

__device__ __forceinline__ float span_xval(const SpanX a, uint32_t e, float scale) {
    if (e >= a.xcols) return 0.f;
    const float x = __ldcg(a.x + e);
    if (a.pro == PRO_RMSNORM) return __fmul_rn(__fmul_rn(x, scale), __ldcg(a.x2 + e));
    if (a.pro == PRO_SWIGLU) return ffn_silu_mul(x, __ldcg(a.x2 + e));
    return x;
}

// The 16 x values of item `it` (span it / 8, quarter it % 8) of a GEMV input:
// plain, ops::rmsnorm with `scale` (ops.rs:262-274) or silu(gate) * up.  Zero
// past xcols and for dead items.
__device__ __forceinline__ void span_item_load(const SpanX a, uint32_t it, bool live, float scale, float (&v)[16]) {
    const uint32_t sp = it >> 3, q = it & 7;
    const uint32_t e0 = sp * SPAN + 16 * q;
#pragma unroll
    for (int k = 0; k < 16; ++k) v[k] = 0.f;
    if (live && e0 + 16 <= a.xcols) {
        const float4* x4 = reinterpret_cast<const float4*>(a.x + e0);
        float4 xa[4], ya[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) xa[k] = __ldcg(x4 + k);
        if (a.pro != PRO_PLAIN) {
            const float4* y4 = reinterpret_cast<const float4*>(a.x2 + e0);
#pragma unroll
            for (int k = 0; k < 4; ++k) ya[k] = __ldcg(y4 + k);
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float xx[4] = {xa[k].x, xa[k].y, xa[k].z, xa[k].w};
            const float yy[4] = {ya[k].x, ya[k].y, ya[k].z, ya[k].w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                v[4 * k + j] = a.pro == PRO_RMSNORM ? __fmul_rn(__fmul_rn(xx[j], scale), yy[j])   // ops.rs:272
                             : a.pro == PRO_SWIGLU ? ffn_silu_mul(xx[j], yy[j])
                             : xx[j];
            }
        }
    } else if (live) {
#pragma unroll
        for (int k = 0; k < 16; ++k) v[k] = span_xval(a, e0 + k, scale);   // checks e < xcols
    }
}

// Item `it`'s 16 values -> the span's power-of-two scale gs (max |x| of the span
// below 2^22 gs), three 8-bit limb words per step in xl, and the quarter / half
// sums in xfs.  Called by all 32 lanes of a warp together (the 8 quarters of a
// span are 8 consecutive lanes).
template <int DT>
__device__ __forceinline__ void span_item_store(const float (&v)[16], uint32_t it, bool live, uint32_t* xl, float* xfs) {
    using F = SpanFmt<DT>;
    const uint32_t sp = it >> 3, q = it & 7;
    float mx = 0.f, sum = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k) { mx = fmaxf(mx, fabsf(v[k])); sum += v[k]; }
    bool finite = isfinite(mx) && isfinite(sum);
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        finite = __shfl_xor_sync(0xffffffffu, (int)finite, o) && finite;
    }
    const float pair = __shfl_xor_sync(0xffffffffu, sum, 1);   // the other quarter of the 32-element half
    int ex = 0;
    frexpf(mx, &ex);
    const float mul = (mx > 0.f && finite) ? ldexpf(1.f, 22 - ex) : 0.f;
    const float gs = !finite ? __int_as_float(0x7FC00000) : (mx > 0.f ? ldexpf(1.f, ex - 22) : 0.f);
    if (live) {
        const uint32_t ct = sp / SPAN_LANES, l = sp % SPAN_LANES;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const int s = F::step_of((int)q, t);
            uint32_t w0 = 0, w1 = 0, w2 = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int xi = __float2int_rn(v[F::qoff(t, j)] * mul);
                w0 |= (uint32_t)(xi & 0xFF) << (8 * j);
                w1 |= (uint32_t)((xi >> 8) & 0xFF) << (8 * j);
                w2 |= (uint32_t)((xi >> 16) & 0xFF) << (8 * j);
            }
            const uint32_t wi[3] = {(uint32_t)(3 * s), (uint32_t)(3 * s + 1), (uint32_t)(3 * s + 2)};
            const uint32_t wv[3] = {w0, w1, w2};
#pragma unroll
            for (int k = 0; k < 3; ++k)
                xl[(((size_t)ct * 24 + wi[k] / 4) * SPAN_LANES + l) * 4 + wi[k] % 4] = wv[k];
        }
        float* xc = xfs + (size_t)ct * GS_XF * SPAN_LANES;   // [gs x 32][3][32] float4
        xc[SPAN_LANES + ((q >> 2) * SPAN_LANES + l) * 4 + (q & 3)] = sum;
        if ((q & 1) == 0) xc[SPAN_LANES + (2 * SPAN_LANES + l) * 4 + (q >> 1)] = sum + pair;
        if (q == 0) xc[l] = gs;
    }
}

// The RMSNorm weight of the one-item-per-thread prologue (x of at most one column
// tile), read into registers before griddepcontrol.wait: the norm weight is a
// model constant, so its load latency (HBM: the weight stream evicts it from L2
// every step) overlaps the wait for the predecessor instead of following it.
struct NormW {
    float v[16];
    bool ok;
};
template <int NWARPS = GS_WARPS>
__device__ __forceinline__ NormW span_norm_preload(const SpanX a, uint32_t nct) {
    NormW w;
    const int tid = threadIdx.x;
    const uint32_t items = nct * SPAN_LANES * 8;
    w.ok = a.pro == PRO_RMSNORM && items <= (uint32_t)NWARPS * 32;
    const uint32_t e0 = (tid >> 3) * SPAN + 16 * (tid & 7);
    if (w.ok && (uint32_t)tid < items && e0 + 16 <= a.xcols) {
        const float4* w4 = reinterpret_cast<const float4*>(a.x2 + e0);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float4 v = __ldg(w4 + q);
            w.v[4 * q] = v.x; w.v[4 * q + 1] = v.y; w.v[4 * q + 2] = v.z; w.v[4 * q + 3] = v.w;
        }
    } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) w.v[e] = w.ok && (uint32_t)tid < items && e0 + e < a.xcols ? __ldg(a.x2 + e0 + e) : 0.f;
    }
    return w;
}

// Returns (thread 0) whether the RMSNorm sum of squares is NaN; the caller reports it.
// `pre`: the norm weight already in registers (span_norm_preload), or none.
template <int DT, int NWARPS = GS_WARPS>
__device__ bool span_x_prologue(const SpanX a, uint32_t nct, uint32_t* xl, float* xfs, double* red, float* s_scale,
                                const NormW* pre = nullptr) {
    constexpr uint32_t CT = NWARPS * 32;
    auto cbar = [] { asm volatile("bar.sync 1, %0;" ::"r"(CT) : "memory"); };
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t items = nct * SPAN_LANES * 8;
    if (a.pro == PRO_RMSNORM && items <= CT) {
        // one item per thread: x and the norm weight read once (one L2 round trip),
        // the sum of squares and the limbs from the same registers
        const uint32_t e0 = (tid >> 3) * SPAN + 16 * (tid & 7);
        float xv[16], wv[16];
        if ((uint32_t)tid < items && e0 + 16 <= a.xcols) {
            const float4* x4 = reinterpret_cast<const float4*>(a.x + e0);
            const float4* w4 = reinterpret_cast<const float4*>(a.x2 + e0);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float4 v = __ldcg(x4 + q);
                xv[4 * q] = v.x; xv[4 * q + 1] = v.y; xv[4 * q + 2] = v.z; xv[4 * q + 3] = v.w;
                if (!pre) {
                    const float4 w = __ldg(w4 + q);
                    wv[4 * q] = w.x; wv[4 * q + 1] = w.y; wv[4 * q + 2] = w.z; wv[4 * q + 3] = w.w;
                }
            }
        } else {
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                const bool in = (uint32_t)tid < items && e0 + e < a.xcols;
                xv[e] = in ? __ldcg(a.x + e0 + e) : 0.f;
                if (!pre) wv[e] = in ? __ldg(a.x2 + e0 + e) : 0.f;
            }
        }
        if (pre) {
#pragma unroll
            for (int e = 0; e < 16; ++e) wv[e] = pre->v[e];
        }
        double ss = 0.0;
#pragma unroll
        for (int e = 0; e < 16; ++e) ss += (double)xv[e] * (double)xv[e];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) red[warp] = ss;
        cbar();
        double t = 0.0;
#pragma unroll
        for (int w = 0; w < NWARPS; ++w) t += red[w];
        const float scale = (float)sqrt(1.0 / (t / (double)a.xcols + (double)1e-6f));   // ops.rs:262-274
        float v[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) v[e] = __fmul_rn(__fmul_rn(xv[e], scale), wv[e]);   // ops.rs:272
        span_item_store<DT>(v, (uint32_t)tid, (uint32_t)tid < items, xl, xfs);
        cbar();
        return tid == 0 && isnan(t);   // NaN in x <=> NaN sum
    }
    float scale = 0.f;
    bool x_nan = false;
    if (a.pro == PRO_RMSNORM) {
        double ss = 0.0;
        if ((a.xcols & 3) == 0) {
            const float4* x4 = reinterpret_cast<const float4*>(a.x);
            for (uint32_t i = tid; i < a.xcols / 4; i += CT) {
                const float4 v = __ldcg(x4 + i);
                ss += (double)v.x * (double)v.x + (double)v.y * (double)v.y + (double)v.z * (double)v.z +
                      (double)v.w * (double)v.w;
            }
        } else {
            for (uint32_t i = tid; i < a.xcols; i += CT) { const double v = (double)__ldcg(a.x + i); ss += v * v; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) red[warp] = ss;
        cbar();
        if (tid == 0) {
            double t = 0.0;
            for (int w = 0; w < NWARPS; ++w) t += red[w];
            *s_scale = (float)sqrt(1.0 / (t / (double)a.xcols + (double)1e-6f));   // ops.rs:262-274
            x_nan = isnan(t);   // NaN in x <=> NaN sum
        }
        cbar();
        scale = *s_scale;
    }
    // x -> limbs: 8 threads per span (one quarter of 16 elements each)
    {
        for (uint32_t base = 0; base < items; base += CT) {
            const uint32_t it = base + tid;
            const bool live = it < items;
            float v[16];
            span_item_load(a, it, live, scale, v);
            span_item_store<DT>(v, it, live, xl, xfs);
        }
    }
    cbar();
    return x_nan;
}

// ---- the kernel ------------------------------------------------------------
template <int DT>
__global__ void __launch_bounds__(GS_THREADS, 1) k_gemv_span(const GemvArgs a, const SpanCfg cfg) {
    using F = SpanFmt<DT>;
    constexpr SpanSpec SP = span_spec(DT);
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ Seg sseg[3];
    __shared__ double red[GS_WARPS];
    __shared__ float s_scale;
    __shared__ unsigned long long s_best[GS_WARPS];
    __shared__ int s_dead;   // a tile never arrived: no more waits, no epilogues

    uint32_t* xl = reinterpret_cast<uint32_t*>(smem);                                // [ct][24][lane][4]
    const uint32_t nct = a.seg[0].m.L.nct;
    float* xfs = reinterpret_cast<float*>(smem + (size_t)nct * SPAN_LANES * GS_WORDS * 4);   // [ct][9][lane]
    float* part = reinterpret_cast<float*>(smem + cfg.xl_bytes);                      // [part_rows]
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + cfg.xl_bytes + cfg.part_rows * 4u);
    uint64_t* empty = full + GS_MAX_STAGES;
    uint8_t* stages = reinterpret_cast<uint8_t*>(full) + 128;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid < a.nseg) sseg[tid] = a.seg[tid];
    if (tid == 0) {
        for (uint32_t s = 0; s < cfg.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], GS_WARPS);
        }
        s_dead = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (tid < GS_WARPS) s_best[tid] = 0ull;
    __syncthreads();
    pdl_trigger();

    // contiguous range of row blocks (over all segments); tiles column-tile-major
    uint32_t total_rb = 0;
    for (int i = 0; i < a.nseg; ++i) total_rb += sseg[i].m.L.nrb;
    const uint32_t rb0 = (uint32_t)((uint64_t)total_rb * blockIdx.x / gridDim.x);
    const uint32_t rb1 = (uint32_t)((uint64_t)total_rb * (blockIdx.x + 1) / gridDim.x);
    const uint32_t nrb = rb1 - rb0, ntiles = nrb * nct;
    auto locate = [&](uint32_t g, int& si, uint32_t& rb) {
        si = 0;
        rb = g;
        while (si + 1 < a.nseg && rb >= sseg[si].m.L.nrb) { rb -= sseg[si].m.L.nrb; ++si; }
    };
    auto skip = [&]() { return (a.st_done && *a.st_done) || (a.st_skip && a.st_skip[0] < a.st_skip[1]); };

    if (warp == GS_WARPS) {
        // ---------------- producer warp ----------------
        const uint32_t prefetch = ntiles < cfg.stages ? ntiles : cfg.stages;
        bool waited = false;
        uint32_t s = 0, ph = 1, rbl = 0, ct = 0, rb = 0;   // empty[s] phase: the first round needs no wait
        int si = 0;
        locate(rb0, si, rb);
        for (uint32_t i = 0; i < ntiles; ++i) {
            if (i == prefetch) {
                pdl_wait();
                waited = true;
                if (skip()) break;
            }
            if (i >= cfg.stages && !mbar_wait(&empty[s], ph, a.errf)) break;
            if (lane == 0) {
                const QMat& m = sseg[si].m;
                uint32_t bytes = 0;
#pragma unroll
                for (int p = 0; p < SP.n; ++p) bytes += TILE_ROWS * tile_pitch(m.L, p, ct);
                mbar_arrive_expect_tx(&full[s], bytes);
                uint8_t* st = stages + (size_t)s * cfg.stage_bytes;
#pragma unroll
                for (int p = 0; p < SP.n; ++p)
                    bulk_g2s(st + cfg.poff[p], m.p[p] + tile_offset(m.L, p, rb, ct), TILE_ROWS * tile_pitch(m.L, p, ct),
                             &full[s]);
            }
            __syncwarp();
            if (++s == cfg.stages) { s = 0; ph ^= 1u; }
            if (++rbl == nrb) {
                rbl = 0;
                ++ct;
                locate(rb0, si, rb);
            } else if (++rb == sseg[si].m.L.nrb) {
                rb = 0;
                ++si;
            }
        }
        if (!waited) pdl_wait();
        return;
    }

    // ---------------- consumer warps ----------------
    const NormW normw = span_norm_preload(span_x_of(a), nct);
    pdl_wait();
    // the skip flags' loads are issued here and used after the x prologue, so
    // their latency overlaps it (the prologue only reads x, and its NaN report
    // waits for the flags)
    const bool skipping = skip();
    constexpr uint32_t CT = GS_WARPS * 32;
    auto cbar = [] { asm volatile("bar.sync 1, %0;" ::"r"(CT) : "memory"); };
    const bool x_nan = span_x_prologue<DT>(span_x_of(a), nct, xl, xfs, red, &s_scale, normw.ok ? &normw : nullptr);
    if (skipping) {   // drain the copies issued before the flag was seen
        const uint32_t n = ntiles < cfg.stages ? ntiles : cfg.stages;
        for (uint32_t i = 0; i < n; ++i) mbar_wait(&full[i], 0, a.errf);
        return;
    }
    if (tid == 0 && x_nan && a.pro_err_val) atomicCAS(&a.errf[a.pro_err_slot], 0, a.pro_err_val);
    for (uint32_t i = tid; i < cfg.part_rows; i += CT) part[i] = 0.f;
    cbar();

    const int r0 = 2 * warp;   // this warp's row pair in every tile
    uint32_t L[GS_WORDS];
    float gs = 0.f;             // x scale of this lane's span in the current column tile
    const float* xq = nullptr;  // its x sums (shared memory)
    // tile i = (column tile ct, row block rb0 + rbl); counters advance instead of dividing
    uint32_t s = 0, ph = 0, rbl = 0, ct = 0;
    int nl = 0;
    uint32_t rowoff[2][4];
    for (uint32_t i = 0; i < ntiles; ++i) {
        // a tile that never arrives ends all waiting; the warps still meet below
        if (!*(volatile int*)&s_dead && !mbar_wait(&full[s], ph, a.errf)) s_dead = 1;
        if (*(volatile int*)&s_dead) {
            if (++s == cfg.stages) { s = 0; ph ^= 1u; }
            if (++rbl == nrb) { rbl = 0; ++ct; }
            continue;
        }
        if (rbl == 0) {   // a new column tile: x of this lane's span into registers, tile geometry
            const TileLayout& L0 = sseg[0].m.L;
            nl = ct + 1 == L0.nct ? (int)((L0.pcols - ct * SPAN_KC) / SPAN) : SPAN_LANES;
#pragma unroll
            for (int p = 0; p < 4; ++p) {
                const uint32_t pitch = tile_pitch(L0, p, ct);
                rowoff[0][p] = cfg.poff[p] + (uint32_t)r0 * pitch;
                rowoff[1][p] = rowoff[0][p] + pitch;
            }
#pragma unroll
            for (int k = 0; k < GS_WORDS / 4; ++k) {
                const uint4 w4 = *reinterpret_cast<const uint4*>(xl + (((size_t)ct * 24 + k) * SPAN_LANES + lane) * 4);
                L[4 * k] = w4.x; L[4 * k + 1] = w4.y; L[4 * k + 2] = w4.z; L[4 * k + 3] = w4.w;
            }
            gs = xfs[(size_t)ct * GS_XF * SPAN_LANES + lane];
            xq = xfs + (size_t)ct * GS_XF * SPAN_LANES + SPAN_LANES + lane * 4;
        }
        const uint8_t* st = stages + (size_t)s * cfg.stage_bytes;
        float y[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            SpanRow R;
#pragma unroll
            for (int p = 0; p < 4; ++p) R.p[p] = st + rowoff[k][p];
            R.nl = nl;
            y[k] = lane < nl ? F::dot(R, lane, L, gs, xq) : 0.f;
        }
        // two row sums: halve the exchange (lanes < 16 keep row 0), then reduce
        {
            const bool up = lane & 16;
            const float send = up ? y[0] : y[1];
            float v = (up ? y[1] : y[0]) + __shfl_xor_sync(0xffffffffu, send, 16);
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            y[0] = __shfl_sync(0xffffffffu, v, 0);
            y[1] = __shfl_sync(0xffffffffu, v, 16);
        }
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(&empty[s]);
            float* pp = part + rbl * TILE_ROWS + r0;   // row sums of the CTA's rows (added over column tiles)
            pp[0] += y[0];
            pp[1] += y[1];
        }
        if (++s == cfg.stages) { s = 0; ph ^= 1u; }
        if (++rbl == nrb) { rbl = 0; ++ct; }
    }
    // epilogues of all the CTA's rows at once, a row pair per thread, so their global
    // loads (residual, RoPE position and table, bias) overlap instead of following each tile
    cbar();
    if (*(volatile int*)&s_dead) return;
    unsigned long long best = 0ull;
    bool nan_logit = false;
    for (uint32_t p = tid; p < nrb * (TILE_ROWS / 2); p += CT) {
        int psi;
        uint32_t prb;
        locate(rb0 + p / (TILE_ROWS / 2), psi, prb);
        const Seg& sg = sseg[psi];
        const uint32_t row = prb * TILE_ROWS + 2 * (p % (TILE_ROWS / 2));
        if (row >= sg.m.L.rows) continue;
        const uint32_t nv = min(2u, sg.m.L.rows - row);
        const float* yy = part + 2 * p;
        if (sg.epi == EPI_LOGITS) {   // logits + greedy argmax (one atomic per warp)
            for (uint32_t k = 0; k < nv; ++k) {
                sg.out[row + k] = yy[k];
                nan_logit |= isnan(yy[k]);
                const unsigned long long key = argmax_key_of(yy[k], row + k);
                best = key > best ? key : best;
            }
        } else {
            gemv_epilogue(a, sg, row, nv, yy);
        }
    }
    if (sseg[0].epi == EPI_LOGITS) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
            best = other > best ? other : best;
        }
        nan_logit = __any_sync(0xffffffffu, nan_logit);
        if (lane == 0 && (best || nan_logit)) {
            if (nan_logit) atomicMax(&a.errf[ERRF_NAN_LOGITS], 1);
            atomicMax(a.argmax_key, best);
        }
    }
    if (a.ar_k)   // tensor parallel: this warp's row pair of each row block, summed over the ranks
        ar_reduce_rows(
            a.ar, a.ar_k, 2 * nrb, [&](uint32_t j) { return (rb0 + j / 2) * TILE_ROWS + (uint32_t)r0 + (j & 1); },
            sseg[0].m.L.rows, sseg[0].out, a.errf, a.err_slot, a.err_val);
}

}  // namespace ggc
