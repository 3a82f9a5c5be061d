// repack.cuh -- the split of raw GGUF rows into the tiled plane / span layout
// (planes.cuh), written once for the host and the device.
//
// The model loader uploads a weight's raw GGUF rows and runs k_repack on the
// GPU: one thread per (row, unit), a unit being one 128-element span (span
// formats) or one block (plane formats, one element for F16/BF16/F32).  Every
// unit's destination is a pure function of (row, unit) and the layout, so the
// units are independent and the device output is the host output byte for byte
// (repack_rows_host runs the same functions on host threads; GGC_REPACK=host
// selects it at upload).
#pragma once
#include "common.cuh"
#include "planes.cuh"

namespace ggc {
namespace rp {

__host__ __device__ inline uint32_t rd32(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
__host__ __device__ inline void wr32(uint8_t* p, uint32_t v) {
    p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); p[2] = (uint8_t)(v >> 16); p[3] = (uint8_t)(v >> 24);
}
__host__ __device__ inline void cpy(uint8_t* d, const uint8_t* s, int n) {
    for (int i = 0; i < n; ++i) d[i] = s[i];
}

// Q5_0 / Q5_1 qh: element i (i<16) uses bit i, element 16+i uses bit 16+i.
// Plane bit 8k+w   <- qh bit 4w+k      (low nibbles of chunk word w, byte k)
// Plane bit 8k+4+w <- qh bit 16+4w+k   (high nibbles of chunk word w, byte k)
__host__ __device__ inline uint32_t permute_q5_qh(uint32_t qh) {
    uint32_t o = 0;
    for (int w = 0; w < 4; ++w)
        for (int k = 0; k < 4; ++k) {
            o |= ((qh >> (4 * w + k)) & 1u) << (8 * k + w);
            o |= ((qh >> (16 + 4 * w + k)) & 1u) << (8 * k + 4 + w);
        }
    return o;
}

// quant.rs:116-124 k_scale_min_6bit for j = 0..7 -> sc[j] at out[j], mn[j] at out[8 + j]
__host__ __device__ inline void unpack_scale_min(const uint8_t* q, uint8_t* out) {
    for (int j = 0; j < 8; ++j) {
        uint8_t sc, mn;
        if (j < 4) {
            sc = q[j] & 0x3F;
            mn = q[j + 4] & 0x3F;
        } else {
            sc = (uint8_t)((q[j + 4] & 0x0F) | ((q[j - 4] >> 6) << 4));
            mn = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
        }
        out[j] = sc;
        out[8 + j] = mn;
    }
}

// One raw block b into the planes pl at block index blk of the tile row.
__host__ __device__ inline void repack_block(int dt, const uint8_t* b, uint64_t blk, uint8_t* const pl[4]) {
    switch (dt) {
        case GGC_Q4_0:
            cpy(pl[0] + blk * 16, b + 2, 16);
            cpy(pl[1] + blk * 2, b, 2);
            break;
        case GGC_Q4_1:
            cpy(pl[0] + blk * 16, b + 4, 16);
            cpy(pl[1] + blk * 4, b, 4);
            break;
        case GGC_Q5_0:
            cpy(pl[0] + blk * 16, b + 6, 16);
            wr32(pl[1] + blk * 4, permute_q5_qh(rd32(b + 2)));
            cpy(pl[2] + blk * 2, b, 2);
            break;
        case GGC_Q5_1:
            cpy(pl[0] + blk * 16, b + 8, 16);
            wr32(pl[1] + blk * 4, permute_q5_qh(rd32(b + 4)));
            cpy(pl[2] + blk * 4, b, 4);
            break;
        case GGC_Q8_0:
            cpy(pl[0] + blk * 32, b + 2, 32);
            cpy(pl[1] + blk * 2, b, 2);
            break;
        case GGC_Q2_K:
            cpy(pl[0] + blk * 64, b + 16, 64);
            cpy(pl[1] + blk * 16, b, 16);
            cpy(pl[2] + blk * 4, b + 80, 4);
            break;
        case GGC_Q3_K_S: case GGC_Q3_K_L: case GGC_Q3_K_M: {
            cpy(pl[0] + blk * 64, b + 32, 64);
            // hmask: element e uses bit e%8 of byte e/8.  Chunk p covers elements
            // 64p + 16w + 4k + s; plane word (2p + w/2), bit 8k + s + 4(w%2).
            uint32_t words[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            for (int e = 0; e < 256; ++e) {
                const uint32_t bit = (b[e / 8] >> (e % 8)) & 1u;
                const int p = e / 64, r = e % 64, w = r / 16, k = (r % 16) / 4, s = r % 4;
                words[2 * p + w / 2] |= bit << (8 * k + s + 4 * (w % 2));
            }
            for (int i = 0; i < 8; ++i) wr32(pl[1] + blk * 32 + 4 * i, words[i]);
            cpy(pl[2] + blk * 12, b + 96, 12);
            cpy(pl[3] + blk * 2, b + (dt == GGC_Q3_K_M ? 112 : 108), 2);
            break;
        }
        case GGC_Q4_K:
            cpy(pl[0] + blk * 128, b + 16, 128);
            cpy(pl[1] + blk * 4, b, 4);
            unpack_scale_min(b + 4, pl[2] + blk * 16);
            break;
        case GGC_Q5_K: {
            cpy(pl[0] + blk * 128, b + 48, 128);
            // qs byte B (0..127) takes its 5th bit from bit B%8 of qh[B/8] (only
            // qh[0..16) is read).  Chunk p = bytes 16p + 4w + k -> plane word p/2,
            // bit 8k + w + 4(p%2).
            uint32_t words[4] = {0, 0, 0, 0};
            for (int B = 0; B < 128; ++B) {
                const uint32_t bit = (b[16 + B / 8] >> (B % 8)) & 1u;
                const int p = B / 16, i = B % 16, w = i / 4, k = i % 4;
                words[p / 2] |= bit << (8 * k + w + 4 * (p % 2));
            }
            for (int i = 0; i < 4; ++i) wr32(pl[1] + blk * 16 + 4 * i, words[i]);
            cpy(pl[2] + blk * 4, b, 4);
            unpack_scale_min(b + 4, pl[3] + blk * 16);
            break;
        }
        case GGC_Q6_K:
            cpy(pl[0] + blk * 128, b, 128);
            cpy(pl[1] + blk * 64, b + 128, 64);
            cpy(pl[2] + blk * 16, b + 192, 16);
            cpy(pl[3] + blk * 2, b + 208, 2);
            break;
        case GGC_Q8_K:
            cpy(pl[0] + blk * 256, b + 4, 256);
            cpy(pl[1] + blk * 4, b, 4);
            break;
        case GGC_F16: case GGC_BF16:
            cpy(pl[0] + blk * 2, b, 2);
            break;
        case GGC_F32:
            cpy(pl[0] + blk * 4, b, 4);
            break;
        default:
            break;
    }
}

// One 128-element span (lane l of a column tile with nl lanes) of one row into
// the span layout; row[p] is the plane's row base in the tile.  Blocks past the
// row's end stay zero.
__host__ __device__ inline void repack_span(int dt, const uint8_t* src, uint64_t nb, uint64_t sp, uint32_t l,
                                            uint32_t nl, uint8_t* const row[4]) {
    auto unit = [&](int p, int k) { return row[p] + ((uint64_t)k * nl + l) * 16; };
    switch (dt) {
        case GGC_Q4_K: {   // span = half n of block sp / 2
            const uint64_t b = sp / 2;
            const int n = (int)(sp % 2);
            if (b >= nb) return;
            const uint8_t* blk = src + b * 144;
            for (int k = 0; k < 4; ++k) cpy(unit(0, k), blk + 16 + 64 * n + 16 * k, 16);
            if (n == 0) cpy(row[1] + (l / 2) * 4, blk, 4);
            uint8_t scm[16];
            unpack_scale_min(blk + 4, scm);
            cpy(row[2] + l * 8, scm + 4 * n, 4);
            cpy(row[2] + l * 8 + 4, scm + 8 + 4 * n, 4);
            break;
        }
        case GGC_Q6_K: {
            const uint64_t b = sp / 2;
            const int n = (int)(sp % 2);
            if (b >= nb) return;
            const uint8_t* blk = src + b * 210;
            for (int k = 0; k < 4; ++k) cpy(unit(0, k), blk + 64 * n + 16 * k, 16);
            for (int k = 0; k < 2; ++k) cpy(unit(1, k), blk + 128 + 32 * n + 16 * k, 16);
            cpy(row[2] + l * 8, blk + 192 + 8 * n, 8);
            if (n == 0) cpy(row[3] + (l / 2) * 2, blk + 208, 2);
            break;
        }
        case GGC_Q4_0:
            for (int k = 0; k < 4; ++k) {
                const uint64_t b = sp * 4 + k;
                if (b >= nb) break;
                cpy(unit(0, k), src + b * 18 + 2, 16);
                cpy(row[1] + l * 8 + 2 * k, src + b * 18, 2);
            }
            break;
        case GGC_Q8_0:
            for (int k = 0; k < 4; ++k) {
                const uint64_t b = sp * 4 + k;
                if (b >= nb) break;
                cpy(unit(0, 2 * k), src + b * 34 + 2, 16);
                cpy(unit(0, 2 * k + 1), src + b * 34 + 18, 16);
                cpy(row[1] + l * 8 + 2 * k, src + b * 34, 2);
            }
            break;
        case GGC_Q4_1:   // d, m, qs[16] (quant.rs:137-145): qs unit per block, d[4] then m[4]
            for (int k = 0; k < 4; ++k) {
                const uint64_t b = sp * 4 + k;
                if (b >= nb) break;
                cpy(unit(0, k), src + b * 20 + 4, 16);
                cpy(row[1] + l * 16 + 2 * k, src + b * 20, 2);
                cpy(row[1] + l * 16 + 8 + 2 * k, src + b * 20 + 2, 2);
            }
            break;
        case GGC_Q5_0: case GGC_Q5_1: {   // [d, (m,)] qh, qs[16] (quant.rs:147-186)
            const int bb = dt == GGC_Q5_0 ? 22 : 24, qh = dt == GGC_Q5_0 ? 2 : 4;
            for (int k = 0; k < 4; ++k) {
                const uint64_t b = sp * 4 + k;
                if (b >= nb) break;
                const uint8_t* blk = src + b * bb;
                cpy(unit(0, k), blk + qh + 4, 16);
                wr32(row[1] + l * 16 + 4 * k, permute_q5_qh(rd32(blk + qh)));
                if (dt == GGC_Q5_0) {
                    cpy(row[2] + l * 8 + 2 * k, blk, 2);
                } else {
                    cpy(row[2] + l * 16 + 2 * k, blk, 2);
                    cpy(row[2] + l * 16 + 8 + 2 * k, blk + 2, 2);
                }
            }
            break;
        }
        case GGC_Q2_K: {   // scales[16], qs[64], d, dmin (quant.rs:190-205); span = half n of block sp / 2
            const uint64_t b = sp / 2;
            const int n = (int)(sp % 2);
            if (b >= nb) return;
            const uint8_t* blk = src + b * 84;
            for (int k = 0; k < 2; ++k) cpy(unit(0, k), blk + 16 + 32 * n + 16 * k, 16);
            // local sub-block w = sub-block j = 8n + w: k_scale4 (quant.rs:100-108), nibble w of the record
            uint32_t sc = 0;
            for (int w = 0; w < 8; ++w) {
                const int j = 8 * n + w, byte = 15 - j / 2;
                sc |= (uint32_t)((j % 2 == 0) ? (blk[byte] & 0xF) : ((blk[byte] >> 4) & 0xF)) << (4 * w);
            }
            wr32(row[1] + l * 4, sc);
            if (n == 0) cpy(row[2] + (l / 2) * 4, blk + 80, 4);
            break;
        }
        case GGC_Q3_K_S: case GGC_Q3_K_M: case GGC_Q3_K_L: {   // quant.rs:209-245
            const uint64_t b = sp / 2;
            const int n = (int)(sp % 2);
            if (b >= nb) return;
            const int bb = dt == GGC_Q3_K_M ? 114 : 110, doff = dt == GGC_Q3_K_M ? 112 : 108;
            const uint8_t* blk = src + b * bb;
            // qs stored inverted (2-bit code ql -> ql ^ 3), hmask inverted (h -> h ^ 1): the
            // GEMV then reads u = q + 3 = (ql ^ 3) | (h ^ 1) << 2 with a shift and a mask
            for (int k = 0; k < 2; ++k) {
                uint8_t* d = unit(0, k);
                const uint8_t* q = blk + 32 + 32 * n + 16 * k;
                for (int i = 0; i < 16; ++i) d[i] = (uint8_t)~q[i];
            }
            // element e = 128 n + 16 w + 4 j + s (word w / 4 of unit w / 4, byte j, shift 2 s):
            // inverted h at bit 8 j + s + 4 (w % 2) of hmask word w / 2
            uint32_t hw[4] = {0, 0, 0, 0};
            for (int w = 0; w < 8; ++w)
                for (int j = 0; j < 4; ++j)
                    for (int t = 0; t < 4; ++t) {
                        const int e = 128 * n + 16 * w + 4 * j + t;
                        const uint32_t h = ((blk[e / 8] >> (e % 8)) & 1u) ^ 1u;
                        hw[w / 2] |= h << (8 * j + t + 4 * (w % 2));
                    }
            for (int i = 0; i < 4; ++i) wr32(row[1] + l * 16 + 4 * i, hw[i]);
            for (int w = 0; w < 8; ++w) {   // scale of sub-block g = 8n + w, as int8 (lo | hi << 4) - 32
                const int g = 8 * n + w;
                const int lo = (blk[96 + g / 2] >> ((g % 2) * 4)) & 0xF, hi = (blk[104 + g / 4] >> ((g % 4) * 2)) & 3;
                row[2][l * 8 + w] = (uint8_t)(int8_t)((lo | (hi << 4)) - 32);
            }
            if (n == 0) cpy(row[3] + (l / 2) * 2, blk + doff, 2);
            break;
        }
        case GGC_Q5_K: {   // d, dmin, scales[12], qh[32], qs[128] (quant.rs:287-307)
            const uint64_t b = sp / 2;
            const int n = (int)(sp % 2);
            if (b >= nb) return;
            const uint8_t* blk = src + b * 176;
            for (int k = 0; k < 4; ++k) cpy(unit(0, k), blk + 48 + 64 * n + 16 * k, 16);
            if (n == 0) cpy(row[1] + (l / 2) * 4, blk, 4);
            uint8_t scm[16];
            unpack_scale_min(blk + 4, scm);
            cpy(row[2] + l * 8, scm + 4 * n, 4);
            cpy(row[2] + l * 8 + 4, scm + 8 + 4 * n, 4);
            // qs byte B = 64n + 4w + j (both nibbles) takes its 5th bit from bit B % 8 of
            // qh[B / 8]: stored at bit 8 j + w % 8 of word w / 8
            uint32_t hw[2] = {0, 0};
            for (int w = 0; w < 16; ++w)
                for (int j = 0; j < 4; ++j) {
                    const int B = 64 * n + 4 * w + j;
                    hw[w / 8] |= (uint32_t)((blk[16 + B / 8] >> (B % 8)) & 1u) << (8 * j + w % 8);
                }
            wr32(row[3] + l * 8, hw[0]);
            wr32(row[3] + l * 8 + 4, hw[1]);
            break;
        }
        case GGC_Q8_K: {   // f32 d, qs[256], bsums (quant.rs:338-344)
            const uint64_t b = sp / 2;
            const int n = (int)(sp % 2);
            if (b >= nb) return;
            const uint8_t* blk = src + b * 292;
            for (int k = 0; k < 8; ++k) cpy(unit(0, k), blk + 4 + 128 * n + 16 * k, 16);
            if (n == 0) cpy(row[1] + (l / 2) * 4, blk, 4);
            break;
        }
        default:
            break;
    }
}

// Units per row: spans (span formats) or blocks.
__host__ __device__ inline uint64_t units_per_row(int dt, const TileLayout& L, uint64_t cols) {
    return is_span_dt(dt) ? (uint64_t)L.pcols / SPAN : cols / (uint64_t)block_size_of(dt);
}

// Unit u of output row r (source row bytes at src) into the planes.
__host__ __device__ inline void repack_unit(int dt, const uint8_t* src, uint64_t r, uint64_t u, uint64_t cols,
                                            const TileLayout& L, uint8_t* const planes[4]) {
    const uint32_t rb = (uint32_t)(r / TILE_ROWS), rl = (uint32_t)(r % TILE_ROWS);
    uint8_t* dst[4] = {nullptr, nullptr, nullptr, nullptr};
    if (is_span_dt(dt)) {
        const SpanSpec sp = span_spec(dt);
        const uint64_t nsp = L.pcols / SPAN, nb = cols / (uint64_t)block_size_of(dt);
        const uint32_t ct = (uint32_t)(u / SPAN_LANES), l = (uint32_t)(u % SPAN_LANES);
        const uint32_t nl = ct + 1 == L.nct ? (uint32_t)(nsp - (uint64_t)ct * SPAN_LANES) : SPAN_LANES;
        for (int p = 0; p < sp.n; ++p) dst[p] = planes[p] + tile_offset(L, p, rb, ct) + (uint64_t)rl * tile_pitch(L, p, ct);
        repack_span(dt, src, nb, u, l, nl, dst);
        return;
    }
    const PlaneSpec s = plane_spec(dt);
    const uint64_t bs = (uint64_t)block_size_of(dt), bb = (uint64_t)block_bytes_of(dt);
    const uint64_t per_tile = L.kc / bs;
    const uint32_t ct = (uint32_t)(u / per_tile);
    for (int p = 0; p < s.n; ++p) dst[p] = planes[p] + tile_offset(L, p, rb, ct) + (uint64_t)rl * tile_pitch(L, p, ct);
    repack_block(dt, src + u * bb, u - (uint64_t)ct * per_tile, dst);
}

}  // namespace rp

}  // namespace ggc
