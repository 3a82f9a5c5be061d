// planes.cuh -- the tiled layouts of uploaded weight tensors.
//
// A raw GGUF tensor stores each block's scale fields and quant bits together
// (e.g. Q4_K: d, dmin, scales[12], qs[128] = 144 bytes).  At upload the raw rows
// are split (on the GPU by k_repack, or on host threads; repack.cuh) into up to
// four planes: the quant payload and the side data (scales, d, dmin, high bits).
//
// Each plane is stored tile by tile: a tile is TILE_ROWS (16) rows x one column
// tile, and the bytes of one tile of one plane are contiguous in HBM (rows at a
// 16-byte-aligned tile pitch).  The GEMV therefore moves a tile with one large
// bulk copy per plane: bulk copies of 1 KB or less reach only ~3-4 TB/s on B200,
// copies of >= 4 KB with >= 128 KB in flight per SM reach > 7 TB/s.
//
// Block formats use the span layout below (k_gemv_span); F16 / BF16 / F32 use the
// plane layout of plane_spec (k_gemv: 16-byte chunks, 128 per tile row).  The
// plane_spec entries of the block formats describe the plane layout that k_gemv
// (instantiated for every format) reads; uploads of block formats use spans.
//
// The split keeps every value the reference's dequantiser reads and drops the
// bytes it never reads (Q3_K_M's 4 bytes at 108..111, Q5_K's qh[16..32), Q8_K's
// bsums).  High-bit fields (Q5_0/Q5_1/Q5_K qh, Q3_K hmask) are bit-permuted so
// that the bits a lane needs for four consecutive bytes sit one per byte of a
// 32-bit word (one shift + one mask).  The 12 packed bytes of the Q4_K/Q5_K 6-bit
// (scale, min) pairs are unpacked with the reference's k_scale_min_6bit
// (quant.rs:116-124), so the GEMV reads a scale with one byte extract.
#pragma once
#include "common.cuh"

namespace ggc {

constexpr int TILE_ROWS = 16;

struct PlaneSpec {
    int n;           // number of planes
    int bpb[4];      // bytes per block in each plane
    int chunk_elems; // elements covered by one 16-byte chunk of plane 0
};

__host__ __device__ constexpr PlaneSpec plane_spec(int dt) {
    return dt == GGC_Q4_0 ? PlaneSpec{2, {16, 2, 0, 0}, 32}
         : dt == GGC_Q4_1 ? PlaneSpec{2, {16, 4, 0, 0}, 32}
         : dt == GGC_Q5_0 ? PlaneSpec{3, {16, 4, 2, 0}, 32}
         : dt == GGC_Q5_1 ? PlaneSpec{3, {16, 4, 4, 0}, 32}
         : dt == GGC_Q8_0 ? PlaneSpec{2, {32, 2, 0, 0}, 16}
         : dt == GGC_Q2_K ? PlaneSpec{3, {64, 16, 4, 0}, 64}
         : (dt == GGC_Q3_K_S || dt == GGC_Q3_K_M || dt == GGC_Q3_K_L) ? PlaneSpec{4, {64, 32, 12, 2}, 64}
         : dt == GGC_Q4_K ? PlaneSpec{3, {128, 4, 16, 0}, 32}
         : dt == GGC_Q5_K ? PlaneSpec{4, {128, 16, 4, 16}, 32}
         : dt == GGC_Q6_K ? PlaneSpec{4, {128, 64, 16, 2}, 32}
         : dt == GGC_Q8_K ? PlaneSpec{2, {256, 4, 0, 0}, 16}
         : dt == GGC_F16 ? PlaneSpec{1, {2, 0, 0, 0}, 8}
         : dt == GGC_BF16 ? PlaneSpec{1, {2, 0, 0, 0}, 8}
         : dt == GGC_F32 ? PlaneSpec{1, {4, 0, 0, 0}, 4}
         : PlaneSpec{0, {0, 0, 0, 0}, 0};
}

// Span layout (every block format: the integer GEMV).  A column tile is 4096
// columns = 32 lanes x one 128-element "span" per lane; the bytes a lane reads for
// its span of a row are, per plane, either 16-byte units interleaved by lane
// (unit k of lane l at (k * nl + l) * 16, nl = lanes of the column tile) or a
// small per-lane record (at l * bps), or a per-block record shared by a lane pair
// (256-element blocks: d|dmin, d).  Rows are padded with zero bytes to a multiple
// of 128 columns.
constexpr int SPAN = 128;
constexpr int SPAN_LANES = 32;
constexpr uint32_t SPAN_KC = SPAN * SPAN_LANES;

__host__ __device__ constexpr bool is_span_dt(int dt) {
    return dt == GGC_Q4_0 || dt == GGC_Q4_1 || dt == GGC_Q5_0 || dt == GGC_Q5_1 || dt == GGC_Q8_0 || dt == GGC_Q2_K ||
           dt == GGC_Q3_K_S || dt == GGC_Q3_K_M || dt == GGC_Q3_K_L || dt == GGC_Q4_K || dt == GGC_Q5_K ||
           dt == GGC_Q6_K || dt == GGC_Q8_K;
}
struct SpanSpec {
    int n;          // planes
    int bps[4];     // bytes per span (per lane) in each plane
};
__host__ __device__ constexpr SpanSpec span_spec(int dt) {
    return dt == GGC_Q4_K ? SpanSpec{3, {64, 2, 8, 0}}     // qs units | d,dmin per block | sc[4] mn[4]
         : dt == GGC_Q6_K ? SpanSpec{4, {64, 32, 8, 1}}    // ql units | qh units | sc[8] | d per block
         : dt == GGC_Q4_0 ? SpanSpec{2, {64, 8, 0, 0}}     // qs units (4 blocks) | d[4]
         : dt == GGC_Q8_0 ? SpanSpec{2, {128, 8, 0, 0}}    // qs units (4 blocks) | d[4]
         : dt == GGC_Q4_1 ? SpanSpec{2, {64, 16, 0, 0}}    // qs units (4 blocks) | d[4] m[4]
         : dt == GGC_Q5_0 ? SpanSpec{3, {64, 16, 8, 0}}    // qs units | permuted qh word per block | d[4]
         : dt == GGC_Q5_1 ? SpanSpec{3, {64, 16, 16, 0}}   // qs units | permuted qh word per block | d[4] m[4]
         : dt == GGC_Q2_K ? SpanSpec{3, {32, 4, 2, 0}}     // qs units | scale nibbles[8] | d,dmin per block
         : (dt == GGC_Q3_K_S || dt == GGC_Q3_K_M || dt == GGC_Q3_K_L)
             ? SpanSpec{4, {32, 16, 8, 1}}                 // inverted qs units | inverted hmask words[4] | sc[8] | d per block
         : dt == GGC_Q5_K ? SpanSpec{4, {64, 2, 8, 8}}     // qs units | d,dmin per block | sc[4] mn[4] | qh words[2]
         : dt == GGC_Q8_K ? SpanSpec{2, {128, 2, 0, 0}}    // qs units | f32 d per block
         : SpanSpec{0, {0, 0, 0, 0}};
}

// Geometry of a tiled weight (computed identically on host and device).
struct TileLayout {
    uint32_t rows, pcols;      // rows, columns padded to the chunk width
    uint32_t kc, nct, nrb;     // columns of a full column tile, column tiles, row blocks
    uint32_t tp_full[4];       // tile row pitch of plane p in a full column tile
    uint32_t tp_last[4];       // ... in the last column tile
    uint64_t rb_bytes[4];      // bytes of one row block of plane p
};

__host__ __device__ inline uint32_t round16(uint32_t b) { return (b + 15u) / 16u * 16u; }

__host__ __device__ inline TileLayout make_layout(int dt, uint32_t rows, uint32_t pcols) {
    if (is_span_dt(dt)) {   // pcols: a multiple of SPAN
        const SpanSpec sp = span_spec(dt);
        TileLayout L{};
        L.rows = rows;
        L.pcols = pcols;
        L.kc = SPAN_KC;
        L.nct = (pcols + SPAN_KC - 1) / SPAN_KC;
        L.nrb = (rows + TILE_ROWS - 1) / TILE_ROWS;
        const uint32_t nl_last = (pcols - (L.nct - 1) * SPAN_KC) / SPAN;
        for (int p = 0; p < 4; ++p) {
            const uint32_t bps = p < sp.n ? (uint32_t)sp.bps[p] : 0u;
            L.tp_full[p] = round16(bps * SPAN_LANES);
            L.tp_last[p] = round16(bps * nl_last);
            L.rb_bytes[p] = (uint64_t)TILE_ROWS * ((uint64_t)(L.nct - 1) * L.tp_full[p] + L.tp_last[p]);
        }
        return L;
    }
    const PlaneSpec s = plane_spec(dt);
    const uint32_t bs = (uint32_t)block_size_of(dt);
    TileLayout L{};
    L.rows = rows;
    L.pcols = pcols;
    const uint32_t kmax = 128u * (uint32_t)s.chunk_elems;
    L.kc = pcols < kmax ? pcols : kmax;
    L.nct = (pcols + L.kc - 1) / L.kc;
    L.nrb = (rows + TILE_ROWS - 1) / TILE_ROWS;
    const uint32_t last = pcols - (L.nct - 1) * L.kc;
    for (int p = 0; p < 4; ++p) {
        const uint32_t bpb = p < s.n ? (uint32_t)s.bpb[p] : 0u;
        L.tp_full[p] = round16(L.kc / bs * bpb);
        L.tp_last[p] = round16(last / bs * bpb);
        L.rb_bytes[p] = (uint64_t)TILE_ROWS * ((uint64_t)(L.nct - 1) * L.tp_full[p] + L.tp_last[p]);
    }
    return L;
}

// Byte offset of tile (rb, ct) inside plane p.
__host__ __device__ inline uint64_t tile_offset(const TileLayout& L, int p, uint32_t rb, uint32_t ct) {
    return (uint64_t)rb * L.rb_bytes[p] + (uint64_t)TILE_ROWS * L.tp_full[p] * ct;
}
__host__ __device__ inline uint32_t tile_pitch(const TileLayout& L, int p, uint32_t ct) {
    return ct + 1 == L.nct ? L.tp_last[p] : L.tp_full[p];
}

// A tiled weight on the device.
struct QMat {
    const uint8_t* p[4];
    TileLayout L;
};

// A view of one tile (in shared memory): plane bases and row pitches.
struct TileView {
    const uint8_t* p[4];
    uint32_t pitch[4];
};

// Host: split `rows` raw GGUF rows into tiled planes (the span layout for the
// span formats).  `row_src[r]` names the raw row that becomes row r (NULL =
// identity).  planes[p] must hold L.nrb * L.rb_bytes[p] zeroed bytes.
void repack_rows_host(int dt, const uint8_t* raw, uint64_t rows, uint64_t cols, const uint32_t* row_src,
                      const TileLayout& L, uint8_t* const planes[4], int nthreads);

}  // namespace ggc
