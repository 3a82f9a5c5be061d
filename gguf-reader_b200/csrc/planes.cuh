// planes.cuh -- the coalesced "plane" layout of uploaded weight tensors.
//
// A raw GGUF tensor stores each block's scale fields and quant bits together
// (e.g. Q4_K: d, dmin, scales[12], qs[128] = 144 bytes).  At upload the host
// splits every block into up to four planes, each a row-major array with a row
// pitch padded to 16 bytes:
//
//   plane 0  the quant payload (qs / ql), always a multiple of 16 bytes per block,
//            read by the GEMV as one 16-byte "chunk" per lane, coalesced across
//            the warp (32 lanes x 16 B = 512 contiguous bytes);
//   plane 1+ the per-block side data (scales, d, dmin, high bits).
//
// The split is a lossless byte permutation, except that bytes the reference's
// dequantiser never reads are dropped (Q3_K_M's 4 bytes at 108..111, Q5_K's
// qh[16..32), Q8_K's bsums).  High-bit fields (Q5_0/Q5_1/Q5_K qh, Q3_K hmask)
// are bit-permuted so that the four bits a lane needs for four consecutive
// bytes sit at bit k of byte k of one 32-bit word (one shift + one mask).
#pragma once
#include "common.cuh"

namespace ggc {

struct PlaneSpec {
    int n;          // number of planes
    int bpb[4];     // bytes per block in each plane
    int chunk_elems;// elements covered by one 16-byte chunk of plane 0
};

__host__ __device__ constexpr PlaneSpec plane_spec(int dt) {
    return dt == GGC_Q4_0 ? PlaneSpec{2, {16, 2, 0, 0}, 32}
         : dt == GGC_Q4_1 ? PlaneSpec{2, {16, 4, 0, 0}, 32}
         : dt == GGC_Q5_0 ? PlaneSpec{3, {16, 4, 2, 0}, 32}
         : dt == GGC_Q5_1 ? PlaneSpec{3, {16, 4, 4, 0}, 32}
         : dt == GGC_Q8_0 ? PlaneSpec{2, {32, 2, 0, 0}, 16}
         : dt == GGC_Q2_K ? PlaneSpec{3, {64, 16, 4, 0}, 64}
         : (dt == GGC_Q3_K_S || dt == GGC_Q3_K_M || dt == GGC_Q3_K_L) ? PlaneSpec{4, {64, 32, 12, 2}, 64}
         : dt == GGC_Q4_K ? PlaneSpec{2, {128, 16, 0, 0}, 32}
         : dt == GGC_Q5_K ? PlaneSpec{3, {128, 16, 16, 0}, 32}
         : dt == GGC_Q6_K ? PlaneSpec{4, {128, 64, 16, 2}, 32}
         : dt == GGC_Q8_K ? PlaneSpec{2, {256, 4, 0, 0}, 16}
         : dt == GGC_F16 ? PlaneSpec{1, {2, 0, 0, 0}, 8}
         : dt == GGC_BF16 ? PlaneSpec{1, {2, 0, 0, 0}, 8}
         : dt == GGC_F32 ? PlaneSpec{1, {4, 0, 0, 0}, 4}
         : PlaneSpec{0, {0, 0, 0, 0}, 0};
}

// A repacked 2-D weight: `rows` x `cols`, blocks along cols.
struct QMat {
    const uint8_t* p[4];
    uint32_t pitch[4];
    uint32_t rows, cols;
};

// Bytes of one row in plane p, padded to 16.
inline uint64_t plane_pitch(int dt, int p, uint64_t cols) {
    PlaneSpec s = plane_spec(dt);
    uint64_t nb = cols / (uint64_t)block_size_of(dt);
    uint64_t b = nb * (uint64_t)s.bpb[p];
    return (b + 15) / 16 * 16;
}

// Host: split `rows` raw rows into planes.  `row_src[r]` names the raw row that
// becomes plane row r (NULL = identity).  Plane buffers must hold rows*pitch.
void repack_rows_host(int dt, const uint8_t* raw, uint64_t rows, uint64_t cols, const uint32_t* row_src,
                      uint8_t* const planes[4], int nthreads);

}  // namespace ggc
