// noalloc.cuh -- split-K matvec over raw GGUF blocks whose scratch is a
// file-scope device array, for ggc_quant_matvec_static (no allocation at all).
//
// The row-parallel k_matvec_raw gives each output row to one warp, so a matrix
// with few rows and long rows (e.g. 64 x 65536) occupies a handful of SMs.  This
// variant also splits the columns: CTA (g, s) computes the partial dot products of
// the 8 rows of row group g over block range s, stores them in the static scratch,
// and the last CTA of the group to finish (an atomic ticket per row group) sums
// the `nsplit` partials in split order and writes y.
//
// Scratch (g_noalloc_scratch, NOALLOC_SCRATCH_BYTES = 4 MiB + 32 KiB):
//   tickets   NOALLOC_MAX_GROUPS u32 -- must be zero when a call starts; the
//             entry clears the ones it uses on the caller's stream before the
//             launch, and the last CTA of each group resets its ticket to zero;
//   partials  NOALLOC_MAX_PARTIALS f32 -- [split][row], written before read within
//             one call, no initial value needed.
// One scratch per device: calls that overlap on the device (two streams, two host
// threads) race on it and give wrong results.
#pragma once
#include "common.cuh"
#include "dequant.cuh"

namespace ggc {

constexpr int NOALLOC_ROWS_PER_CTA = 8;                               // one warp per row
constexpr uint64_t NOALLOC_MAX_ROWS = 65536;
constexpr uint32_t NOALLOC_MAX_GROUPS = NOALLOC_MAX_ROWS / NOALLOC_ROWS_PER_CTA;
constexpr uint64_t NOALLOC_MAX_PARTIALS = 1u << 20;                   // 4 MiB of f32
constexpr uint32_t NOALLOC_MAX_SPLIT = 32;
constexpr size_t NOALLOC_TICKET_BYTES = NOALLOC_MAX_GROUPS * sizeof(uint32_t);
constexpr size_t NOALLOC_SCRATCH_BYTES = NOALLOC_TICKET_BYTES + NOALLOC_MAX_PARTIALS * sizeof(float);
static_assert(NOALLOC_MAX_PARTIALS >= NOALLOC_MAX_ROWS * 16, "every admissible row count gets >= 16 splits");

static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

template <int DT>
__global__ void __launch_bounds__(256) k_matvec_raw_splitk(const uint8_t* __restrict__ w, uint64_t rows,
                                                           uint64_t cols, const float* __restrict__ x,
                                                           float* __restrict__ y, uint32_t nsplit,
                                                           uint64_t blk_per_split, unsigned char* scratch) {
    constexpr int BS = block_size_of(DT), BB = block_bytes_of(DT);
    uint32_t* tickets = reinterpret_cast<uint32_t*>(scratch);
    float* part = reinterpret_cast<float*>(scratch + NOALLOC_TICKET_BYTES);
    __shared__ uint32_t last;
    const int lane = threadIdx.x & 31;
    const uint64_t r = (uint64_t)blockIdx.x * NOALLOC_ROWS_PER_CTA + (threadIdx.x >> 5);
    const uint64_t nblk = cols / BS, row_bytes = nblk * BB;
    const uint64_t b0 = (uint64_t)blockIdx.y * blk_per_split;
    const uint64_t b1 = b0 + blk_per_split < nblk ? b0 + blk_per_split : nblk;
    if (r < rows) {
        const uint8_t* row = w + r * row_bytes;
        float acc = 0.0f;
        for (uint64_t b = b0 + lane; b < b1; b += 32) {
            const uint8_t* blk = row + b * BB;
            const float* xb = x + b * BS;
#pragma unroll 4
            for (int e = 0; e < BS; ++e) acc = __fadd_rn(acc, __fmul_rn(deq_elem<DT>(blk, e), xb[e]));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) part[(uint64_t)blockIdx.y * rows + r] = acc;
    }
    // publish the partials, then take a ticket; the last CTA of the group combines
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(&tickets[blockIdx.x], 1u) == nsplit - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (r < rows && lane == 0) {
        float s = 0.0f;
        for (uint32_t k = 0; k < nsplit; ++k) s += __ldcg(&part[(uint64_t)k * rows + r]);
        y[r] = s;
    }
    if (threadIdx.x == 0) tickets[blockIdx.x] = 0;
}

}  // namespace ggc
