// allreduce.cuh -- the tensor-parallel all-reduce of a row-parallel GEMV
// (attn_output, ffn_down) fused into the GEMV itself over peer memory: NVLink
// stores and loads between the ranks' GPUs, no collective library call and no
// memory fence.
//
//  * The epilogue (EPI_AR) sends each partial output row to every rank as one
//    64-bit word, (epoch << 32) | f32 bits, stored into this rank's slot of the
//    receiver's buffer, buf[p][phase][rank][row].  A 64-bit aligned store is
//    single-copy atomic, so a reader that sees the epoch sees the value with it
//    (the low-latency protocol of collective libraries): no flag, no fence.
//    Rank 0's partial includes the residual (the hidden state), the others' not.
//  * After its last tile every consumer warp sums a fixed share of its CTA's rows:
//    for each row it polls the ranks' words in rank order until each carries this
//    all-reduce's epoch (bounded by AR_WAIT_LIMIT polls, then ERRF_TIMEOUT) and
//    adds them in that order.  Every rank computes the same sums in the same
//    order, so the ranks' hidden states stay bit-identical, and the NaN guard of
//    the residual (llama.rs:300-307) runs on the sum.
//  * epoch = step * per_step + k (k = 1-based index of the all-reduce inside a
//    step; the step counter advances on every replay of the step on every rank).
//    Two phases alternate (attn_output, ffn_down): a rank writes a phase's slots
//    again only after every rank has read them, because that next write depends
//    on the other ranks' partials of the phase in between.
//
// The ranks run on distinct GPUs (the host checks device UUIDs and processes), so
// the waits of one rank's kernel on another's never share a GPU.
#pragma once
#include "common.cuh"
#include "planes.cuh"

namespace ggc {

constexpr int AR_MAX_WORLD = 8;
constexpr uint32_t AR_WAIT_LIMIT = 1u << 22;   // polls of one word (~0.5 s with the back-off) before ERRF_TIMEOUT

struct ArGroup {
    unsigned long long* buf[AR_MAX_WORLD];   // rank p's receive words: [2 phases][world][stride]
    int world, rank;
    uint32_t stride;                         // words per (phase, rank) slot (>= rows)
    const uint32_t* step;                    // decode-step counter (device)
    uint32_t per_step;                       // all-reduces per step
};

__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint32_t ar_epoch(const ArGroup& g, uint32_t k) { return *g.step * g.per_step + k; }

// EPI_AR epilogue for `nvalid` rows from r0: tagged partials (+ residual on rank 0) to every rank.
__device__ __forceinline__ void ar_store_rows(const ArGroup& g, uint32_t k, const float* resid, uint32_t r0,
                                              uint32_t nvalid, const float* acc) {
    const uint32_t ph = (k - 1u) & 1u;
    const unsigned long long tag = (unsigned long long)ar_epoch(g, k) << 32;
    const size_t off = ((size_t)ph * g.world + g.rank) * g.stride + r0;
    for (uint32_t r = 0; r < nvalid; ++r) {
        const float v = g.rank == 0 ? __fadd_rn(resid[r0 + r], acc[r]) : acc[r];
        const unsigned long long w = tag | __float_as_uint(v);
        for (int p = 0; p < g.world; ++p) st_relaxed_sys_u64(g.buf[p] + off + r, w);
    }
}

// Sum of the ranks' partials of one row, in rank order, into out[row].
// The world's words are loaded together (one memory round trip, not one per
// rank) and only the ones still missing are polled again.  Returns false when a
// word did not arrive within the poll limit.
__device__ __forceinline__ bool ar_reduce_row(const ArGroup& g, uint32_t ph, uint32_t epoch, uint32_t row, float* out,
                                              const int* errf, bool* nan) {
    const unsigned long long* b = g.buf[g.rank] + (size_t)ph * g.world * g.stride + row;
    unsigned long long w[AR_MAX_WORLD];
    uint32_t missing = (1u << g.world) - 1u;
    for (uint32_t it = 0;; ++it) {
#pragma unroll
        for (int r = 0; r < AR_MAX_WORLD; ++r)
            if ((missing >> r) & 1u) w[r] = ld_relaxed_sys_u64(b + (size_t)r * g.stride);
#pragma unroll
        for (int r = 0; r < AR_MAX_WORLD; ++r)
            if (((missing >> r) & 1u) && (uint32_t)(w[r] >> 32) == epoch) missing &= ~(1u << r);
        if (!missing) break;
        if (it >= AR_WAIT_LIMIT || ((it & 1023u) == 1023u && *(volatile const int*)&errf[ERRF_TIMEOUT])) return false;
        __nanosleep(it < 64 ? 20 : 100);
    }
    float v = 0.f;
#pragma unroll
    for (int r = 0; r < AR_MAX_WORLD; ++r) {
        if (r < g.world) {
            const float x = __uint_as_float((uint32_t)w[r]);
            v = r == 0 ? x : __fadd_rn(v, x);
        }
    }
    out[row] = v;
    *nan |= isnan(v);
    return true;
}

// Called by every lane of a consumer warp after its last tile: sums the rows
// row_of(j), j < count, that lie below `rows`, into out.  NaN -> errf[err_slot] =
// err_val (first wins).
template <class RowOf>
__device__ __forceinline__ void ar_reduce_rows(const ArGroup* gp, uint32_t k, uint32_t count, RowOf row_of,
                                               uint32_t rows, float* out, int* errf, int err_slot, int err_val) {
    const ArGroup& g = *gp;
    const uint32_t ph = (k - 1u) & 1u, epoch = ar_epoch(g, k);
    bool ok = true, nan = false;
    for (uint32_t j = threadIdx.x & 31; j < count && ok; j += 32) {
        const uint32_t row = row_of(j);
        if (row < rows) ok = ar_reduce_row(g, ph, epoch, row, out, errf, &nan);
    }
    const unsigned bad = __ballot_sync(0xffffffffu, !ok), nans = __ballot_sync(0xffffffffu, nan);
    if ((threadIdx.x & 31) == 0) {
        if (bad) atomicMax(&errf[ERRF_TIMEOUT], 1);
        if (nans && err_val) atomicCAS(&errf[err_slot], 0, err_val);
    }
}

// One fused all-reduce step of a world-2 group run on a single GPU (the probe of
// ggc_allreduce_probe): this rank's partial words are stored by the kernel, the
// peer's too when peer_writes, else never, so the bounded poll must give up.
// One warp: ar_reduce_rows strides a row list over the lanes of a warp.
__global__ void k_ar_probe(const ArGroup* g, uint32_t rows, const float* part0, const float* part1, int peer_writes,
                           float* out, int* errf) {
    const uint32_t k = 1u, ph = 0u;
    const unsigned long long tag = (unsigned long long)ar_epoch(*g, k) << 32;
    for (uint32_t r = threadIdx.x; r < rows; r += 32) {
        st_relaxed_sys_u64(g->buf[0] + ((size_t)ph * g->world + 0) * g->stride + r, tag | __float_as_uint(part0[r]));
        if (peer_writes)
            st_relaxed_sys_u64(g->buf[0] + ((size_t)ph * g->world + 1) * g->stride + r, tag | __float_as_uint(part1[r]));
    }
    __syncwarp();
    ar_reduce_rows(g, k, rows, [](uint32_t j) { return j; }, rows, out, errf, ERRF_NAN_ATTN, 0);
}

}  // namespace ggc
