// chain.cuh -- a run of decode GEMVs (one layer's attn_output, fused up/gate and
// ffn_down, then the next layer's q/k/v or the output head) in ONE persistent
// launch over the span-layout formats.
//
// Why.  A decode GEMV streams 4-50 MB; at ~6.5 TB/s that is 1.5-8 us, the same
// order as what a separate launch loses to its start, to waiting for its
// predecessor's slowest CTA and to its x prologue.  Here one CTA per SM runs
// every op of the chain: its producer warp streams the weight tiles of ALL the
// ops it will consume, in order, into one shared-memory ring, never waiting on
// data (weights do not depend on activations), so HBM stays busy while the
// consumers wait for an op's input, convert x and run the epilogues.
//
// Block.  4 consumer warps + 1 producer warp.  A consumer warp owns 4 adjacent
// rows of every 16-row tile (RoPE and SwiGLU row pairs stay in one warp), so it
// loads a column tile's x limbs into registers once for 4 rows and keeps 4
// independent dp4a chains in flight.  With 5 warps no SM sub-partition holds more
// than 2 of them, so a thread may use up to 255 registers (a 9-warp block puts 3
// warps on one sub-partition and caps a thread at 168, which the 96 limb words
// plus the chain's state exceed).
//
// Ring.  Byte-granular, ring_bytes long, with CH_DESC tile descriptors (a full
// and an empty mbarrier each).  Tile j of the CTA's sequence uses descriptor j %
// CH_DESC; its bytes start at the running offset, wrapped to 0 when the tile
// would cross the end.  Producer and consumers compute the same offsets.  The
// producer issues tile j once its descriptor and its bytes are free (the tiles
// in flight that overlap it have been released, oldest first).
//
// Dependencies.  Op k waits for ops [dep, dep + ndep) of the same chain (none:
// the launch's predecessor, griddepcontrol.wait): a per-op counter that every
// CTA increments after its rows (and, for EPI_AR, its all-reduce) are written,
// release-ordered; op k's consumers acquire it at step * gridDim.x, step being
// the decode-step counter that k_step_begin advances on every replay, so the
// counters are never reset.  Every wait is bounded; on expiry the CTA flags
// ERRF_TIMEOUT, stops computing, still drains every tile its producer issued and
// still counts its ops, so no CTA waits forever.
//
// Formats.  The consumer body switches on the op's format (a uniform branch) among
// the formats of the kernel instance's mask: each chain launches the instance of
// exactly its ops' formats (15 instances), so the instruction cache holds only
// their code.  One body per format, inlined side by side into the op loop of a
// single all-format instance, made the compiler spill and the warps wait on
// instruction fetch.
//
// x.  Per op the consumers convert x into span limbs as k_gemv_span does; for an
// RMSNorm input of up to 4096 elements x and the norm weight are read once into
// registers (one L2 round trip instead of two), the sum of squares and the limbs
// coming from the same registers.  Numerics equal k_gemv_span's.
#pragma once
#include "gemv_span.cuh"

namespace ggc {

constexpr int CH_MAX_OPS = 8;
constexpr int CH_DESC = 8;
constexpr int CH_WARPS = 4;                     // consumer warps
constexpr int CH_THREADS = CH_WARPS * 32 + 32;  // + the producer warp
constexpr int CH_R = TILE_ROWS / CH_WARPS;      // rows per consumer warp and tile
constexpr int CH_RMS_ITEMS = 2;                 // RMSNorm x items held in registers per thread (xcols <= 4096)
constexpr int CH_PLAIN_ITEMS = 4;               // plain x items loaded per batch per thread (8192 columns)
constexpr uint32_t CH_WAIT_LIMIT = 1u << 22;    // polls of a completion counter (~1 s with the back-off)

struct ChainOp {
    GemvArgs a;
    int dt;                  // span dtype of every segment
    int dep, ndep;           // ops [dep, dep + ndep) of the chain this one waits for (ndep 0: the
                             // launch's predecessor, griddepcontrol.wait)
    uint32_t poff[4];        // plane offsets inside a tile slot
    uint32_t slot_bytes;     // bytes a tile takes in the ring (a full column tile, 128-aligned)
    uint32_t part_rows;      // row sums per CTA (the rows of its row blocks)
};

struct ChainArgs {
    const ChainOp* ops;      // device memory
    int nops;
    uint32_t* cnt;           // completion counter per op
    const uint32_t* step;    // decode-step counter
    int* errf;
    uint32_t ring_bytes;
    uint32_t xl_bytes;       // limb region (max over the ops)
    uint32_t part_bytes;     // row-sum region (max over the ops)
};

__device__ __forceinline__ uint32_t ld_acquire_gpu_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_gpu_add(uint32_t* p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Row blocks [rb0, rb1) of an op for this CTA (all segments together).
__device__ __forceinline__ void chain_rows(const GemvArgs& a, uint32_t& rb0, uint32_t& rb1) {
    uint32_t total = 0;
    for (int i = 0; i < a.nseg; ++i) total += a.seg[i].m.L.nrb;
    rb0 = (uint32_t)((uint64_t)total * blockIdx.x / gridDim.x);
    rb1 = (uint32_t)((uint64_t)total * (blockIdx.x + 1) / gridDim.x);
}
__device__ __forceinline__ void chain_locate(const GemvArgs& a, uint32_t g, int& si, uint32_t& rb) {
    si = 0;
    rb = g;
    while (si + 1 < a.nseg && rb >= a.seg[si].m.L.nrb) { rb -= a.seg[si].m.L.nrb; ++si; }
}
__device__ __forceinline__ void chain_locate_s(int nseg, uint32_t g, int& si, uint32_t& rb);

// Offset of the next tile of `size` bytes after `off` (a tile never crosses the ring's end).
__device__ __forceinline__ uint32_t ring_place(uint32_t off, uint32_t size, uint32_t ring) {
    return off + size > ring ? 0u : off;
}

// Formats a kernel instance serves: one bit per span format.  Each chain launches
// the instance of exactly its ops' formats, so the code in the instruction cache
// is only theirs (one instance for all four formats was instruction-fetch bound).
constexpr uint32_t CH_Q4_K = 1u, CH_Q6_K = 2u, CH_Q4_0 = 4u, CH_Q8_0 = 8u;
__host__ __device__ constexpr uint32_t chain_bit(int dt) {
    return dt == GGC_Q4_K ? CH_Q4_K : dt == GGC_Q6_K ? CH_Q6_K : dt == GGC_Q4_0 ? CH_Q4_0 : dt == GGC_Q8_0 ? CH_Q8_0 : 0u;
}
template <int V> struct DtTag { static constexpr int value = V; };
// Calls f(DtTag<DT>) for the op's format among those of the mask M.
template <uint32_t M, class F>
__device__ __forceinline__ void chain_dispatch(int dt, F&& f) {
    if constexpr ((M & CH_Q4_K) != 0) if (dt == GGC_Q4_K) { f(DtTag<GGC_Q4_K>{}); return; }
    if constexpr ((M & CH_Q6_K) != 0) if (dt == GGC_Q6_K) { f(DtTag<GGC_Q6_K>{}); return; }
    if constexpr ((M & CH_Q4_0) != 0) if (dt == GGC_Q4_0) { f(DtTag<GGC_Q4_0>{}); return; }
    if constexpr ((M & CH_Q8_0) != 0) if (dt == GGC_Q8_0) { f(DtTag<GGC_Q8_0>{}); return; }
}

// Per-CTA state of the consumers (shared memory at file scope: addressed without pointers).
__shared__ Seg ch_sseg[3];
__shared__ double ch_red[CH_WARPS];
__shared__ float ch_scale;
__shared__ int ch_flags[4];   // [0] abort (stop computing), [1] the step is done, [2] this op is skipped, [3] no more waits
__shared__ uint32_t ch_target;
extern __shared__ __align__(128) uint8_t ch_smem[];   // [xl | part | full, empty barriers | ring]

__device__ __forceinline__ void chain_locate_s(int nseg, uint32_t g, int& si, uint32_t& rb) {
    si = 0;
    rb = g;
    while (si + 1 < nseg && rb >= ch_sseg[si].m.L.nrb) { rb -= ch_sseg[si].m.L.nrb; ++si; }
}

// ---------------------------------------------------------------- producer --
__device__ void chain_producer(const ChainArgs& c, uint8_t* ring, uint64_t* full, uint64_t* empty) {
    if ((threadIdx.x & 31) != 0) return;
    uint32_t q_off[CH_DESC], q_end[CH_DESC];
    uint32_t j = 0, oldest = 0, head = 0;
    for (int k = 0; k < c.nops; ++k) {
        const ChainOp& op = c.ops[k];
        const GemvArgs& a = op.a;
        uint32_t rb0, rb1;
        chain_rows(a, rb0, rb1);
        const uint32_t nrb = rb1 - rb0, nct = a.seg[0].m.L.nct;
        const SpanSpec SP = span_spec(op.dt);
        for (uint32_t ct = 0; ct < nct; ++ct) {
            int si;
            uint32_t rb;
            chain_locate(a, rb0, si, rb);
            for (uint32_t rbl = 0; rbl < nrb; ++rbl) {
                const uint32_t size = op.slot_bytes;
                const uint32_t off = ring_place(head, size, c.ring_bytes);
                // release the oldest tiles until a descriptor and the bytes are free
                for (;;) {
                    bool ok = j - oldest < (uint32_t)CH_DESC;
                    for (uint32_t i = oldest; ok && i < j; ++i)
                        if (off < q_end[i % CH_DESC] && q_off[i % CH_DESC] < off + size) ok = false;
                    if (ok) break;
                    if (!mbar_wait(&empty[oldest % CH_DESC], (oldest / CH_DESC) & 1u, c.errf))
                        return;   // the consumers stopped releasing: issue nothing more
                    ++oldest;
                }
                const QMat& m = a.seg[si].m;
                uint32_t bytes = 0;
                for (int p = 0; p < SP.n; ++p) bytes += TILE_ROWS * tile_pitch(m.L, p, ct);
                uint64_t* fb = &full[j % CH_DESC];
                mbar_arrive_expect_tx(fb, bytes);
                for (int p = 0; p < SP.n; ++p)
                    bulk_g2s(ring + off + op.poff[p], m.p[p] + tile_offset(m.L, p, rb, ct),
                             TILE_ROWS * tile_pitch(m.L, p, ct), fb);
                q_off[j % CH_DESC] = off;
                q_end[j % CH_DESC] = off + size;
                head = off + size;
                ++j;
                if (++rb == a.seg[si].m.L.nrb) { rb = 0; ++si; }
            }
        }
    }
}

// ---------------------------------------------------------------- consumers --
// Waits (thread 0) for op `dep`'s counter to reach the step's target; false on timeout.
__device__ __forceinline__ bool chain_wait_dep(const ChainArgs& c, int dep, uint32_t target) {
    const uint32_t* p = c.cnt + dep;
    for (uint32_t it = 0; it < CH_WAIT_LIMIT; ++it) {
        if ((int32_t)(ld_acquire_gpu_u32(p) - target) >= 0) return true;
        if ((it & 255u) == 255u && *(volatile const int*)&c.errf[ERRF_TIMEOUT]) return false;
        if (it >= 512) __nanosleep(64);   // spin first: the wait is on the critical path
    }
    atomicExch(&c.errf[ERRF_TIMEOUT], 1);
    return false;
}

// The warp's 4 rows of a tile (rp: plane bases of its first row, pitch: plane row
// pitches) as two pairs; a pair's two integer chains interleave.  Lanes past the
// tile's width (nl) read padding inside the ring slot, which holds a full 32-lane
// tile, and return 0.
template <int DT>
__device__ __forceinline__ void chain_rows4(const uint8_t* const (&rp)[4], const uint32_t (&pitch)[4], int nl, int lane,
                                            const uint32_t* L, float gs, const float* xq, float (&y)[CH_R]) {
    float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
#pragma unroll 1
    for (int h = 0; h < 2; ++h) {
        SpanRow R0, R1;
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            R0.p[p] = rp[p] + (uint32_t)(2 * h) * pitch[p];
            R1.p[p] = R0.p[p] + pitch[p];
        }
        R0.nl = R1.nl = nl;
        const float u0 = SpanFmt<DT>::dot(R0, lane, L, gs, xq);
        const float u1 = SpanFmt<DT>::dot(R1, lane, L, gs, xq);
        if (h == 0) { a0 = u0; a1 = u1; } else { b0 = u0; b1 = u1; }
    }
    const bool live = lane < nl;
    y[0] = live ? a0 : 0.f;
    y[1] = live ? a1 : 0.f;
    y[2] = live ? b0 : 0.f;
    y[3] = live ? b1 : 0.f;
}
template <uint32_t M>
__device__ __forceinline__ void chain_item_store(int dt, const float (&v)[16], uint32_t it, bool live, uint32_t* xl,
                                                 float* xfs) {
    chain_dispatch<M>(dt, [&](auto t) { span_item_store<decltype(t)::value>(v, it, live, xl, xfs); });
}
template <uint32_t M>
__device__ __forceinline__ bool chain_span_prologue(int dt, const SpanX a, uint32_t nct, uint32_t* xl, float* xfs) {
    bool nan = false;
    chain_dispatch<M>(dt, [&](auto t) {
        nan = span_x_prologue<decltype(t)::value, CH_WARPS>(a, nct, xl, xfs, ch_red, &ch_scale);
    });
    return nan;
}

// The 16 x values of item `it` (zeros past the items or xcols), read through L2.
__device__ __forceinline__ void chain_load_item(const SpanX X, uint32_t it, uint32_t items, float (&v)[16]) {
    const uint32_t e0 = (it >> 3) * SPAN + 16 * (it & 7);
    if (it < items && e0 + 16 <= X.xcols) {
        const float4* x4 = reinterpret_cast<const float4*>(X.x + e0);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float4 f = __ldcg(x4 + q);
            v[4 * q] = f.x; v[4 * q + 1] = f.y; v[4 * q + 2] = f.z; v[4 * q + 3] = f.w;
        }
    } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) v[e] = (it < items && e0 + e < X.xcols) ? __ldcg(X.x + e0 + e) : 0.f;
    }
}

// x of an op into the span limbs (xl, xfs); whether the RMSNorm sum of squares is NaN (thread 0).
template <uint32_t M>
__device__ __forceinline__ bool chain_prologue(int dt, const SpanX X, uint32_t nct, uint32_t* xl, float* xfs) {
    constexpr uint32_t CT = CH_WARPS * 32;
    auto cbar = [] { asm volatile("bar.sync 1, %0;" ::"r"(CT) : "memory"); };
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t items = nct * SPAN_LANES * 8;
    if (X.pro == PRO_PLAIN) {
        // the next item's loads are in flight while the current one is converted
        const uint32_t n = (items + CT - 1) / CT;   // the same count on every thread (the converter shuffles)
        float cur[16];
        chain_load_item(X, tid, items, cur);
#pragma unroll 1
        for (uint32_t i = 0; i < n; ++i) {
            const uint32_t it = tid + i * CT;
            float nxt[16];
            chain_load_item(X, it + CT, i + 1 < n ? items : 0u, nxt);
            chain_item_store<M>(dt, cur, it, it < items, xl, xfs);
#pragma unroll
            for (int e = 0; e < 16; ++e) cur[e] = nxt[e];
        }
        cbar();
        return false;
    }
    if (X.pro != PRO_RMSNORM || items > CH_RMS_ITEMS * CT) {
        const bool nan = chain_span_prologue<M>(dt, X, nct, xl, xfs);
        return tid == 0 && nan;
    }
    float xv[CH_RMS_ITEMS][16], wv[CH_RMS_ITEMS][16];   // x and the norm weight: one L2 round trip
    double ss = 0.0;
#pragma unroll
    for (int i = 0; i < CH_RMS_ITEMS; ++i) {
        const uint32_t it = tid + i * CT, e0 = (it >> 3) * SPAN + 16 * (it & 7);
        if (it < items && e0 + 16 <= X.xcols) {
            const float4* x4 = reinterpret_cast<const float4*>(X.x + e0);
            const float4* w4 = reinterpret_cast<const float4*>(X.x2 + e0);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float4 v = __ldcg(x4 + q), w = __ldg(w4 + q);
                xv[i][4 * q] = v.x; xv[i][4 * q + 1] = v.y; xv[i][4 * q + 2] = v.z; xv[i][4 * q + 3] = v.w;
                wv[i][4 * q] = w.x; wv[i][4 * q + 1] = w.y; wv[i][4 * q + 2] = w.z; wv[i][4 * q + 3] = w.w;
            }
        } else {
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                const bool in = it < items && e0 + e < X.xcols;
                xv[i][e] = in ? __ldcg(X.x + e0 + e) : 0.f;
                wv[i][e] = in ? __ldg(X.x2 + e0 + e) : 0.f;
            }
        }
#pragma unroll
        for (int e = 0; e < 16; ++e) ss += (double)xv[i][e] * (double)xv[i][e];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) ch_red[warp] = ss;
    cbar();
    double t = 0.0;
#pragma unroll
    for (int w = 0; w < CH_WARPS; ++w) t += ch_red[w];
    const float scale = (float)sqrt(1.0 / (t / (double)X.xcols + (double)1e-6f));   // ops.rs:262-274
#pragma unroll
    for (int i = 0; i < CH_RMS_ITEMS; ++i) {
        const uint32_t it = tid + i * CT;
        float v[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) v[e] = __fmul_rn(__fmul_rn(xv[i][e], scale), wv[i][e]);   // ops.rs:272
        chain_item_store<M>(dt, v, it, it < items, xl, xfs);
    }
    cbar();
    return tid == 0 && isnan(t);   // NaN in x <=> NaN sum
}

// The consumers' part of op k.  `j` / `head`: the ring position, advanced over
// every tile of the op whether it is computed or only drained.
template <uint32_t M>
__device__ __forceinline__ void chain_consume(const ChainArgs& c, const ChainOp& op, int k, uint32_t& j,
                                              uint32_t& head) {
    const int dt = op.dt;
    constexpr uint32_t CT = CH_WARPS * 32;
    auto cbar = [] { asm volatile("bar.sync 1, %0;" ::"r"(CT) : "memory"); };
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const GemvArgs& a = op.a;
    uint32_t rb0, rb1;
    chain_rows(a, rb0, rb1);
    const uint32_t nrb = rb1 - rb0, nct = a.seg[0].m.L.nct, ntiles = nrb * nct;
    uint32_t* const xl = reinterpret_cast<uint32_t*>(ch_smem);
    float* const xfs = reinterpret_cast<float*>(ch_smem + (size_t)nct * SPAN_LANES * GS_WORDS * 4);
    float* const part = reinterpret_cast<float*>(ch_smem + c.xl_bytes);
    uint64_t* const full = reinterpret_cast<uint64_t*>(ch_smem + c.xl_bytes + c.part_bytes);
    uint64_t* const empty = full + CH_DESC;
    const uint8_t* const ring = ch_smem + c.xl_bytes + c.part_bytes + 128;

    // dependency, skip flags
    if (tid == 0) {
        bool ok = true;
        for (int d = 0; d < op.ndep && ok && !ch_flags[0]; ++d) ok = chain_wait_dep(c, op.dep + d, ch_target);
        if (!ok) ch_flags[0] = 1;
        ch_flags[2] = (a.st_skip && a.st_skip[0] < a.st_skip[1]) ? 1 : 0;
    }
    if (tid < a.nseg) ch_sseg[tid] = a.seg[tid];
    cbar();
    const bool drain = ch_flags[0] || ch_flags[1] || ch_flags[2];
    if (!drain) {
        const bool x_nan = chain_prologue<M>(dt, span_x_of(a), nct, xl, xfs);
        if (x_nan && a.pro_err_val) atomicCAS(&a.errf[a.pro_err_slot], 0, a.pro_err_val);
        for (uint32_t i = tid; i < nrb * TILE_ROWS; i += CT) part[i] = 0.f;
        cbar();
    }

    // ---- tiles ----
    const int r0 = CH_R * warp;   // this warp's rows in every tile
    uint32_t L[GS_WORDS];
    float gs = 0.f;
    const float* xq = nullptr;
    uint32_t rbl = 0, ct = 0;
    int nl = 0;
    uint32_t pitch[4];
    for (uint32_t i = 0; i < ntiles; ++i) {
        const uint32_t off = ring_place(head, op.slot_bytes, c.ring_bytes);
        head = off + op.slot_bytes;
        uint64_t* fb = &full[j % CH_DESC];
        uint64_t* eb = &empty[j % CH_DESC];
        const uint32_t par = (j / CH_DESC) & 1u;
        ++j;
        // a tile that never arrives (the producer gave up) ends all waiting: the
        // CTA still passes every barrier and counts its ops, computing nothing
        if (!*(volatile int*)&ch_flags[3] && !mbar_wait(fb, par, c.errf)) {
            ch_flags[3] = 1;
            ch_flags[0] = 1;
        }
        if (drain || *(volatile int*)&ch_flags[0]) {
            __syncwarp();
            if (lane == 0) mbar_arrive(eb);
            if (++rbl == nrb) { rbl = 0; ++ct; }
            continue;
        }
        if (rbl == 0) {   // a new column tile: this lane's x limbs, the tile geometry
            const TileLayout& L0 = ch_sseg[0].m.L;
            nl = ct + 1 == L0.nct ? (int)((L0.pcols - ct * SPAN_KC) / SPAN) : SPAN_LANES;
#pragma unroll
            for (int p = 0; p < 4; ++p) pitch[p] = tile_pitch(L0, p, ct);
#pragma unroll
            for (int q = 0; q < GS_WORDS / 4; ++q) {
                const uint4 w4 = *reinterpret_cast<const uint4*>(xl + (((size_t)ct * 24 + q) * SPAN_LANES + lane) * 4);
                L[4 * q] = w4.x; L[4 * q + 1] = w4.y; L[4 * q + 2] = w4.z; L[4 * q + 3] = w4.w;
            }
            gs = xfs[(size_t)ct * GS_XF * SPAN_LANES + lane];
            xq = xfs + (size_t)ct * GS_XF * SPAN_LANES + SPAN_LANES + lane * 4;
        }
        const uint8_t* st = ring + off;
        float y[CH_R];
        {
            const uint8_t* rp[4];
#pragma unroll
            for (int p = 0; p < 4; ++p) rp[p] = st + op.poff[p] + (uint32_t)r0 * pitch[p];
            chain_dispatch<M>(dt, [&](auto t) {   // one branch per tile
                chain_rows4<decltype(t)::value>(rp, pitch, nl, lane, L, gs, xq, y);
            });
        }
        // four row sums over the warp: halve the exchange twice (xor 16, xor 8),
        // then reduce inside groups of 8; row q ends in lane 8 q
        {
            const bool h16 = lane & 16, h8 = lane & 8;
            const float a0 = (h16 ? y[2] : y[0]) + __shfl_xor_sync(0xffffffffu, h16 ? y[0] : y[2], 16);
            const float a1 = (h16 ? y[3] : y[1]) + __shfl_xor_sync(0xffffffffu, h16 ? y[1] : y[3], 16);
            float v = (h8 ? a1 : a0) + __shfl_xor_sync(0xffffffffu, h8 ? a0 : a1, 8);
#pragma unroll
            for (int o = 4; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
#pragma unroll
            for (int q = 0; q < CH_R; ++q) y[q] = __shfl_sync(0xffffffffu, v, 8 * q);
        }
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(eb);
            // row sums gathered per row of the CTA (added over the column tiles)
            float* pp = part + rbl * TILE_ROWS + r0;
#pragma unroll
            for (int q = 0; q < CH_R; ++q) pp[q] += y[q];
        }
        if (++rbl == nrb) { rbl = 0; ++ct; }
    }
    if (!drain && !*(volatile int*)&ch_flags[0]) {
        // epilogues of all the CTA's rows at once, a row pair per thread, so their
        // global loads (residual, RoPE position and table, bias) overlap
        cbar();
        unsigned long long best = 0ull;
        bool nan_logit = false;
        for (uint32_t p = tid; p < nrb * (TILE_ROWS / 2); p += CT) {
            int psi;
            uint32_t prb;
            chain_locate_s(a.nseg, rb0 + p / (TILE_ROWS / 2), psi, prb);
            const Seg& sg = ch_sseg[psi];
            const uint32_t row = prb * TILE_ROWS + 2 * (p % (TILE_ROWS / 2));
            if (row >= sg.m.L.rows) continue;
            const uint32_t nv = min(2u, sg.m.L.rows - row);
            const float* yy = part + 2 * p;
            if (sg.epi == EPI_LOGITS) {
                for (uint32_t q = 0; q < nv; ++q) {
                    sg.out[row + q] = yy[q];
                    nan_logit |= isnan(yy[q]);
                    const unsigned long long key = argmax_key_of(yy[q], row + q);
                    best = key > best ? key : best;
                }
            } else {
                gemv_epilogue(a, sg, row, nv, yy);
            }
        }
        if (ch_sseg[0].epi == EPI_LOGITS) {   // one atomic per warp
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
        if (a.ar_k)   // tensor parallel: this warp's rows of each row block, summed over the ranks
            ar_reduce_rows(
                a.ar, a.ar_k, CH_R * nrb,
                [&](uint32_t q) { return (rb0 + q / CH_R) * TILE_ROWS + (uint32_t)r0 + (q % CH_R); },
                ch_sseg[0].m.L.rows, ch_sseg[0].out, a.errf, a.err_slot, a.err_val);
    }
    // this CTA's part of op k is written: count it.  The barrier orders the other
    // consumer threads' writes before thread 0's release, which is cumulative.
    cbar();
    if (tid == 0) red_release_gpu_add(c.cnt + k, 1u);
}

template <uint32_t M>
__global__ void __launch_bounds__(CH_THREADS, 1) k_gemv_chain(const ChainArgs c) {
    uint64_t* const full = reinterpret_cast<uint64_t*>(ch_smem + c.xl_bytes + c.part_bytes);
    uint64_t* const empty = full + CH_DESC;
    const int tid = threadIdx.x, warp = tid >> 5;
    if (tid == 0) {
        for (int d = 0; d < CH_DESC; ++d) {
            mbar_init(&full[d], 1);
            mbar_init(&empty[d], CH_WARPS);
        }
        ch_flags[0] = ch_flags[1] = ch_flags[2] = ch_flags[3] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    pdl_trigger();

    if (warp == CH_WARPS) {
        chain_producer(c, ch_smem + c.xl_bytes + c.part_bytes + 128, full, empty);
        pdl_wait();
        return;
    }
    pdl_wait();
    if (tid == 0) {
        ch_target = *c.step * gridDim.x;
        const int* done = c.ops[0].a.st_done;
        ch_flags[1] = (done && *done) ? 1 : 0;
    }
    asm volatile("bar.sync 1, %0;" ::"r"(CH_WARPS * 32) : "memory");
    uint32_t j = 0, head = 0;
    for (int k = 0; k < c.nops; ++k) chain_consume<M>(c, c.ops[k], k, j, head);
}

// Host: the kernel instance for a set of formats (mask of chain_bit), every
// non-empty subset of the four instantiated.
using ChainKernel = void (*)(const ChainArgs);
template <uint32_t M>
constexpr ChainKernel chain_kernel_of() { return k_gemv_chain<M>; }
inline ChainKernel chain_kernel(uint32_t mask) {
    constexpr ChainKernel tab[16] = {
        nullptr, chain_kernel_of<1>(), chain_kernel_of<2>(), chain_kernel_of<3>(),
        chain_kernel_of<4>(), chain_kernel_of<5>(), chain_kernel_of<6>(), chain_kernel_of<7>(),
        chain_kernel_of<8>(), chain_kernel_of<9>(), chain_kernel_of<10>(), chain_kernel_of<11>(),
        chain_kernel_of<12>(), chain_kernel_of<13>(), chain_kernel_of<14>(), chain_kernel_of<15>()};
    return tab[mask & 15u];
}

}  // namespace ggc
