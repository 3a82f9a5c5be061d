// stream.cuh -- the decode step as one persistent launch over a list of ops.
//
// One CTA per SM (cooperative launch: all CTAs resident) walks the same op list:
//   SOP_GEMV  span-layout GEMV (Q4_K / Q6_K / Q4_0 / Q8_0), rows split over CTAs
//             by contiguous 16-row blocks, with the k_gemv_span prologue,
//             decoders and epilogues;
//   SOP_ATTN  split decode attention (the k_attn_decode algorithm), (kv head,
//             split) items spread over CTAs, last CTA of a head combines.
// A producer warp streams every tile this CTA will consume -- weight tiles of
// all GEMVs, K/V tiles of attention -- through one ring of shared-memory stages
// in consumption order, so the weights of op k+1 load while op k computes.  The
// consumers of op k wait until every CTA has finished op `dep` (a completion
// counter per op, bounded spin); the producer waits on that counter only before
// the K/V tiles of an attention op (they include the row the QKV op writes).
// Data written by other CTAs is read through L2 (ld.cg) or by bulk copy after a
// proxy fence.  Counters are zero between launches: the last CTA to leave
// resets them.  Every wait is bounded (ERRF_TIMEOUT).
#pragma once
#include "common.cuh"
#include "mbarrier.cuh"
#include "gemv.cuh"
#include "gemv_span.cuh"
#include "attention.cuh"

namespace ggc {

enum StreamOpKind : int { SOP_GEMV = 0, SOP_ATTN = 1 };

struct StreamOp {
    int kind;
    int dtype;          // SOP_GEMV
    int dep;            // op whose completion (on every CTA) this op's inputs need; -1: none
    int logits;         // SOP_GEMV: the lm_head (skipped while the step state says so)
    uint32_t poff[4];   // SOP_GEMV: plane offsets inside a stage
    uint32_t part_rows; // SOP_GEMV: partial row sums needed per CTA (multi-tile rows)
    GemvArgs g;         // SOP_GEMV
    AttnArgs at;        // SOP_ATTN
};

struct StreamArgs {
    const StreamOp* ops;
    int n_ops;
    unsigned* done;          // [n_ops + 1]: per-op completion counters + the exit counter
    const int* st_done;      // the decode loop has stopped: the launch does nothing
    const int* st_skip;      // st_skip[0] < st_skip[1]: a prompt token, skip the lm_head
    int* errf;
    unsigned long long* argmax_key;
    uint32_t stage_bytes, stages;
    uint32_t xl_bytes;       // x limbs (GEMV) / scores + cross-warp sums (attention)
    uint32_t part_bytes;
};

constexpr uint32_t STREAM_WAIT_LIMIT = 1u << 22;   // x 64..256 ns sleeps: about a second

// Any expired wait of the grid raises ERRF_TIMEOUT; every wait of the stream
// also gives up as soon as it sees that flag, so one expiry ends the launch
// quickly instead of running every later wait to its own limit.
__device__ __forceinline__ bool stream_aborted(const int* errf) {
    return *reinterpret_cast<const volatile int*>(&errf[ERRF_TIMEOUT]) != 0;
}

// Waits (one thread) until counter >= target; false (ERRF_TIMEOUT) on expiry or abort.
__device__ __forceinline__ bool wait_counter(const unsigned* c, unsigned target, int* errf) {
    unsigned ns = 32;
    for (uint32_t i = 0; i < STREAM_WAIT_LIMIT; ++i) {
        unsigned v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(c) : "memory");
        if (v >= target) return true;
        if (stream_aborted(errf)) return false;
        __nanosleep(ns);
        if (ns < 256) ns <<= 1;
    }
    atomicExch(&errf[ERRF_TIMEOUT], 1);
    return false;
}

// Bounded mbarrier wait that also stops on a grid-wide abort.
__device__ __forceinline__ bool stream_mbar_wait(uint64_t* bar, uint32_t parity, int* errf) {
    for (uint32_t i = 0; i < BULK_WAIT_LIMIT; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (stream_aborted(errf)) return false;
    }
    atomicExch(&errf[ERRF_TIMEOUT], 1);
    return false;
}

__device__ __forceinline__ void stream_range(uint32_t total, uint32_t& b0, uint32_t& b1) {
    b0 = (uint32_t)((uint64_t)total * blockIdx.x / gridDim.x);
    b1 = (uint32_t)((uint64_t)total * (blockIdx.x + 1) / gridDim.x);
}

// ring position shared by the producer's and the consumers' walk over tiles
struct Ring {
    uint32_t s, ph;
    __device__ void advance(uint32_t n) { if (++s == n) { s = 0; ph ^= 1u; } }
};

// ---- GEMV ops ----------------------------------------------------------------
__device__ __forceinline__ uint32_t gemv_total_rb(const GemvArgs& g) {
    uint32_t t = 0;
    for (int i = 0; i < g.nseg; ++i) t += g.seg[i].m.L.nrb;
    return t;
}
__device__ __forceinline__ void gemv_locate(const GemvArgs& g, uint32_t rbg, int& si, uint32_t& rb) {
    si = 0;
    rb = rbg;
    while (si + 1 < g.nseg && rb >= g.seg[si].m.L.nrb) { rb -= g.seg[si].m.L.nrb; ++si; }
}

// producer: issue this CTA's tiles of one GEMV (column-tile-major)
static __device__ void stream_gemv_produce(const StreamOp& op, const StreamArgs& P, uint64_t* full, uint64_t* empty,
                                    uint8_t* stages, Ring& r, uint32_t& issued, int lane) {
    const GemvArgs& g = op.g;
    uint32_t rb0, rb1;
    stream_range(gemv_total_rb(g), rb0, rb1);
    const uint32_t nrb = rb1 - rb0, nct = g.seg[0].m.L.nct;
    const SpanSpec SP = span_spec(op.dtype);
    for (uint32_t ct = 0; ct < nct && nrb; ++ct) {
        int si; uint32_t rb;
        gemv_locate(g, rb0, si, rb);
        for (uint32_t k = 0; k < nrb; ++k) {
            if (issued >= P.stages) stream_mbar_wait(&empty[r.s], r.ph, P.errf);   // on abort: issue anyway (in bounds)
            if (lane == 0) {
                const QMat& m = g.seg[si].m;
                uint32_t bytes = 0;
                for (int p = 0; p < SP.n; ++p) bytes += TILE_ROWS * tile_pitch(m.L, p, ct);
                mbar_arrive_expect_tx(&full[r.s], bytes);
                uint8_t* st = stages + (size_t)r.s * P.stage_bytes;
                for (int p = 0; p < SP.n; ++p)
                    bulk_g2s(st + op.poff[p], m.p[p] + tile_offset(m.L, p, rb, ct), TILE_ROWS * tile_pitch(m.L, p, ct),
                             &full[r.s]);
            }
            __syncwarp();
            r.advance(P.stages);
            ++issued;
            if (++rb == g.seg[si].m.L.nrb) { rb = 0; ++si; }
        }
    }
}

// one copy of the epilogues for every format path (called by one lane per row pair)
static __device__ __noinline__ void stream_epilogue(const GemvArgs& g, const Seg& sg, uint32_t row, uint32_t nv,
                                                    float y0, float y1) {
    const float y[2] = {y0, y1};
    if (sg.epi == EPI_RESID) {   // hidden (written by other CTAs) through L2
        bool nan = false;
        for (uint32_t k = 0; k < nv; ++k) {
            nan |= isnan(y[k]);
            sg.out[row + k] = __fadd_rn(__ldcg(sg.out + row + k), y[k]);
        }
        if (nan) atomicCAS(&g.errf[g.err_slot], 0, g.err_val);
    } else {
        gemv_epilogue(g, sg, row, nv, y);
    }
}

// consumers: this CTA's rows of one GEMV; false on an expired wait
template <int DT>
__device__ __noinline__ bool stream_gemv_consume(const StreamOp& op, const StreamArgs& P, uint8_t* smem, uint64_t* full,
                                    uint64_t* empty, uint8_t* stages, Ring& r, double* red, float* s_scale) {
    using F = SpanFmt<DT>;
    constexpr uint32_t CT = GS_WARPS * 32;
    const GemvArgs& g = op.g;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint32_t rb0, rb1;
    stream_range(gemv_total_rb(g), rb0, rb1);
    const uint32_t nrb = rb1 - rb0, nct = g.seg[0].m.L.nct;
    uint32_t* xl = reinterpret_cast<uint32_t*>(smem);
    float* xfs = reinterpret_cast<float*>(smem + (size_t)nct * SPAN_LANES * GS_WORDS * 4);
    float* part = reinterpret_cast<float*>(smem + P.xl_bytes);
    bool ok = true;   // an expired wait is recorded, never taken as a branch: every warp keeps the same barriers
    span_x_prologue<DT>(span_x_of(g), nct, xl, xfs, red, s_scale);   // ends with a consumer barrier
    if (nct > 1) {
        for (uint32_t i = tid; i < nrb * TILE_ROWS; i += CT) part[i] = 0.f;
        asm volatile("bar.sync 1, %0;" ::"r"(CT) : "memory");
    }
    const int r0 = 2 * warp;
    uint32_t L[GS_WORDS];
    float gs = 0.f;
    const float* xq = nullptr;
    unsigned long long best = 0ull;
    bool nan_logit = false;
    const TileLayout& L0 = g.seg[0].m.L;
    for (uint32_t ct = 0; ct < nct && nrb; ++ct) {
        const int nl = ct + 1 == L0.nct ? (int)((L0.pcols - ct * SPAN_KC) / SPAN) : SPAN_LANES;
        uint32_t rowoff[4], pitch[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            pitch[p] = tile_pitch(L0, p, ct);
            rowoff[p] = op.poff[p] + (uint32_t)r0 * pitch[p];
        }
#pragma unroll
        for (int k = 0; k < GS_WORDS / 4; ++k) {
            const uint4 w4 = *reinterpret_cast<const uint4*>(xl + (((size_t)ct * 24 + k) * SPAN_LANES + lane) * 4);
            L[4 * k] = w4.x; L[4 * k + 1] = w4.y; L[4 * k + 2] = w4.z; L[4 * k + 3] = w4.w;
        }
        gs = xfs[(size_t)ct * GS_XF * SPAN_LANES + lane];
        xq = xfs + (size_t)ct * GS_XF * SPAN_LANES + SPAN_LANES + lane * 4;
        int si; uint32_t rb;
        gemv_locate(g, rb0, si, rb);
        for (uint32_t rbl = 0; rbl < nrb; ++rbl) {
            ok &= stream_mbar_wait(&full[r.s], r.ph, P.errf);
            const uint8_t* st = stages + (size_t)r.s * P.stage_bytes;
            float y[2] = {0.f, 0.f};
#pragma unroll 1
            for (int k = 0; k < 2; ++k) {   // one row at a time: the kernel's register budget is 168
                SpanRow R;
#pragma unroll
                for (int p = 0; p < 4; ++p) R.p[p] = st + rowoff[p] + (uint32_t)k * pitch[p];
                R.nl = nl;
                const float v = lane < nl ? F::dot(R, lane, L, gs, xq) : 0.f;
                if (k == 0) y[0] = v; else y[1] = v;
            }
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
            if (lane == 0) mbar_arrive(&empty[r.s]);
            r.advance(P.stages);
            const int tsi = si;
            const uint32_t trb = rb;
            if (++rb == g.seg[si].m.L.nrb) { rb = 0; ++si; }
            const uint32_t nrows = min((uint32_t)TILE_ROWS, g.seg[tsi].m.L.rows - trb * TILE_ROWS);
            if ((uint32_t)r0 >= nrows) continue;
            const uint32_t nv = min(2u, nrows - (uint32_t)r0);
            if (nct > 1) {
                float* pp = part + rbl * TILE_ROWS + r0;
                if (ct + 1 < nct) {
                    if (lane == 0) { pp[0] += y[0]; pp[1] += y[1]; }
                    continue;
                }
                y[0] += pp[0];
                y[1] += pp[1];
            }
            if (lane == 0) {
                const Seg& sg = g.seg[tsi];
                const uint32_t row = trb * TILE_ROWS + (uint32_t)r0;
                if (sg.epi == EPI_LOGITS) {
                    for (uint32_t k = 0; k < nv; ++k) {
                        sg.out[row + k] = y[k];
                        nan_logit |= isnan(y[k]);
                        const unsigned long long key = argmax_key_of(y[k], row + k);
                        best = key > best ? key : best;
                    }
                } else {
                    stream_epilogue(g, sg, row, nv, y[0], y[1]);
                }
            }
        }
    }
    if (lane == 0 && (best || nan_logit)) {
        if (nan_logit) atomicMax(&P.errf[ERRF_NAN_LOGITS], 1);
        atomicMax(P.argmax_key, best);
    }
    return ok;
}

// ---- attention ops ---------------------------------------------------------------
template <int HD, bool F16, int MAXG>
struct StreamAttn {
    using C = FaCfg<HD, F16, MAXG>;
    static constexpr int TR = C::TR;
    static constexpr uint32_t TB = C::TILE_BYTES;

    __device__ static uint32_t items(const AttnArgs& a) { return a.kvh * a.nsplit; }

    // producer: K and V tiles of this CTA's items (after the QKV op finished everywhere)
    __device__ static void produce(const StreamOp& op, const StreamArgs& P, uint64_t* full, uint64_t* empty,
                                   uint8_t* stages, Ring& r, uint32_t& issued, int lane) {
        const AttnArgs& a = op.at;
        if (lane == 0 && op.dep >= 0) {
            wait_counter(&P.done[op.dep], gridDim.x, P.errf);   // on expiry the tiles are still issued (in bounds)
            asm volatile("fence.proxy.async.global;" ::: "memory");
        }
        __syncwarp();
        uint32_t i0, i1;
        stream_range(items(a), i0, i1);
        for (uint32_t it = i0; it < i1; ++it) {
            const uint32_t kvhead = it / a.nsplit, split = it % a.nsplit;
            uint32_t s0, s1, visible;
            attn_range(a, split, s0, s1, visible);
            const uint32_t n = s1 - s0, nt = (n + TR - 1) / TR;
            const uint8_t* kg = reinterpret_cast<const uint8_t*>(a.kc) + ((uint64_t)kvhead * a.max_ctx + s0) * C::ROWB;
            const uint8_t* vg = reinterpret_cast<const uint8_t*>(a.vc) + ((uint64_t)kvhead * a.max_ctx + s0) * C::ROWB;
            for (uint32_t t = 0; t < nt; ++t) {
                if (issued >= P.stages) stream_mbar_wait(&empty[r.s], r.ph, P.errf);
                if (lane == 0) {
                    const uint32_t rows = min((uint32_t)TR, n - t * TR), bytes = rows * C::ROWB;
                    uint8_t* st = stages + (size_t)r.s * P.stage_bytes;
                    mbar_arrive_expect_tx(&full[r.s], 2 * bytes);
                    bulk_g2s(st, kg + (uint64_t)t * TB, bytes, &full[r.s]);
                    bulk_g2s(st + TB, vg + (uint64_t)t * TB, bytes, &full[r.s]);
                }
                __syncwarp();
                r.advance(P.stages);
                ++issued;
            }
        }
    }

    // consumers: every item of this CTA (scores, online softmax, V sum, split
    // partials, last-CTA combine); false on an expired wait
    __device__ __noinline__ static bool consume(const StreamOp& op, const StreamArgs& P, uint8_t* smem, uint64_t* full,
                                   uint64_t* empty, uint8_t* stages, Ring& r, float* s_fin, bool* s_last) {
        using IsF16 = std::integral_constant<bool, F16>;
        constexpr int LPR = C::LPR, GPL = C::GPL, RPW = C::RPW, WR = C::WR, U = C::U, RL = C::RL;
        constexpr int NV = C::NV, CF = C::CF;
        constexpr uint32_t CT = GS_WARPS * 32;
        auto cbar = [] { asm volatile("bar.sync 1, %0;" ::"r"(CT) : "memory"); };
        const AttnArgs& a = op.at;
        const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
        const int sub = lane / LPR, gl = lane % LPR;
        float* ssc = reinterpret_cast<float*>(smem);                         // [TR][MAXG]
        float* sred = reinterpret_cast<float*>(smem) + TR * MAXG;            // [warps][MAXG][HD]
        const uint32_t G = a.n_heads / a.kvh;
        uint32_t i0, i1;
        stream_range(items(a), i0, i1);
        bool ok = true;   // recorded, never branched on (see stream_gemv_consume)
        for (uint32_t it = i0; it < i1; ++it) {
            const uint32_t kvhead = it / a.nsplit, split = it % a.nsplit, h0 = kvhead * G;
            uint32_t s0, s1, visible;
            attn_range(a, split, s0, s1, visible);
            const uint32_t n = s1 - s0, nt = (n + TR - 1) / TR;
            float4 qv[MAXG][GPL];
#pragma unroll
            for (int g = 0; g < MAXG; ++g)
#pragma unroll
                for (int j = 0; j < GPL; ++j)
                    qv[g][j] = g < (int)G ? __ldcg(reinterpret_cast<const float4*>(a.q + (size_t)(h0 + g) * HD + 4 * (gl + j * LPR)))
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
            float m_run[MAXG], l_run[MAXG];
            float4 acc[MAXG][GPL];
#pragma unroll
            for (int g = 0; g < MAXG; ++g) {
                m_run[g] = -INFINITY;
                l_run[g] = 0.f;
#pragma unroll
                for (int j = 0; j < GPL; ++j) acc[g][j] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
            for (uint32_t t = 0; t < nt; ++t) {
                ok &= stream_mbar_wait(&full[r.s], r.ph, P.errf);
                const uint8_t* kt = stages + (size_t)r.s * P.stage_bytes;
                const uint8_t* vt = kt + TB;
                {
                    float v[NV];
#pragma unroll
                    for (int u = 0; u < U; ++u) {
                        const int row = warp * WR + u * RPW + sub;
                        float4 kq[GPL];
#pragma unroll
                        for (int j = 0; j < GPL; ++j) kq[j] = fa_ld(kt + row * C::ROWB + (gl + j * LPR) * C::GB, IsF16{});
#pragma unroll
                        for (int g = 0; g < MAXG; ++g) {
                            float d = 0.f;
#pragma unroll
                            for (int j = 0; j < GPL; ++j) d = dot4(qv[g][j], kq[j], d);
                            v[u * MAXG + g] = d;
                        }
                    }
                    int base = 0;
                    fa_butterfly<NV, LPR / 2>(v, gl, base);
#pragma unroll
                    for (int i = 0; i < CF; ++i) {
                        const int idx = base + i, u = idx / MAXG, g = idx % MAXG;
                        ssc[(warp * WR + u * RPW + sub) * MAXG + g] = __fmul_rn(v[i], a.inv);
                    }
                }
                cbar();
                const uint32_t valid = min((uint32_t)TR, n - t * TR);
                float p[RL][MAXG];
#pragma unroll
                for (int g = 0; g < MAXG; ++g) {
                    float mt = -INFINITY;
#pragma unroll
                    for (int k = 0; k < RL; ++k) {
                        const uint32_t row = (uint32_t)(lane + 32 * k);
                        p[k][g] = row < valid ? ssc[row * MAXG + g] : -INFINITY;
                        mt = fmaxf(mt, p[k][g]);
                    }
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o));
                    const float mn = fmaxf(m_run[g], mt);
                    const float alpha = mn == -INFINITY ? 1.f : expf(m_run[g] - mn);
                    float ps = 0.f;
#pragma unroll
                    for (int k = 0; k < RL; ++k) {
                        p[k][g] = mn == -INFINITY ? 0.f : expf(p[k][g] - mn);
                        ps += p[k][g];
                    }
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
                    l_run[g] = l_run[g] * alpha + ps;
                    m_run[g] = mn;
#pragma unroll
                    for (int j = 0; j < GPL; ++j) {
                        acc[g][j].x *= alpha; acc[g][j].y *= alpha; acc[g][j].z *= alpha; acc[g][j].w *= alpha;
                    }
                }
                const int kk = (warp * WR) / 32;
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int row = warp * WR + u * RPW + sub;
                    const bool rv = (uint32_t)row < valid;
                    float4 vq[GPL];
#pragma unroll
                    for (int j = 0; j < GPL; ++j) {
                        vq[j] = fa_ld(vt + row * C::ROWB + (gl + j * LPR) * C::GB, IsF16{});
                        if (!rv) vq[j] = make_float4(0.f, 0.f, 0.f, 0.f);
                    }
#pragma unroll
                    for (int g = 0; g < MAXG; ++g) {
                        float src = p[0][g];
#pragma unroll
                        for (int k = 1; k < RL; ++k) src = kk == k ? p[k][g] : src;
                        const float w = __shfl_sync(0xffffffffu, src, row & 31);
#pragma unroll
                        for (int j = 0; j < GPL; ++j) {
                            acc[g][j].x = fmaf(w, vq[j].x, acc[g][j].x);
                            acc[g][j].y = fmaf(w, vq[j].y, acc[g][j].y);
                            acc[g][j].z = fmaf(w, vq[j].z, acc[g][j].z);
                            acc[g][j].w = fmaf(w, vq[j].w, acc[g][j].w);
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[r.s]);
                r.advance(P.stages);
                cbar();   // the score tile is free
            }
            // item partial: rows of a warp pass, then warps in fixed order
#pragma unroll
            for (int o = 16; o >= LPR; o >>= 1)
#pragma unroll
                for (int g = 0; g < MAXG; ++g)
#pragma unroll
                    for (int j = 0; j < GPL; ++j) {
                        acc[g][j].x += __shfl_xor_sync(0xffffffffu, acc[g][j].x, o);
                        acc[g][j].y += __shfl_xor_sync(0xffffffffu, acc[g][j].y, o);
                        acc[g][j].z += __shfl_xor_sync(0xffffffffu, acc[g][j].z, o);
                        acc[g][j].w += __shfl_xor_sync(0xffffffffu, acc[g][j].w, o);
                    }
            if (sub == 0) {
#pragma unroll
                for (int g = 0; g < MAXG; ++g)
#pragma unroll
                    for (int j = 0; j < GPL; ++j)
                        *reinterpret_cast<float4*>(sred + ((size_t)warp * MAXG + g) * HD + 4 * (gl + j * LPR)) = acc[g][j];
            }
            cbar();
            for (uint32_t e = tid; e < G * HD; e += CT) {
                const uint32_t g = e / HD, i = e % HD;
                float sum = 0.f;
#pragma unroll
                for (int w = 0; w < GS_WARPS; ++w) sum += sred[((size_t)w * MAXG + g) * HD + i];
                a.opart[((size_t)split * a.n_heads + h0 + g) * HD + i] = sum;
            }
            if (warp == 0) {
#pragma unroll
                for (int g = 0; g < MAXG; ++g)
                    if (lane == g && g < (int)G) {
                        a.pmax[(size_t)split * a.n_heads + h0 + g] = m_run[g];
                        a.psum[(size_t)split * a.n_heads + h0 + g] = l_run[g];
                    }
            }
            __threadfence();
            cbar();
            if (tid == 0) *s_last = atomicAdd(&a.tickets[kvhead], 1u) == a.nsplit - 1;
            cbar();
            if (*s_last) {
                __threadfence();
                if (warp < (int)G) {
                    const uint32_t h = h0 + warp;
                    float M = -INFINITY;
                    for (uint32_t k = lane; k < a.nsplit; k += 32) M = fmaxf(M, __ldcg(&a.pmax[(size_t)k * a.n_heads + h]));
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
                    float S = 0.f;
                    for (uint32_t k = lane; k < a.nsplit; k += 32) {
                        const float mk = __ldcg(&a.pmax[(size_t)k * a.n_heads + h]);
                        if (mk != -INFINITY) S += expf(mk - M) * __ldcg(&a.psum[(size_t)k * a.n_heads + h]);
                    }
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) S += __shfl_xor_sync(0xffffffffu, S, o);
                    if (lane == 0) {
                        s_fin[warp] = M;
                        s_fin[8 + warp] = __fdiv_rn(1.0f, S);
                    }
                }
                cbar();
                for (uint32_t e = tid; e < G * HD; e += CT) {
                    const uint32_t g = e / HD, i = e % HD, h = h0 + g;
                    const float M = s_fin[g];
                    float sum = 0.f;
                    for (uint32_t k = 0; k < a.nsplit; ++k) {
                        const float mk = __ldcg(&a.pmax[(size_t)k * a.n_heads + h]);
                        if (mk != -INFINITY) sum += expf(mk - M) * __ldcg(&a.opart[((size_t)k * a.n_heads + h) * HD + i]);
                    }
                    a.o[(size_t)h * HD + i] = sum * s_fin[8 + g];
                }
                if (tid == 0) a.tickets[kvhead] = 0;
            }
            cbar();   // sred / s_fin / s_last reuse by the next item
        }
        return ok;
    }
};

// ---- the kernel ------------------------------------------------------------------
template <int HD, bool F16, int MAXG>
__global__ void __launch_bounds__(GS_THREADS, 1) k_stream(const StreamArgs P) {
    using A = StreamAttn<HD, F16, MAXG>;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ double red[GS_WARPS];
    __shared__ float s_scale;
    __shared__ float s_fin[16];
    __shared__ bool s_last;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + P.xl_bytes + P.part_bytes);
    uint64_t* empty = full + GS_MAX_STAGES;
    uint8_t* stages = reinterpret_cast<uint8_t*>(full) + 128;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (uint32_t s = 0; s < P.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], GS_WARPS);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    pdl_trigger();
    pdl_wait();
    if (*P.st_done) return;   // the whole grid leaves (the step state is stable during the launch)
    const bool skip_logits = P.st_skip && P.st_skip[0] < P.st_skip[1];

    if (warp == GS_WARPS) {
        // ---------------- producer warp ----------------
        Ring r{0, 1};   // empty-barrier phase: the first round needs no wait
        uint32_t issued = 0;
        for (int k = 0; k < P.n_ops; ++k) {
            const StreamOp& op = P.ops[k];
            if (op.kind == SOP_GEMV) {
                if (op.logits && skip_logits) continue;
                stream_gemv_produce(op, P, full, empty, stages, r, issued, lane);
            } else {
                A::produce(op, P, full, empty, stages, r, issued, lane);
            }
        }
        // copies still in flight (only after an abort) land before the CTA leaves
        if (lane == 0) {
            const uint32_t n = issued < P.stages ? issued : P.stages;
            for (uint32_t k = 0; k < n; ++k) {
                const uint32_t i = issued - 1 - k, st = i % P.stages, par = (i / P.stages) & 1u;
                for (uint32_t w = 0; w < BULK_WAIT_LIMIT && !mbar_try_wait(&full[st], par); ++w) {}
            }
        }
    } else {
        // ---------------- consumer warps ----------------
        constexpr uint32_t CT = GS_WARPS * 32;
        Ring r{0, 0};
        for (int k = 0; k < P.n_ops; ++k) {   // every warp walks every op, failed waits included
            const StreamOp& op = P.ops[k];
            if (op.dep >= 0) {
                if (tid == 0) wait_counter(&P.done[op.dep], gridDim.x, P.errf);
                asm volatile("bar.sync 1, %0;" ::"r"(CT) : "memory");
            }
            if (op.kind == SOP_GEMV) {
                if (!(op.logits && skip_logits)) {
                    switch (op.dtype) {
                        case GGC_Q4_K: stream_gemv_consume<GGC_Q4_K>(op, P, smem, full, empty, stages, r, red, &s_scale); break;
                        case GGC_Q6_K: stream_gemv_consume<GGC_Q6_K>(op, P, smem, full, empty, stages, r, red, &s_scale); break;
                        case GGC_Q4_0: stream_gemv_consume<GGC_Q4_0>(op, P, smem, full, empty, stages, r, red, &s_scale); break;
                        case GGC_Q8_0: stream_gemv_consume<GGC_Q8_0>(op, P, smem, full, empty, stages, r, red, &s_scale); break;
                        default: break;
                    }
                }
            } else {
                A::consume(op, P, smem, full, empty, stages, r, s_fin, &s_last);
            }
            // this CTA's part of op k is written: publish it
            asm volatile("bar.sync 1, %0;" ::"r"(CT) : "memory");
            if (tid == 0) {
                __threadfence();
                atomicAdd(&P.done[k], 1u);
            }
        }
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(&P.done[P.n_ops], 1u) == gridDim.x - 1) {   // last CTA out: counters back to zero
            for (int k = 0; k <= P.n_ops; ++k) P.done[k] = 0;
            __threadfence();
        }
    }
}

}  // namespace ggc

namespace ggc {
// host side (stream.cu)
bool stream_supported(uint32_t hd, bool f16, uint32_t G);
void stream_attn_geometry(uint32_t hd, bool f16, uint32_t G, uint32_t* tile_bytes, uint32_t* scratch_bytes);
cudaError_t stream_prepare(uint32_t hd, bool f16, uint32_t G, size_t smem, int* max_blocks_per_sm);
cudaError_t stream_launch(uint32_t hd, bool f16, uint32_t G, const StreamArgs& P, unsigned grid, size_t smem,
                          cudaStream_t st);
}  // namespace ggc
