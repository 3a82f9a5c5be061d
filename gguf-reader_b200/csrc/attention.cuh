// attention.cuh -- decode attention over the HBM-resident KV cache.
//
// Replaces LlamaModel::attend (src/infer/model/llama.rs:499-545) for one new
// token: for q-head h (kv head h / (n_heads / n_kv_heads)),
//   score_s = (q . k_s) * (1/sqrt(hd))   for s <= pos, -inf otherwise
//   w = softmax(score)                    (ops::softmax, ops.rs:295-308)
//   o = sum_{s: |w_s| > 1e-9} w_s v_s
// The current token's K/V is already at cache index `slot`.
//
// HBM layout of one layer's cache: head-major [kv head][max_ctx][hd] (the
// reference keeps [slot][kv head][hd], cache.rs:12-17).  A (kv head, position
// range) is then one contiguous run of rows, read with 16-byte vector loads
// that cover whole rows per warp instruction.
//
// k_attn_decode<HD, F16, MAXG> (hd in {64, 128, 256}, GQA group <= 8): one
// kernel per layer, grid (kv head, split).  A CTA computes the scores of its
// position range for the group's q heads (kept in shared memory), their local
// max m and sum l of exp(score - m), and the exp-weighted V sum; the last CTA
// of the kv head (atomic ticket) rescales the split partials by exp(m_k - M)
// and adds them in split order (deterministic).  The |w| <= 1e-9 skip of
// llama.rs:533-537 needs the global max and sum before V is read and is not
// applied: its effect on an output element is below 1e-9 * visible * max|v|.
//
// k_attn_scores + k_attn_av: the general pair (any even hd <= 256), which
// follows the reference's order exactly: all scores, then max and sum over the
// whole row, then w = exp(score - max) * (1/sum) with the skip.
#pragma once
#include <type_traits>
#include "common.cuh"
#include "mbarrier.cuh"

namespace ggc {

struct AttnArgs {
    const float* q;          // [n_heads * hd]
    const void* kc;          // this layer's K cache [max_ctx][kvh * hd]
    const void* vc;          // this layer's V cache
    float* scores;           // [n_heads][max_ctx]
    float* pmax;             // [n_heads][nsplit] (k_attn_scores); [nsplit][n_heads] split max (k_attn_decode)
    float* psum;             // [nsplit][n_heads] split sum of exp (k_attn_decode)
    float2* stats;           // [n_heads] (max, 1/sum)
    float* opart;            // [nsplit][n_heads][hd] split partial outputs
    float* o;                // [n_heads * hd]
    unsigned* tickets;       // [2][kvh], zero between launches (k_attn_decode uses [0][kvh])
    const uint32_t* slot;
    const int64_t* pos;
    const int* done;
    int* errf;               // ERRF_TIMEOUT on an expired wait (k_attn_decode)
    uint32_t n_heads, kvh, hd, max_ctx, nsplit;
    float inv;               // 1/sqrt(hd) as f32 (llama.rs:285)
    int kv_f16;
};

constexpr int ATTN_WARPS = 8;
constexpr int ATTN_MAX_G = 8;      // q heads per kv head
constexpr int ATTN_MAX_NI = 8;     // hd / 32 (hd <= 256)

__device__ __forceinline__ float kv_load(const void* base, uint64_t idx, int f16) {
    return f16 ? __half2float(reinterpret_cast<const __half*>(base)[idx]) : reinterpret_cast<const float*>(base)[idx];
}

__device__ __forceinline__ void attn_range(const AttnArgs& a, uint32_t split, uint32_t& s0, uint32_t& s1, uint32_t& visible) {
    const uint32_t seq = *a.slot + 1;
    const int64_t pos = *a.pos;
    visible = (pos + 1 < (int64_t)seq) ? (uint32_t)(pos + 1) : seq;
    const uint32_t chunk = cdiv(visible, a.nsplit);
    s0 = min(split * chunk, visible);
    s1 = min(s0 + chunk, visible);
}

static __global__ void __launch_bounds__(ATTN_WARPS * 32) k_attn_scores(const AttnArgs a) {
    pdl_trigger();
    pdl_wait();
    if (*a.done) return;
    const uint32_t kvhead = blockIdx.x, split = blockIdx.y;
    const uint32_t G = a.n_heads / a.kvh, h0 = kvhead * G, hd = a.hd;
    uint32_t s0, s1, visible;
    attn_range(a, split, s0, s1, visible);
    __shared__ float sq[ATTN_MAX_G * 256];
    __shared__ float smax[ATTN_WARPS][ATTN_MAX_G];
    __shared__ bool s_last;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (uint32_t i = tid; i < G * hd; i += blockDim.x) sq[i] = a.q[h0 * hd + i];
    __syncthreads();
    float lmax[ATTN_MAX_G];
#pragma unroll
    for (int g = 0; g < ATTN_MAX_G; ++g) lmax[g] = -INFINITY;
    const uint64_t hbase = (uint64_t)kvhead * a.max_ctx * hd;
    for (uint32_t s = s0 + warp; s < s1; s += ATTN_WARPS) {
        float kv[ATTN_MAX_NI];
#pragma unroll
        for (int k = 0; k < ATTN_MAX_NI; ++k) {
            const uint32_t i = lane + 32 * k;
            kv[k] = (i < hd) ? kv_load(a.kc, hbase + (uint64_t)s * hd + i, a.kv_f16) : 0.f;
        }
#pragma unroll
        for (int g = 0; g < ATTN_MAX_G; ++g) {
            if (g >= (int)G) break;
            float dot = 0.f;
#pragma unroll
            for (int k = 0; k < ATTN_MAX_NI; ++k) {
                const uint32_t i = lane + 32 * k;
                if (i < hd) dot = fmaf(sq[g * hd + i], kv[k], dot);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
            const float sc = __fmul_rn(dot, a.inv);
            if (lane == 0) a.scores[(uint64_t)(h0 + g) * a.max_ctx + s] = sc;
            lmax[g] = fmaxf(lmax[g], sc);
        }
    }
    if (lane == 0) {
#pragma unroll
        for (int g = 0; g < ATTN_MAX_G; ++g)
            if (g < (int)G) smax[warp][g] = lmax[g];
    }
    __syncthreads();
    if (tid < (int)G) {
        float m = -INFINITY;
        for (int w = 0; w < ATTN_WARPS; ++w) m = fmaxf(m, smax[w][tid]);
        a.pmax[(uint64_t)(h0 + tid) * a.nsplit + split] = m;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = (atomicAdd(&a.tickets[kvhead], 1u) == a.nsplit - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // last CTA of this kv head: global max and sum of exp for each of its q heads
    __shared__ float ssum[ATTN_WARPS];
    for (uint32_t g = 0; g < G; ++g) {
        const uint32_t h = h0 + g;
        float m = -INFINITY;
        for (uint32_t k = 0; k < a.nsplit; ++k) m = fmaxf(m, __ldcg(&a.pmax[(uint64_t)h * a.nsplit + k]));
        float sum = 0.f;
        for (uint32_t s = tid; s < visible; s += blockDim.x) sum += expf(__ldcg(&a.scores[(uint64_t)h * a.max_ctx + s]) - m);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) ssum[warp] = sum;
        __syncthreads();
        if (tid == 0) {
            float t = 0.f;
            for (int w = 0; w < ATTN_WARPS; ++w) t += ssum[w];
            a.stats[h] = make_float2(m, __fdiv_rn(1.0f, t));
        }
        __syncthreads();
    }
    if (tid == 0) a.tickets[kvhead] = 0;
}

static __global__ void __launch_bounds__(ATTN_WARPS * 32) k_attn_av(const AttnArgs a) {
    pdl_trigger();
    pdl_wait();
    if (*a.done) return;
    const uint32_t kvhead = blockIdx.x, split = blockIdx.y;
    const uint32_t G = a.n_heads / a.kvh, h0 = kvhead * G, hd = a.hd;
    uint32_t s0, s1, visible;
    attn_range(a, split, s0, s1, visible);
    __shared__ float2 sst[ATTN_MAX_G];
    extern __shared__ float dyn[];   // [ATTN_WARPS][G][hd]
    __shared__ bool s_last;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid < (int)G) sst[tid] = a.stats[h0 + tid];
    __syncthreads();
    float acc[ATTN_MAX_G][ATTN_MAX_NI];
#pragma unroll
    for (int g = 0; g < ATTN_MAX_G; ++g)
#pragma unroll
        for (int k = 0; k < ATTN_MAX_NI; ++k) acc[g][k] = 0.f;
    const uint64_t hbase = (uint64_t)kvhead * a.max_ctx * hd;
    for (uint32_t s = s0 + warp; s < s1; s += ATTN_WARPS) {
        float vv[ATTN_MAX_NI];
#pragma unroll
        for (int k = 0; k < ATTN_MAX_NI; ++k) {
            const uint32_t i = lane + 32 * k;
            vv[k] = (i < hd) ? kv_load(a.vc, hbase + (uint64_t)s * hd + i, a.kv_f16) : 0.f;
        }
#pragma unroll
        for (int g = 0; g < ATTN_MAX_G; ++g) {
            if (g >= (int)G) break;
            const float sc = a.scores[(uint64_t)(h0 + g) * a.max_ctx + s];
            const float w = __fmul_rn(expf(sc - sst[g].x), sst[g].y);
            if (fabsf(w) > 1e-9f) {
#pragma unroll
                for (int k = 0; k < ATTN_MAX_NI; ++k) acc[g][k] = fmaf(w, vv[k], acc[g][k]);
            }
        }
    }
    // reduce the warps' partials in fixed order
#pragma unroll
    for (int g = 0; g < ATTN_MAX_G; ++g) {
        if (g >= (int)G) break;
#pragma unroll
        for (int k = 0; k < ATTN_MAX_NI; ++k) {
            const uint32_t i = lane + 32 * k;
            if (i < hd) dyn[((size_t)warp * G + g) * hd + i] = acc[g][k];
        }
    }
    __syncthreads();
    for (uint32_t q = tid; q < G * hd; q += blockDim.x) {
        float t = 0.f;
        for (int w = 0; w < ATTN_WARPS; ++w) t += dyn[(size_t)w * G * hd + q];
        a.opart[((uint64_t)split * a.n_heads + h0) * hd + q] = t;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = (atomicAdd(&a.tickets[a.kvh + kvhead], 1u) == a.nsplit - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (uint32_t q = tid; q < G * hd; q += blockDim.x) {
        float t = 0.f;
        for (uint32_t k = 0; k < a.nsplit; ++k) t += __ldcg(&a.opart[((uint64_t)k * a.n_heads + h0) * hd + q]);
        a.o[(uint64_t)h0 * hd + q] = t;
    }
    if (tid == 0) a.tickets[a.kvh + kvhead] = 0;
}

inline size_t attn_av_smem(uint32_t G, uint32_t hd) { return (size_t)ATTN_WARPS * G * hd * sizeof(float); }

// ---------------------------------------------------------------------------
// k_attn_decode: one-pass split attention (see the file header).
// ---------------------------------------------------------------------------
constexpr int FA_WARPS = 8;
constexpr int FA_THREADS = FA_WARPS * 32;
constexpr int FA_STAGES = 3;
constexpr uint32_t FA_MAX_SPLITS = 64;   // splits of a kv head's positions (the combine's weights)

template <int HD, bool F16, int MAXG>
struct FaCfg {
    static constexpr int ESZ = F16 ? 2 : 4;
    static constexpr int ROWB = HD * ESZ;                 // bytes of one cache row
    static constexpr int GB = 4 * ESZ;                    // bytes of a 4-element group
    static constexpr int NG = HD / 4;                     // groups per row
    static constexpr int LPR = NG < 32 ? NG : 32;         // lanes per row
    static constexpr int GPL = NG / LPR;                  // groups per lane
    static constexpr int RPW = 32 / LPR;                  // rows per warp pass
    static constexpr int TR0 = 16384 / ROWB;
    static constexpr int TR = TR0 > 64 ? 64 : (TR0 < 16 ? 16 : TR0);   // rows per tile (16 KB of K)
    static constexpr int WR = TR / FA_WARPS;              // rows of a tile per warp
    static constexpr int U = WR / RPW;                    // warp passes per tile
    static constexpr int RL = TR > 32 ? TR / 32 : 1;      // rows per lane in the softmax step
    static constexpr int NV = U * MAXG;                   // dot products per lane per tile
    static constexpr int CF = NV > LPR ? NV / LPR : 1;    // totals per lane after the butterfly
    static constexpr uint32_t TILE_BYTES = (uint32_t)TR * ROWB;
    static constexpr size_t SMEM = (size_t)FA_STAGES * 2 * TILE_BYTES + (size_t)TR * MAXG * sizeof(float);
    static_assert(HD % 4 == 0 && 32 % LPR == 0 && WR % RPW == 0 && U >= 1, "tile geometry");
    static_assert(TR % 32 == 0 || TR < 32, "softmax rows per lane");
    static_assert((size_t)FA_WARPS * MAXG * HD * sizeof(float) <= (size_t)FA_STAGES * 2 * TILE_BYTES,
                  "cross-warp reduction fits in the stage area");
};

__device__ __forceinline__ float4 fa_ld(const uint8_t* p, std::false_type) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(smem_addr(p)));
    return v;
}
__device__ __forceinline__ float4 fa_ld(const uint8_t* p, std::true_type) {
    uint32_t a, b;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(a), "=r"(b) : "r"(smem_addr(p)));
    const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&a));
    const float2 y = __half22float2(*reinterpret_cast<const __half2*>(&b));
    return make_float4(x.x, x.y, y.x, y.y);
}
__device__ __forceinline__ float dot4(float4 a, float4 b, float acc) {
    return fmaf(a.w, b.w, fmaf(a.z, b.z, fmaf(a.y, b.y, fmaf(a.x, b.x, acc))));
}

// Sums C values per lane over the lanes that differ in bits O, O/2, .., 1.  While
// more than one value is left, partners swap halves (each keeps one half, sums
// it with the partner's copy), so C values cost C-1 shuffles, not C log2(lanes).
// On return v[0 .. max(C / (2O), 1)) are totals of the original indices base + i.
template <int C, int O>
__device__ __forceinline__ void fa_butterfly(float* v, int lane, int& base) {
    if constexpr (O >= 1) {
        if constexpr (C > 1) {
            const bool up = (lane & O) != 0;
#pragma unroll
            for (int i = 0; i < C / 2; ++i) {
                const float send = up ? v[i] : v[i + C / 2];
                const float keep = up ? v[i + C / 2] : v[i];
                v[i] = keep + __shfl_xor_sync(0xffffffffu, send, O);
            }
            if (up) base += C / 2;
            fa_butterfly<C / 2, O / 2>(v, lane, base);
        } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], O);
            fa_butterfly<1, O / 2>(v, lane, base);
        }
    }
}

template <int HD, bool F16, int MAXG>
__global__ void __launch_bounds__(FA_THREADS, 2) k_attn_decode(const AttnArgs a) {
    using C = FaCfg<HD, F16, MAXG>;
    using IsF16 = std::integral_constant<bool, F16>;
    constexpr int LPR = C::LPR, GPL = C::GPL, RPW = C::RPW, TR = C::TR, WR = C::WR, U = C::U, RL = C::RL;
    constexpr int NV = C::NV, CF = C::CF;
    constexpr uint32_t TB = C::TILE_BYTES;
    extern __shared__ __align__(128) uint8_t fsm[];
    uint8_t* kst = fsm;                                                    // [stage] K tile
    uint8_t* vst = fsm + FA_STAGES * TB;                                   // [stage] V tile
    float* ssc = reinterpret_cast<float*>(fsm + 2 * FA_STAGES * TB);       // [TR][MAXG] scores of a tile
    __shared__ __align__(8) uint64_t full[FA_STAGES];
    __shared__ float s_fin[2][MAXG];
    __shared__ float s_w[MAXG][FA_MAX_SPLITS];   // split weights exp(m_k - M) of the combine
    __shared__ bool s_last;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int sub = lane / LPR, gl = lane % LPR;

    if (tid == 0) {
        for (int s = 0; s < FA_STAGES; ++s) mbar_init(&full[s], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    pdl_trigger();
    pdl_wait();
    if (*a.done) return;

    const uint32_t kvhead = blockIdx.x, split = blockIdx.y;
    const uint32_t G = a.n_heads / a.kvh, h0 = kvhead * G;
    uint32_t s0, s1, visible;
    attn_range(a, split, s0, s1, visible);
    const uint32_t n = s1 - s0, ntiles = (n + TR - 1) / TR;
    const uint8_t* kg = reinterpret_cast<const uint8_t*>(a.kc) + ((uint64_t)kvhead * a.max_ctx + s0) * C::ROWB;
    const uint8_t* vg = reinterpret_cast<const uint8_t*>(a.vc) + ((uint64_t)kvhead * a.max_ctx + s0) * C::ROWB;
    auto issue = [&](uint32_t t) {
        const uint32_t rows = min((uint32_t)TR, n - t * TR), bytes = rows * C::ROWB, s = t % FA_STAGES;
        mbar_arrive_expect_tx(&full[s], 2 * bytes);
        bulk_g2s(kst + s * TB, kg + (uint64_t)t * TB, bytes, &full[s]);
        bulk_g2s(vst + s * TB, vg + (uint64_t)t * TB, bytes, &full[s]);
    };
    if (tid == 0)
        for (uint32_t t = 0; t < ntiles && t < (uint32_t)FA_STAGES; ++t) issue(t);

    float4 qv[MAXG][GPL];
#pragma unroll
    for (int g = 0; g < MAXG; ++g)
#pragma unroll
        for (int j = 0; j < GPL; ++j)
            qv[g][j] = g < (int)G ? *reinterpret_cast<const float4*>(a.q + (size_t)(h0 + g) * HD + 4 * (gl + j * LPR))
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

    uint32_t t = 0;
    for (; t < ntiles; ++t) {
        const uint32_t s = t % FA_STAGES;
        const bool got = mbar_wait(&full[s], (t / FA_STAGES) & 1, a.errf);
        const uint8_t* kt = kst + s * TB;
        const uint8_t* vt = vst + s * TB;
        if (got) {
            // scores of this warp's rows: q . k for every (pass, head), one butterfly
            float v[NV];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int r = warp * WR + u * RPW + sub;
                float4 kq[GPL];
#pragma unroll
                for (int j = 0; j < GPL; ++j) kq[j] = fa_ld(kt + r * C::ROWB + (gl + j * LPR) * C::GB, IsF16{});
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
        if (!__syncthreads_and(got)) break;
        // running max / sum (every warp computes the same values), then V
        const uint32_t valid = min((uint32_t)TR, n - t * TR);
        float p[RL][MAXG];
#pragma unroll
        for (int g = 0; g < MAXG; ++g) {
            float mt = -INFINITY;
#pragma unroll
            for (int k = 0; k < RL; ++k) {
                const uint32_t r = (uint32_t)(lane + 32 * k);
                p[k][g] = r < valid ? ssc[r * MAXG + g] : -INFINITY;
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
        const int kk = (warp * WR) / 32;   // the warp's rows share one softmax register slot
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int r = warp * WR + u * RPW + sub;
            const bool rv = (uint32_t)r < valid;
            float4 vq[GPL];
#pragma unroll
            for (int j = 0; j < GPL; ++j) {
                vq[j] = fa_ld(vt + r * C::ROWB + (gl + j * LPR) * C::GB, IsF16{});
                if (!rv) vq[j] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int g = 0; g < MAXG; ++g) {
                float src = p[0][g];
#pragma unroll
                for (int k = 1; k < RL; ++k) src = kk == k ? p[k][g] : src;
                const float w = __shfl_sync(0xffffffffu, src, r & 31);
#pragma unroll
                for (int j = 0; j < GPL; ++j) {
                    acc[g][j].x = fmaf(w, vq[j].x, acc[g][j].x);
                    acc[g][j].y = fmaf(w, vq[j].y, acc[g][j].y);
                    acc[g][j].z = fmaf(w, vq[j].z, acc[g][j].z);
                    acc[g][j].w = fmaf(w, vq[j].w, acc[g][j].w);
                }
            }
        }
        __syncthreads();   // stage s and the score tile are free
        if (tid == 0 && t + FA_STAGES < ntiles) {
            fence_proxy_async_smem();
            issue(t + FA_STAGES);
        }
    }
    if (t < ntiles) {   // a wait expired (ERRF_TIMEOUT is set): let issued copies land, then leave
        if (tid == 0)
            for (uint32_t u = t; u < ntiles && u < t + FA_STAGES; ++u) mbar_wait(&full[u % FA_STAGES], (u / FA_STAGES) & 1, nullptr);
        return;
    }

    // rows of a warp pass -> one partial per warp; warps -> fixed-order sum
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
    float* sred = reinterpret_cast<float*>(fsm);   // [FA_WARPS][MAXG][HD] over the free stages
    if (sub == 0) {
#pragma unroll
        for (int g = 0; g < MAXG; ++g)
#pragma unroll
            for (int j = 0; j < GPL; ++j)
                *reinterpret_cast<float4*>(sred + ((size_t)warp * MAXG + g) * HD + 4 * (gl + j * LPR)) = acc[g][j];
    }
    __syncthreads();
    for (uint32_t e = tid; e < G * HD; e += FA_THREADS) {
        const uint32_t g = e / HD, i = e % HD;
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < FA_WARPS; ++w) sum += sred[((size_t)w * MAXG + g) * HD + i];
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
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(&a.tickets[kvhead], 1u) == a.nsplit - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // last CTA of the kv head: M = max m_k, S = sum exp(m_k - M) l_k,
    // o = (sum exp(m_k - M) o_k) * (1/S), splits in index order.  The split weights
    // exp(m_k - M) go to shared memory once, so the output sums load the partials
    // without a data-dependent branch (several loads in flight).
    if (warp < (int)G) {
        const uint32_t h = h0 + warp;
        float M = -INFINITY;
        for (uint32_t k = lane; k < a.nsplit; k += 32) M = fmaxf(M, __ldcg(&a.pmax[(size_t)k * a.n_heads + h]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        float S = 0.f;
        for (uint32_t k = lane; k < a.nsplit; k += 32) {
            const float mk = __ldcg(&a.pmax[(size_t)k * a.n_heads + h]);
            const float w = mk != -INFINITY ? expf(mk - M) : 0.f;
            s_w[warp][k] = w;
            if (mk != -INFINITY) S += w * __ldcg(&a.psum[(size_t)k * a.n_heads + h]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) S += __shfl_xor_sync(0xffffffffu, S, o);
        if (lane == 0) s_fin[1][warp] = __fdiv_rn(1.0f, S);
    }
    __syncthreads();
    for (uint32_t e = tid; e < G * HD; e += FA_THREADS) {
        const uint32_t g = e / HD, i = e % HD, h = h0 + g;
        const float* op = a.opart + (size_t)h * HD + i;
        const size_t stride = (size_t)a.n_heads * HD;
        float sum = 0.f;
        uint32_t k = 0;
        for (; k + 8 <= a.nsplit; k += 8) {
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = __ldcg(op + (k + u) * stride);
#pragma unroll
            for (int u = 0; u < 8; ++u) sum += s_w[g][k + u] * v[u];
        }
        for (; k < a.nsplit; ++k) sum += s_w[g][k] * __ldcg(op + k * stride);
        a.o[(size_t)h * HD + i] = sum * s_fin[1][g];
    }
    if (tid == 0) a.tickets[kvhead] = 0;
}

}  // namespace ggc
