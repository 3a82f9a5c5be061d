// attention.cuh -- decode attention over the HBM-resident KV cache.
//
// Replaces LlamaModel::attend (src/infer/model/llama.rs:499-545) for one new
// token: for q-head h (kv head h / (n_heads / n_kv_heads)),
//   score_s = (q . k_s) * (1/sqrt(hd))   for s <= pos, -inf otherwise
//   w = softmax(score)                    (ops::softmax, ops.rs:295-308)
//   o = sum_{s: |w_s| > 1e-9} w_s v_s
// The cache is [slot][n_kv][hd] like cache.rs:12-17; the current token's K/V is
// already at index `slot`.
//
// Two kernels, each over a (kv head, sequence split) grid so that K and V are
// each read once by all SMs:
//   k_attn_scores  q.k for its split, per-split maxima; the last CTA of a kv head
//                  (atomic ticket) reduces max and sum exp over the whole row.
//   k_attn_av      w = exp(score - max) * (1/sum) as the reference computes it,
//                  the weighted V sum of its split; the last CTA adds the split
//                  partials in fixed order (deterministic) into o.
#pragma once
#include "common.cuh"

namespace ggc {

struct AttnArgs {
    const float* q;          // [n_heads * hd]
    const void* kc;          // this layer's K cache [max_ctx][kvh * hd]
    const void* vc;          // this layer's V cache
    float* scores;           // [n_heads][max_ctx]
    float* pmax;             // [n_heads][nsplit]
    float2* stats;           // [n_heads] (max, 1/sum)
    float* opart;            // [nsplit][n_heads][hd]
    float* o;                // [n_heads * hd]
    unsigned* tickets;       // [2][kvh], zero between launches
    const uint32_t* slot;
    const int64_t* pos;
    const int* done;
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

__global__ void __launch_bounds__(ATTN_WARPS * 32) k_attn_scores(const AttnArgs a) {
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
    const uint64_t row = (uint64_t)a.kvh * hd;
    for (uint32_t s = s0 + warp; s < s1; s += ATTN_WARPS) {
        float kv[ATTN_MAX_NI];
#pragma unroll
        for (int k = 0; k < ATTN_MAX_NI; ++k) {
            const uint32_t i = lane + 32 * k;
            kv[k] = (i < hd) ? kv_load(a.kc, s * row + kvhead * hd + i, a.kv_f16) : 0.f;
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

__global__ void __launch_bounds__(ATTN_WARPS * 32) k_attn_av(const AttnArgs a) {
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
    const uint64_t row = (uint64_t)a.kvh * hd;
    for (uint32_t s = s0 + warp; s < s1; s += ATTN_WARPS) {
        float vv[ATTN_MAX_NI];
#pragma unroll
        for (int k = 0; k < ATTN_MAX_NI; ++k) {
            const uint32_t i = lane + 32 * k;
            vv[k] = (i < hd) ? kv_load(a.vc, s * row + kvhead * hd + i, a.kv_f16) : 0.f;
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

}  // namespace ggc
