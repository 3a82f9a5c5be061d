// sample.cuh -- Sampler::sample (src/infer/sampler.rs:86-186) on the device, so a
// decode loop that samples reads back one token id instead of the logits.
//
// The random draw stays with the caller: `u` is the rng.gen_range(0.0..1.0) value
// the reference draws once per sample (step 7), so a host that keeps the
// reference's RNG gets the reference's stream of draws.
//
// One CTA of SAMPLE_THREADS threads:
//   1. v = logits with the repeat penalty on the seen ids (divide if > 0, else
//      multiply), NaN -> error (the reference panics in partial_cmp);
//   2. temperature <= 1e-6: greedy argmax of v, the last maximum (max_by);
//   3. s = v / T; p_i = exp(s_i - max s) / sum (the sum is a block reduction, not
//      the reference's serial f32 sum: the probabilities share a common factor
//      within a few ulp of the reference's, so a pick can differ only when u lands
//      that close to a cumulative boundary);
//   4. top-k: the k-th largest p by a 4-pass radix select on the f32 bits (p >= 0,
//      so the bits order like the values), then every p above it plus the first
//      ones equal to it in index order (the stable sort keeps ties in index
//      order), bitonic-sorted by (p descending, index ascending);
//   5-7. top-p, min-p and the pick walk the <= SAMPLE_MAX_K candidates serially
//      in the reference's f32 order; an empty set falls back to argmax of s.
// Without top-k (k = 0 or k >= vocab) the candidates are the whole vocabulary,
// supported up to SAMPLE_MAX_K entries (in index order unless top-p sorts them).
#pragma once
#include "common.cuh"

namespace ggc {

constexpr int SAMPLE_THREADS = 1024;
constexpr int SAMPLE_MAX_K = 1024;

struct SampleCfg {
    float temperature;
    uint32_t top_k;
    float top_p;
    float min_p;
    float repeat_penalty;
};

// key of the last maximum: order-preserving float bits, ties -> larger index
__device__ __forceinline__ unsigned long long sample_max_key(float v, uint32_t idx) {
    uint32_t b = __float_as_uint(v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)b << 32) | idx;
}

__device__ __forceinline__ unsigned long long block_max_u64(unsigned long long v, unsigned long long* red) {
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
        v = w > v ? w : v;
    }
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    unsigned long long m = 0;
    for (int w = 0; w < SAMPLE_THREADS / 32; ++w) m = red[w] > m ? red[w] : m;
    return m;
}

__device__ __forceinline__ float block_sum_f32(float v, float* red) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float s = 0.f;
    for (int w = 0; w < SAMPLE_THREADS / 32; ++w) s += red[w];
    return s;
}

// exclusive prefix over the block of a 0/1 flag, and the block total
__device__ __forceinline__ uint32_t block_excl_scan(uint32_t flag, uint32_t* wsum, uint32_t* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const unsigned bal = __ballot_sync(0xffffffffu, flag);
    const uint32_t in_warp = __popc(bal & ((1u << lane) - 1u));
    __syncthreads();
    if (lane == 0) wsum[warp] = __popc(bal);
    __syncthreads();
    uint32_t before = 0, all = 0;
    for (int w = 0; w < SAMPLE_THREADS / 32; ++w) {
        if (w < warp) before += wsum[w];
        all += wsum[w];
    }
    *total = all;
    return before + in_warp;
}

// work: vocab floats of scratch (the penalised / scaled values); out[0] = the
// token id; err[0] = 1 on a NaN logit.
__global__ void __launch_bounds__(SAMPLE_THREADS) k_sample(const float* __restrict__ logits, uint32_t vocab,
                                                           const uint32_t* __restrict__ seen, uint32_t n_seen,
                                                           const SampleCfg cfg, float u, float* work, uint32_t* out,
                                                           int* err) {
    __shared__ unsigned long long sred[SAMPLE_THREADS / 32];
    __shared__ float fred[SAMPLE_THREADS / 32];
    __shared__ uint32_t wsum[SAMPLE_THREADS / 32];
    __shared__ uint32_t hist[256];
    __shared__ unsigned long long cand[SAMPLE_MAX_K];
    __shared__ uint32_t s_digit, s_above;
    const uint32_t tid = threadIdx.x;
    pdl_trigger();
    pdl_wait();
    // 1. copy + NaN check, then the penalty on the seen ids (sampler.rs:95-110)
    bool nan = false;
    for (uint32_t i = tid; i < vocab; i += SAMPLE_THREADS) {
        const float x = logits[i];
        nan |= isnan(x);
        work[i] = x;
    }
    if (__syncthreads_or(nan)) {
        if (tid == 0) { err[0] = 1; out[0] = 0; }
        return;
    }
    if (cfg.repeat_penalty != 1.0f)
        for (uint32_t k = tid; k < n_seen; k += SAMPLE_THREADS) {
            const uint32_t idx = seen[k];
            if (idx < vocab) {
                const float x = work[idx];
                work[idx] = x > 0.0f ? x / cfg.repeat_penalty : x * cfg.repeat_penalty;
            }
        }
    __syncthreads();
    // 2. greedy (:112-124)
    if (!(cfg.temperature > 1e-6f)) {
        unsigned long long best = 0;
        for (uint32_t i = tid; i < vocab; i += SAMPLE_THREADS) {
            const unsigned long long k = sample_max_key(work[i], i);
            best = k > best ? k : best;
        }
        best = block_max_u64(best, sred);
        if (tid == 0) out[0] = (uint32_t)(best & 0xFFFFFFFFull);
        return;
    }
    // 3. temperature and softmax (:112-130); the argmax of s is kept for step 7's fallback
    unsigned long long best = 0;
    for (uint32_t i = tid; i < vocab; i += SAMPLE_THREADS) {
        const float s = work[i] / cfg.temperature;
        work[i] = s;
        const unsigned long long k = sample_max_key(s, i);
        best = k > best ? k : best;
    }
    best = block_max_u64(best, sred);
    const uint32_t arg_s = (uint32_t)(best & 0xFFFFFFFFull);
    const float max_v = work[arg_s];   // written by this block, visible after the barriers above
    float part = 0.f;
    for (uint32_t i = tid; i < vocab; i += SAMPLE_THREADS) part += expf(work[i] - max_v);
    const float sum = block_sum_f32(part, fred);
    for (uint32_t i = tid; i < vocab; i += SAMPLE_THREADS) work[i] = expf(work[i] - max_v) / sum;   // p_i
    __syncthreads();
    // 4. the candidate set
    const bool use_k = cfg.top_k > 0 && cfg.top_k < vocab;
    const uint32_t k = use_k ? cfg.top_k : vocab;   // <= SAMPLE_MAX_K (checked on the host)
    uint32_t thr = 0, take_eq = k;                  // p bits of the k-th largest; ties to take
    if (use_k) {
        uint32_t prefix = 0, mask = 0, need = k;
        for (int shift = 24; shift >= 0; shift -= 8) {
            for (uint32_t i = tid; i < 256; i += SAMPLE_THREADS) hist[i] = 0;
            __syncthreads();
            for (uint32_t i = tid; i < vocab; i += SAMPLE_THREADS) {
                const uint32_t b = __float_as_uint(work[i]);
                if ((b & mask) == prefix) atomicAdd(&hist[(b >> shift) & 0xFF], 1u);
            }
            __syncthreads();
            if (tid == 0) {
                uint32_t above = 0, d = 255;
                for (;; --d) {
                    if (above + hist[d] >= need || d == 0) break;
                    above += hist[d];
                }
                s_digit = d;
                s_above = above;
            }
            __syncthreads();
            prefix |= s_digit << shift;
            mask |= 0xFFu << shift;
            need -= s_above;
            __syncthreads();
        }
        thr = prefix;
        take_eq = need;
    }
    // ordered compaction: p > thr anywhere, p == thr by index up to take_eq
    // (without top-k: every index, in index order)
    uint32_t n_gt = 0, n_eq = 0;
    for (uint32_t base = 0; base < vocab; base += SAMPLE_THREADS) {
        const uint32_t i = base + tid;
        const uint32_t b = i < vocab ? __float_as_uint(work[i]) : 0u;
        const bool in = i < vocab;
        const bool gt = in && (!use_k || b > thr), eq = in && use_k && b == thr;
        uint32_t tot_gt, tot_eq;
        const uint32_t r_gt = block_excl_scan(gt ? 1u : 0u, wsum, &tot_gt);
        const uint32_t r_eq = block_excl_scan(eq ? 1u : 0u, wsum, &tot_eq);
        if (gt && n_gt + r_gt < (uint32_t)SAMPLE_MAX_K)
            cand[n_gt + r_gt] = ((unsigned long long)b << 32) | (0xFFFFFFFFu - i);
        if (eq && n_eq + r_eq < take_eq) {
            const uint32_t slot = (k - take_eq) + n_eq + r_eq;   // after the k - take_eq larger ones
            if (slot < (uint32_t)SAMPLE_MAX_K) cand[slot] = ((unsigned long long)b << 32) | (0xFFFFFFFFu - i);
        }
        n_gt += tot_gt;
        n_eq += tot_eq;
    }
    const uint32_t n = use_k ? k : vocab;
    for (uint32_t i = n + tid; i < (uint32_t)SAMPLE_MAX_K; i += SAMPLE_THREADS) cand[i] = 0ull;   // pad: sorts last
    __syncthreads();
    // sort (p descending, index ascending) when the reference sorts: top-k or top-p
    if (use_k || cfg.top_p < 1.0f) {
        for (uint32_t size = 2; size <= (uint32_t)SAMPLE_MAX_K; size <<= 1)
            for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
                for (uint32_t i = tid; i < (uint32_t)SAMPLE_MAX_K; i += SAMPLE_THREADS) {
                    const uint32_t j = i ^ stride;
                    if (j > i) {
                        const bool desc = (i & size) == 0;
                        const unsigned long long a = cand[i], c = cand[j];
                        if (desc ? (a < c) : (a > c)) { cand[i] = c; cand[j] = a; }
                    }
                }
                __syncthreads();
            }
    }
    if (tid != 0) return;
    // 5-7: serial, in the reference's order (:142-184)
    auto pv = [&](uint32_t q) { return __uint_as_float((uint32_t)(cand[q] >> 32)); };
    auto id = [&](uint32_t q) { return 0xFFFFFFFFu - (uint32_t)(cand[q] & 0xFFFFFFFFull); };
    uint32_t cnt = n;
    if (cfg.top_p < 1.0f) {
        float total = 0.0f;
        for (uint32_t q = 0; q < cnt; ++q) total = __fadd_rn(total, pv(q));
        const float threshold = __fmul_rn(total, cfg.top_p);
        float cum = 0.0f;
        uint32_t cut = cnt;
        for (uint32_t q = 0; q < cnt; ++q) {
            cum = __fadd_rn(cum, pv(q));
            if (cum >= threshold) { cut = q + 1; break; }
        }
        cnt = cut;
    }
    float min_thr = -1.0f;   // min-p keeps p >= max * min_p, in order
    if (cfg.min_p > 0.0f) {
        float mp = 0.0f;
        for (uint32_t q = 0; q < cnt; ++q) mp = fmaxf(mp, pv(q));
        min_thr = __fmul_rn(mp, cfg.min_p);
    }
    float total = 0.0f;
    uint32_t kept = 0, last = 0;
    for (uint32_t q = 0; q < cnt; ++q)
        if (pv(q) >= min_thr) { total = __fadd_rn(total, pv(q)); ++kept; last = q; }
    if (kept == 0) { out[0] = arg_s; return; }
    float r = __fmul_rn(u, total);
    for (uint32_t q = 0; q < cnt; ++q) {
        if (!(pv(q) >= min_thr)) continue;
        r = __fsub_rn(r, pv(q));
        if (r <= 0.0f) { out[0] = id(q); return; }
    }
    out[0] = id(last);
}

}  // namespace ggc
