// ops.cuh -- the standalone functions of src/infer/ops.rs on the device (API
// surface: the model's forward uses its own fused kernels).  Products and sums
// run serially per output in the reference's order (one thread per output row /
// vector, no FMA contraction: the file is built with -fmad=false), so matvec,
// matmul, the column-major variants, rmsnorm and layernorm give the reference's
// bits; silu, gelu, softmax and rope call CUDA's expf / tanhf / sincosf, within a
// few ulp of the host libm the reference calls.
#pragma once
#include "common.cuh"

namespace ggc {

// y[i] = sum_j a[i*rs + j*cs] * x[j] (+ b[i]) serially in j: rs/cs pick the layout
//   matvec / colmajor_trans: a[i*cols + j] (rs = cols, cs = 1); colmajor: a[j*rows + i]
__global__ void __launch_bounds__(128) k_ops_matvec(const float* __restrict__ a, uint64_t rows, uint64_t cols,
                                                    uint64_t rs, uint64_t cs, const float* __restrict__ x,
                                                    const float* __restrict__ b, float* __restrict__ y) {
    pdl_trigger();
    pdl_wait();
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows) return;
    float acc = 0.f;
    for (uint64_t j = 0; j < cols; ++j) acc = __fadd_rn(acc, __fmul_rn(a[i * rs + j * cs], x[j]));
    y[i] = __fadd_rn(acc, b ? b[i] : 0.0f);
}

// c[i][j] = sum_k a[i][k] * b[k][j] serially in k (ops.rs:74-113)
__global__ void __launch_bounds__(256) k_ops_matmul(const float* __restrict__ a, const float* __restrict__ b,
                                                    uint64_t ra, uint64_t ca, uint64_t cb, float* __restrict__ c) {
    pdl_trigger();
    pdl_wait();
    const uint64_t j = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x, i = blockIdx.y;
    if (j >= cb || i >= ra) return;
    float acc = 0.f;
    for (uint64_t k = 0; k < ca; ++k) acc = __fadd_rn(acc, __fmul_rn(a[i * ca + k], b[k * cb + j]));
    c[i * cb + j] = acc;
}

// silu (ops.rs:237-247, sign branch) and gelu (tanh form, ops.rs:250-256)
__global__ void __launch_bounds__(256) k_ops_act(float* x, uint64_t n, int gelu) {
    pdl_trigger();
    pdl_wait();
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        const float v = x[i];
        if (gelu) {
            const float v3 = __fmul_rn(__fmul_rn(v, v), v);
            const float t = __fmul_rn(0.7978846f, __fadd_rn(v, __fmul_rn(0.044715f, v3)));
            x[i] = __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, tanhf(t)));
        } else {
            float sig;
            if (v >= 0.0f) sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v)));
            else { const float e = expf(v); sig = __fdiv_rn(e, __fadd_rn(1.0f, e)); }
            x[i] = __fmul_rn(v, sig);
        }
    }
}

// one vector per CTA: rmsnorm (ops.rs:262-274, f64 serial sum of squares) and
// layernorm (:279-291, f32 serial mean and variance); thread 0 reduces serially
__global__ void __launch_bounds__(256) k_ops_norm(float* x, uint64_t n, const float* __restrict__ w,
                                                  const float* __restrict__ b, float eps, int layer) {
    __shared__ float s_a, s_b;
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x == 0) {
        if (layer) {
            float sum = 0.f;
            for (uint64_t i = 0; i < n; ++i) sum = __fadd_rn(sum, x[i]);
            const float mean = __fdiv_rn(sum, (float)n);
            float var = 0.f;
            for (uint64_t i = 0; i < n; ++i) {
                const float d = __fsub_rn(x[i], mean);
                var = __fadd_rn(var, __fmul_rn(d, d));
            }
            var = __fdiv_rn(var, (float)n);
            s_a = mean;
            s_b = __fsqrt_rn(__fdiv_rn(1.0f, __fadd_rn(var, eps)));
        } else {
            double ss = 0.0;
            for (uint64_t i = 0; i < n; ++i) ss = __dadd_rn(ss, __dmul_rn((double)x[i], (double)x[i]));
            s_b = (float)__dsqrt_rn(__ddiv_rn(1.0, __dadd_rn(__ddiv_rn(ss, (double)n), (double)eps)));
        }
    }
    __syncthreads();
    for (uint64_t i = threadIdx.x; i < n; i += blockDim.x) {
        if (layer) x[i] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(x[i], s_a), s_b), w[i]), b[i]);
        else x[i] = __fmul_rn(__fmul_rn(x[i], s_b), w[i]);
    }
}

// softmax (ops.rs:295-308): max from -inf, serial sum of exp, times 1/sum
__global__ void __launch_bounds__(256) k_ops_softmax(float* x, uint64_t n) {
    __shared__ float s_max, s_inv;
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x == 0) {
        float mx = -INFINITY;
        for (uint64_t i = 0; i < n; ++i) mx = fmaxf(mx, x[i]);
        float sum = 0.f;
        for (uint64_t i = 0; i < n; ++i) sum = __fadd_rn(sum, expf(__fsub_rn(x[i], mx)));
        s_max = mx;
        s_inv = __fdiv_rn(1.0f, sum);
    }
    __syncthreads();
    for (uint64_t i = threadIdx.x; i < n; i += blockDim.x) x[i] = __fmul_rn(expf(__fsub_rn(x[i], s_max)), s_inv);
}

// rope (ops.rs:318-337): token t (position pos[t], 0 past the list) rotates its
// pairs (i, i + half) by pos * freqs[i]
__global__ void __launch_bounds__(256) k_ops_rope(float* x, uint64_t n_tok, const int64_t* __restrict__ pos,
                                                  uint64_t n_pos, const float* __restrict__ freqs, uint32_t half) {
    pdl_trigger();
    pdl_wait();
    const uint64_t total = n_tok * half;
    for (uint64_t q = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; q < total; q += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t t = q / half;
        const uint32_t i = (uint32_t)(q - t * half);
        const float p = (float)(t < n_pos ? pos[t] : 0);
        float s, c;
        sincosf(__fmul_rn(p, freqs[i]), &s, &c);
        float* base = x + t * 2 * half;
        const float a = base[i], bb = base[i + half];
        base[i] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(bb, s));
        base[i + half] = __fadd_rn(__fmul_rn(bb, c), __fmul_rn(a, s));
    }
}

}  // namespace ggc
