// prefill.cuh -- the batched (prompt / prefill) path: a quantized-weight matrix
// product on the 5th-generation tensor cores, and the per-token kernels around it.
//
// k_mm_tc<DT>: Y[m][n] (+)= X[m][k] . W[n][k]^T with W in raw GGUF blocks.
//   * CTA = 64 weight rows (MM_BN) x up to 512 tokens (MM_MB M-blocks of 128):
//     the f32 accumulators of all its tokens live in tensor memory (4 x 64
//     columns of 128 lanes), so each W tile is read from HBM and dequantised
//     (bit-exact, dequant.cuh) once per CTA and X tiles come from L2.
//   * Precision: W and X are each split into bf16 hi + lo (v = hi + lo to ~16
//     mantissa bits) and D accumulates hi.hi + hi.lo + lo.hi in f32
//     (tcgen05.mma kind::f16, bf16 operands): ~1e-5 relative per product, within
//     the 1e-4 relative-L2 parity bar that plain bf16 (~1e-3) misses.
//   * Per K step of 64: the 256 threads dequantise the W tile and copy the X
//     tiles into shared memory in the canonical K-major layout without swizzle
//     (8-row x 16-byte core matrices: byte (row, kchunk) = kchunk*rows*16 +
//     row*16, so LBO = rows*16 between K chunks, SBO = 128 between 8-row groups),
//     then one thread issues 3 MMAs of K = 16 per M-block and K/16 step and
//     commits them to an mbarrier, which the threads wait on (bounded) before
//     overwriting the tiles.
//   * Epilogue: warps 0-3 read their 32 TMEM lanes (tokens) with tcgen05.ld and
//     write Y rows (+ the residual when given).  TMEM is freed on every path.
#pragma once
#include <cuda_bf16.h>
#include "common.cuh"
#include "dequant.cuh"
#include "mbarrier.cuh"
#include "gemv.cuh"

namespace ggc {

constexpr int MM_BN = 64;                  // weight rows per CTA (UMMA N)
constexpr int MM_BM = 128;                 // tokens per M-block (UMMA M, TMEM lanes)
constexpr int MM_MB = 4;                   // M-blocks per CTA
constexpr int MM_BK = 64;                  // K per stage
constexpr int MM_THREADS = 256;
constexpr uint32_t MM_TOKENS = MM_BM * MM_MB;
constexpr uint32_t MM_TMEM_COLS = MM_MB * MM_BN;            // 256 (a power of two >= 32)
constexpr uint32_t MM_W_BYTES = MM_BN * MM_BK * 2;          // one bf16 W tile
constexpr uint32_t MM_X_BYTES = MM_BM * MM_BK * 2;          // one bf16 X tile
constexpr uint32_t MM_SMEM = 2 * MM_W_BYTES + 2 * MM_MB * MM_X_BYTES;   // 144 KB
// instruction descriptor: D f32, A/B bf16, both K-major, N = 64, M = 128
constexpr uint32_t MM_IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(MM_BN >> 3) << 17) |
                              ((uint32_t)(MM_BM >> 4) << 24);

// shared-memory matrix descriptor: K-major, no swizzle, version 1
__device__ __forceinline__ uint64_t mm_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_ld16(uint32_t taddr, float* v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
        "[%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// hi + lo bf16 split of 8 floats, packed as two 16-byte rows
__device__ __forceinline__ void split8(const float* v, uint4& hi, uint4& lo) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const __nv_bfloat16 h0 = __float2bfloat16_rn(v[2 * j]), h1 = __float2bfloat16_rn(v[2 * j + 1]);
        const __nv_bfloat16 l0 = __float2bfloat16_rn(v[2 * j] - __bfloat162float(h0));
        const __nv_bfloat16 l1 = __float2bfloat16_rn(v[2 * j + 1] - __bfloat162float(h1));
        h[j] = (uint32_t)__bfloat16_as_ushort(h0) | ((uint32_t)__bfloat16_as_ushort(h1) << 16);
        l[j] = (uint32_t)__bfloat16_as_ushort(l0) | ((uint32_t)__bfloat16_as_ushort(l1) << 16);
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// X rows -> bf16 hi / lo [mpad][kpad] (zero beyond m and k), with the row's
// RMSNorm (ops.rs:262-274, f64 sum of squares) or silu(gate) * up applied first.
enum MmPro : int { MMP_PLAIN = 0, MMP_RMSNORM = 1, MMP_SWIGLU = 2 };
constexpr int SPLIT_THREADS = 256;

__global__ void __launch_bounds__(SPLIT_THREADS) k_x_split(const float* __restrict__ x, const float* __restrict__ x2,
                                                           uint32_t m, uint32_t k, uint32_t ldx, uint32_t kpad, int pro,
                                                           __nv_bfloat16* __restrict__ xh,
                                                           __nv_bfloat16* __restrict__ xl) {
    pdl_trigger();
    pdl_wait();
    const uint32_t row = blockIdx.x;
    __shared__ double red[SPLIT_THREADS / 32];
    __shared__ float s_scale;
    const float* xr = x + (size_t)row * ldx;
    float scale = 0.f;
    if (row < m && pro == MMP_RMSNORM) {
        double ss = 0.0;
        for (uint32_t i = threadIdx.x; i < k; i += SPLIT_THREADS) { const double v = (double)xr[i]; ss += v * v; }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
        __syncthreads();
        if (threadIdx.x == 0) {
            double t = 0.0;
            for (int w = 0; w < SPLIT_THREADS / 32; ++w) t += red[w];
            s_scale = (float)sqrt(1.0 / (t / (double)k + (double)1e-6f));
        }
        __syncthreads();
        scale = s_scale;
    }
    for (uint32_t c = threadIdx.x; c < kpad / 8; c += SPLIT_THREADS) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t e = c * 8 + j;
            float t = 0.f;
            if (row < m && e < k) {
                t = xr[e];
                if (pro == MMP_RMSNORM) t = __fmul_rn(__fmul_rn(t, scale), x2[e]);
                else if (pro == MMP_SWIGLU) t = ffn_silu_mul(t, x2[(size_t)row * ldx + e]);
            }
            v[j] = t;
        }
        uint4 h, l;
        split8(v, h, l);
        *reinterpret_cast<uint4*>(xh + (size_t)row * kpad + c * 8) = h;
        *reinterpret_cast<uint4*>(xl + (size_t)row * kpad + c * 8) = l;
    }
}

template <int DT>
__global__ void __launch_bounds__(MM_THREADS, 1)
    k_mm_tc(const uint8_t* __restrict__ w, uint32_t n_rows, uint32_t k_cols, const __nv_bfloat16* __restrict__ xh,
            const __nv_bfloat16* __restrict__ xl, uint32_t m, uint32_t kpad, float* y, uint32_t ldy,
            const float* resid, int* errf) {
    constexpr int BS = block_size_of(DT), BB = block_bytes_of(DT);
    extern __shared__ __align__(128) uint8_t smem[];   // no-swizzle descriptors need 16-byte alignment
    __shared__ uint64_t mbar;
    __shared__ uint32_t s_tmem;
    uint8_t* wsh = smem;
    uint8_t* wsl = smem + MM_W_BYTES;
    uint8_t* xsh = smem + 2 * MM_W_BYTES;
    uint8_t* xsl = xsh + MM_MB * MM_X_BYTES;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t n0 = blockIdx.x * MM_BN, m0 = blockIdx.y * MM_TOKENS;
    const uint32_t left = m - m0, nmb = min((uint32_t)MM_MB, (left + MM_BM - 1) / MM_BM);
    const uint64_t row_bytes = (uint64_t)(k_cols / BS) * BB;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&s_tmem)),
                     "r"(MM_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        mbar_init(&mbar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    pdl_trigger();
    pdl_wait();

    const uint32_t nk = kpad / MM_BK;
    bool ok = true;
    uint32_t commits = 0;   // commit groups issued (one per K step)
    for (uint32_t kb = 0; kb < nk; ++kb) {
        if (kb > 0 && !__syncthreads_and(mbar_wait(&mbar, (kb - 1) & 1, errf))) {   // previous MMAs read the tiles
            ok = false;
            break;
        }
        // W tile: 64 rows x 8 chunks of 8 consecutive elements, dequantised and split
        for (uint32_t it = tid; it < MM_BN * 8; it += MM_THREADS) {
            const uint32_t r = it >> 3, kc = it & 7, n = n0 + r, k0 = kb * MM_BK + kc * 8;
            float v[8];
            if (n < n_rows && k0 < k_cols) {
                const uint8_t* rowp = w + (uint64_t)n * row_bytes;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint32_t e = k0 + j;
                    v[j] = e < k_cols ? deq_elem<DT>(rowp + (uint64_t)(e / BS) * BB, (int)(e % BS)) : 0.f;
                }
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) v[j] = 0.f;
            }
            uint4 h, l;
            split8(v, h, l);
            *reinterpret_cast<uint4*>(wsh + kc * (MM_BN * 16) + r * 16) = h;
            *reinterpret_cast<uint4*>(wsl + kc * (MM_BN * 16) + r * 16) = l;
        }
        // X tiles of the CTA's M-blocks
        for (uint32_t it = tid; it < nmb * MM_BM * 8; it += MM_THREADS) {
            const uint32_t mb = it / (MM_BM * 8), rem = it % (MM_BM * 8), r = rem >> 3, kc = rem & 7;
            const uint32_t row = m0 + mb * MM_BM + r;
            uint4 h = make_uint4(0, 0, 0, 0), l = h;
            if (row < m) {
                const size_t off = (size_t)row * kpad + kb * MM_BK + kc * 8;
                h = *reinterpret_cast<const uint4*>(xh + off);
                l = *reinterpret_cast<const uint4*>(xl + off);
            }
            const uint32_t so = mb * MM_X_BYTES + kc * (MM_BM * 16) + r * 16;
            *reinterpret_cast<uint4*>(xsh + so) = h;
            *reinterpret_cast<uint4*>(xsl + so) = l;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // generic stores -> tensor-core reads
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            const uint32_t a_h = smem_addr(xsh), a_l = smem_addr(xsl), b_h = smem_addr(wsh), b_l = smem_addr(wsl);
            for (uint32_t mb = 0; mb < nmb; ++mb) {
                const uint32_t d = tmem + mb * MM_BN;
#pragma unroll
                for (uint32_t j = 0; j < MM_BK / 16; ++j) {
                    const uint32_t ao = mb * MM_X_BYTES + 2 * j * (MM_BM * 16), bo = 2 * j * (MM_BN * 16);
                    const uint64_t ah = mm_desc(a_h + ao, MM_BM * 16, 128), al = mm_desc(a_l + ao, MM_BM * 16, 128);
                    const uint64_t bh = mm_desc(b_h + bo, MM_BN * 16, 128), bl = mm_desc(b_l + bo, MM_BN * 16, 128);
                    tc_mma(d, ah, bh, MM_IDESC, (kb > 0 || j > 0) ? 1u : 0u);
                    tc_mma(d, ah, bl, MM_IDESC, 1u);
                    tc_mma(d, al, bh, MM_IDESC, 1u);
                }
            }
            tc_commit(&mbar);
        }
        commits = kb + 1;
    }
    if (ok && commits > 0) ok = __syncthreads_and(mbar_wait(&mbar, (commits - 1) & 1, errf));
    if (ok) {
        tc_fence_after();
        if (warp < 4) {
            for (uint32_t mb = 0; mb < nmb; ++mb) {
                const uint32_t row = m0 + mb * MM_BM + warp * 32 + lane;
#pragma unroll 1
                for (uint32_t c0 = 0; c0 < MM_BN; c0 += 16) {
                    float v[16];
                    tc_ld16(tmem + ((uint32_t)(warp * 32) << 16) + mb * MM_BN + c0, v);
                    if (row < m) {
#pragma unroll
                        for (int c = 0; c < 16; ++c) {
                            const uint32_t n = n0 + c0 + c;
                            if (n < n_rows) {
                                const size_t idx = (size_t)row * ldy + n;
                                y[idx] = resid ? __fadd_rn(resid[idx], v[c]) : v[c];
                            }
                        }
                    }
                }
            }
        }
    } else if (commits > 0) {
        // a wait gave up: wait once more (bounded) for the MMAs in flight before freeing TMEM
        mbar_wait(&mbar, (commits - 1) & 1, errf);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(MM_TMEM_COLS) : "memory");
    }
}


// ---- the per-token kernels of the batched forward ---------------------------

// embed (llama.rs:367-380): row tok[t] of token_embd, dequantised, into h[t][:]
template <int DT>
__global__ void __launch_bounds__(256) k_embed_rows(const uint8_t* __restrict__ raw, uint64_t n_rows, uint32_t d,
                                                    const uint32_t* __restrict__ tok, float* __restrict__ h,
                                                    int* __restrict__ errf) {
    constexpr int BS = block_size_of(DT), BB = block_bytes_of(DT);
    pdl_trigger();
    pdl_wait();
    const uint32_t t = blockIdx.x, id = tok[t];
    if ((uint64_t)id >= n_rows) {
        if (threadIdx.x == 0) atomicCAS(&errf[ERRF_EMBED_OOB], 0, (int)id + 1);
        return;
    }
    const uint8_t* row = raw + (uint64_t)id * (uint64_t)(d / BS) * BB;
    for (uint32_t i = threadIdx.x; i < d; i += blockDim.x) {
        const uint32_t blk = i / BS;
        h[(size_t)t * d + i] = deq_elem<DT>(row + (uint64_t)blk * BB, (int)(i - blk * BS));
    }
}

// Q/K/V of the batch (one row per token, columns [q | k | v] at ldy): bias,
// RoPE (ops.rs:318-337, pairs (j, j + hd/2), the decode path's table and
// arithmetic), q into qo[t], k / v into the cache at slot base + t
// (llama.rs:441-479, cache.rs:46-54).  q is skipped when qo is null.
__global__ void __launch_bounds__(256) k_qkv_post(const float* __restrict__ y, uint32_t ldy, uint32_t qdim,
                                                  uint32_t kvdim, uint32_t hd, const float* __restrict__ bq,
                                                  const float* __restrict__ bk, const float* __restrict__ bv,
                                                  const int64_t* __restrict__ pos, const float2* __restrict__ rope,
                                                  uint32_t base, float* __restrict__ qo, void* kc, void* vc,
                                                  uint32_t kv_ctx, int kv_f16) {
    pdl_trigger();
    pdl_wait();
    const uint32_t t = blockIdx.x, half = hd / 2;
    const float* yr = y + (size_t)t * ldy;
    const int64_t p = pos[t];
    const float2* cs = rope + (uint64_t)p * half;
    // RoPE pairs: q (qdim / 2 pairs), then k (kvdim / 2 pairs); then v elements
    const uint32_t nq = qo ? qdim / 2 : 0, nk = kvdim / 2;
    for (uint32_t i = threadIdx.x; i < nq + nk + kvdim; i += blockDim.x) {
        if (i < nq + nk) {
            const bool isq = i < nq;
            const uint32_t pm = isq ? i : i - nq, head = pm / half, j = pm % half;
            const uint32_t l0 = head * hd + j, l1 = l0 + half;
            const float* src = isq ? yr : yr + qdim;
            const float* b = isq ? bq : bk;
            float v0 = src[l0], v1 = src[l1];
            if (b) { v0 = __fadd_rn(v0, b[l0]); v1 = __fadd_rn(v1, b[l1]); }
            const float2 c = cs[j];
            const float n0 = __fsub_rn(__fmul_rn(v0, c.x), __fmul_rn(v1, c.y));
            const float n1 = __fadd_rn(__fmul_rn(v1, c.x), __fmul_rn(v0, c.y));
            if (isq) {
                qo[(size_t)t * qdim + l0] = n0;
                qo[(size_t)t * qdim + l1] = n1;
            } else {
                const uint64_t o = ((uint64_t)head * kv_ctx + base + t) * hd;
                if (kv_f16) {
                    reinterpret_cast<__half*>(kc)[o + j] = __float2half_rn(n0);
                    reinterpret_cast<__half*>(kc)[o + j + half] = __float2half_rn(n1);
                } else {
                    reinterpret_cast<float*>(kc)[o + j] = n0;
                    reinterpret_cast<float*>(kc)[o + j + half] = n1;
                }
            }
        } else {
            const uint32_t lr = i - nq - nk, head = lr / hd;
            float v = yr[qdim + kvdim + lr];
            if (bv) v = __fadd_rn(v, bv[lr]);
            const uint64_t o = ((uint64_t)head * kv_ctx + base + t) * hd + (lr - head * hd);
            if (kv_f16) reinterpret_cast<__half*>(vc)[o] = __float2half_rn(v);
            else reinterpret_cast<float*>(vc)[o] = v;
        }
    }
}

// Causal attention of the batch (llama.rs:499-545) on the CUDA cores: CTA = one
// q head x PA_Q tokens (4 warps x 4 tokens), K/V tiles of 32 cache rows in
// shared memory (K rows padded by one float: lane j reads row j without bank
// conflicts).  Token t (cache slot base + t, position pos[t]) sees the rows
// s < min(pos[t] + 1, base + t + 1), as the decode kernels do; the softmax runs
// online (running max / sum, o rescaled per tile) and o is divided by the sum
// at the end.  Output o[t][head * hd + i].
constexpr int PA_WARPS = 4, PA_QW = 4, PA_Q = PA_WARPS * PA_QW, PA_KT = 32;

template <int HD>
__global__ void __launch_bounds__(PA_WARPS * 32) k_attn_prefill(const float* __restrict__ q, const void* kc,
                                                                 const void* vc, const int64_t* __restrict__ pos,
                                                                 uint32_t base, uint32_t m, uint32_t n_heads,
                                                                 uint32_t kvh, uint32_t kv_ctx, int kv_f16, float inv,
                                                                 float* __restrict__ o) {
    constexpr int NI = HD / 32;
    __shared__ float sk[PA_KT][HD + 1];
    __shared__ float sv[PA_KT][HD];
    __shared__ float sq[PA_Q][HD];
    pdl_trigger();
    pdl_wait();
    const uint32_t head = blockIdx.x, t0 = blockIdx.y * PA_Q, kvhead = head / (n_heads / kvh);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t qdim = n_heads * HD;
    for (uint32_t i = tid; i < PA_Q * HD; i += blockDim.x) {
        const uint32_t r = i / HD, t = t0 + r;
        sq[r][i % HD] = t < m ? q[(size_t)t * qdim + head * HD + i % HD] : 0.f;
    }
    // visible rows per token of this warp, and of the whole CTA
    uint32_t vis[PA_QW];
    uint32_t vmax = 0;
    for (int k = 0; k < PA_QW; ++k) {
        const uint32_t t = t0 + warp * PA_QW + k;
        uint32_t v = 0;
        if (t < m) {
            const int64_t p = pos[t];
            const uint32_t seq = base + t + 1;
            v = (p + 1 < (int64_t)seq) ? (uint32_t)(p + 1) : seq;
        }
        vis[k] = v;
    }
    for (uint32_t r = 0; r < PA_Q; ++r) {
        const uint32_t t = t0 + r;
        if (t < m) {
            const int64_t p = pos[t];
            const uint32_t seq = base + t + 1, v = (p + 1 < (int64_t)seq) ? (uint32_t)(p + 1) : seq;
            vmax = v > vmax ? v : vmax;
        }
    }
    float mx[PA_QW], sum[PA_QW], acc[PA_QW][NI];
#pragma unroll
    for (int k = 0; k < PA_QW; ++k) {
        mx[k] = -INFINITY;
        sum[k] = 0.f;
#pragma unroll
        for (int c = 0; c < NI; ++c) acc[k][c] = 0.f;
    }
    const uint64_t hb = (uint64_t)kvhead * kv_ctx * HD;
    for (uint32_t s0 = 0; s0 < vmax; s0 += PA_KT) {
        __syncthreads();   // previous tile consumed (and sq written, first time)
        for (uint32_t i = tid; i < PA_KT * HD; i += blockDim.x) {
            const uint32_t r = i / HD, c = i % HD, s = s0 + r;
            float kv = 0.f, vv = 0.f;
            if (s < vmax) {
                const uint64_t idx = hb + (uint64_t)s * HD + c;
                kv = kv_f16 ? __half2float(reinterpret_cast<const __half*>(kc)[idx]) : reinterpret_cast<const float*>(kc)[idx];
                vv = kv_f16 ? __half2float(reinterpret_cast<const __half*>(vc)[idx]) : reinterpret_cast<const float*>(vc)[idx];
            }
            sk[r][c] = kv;
            sv[r][c] = vv;
        }
        __syncthreads();
        const uint32_t s = s0 + lane;   // this lane's key
#pragma unroll
        for (int k = 0; k < PA_QW; ++k) {
            if (s0 >= vis[k]) continue;   // warp-uniform
            const float* qr = sq[warp * PA_QW + k];
            float dot = 0.f;
#pragma unroll 8
            for (int i = 0; i < HD; ++i) dot = fmaf(qr[i], sk[lane][i], dot);
            const float sc = s < vis[k] ? __fmul_rn(dot, inv) : -INFINITY;
            float tmax = sc;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
            const float mnew = fmaxf(mx[k], tmax);
            const float scale = expf(mx[k] - mnew);   // 0 on the first tile (mx = -inf)
            const float pj = s < vis[k] ? expf(sc - mnew) : 0.f;
            float ps = pj;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
            sum[k] = sum[k] * scale + ps;
            mx[k] = mnew;
#pragma unroll
            for (int c = 0; c < NI; ++c) acc[k][c] *= scale;
            for (int j = 0; j < PA_KT; ++j) {
                const float pb = __shfl_sync(0xffffffffu, pj, j);
#pragma unroll
                for (int c = 0; c < NI; ++c) acc[k][c] = fmaf(pb, sv[j][lane + 32 * c], acc[k][c]);
            }
        }
    }
#pragma unroll
    for (int k = 0; k < PA_QW; ++k) {
        const uint32_t t = t0 + warp * PA_QW + k;
        if (t >= m) continue;
        const float rs = vis[k] ? 1.0f / sum[k] : 0.f;
#pragma unroll
        for (int c = 0; c < NI; ++c) o[(size_t)t * qdim + head * HD + lane + 32 * c] = acc[k][c] * rs;
    }
}

// NaN anywhere in x[0, n) -> errf[slot] = val (first wins); the NaN guards of
// llama.rs:300-307 for the batch
__global__ void __launch_bounds__(256) k_nan_scan(const float* __restrict__ x, uint64_t n, int* errf, int slot, int val) {
    pdl_trigger();
    pdl_wait();
    bool nan = false;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
        nan |= isnan(x[i]);
    if (__any_sync(0xffffffffu, nan) && (threadIdx.x & 31) == 0) atomicCAS(&errf[slot], 0, val);
}

}  // namespace ggc
