// prefill.cuh -- the batched (prompt / prefill) path: a quantized-weight matrix
// product on the 5th-generation tensor cores, and the per-token kernels around it.
//
// k_mm_tc<DT, BN, STAGE>: Y[m][n] (+)= X[m][k] . W[n][k]^T with W in raw GGUF blocks.
//   * CTA = 128 weight rows x up to 512 tokens: D = W . X^T with the weight rows
//     as the UMMA M side (TMEM lanes) and two 256-token groups as N (2 x 256 f32
//     columns = all of TMEM), so each W tile is read from HBM and dequantised
//     (bit-exact, dequant.cuh) once per CTA and X tiles come from L2.
//   * Precision: W and X are each split into bf16 hi + lo (v = hi + lo to ~16
//     mantissa bits) and D accumulates Wh.Xh + Wl.Xh + Wh.Xl in f32
//     (tcgen05.mma kind::f16, bf16 operands): ~1e-5 relative per product, within
//     the 1e-4 relative-L2 parity bar that plain bf16 (~1e-3) misses.
//   * Shared-memory operands use the canonical K-major layout without swizzle
//     (8-row x 16-byte core matrices: byte (row, kchunk) = kchunk*rows*16 +
//     row*16, so LBO = rows*16 between K chunks, SBO = 128 between 8-row
//     groups); X arrives in that layout by bulk copy (k_x_split writes it so),
//     W is dequantised into it by 8 warps while a copy warp keeps the X (and raw
//     W) rings full and one issuer thread the MMAs (mbarrier rings, see the kernel).
//   * Epilogue: tcgen05.ld of the TMEM lanes (weight rows): for each token a
//     warp stores 32 consecutive floats of a Y row (+ residual).
//     TMEM is freed on every path; every wait is bounded.
#pragma once
#include <cuda.h>   // CUtensorMap (the tensor-map type only)
#include <cuda_bf16.h>
#include "common.cuh"
#include "dequant.cuh"
#include "mbarrier.cuh"
#include "gemv.cuh"

namespace ggc {

constexpr int MM_TG = 256;                 // tokens per token group (UMMA N: TMEM columns of one accumulator)
constexpr int MM_NTG = 2;                  // token groups per CTA (512 tokens: W dequantised once)
constexpr int MM_BK = 64;                  // K per stage
constexpr int MM_DQ_THREADS = 256;         // 8 dequantising / epilogue warps
constexpr int MM_THREADS = MM_DQ_THREADS + 64;   // + the MMA issuer warp (TMEM owner) + the copy warp
constexpr int MM_XS = 8;                   // X quarter-tile ring slots
constexpr uint32_t MM_TOKENS = MM_TG * MM_NTG;
constexpr uint32_t MM_X_BYTES = MM_TG * MM_BK * 2;          // one bf16 X tile (hi or lo): token group x K step, 32 KB
constexpr uint32_t MM_XQ_BYTES = MM_X_BYTES / 4;            // its K quarter (16 columns), 8 KB
constexpr int MM_BN = 128;                 // weight rows per CTA (UMMA M = TMEM lanes); TMEM: 2 x 256 = all 512 columns
constexpr uint32_t mm_w_bytes(int bn) { return (uint32_t)bn * MM_BK * 2; }
// formats whose raw blocks the product stages in shared memory by TMA (256-element
// blocks of a 16-byte multiple: every block of a raw row starts 16-byte aligned)
constexpr bool mm_staged(int dt) { return dt == GGC_Q4_K || dt == GGC_Q5_K; }
// raw staging modes of the product: none; one 2-D TMA copy per block step (Q4_K /
// Q5_K); one bulk copy per row of the 16-byte-aligned window around the row's
// block (Q6_K: 210-byte blocks start at any even offset)
enum MmStage : int { MMS_NONE = 0, MMS_TMA = 1, MMS_ROWS = 2 };
constexpr int mm_xs(bool staged) { return staged ? 6 : MM_XS; }   // X ring slots (smem for the raw ring)
// bytes a staged row takes in the raw ring: the block, or its aligned window
constexpr uint32_t mm_raw_pitch(int sm, int bb) { return sm == MMS_ROWS ? ((uint32_t)bb + 14u + 15u) / 16u * 16u : (uint32_t)bb; }
// dynamic shared memory: W ring [2][hi, lo], X ring [XS][hi, lo] quarter tiles, staged: raw ring
// [2][bn rows][raw pitch] at the next 128-byte boundary (the TMA destination alignment)
constexpr uint32_t mm_smem(int bn, int sm = MMS_NONE, int bb = 0) {
    return 2 * 2 * mm_w_bytes(bn) + mm_xs(sm != MMS_NONE) * 2 * MM_XQ_BYTES +
           (sm != MMS_NONE ? 2u * bn * mm_raw_pitch(sm, bb) + 128u : 0u);
}
// instruction descriptor: D f32, A/B bf16, both K-major, M = bn weight rows, N = MM_TG tokens
constexpr uint32_t mm_idesc(int bn) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(MM_TG >> 3) << 17) | ((uint32_t)(bn >> 4) << 24);
}

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

// 32 consecutive TMEM columns of this thread's lane (32x32b shape, 32 repeats)
__device__ __forceinline__ void tc_ld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
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

// Elements e0 .. e0+7 (e0 % 8 == 0) of one block of >= 8 elements: the deq_elem arithmetic with
// the per-sub-block factors computed once (the same operations per element, so
// the values are bit-identical to deq_elem's).
template <int DT>
__device__ __forceinline__ void deq8(const uint8_t* b, int e0, float* v) {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = deq_elem<DT>(b, e0 + j);
}
// (blocks of 18 / 34 / 210 bytes start 2-byte aligned in a raw row, 144-byte
// blocks 16-byte aligned: the loads below use the widest access that allows)
__device__ __forceinline__ uint16_t ld_a16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }
template <> __device__ __forceinline__ void deq8<GGC_Q4_0>(const uint8_t* b, int e0, float* v) {
    const float d = f16_ref(ld_a16(b));
    const uint32_t w = (uint32_t)ld_a16(b + 2 + (e0 >> 1)) | ((uint32_t)ld_a16(b + 4 + (e0 >> 1)) << 16);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t byte = (w >> (8 * j)) & 0xFF;
        v[2 * j] = __fmul_rn(d, (float)((int)(byte & 0xF) - 8));
        v[2 * j + 1] = __fmul_rn(d, (float)((int)(byte >> 4) - 8));
    }
}
template <> __device__ __forceinline__ void deq8<GGC_Q8_0>(const uint8_t* b, int e0, float* v) {
    const float d = f16_ref(ld_a16(b));
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint16_t h = ld_a16(b + 2 + e0 + 2 * j);
        v[2 * j] = __fmul_rn(d, (float)(int8_t)(h & 0xFF));
        v[2 * j + 1] = __fmul_rn(d, (float)(int8_t)(h >> 8));
    }
}
template <> __device__ __forceinline__ void deq8<GGC_Q4_K>(const uint8_t* b, int e0, float* v) {
    const uint4 h = *reinterpret_cast<const uint4*>(b);   // d, dmin, 12 scale bytes
    const float d = f16_ref((uint16_t)(h.x & 0xFFFF)), dmin = f16_ref((uint16_t)(h.x >> 16));
    const int group = e0 >> 6, in_grp = e0 & 63, is_high = in_grp >> 5, j = group * 2 + is_high;
    const uint32_t sw[3] = {h.y, h.z, h.w};
    auto sb = [&](int i) { return (sw[i >> 2] >> (8 * (i & 3))) & 0xFFu; };   // scale byte i (quant.rs:116-124)
    uint32_t sc, mn;
    if (j < 4) {
        sc = sb(j) & 0x3F;
        mn = sb(j + 4) & 0x3F;
    } else {
        sc = (sb(j + 4) & 0x0F) | ((sb(j - 4) >> 6) << 4);
        mn = (sb(j + 4) >> 4) | ((sb(j) >> 6) << 4);
    }
    const float s1 = __fmul_rn((float)sc, d), s2 = __fmul_rn((float)mn, dmin);
    const uint2 q8 = *reinterpret_cast<const uint2*>(b + 16 + group * 32 + (in_grp & 31));
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t byte = ((i < 4 ? q8.x : q8.y) >> (8 * (i & 3))) & 0xFF;
        const uint32_t val = is_high ? (byte >> 4) : (byte & 0x0F);
        v[i] = __fsub_rn(__fmul_rn(s1, (float)val), s2);
    }
}
template <> __device__ __forceinline__ void deq8<GGC_Q6_K>(const uint8_t* b, int e0, float* v) {
    const float d = f16_ref(ld_a16(b + 208));
    const int n = e0 >> 7, r = e0 & 127, t = r >> 5, l = r & 31, is = l / 16;
    const uint8_t* ql = b + n * 64 + ((t & 1) ? 32 : 0) + l;
    const uint8_t* qh = b + 128 + n * 32 + l;
    const float ds = __fmul_rn(d, (float)(int8_t)b[192 + n * 8 + is + 2 * t]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint16_t lw = ld_a16(ql + 2 * j), hw = ld_a16(qh + 2 * j);
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const uint32_t lb = (lw >> (8 * k)) & 0xFF, hb = (hw >> (8 * k)) & 0xFF;
            const uint32_t q = ((t < 2) ? (lb & 0xF) : (lb >> 4)) | (((hb >> (2 * t)) & 3) << 4);
            v[2 * j + k] = __fmul_rn(ds, (float)((int32_t)q - 32));
        }
    }
}

// X rows -> bf16 hi / lo in the blocked tile layout the product loads with bulk
// copies: tile (256-token group g, K step kb) is 32 KB at ((g * nk + kb) * 32 KB),
// inside it byte kchunk * 4096 + row * 16 (the no-swizzle core-matrix layout;
// the 16 columns of a copy slot are 8 KB contiguous).  Rows m .. mpad-1 and
// columns k .. kpad-1 are zero.  The row's RMSNorm (ops.rs:262-274, f64 sum of
// squares) or silu(gate) * up comes first.  With RMSNorm and nan_val != 0 the
// split is also the NaN guard of its input (llama.rs:300-307): a row's sum of
// squares is NaN exactly when the row holds a NaN -> errf[nan_slot] = nan_val
// (first wins).
enum MmPro : int { MMP_PLAIN = 0, MMP_RMSNORM = 1, MMP_SWIGLU = 2 };
constexpr int SPLIT_THREADS = 256;

__global__ void __launch_bounds__(SPLIT_THREADS) k_x_split(const float* __restrict__ x, const float* __restrict__ x2,
                                                           uint32_t m, uint32_t k, uint32_t ldx, uint32_t kpad, int pro,
                                                           int vec, uint8_t* __restrict__ xh, uint8_t* __restrict__ xl,
                                                           int* errf, int nan_slot, int nan_val) {
    pdl_trigger();
    pdl_wait();
    const uint32_t row = blockIdx.x, nk = kpad / MM_BK;
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
            if (nan_val && isnan(t)) atomicCAS(&errf[nan_slot], 0, nan_val);
        }
        __syncthreads();
        scale = s_scale;
    }
    const size_t tile0 = (size_t)(row / MM_TG) * nk * MM_X_BYTES + (row % MM_TG) * 16;
    // whole 8-element chunks by float4 loads when the rows allow it (vec: x, x2
    // 16-byte aligned, ldx a multiple of 4); the same arithmetic per element
    const float* x2r = pro == MMP_SWIGLU ? x2 + (size_t)row * ldx : x2;
    for (uint32_t c = threadIdx.x; c < kpad / 8; c += SPLIT_THREADS) {
        float v[8];
        if (vec && row < m && c * 8 + 8 <= k) {
            const float4 a0 = *reinterpret_cast<const float4*>(xr + c * 8);
            const float4 a1 = *reinterpret_cast<const float4*>(xr + c * 8 + 4);
            v[0] = a0.x; v[1] = a0.y; v[2] = a0.z; v[3] = a0.w; v[4] = a1.x; v[5] = a1.y; v[6] = a1.z; v[7] = a1.w;
            if (pro != MMP_PLAIN) {
                const float4 b0 = *reinterpret_cast<const float4*>(x2r + c * 8);
                const float4 b1 = *reinterpret_cast<const float4*>(x2r + c * 8 + 4);
                const float w[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    v[j] = pro == MMP_RMSNORM ? __fmul_rn(__fmul_rn(v[j], scale), w[j]) : ffn_silu_mul(v[j], w[j]);
            }
        } else {
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
        }
        uint4 h, l;
        split8(v, h, l);
        const size_t off = tile0 + (size_t)(c / 8) * MM_X_BYTES + (c % 8) * (MM_TG * 16);
        *reinterpret_cast<uint4*>(xh + off) = h;
        *reinterpret_cast<uint4*>(xl + off) = l;
    }
}

// Y[m][n] (+)= X . W^T as D = W . X^T.  Block = 8 dequantising warps + the MMA
// warp + the copy warp.
//   dequant warps: W tile of K step kb (BN rows x 64) -> bf16 hi / lo into W
//     slot kb % 2 (after the MMAs of kb - 2 freed it: wfree), arrive on wfull;
//   copy warp (warp 9, one lane): keeps the X ring full by bulk copy -- one slot
//     = one 256-token group x 16 columns of a K step, hi + lo, 16 KB (xfull; a
//     slot is refilled after the MMAs that read it completed: xfree) -- and, for
//     the staged formats, the raw ring;
//   MMA warp (warp 8, one lane, TMEM owner): for each K step waits for the W
//     slot, then per token group and 16 columns for its X slot, issues 3 MMAs
//     (A = the W rows of the slot, B = the X slot) into the group's 256 TMEM
//     columns and commits them to xfree; the step's commit frees the W slot, the
//     last one signals `done`.  It never waits on a free slot, so the tensor
//     pipe's queue stays full while copies are in flight;
//   epilogue: the 8 warps read TMEM (warp w: lanes 32 (w % 4).. = weight rows,
//     columns of token group w / 4) and write Y (+ the residual).
// Every wait is bounded (ERRF_TIMEOUT); no thread leaves early, warp 8 frees TMEM.
//
// SM = MMS_TMA (Q4_K, Q5_K): the copy warp also loads the CTA's raw blocks of
// each 256-element K range (BN rows x one block, rows past the matrix
// zero-filled) with one 2-D TMA copy (tensor map over the raw rows as bytes, no
// multicast) into a 2-slot ring (rfull / rfree), so the dequantising warps read
// shared memory only; SM = MMS_ROWS (Q6_K): the same ring, filled with one bulk
// copy per row of the 16-byte-aligned window around the row's block (rows past
// the matrix not loaded, their values zero).  Split-K ranges are whole blocks.
template <int DT, int BN, int SM>
__global__ void __launch_bounds__(MM_THREADS, 1)
    k_mm_tc(const uint8_t* __restrict__ w, uint32_t n_rows, uint32_t k_cols, const uint8_t* __restrict__ xh,
            const uint8_t* __restrict__ xl, uint32_t m, uint32_t kpad, uint32_t kb_per, float* y, uint32_t ldy,
            const float* resid, int* errf, const __grid_constant__ CUtensorMap wmap) {
    constexpr int BS = block_size_of(DT), BB = block_bytes_of(DT);
    constexpr bool STAGE = SM != MMS_NONE;
    static_assert(SM != MMS_TMA || (mm_staged(DT) && BS == 4 * MM_BK && BB % 16 == 0 && (BN * BB) % 128 == 0),
                  "TMA staging: 256-element blocks of a 16-byte multiple");
    static_assert(SM != MMS_ROWS || (DT == GGC_Q6_K && BS == 4 * MM_BK), "row-window staging: Q6_K");
    constexpr int XS = mm_xs(STAGE);
    static_assert(BN == 128, "UMMA M = 128 weight rows (all TMEM lanes)");
    constexpr uint32_t RP = mm_raw_pitch(SM, BB);   // bytes of a staged row
    constexpr uint32_t WB = mm_w_bytes(BN), TCOLS = MM_NTG * MM_TG, IDESC = mm_idesc(BN), RB = (uint32_t)BN * RP;
    static_assert(!STAGE || (RP % 16 == 0 && RB % 128 == 0), "raw ring slots 128-byte aligned, rows 16-byte aligned");
    constexpr uint32_t KSTEPS_PER_BLOCK = STAGE ? BS / MM_BK : 1;   // K steps per staged raw block (4)
    extern __shared__ __align__(128) uint8_t smem[];   // no-swizzle descriptors need 16-byte alignment
    __shared__ uint64_t wfull[2], wfree[2], xfull[MM_XS], xfree[MM_XS], rfull[2], rfree[2], done;
    __shared__ uint32_t s_tmem;
    uint8_t* wsm = smem;                  // [2 slots][hi, lo][WB]
    uint8_t* xsm = smem + 4 * WB;         // [XS slots][hi, lo][MM_XQ_BYTES]
    uint8_t* rsm = xsm + XS * 2 * MM_XQ_BYTES;   // staged: [2 slots][BN rows][RP] raw blocks
    rsm += (128u - (smem_addr(rsm) & 127u)) & 127u;   // RB is a multiple of 128: both slots aligned
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t n0 = blockIdx.x * BN, gtg0 = blockIdx.y * MM_NTG;
    const uint32_t mpad = (m + MM_TG - 1) / MM_TG * MM_TG, ntg = min((uint32_t)MM_NTG, mpad / MM_TG - gtg0);
    // split K: this CTA's K steps [kb0, kb0 + nk) of the kpad / 64; its output
    // (a partial sum when gridDim.z > 1) goes to slice blockIdx.z of y
    const uint32_t nk_all = kpad / MM_BK, kb0 = blockIdx.z * kb_per;
    const uint32_t nk = kb0 < nk_all ? min(kb_per, nk_all - kb0) : 0u;
    y += (size_t)blockIdx.z * m * ldy;
    const uint64_t row_bytes = (uint64_t)(k_cols / BS) * BB;

    if (warp == 8) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&s_tmem)),
                     "r"(TCOLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        for (int i = 0; i < 2; ++i) { mbar_init(&wfull[i], MM_DQ_THREADS); mbar_init(&wfree[i], 1); }
        for (int i = 0; i < 2; ++i) { mbar_init(&rfull[i], 1); mbar_init(&rfree[i], MM_DQ_THREADS); }
        for (int i = 0; i < XS; ++i) { mbar_init(&xfull[i], 1); mbar_init(&xfree[i], 1); }
        mbar_init(&done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    pdl_trigger();
    pdl_wait();

    if (warp < 8) {
        // ---------------- dequantising warps ----------------
        for (uint32_t kb = 0; kb < nk; ++kb) {
            const uint32_t slot = kb & 1, use = kb >> 1;
            if (use > 0) mbar_wait(&wfree[slot], (use - 1) & 1, errf);
            uint8_t* wh = wsm + slot * 2 * WB;
            uint8_t* wl = wh + WB;
            const uint32_t lb = kb / KSTEPS_PER_BLOCK;   // staged: the raw block step of this K step
            if (STAGE && kb % KSTEPS_PER_BLOCK == 0) mbar_wait(&rfull[lb & 1], (lb >> 1) & 1, errf);
            const uint8_t* rblk = rsm + (lb & 1) * RB;
#pragma unroll
            for (uint32_t it = tid; it < (uint32_t)BN * 8; it += MM_DQ_THREADS) {   // BN / 32 independent items
                const uint32_t r = it % BN, kc = it / BN, n = n0 + r, k0 = (kb0 + kb) * MM_BK + kc * 8;
                float v[8];
                if (STAGE) {
                    if (n < n_rows) {
                        // MMS_ROWS: the block sits at its global address's offset in the aligned window
                        const uint32_t off = SM == MMS_ROWS
                                                 ? (uint32_t)(((uint64_t)n * row_bytes + (uint64_t)(k0 / BS) * BB) & 15u)
                                                 : 0u;
                        deq8<DT>(rblk + r * RP + off, (int)(k0 % BS), v);
                    } else {
#pragma unroll
                        for (int j = 0; j < 8; ++j) v[j] = 0.f;
                    }
                } else if (BS >= 8 && n < n_rows && k0 + 8 <= k_cols) {   // the 8 elements share one block
                    deq8<DT>(w + (uint64_t)n * row_bytes + (uint64_t)(k0 / BS) * BB, (int)(k0 % BS), v);
                } else {
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const uint32_t e = k0 + j;
                        v[j] = (n < n_rows && e < k_cols)
                                   ? deq_elem<DT>(w + (uint64_t)n * row_bytes + (uint64_t)(e / BS) * BB, (int)(e % BS))
                                   : 0.f;
                    }
                }
                uint4 h, l;
                split8(v, h, l);
                *reinterpret_cast<uint4*>(wh + kc * (BN * 16) + r * 16) = h;
                *reinterpret_cast<uint4*>(wl + kc * (BN * 16) + r * 16) = l;
            }
            if (STAGE && (kb % KSTEPS_PER_BLOCK == KSTEPS_PER_BLOCK - 1 || kb + 1 == nk))
                mbar_arrive(&rfree[lb & 1]);   // this raw slot is read
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // generic stores -> tensor-core reads
            mbar_arrive(&wfull[slot]);
        }
    } else if (warp == 9 && lane == 0) {
        // ---------------- copy warp ----------------
        // X slot seq = (K step, token group, K quarter), K-step-major; its source is
        // quarter kq of the pre-tiled X tile (token group, K step)
        auto load_x = [&](uint32_t seq) {
            const uint32_t q = seq % XS, kq = seq & 3, tg = (seq >> 2) % ntg, kb = (seq >> 2) / ntg;
            if (seq >= (uint32_t)XS) mbar_wait(&xfree[q], ((seq / XS) - 1) & 1, errf);
            mbar_arrive_expect_tx(&xfull[q], 2 * MM_XQ_BYTES);
            const size_t src = ((size_t)(gtg0 + tg) * nk_all + kb0 + kb) * MM_X_BYTES + kq * MM_XQ_BYTES;
            bulk_g2s(xsm + q * 2 * MM_XQ_BYTES, xh + src, MM_XQ_BYTES, &xfull[q]);
            bulk_g2s(xsm + q * 2 * MM_XQ_BYTES + MM_XQ_BYTES, xl + src, MM_XQ_BYTES, &xfull[q]);
        };
        // staged: raw blocks of block step lb (x = byte offset of the block in a row, y = first row)
        const uint32_t nblk = STAGE ? nk / KSTEPS_PER_BLOCK : 0u;
        auto load_raw = [&](uint32_t lb) {
            const uint32_t q = lb & 1;
            if (lb >= 2) mbar_wait(&rfree[q], ((lb >> 1) - 1) & 1, errf);
            if constexpr (SM == MMS_TMA) {
                mbar_arrive_expect_tx(&rfull[q], RB);
                const int x = (int)((kb0 / KSTEPS_PER_BLOCK + lb) * BB), yrow = (int)n0;
                asm volatile(
                    "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
                    "%3}], [%4];" ::"r"(smem_addr(rsm + q * RB)),
                    "l"(reinterpret_cast<uint64_t>(&wmap)), "r"(x), "r"(yrow), "r"(smem_addr(&rfull[q]))
                    : "memory");
            } else {
                // one RP-byte copy per row from the 16-byte boundary at or below its block
                // (the weight base is 16-byte aligned; the allocation has 16 bytes of slack)
                const uint32_t rows = min((uint32_t)BN, n_rows - n0);
                const uint64_t boff = (uint64_t)(kb0 / KSTEPS_PER_BLOCK + lb) * BB;
                mbar_arrive_expect_tx(&rfull[q], rows * RP);
                for (uint32_t r = 0; r < rows; ++r) {
                    const uint64_t src = ((uint64_t)(n0 + r) * row_bytes + boff) & ~(uint64_t)15;
                    bulk_g2s(rsm + q * RB + r * RP, w + src, RP, &rfull[q]);
                }
            }
        };
        if constexpr (STAGE) {
            for (uint32_t lb = 0; lb < 2 && lb < nblk; ++lb) load_raw(lb);
        } else {
            // the CTA's weight rows into L2 ahead of the dequantising warps: one bulk
            // prefetch per row (16-byte aligned, clipped to the matrix)
            const uintptr_t wend = ((uintptr_t)w + (uint64_t)n_rows * row_bytes) & ~(uintptr_t)15;
            const uint64_t c0 = (uint64_t)(kb0 * MM_BK) / BS * BB;
            const uint64_t c1 = min((uint64_t)((kb0 + nk) * MM_BK + BS - 1) / BS * BB, row_bytes);
            for (uint32_t r = 0; r < (uint32_t)BN && n0 + r < n_rows; ++r) {
                const uintptr_t a = ((uintptr_t)w + (uint64_t)(n0 + r) * row_bytes + c0) & ~(uintptr_t)15;
                uintptr_t e = ((uintptr_t)w + (uint64_t)(n0 + r) * row_bytes + c1 + 15) & ~(uintptr_t)15;
                e = e < wend ? e : wend;
                if (e > a)
                    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a), "r"((uint32_t)(e - a)) : "memory");
            }
        }
        for (uint32_t kb = 0; kb < nk; ++kb) {
            // raw block lb + 1 when K step 4 lb is next: its slot held block lb - 1,
            // which the dequantising warps finished before the MMAs of K step 4 lb - 1
            if (STAGE && kb % KSTEPS_PER_BLOCK == 0 && kb >= KSTEPS_PER_BLOCK && kb / KSTEPS_PER_BLOCK + 1 < nblk)
                load_raw(kb / KSTEPS_PER_BLOCK + 1);
            for (uint32_t i = 0; i < 4 * ntg; ++i) load_x(kb * 4 * ntg + i);
        }
    } else if (warp == 8 && lane == 0) {
        // ---------------- MMA issuer ----------------
        const uint32_t w0 = smem_addr(wsm), x0 = smem_addr(xsm);
        for (uint32_t kb = 0; kb < nk; ++kb) {
            const uint32_t slot = kb & 1;
            mbar_wait(&wfull[slot], (kb >> 1) & 1, errf);
            tc_fence_after();
            const uint32_t wh = w0 + slot * 2 * WB, wl = wh + WB;
            for (uint32_t i = 0; i < 4 * ntg; ++i) {
                const uint32_t seq = kb * 4 * ntg + i, q = seq % XS, kk = i & 3, tg = i >> 2;
                mbar_wait(&xfull[q], (seq / XS) & 1, errf);
                tc_fence_after();
                // A = W rows (16-column step kk of the W slot), B = X tokens (this quarter slot)
                const uint32_t xh_s = x0 + q * 2 * MM_XQ_BYTES, xl_s = xh_s + MM_XQ_BYTES;
                const uint64_t dwh = mm_desc(wh + 2 * kk * (BN * 16), BN * 16, 128);
                const uint64_t dwl = mm_desc(wl + 2 * kk * (BN * 16), BN * 16, 128);
                const uint64_t dxh = mm_desc(xh_s, MM_TG * 16, 128);
                const uint64_t dxl = mm_desc(xl_s, MM_TG * 16, 128);
                const uint32_t d = tmem + tg * MM_TG;
                tc_mma(d, dwh, dxh, IDESC, (kb > 0 || kk > 0) ? 1u : 0u);
                tc_mma(d, dwl, dxh, IDESC, 1u);
                tc_mma(d, dwh, dxl, IDESC, 1u);
                tc_commit(&xfree[q]);
            }
            tc_commit(&wfree[slot]);
        }
        tc_commit(&done);
    }
    // ---------------- epilogue ----------------
    // warp w reads TMEM lanes 32 (w % 4).. (weight rows n0 + 32 (w % 4) + lane) of
    // token group w / 4 in 32-column chunks (tokens); for each token the warp's 32
    // lanes store 32 consecutive floats of its y row (one 128-byte line)
    if (warp < 8) {
        mbar_wait(&done, 0, errf);
        tc_fence_after();
        const uint32_t quarter = warp & 3, tg = warp >> 2;
        const uint32_t n = n0 + quarter * 32 + lane;
        if (tg < ntg) {
#pragma unroll 1
            for (uint32_t c0 = 0; c0 < (uint32_t)MM_TG; c0 += 32) {
                float v[32];
                tc_ld32(tmem + ((quarter * 32) << 16) + tg * MM_TG + c0, v);
                const uint32_t tok0 = (gtg0 + tg) * MM_TG + c0;
#pragma unroll
                for (uint32_t j = 0; j < 32; ++j) {
                    const uint32_t tok = tok0 + j;
                    if (tok < m && n < n_rows) {
                        const size_t idx = (size_t)tok * ldy + n;
                        y[idx] = resid ? __fadd_rn(resid[idx], v[j]) : v[j];
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 8) {
        __syncwarp();   // .sync.aligned: the whole warp, converged
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TCOLS) : "memory");
    }
}

// y[r][c] = (resid[r][c] +) sum over s of part[s][r][c], s in order: the split-K
// partial products of k_mm_tc summed deterministically
__global__ void __launch_bounds__(256) k_mm_reduce(const float* __restrict__ part, uint32_t ks, uint32_t m, uint32_t n,
                                                   float* y, uint32_t ldy, const float* resid) {
    pdl_trigger();
    pdl_wait();
    const uint64_t total = (uint64_t)m * n, slice = (uint64_t)m * n;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t r = i / n, c = i - r * n;
        float v = part[i];
        for (uint32_t s = 1; s < ks; ++s) v = __fadd_rn(v, part[s * slice + i]);
        const size_t idx = (size_t)r * ldy + c;
        y[idx] = resid ? __fadd_rn(resid[idx], v) : v;
    }
}

// k_mm_reduce over float4 columns (n, ldy multiples of 4, every pointer 16-byte
// aligned): the same additions in the same order, four columns per thread, the
// ks loads of a thread independent of one another
__global__ void __launch_bounds__(256) k_mm_reduce4(const float4* __restrict__ part, uint32_t ks, uint32_t m,
                                                    uint32_t n4, float* y, uint32_t ldy, const float* resid) {
    pdl_trigger();
    pdl_wait();
    const uint64_t total = (uint64_t)m * n4, slice = total;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t r = i / n4, c = (i - r * n4) * 4;
        float4 v = __ldcs(part + i);
#pragma unroll 4
        for (uint32_t s = 1; s < ks; ++s) {
            const float4 t = __ldcs(part + s * slice + i);
            v.x = __fadd_rn(v.x, t.x);
            v.y = __fadd_rn(v.y, t.y);
            v.z = __fadd_rn(v.z, t.z);
            v.w = __fadd_rn(v.w, t.w);
        }
        const size_t idx = (size_t)r * ldy + c;
        if (resid) {
            const float4 q = *reinterpret_cast<const float4*>(resid + idx);
            v = make_float4(__fadd_rn(q.x, v.x), __fadd_rn(q.y, v.y), __fadd_rn(q.z, v.z), __fadd_rn(q.w, v.w));
        }
        *reinterpret_cast<float4*>(y + idx) = v;
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
// q head x PA_Q tokens (8 warps x 8 tokens), K/V tiles of PA_KT cache rows in
// shared memory.  Token t (cache slot base + t, position pos[t]) sees the rows
// s < min(pos[t] + 1, base + t + 1), as the decode kernels do.
//   scores: lane l holds keys l and l + 32 of the tile for the warp's 8 tokens;
//     each dot product runs over the head dimension in order (fmaf chain), from
//     float4 loads of K rows (padded by 4 floats: conflict-free) and broadcast q;
//   softmax: online per token (running max / sum, o rescaled per tile), the
//     tile's probabilities through a per-warp shared row;
//   o: lane l owns dimensions [l NI, l NI + NI) of the 8 tokens and adds
//     p . V over the tile's keys in order; o is divided by the sum at the end.
// Token tiles run heaviest (latest) first.  Output o[t][head * hd + i].
constexpr int PA_WARPS = 8, PA_QW = 8, PA_Q = PA_WARPS * PA_QW, PA_KT = 64;
template <int HD>
constexpr size_t pa_smem() {
    return sizeof(float) * ((size_t)PA_Q * HD + (size_t)PA_KT * (HD + 4) + (size_t)PA_KT * HD + (size_t)PA_WARPS * PA_QW * PA_KT);
}
template <int HD>
__global__ void __launch_bounds__(PA_WARPS * 32, 1) k_attn_prefill(const float* __restrict__ q, const void* kc,
                                                                 const void* vc, const int64_t* __restrict__ pos,
                                                                 uint32_t base, uint32_t m, uint32_t n_heads,
                                                                 uint32_t kvh, uint32_t kv_ctx, int kv_f16, float inv,
                                                                 float* __restrict__ o) {
    constexpr int NI = HD / 32, KP = HD + 4;
    static_assert(NI == 2 || NI == 4, "head dim 64 or 128");
    extern __shared__ __align__(16) float pa_sm[];
    float* sq = pa_sm;                       // [PA_Q][HD]
    float* sk = sq + PA_Q * HD;              // [PA_KT][KP]
    float* sv = sk + PA_KT * KP;             // [PA_KT][HD]
    float* sp = sv + PA_KT * HD;             // [warp][PA_QW][PA_KT]
    pdl_trigger();
    pdl_wait();
    const uint32_t head = blockIdx.x, t0 = (gridDim.y - 1 - blockIdx.y) * PA_Q, kvhead = head / (n_heads / kvh);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t qdim = n_heads * HD;
    for (uint32_t i = tid; i < PA_Q * HD / 4; i += blockDim.x) {
        const uint32_t r = i / (HD / 4), c = (i % (HD / 4)) * 4, t = t0 + r;
        const float4 v = t < m ? *reinterpret_cast<const float4*>(q + (size_t)t * qdim + head * HD + c)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4*>(sq + r * HD + c) = v;
    }
    // visible rows per token of this warp, and of the whole CTA
    uint32_t vis[PA_QW];
    uint32_t vmax = 0, vwarp = 0;
#pragma unroll
    for (int k = 0; k < PA_QW; ++k) {
        const uint32_t t = t0 + warp * PA_QW + k;
        uint32_t v = 0;
        if (t < m) {
            const int64_t p = pos[t];
            const uint32_t seq = base + t + 1;
            v = (p + 1 < (int64_t)seq) ? (uint32_t)(p + 1) : seq;
        }
        vis[k] = v;
        vwarp = v > vwarp ? v : vwarp;
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
    const float* sqw = sq + warp * PA_QW * HD;
    float* spw = sp + warp * PA_QW * PA_KT;
    for (uint32_t s0 = 0; s0 < vmax; s0 += PA_KT) {
        __syncthreads();   // previous tile consumed (and sq written, first time)
        for (uint32_t i = tid; i < PA_KT * HD / 4; i += blockDim.x) {
            const uint32_t r = i / (HD / 4), c = (i % (HD / 4)) * 4, s = s0 + r;
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
            if (s < vmax) {
                const uint64_t idx = hb + (uint64_t)s * HD + c;
                if (kv_f16) {
                    const __half* kh = reinterpret_cast<const __half*>(kc) + idx;
                    const __half* vh = reinterpret_cast<const __half*>(vc) + idx;
                    kv = make_float4(__half2float(kh[0]), __half2float(kh[1]), __half2float(kh[2]), __half2float(kh[3]));
                    vv = make_float4(__half2float(vh[0]), __half2float(vh[1]), __half2float(vh[2]), __half2float(vh[3]));
                } else {
                    kv = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(kc) + idx);
                    vv = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(vc) + idx);
                }
            }
            *reinterpret_cast<float4*>(sk + r * KP + c) = kv;
            *reinterpret_cast<float4*>(sv + r * HD + c) = vv;
        }
        __syncthreads();
        if (s0 >= vwarp) continue;   // no key of this tile is visible to the warp's tokens
        // scores of keys s0 + lane and s0 + lane + 32
        float sc[PA_QW][2];
#pragma unroll
        for (int k = 0; k < PA_QW; ++k) sc[k][0] = sc[k][1] = 0.f;
        const float* ka = sk + lane * KP;
        const float* kb = sk + (lane + 32) * KP;
#pragma unroll 2
        for (int d = 0; d < HD; d += 4) {
            const float4 a = *reinterpret_cast<const float4*>(ka + d);
            const float4 b = *reinterpret_cast<const float4*>(kb + d);
#pragma unroll
            for (int k = 0; k < PA_QW; ++k) {
                const float4 qv = *reinterpret_cast<const float4*>(sqw + k * HD + d);
                sc[k][0] = fmaf(qv.x, a.x, sc[k][0]);
                sc[k][0] = fmaf(qv.y, a.y, sc[k][0]);
                sc[k][0] = fmaf(qv.z, a.z, sc[k][0]);
                sc[k][0] = fmaf(qv.w, a.w, sc[k][0]);
                sc[k][1] = fmaf(qv.x, b.x, sc[k][1]);
                sc[k][1] = fmaf(qv.y, b.y, sc[k][1]);
                sc[k][1] = fmaf(qv.z, b.z, sc[k][1]);
                sc[k][1] = fmaf(qv.w, b.w, sc[k][1]);
            }
        }
        // online softmax per token; probabilities into this warp's shared rows
#pragma unroll
        for (int k = 0; k < PA_QW; ++k) {
            const uint32_t sa = s0 + lane, sb = s0 + lane + 32;
            if (s0 >= vis[k]) {   // warp-uniform: no visible key in this tile
                spw[k * PA_KT + lane] = 0.f;
                spw[k * PA_KT + lane + 32] = 0.f;
                continue;
            }
            const float xa = sa < vis[k] ? __fmul_rn(sc[k][0], inv) : -INFINITY;
            const float xb = sb < vis[k] ? __fmul_rn(sc[k][1], inv) : -INFINITY;
            float tmax = fmaxf(xa, xb);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
            const float mnew = fmaxf(mx[k], tmax);
            const float scale = expf(mx[k] - mnew);   // 0 on the first visible tile (mx = -inf)
            const float pa = sa < vis[k] ? expf(xa - mnew) : 0.f;
            const float pb = sb < vis[k] ? expf(xb - mnew) : 0.f;
            float ps = pa + pb;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
            sum[k] = sum[k] * scale + ps;
            mx[k] = mnew;
#pragma unroll
            for (int c = 0; c < NI; ++c) acc[k][c] *= scale;
            spw[k * PA_KT + lane] = pa;
            spw[k * PA_KT + lane + 32] = pb;
        }
        __syncwarp();
        // o += p . V over the tile's keys in order
        const uint32_t kend = min((uint32_t)PA_KT, vmax - s0);
        for (uint32_t j = 0; j < kend; j += 4) {
            float4 p4[PA_QW];
#pragma unroll
            for (int k = 0; k < PA_QW; ++k) p4[k] = *reinterpret_cast<const float4*>(spw + k * PA_KT + j);
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                float vr[NI];
                if constexpr (NI == 4) {
                    const float4 t4 = *reinterpret_cast<const float4*>(sv + (j + jj) * HD + lane * 4);
                    vr[0] = t4.x; vr[1] = t4.y; vr[2] = t4.z; vr[3] = t4.w;
                } else {
                    const float2 t2 = *reinterpret_cast<const float2*>(sv + (j + jj) * HD + lane * 2);
                    vr[0] = t2.x; vr[1] = t2.y;
                }
#pragma unroll
                for (int k = 0; k < PA_QW; ++k) {
                    const float pk = jj == 0 ? p4[k].x : jj == 1 ? p4[k].y : jj == 2 ? p4[k].z : p4[k].w;
#pragma unroll
                    for (int c = 0; c < NI; ++c) acc[k][c] = fmaf(pk, vr[c], acc[k][c]);
                }
            }
        }
        __syncwarp();
    }
#pragma unroll
    for (int k = 0; k < PA_QW; ++k) {
        const uint32_t t = t0 + warp * PA_QW + k;
        if (t >= m) continue;
        const float rs = vis[k] ? 1.0f / sum[k] : 0.f;
        float* dst = o + (size_t)t * qdim + head * HD + lane * NI;
#pragma unroll
        for (int c = 0; c < NI; ++c) dst[c] = acc[k][c] * rs;
    }
}

}  // namespace ggc
