// stream.cu -- instantiations and the cooperative launch of k_stream (its own
// translation unit: the kernels are large and compile in parallel with the rest).
#include "stream.cuh"

namespace ggc {
namespace {

template <int HD, bool F16, int MAXG>
struct StreamKernel {
    static constexpr auto kernel = k_stream<HD, F16, MAXG>;
};

using KernelFn = void (*)(const StreamArgs);

template <int HD, bool F16>
KernelFn pick_g(uint32_t G) {
    if (G == 1) return StreamKernel<HD, F16, 1>::kernel;
    if (G <= 4) return StreamKernel<HD, F16, 4>::kernel;
    if constexpr (HD < 256)
        if (G <= 8) return StreamKernel<HD, F16, 8>::kernel;
    return nullptr;
}

KernelFn pick(uint32_t hd, bool f16, uint32_t G) {
    switch (hd) {
        case 64: return f16 ? pick_g<64, true>(G) : pick_g<64, false>(G);
        case 128: return f16 ? pick_g<128, true>(G) : pick_g<128, false>(G);
        case 256: return f16 ? pick_g<256, true>(G) : pick_g<256, false>(G);
        default: return nullptr;
    }
}

template <int HD, bool F16>
void attn_geom_g(uint32_t G, uint32_t* tile, uint32_t* scratch) {
    auto set = [&](auto cfg, int maxg) {
        using C = decltype(cfg);
        *tile = 2 * C::TILE_BYTES;
        *scratch = (uint32_t)((C::TR * maxg + GS_WARPS * maxg * HD) * sizeof(float));
    };
    if (G == 1) set(FaCfg<HD, F16, 1>{}, 1);
    else if (G <= 4) set(FaCfg<HD, F16, 4>{}, 4);
    else set(FaCfg<HD, F16, 8>{}, 8);
}

}  // namespace

bool stream_supported(uint32_t hd, bool f16, uint32_t G) { return pick(hd, f16, G) != nullptr; }

void stream_attn_geometry(uint32_t hd, bool f16, uint32_t G, uint32_t* tile_bytes, uint32_t* scratch_bytes) {
    *tile_bytes = 0;
    *scratch_bytes = 0;
    if (!stream_supported(hd, f16, G)) return;
    switch (hd) {
        case 64: f16 ? attn_geom_g<64, true>(G, tile_bytes, scratch_bytes) : attn_geom_g<64, false>(G, tile_bytes, scratch_bytes); break;
        case 128: f16 ? attn_geom_g<128, true>(G, tile_bytes, scratch_bytes) : attn_geom_g<128, false>(G, tile_bytes, scratch_bytes); break;
        default: f16 ? attn_geom_g<256, true>(G, tile_bytes, scratch_bytes) : attn_geom_g<256, false>(G, tile_bytes, scratch_bytes); break;
    }
}

cudaError_t stream_prepare(uint32_t hd, bool f16, uint32_t G, size_t smem, int* max_blocks_per_sm) {
    KernelFn k = pick(hd, f16, G);
    if (!k) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(max_blocks_per_sm, k, GS_THREADS, smem);
}

// Cooperative (all CTAs co-resident; their waits on one another need it) and
// without programmatic serialization: the launch starts after its predecessor ends.
cudaError_t stream_launch(uint32_t hd, bool f16, uint32_t G, const StreamArgs& P, unsigned grid, size_t smem,
                          cudaStream_t st) {
    KernelFn k = pick(hd, f16, G);
    if (!k) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(GS_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k, P);
}

}  // namespace ggc
