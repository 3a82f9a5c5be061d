// repack.cpp -- host-side split of raw GGUF rows into the plane layout
// (planes.cuh), on host threads with the same per-unit functions the device
// repack (k_repack) runs (repack.cuh).  Used when GGC_REPACK=host.
#include <thread>
#include <vector>

#include "repack.cuh"

namespace ggc {

void repack_rows_host(int dt, const uint8_t* raw, uint64_t rows, uint64_t cols, const uint32_t* row_src,
                      const TileLayout& L, uint8_t* const planes[4], int nthreads) {
    const uint64_t bs = (uint64_t)block_size_of(dt), bb = (uint64_t)block_bytes_of(dt);
    const uint64_t row_bytes = cols / bs * bb;
    const uint64_t upr = rp::units_per_row(dt, L, cols);
    auto work = [&](uint64_t r0, uint64_t r1) {
        for (uint64_t r = r0; r < r1; ++r) {
            const uint8_t* src = raw + (uint64_t)(row_src ? row_src[r] : r) * row_bytes;
            for (uint64_t u = 0; u < upr; ++u) rp::repack_unit(dt, src, r, u, cols, L, planes);
        }
    };
    if (nthreads <= 1 || rows < 64) {
        work(0, rows);
        return;
    }
    std::vector<std::thread> pool;
    for (int t = 0; t < nthreads; ++t) {
        uint64_t r0 = rows * t / nthreads, r1 = rows * (t + 1) / nthreads;
        pool.emplace_back(work, r0, r1);
    }
    for (auto& th : pool) th.join();
}

}  // namespace ggc
