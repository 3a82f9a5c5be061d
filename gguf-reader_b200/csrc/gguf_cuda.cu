// gguf_cuda.cu -- libgguf_cuda.so: the C ABI declared in include/gguf_cuda.h.
//
// One translation unit holds the context, the quant.rs entry points, device
// tensors and the LlamaModel forward / Engine greedy loop.  Kernels live in the
// included .cuh files.  Built with -fmad=false so that the dequantisers' f32
// arithmetic is never contracted into FMAs (bit-exact with the reference).
#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include <dlfcn.h>
#include <unistd.h>
#include <nccl.h>

#include "common.cuh"
#include "dequant.cuh"
#include "planes.cuh"
#include "repack.cuh"
#include "gemv.cuh"
#include "gemv_span.cuh"
#include "chain.cuh"
#include "attention.cuh"
#include "noalloc.cuh"
#include "prefill.cuh"
#include "sample.cuh"
#include "ops.cuh"

using namespace ggc;

// ===========================================================================
// errors
// ===========================================================================
namespace ggc {
ggc_error_info& tls_error() {
    static thread_local ggc_error_info e;
    return e;
}
int set_error(int status, const char* fmt, ...) {
    ggc_error_info& e = tls_error();
    memset(&e, 0, sizeof(e));
    e.status = status;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(e.message, sizeof(e.message), fmt, ap);
    va_end(ap);
    return status;
}
int set_dequant_error(int dtype, uint64_t expected, uint64_t actual, const char* what) {
    set_error(GGC_ERR_DEQUANT, "DequantError { dtype: %s, expected: %llu, actual: %llu } (%s)", dtype_name(dtype),
              (unsigned long long)expected, (unsigned long long)actual, what);
    ggc_error_info& e = tls_error();
    snprintf(e.dtype, sizeof(e.dtype), "%s", dtype_name(dtype));
    e.expected = expected;
    e.actual = actual;
    return GGC_ERR_DEQUANT;
}
int set_shape_error(uint64_t elements, uint64_t block, const char* what) {
    set_error(GGC_ERR_INVALID_TENSOR_SHAPE, "InvalidTensorShape { elements: %llu, block: %llu } (%s)",
              (unsigned long long)elements, (unsigned long long)block, what);
    tls_error().elements = elements;
    tls_error().block = block;
    return GGC_ERR_INVALID_TENSOR_SHAPE;
}
}  // namespace ggc

// ===========================================================================
// NCCL, loaded on first use (no link-time dependency): the library then shares
// whichever libnccl.so.2 the process already has (e.g. PyTorch's).
// ===========================================================================
namespace {
struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    bool ok = false;
};

NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        api.GetUniqueId = (decltype(api.GetUniqueId))dlsym(h, "ncclGetUniqueId");
        api.CommInitRank = (decltype(api.CommInitRank))dlsym(h, "ncclCommInitRank");
        api.CommDestroy = (decltype(api.CommDestroy))dlsym(h, "ncclCommDestroy");
        api.CommAbort = (decltype(api.CommAbort))dlsym(h, "ncclCommAbort");
        api.CommGetAsyncError = (decltype(api.CommGetAsyncError))dlsym(h, "ncclCommGetAsyncError");
        api.GetErrorString = (decltype(api.GetErrorString))dlsym(h, "ncclGetErrorString");
        api.AllReduce = (decltype(api.AllReduce))dlsym(h, "ncclAllReduce");
        api.AllGather = (decltype(api.AllGather))dlsym(h, "ncclAllGather");
        api.ok = api.GetUniqueId && api.CommInitRank && api.CommDestroy && api.AllReduce && api.AllGather &&
                 api.GetErrorString;
    });
    return api;
}

int nccl_error(const char* what, ncclResult_t r) {
    return set_error(GGC_ERR_NCCL, "%s: %s", what, nccl().GetErrorString ? nccl().GetErrorString(r) : "?");
}

// Host deadline of a wait on work that includes collectives (GGC_NCCL_TIMEOUT_MS,
// default 10 minutes).
double nccl_deadline_ms() {
    const char* e = getenv("GGC_NCCL_TIMEOUT_MS");
    const double v = e ? atof(e) : 0.0;
    return v > 0.0 ? v : 600000.0;
}
}  // namespace

// ===========================================================================
// context
// ===========================================================================
struct ggc_ctx {
    int device = 0;
    int num_sms = 148;
    cudaStream_t stream = nullptr;
    int rank = 0, world = 1;
    ncclComm_t comm = nullptr;
    uint64_t launches = 0;
    // owner + one per live model / tensor: the context outlives everything made on it
    std::atomic<int> refs{1};
    // staging buffers for host arguments (0-2), matmul operands (3-4), split-K
    // partials (5), sampling scratch (6) and the sampler's seen ids + result (7)
    void* stage[8] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
    size_t stage_cap[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int* errf = nullptr;   // device error flags of the context's own launches
    bool comm_failed = false;   // the communicator was aborted (a rank lost or an NCCL error)
};

namespace {

// Waits for the context stream.  Without a communicator: cudaStreamSynchronize.
// With one (tensor parallelism), a rank that died or stalls would leave the others
// blocked in a collective forever, so the stream is polled against a host
// deadline together with ncclCommGetAsyncError; on an NCCL error or expiry the
// communicator is aborted (its kernels in flight return; the fused all-reduce's
// own waits are bounded) and the call fails with GGC_ERR_NCCL.  The context's
// collectives fail from then on.
// Waits for the context stream, or with `ev` only for the work queued before that
// event was recorded.
int ctx_sync(ggc_ctx* ctx, cudaEvent_t ev = nullptr) {
    if (ctx->comm_failed) return set_error(GGC_ERR_NCCL, "communicator aborted earlier (a rank was lost)");
    if (!ctx->comm) {
        GGC_CUDA_TRY(ev ? cudaEventSynchronize(ev) : cudaStreamSynchronize(ctx->stream));
        return GGC_OK;
    }
    const auto t0 = std::chrono::steady_clock::now();
    for (uint64_t it = 0;; ++it) {
        const cudaError_t e = ev ? cudaEventQuery(ev) : cudaStreamQuery(ctx->stream);
        if (e == cudaSuccess) return GGC_OK;
        if (e != cudaErrorNotReady) return set_error(GGC_ERR_CUDA, "stream: %s", cudaGetErrorString(e));
        ncclResult_t ar = ncclSuccess;
        const bool async_err = nccl().CommGetAsyncError && nccl().CommGetAsyncError(ctx->comm, &ar) == ncclSuccess &&
                               ar != ncclSuccess && ar != ncclInProgress;
        const double ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
        if (async_err || ms > nccl_deadline_ms()) {
            if (nccl().CommAbort) nccl().CommAbort(ctx->comm);
            ctx->comm = nullptr;
            ctx->comm_failed = true;
            if (async_err) return nccl_error("NCCL asynchronous error (communicator aborted)", ar);
            return set_error(GGC_ERR_NCCL, "no progress within %.0f ms: a rank lost? (communicator aborted)", ms);
        }
        if (it > 2000) std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

bool is_device_ptr(const void* p) {
    if (!p) return false;
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged;
}

int ensure_stage(ggc_ctx* ctx, int i, size_t bytes) {
    if (ctx->stage_cap[i] >= bytes) return GGC_OK;
    GGC_TRY(ctx_sync(ctx));
    if (ctx->stage[i]) cudaFree(ctx->stage[i]);
    ctx->stage[i] = nullptr;
    ctx->stage_cap[i] = 0;
    size_t cap = bytes < 4096 ? 4096 : bytes;
    GGC_CUDA_TRY(cudaMalloc(&ctx->stage[i], cap));
    ctx->stage_cap[i] = cap;
    return GGC_OK;
}

// Device view of a caller argument: device pointers pass through, host data is
// copied into staging buffer `i`.
int dev_in(ggc_ctx* ctx, int i, const void* p, size_t bytes, const void** out) {
    if (is_device_ptr(p) || bytes == 0) { *out = p; return GGC_OK; }
    GGC_TRY(ensure_stage(ctx, i, bytes));
    GGC_CUDA_TRY(cudaMemcpyAsync(ctx->stage[i], p, bytes, cudaMemcpyHostToDevice, ctx->stream));
    *out = ctx->stage[i];
    return GGC_OK;
}
int dev_out(ggc_ctx* ctx, int i, void* p, size_t bytes, void** out, bool* staged) {
    *staged = !is_device_ptr(p);
    if (!*staged) { *out = p; return GGC_OK; }
    GGC_TRY(ensure_stage(ctx, i, bytes));
    *out = ctx->stage[i];
    return GGC_OK;
}

// Launch with programmatic stream serialization (PDL): the next kernel may be
// scheduled while this one drains; every kernel calls griddepcontrol.wait.
template <class... KArgs, class... Args>
cudaError_t launch(ggc_ctx* ctx, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    ctx->launches++;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

int host_threads() {
    unsigned h = std::thread::hardware_concurrency();
    return h ? (int)(h > 32 ? 32 : h) : 4;
}

}  // namespace

// ===========================================================================
// quant.rs entry points
// ===========================================================================
namespace {

template <int DT>
struct RunDequant {
    static void run(ggc_ctx* ctx, const uint8_t* raw, uint64_t n, float* out, cudaError_t* err) {
        uint64_t blocks = cdiv<uint64_t>(n, 256);
        unsigned grid = (unsigned)(blocks < (uint64_t)ctx->num_sms * 16 ? blocks : (uint64_t)ctx->num_sms * 16);
        if (grid == 0) grid = 1;
        *err = launch(ctx, k_dequantize<DT>, dim3(grid), dim3(256), 0, raw, n, out);
    }
};

template <int DT>
struct RunMatvecRaw {
    static void run(ggc_ctx* ctx, const uint8_t* w, uint64_t rows, uint64_t cols, const float* x, float* y,
                    cudaError_t* err) {
        uint64_t ctas = cdiv<uint64_t>(rows, 8);
        unsigned grid = (unsigned)(ctas < (uint64_t)ctx->num_sms * 8 ? ctas : (uint64_t)ctx->num_sms * 8);
        if (grid == 0) grid = 1;
        *err = launch(ctx, k_matvec_raw<DT>, dim3(grid), dim3(256), 0, w, rows, cols, x, y);
    }
};

}  // namespace

extern "C" int ggc_last_error(ggc_error_info* out) {
    if (out) *out = tls_error();
    return tls_error().status;
}

extern "C" int64_t ggc_block_size(int dtype) { return block_size_of(dtype); }
extern "C" int64_t ggc_block_bytes(int dtype) { return block_bytes_of(dtype); }

extern "C" int ggc_nccl_unique_id(void* out128) {
    if (!out128) return set_error(GGC_ERR_INVALID_ARG, "null id buffer");
    if (!nccl().ok) return set_error(GGC_ERR_NCCL, "libnccl.so.2 not loadable");
    ncclUniqueId id;
    ncclResult_t r = nccl().GetUniqueId(&id);
    if (r != ncclSuccess) return nccl_error("ncclGetUniqueId", r);
    memcpy(out128, &id, sizeof(id));
    return GGC_OK;
}

static int ctx_init(ggc_ctx* c, int device) {
    int n = 0;
    GGC_CUDA_TRY(cudaGetDeviceCount(&n));
    if (device < 0 || device >= n) return set_error(GGC_ERR_INVALID_ARG, "device %d out of range (%d GPUs)", device, n);
    c->device = device;
    DeviceGuard g(device);
    GGC_CUDA_TRY(cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, device));
    GGC_CUDA_TRY(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
    return GGC_OK;
}

extern "C" int ggc_ctx_create(int device, ggc_ctx** out) {
    if (!out) return set_error(GGC_ERR_INVALID_ARG, "null out");
    std::unique_ptr<ggc_ctx> c(new ggc_ctx());
    GGC_TRY(ctx_init(c.get(), device));
    *out = c.release();
    return GGC_OK;
}

extern "C" int ggc_ctx_create_tp(int device, int rank, int world, const void* nccl_id, ggc_ctx** out) {
    if (!out || !nccl_id || world < 1 || rank < 0 || rank >= world)
        return set_error(GGC_ERR_INVALID_ARG, "bad tensor-parallel arguments");
    std::unique_ptr<ggc_ctx> c(new ggc_ctx());
    GGC_TRY(ctx_init(c.get(), device));
    c->rank = rank;
    c->world = world;
    if (world > 1) {
        DeviceGuard g(device);
        if (!nccl().ok) return set_error(GGC_ERR_NCCL, "libnccl.so.2 not loadable");
        ncclUniqueId id;
        memcpy(&id, nccl_id, sizeof(id));
        ncclResult_t r = nccl().CommInitRank(&c->comm, world, id, rank);
        if (r != ncclSuccess) return nccl_error("ncclCommInitRank", r);
    }
    *out = c.release();
    return GGC_OK;
}

namespace {
void ctx_release(ggc_ctx* ctx) {
    if (ctx->refs.fetch_sub(1) != 1) return;
    {
        DeviceGuard g(ctx->device);
        cudaStreamSynchronize(ctx->stream);
        for (int i = 0; i < 8; ++i)
            if (ctx->stage[i]) cudaFree(ctx->stage[i]);
        if (ctx->errf) cudaFree(ctx->errf);
        if (ctx->comm) nccl().CommDestroy(ctx->comm);
        cudaStreamDestroy(ctx->stream);
    }
    delete ctx;
}
}  // namespace

// Releases the caller's reference; the context is freed once the models and
// tensors made on it are destroyed too (in any order).
extern "C" int ggc_ctx_destroy(ggc_ctx* ctx) {
    if (ctx) ctx_release(ctx);
    return GGC_OK;
}

extern "C" void* ggc_ctx_stream(ggc_ctx* ctx) { return ctx ? (void*)ctx->stream : nullptr; }
extern "C" uint64_t ggc_ctx_kernel_launches(ggc_ctx* ctx) { return ctx ? ctx->launches : 0; }

extern "C" int ggc_ctx_synchronize(ggc_ctx* ctx) {
    if (!ctx) return set_error(GGC_ERR_INVALID_ARG, "null ctx");
    DeviceGuard g(ctx->device);
    GGC_TRY(ctx_sync(ctx));
    return GGC_OK;
}

// quant.rs:403-448
extern "C" int ggc_dequantize(ggc_ctx* ctx, int dtype, const void* raw, uint64_t raw_len, uint64_t n, float* out) {
    const int bs = block_size_of(dtype);
    if (bs < 0) return set_dequant_error(dtype, 0, 0, "unsupported dtype");
    if (n % (uint64_t)bs != 0) return set_shape_error(n, (uint64_t)bs, "dequantize");
    const uint64_t need = n / bs * (uint64_t)block_bytes_of(dtype);
    if (raw_len < need) return set_dequant_error(dtype, need, raw_len, "data shorter than tensor");
    if (n == 0) return GGC_OK;
    if (!ctx) return set_error(GGC_ERR_INVALID_ARG, "null ctx");
    if (!raw || !out) return set_error(GGC_ERR_INVALID_ARG, "null buffer");
    DeviceGuard g(ctx->device);
    const void* draw;
    void* dout;
    bool staged;
    GGC_TRY(dev_in(ctx, 0, raw, need, &draw));
    GGC_TRY(dev_out(ctx, 1, out, n * sizeof(float), &dout, &staged));
    cudaError_t err = cudaSuccess;
    dispatch_dtype<RunDequant>(dtype, ctx, (const uint8_t*)draw, n, (float*)dout, &err);
    GGC_CUDA_TRY(err);
    if (staged) {
        GGC_CUDA_TRY(cudaMemcpyAsync(out, dout, n * sizeof(float), cudaMemcpyDeviceToHost, ctx->stream));
        GGC_TRY(ctx_sync(ctx));
    }
    return GGC_OK;
}

// quant.rs:526-570 (checks in the order of :534-555)
extern "C" int ggc_quant_matvec(ggc_ctx* ctx, int dtype, const void* w, uint64_t w_len, uint64_t rows, uint64_t cols,
                                const float* x, uint64_t x_len, float* y, uint64_t y_len) {
    const int bs = block_size_of(dtype), bb = block_bytes_of(dtype);
    if (bs < 0 || bb < 0) return set_dequant_error(dtype, 0, 0, "unsupported dtype");
    if (cols % (uint64_t)bs != 0) return set_shape_error(cols, (uint64_t)bs, "row_bytes");
    const uint64_t rb = cols / bs * (uint64_t)bb;
    if (x_len != cols) return set_dequant_error(dtype, cols, x_len, "x length != cols");
    if (y_len != rows) return set_dequant_error(dtype, rows, y_len, "y length != rows");
    if (rows * rb > w_len) return set_dequant_error(dtype, rows * rb, w_len, "w shorter than rows*row_bytes");
    if (rows == 0) return GGC_OK;
    if (!ctx) return set_error(GGC_ERR_INVALID_ARG, "null ctx");
    if (!w || !y || (!x && cols)) return set_error(GGC_ERR_INVALID_ARG, "null buffer");
    DeviceGuard g(ctx->device);
    const void *dw, *dx;
    void* dy;
    bool staged;
    GGC_TRY(dev_in(ctx, 0, w, rows * rb, &dw));
    GGC_TRY(dev_in(ctx, 1, x, cols * sizeof(float), &dx));
    GGC_TRY(dev_out(ctx, 2, y, rows * sizeof(float), &dy, &staged));
    cudaError_t err = cudaSuccess;
    dispatch_dtype<RunMatvecRaw>(dtype, ctx, (const uint8_t*)dw, rows, cols, (const float*)dx, (float*)dy, &err);
    GGC_CUDA_TRY(err);
    if (staged) {
        GGC_CUDA_TRY(cudaMemcpyAsync(y, dy, rows * sizeof(float), cudaMemcpyDeviceToHost, ctx->stream));
        GGC_TRY(ctx_sync(ctx));
    }
    return GGC_OK;
}

// ---------------------------------------------------------------------------
// ggc_quant_matvec_static: the same product as ggc_quant_matvec over device
// buffers, split over columns, with its scratch in g_noalloc_scratch.  It calls
// no allocating routine: the first call on a device looks the scratch up with
// cudaGetSymbolAddress (device current) and caches the pointer; every call then
// clears the tickets it uses and launches on the caller's stream.
// ---------------------------------------------------------------------------
namespace {

constexpr int NOALLOC_MAX_DEVICES = 64;

int noalloc_scratch(int dev, unsigned char** out) {
    static std::mutex mu;
    static unsigned char* ptr[NOALLOC_MAX_DEVICES] = {};
    if (dev < 0 || dev >= NOALLOC_MAX_DEVICES) return set_error(GGC_ERR_INVALID_ARG, "device %d out of range", dev);
    std::lock_guard<std::mutex> lk(mu);
    if (!ptr[dev]) {
        void* p = nullptr;
        GGC_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
        ptr[dev] = static_cast<unsigned char*>(p);
    }
    *out = ptr[dev];
    return GGC_OK;
}

template <int DT>
struct RunMatvecSplitK {
    static void run(const uint8_t* w, uint64_t rows, uint64_t cols, const float* x, float* y, dim3 grid,
                    uint32_t nsplit, uint64_t per, unsigned char* scratch, cudaStream_t st, cudaError_t* err) {
        k_matvec_raw_splitk<DT><<<grid, 256, 0, st>>>(w, rows, cols, x, y, nsplit, per, scratch);
        *err = cudaGetLastError();
    }
};

}  // namespace

extern "C" int ggc_quant_matvec_static(int dtype, const void* w, uint64_t w_len, uint64_t rows, uint64_t cols,
                                       const float* x, uint64_t x_len, float* y, uint64_t y_len, void* stream) {
    const int bs = block_size_of(dtype), bb = block_bytes_of(dtype);
    if (bs < 0 || bb < 0) return set_dequant_error(dtype, 0, 0, "unsupported dtype");
    if (cols % (uint64_t)bs != 0) return set_shape_error(cols, (uint64_t)bs, "row_bytes");
    const uint64_t rb = cols / bs * (uint64_t)bb;
    if (x_len != cols) return set_dequant_error(dtype, cols, x_len, "x length != cols");
    if (y_len != rows) return set_dequant_error(dtype, rows, y_len, "y length != rows");
    if (rows * rb > w_len) return set_dequant_error(dtype, rows * rb, w_len, "w shorter than rows*row_bytes");
    if (rows > NOALLOC_MAX_ROWS)
        return set_error(GGC_ERR_INVALID_ARG, "rows %llu exceed the static scratch (at most %llu rows)",
                         (unsigned long long)rows, (unsigned long long)NOALLOC_MAX_ROWS);
    if (rows == 0) return GGC_OK;
    if (!w || !y || (!x && cols)) return set_error(GGC_ERR_INVALID_ARG, "null buffer");
    if (!is_device_ptr(w) || !is_device_ptr(y) || (cols && !is_device_ptr(x)))
        return set_error(GGC_ERR_INVALID_ARG, "w, x and y must be device buffers");
    int dev = 0, sms = 148;
    GGC_CUDA_TRY(cudaGetDevice(&dev));
    GGC_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    unsigned char* scratch = nullptr;
    GGC_TRY(noalloc_scratch(dev, &scratch));
    // enough CTAs for ~8 per SM, at most NOALLOC_MAX_SPLIT splits, partials in scratch
    const uint64_t groups = cdiv<uint64_t>(rows, NOALLOC_ROWS_PER_CTA), nblk = cols / bs;
    uint64_t ns = cdiv<uint64_t>((uint64_t)sms * 8, groups);
    if (ns > NOALLOC_MAX_SPLIT) ns = NOALLOC_MAX_SPLIT;
    if (ns > NOALLOC_MAX_PARTIALS / rows) ns = NOALLOC_MAX_PARTIALS / rows;
    if (ns > nblk) ns = nblk;
    if (ns < 1) ns = 1;
    const uint64_t per = cdiv<uint64_t>(nblk ? nblk : 1, ns);
    ns = cdiv<uint64_t>(nblk ? nblk : 1, per);   // no empty split
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    GGC_CUDA_TRY(cudaMemsetAsync(scratch, 0, groups * sizeof(uint32_t), st));
    cudaError_t err = cudaSuccess;
    dispatch_dtype<RunMatvecSplitK>(dtype, (const uint8_t*)w, rows, cols, x, y, dim3((unsigned)groups, (unsigned)ns),
                                    (uint32_t)ns, per, scratch, st, &err);
    GGC_CUDA_TRY(err);
    return GGC_OK;
}

// model/llama.rs:656-710
extern "C" int ggc_infer_k_quant_dtype(uint64_t span, uint64_t n, int marked) {
    switch (marked) {
        case GGC_Q4_0: case GGC_Q4_1: case GGC_Q5_0: case GGC_Q5_1: case GGC_Q8_0: case GGC_Q2_K:
        case GGC_Q3_K_S: case GGC_Q3_K_M: case GGC_Q3_K_L: case GGC_Q4_K: case GGC_Q5_K:
        case GGC_Q6_K: case GGC_Q8_K: break;
        default: return -1;
    }
    if (n == 0) return -1;
    const int bs = block_size_of(marked);
    const uint64_t blocks = bs == 32 ? n / 32 : n / 256;
    if (blocks == 0) return -1;
    const uint64_t per256 = bs == 32 ? span * 8 / blocks : span / blocks;
    if (span % blocks > 256) return -1;
    static const struct { uint64_t b; int dt; } table[] = {{84, GGC_Q2_K}, {110, GGC_Q3_K_S}, {114, GGC_Q3_K_M},
                                                            {144, GGC_Q4_K}, {176, GGC_Q5_K}, {210, GGC_Q6_K},
                                                            {292, GGC_Q8_K}};
    for (auto& e : table)
        if (e.b == per256) return e.dt;
    return -1;
}

// ===========================================================================
// device tensors in plane layout
// ===========================================================================
struct DevMat {
    int dtype = -1;
    uint32_t rows = 0, cols = 0;      // cols padded to the chunk width for float formats
    uint32_t xcols = 0;               // logical cols
    uint8_t* base = nullptr;          // one allocation holding all planes
    QMat q{};
    uint64_t bytes = 0;
};

namespace {

void free_mat(DevMat& m) {
    if (m.base) cudaFree(m.base);
    m.base = nullptr;
}

int chunk_elems(int dt) { return plane_spec(dt).chunk_elems; }

// Raw rows (in output order, contiguous) into the zeroed planes: one thread per
// (row, unit) of the layout, the same per-unit split the host repack runs
// (repack.cuh), so the planes are the host's byte for byte.
__global__ void __launch_bounds__(256) k_repack(int dt, const uint8_t* __restrict__ raw, uint64_t rows, uint64_t cols,
                                                uint64_t row_bytes, TileLayout L, uint8_t* p0, uint8_t* p1, uint8_t* p2,
                                                uint8_t* p3) {
    pdl_wait();
    uint8_t* const planes[4] = {p0, p1, p2, p3};
    const uint64_t upr = rp::units_per_row(dt, L, cols), n = rows * upr;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t r = i / upr, u = i % upr;
        rp::repack_unit(dt, raw + r * row_bytes, r, u, cols, L, planes);
    }
}

bool host_repack() {
    const char* e = getenv("GGC_REPACK");
    return e && strcmp(e, "host") == 0;
}

// Splits raw rows into planes and uploads them.  Default: the raw rows go to the
// GPU (gathered in output order on the host when row_src selects or reorders
// them) and k_repack splits them there; GGC_REPACK=host splits them on host
// threads and uploads the planes.  `raw` is host memory, or device memory when
// row_src is null and the split runs on the GPU.
int upload_mat(ggc_ctx* ctx, const void* raw, uint64_t raw_bytes, int dt, uint64_t rows, uint64_t cols,
               const uint32_t* row_src, DevMat& out) {
    const int bs = block_size_of(dt), bb = block_bytes_of(dt);
    PlaneSpec ps = plane_spec(dt);
    if (bs < 0 || ps.n == 0) return set_dequant_error(dt, 0, 0, "unsupported dtype");
    if (cols % (uint64_t)bs != 0) return set_shape_error(cols, bs, "matrix columns");
    const uint64_t E = (uint64_t)chunk_elems(dt);
    uint64_t pcols = cols;
    if (is_span_dt(dt)) {
        pcols = (cols + SPAN - 1) / SPAN * SPAN;   // zero-padded spans
    } else if (cols % E != 0) {
        if (bs != 1) return set_shape_error(cols, E, "matrix columns (chunk)");
        pcols = (cols + E - 1) / E * E;
    }
    const uint64_t row_bytes = cols / bs * (uint64_t)bb;
    if (raw_bytes < rows * row_bytes) return set_dequant_error(dt, rows * row_bytes, raw_bytes, "tensor data too short");
    if (rows == 0 || rows > 0xFFFFFFFFull || pcols > 0xFFFFFFFFull) return set_error(GGC_ERR_INVALID_ARG, "matrix shape");
    const TileLayout L = make_layout(dt, (uint32_t)rows, (uint32_t)pcols);
    uint64_t off[4] = {0, 0, 0, 0}, total = 0;
    if (is_span_dt(dt)) ps.n = span_spec(dt).n;
    for (int p = 0; p < ps.n; ++p) {
        off[p] = total;
        total += ((uint64_t)L.nrb * L.rb_bytes[p] + 255) / 256 * 256;
    }
    DevMat m;
    m.dtype = dt;
    m.rows = (uint32_t)rows;
    m.cols = (uint32_t)pcols;
    m.xcols = (uint32_t)cols;
    m.bytes = total;
    GGC_CUDA_TRY(cudaMalloc(&m.base, total));
    cudaError_t e = cudaSuccess;
    if (host_repack()) {
        std::vector<uint8_t> host(total, 0);
        uint8_t* planes[4] = {nullptr, nullptr, nullptr, nullptr};
        for (int p = 0; p < ps.n; ++p) planes[p] = host.data() + off[p];
        repack_rows_host(dt, (const uint8_t*)raw, rows, cols, row_src, L, planes, host_threads());
        e = cudaMemcpyAsync(m.base, host.data(), total, cudaMemcpyHostToDevice, ctx->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    } else {
        const uint8_t* src = (const uint8_t*)raw;
        std::vector<uint8_t> gathered;
        if (row_src) {
            gathered.resize(rows * row_bytes);
            for (uint64_t r = 0; r < rows; ++r)
                memcpy(gathered.data() + r * row_bytes, src + (uint64_t)row_src[r] * row_bytes, row_bytes);
            src = gathered.data();
        }
        uint8_t* draw = nullptr;
        e = cudaMalloc(&draw, rows * row_bytes);
        if (e == cudaSuccess) e = cudaMemsetAsync(m.base, 0, total, ctx->stream);
        if (e == cudaSuccess) e = cudaMemcpyAsync(draw, src, rows * row_bytes, cudaMemcpyDefault, ctx->stream);
        if (e == cudaSuccess) {
            const uint64_t n = rows * rp::units_per_row(dt, L, cols);
            const uint64_t grid = std::min<uint64_t>((n + 255) / 256, (uint64_t)ctx->num_sms * 16);
            uint8_t* pp[4];
            for (int p = 0; p < 4; ++p) pp[p] = p < ps.n ? m.base + off[p] : nullptr;
            e = launch(ctx, k_repack, dim3((unsigned)grid), dim3(256), 0, dt, (const uint8_t*)draw, rows, cols, row_bytes,
                       L, pp[0], pp[1], pp[2], pp[3]);
        }
        if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
        if (draw) {
            const cudaError_t f = cudaFree(draw);
            if (e == cudaSuccess) e = f;
        }
    }
    if (e != cudaSuccess) {
        cudaFree(m.base);
        return set_error(GGC_ERR_CUDA, "upload: %s", cudaGetErrorString(e));
    }
    for (int p = 0; p < 4; ++p) m.q.p[p] = p < ps.n ? m.base + off[p] : nullptr;
    m.q.L = L;
    out = m;
    return GGC_OK;
}

constexpr size_t GEMV_SMEM_LIMIT = 227 * 1024 - 4096;   // dynamic shared bytes per CTA (static use < 4 KB)

template <int DT>
struct SetGemvSmem {
    static void run(int* ok) {
        cudaError_t e;
        if constexpr (is_span_dt(DT))
            e = cudaFuncSetAttribute(k_gemv_span<DT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GEMV_SMEM_LIMIT);
        else
            e = cudaFuncSetAttribute(k_gemv<DT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GEMV_SMEM_LIMIT);
        if (e != cudaSuccess) *ok = 0;
    }
};

// Every k_attn_decode instantiation (head dim 64/128/256, f32/f16 cache, group
// bound 1/4/8) with its dynamic shared memory.
template <int HD, bool F16, int MAXG>
struct AttnDecodeKernel {
    static constexpr auto kernel = k_attn_decode<HD, F16, MAXG>;
    static constexpr size_t smem = FaCfg<HD, F16, MAXG>::SMEM;
};
// group bound 8 at hd 256 would hold 128 registers of q and accumulators alone:
// that shape takes the general pair
template <int HD>
constexpr bool attn_decode_g8 = HD < 256;
template <int HD, bool F16, class F>
void for_each_attn_decode_g(F& f) {
    f(AttnDecodeKernel<HD, F16, 1>::kernel, AttnDecodeKernel<HD, F16, 1>::smem);
    f(AttnDecodeKernel<HD, F16, 4>::kernel, AttnDecodeKernel<HD, F16, 4>::smem);
    if constexpr (attn_decode_g8<HD>) f(AttnDecodeKernel<HD, F16, 8>::kernel, AttnDecodeKernel<HD, F16, 8>::smem);
}
template <class F>
void for_each_attn_decode(F&& f) {
    for_each_attn_decode_g<64, false>(f); for_each_attn_decode_g<64, true>(f);
    for_each_attn_decode_g<128, false>(f); for_each_attn_decode_g<128, true>(f);
    for_each_attn_decode_g<256, false>(f); for_each_attn_decode_g<256, true>(f);
}

// The k_attn_decode instantiation for (hd, f16 cache, group), or null when the
// shape needs the general k_attn_scores / k_attn_av pair.
struct AttnDecodeSel {
    void (*kernel)(const AttnArgs) = nullptr;
    size_t smem = 0;
};
template <int HD, bool F16>
AttnDecodeSel attn_decode_sel_g(uint32_t G) {
    if (G == 1) return {AttnDecodeKernel<HD, F16, 1>::kernel, AttnDecodeKernel<HD, F16, 1>::smem};
    if (G <= 4) return {AttnDecodeKernel<HD, F16, 4>::kernel, AttnDecodeKernel<HD, F16, 4>::smem};
    if constexpr (attn_decode_g8<HD>)
        if (G <= 8) return {AttnDecodeKernel<HD, F16, 8>::kernel, AttnDecodeKernel<HD, F16, 8>::smem};
    return {};
}
AttnDecodeSel attn_decode_sel(uint32_t hd, bool f16, uint32_t G) {
    switch (hd) {
        case 64: return f16 ? attn_decode_sel_g<64, true>(G) : attn_decode_sel_g<64, false>(G);
        case 128: return f16 ? attn_decode_sel_g<128, true>(G) : attn_decode_sel_g<128, false>(G);
        case 256: return f16 ? attn_decode_sel_g<256, true>(G) : attn_decode_sel_g<256, false>(G);
        default: return {};
    }
}

// Kernel attributes are per device: set once for every device a context runs on
// (the caller's device guard makes it current).
constexpr int GGC_MAX_DEVICES = 64;
int current_device() {
    int d = -1;
    return cudaGetDevice(&d) == cudaSuccess && d >= 0 && d < GGC_MAX_DEVICES ? d : -1;
}

int init_kernel_attrs() {
    static std::once_flag once_dev[GGC_MAX_DEVICES];
    static int ok_dev[GGC_MAX_DEVICES];
    const int dev = current_device();
    if (dev < 0) return set_error(GGC_ERR_CUDA, "no current device below %d", GGC_MAX_DEVICES);
    int& ok = ok_dev[dev];
    std::call_once(once_dev[dev], [&ok] {
        ok = 1;
        const int dts[] = {GGC_F32, GGC_F16, GGC_BF16, GGC_Q4_0, GGC_Q4_1, GGC_Q5_0, GGC_Q5_1, GGC_Q8_0,
                           GGC_Q2_K, GGC_Q3_K_S, GGC_Q3_K_M, GGC_Q3_K_L, GGC_Q4_K, GGC_Q5_K, GGC_Q6_K, GGC_Q8_K};
        for (int dt : dts) dispatch_dtype<SetGemvSmem>(dt, &ok);
        if (cudaFuncSetAttribute(k_attn_av, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024) != cudaSuccess) ok = 0;
        for (uint32_t mask = 1; mask < 16; ++mask)
            if (cudaFuncSetAttribute(chain_kernel(mask), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)GEMV_SMEM_LIMIT) != cudaSuccess)
                ok = 0;
        if (cudaFuncSetAttribute(k_attn_prefill<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pa_smem<64>()) !=
                cudaSuccess ||
            cudaFuncSetAttribute(k_attn_prefill<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pa_smem<128>()) !=
                cudaSuccess)
            ok = 0;
        for_each_attn_decode([&ok](auto kernel, size_t smem) {
            if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) ok = 0;
        });
    });
    if (!ok) return set_error(GGC_ERR_CUDA, "cudaFuncSetAttribute failed");
    return GGC_OK;
}

// One k_gemv launch over up to three same-dtype segments.
struct GemvLaunch {
    GemvArgs a{};
    int dtype = -1;
    uint32_t xcols = 0;
};

template <int DT>
struct RunGemv {
    static void run(ggc_ctx* ctx, const GemvArgs* a, cudaError_t* err) {
        uint32_t total_rb = 0;
        for (int i = 0; i < a->nseg; ++i) total_rb += a->seg[i].m.L.nrb;
        uint32_t ctas = total_rb < (uint32_t)ctx->num_sms ? total_rb : (uint32_t)ctx->num_sms;
        if (ctas == 0) ctas = 1;
        if constexpr (is_span_dt(DT)) {
            const SpanCfg c = make_span_cfg<DT>(a->cols, total_rb, ctas, GEMV_SMEM_LIMIT);
            if (c.stages < 2) { *err = cudaErrorInvalidConfiguration; return; }
            *err = launch(ctx, k_gemv_span<DT>, dim3(ctas), dim3(GS_THREADS), c.smem, *a, c);
        } else {
            const TileCfg tc = make_tile_cfg<DT>(a->cols, GEMV_SMEM_LIMIT);
            if (tc.stages < 2) { *err = cudaErrorInvalidConfiguration; return; }
            *err = launch(ctx, k_gemv<DT>, dim3(ctas), dim3(GEMV_THREADS), gemv_smem_bytes(tc), *a, tc);
        }
    }
};

int run_gemv(ggc_ctx* ctx, int dt, const GemvArgs& a) {
    cudaError_t err = cudaSuccess;
    if (!dispatch_dtype<RunGemv>(dt, ctx, &a, &err)) return set_dequant_error(dt, 0, 0, "gemv dtype");
    GGC_CUDA_TRY(err);
    return GGC_OK;
}

Seg make_seg(const DevMat& m, int epi, float* out, void* cache, const float* bias) {
    Seg s{};
    s.m = m.q;
    s.epi = epi;
    s.out = out;
    s.cache = cache;
    s.bias = bias;
    return s;
}

}  // namespace

struct ggc_tensor {
    ggc_ctx* ctx = nullptr;
    int dtype = -1;
    uint64_t ne[4] = {1, 1, 1, 1};
    int ndim = 0;
    bool repacked = false;
    DevMat mat;               // repacked planes
    uint8_t* raw = nullptr;   // raw bytes when not repacked
    uint64_t raw_bytes = 0;
    uint64_t n_elements = 0;
};

extern "C" int ggc_tensor_upload(ggc_ctx* ctx, const void* raw, uint64_t bytes, int dtype, const uint64_t* ne, int ndim,
                                 int repack, ggc_tensor** out) {
    if (!ctx || !raw || !ne || !out || ndim < 1 || ndim > 4) return set_error(GGC_ERR_INVALID_ARG, "bad upload arguments");
    const int bs = block_size_of(dtype), bb = block_bytes_of(dtype);
    if (bs < 0) return set_dequant_error(dtype, 0, 0, "unsupported dtype");
    DeviceGuard g(ctx->device);
    GGC_TRY(init_kernel_attrs());
    std::unique_ptr<ggc_tensor> t(new ggc_tensor());
    t->ctx = ctx;
    t->dtype = dtype;
    t->ndim = ndim;
    uint64_t n = 1;
    for (int i = 0; i < ndim; ++i) { t->ne[i] = ne[i]; n *= ne[i]; }
    t->n_elements = n;
    if (n % (uint64_t)bs != 0) return set_shape_error(n, bs, "tensor elements");
    const uint64_t need = n / bs * (uint64_t)bb;
    if (bytes < need) return set_dequant_error(dtype, need, bytes, "tensor data too short");
    const uint64_t cols = ne[0], rows = n / (cols ? cols : 1);
    if (repack) {
        GGC_TRY(upload_mat(ctx, raw, bytes, dtype, rows, cols, nullptr, t->mat));
        t->repacked = true;
    } else {
        GGC_CUDA_TRY(cudaMalloc(&t->raw, need + 16));   // 16 bytes of slack: the product's aligned row windows
        GGC_CUDA_TRY(cudaMemcpyAsync(t->raw, raw, need, cudaMemcpyDefault, ctx->stream));
        GGC_TRY(ctx_sync(ctx));
        t->raw_bytes = need;
    }
    ctx->refs++;
    *out = t.release();
    return GGC_OK;
}

extern "C" int ggc_tensor_free(ggc_tensor* t) {
    if (!t) return GGC_OK;
    ggc_ctx* ctx = t->ctx;
    {
        DeviceGuard g(ctx->device);
        cudaStreamSynchronize(ctx->stream);
        free_mat(t->mat);
        if (t->raw) cudaFree(t->raw);
    }
    delete t;
    ctx_release(ctx);
    return GGC_OK;
}

extern "C" int ggc_tensor_matvec(ggc_ctx* ctx, const ggc_tensor* t, const float* x, float* y) {
    if (!ctx || !t || !x || !y) return set_error(GGC_ERR_INVALID_ARG, "null argument");
    DeviceGuard g(ctx->device);
    const uint64_t cols = t->ne[0], rows = t->n_elements / (cols ? cols : 1);
    const void* dx;
    void* dy;
    bool staged;
    GGC_TRY(dev_in(ctx, 1, x, cols * sizeof(float), &dx));
    GGC_TRY(dev_out(ctx, 2, y, rows * sizeof(float), &dy, &staged));
    if (t->repacked) {
        GemvArgs a{};
        a.seg[0] = make_seg(t->mat, EPI_STORE, (float*)dy, nullptr, nullptr);
        a.nseg = 1;
        a.pro = PRO_PLAIN;
        a.x = (const float*)dx;
        a.cols = t->mat.cols;
        a.xcols = t->mat.xcols;
        GGC_TRY(run_gemv(ctx, t->dtype, a));
    } else {
        cudaError_t err = cudaSuccess;
        dispatch_dtype<RunMatvecRaw>(t->dtype, ctx, (const uint8_t*)t->raw, rows, cols, (const float*)dx, (float*)dy, &err);
        GGC_CUDA_TRY(err);
    }
    if (staged) {
        GGC_CUDA_TRY(cudaMemcpyAsync(y, dy, rows * sizeof(float), cudaMemcpyDeviceToHost, ctx->stream));
        GGC_TRY(ctx_sync(ctx));
    }
    return GGC_OK;
}

extern "C" int ggc_tensor_matvec_batch(ggc_ctx* ctx, const ggc_tensor* const* ts, uint64_t n, const float* x, float* y) {
    if (!ctx || (!ts && n) || !x || !y) return set_error(GGC_ERR_INVALID_ARG, "null argument");
    if (!is_device_ptr(x) || !is_device_ptr(y)) return set_error(GGC_ERR_INVALID_ARG, "x and y must be device buffers");
    DeviceGuard g(ctx->device);
    for (uint64_t i = 0; i < n; ++i) {
        const ggc_tensor* t = ts[i];
        if (!t || !t->repacked) return set_error(GGC_ERR_INVALID_ARG, "tensor %llu missing or not in plane layout",
                                                 (unsigned long long)i);
        GemvArgs a{};
        a.seg[0] = make_seg(t->mat, EPI_STORE, y, nullptr, nullptr);
        a.nseg = 1;
        a.pro = PRO_PLAIN;
        a.x = x;
        a.cols = t->mat.cols;
        a.xcols = t->mat.xcols;
        GGC_TRY(run_gemv(ctx, t->dtype, a));
    }
    return GGC_OK;
}

extern "C" int ggc_tensor_dequantize(ggc_ctx* ctx, const ggc_tensor* t, float* out) {
    if (!ctx || !t || !out) return set_error(GGC_ERR_INVALID_ARG, "null argument");
    if (t->repacked) return set_error(GGC_ERR_INVALID_ARG, "tensor was uploaded in plane layout; upload with repack=0");
    return ggc_dequantize(ctx, t->dtype, t->raw, t->raw_bytes, t->n_elements, out);
}

namespace {

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link)
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return (EncodeTiledFn)p;
    }();
    return fn;
}

// The raw rows of a block matrix as a 2-D byte tensor (x = byte in the row,
// y = row) with a box of one block x `box_rows` rows; false when the layout does
// not allow it (base or row pitch not 16-byte aligned, no driver entry point).
bool raw_row_map(CUtensorMap* map, const uint8_t* w, uint32_t rows, uint64_t row_bytes, uint32_t block_bytes,
                 uint32_t box_rows) {
    EncodeTiledFn enc = encode_tiled();
    if (!enc || ((uintptr_t)w & 15) || (row_bytes & 15) || (block_bytes & 15) || block_bytes > 256 || box_rows > 256)
        return false;
    const cuuint64_t dims[2] = {row_bytes, rows}, strides[1] = {row_bytes};
    const cuuint32_t box[2] = {block_bytes, box_rows}, estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void*)w, dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// K split of the product: ks ranges of kb_per K steps (kb_per a multiple of
// `step`, no empty range) minimising the estimated time in K steps of one CTA:
// waves of `tiles` x ks CTAs over the SMs times kb_per, plus the partial slices'
// write + read (m x n x 8 bytes a split, about 12 MB per K step's time).
void mm_split(uint32_t nk, uint32_t step, uint32_t tiles, uint32_t sms, uint32_t m, uint32_t n, uint32_t* ks_out,
              uint32_t* kb_per_out) {
    const double part = (double)m * n * 8.0 / 12e6;
    double best = 1e300;
    for (uint32_t c = 1; c <= std::max(nk / step, 1u); ++c) {
        const uint32_t kb_per = cdiv<uint32_t>(cdiv<uint32_t>(nk, c), step) * step, ks = cdiv<uint32_t>(nk, kb_per);
        if (ks != c) continue;
        const double cost = (double)cdiv<uint32_t>(tiles * ks, sms) * kb_per + (ks > 1 ? ks * part : 0.0);
        if (cost < best) {
            best = cost;
            *ks_out = ks;
            *kb_per_out = kb_per;
        }
    }
}

// 128 weight rows x 512 tokens per CTA; K split over enough CTAs to fill the
// SMs (partials summed in split order by k_mm_reduce).  Q4_K / Q5_K stage their
// raw blocks by TMA (split ranges of whole 256-element blocks) when the tensor
// map can be made, else they read the blocks from global memory as the rest do.
template <int DT>
struct RunMM {
    template <int SM>
    static cudaError_t set_attr() {
        static std::once_flag once_dev[GGC_MAX_DEVICES];
        static cudaError_t attr_dev[GGC_MAX_DEVICES];
        const int dev = current_device();
        if (dev < 0) return cudaErrorInvalidDevice;
        cudaError_t& attr = attr_dev[dev];
        std::call_once(once_dev[dev], [&attr] {
            attr = cudaFuncSetAttribute(k_mm_tc<DT, MM_BN, SM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)mm_smem(MM_BN, SM, block_bytes_of(DT)));
        });
        return attr;
    }
    template <int SM>
    static void go(ggc_ctx* ctx, const uint8_t* w, uint32_t n, uint32_t k, const uint8_t* xh, const uint8_t* xl,
                   uint32_t m, uint32_t kpad, float* y, uint32_t ldy, const float* resid, int* errf,
                   const CUtensorMap& map, cudaError_t* err) {
        constexpr bool STAGE = SM != MMS_NONE;
        *err = set_attr<SM>();
        if (*err != cudaSuccess) return;
        const uint32_t smem = mm_smem(MM_BN, SM, block_bytes_of(DT));
        const uint32_t gx = cdiv<uint32_t>(n, MM_BN), gy = cdiv<uint32_t>(cdiv<uint32_t>(m, MM_TG), MM_NTG);
        const uint32_t nk = kpad / MM_BK, step = STAGE ? (uint32_t)(block_size_of(DT) / MM_BK) : 1u;
        uint32_t ks = 1, kb_per = nk;
        mm_split(nk, step, gx * gy, (uint32_t)ctx->num_sms, m, n, &ks, &kb_per);
        if (ks == 1) {
            *err = launch(ctx, k_mm_tc<DT, MM_BN, SM>, dim3(gx, gy, 1), dim3(MM_THREADS), smem, w, n, k, xh, xl,
                          m, kpad, kb_per, y, ldy, resid, errf, map);
            return;
        }
        const size_t pbytes = (size_t)ks * m * n * sizeof(float);
        int st = ensure_stage(ctx, 5, pbytes);
        if (st != GGC_OK) { *err = cudaErrorMemoryAllocation; return; }
        float* part = (float*)ctx->stage[5];
        *err = launch(ctx, k_mm_tc<DT, MM_BN, SM>, dim3(gx, gy, ks), dim3(MM_THREADS), smem, w, n, k, xh, xl, m,
                      kpad, kb_per, part, n, (const float*)nullptr, errf, map);
        if (*err != cudaSuccess) return;
        const bool vec4 = n % 4 == 0 && ldy % 4 == 0 && (uintptr_t)y % 16 == 0 && (uintptr_t)resid % 16 == 0;
        const uint64_t total = (uint64_t)m * (vec4 ? n / 4 : n);
        const unsigned grid = (unsigned)std::min<uint64_t>(cdiv<uint64_t>(total, 256), (uint64_t)ctx->num_sms * 8);
        if (vec4)
            *err = launch(ctx, k_mm_reduce4, dim3(grid), dim3(256), 0, (const float4*)part, ks, m, n / 4, y, ldy, resid);
        else
            *err = launch(ctx, k_mm_reduce, dim3(grid), dim3(256), 0, (const float*)part, ks, m, n, y, ldy, resid);
    }
    static void run(ggc_ctx* ctx, const uint8_t* w, uint32_t n, uint32_t k, const uint8_t* xh, const uint8_t* xl,
                    uint32_t m, uint32_t kpad, float* y, uint32_t ldy, const float* resid, int* errf,
                    cudaError_t* err) {
        CUtensorMap map;
        std::memset(&map, 0, sizeof(map));
        if constexpr (mm_staged(DT)) {
            const uint64_t row_bytes = (uint64_t)(k / block_size_of(DT)) * block_bytes_of(DT);
            if (k % block_size_of(DT) == 0 && kpad == k &&
                raw_row_map(&map, w, n, row_bytes, (uint32_t)block_bytes_of(DT), MM_BN))
                return go<MMS_TMA>(ctx, w, n, k, xh, xl, m, kpad, y, ldy, resid, errf, map, err);
        }
        if constexpr (DT == GGC_Q6_K) {   // raw weights carry 16 bytes of slack past their end
            if (k % block_size_of(DT) == 0 && kpad == k && ((uintptr_t)w & 15) == 0)
                return go<MMS_ROWS>(ctx, w, n, k, xh, xl, m, kpad, y, ldy, resid, errf, map, err);
        }
        go<MMS_NONE>(ctx, w, n, k, xh, xl, m, kpad, y, ldy, resid, errf, map, err);
    }
};

int ctx_errf(ggc_ctx* ctx, int** out) {
    if (!ctx->errf) {
        GGC_CUDA_TRY(cudaMalloc(&ctx->errf, sizeof(int) * ERRF_COUNT));
        GGC_CUDA_TRY(cudaMemsetAsync(ctx->errf, 0, sizeof(int) * ERRF_COUNT, ctx->stream));
    }
    *out = ctx->errf;
    return GGC_OK;
}

// x [m][k] f32 (device) -> bf16 hi / lo tiles (k_x_split's blocked layout,
// rows padded to 128, columns to 64) in staging buffers 3 / 4
int split_rows(ggc_ctx* ctx, const float* x, const float* x2, uint32_t m, uint32_t k, uint32_t ldx, int pro,
               uint8_t** xh, uint8_t** xl, uint32_t* kpad, int* errf = nullptr, int nan_slot = 0, int nan_val = 0) {
    *kpad = (k + MM_BK - 1) / MM_BK * MM_BK;
    const uint32_t mpad = (m + MM_TG - 1) / MM_TG * MM_TG;
    const size_t bytes = (size_t)mpad * *kpad * 2;
    GGC_TRY(ensure_stage(ctx, 3, bytes));
    GGC_TRY(ensure_stage(ctx, 4, bytes));
    *xh = (uint8_t*)ctx->stage[3];
    *xl = (uint8_t*)ctx->stage[4];
    const int vec = ((uintptr_t)x % 16 == 0) && (!x2 || (uintptr_t)x2 % 16 == 0) && ldx % 4 == 0;
    GGC_CUDA_TRY(launch(ctx, k_x_split, dim3(mpad), dim3(SPLIT_THREADS), 0, x, x2, m, k, ldx, *kpad, pro, vec, *xh, *xl,
                        errf, nan_slot, errf ? nan_val : 0));
    return GGC_OK;
}

}  // namespace

// ops::matmul over a quantized weight (ops.rs:74 computes a @ b for f32
// matrices; here b is an uploaded GGUF tensor used transposed, as every model
// projection does): y[m][rows] = x[m][cols] . W^T on the tensor cores
// (k_mm_tc, split-bf16 operands, f32 accumulation).
extern "C" int ggc_tensor_matmul(ggc_ctx* ctx, const ggc_tensor* t, const float* x, uint64_t m, float* y) {
    if (!ctx || !t || !x || !y) return set_error(GGC_ERR_INVALID_ARG, "null argument");
    if (t->repacked) return set_error(GGC_ERR_INVALID_ARG, "tensor was uploaded in plane layout; upload with repack=0");
    if (m == 0) return set_error(GGC_ERR_INFERENCE, "empty input");
    const uint64_t cols = t->ne[0], rows = t->n_elements / (cols ? cols : 1);
    if (m > 0xFFFFFFFFull / (cols ? cols : 1) || rows > 0xFFFFFFFFull) return set_error(GGC_ERR_INVALID_ARG, "matmul shape");
    DeviceGuard g(ctx->device);
    const void* dx;
    void* dy;
    bool staged;
    GGC_TRY(dev_in(ctx, 0, x, m * cols * sizeof(float), &dx));
    GGC_TRY(dev_out(ctx, 2, y, m * rows * sizeof(float), &dy, &staged));
    int* errf = nullptr;
    GGC_TRY(ctx_errf(ctx, &errf));
    uint8_t *xh, *xl;
    uint32_t kpad = 0;
    GGC_TRY(split_rows(ctx, (const float*)dx, nullptr, (uint32_t)m, (uint32_t)cols, (uint32_t)cols, MMP_PLAIN, &xh, &xl,
                       &kpad));
    cudaError_t err = cudaSuccess;
    if (!dispatch_dtype<RunMM>(t->dtype, ctx, (const uint8_t*)t->raw, (uint32_t)rows, (uint32_t)cols,
                               (const uint8_t*)xh, (const uint8_t*)xl, (uint32_t)m, kpad, (float*)dy,
                               (uint32_t)rows, (const float*)nullptr, errf, &err))
        return set_dequant_error(t->dtype, 0, 0, "matmul dtype");
    GGC_CUDA_TRY(err);
    int hf[ERRF_COUNT];
    GGC_CUDA_TRY(cudaMemcpyAsync(hf, errf, sizeof(hf), cudaMemcpyDeviceToHost, ctx->stream));
    if (staged) GGC_CUDA_TRY(cudaMemcpyAsync(y, dy, m * rows * sizeof(float), cudaMemcpyDeviceToHost, ctx->stream));
    GGC_TRY(ctx_sync(ctx));
    if (hf[ERRF_TIMEOUT]) {
        cudaMemsetAsync(errf, 0, sizeof(int) * ERRF_COUNT, ctx->stream);
        return set_error(GGC_ERR_TIMEOUT, "a bounded device wait expired");
    }
    return GGC_OK;
}

// ===========================================================================
// ops.rs standalone functions (ops.cuh)
// ===========================================================================
namespace {

// a caller's in/out vector: device pointers pass through, host data is staged
// in buffer `i` and copied back by done()
struct InOut {
    ggc_ctx* ctx;
    void* user;
    void* dev = nullptr;
    size_t bytes = 0;
    bool staged = false;
    int open(ggc_ctx* c, int i, void* p, size_t n) {
        ctx = c;
        user = p;
        bytes = n;
        staged = !is_device_ptr(p);
        if (!staged || n == 0) { dev = p; return GGC_OK; }
        GGC_TRY(ensure_stage(c, i, n));
        dev = c->stage[i];
        GGC_CUDA_TRY(cudaMemcpyAsync(dev, p, n, cudaMemcpyHostToDevice, c->stream));
        return GGC_OK;
    }
    int done() {
        if (staged && bytes) GGC_CUDA_TRY(cudaMemcpyAsync(user, dev, bytes, cudaMemcpyDeviceToHost, ctx->stream));
        GGC_TRY(ctx_sync(ctx));
        return GGC_OK;
    }
};

// the three matvec layouts share one kernel and the reference's checks
int ops_matvec(ggc_ctx* ctx, const float* a, uint64_t a_len, uint64_t rows, uint64_t cols, uint64_t rs, uint64_t cs,
               const float* x, uint64_t x_len, float* y, uint64_t y_len, const float* b) {
    if (!ctx || (!a && a_len) || (!x && x_len) || (!y && y_len)) return set_error(GGC_ERR_INVALID_ARG, "null argument");
    if (a_len < rows * cols) return set_dequant_error(GGC_F32, rows * cols, a_len, "matvec a");
    if (x_len != cols) return set_dequant_error(GGC_F32, cols, x_len, "matvec x");
    if (y_len != rows) return set_dequant_error(GGC_F32, rows, y_len, "matvec y");
    if (rows == 0) return GGC_OK;
    DeviceGuard g(ctx->device);
    const void *da, *dx, *db = nullptr;
    GGC_TRY(dev_in(ctx, 0, a, rows * cols * sizeof(float), &da));
    GGC_TRY(dev_in(ctx, 1, x, cols * sizeof(float), &dx));
    if (b) GGC_TRY(dev_in(ctx, 3, b, rows * sizeof(float), &db));
    InOut yo;
    GGC_TRY(yo.open(ctx, 2, y, rows * sizeof(float)));
    GGC_CUDA_TRY(launch(ctx, k_ops_matvec, dim3((unsigned)cdiv<uint64_t>(rows, 128)), dim3(128), 0, (const float*)da, rows,
                        cols, rs, cs, (const float*)dx, (const float*)db, (float*)yo.dev));
    return yo.done();
}

}  // namespace

// ops::matvec (ops.rs:14-72): y = A x (+ b), A row-major rows x cols
extern "C" int ggc_ops_matvec(ggc_ctx* ctx, const float* a, uint64_t a_len, uint64_t rows, uint64_t cols,
                              const float* x, uint64_t x_len, float* y, uint64_t y_len, const float* b) {
    return ops_matvec(ctx, a, a_len, rows, cols, cols, 1, x, x_len, y, y_len, b);
}
// ops::matvec_colmajor (ops.rs:121-170): y[i] = sum_j a[j * rows + i] x[j] (+ b)
extern "C" int ggc_ops_matvec_colmajor(ggc_ctx* ctx, const float* a, uint64_t a_len, uint64_t rows, uint64_t cols,
                                       const float* x, uint64_t x_len, float* y, uint64_t y_len, const float* b) {
    return ops_matvec(ctx, a, a_len, rows, cols, 1, rows, x, x_len, y, y_len, b);
}
// ops::matvec_colmajor_trans (ops.rs:172-227): y[i] = sum_j a[i * dim0 + j] x[j] (+ b), i < dim1
extern "C" int ggc_ops_matvec_colmajor_trans(ggc_ctx* ctx, const float* a, uint64_t a_len, uint64_t dim0, uint64_t dim1,
                                             const float* x, uint64_t x_len, float* y, uint64_t y_len, const float* b) {
    if (a_len < dim0 * dim1) return set_dequant_error(GGC_F32, dim0 * dim1, a_len, "matvec a");
    return ops_matvec(ctx, a, a_len, dim1, dim0, dim0, 1, x, x_len, y, y_len, b);
}
// ops::matmul (ops.rs:74-113): C = A B, row-major
extern "C" int ggc_ops_matmul(ggc_ctx* ctx, const float* a, uint64_t a_len, uint64_t ra, uint64_t ca, const float* b,
                              uint64_t b_len, uint64_t cb, float* c, uint64_t c_len) {
    if (!ctx || (!a && a_len) || (!b && b_len) || (!c && c_len)) return set_error(GGC_ERR_INVALID_ARG, "null argument");
    if (a_len < ra * ca) return set_dequant_error(GGC_F32, ra * ca, a_len, "matmul a");
    if (b_len < ca * cb) return set_dequant_error(GGC_F32, ca * cb, b_len, "matmul b");
    if (c_len < ra * cb) return set_dequant_error(GGC_F32, ra * cb, c_len, "matmul c");
    if (ra == 0 || cb == 0) return GGC_OK;
    if (ra > 65535) return set_error(GGC_ERR_INVALID_ARG, "matmul: at most 65535 rows");
    DeviceGuard g(ctx->device);
    const void *da, *db;
    GGC_TRY(dev_in(ctx, 0, a, ra * ca * sizeof(float), &da));
    GGC_TRY(dev_in(ctx, 1, b, ca * cb * sizeof(float), &db));
    InOut co;
    GGC_TRY(co.open(ctx, 2, c, ra * cb * sizeof(float)));
    GGC_CUDA_TRY(launch(ctx, k_ops_matmul, dim3((unsigned)cdiv<uint64_t>(cb, 256), (unsigned)ra), dim3(256), 0,
                        (const float*)da, (const float*)db, ra, ca, cb, (float*)co.dev));
    return co.done();
}

namespace {
int ops_act(ggc_ctx* ctx, float* x, uint64_t n, int gelu) {
    if (!ctx || (!x && n)) return set_error(GGC_ERR_INVALID_ARG, "null argument");
    if (n == 0) return GGC_OK;
    DeviceGuard g(ctx->device);
    InOut xo;
    GGC_TRY(xo.open(ctx, 0, x, n * sizeof(float)));
    const unsigned grid = (unsigned)std::min<uint64_t>(cdiv<uint64_t>(n, 256), (uint64_t)ctx->num_sms * 8);
    GGC_CUDA_TRY(launch(ctx, k_ops_act, dim3(grid), dim3(256), 0, (float*)xo.dev, n, gelu));
    return xo.done();
}
int ops_norm(ggc_ctx* ctx, float* x, uint64_t n, const float* w, const float* b, float eps, int layer) {
    DeviceGuard g(ctx->device);
    InOut xo;
    GGC_TRY(xo.open(ctx, 0, x, n * sizeof(float)));
    const void *dw, *db = nullptr;
    GGC_TRY(dev_in(ctx, 1, w, n * sizeof(float), &dw));
    if (layer) GGC_TRY(dev_in(ctx, 3, b, n * sizeof(float), &db));
    GGC_CUDA_TRY(launch(ctx, k_ops_norm, dim3(1), dim3(256), 0, (float*)xo.dev, n, (const float*)dw, (const float*)db,
                        eps, layer));
    return xo.done();
}
}  // namespace

// ops::silu / ops::gelu (ops.rs:237-256), in place
extern "C" int ggc_ops_silu(ggc_ctx* ctx, float* x, uint64_t n) { return ops_act(ctx, x, n, 0); }
extern "C" int ggc_ops_gelu(ggc_ctx* ctx, float* x, uint64_t n) { return ops_act(ctx, x, n, 1); }

// ops::rmsnorm (ops.rs:262-274), in place; a length mismatch leaves x as is (as the reference)
extern "C" int ggc_ops_rmsnorm(ggc_ctx* ctx, float* x, uint64_t n, const float* w, uint64_t w_len, float eps) {
    if (!ctx || (!x && n) || (!w && w_len)) return set_error(GGC_ERR_INVALID_ARG, "null argument");
    if (n != w_len || n == 0) return GGC_OK;
    return ops_norm(ctx, x, n, w, nullptr, eps, 0);
}
// ops::layernorm (ops.rs:279-291), in place; empty or mismatched lengths leave x as is
extern "C" int ggc_ops_layernorm(ggc_ctx* ctx, float* x, uint64_t n, const float* w, uint64_t w_len, const float* b,
                                 uint64_t b_len, float eps) {
    if (!ctx || (!x && n) || (!w && w_len) || (!b && b_len)) return set_error(GGC_ERR_INVALID_ARG, "null argument");
    if (n == 0 || n != w_len || n != b_len) return GGC_OK;
    return ops_norm(ctx, x, n, w, b, eps, 1);
}
// ops::softmax (ops.rs:295-308), in place
extern "C" int ggc_ops_softmax(ggc_ctx* ctx, float* x, uint64_t n) {
    if (!ctx || (!x && n)) return set_error(GGC_ERR_INVALID_ARG, "null argument");
    if (n == 0) return GGC_OK;
    DeviceGuard g(ctx->device);
    InOut xo;
    GGC_TRY(xo.open(ctx, 0, x, n * sizeof(float)));
    GGC_CUDA_TRY(launch(ctx, k_ops_softmax, dim3(1), dim3(256), 0, (float*)xo.dev, n));
    return xo.done();
}
// ops::rope (ops.rs:318-337), in place: x holds n_x / head_dim tokens, head_dim = 2 * n_freqs
extern "C" int ggc_ops_rope(ggc_ctx* ctx, float* x, uint64_t n_x, const int64_t* positions, uint64_t n_pos,
                            const float* freqs, uint64_t n_freqs) {
    if (!ctx || (!x && n_x) || (!positions && n_pos) || (!freqs && n_freqs))
        return set_error(GGC_ERR_INVALID_ARG, "null argument");
    if (n_x == 0 || n_pos == 0 || n_freqs == 0) return GGC_OK;
    if (n_freqs > 0xFFFFFFFFull) return set_error(GGC_ERR_INVALID_ARG, "rope: too many frequencies");
    const uint64_t n_tok = n_x / (2 * n_freqs);
    if (n_tok == 0) return GGC_OK;
    DeviceGuard g(ctx->device);
    InOut xo;
    GGC_TRY(xo.open(ctx, 0, x, n_x * sizeof(float)));
    const void *dp, *df;
    GGC_TRY(dev_in(ctx, 1, positions, n_pos * sizeof(int64_t), &dp));
    GGC_TRY(dev_in(ctx, 3, freqs, n_freqs * sizeof(float), &df));
    const unsigned grid = (unsigned)std::min<uint64_t>(cdiv<uint64_t>(n_tok * n_freqs, 256), (uint64_t)ctx->num_sms * 8);
    GGC_CUDA_TRY(launch(ctx, k_ops_rope, dim3(grid), dim3(256), 0, (float*)xo.dev, n_tok, (const int64_t*)dp, n_pos,
                        (const float*)df, (uint32_t)n_freqs));
    return xo.done();
}

// ===========================================================================
// LlamaModel
// ===========================================================================
namespace ggc {
// Device-side state of the token loop (Engine::generate, engine.rs:89-138).
struct StepState {
    int32_t in_idx;     // next prompt token to consume
    int32_t n_in;       // prompt tokens of this run
    int32_t max_new;    // sampling budget (max_tokens)
    int32_t eos;        // < 0: none
    int32_t n_out;      // tokens generated in this run
    int32_t done;       // run finished (EOS, budget, or error)
    uint32_t tok;       // token of the current step
    uint32_t slot;      // KV cache length before this step (= write index)
    int64_t pos;        // position of the current step
    int64_t next_pos;
    uint32_t next_tok;
    uint32_t max_ctx;
    uint32_t ar_step;   // replays of the step graph (the epoch base of the fused all-reduce)
};
}  // namespace ggc

namespace {

__global__ void k_step_begin(StepState* st, const uint32_t* in_tok, const int64_t* in_pos,
                             unsigned long long* argmax_key, int* errf) {
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x != 0) return;
    st->ar_step += 1;   // every replay, on every rank alike
    if (st->done) return;
    if (st->in_idx < st->n_in) {
        st->tok = in_tok[st->in_idx];
        st->pos = in_pos[st->in_idx];
        st->in_idx += 1;
    } else {
        st->tok = st->next_tok;
        st->pos = st->next_pos;
    }
    *argmax_key = 0ull;
    if (st->slot >= st->max_ctx) {   // KvCacheOverflow (error.rs:46-51)
        errf[ERRF_KV_OVERFLOW] = (int)st->slot + 1;
        st->done = 1;
    } else if (st->pos < 0 || st->pos >= (int64_t)st->max_ctx) {
        errf[ERRF_BAD_POS] = 1;
        st->done = 1;
    }
}

// `nan_vec` (tensor parallel only): the reduced hidden state after the last layer,
// checked here because the NaN guards of a sharded model run on reduced vectors
// (the next RMSNorm prologue) and the lm_head GEMV skips prompt tokens.
__global__ void k_step_end(StepState* st, const unsigned long long* argmax_key, uint32_t* out_ids, int* errf,
                           const float* nan_vec, uint32_t nan_n, int nan_val) {
    pdl_trigger();
    pdl_wait();
    if (nan_vec && !st->done) {   // llama.rs:300-307 for the last layer's ffn
        bool nan = false;
        for (uint32_t i = threadIdx.x; i < nan_n; i += blockDim.x) nan |= isnan(nan_vec[i]);
        if (__syncthreads_or(nan) && threadIdx.x == 0) atomicCAS(&errf[ERRF_NAN_FFN], 0, nan_val);
    }
    if (threadIdx.x != 0 || st->done) return;
    st->slot += 1;   // this step's K/V were appended
    for (int i = 0; i < ERRF_COUNT; ++i)
        if (errf[i]) { st->done = 1; return; }
    if (st->in_idx < st->n_in) return;          // inside the prompt: logits not sampled
    if (st->n_out >= st->max_new) { st->done = 1; return; }
    const uint32_t id = (uint32_t)(*argmax_key & 0xFFFFFFFFull);   // Sampler greedy (sampler.rs:113-123)
    if (st->eos >= 0 && (int64_t)id == (int64_t)st->eos) { st->done = 1; return; }
    out_ids[st->n_out] = id;
    st->n_out += 1;
    st->next_tok = id;
    st->next_pos = st->pos + 1;
}

// Greedy-samples the last forward's logits to start a decode continuation
// (the first `sample` of the engine.rs:104-138 loop).
__global__ void k_decode_start(StepState* st, const unsigned long long* argmax_key, uint32_t* out_ids, int* errf) {
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x != 0 || st->done) return;
    if (st->max_new <= 0 || errf[ERRF_NAN_LOGITS]) { st->done = 1; return; }
    const uint32_t id = (uint32_t)(*argmax_key & 0xFFFFFFFFull);
    if (st->eos >= 0 && (int64_t)id == (int64_t)st->eos) { st->done = 1; return; }
    out_ids[0] = id;
    st->n_out = 1;
    st->next_tok = id;
    st->next_pos = st->pos + 1;
}

template <int DT>
__global__ void __launch_bounds__(256) k_embed(const uint8_t* __restrict__ raw, uint64_t n_rows, uint32_t d,
                                               StepState* st, float* __restrict__ hidden, int* __restrict__ errf) {
    constexpr int BS = block_size_of(DT), BB = block_bytes_of(DT);
    pdl_trigger();
    pdl_wait();
    if (st->done) return;
    const uint32_t tok = st->tok;
    if ((uint64_t)tok >= n_rows) {   // llama.rs:374-379 embed out of bounds
        if (threadIdx.x == 0 && blockIdx.x == 0) { errf[ERRF_EMBED_OOB] = (int)tok + 1; }
        return;
    }
    const uint64_t row_bytes = (uint64_t)(d / BS) * BB;
    const uint8_t* row = raw + (uint64_t)tok * row_bytes;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < d; i += gridDim.x * blockDim.x) {
        const uint32_t blk = i / BS;
        hidden[i] = deq_elem<DT>(row + (uint64_t)blk * BB, (int)(i - blk * BS));
    }
}

template <int DT>
struct RunEmbed {
    static void run(ggc_ctx* ctx, const uint8_t* raw, uint64_t rows, uint32_t d, StepState* st, float* hidden, int* errf,
                    cudaError_t* err) {
        unsigned grid = cdiv<uint32_t>(d, 256);
        *err = launch(ctx, k_embed<DT>, dim3(grid), dim3(256), 0, raw, rows, d, st, hidden, errf);
    }
};

}  // namespace

// Raw GGUF rows of a weight (row-major blocks, the logical row order) for the
// batched prefill product (k_mm_tc).
struct RawMat {
    int dtype = -1;
    uint32_t rows = 0, cols = 0;
    uint8_t* p = nullptr;
};

struct ModelLayer {
    float* attn_norm = nullptr;
    float* ffn_norm = nullptr;
    float* bq = nullptr;
    float* bk = nullptr;
    float* bv = nullptr;
    DevMat wq, wk, wv, wo, up, gate, down;
    DevMat ug;   // ffn_up / ffn_gate rows interleaved (same dtype): one GEMV with the SwiGLU epilogue
    uint32_t f_l = 0;   // ffn rows held (all of them, or this rank's shard)
    RawMat rq, rk, rv, ro, rup, rgate, rdown;   // the same weights for the batched prefill
};

struct ggc_model {
    ggc_ctx* ctx = nullptr;
    ggc_hparams hp{};   // the whole model's
    uint32_t hd = 0, qdim = 0, kvdim = 0, nsplit = 1;   // qdim / kvdim: this rank's heads x hd
    uint32_t heads_l = 0, kv_heads_l = 0;                // heads held (all, or this rank's shard)
    int embd_dtype = -1;
    uint8_t* embd = nullptr;
    uint64_t embd_rows = 0;
    float* output_norm = nullptr;
    DevMat output;
    std::vector<ModelLayer> layers;
    void* kcache = nullptr;
    void* vcache = nullptr;
    size_t kv_elem = 4;
    float2* rope = nullptr;
    // activations / scratch
    float *hidden = nullptr, *q = nullptr, *o = nullptr, *ubuf = nullptr, *gbuf = nullptr, *logits = nullptr;
    float* logits_host = nullptr;   // pinned mirror of logits (host copies out of forward)
    float *scores = nullptr, *pmax = nullptr, *psum = nullptr, *opart = nullptr;
    AttnDecodeSel attn;   // fused decode attention, or null for the general pair
    float2* stats = nullptr;
    unsigned* tickets = nullptr;
    unsigned long long* argmax_key = nullptr;
    int* errf = nullptr;
    StepState* st = nullptr;
    uint32_t* in_tok = nullptr;
    int64_t* in_pos = nullptr;
    uint32_t* out_ids = nullptr;
    // pinned host mirror for readback
    struct Readback {
        int32_t ctl[6];
        StepState st;
        int errf[ERRF_COUNT];
        unsigned long long key;
    }* rb = nullptr;
    cudaEvent_t ctl_done = nullptr;   // recorded after each copy of rb->ctl to the device
    // batched prefill (prefill.cuh): raw weights in the layers, activations for
    // PF_CHUNK tokens
    bool prefill = false;
    float *pf_h = nullptr, *pf_y = nullptr, *pf_q = nullptr, *pf_o = nullptr;
    uint32_t* pf_tok = nullptr;
    int64_t* pf_pos = nullptr;
    uint32_t pf_ldy = 0;
    // tensor parallel: the fused all-reduce over peer memory (allreduce.cuh), else NCCL
    bool ar_p2p = false;
    ArGroup* ar = nullptr;                 // device copy
    std::vector<void*> ar_peer_maps;       // IPC mappings of the other ranks' buffers
    // decode-step GEMVs run as chains (chain.cuh): per chain CH_MAX_OPS op slots
    // and completion counters on the device, filled from chain_host after capture
    bool chain = false;
    ChainOp* chain_ops = nullptr;
    uint32_t* chain_cnt = nullptr;
    std::vector<ChainOp> chain_host;
    cudaGraphExec_t graph = nullptr;
    uint64_t launches_per_step = 0;
    uint64_t cache_len = 0;
    std::vector<void*> allocs;
};

namespace {

template <class T>
int dalloc(ggc_model* m, T** p, size_t count) {
    void* q = nullptr;
    GGC_CUDA_TRY(cudaMalloc(&q, count * sizeof(T) + 16));
    // on the context stream: it is non-blocking, so a fill on the legacy default
    // stream is not ordered with the uploads and kernels that follow on it (a late
    // fill once zeroed freshly uploaded norm weights)
    GGC_CUDA_TRY(cudaMemsetAsync(q, 0, count * sizeof(T) + 16, m->ctx->stream));
    m->allocs.push_back(q);
    *p = (T*)q;
    return GGC_OK;
}

// dequantises a (norm / bias) tensor to an f32 device vector (LlamaModel::materialize)
int upload_vec(ggc_model* m, const ggc_tensor_desc& t, uint64_t expect, float** out, const char* what) {
    *out = nullptr;
    if (!t.data) return GGC_OK;
    const int bs = block_size_of(t.dtype), bb = block_bytes_of(t.dtype);
    if (bs < 0) return set_dequant_error(t.dtype, 0, 0, what);
    const uint64_t elements = t.nbytes / (uint64_t)bb * (uint64_t)bs;   // llama.rs:765-767
    if (elements != t.n_elements)
        return set_error(GGC_ERR_INFERENCE, "materialize(%s): dequantized length %llu != num_elements %llu", what,
                         (unsigned long long)elements, (unsigned long long)t.n_elements);
    if (expect && elements != expect)
        return set_error(GGC_ERR_INFERENCE, "%s: %llu elements, expected %llu", what, (unsigned long long)elements,
                         (unsigned long long)expect);
    float* d = nullptr;
    GGC_TRY(dalloc(m, &d, elements));
    GGC_TRY(ggc_dequantize(m->ctx, t.dtype, t.data, t.nbytes, elements, d));
    GGC_TRY(ctx_sync(m->ctx));
    *out = d;
    return GGC_OK;
}

int upload_weight(ggc_model* m, const ggc_tensor_desc& t, uint64_t rows, uint64_t cols, const uint32_t* row_src,
                  DevMat& out, const char* what) {
    if (!t.data) return set_error(GGC_ERR_MISSING_TENSOR, "MissingTensor { name: %s, kind: tensor }", what);
    if (t.n_elements != rows * cols)
        return set_dequant_error(GGC_F32, rows * cols, t.n_elements, what);   // matvec_colmajor_trans size check
    return upload_mat(m->ctx, t.data, t.nbytes, t.dtype, rows, cols, row_src, out);
}

// ffn_up and ffn_gate (llama.rs:547-580).  With one dtype they become one matrix
// whose rows 2i, 2i+1 are up row i, gate row i, so a row pair of the GEMV yields
// silu(gate_i) * up_i in its epilogue; otherwise two matrices.
int upload_rows(ggc_model* m, const ggc_tensor_desc& t, uint64_t total_rows, uint64_t cols,
                const std::vector<uint32_t>& rows, DevMat& out, const char* what);

// Rows [f0, f0 + fl) of both (all of them, or a tensor-parallel shard).
int upload_ffn_up_gate(ggc_model* m, const ggc_tensor_desc& up, const ggc_tensor_desc& gate, uint64_t f, uint64_t d,
                       uint64_t f0, uint64_t fl, ModelLayer& ML) {
    if (!up.data) return set_error(GGC_ERR_MISSING_TENSOR, "MissingTensor { name: ffn_up, kind: tensor }");
    if (!gate.data) return set_error(GGC_ERR_MISSING_TENSOR, "MissingTensor { name: ffn_gate, kind: tensor }");
    if (up.n_elements != f * d) return set_dequant_error(GGC_F32, f * d, up.n_elements, "ffn_up");
    if (gate.n_elements != f * d) return set_dequant_error(GGC_F32, f * d, gate.n_elements, "ffn_gate");
    const int bs = block_size_of(up.dtype), bb = block_bytes_of(up.dtype);
    ML.f_l = (uint32_t)fl;
    if (up.dtype != gate.dtype || bs < 0 || d % (uint64_t)bs != 0) {
        if (f0 == 0 && fl == f) {
            GGC_TRY(upload_weight(m, up, f, d, nullptr, ML.up, "ffn_up"));
            return upload_weight(m, gate, f, d, nullptr, ML.gate, "ffn_gate");
        }
        std::vector<uint32_t> rows(fl);
        for (uint64_t i = 0; i < fl; ++i) rows[i] = (uint32_t)(f0 + i);
        GGC_TRY(upload_rows(m, up, f, d, rows, ML.up, "ffn_up"));
        return upload_rows(m, gate, f, d, rows, ML.gate, "ffn_gate");
    }
    const uint64_t rb = d / bs * (uint64_t)bb;
    if (up.nbytes < f * rb) return set_dequant_error(up.dtype, f * rb, up.nbytes, "ffn_up");
    if (gate.nbytes < f * rb) return set_dequant_error(gate.dtype, f * rb, gate.nbytes, "ffn_gate");
    std::vector<uint8_t> both(2 * fl * rb);
    for (uint64_t i = 0; i < fl; ++i) {
        memcpy(both.data() + (2 * i) * rb, (const uint8_t*)up.data + (f0 + i) * rb, rb);
        memcpy(both.data() + (2 * i + 1) * rb, (const uint8_t*)gate.data + (f0 + i) * rb, rb);
    }
    return upload_mat(m->ctx, both.data(), both.size(), up.dtype, 2 * fl, d, nullptr, ML.ug);
}

// RoPE pair order: plane row 2m / 2m+1 = logical rows h hd + j / h hd + j + hd/2
std::vector<uint32_t> rope_row_order(uint32_t heads, uint32_t hd) {
    std::vector<uint32_t> v((size_t)heads * hd);
    const uint32_t half = hd / 2;
    for (uint32_t h = 0; h < heads; ++h)
        for (uint32_t j = 0; j < half; ++j) {
            const uint32_t mm = h * half + j;
            v[2 * mm] = h * hd + j;
            v[2 * mm + 1] = h * hd + j + half;
        }
    return v;
}

// Group segments by dtype into as few k_gemv launches as possible.
// The launches of one GEMV over segments: one per dtype (up to three segments each).
std::vector<std::pair<int, GemvArgs>> split_segments(std::vector<std::pair<int, Seg>> segs, int pro, const float* x,
                                                     const float* x2, uint32_t cols, uint32_t xcols,
                                                     const GemvArgs& tmpl) {
    std::vector<std::pair<int, GemvArgs>> out;
    while (!segs.empty()) {
        const int dt = segs.front().first;
        GemvArgs a = tmpl;
        a.nseg = 0;
        std::vector<std::pair<int, Seg>> rest;
        for (auto& s : segs) {
            if (s.first == dt && a.nseg < 3) a.seg[a.nseg++] = s.second;
            else rest.push_back(s);
        }
        a.pro = pro;
        a.x = x;
        a.x2 = x2;
        a.cols = cols;
        a.xcols = xcols;
        out.emplace_back(dt, a);
        segs.swap(rest);
    }
    return out;
}

// The GEMVs between two attention launches of the decode step, gathered into
// groups (a group's ops read what the group before wrote) and launched as one
// k_gemv_chain when every op has a span format and the shared memory holds the
// largest x and two tiles; otherwise each op is its own launch, as before.
struct ChainBuilder {
    ggc_model* m;
    uint32_t index = 0;                              // chains launched so far in this step
    std::vector<std::pair<int, GemvArgs>> ops;
    std::vector<std::pair<int, int>> deps;           // per op: first op waited for, count
    int last0 = 0, last1 = 0;                         // the last group's op range

    explicit ChainBuilder(ggc_model* mm) : m(mm) {}

    // ops that read what the previous group (if any, in this chain) wrote
    int group(std::vector<std::pair<int, GemvArgs>> g) {
        const int b = (int)ops.size();
        for (auto& op : g) {
            ops.push_back(op);
            deps.emplace_back(last0, last1 - last0);
        }
        last0 = b;
        last1 = (int)ops.size();
        return m->chain ? GGC_OK : flush();
    }

    bool chainable(ChainArgs& c) const {
        if (!m->chain || ops.empty() || ops.size() > (size_t)CH_MAX_OPS) return false;
        uint32_t xl = 0, part = 0, slot = 0;
        const uint32_t sms = (uint32_t)m->ctx->num_sms;
        for (auto& op : ops) {
            if (!chain_bit(op.first) || op.second.cols % SPAN) return false;   // Q4_K, Q6_K, Q4_0, Q8_0
            const TileLayout L = make_layout(op.first, TILE_ROWS, op.second.cols);
            const SpanSpec sp = span_spec(op.first);
            uint32_t sb = 0;
            for (int p = 0; p < sp.n; ++p) sb += (TILE_ROWS * L.tp_full[p] + 127u) / 128u * 128u;
            slot = std::max(slot, sb);
            xl = std::max(xl, (L.nct * SPAN_LANES * (GS_WORDS + GS_XF) * 4u + 127u) / 128u * 128u);
            uint32_t total = 0;
            for (int i = 0; i < op.second.nseg; ++i) total += op.second.seg[i].m.L.nrb;
            part = std::max(part, ((total + sms - 1) / sms) * TILE_ROWS * 4u);   // every op's row sums
        }
        part = (part + 127u) / 128u * 128u;
        if ((size_t)xl + part + 128 + 2ull * slot > GEMV_SMEM_LIMIT) return false;
        c.xl_bytes = xl;
        c.part_bytes = part;
        c.ring_bytes = (uint32_t)(GEMV_SMEM_LIMIT - xl - part - 128) / 128u * 128u;
        return true;
    }

    int flush() {
        ChainArgs c{};
        if (!chainable(c)) {
            for (auto& op : ops) GGC_TRY(run_gemv(m->ctx, op.first, op.second));
        } else {
            const uint32_t sms = (uint32_t)m->ctx->num_sms;
            ChainOp* host = m->chain_host.data() + (size_t)index * CH_MAX_OPS;
            for (size_t k = 0; k < ops.size(); ++k) {
                ChainOp& o = host[k];
                o = ChainOp{};
                o.a = ops[k].second;
                o.dt = ops[k].first;
                o.dep = deps[k].first;
                o.ndep = deps[k].second;
                const TileLayout L = make_layout(o.dt, TILE_ROWS, o.a.cols);
                const SpanSpec sp = span_spec(o.dt);
                uint32_t off = 0;
                for (int p = 0; p < 4; ++p) {
                    o.poff[p] = off;
                    off += p < sp.n ? (TILE_ROWS * L.tp_full[p] + 127u) / 128u * 128u : 0u;
                }
                o.slot_bytes = off;
                uint32_t total = 0;
                for (int i = 0; i < o.a.nseg; ++i) total += o.a.seg[i].m.L.nrb;
                o.part_rows = ((total + sms - 1) / sms) * TILE_ROWS;
            }
            c.ops = m->chain_ops + (size_t)index * CH_MAX_OPS;
            c.nops = (int)ops.size();
            c.cnt = m->chain_cnt + (size_t)index * CH_MAX_OPS;
            c.step = &m->st->ar_step;
            c.errf = m->errf;
            uint32_t mask = 0;
            for (auto& op : ops) mask |= chain_bit(op.first);
            GGC_CUDA_TRY(launch(m->ctx, chain_kernel(mask), dim3(sms), dim3(CH_THREADS), (size_t)GEMV_SMEM_LIMIT, c));
            ++index;
        }
        ops.clear();
        deps.clear();
        last0 = last1 = 0;
        return GGC_OK;
    }
};

// Enqueues one decode step (one token through every layer) on the context stream.
int enqueue_step(ggc_model* m) {
    ggc_ctx* ctx = m->ctx;
    const ggc_hparams& hp = m->hp;
    const uint32_t d = hp.embed_dim;
    GGC_CUDA_TRY(launch(ctx, k_step_begin, dim3(1), dim3(32), 0, m->st, (const uint32_t*)m->in_tok,
                        (const int64_t*)m->in_pos, m->argmax_key, m->errf));
    cudaError_t err = cudaSuccess;
    dispatch_dtype<RunEmbed>(m->embd_dtype, ctx, (const uint8_t*)m->embd, m->embd_rows, d, m->st, m->hidden, m->errf, &err);
    GGC_CUDA_TRY(err);
    GemvArgs base{};
    base.st_done = &m->st->done;
    base.slot = &m->st->slot;
    base.pos = &m->st->pos;
    base.rope = m->rope;
    base.hd = m->hd;
    base.kv_ctx = hp.max_ctx;
    base.kv_f16 = hp.kv_f16 ? 1 : 0;
    base.errf = m->errf;
    base.argmax_key = m->argmax_key;
    const size_t layer_kv = (size_t)hp.max_ctx * m->kvdim * m->kv_elem;
    // Tensor parallelism: attn_output / ffn_down give partial sums, the residual
    // added by rank 0 alone, and an all-reduce of the hidden state completes each
    // block.  The NaN guards (llama.rs:300-307) then run on the reduced vector in
    // the next RMSNorm prologue (and k_step_end for the last layer), so every rank
    // takes the same device-side decisions.
    // With the fused all-reduce (m->ar_p2p) the two row-parallel GEMVs push their
    // partials to every rank and sum them into the hidden state themselves
    // (EPI_AR), their NaN guard included; the prologue guards serve the NCCL path.
    const bool tp = ctx->world > 1, p2p = tp && m->ar_p2p, nccl_tp = tp && !p2p;
    const int resid_epi = p2p ? EPI_AR : ((!tp || ctx->rank == 0) ? EPI_RESID : EPI_STORE);
    auto allreduce_hidden = [&]() -> int {
        if (!nccl_tp) return GGC_OK;
        const ncclResult_t r = nccl().AllReduce(m->hidden, m->hidden, d, ncclFloat, ncclSum, ctx->comm, ctx->stream);
        return r == ncclSuccess ? GGC_OK : nccl_error("ncclAllReduce", r);
    };
    // the GEMVs between two attention launches form one chain (chain.cuh)
    ChainBuilder cb(m);
    for (uint32_t l = 0; l < hp.n_layers; ++l) {
        ModelLayer& L = m->layers[l];
        void* kc = (uint8_t*)m->kcache + l * layer_kv;
        void* vc = (uint8_t*)m->vcache + l * layer_kv;
        // attention_block (llama.rs:417-495): rmsnorm -> q/k/v (+bias, RoPE, cache append)
        GemvArgs rq = base;
        if (nccl_tp && l > 0) {
            rq.pro_err_slot = ERRF_NAN_FFN;
            rq.pro_err_val = (int)l;   // layer l - 1
        }
        GGC_TRY(cb.group(split_segments({{L.wq.dtype, make_seg(L.wq, EPI_ROPE_Q, m->q, nullptr, L.bq)},
                                         {L.wk.dtype, make_seg(L.wk, EPI_ROPE_KC, nullptr, kc, L.bk)},
                                         {L.wv.dtype, make_seg(L.wv, EPI_VC, nullptr, vc, L.bv)}},
                                        PRO_RMSNORM, m->hidden, L.attn_norm, L.wq.cols, d, rq)));
        GGC_TRY(cb.flush());
        AttnArgs aa{};
        aa.q = m->q;
        aa.kc = kc;
        aa.vc = vc;
        aa.scores = m->scores;
        aa.pmax = m->pmax;
        aa.stats = m->stats;
        aa.opart = m->opart;
        aa.o = m->o;
        aa.tickets = m->tickets;
        aa.slot = &m->st->slot;
        aa.pos = &m->st->pos;
        aa.done = &m->st->done;
        aa.n_heads = m->heads_l;
        aa.kvh = m->kv_heads_l;
        aa.hd = m->hd;
        aa.max_ctx = hp.max_ctx;
        aa.nsplit = m->nsplit;
        aa.inv = 1.0f / sqrtf((float)m->hd);
        aa.kv_f16 = base.kv_f16;
        aa.psum = m->psum;
        aa.errf = m->errf;
        if (m->attn.kernel) {
            GGC_CUDA_TRY(launch(ctx, m->attn.kernel, dim3(m->kv_heads_l, m->nsplit), dim3(FA_THREADS), m->attn.smem, aa));
        } else {
            GGC_CUDA_TRY(launch(ctx, k_attn_scores, dim3(m->kv_heads_l, m->nsplit), dim3(ATTN_WARPS * 32), 0, aa));
            GGC_CUDA_TRY(launch(ctx, k_attn_av, dim3(m->kv_heads_l, m->nsplit), dim3(ATTN_WARPS * 32),
                                attn_av_smem(hp.n_heads / hp.n_kv_heads, m->hd), aa));
        }
        // output projection + residual (llama.rs:485, :309-311), NaN guard (:300-307)
        GemvArgs ro = base;
        ro.err_slot = ERRF_NAN_ATTN;
        ro.err_val = nccl_tp ? 0 : (int)l + 1;
        if (p2p) {
            ro.ar = m->ar;
            ro.ar_k = 2 * l + 1;
        }
        GGC_TRY(cb.group(split_segments({{L.wo.dtype, make_seg(L.wo, resid_epi, m->hidden, nullptr, nullptr)}},
                                        PRO_PLAIN, m->o, nullptr, L.wo.cols, L.wo.xcols, ro)));
        GGC_TRY(allreduce_hidden());
        // ffn_block (llama.rs:547-580): rmsnorm -> up, gate -> silu(gate)*up -> down + residual
        GemvArgs ru = base;
        if (nccl_tp) {
            ru.pro_err_slot = ERRF_NAN_ATTN;
            ru.pro_err_val = (int)l + 1;
        }
        GemvArgs rd = base;
        rd.err_slot = ERRF_NAN_FFN;
        rd.err_val = nccl_tp ? 0 : (int)l + 1;
        if (p2p) {
            rd.ar = m->ar;
            rd.ar_k = 2 * l + 2;
        }
        if (L.ug.base) {   // fused up/gate: h = silu(gate) * up in the epilogue (into ubuf), then down
            GGC_TRY(cb.group(split_segments({{L.ug.dtype, make_seg(L.ug, EPI_SWIGLU, m->ubuf, nullptr, nullptr)}},
                                            PRO_RMSNORM, m->hidden, L.ffn_norm, L.ug.cols, d, ru)));
            GGC_TRY(cb.group(split_segments({{L.down.dtype, make_seg(L.down, resid_epi, m->hidden, nullptr, nullptr)}},
                                            PRO_PLAIN, m->ubuf, nullptr, L.down.cols, L.f_l, rd)));
        } else {
            GGC_TRY(cb.group(split_segments({{L.up.dtype, make_seg(L.up, EPI_STORE, m->ubuf, nullptr, nullptr)},
                                             {L.gate.dtype, make_seg(L.gate, EPI_STORE, m->gbuf, nullptr, nullptr)}},
                                            PRO_RMSNORM, m->hidden, L.ffn_norm, L.up.cols, d, ru)));
            GGC_TRY(cb.group(split_segments({{L.down.dtype, make_seg(L.down, resid_epi, m->hidden, nullptr, nullptr)}},
                                            PRO_SWIGLU, m->gbuf, m->ubuf, L.down.cols, L.f_l, rd)));
        }
        GGC_TRY(allreduce_hidden());
    }
    // final norm + lm_head for the last token only (llama.rs:333, :582-616) + greedy argmax
    GemvArgs lh = base;
    lh.st_skip = &m->st->in_idx;   // skip while in_idx < n_in (a prompt token that is not the last)
    GGC_TRY(cb.group(split_segments({{m->output.dtype, make_seg(m->output, EPI_LOGITS, m->logits, nullptr, nullptr)}},
                                    PRO_RMSNORM, m->hidden, m->output_norm, m->output.cols, d, lh)));
    GGC_TRY(cb.flush());
    GGC_CUDA_TRY(launch(ctx, k_step_end, dim3(1), dim3(nccl_tp ? 256 : 32), 0, m->st,
                        (const unsigned long long*)m->argmax_key, m->out_ids, m->errf,
                        nccl_tp ? (const float*)m->hidden : nullptr, d, (int)hp.n_layers));
    return GGC_OK;
}

// Tensor parallel: the receive words of the fused all-reduce (allreduce.cuh),
// mapped on every rank through CUDA IPC (handles exchanged with an NCCL
// all-gather).  Used when every rank is a separate process on its own GPU and
// every mapping opens; otherwise (or with GGC_TP_ALLREDUCE=nccl) the step
// all-reduces with NCCL.  The ranks agree through an all-reduce of their verdicts.
int setup_allreduce(ggc_model* m) {
    ggc_ctx* ctx = m->ctx;
    const int world = ctx->world, rank = ctx->rank;
    m->ar_p2p = false;
    if (world < 2) return GGC_OK;
    const char* env = getenv("GGC_TP_ALLREDUCE");
    const bool want = !(env && strcmp(env, "nccl") == 0) && world <= AR_MAX_WORLD;
    const uint32_t d = m->hp.embed_dim;
    const uint32_t stride = (d + 31u) / 32u * 32u;
    const size_t buf_bytes = 2ull * world * stride * sizeof(unsigned long long);
    struct Rec {
        cudaIpcMemHandle_t h;
        uint64_t pid;
        unsigned char uuid[16];
        int32_t ok, pad;
    };
    Rec mine{};
    mine.pid = (uint64_t)getpid();
    cudaDeviceProp prop{};
    GGC_CUDA_TRY(cudaGetDeviceProperties(&prop, ctx->device));
    memcpy(mine.uuid, &prop.uuid, 16);
    uint8_t* base = nullptr;
    if (want) {
        GGC_TRY(dalloc(m, &base, buf_bytes));   // zeroed: tag 0 matches no epoch
        mine.ok = cudaIpcGetMemHandle(&mine.h, base) == cudaSuccess;
        cudaGetLastError();
    }
    Rec* drec = nullptr;
    int32_t* dok = nullptr;
    GGC_TRY(dalloc(m, (uint8_t**)&drec, sizeof(Rec) * (world + 1)));
    GGC_TRY(dalloc(m, &dok, 1));
    GGC_CUDA_TRY(cudaMemcpyAsync(drec + world, &mine, sizeof(Rec), cudaMemcpyHostToDevice, ctx->stream));
    ncclResult_t r = nccl().AllGather(drec + world, drec, sizeof(Rec), ncclChar, ctx->comm, ctx->stream);
    if (r != ncclSuccess) return nccl_error("ncclAllGather", r);
    std::vector<Rec> recs(world);
    GGC_CUDA_TRY(cudaMemcpyAsync(recs.data(), drec, sizeof(Rec) * world, cudaMemcpyDeviceToHost, ctx->stream));
    GGC_TRY(ctx_sync(ctx));
    bool ok = want;
    for (int p = 0; p < world && ok; ++p) {
        ok = recs[p].ok != 0;
        for (int q = 0; q < p && ok; ++q)   // one GPU per rank, one process per rank
            ok = memcmp(recs[p].uuid, recs[q].uuid, 16) != 0 && recs[p].pid != recs[q].pid;
    }
    std::vector<uint8_t*> peer(world, nullptr);
    peer[rank] = base;
    for (int p = 0; p < world && ok; ++p) {
        if (p == rank) continue;
        void* q = nullptr;
        if (cudaIpcOpenMemHandle(&q, recs[p].h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            ok = false;
            break;
        }
        m->ar_peer_maps.push_back(q);
        peer[p] = (uint8_t*)q;
    }
    // every rank takes the same path
    const int32_t vote = ok ? 1 : 0;
    GGC_CUDA_TRY(cudaMemcpyAsync(dok, &vote, sizeof(vote), cudaMemcpyHostToDevice, ctx->stream));
    r = nccl().AllReduce(dok, dok, 1, ncclInt32, ncclMin, ctx->comm, ctx->stream);
    if (r != ncclSuccess) return nccl_error("ncclAllReduce", r);
    int32_t all = 0;
    GGC_CUDA_TRY(cudaMemcpyAsync(&all, dok, sizeof(all), cudaMemcpyDeviceToHost, ctx->stream));
    GGC_TRY(ctx_sync(ctx));
    if (!all) {
        for (void* q : m->ar_peer_maps) cudaIpcCloseMemHandle(q);
        m->ar_peer_maps.clear();
        return GGC_OK;
    }
    ArGroup g{};
    for (int p = 0; p < world; ++p) g.buf[p] = (unsigned long long*)peer[p];
    g.world = world;
    g.rank = rank;
    g.stride = stride;
    g.step = &m->st->ar_step;
    g.per_step = 2u * m->hp.n_layers;
    GGC_TRY(dalloc(m, &m->ar, 1));
    GGC_CUDA_TRY(cudaMemcpyAsync(m->ar, &g, sizeof(g), cudaMemcpyHostToDevice, ctx->stream));
    GGC_TRY(ctx_sync(ctx));
    m->ar_p2p = true;
    return GGC_OK;
}

int build_graph(ggc_model* m) {
    ggc_ctx* ctx = m->ctx;
    uint64_t before = ctx->launches;
    cudaGraph_t g = nullptr;
    GGC_CUDA_TRY(cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
    int st = enqueue_step(m);
    cudaError_t e = cudaStreamEndCapture(ctx->stream, &g);
    if (st != GGC_OK) {
        if (g) cudaGraphDestroy(g);
        return st;
    }
    GGC_CUDA_TRY(e);
    if (m->chain)
        GGC_CUDA_TRY(cudaMemcpyAsync(m->chain_ops, m->chain_host.data(), m->chain_host.size() * sizeof(ChainOp),
                                     cudaMemcpyHostToDevice, ctx->stream));
    e = cudaGraphInstantiate(&m->graph, g, 0);
    cudaGraphDestroy(g);
    GGC_CUDA_TRY(e);
    m->launches_per_step = ctx->launches - before;
    ctx->launches = before;
    return GGC_OK;
}

void destroy_model(ggc_model* m) {
    if (!m) return;
    ggc_ctx* ctx = m->ctx;
    {
        DeviceGuard g(ctx->device);
        cudaStreamSynchronize(ctx->stream);
        if (m->graph) cudaGraphExecDestroy(m->graph);
        for (auto& L : m->layers) {
            free_mat(L.wq); free_mat(L.wk); free_mat(L.wv); free_mat(L.wo);
            free_mat(L.up); free_mat(L.gate); free_mat(L.down); free_mat(L.ug);
        }
        free_mat(m->output);
        for (void* p : m->ar_peer_maps) cudaIpcCloseMemHandle(p);
        for (void* p : m->allocs) cudaFree(p);
        if (m->rb) cudaFreeHost(m->rb);
        if (m->ctl_done) cudaEventDestroy(m->ctl_done);
        if (m->logits_host) cudaFreeHost(m->logits_host);
    }
    delete m;
    ctx_release(ctx);
}

}  // namespace

// Megatron shard of one layer for `rank` of `world`: heads and kv heads in equal
// contiguous ranges, ffn rows in ffn_down blocks with the remainder on the lowest ranks.
extern "C" int ggc_tp_plan(const ggc_hparams* hp, int wo_dtype, int down_dtype, int rank, int world, ggc_tp_shard* out) {
    if (!hp || !out) return set_error(GGC_ERR_INVALID_ARG, "null argument");
    if (world < 1 || rank < 0 || rank >= world) return set_error(GGC_ERR_INVALID_ARG, "rank %d of world %d", rank, world);
    if (hp->n_heads == 0 || hp->n_kv_heads == 0 || hp->embed_dim % hp->n_heads != 0)
        return set_error(GGC_ERR_INFERENCE, "unsupported head configuration");
    if (hp->n_heads % (uint32_t)world != 0 || hp->n_kv_heads % (uint32_t)world != 0)
        return set_error(GGC_ERR_INVALID_ARG, "tensor parallel: world %d does not divide n_heads %u and n_kv_heads %u",
                         world, hp->n_heads, hp->n_kv_heads);
    const int bo = block_size_of(wo_dtype), bd = block_size_of(down_dtype);
    if (bo < 0) return set_dequant_error(wo_dtype, 0, 0, "attn_output");
    if (bd < 0) return set_dequant_error(down_dtype, 0, 0, "ffn_down");
    const uint32_t hd = hp->embed_dim / hp->n_heads, heads = hp->n_heads / (uint32_t)world;
    if (((uint64_t)heads * hd) % (uint64_t)bo != 0)
        return set_error(GGC_ERR_INVALID_ARG, "tensor parallel: %u attn_output columns per rank are not whole %d-element blocks",
                         heads * hd, bo);
    if (hp->ffn_dim % (uint32_t)bd != 0) return set_shape_error(hp->ffn_dim, bd, "ffn_down columns");
    const uint64_t units = hp->ffn_dim / (uint64_t)bd, base = units / (uint64_t)world, extra = units % (uint64_t)world;
    if (base == 0)
        return set_error(GGC_ERR_INVALID_ARG, "tensor parallel: %llu ffn_down blocks for %d ranks",
                         (unsigned long long)units, world);
    const uint64_t r = (uint64_t)rank;
    out->head0 = (uint32_t)rank * heads;
    out->heads = heads;
    out->kv_heads = hp->n_kv_heads / (uint32_t)world;
    out->kv_head0 = (uint32_t)rank * out->kv_heads;
    out->ffn0 = (r * base + (r < extra ? r : extra)) * (uint64_t)bd;
    out->ffn_len = (base + (r < extra ? 1 : 0)) * (uint64_t)bd;
    return GGC_OK;
}

namespace {

// Elements [e0, e0 + n) of a vector tensor as a tensor of its own (whole blocks).
int slice_vec(const ggc_tensor_desc& t, uint64_t e0, uint64_t n, ggc_tensor_desc* out, const char* what) {
    *out = t;
    if (!t.data) return GGC_OK;
    const int bs = block_size_of(t.dtype), bb = block_bytes_of(t.dtype);
    if (bs < 0) return set_dequant_error(t.dtype, 0, 0, what);
    if (e0 % (uint64_t)bs || n % (uint64_t)bs) return set_shape_error(n, bs, what);
    if (t.n_elements < e0 + n || t.nbytes < (e0 + n) / bs * (uint64_t)bb)
        return set_dequant_error(t.dtype, e0 + n, t.n_elements, what);
    out->data = (const uint8_t*)t.data + e0 / bs * (uint64_t)bb;
    out->nbytes = n / bs * (uint64_t)bb;
    out->n_elements = n;
    return GGC_OK;
}

// Columns [c0, c0 + n) of every row of a rows x cols block matrix (whole blocks).
int slice_cols(const ggc_tensor_desc& t, uint64_t rows, uint64_t cols, uint64_t c0, uint64_t n,
               std::vector<uint8_t>& out, const char* what) {
    if (!t.data) return set_error(GGC_ERR_MISSING_TENSOR, "MissingTensor { name: %s, kind: tensor }", what);
    const int bs = block_size_of(t.dtype), bb = block_bytes_of(t.dtype);
    if (bs < 0) return set_dequant_error(t.dtype, 0, 0, what);
    if (t.n_elements != rows * cols) return set_dequant_error(GGC_F32, rows * cols, t.n_elements, what);
    if (cols % (uint64_t)bs || c0 % (uint64_t)bs || n % (uint64_t)bs) return set_shape_error(cols, bs, what);
    const uint64_t rb = cols / bs * (uint64_t)bb, ob = n / bs * (uint64_t)bb, off = c0 / bs * (uint64_t)bb;
    if (t.nbytes < rows * rb) return set_dequant_error(t.dtype, rows * rb, t.nbytes, what);
    out.resize(rows * ob);
    for (uint64_t r = 0; r < rows; ++r) memcpy(out.data() + r * ob, (const uint8_t*)t.data + r * rb + off, ob);
    return GGC_OK;
}

// Rows [r0, r0 + n) of a rows x cols block matrix `data` as a device RawMat.
int upload_raw(ggc_model* m, const void* data, int dt, uint64_t r0, uint64_t n, uint64_t cols, RawMat& out) {
    const uint64_t rb = cols / (uint64_t)block_size_of(dt) * (uint64_t)block_bytes_of(dt);
    uint8_t* d = nullptr;
    GGC_TRY(dalloc(m, &d, n * rb));
    GGC_CUDA_TRY(cudaMemcpyAsync(d, (const uint8_t*)data + r0 * rb, n * rb, cudaMemcpyDefault, m->ctx->stream));
    GGC_TRY(ctx_sync(m->ctx));
    out.dtype = dt;
    out.rows = (uint32_t)n;
    out.cols = (uint32_t)cols;
    out.p = d;
    return GGC_OK;
}

// Rows `rows` (source indices, in plane order) of a total_rows x cols matrix.
int upload_rows(ggc_model* m, const ggc_tensor_desc& t, uint64_t total_rows, uint64_t cols,
                const std::vector<uint32_t>& rows, DevMat& out, const char* what) {
    if (!t.data) return set_error(GGC_ERR_MISSING_TENSOR, "MissingTensor { name: %s, kind: tensor }", what);
    if (t.n_elements != total_rows * cols) return set_dequant_error(GGC_F32, total_rows * cols, t.n_elements, what);
    const int bs = block_size_of(t.dtype), bb = block_bytes_of(t.dtype);
    if (bs < 0) return set_dequant_error(t.dtype, 0, 0, what);
    if (cols % (uint64_t)bs) return set_shape_error(cols, bs, what);
    if (t.nbytes < total_rows * (cols / bs * (uint64_t)bb))
        return set_dequant_error(t.dtype, total_rows * (cols / bs * (uint64_t)bb), t.nbytes, what);
    return upload_mat(m->ctx, t.data, t.nbytes, t.dtype, rows.size(), cols, rows.data(), out);
}

}  // namespace

extern "C" int ggc_model_create(ggc_ctx* ctx, const ggc_hparams* hp_in, const ggc_tensor_desc* t, uint64_t n_tensors,
                                ggc_model** out) {
    if (!ctx || !hp_in || !t || !out) return set_error(GGC_ERR_INVALID_ARG, "null argument");
    const ggc_hparams hp = *hp_in;
    if (n_tensors != 3 + 12ull * hp.n_layers)
        return set_error(GGC_ERR_MISSING_TENSOR, "expected %llu tensors, got %llu",
                         (unsigned long long)(3 + 12ull * hp.n_layers), (unsigned long long)n_tensors);
    if (hp.n_heads == 0 || hp.n_kv_heads == 0 || hp.embed_dim % hp.n_heads != 0 || hp.n_heads % hp.n_kv_heads != 0)
        return set_error(GGC_ERR_INFERENCE, "unsupported head configuration");
    const uint32_t hd = hp.embed_dim / hp.n_heads;
    if (hd % 2 != 0 || hd > 256 || hp.n_heads / hp.n_kv_heads > ATTN_MAX_G)
        return set_error(GGC_ERR_INFERENCE, "head_dim %u / GQA group %u not supported", hd, hp.n_heads / hp.n_kv_heads);
    if (hp.max_ctx == 0) return set_error(GGC_ERR_INVALID_ARG, "max_ctx must be > 0");
    DeviceGuard g(ctx->device);
    GGC_TRY(init_kernel_attrs());
    std::unique_ptr<ggc_model, void (*)(ggc_model*)> m(new ggc_model(), destroy_model);
    m->ctx = ctx;
    ctx->refs++;   // released by destroy_model
    m->hp = hp;
    m->hd = hd;
    const int world = ctx->world;
    m->heads_l = hp.n_heads / (uint32_t)world;
    m->kv_heads_l = hp.n_kv_heads / (uint32_t)world;
    if (world > 1 && (hp.n_heads % (uint32_t)world || hp.n_kv_heads % (uint32_t)world))
        return set_error(GGC_ERR_INVALID_ARG, "tensor parallel: world %d does not divide n_heads %u and n_kv_heads %u",
                         world, hp.n_heads, hp.n_kv_heads);
    m->qdim = m->heads_l * hd;
    m->kvdim = m->kv_heads_l * hd;
    m->kv_elem = hp.kv_f16 ? 2 : 4;
    const uint32_t d = hp.embed_dim, f = hp.ffn_dim;
    // token_embd: kept raw, one row dequantised per token
    {
        const ggc_tensor_desc& e = t[0];
        if (!e.data) return set_error(GGC_ERR_MISSING_TENSOR, "MissingTensor { name: token_embd, kind: tensor }");
        const int bs = block_size_of(e.dtype), bb = block_bytes_of(e.dtype);
        if (bs < 0) return set_dequant_error(e.dtype, 0, 0, "token_embd");
        if (d % bs != 0) return set_shape_error(d, bs, "token_embd row");
        const uint64_t row_bytes = (uint64_t)d / bs * bb;
        m->embd_rows = e.nbytes / row_bytes;
        m->embd_dtype = e.dtype;
        GGC_TRY(dalloc(m.get(), &m->embd, m->embd_rows * row_bytes));
        GGC_CUDA_TRY(cudaMemcpyAsync(m->embd, e.data, m->embd_rows * row_bytes, cudaMemcpyDefault, ctx->stream));
        GGC_TRY(ctx_sync(ctx));
    }
    GGC_TRY(upload_vec(m.get(), t[1], d, &m->output_norm, "output_norm"));
    if (!m->output_norm) return set_error(GGC_ERR_MISSING_TENSOR, "MissingTensor { name: output_norm, kind: tensor }");
    GGC_TRY(upload_weight(m.get(), t[2], hp.vocab_size, d, nullptr, m->output, "output"));
    const std::vector<uint32_t> qorder = rope_row_order(hp.n_heads, hd), korder = rope_row_order(hp.n_kv_heads, hd);
    m->layers.resize(hp.n_layers);
    {   // batched prefill: head dims with a k_attn_prefill instantiation; GGC_PREFILL=0 turns it off
        const char* pe = getenv("GGC_PREFILL");
        m->prefill = (hd == 64 || hd == 128) && !(pe && strcmp(pe, "0") == 0);
    }
    for (uint32_t l = 0; l < hp.n_layers; ++l) {
        const ggc_tensor_desc* L = t + 3 + 12 * l;
        ModelLayer& ML = m->layers[l];
        GGC_TRY(upload_vec(m.get(), L[0], d, &ML.attn_norm, "attn_norm"));
        if (!ML.attn_norm) return set_error(GGC_ERR_MISSING_TENSOR, "MissingTensor { name: blk.%u.attn_norm, kind: tensor }", l);
        if (world == 1) {
            GGC_TRY(upload_weight(m.get(), L[1], m->qdim, d, qorder.data(), ML.wq, "attn_q"));
            GGC_TRY(upload_vec(m.get(), L[2], m->qdim, &ML.bq, "attn_q.bias"));
            GGC_TRY(upload_weight(m.get(), L[3], m->kvdim, d, korder.data(), ML.wk, "attn_k"));
            GGC_TRY(upload_vec(m.get(), L[4], m->kvdim, &ML.bk, "attn_k.bias"));
            GGC_TRY(upload_weight(m.get(), L[5], m->kvdim, d, nullptr, ML.wv, "attn_v"));
            GGC_TRY(upload_vec(m.get(), L[6], m->kvdim, &ML.bv, "attn_v.bias"));
            GGC_TRY(upload_weight(m.get(), L[7], d, m->qdim, nullptr, ML.wo, "attn_output"));
            GGC_TRY(upload_vec(m.get(), L[8], d, &ML.ffn_norm, "ffn_norm"));
            if (!ML.ffn_norm)
                return set_error(GGC_ERR_MISSING_TENSOR, "MissingTensor { name: blk.%u.ffn_norm, kind: tensor }", l);
            GGC_TRY(upload_ffn_up_gate(m.get(), L[9], L[10], f, d, 0, f, ML));
            GGC_TRY(upload_weight(m.get(), L[11], d, f, nullptr, ML.down, "ffn_down"));
            if (m->prefill) {   // raw copies (shapes validated above)
                GGC_TRY(upload_raw(m.get(), L[1].data, L[1].dtype, 0, m->qdim, d, ML.rq));
                GGC_TRY(upload_raw(m.get(), L[3].data, L[3].dtype, 0, m->kvdim, d, ML.rk));
                GGC_TRY(upload_raw(m.get(), L[5].data, L[5].dtype, 0, m->kvdim, d, ML.rv));
                GGC_TRY(upload_raw(m.get(), L[7].data, L[7].dtype, 0, d, m->qdim, ML.ro));
                GGC_TRY(upload_raw(m.get(), L[9].data, L[9].dtype, 0, f, d, ML.rup));
                GGC_TRY(upload_raw(m.get(), L[10].data, L[10].dtype, 0, f, d, ML.rgate));
                GGC_TRY(upload_raw(m.get(), L[11].data, L[11].dtype, 0, d, f, ML.rdown));
            }
            continue;
        }
        // tensor-parallel shard (ggc_tp_plan): q/k/v rows and up/gate rows of this
        // rank, attn_output / ffn_down columns to match (partial sums, all-reduced)
        if (!L[7].data) return set_error(GGC_ERR_MISSING_TENSOR, "MissingTensor { name: attn_output, kind: tensor }");
        if (!L[11].data) return set_error(GGC_ERR_MISSING_TENSOR, "MissingTensor { name: ffn_down, kind: tensor }");
        ggc_tp_shard sh{};
        GGC_TRY(ggc_tp_plan(&hp, L[7].dtype, L[11].dtype, ctx->rank, world, &sh));
        const uint32_t qfull = hp.n_heads * hd, kvfull = hp.n_kv_heads * hd;
        std::vector<uint32_t> qrows = rope_row_order(sh.heads, hd), krows = rope_row_order(sh.kv_heads, hd);
        std::vector<uint32_t> vrows(m->kvdim);
        for (auto& r : qrows) r += sh.head0 * hd;
        for (auto& r : krows) r += sh.kv_head0 * hd;
        for (uint32_t i = 0; i < m->kvdim; ++i) vrows[i] = sh.kv_head0 * hd + i;
        ggc_tensor_desc b{};
        GGC_TRY(upload_rows(m.get(), L[1], qfull, d, qrows, ML.wq, "attn_q"));
        GGC_TRY(slice_vec(L[2], (uint64_t)sh.head0 * hd, m->qdim, &b, "attn_q.bias"));
        GGC_TRY(upload_vec(m.get(), b, m->qdim, &ML.bq, "attn_q.bias"));
        GGC_TRY(upload_rows(m.get(), L[3], kvfull, d, krows, ML.wk, "attn_k"));
        GGC_TRY(slice_vec(L[4], (uint64_t)sh.kv_head0 * hd, m->kvdim, &b, "attn_k.bias"));
        GGC_TRY(upload_vec(m.get(), b, m->kvdim, &ML.bk, "attn_k.bias"));
        GGC_TRY(upload_rows(m.get(), L[5], kvfull, d, vrows, ML.wv, "attn_v"));
        GGC_TRY(slice_vec(L[6], (uint64_t)sh.kv_head0 * hd, m->kvdim, &b, "attn_v.bias"));
        GGC_TRY(upload_vec(m.get(), b, m->kvdim, &ML.bv, "attn_v.bias"));
        std::vector<uint8_t> cols;
        GGC_TRY(slice_cols(L[7], d, qfull, (uint64_t)sh.head0 * hd, m->qdim, cols, "attn_output"));
        GGC_TRY(upload_mat(ctx, cols.data(), cols.size(), L[7].dtype, d, m->qdim, nullptr, ML.wo));
        if (m->prefill) {
            GGC_TRY(upload_raw(m.get(), L[1].data, L[1].dtype, (uint64_t)sh.head0 * hd, m->qdim, d, ML.rq));
            GGC_TRY(upload_raw(m.get(), L[3].data, L[3].dtype, (uint64_t)sh.kv_head0 * hd, m->kvdim, d, ML.rk));
            GGC_TRY(upload_raw(m.get(), L[5].data, L[5].dtype, (uint64_t)sh.kv_head0 * hd, m->kvdim, d, ML.rv));
            GGC_TRY(upload_raw(m.get(), cols.data(), L[7].dtype, 0, d, m->qdim, ML.ro));
        }
        GGC_TRY(upload_vec(m.get(), L[8], d, &ML.ffn_norm, "ffn_norm"));
        if (!ML.ffn_norm) return set_error(GGC_ERR_MISSING_TENSOR, "MissingTensor { name: blk.%u.ffn_norm, kind: tensor }", l);
        GGC_TRY(upload_ffn_up_gate(m.get(), L[9], L[10], f, d, sh.ffn0, sh.ffn_len, ML));
        GGC_TRY(slice_cols(L[11], d, f, sh.ffn0, sh.ffn_len, cols, "ffn_down"));
        GGC_TRY(upload_mat(ctx, cols.data(), cols.size(), L[11].dtype, d, sh.ffn_len, nullptr, ML.down));
        if (m->prefill) {
            GGC_TRY(upload_raw(m.get(), L[9].data, L[9].dtype, sh.ffn0, sh.ffn_len, d, ML.rup));
            GGC_TRY(upload_raw(m.get(), L[10].data, L[10].dtype, sh.ffn0, sh.ffn_len, d, ML.rgate));
            GGC_TRY(upload_raw(m.get(), cols.data(), L[11].dtype, 0, d, sh.ffn_len, ML.rdown));
        }
    }
    // KV cache resident in HBM, head-major: [layer][n_kv][max_ctx][hd]
    const size_t kv_bytes = (size_t)hp.n_layers * hp.max_ctx * m->kvdim * m->kv_elem;
    GGC_TRY(dalloc(m.get(), (uint8_t**)&m->kcache, kv_bytes));
    GGC_TRY(dalloc(m.get(), (uint8_t**)&m->vcache, kv_bytes));
    // RoPE table with the reference's f32 arithmetic (ops.rs:326-330, llama.rs:778-782)
    {
        const uint32_t half = hd / 2;
        std::vector<float> inv(half);
        for (uint32_t i = 0; i < half; ++i) inv[i] = (float)std::pow(hp.rope_freq_base, -2.0 * (double)i / (double)hd);
        std::vector<float2> tab((size_t)hp.max_ctx * half);
        for (uint32_t p = 0; p < hp.max_ctx; ++p)
            for (uint32_t i = 0; i < half; ++i) {
                const float angle = (float)p * inv[i];
                tab[(size_t)p * half + i] = make_float2(cosf(angle), sinf(angle));
            }
        GGC_TRY(dalloc(m.get(), &m->rope, tab.size()));
        GGC_CUDA_TRY(cudaMemcpyAsync(m->rope, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice,
                                     ctx->stream));
        GGC_TRY(ctx_sync(ctx));
    }
    // fused attention: two resident CTAs per SM over (kv head, split); general pair: ~2 per SM, <= 64 splits
    m->attn = attn_decode_sel(hd, hp.kv_f16 != 0, hp.n_heads / hp.n_kv_heads);
    if (m->attn.kernel) {   // at most two CTAs per SM, >= 128 positions per split at max_ctx, <= 64 splits
        uint32_t ns = (uint32_t)ctx->num_sms * 2 / m->kv_heads_l;
        ns = std::min(ns, cdiv<uint32_t>(hp.max_ctx, 128));
        ns = std::min(ns, FA_MAX_SPLITS);
        m->nsplit = ns < 1 ? 1 : ns;
    } else {
        const uint32_t ns = cdiv<uint32_t>((uint32_t)ctx->num_sms * 2, m->kv_heads_l);
        m->nsplit = ns < 1 ? 1 : (ns > 64 ? 64 : ns);
    }
    GGC_TRY(dalloc(m.get(), &m->hidden, d));
    GGC_TRY(dalloc(m.get(), &m->q, m->qdim));
    GGC_TRY(dalloc(m.get(), &m->o, m->qdim));
    GGC_TRY(dalloc(m.get(), &m->ubuf, f));
    GGC_TRY(dalloc(m.get(), &m->gbuf, f));
    GGC_TRY(dalloc(m.get(), &m->logits, hp.vocab_size));
    GGC_TRY(dalloc(m.get(), &m->scores, (size_t)m->heads_l * hp.max_ctx));
    GGC_TRY(dalloc(m.get(), &m->pmax, (size_t)m->heads_l * m->nsplit));
    GGC_TRY(dalloc(m.get(), &m->psum, (size_t)m->heads_l * m->nsplit));
    GGC_TRY(dalloc(m.get(), &m->stats, m->heads_l));
    GGC_TRY(dalloc(m.get(), &m->opart, (size_t)m->nsplit * m->qdim));
    GGC_TRY(dalloc(m.get(), &m->tickets, 2 * m->kv_heads_l));
    GGC_TRY(dalloc(m.get(), &m->argmax_key, 1));
    GGC_TRY(dalloc(m.get(), &m->errf, ERRF_COUNT));
    GGC_TRY(dalloc(m.get(), &m->st, 1));
    GGC_TRY(dalloc(m.get(), &m->in_tok, hp.max_ctx));
    GGC_TRY(dalloc(m.get(), &m->in_pos, hp.max_ctx));
    GGC_TRY(dalloc(m.get(), &m->out_ids, hp.max_ctx));
    GGC_CUDA_TRY(cudaMallocHost((void**)&m->rb, sizeof(*m->rb)));
    GGC_CUDA_TRY(cudaEventCreateWithFlags(&m->ctl_done, cudaEventDisableTiming));
    GGC_CUDA_TRY(cudaMallocHost((void**)&m->logits_host, (size_t)hp.vocab_size * sizeof(float)));
    StepState s0{};
    s0.done = 1;
    s0.max_ctx = hp.max_ctx;
    GGC_CUDA_TRY(cudaMemcpyAsync(m->st, &s0, sizeof(s0), cudaMemcpyHostToDevice, ctx->stream));
    GGC_TRY(setup_allreduce(m.get()));
    {   // decode GEMVs as chains (chain.cuh), opt-in with GGC_DECODE_CHAIN=1 (slower than the per-op
        // kernels today: 369 vs 450 tokens/s on the Llama-2-7B Q4_K_M step), never around an NCCL all-reduce
        const char* ce = getenv("GGC_DECODE_CHAIN");
        m->chain = (ce && strcmp(ce, "1") == 0) && !(ctx->world > 1 && !m->ar_p2p);
        if (m->chain) {
            const size_t slots = (size_t)(hp.n_layers + 1) * CH_MAX_OPS;
            m->chain_host.assign(slots, ChainOp{});
            GGC_TRY(dalloc(m.get(), &m->chain_ops, slots));
            GGC_TRY(dalloc(m.get(), &m->chain_cnt, slots));
        }
    }
    GGC_TRY(build_graph(m.get()));
    GGC_TRY(ctx_sync(ctx));
    *out = m.release();
    return GGC_OK;
}

extern "C" int ggc_model_destroy(ggc_model* m) {
    destroy_model(m);
    return GGC_OK;
}

namespace {

// Runs `steps` graph replays after setting the control block, then reads back.
// Queues the copy of the step control words to the device through the pinned
// block, after the previous copy out of that block has landed (an event, not a
// wait for the whole stream: a forward on an idle stream starts at once).
int put_ctl(ggc_model* m, const int32_t (&ctl)[6]) {
    GGC_TRY(ctx_sync(m->ctx, m->ctl_done));
    memcpy(&m->rb->ctl, ctl, sizeof(ctl));
    GGC_CUDA_TRY(cudaMemcpyAsync(m->st, &m->rb->ctl, sizeof(ctl), cudaMemcpyHostToDevice, m->ctx->stream));
    GGC_CUDA_TRY(cudaEventRecord(m->ctl_done, m->ctx->stream));
    return GGC_OK;
}

int run_steps(ggc_model* m, uint64_t n_in, uint64_t max_new, int64_t eos, uint64_t steps) {
    ggc_ctx* ctx = m->ctx;
    int32_t ctl[6] = {0, (int32_t)n_in, (int32_t)max_new, (int32_t)(eos < 0 ? -1 : eos), 0, 0};
    GGC_TRY(put_ctl(m, ctl));
    for (uint64_t i = 0; i < steps; ++i) {
        GGC_CUDA_TRY(cudaGraphLaunch(m->graph, ctx->stream));
        ctx->launches += m->launches_per_step;
    }
    GGC_CUDA_TRY(cudaMemcpyAsync(&m->rb->st, m->st, sizeof(StepState), cudaMemcpyDeviceToHost, ctx->stream));
    GGC_CUDA_TRY(cudaMemcpyAsync(m->rb->errf, m->errf, sizeof(int) * ERRF_COUNT, cudaMemcpyDeviceToHost, ctx->stream));
    GGC_CUDA_TRY(cudaMemcpyAsync(&m->rb->key, m->argmax_key, sizeof(unsigned long long), cudaMemcpyDeviceToHost, ctx->stream));
    return GGC_OK;
}

// The error of a set of device flags (GgufError variant + message), GGC_OK if none.
int errf_status(const ggc_model* m, const int* e) {
    int status = GGC_OK;
    if (e[ERRF_EMBED_OOB]) status = set_error(GGC_ERR_INFERENCE, "embed out of bounds: tok=%d", e[ERRF_EMBED_OOB] - 1);
    // the earliest NaN site: attention of layer l runs before the ffn of layer l
    else if (e[ERRF_NAN_ATTN] && (!e[ERRF_NAN_FFN] || e[ERRF_NAN_ATTN] <= e[ERRF_NAN_FFN]))
        status = set_error(GGC_ERR_INFERENCE, "NaN after layer %d attention", e[ERRF_NAN_ATTN] - 1);
    else if (e[ERRF_NAN_FFN]) status = set_error(GGC_ERR_INFERENCE, "NaN after layer %d ffn", e[ERRF_NAN_FFN] - 1);
    else if (e[ERRF_NAN_LOGITS]) status = set_error(GGC_ERR_INFERENCE, "NaN in logits");
    else if (e[ERRF_KV_OVERFLOW]) {
        status = set_error(GGC_ERR_KV_CACHE_OVERFLOW, "KvCacheOverflow { seq_len: %d, max_seq: %u }", e[ERRF_KV_OVERFLOW] - 1,
                           m->hp.max_ctx);
    } else if (e[ERRF_BAD_POS]) status = set_error(GGC_ERR_INFERENCE, "position outside [0, %u)", m->hp.max_ctx);
    else if (e[ERRF_TIMEOUT]) status = set_error(GGC_ERR_TIMEOUT, "a bounded device wait expired");
    return status;
}

int check_run(ggc_model* m) {
    m->cache_len = m->rb->st.slot;
    const int status = errf_status(m, m->rb->errf);
    if (status != GGC_OK) {
        cudaMemsetAsync(m->errf, 0, sizeof(int) * ERRF_COUNT, m->ctx->stream);
        cudaStreamSynchronize(m->ctx->stream);
    }
    return status;
}

// ---- batched prefill (prefill.cuh) -------------------------------------------
constexpr uint32_t PF_CHUNK = MM_TOKENS;     // tokens per pass (one k_mm_tc grid row: W dequantised once)
constexpr uint64_t PREFILL_MIN = 64;          // batch the prompt prefix from this many tokens on

template <int DT>
struct RunEmbedRows {
    static void run(ggc_ctx* ctx, const uint8_t* raw, uint64_t rows, uint32_t d, const uint32_t* tok, uint32_t n,
                    float* h, int* errf, cudaError_t* err) {
        *err = launch(ctx, k_embed_rows<DT>, dim3(n), dim3(256), 0, raw, rows, d, tok, h, errf);
    }
};

int ensure_prefill_buffers(ggc_model* m) {
    if (m->pf_h) return GGC_OK;
    const ggc_hparams& hp = m->hp;
    uint32_t fmax = 0;
    for (auto& L : m->layers) fmax = std::max(fmax, L.f_l);
    m->pf_ldy = std::max(m->qdim + 2 * m->kvdim, 2 * fmax);
    GGC_TRY(dalloc(m, &m->pf_h, (size_t)PF_CHUNK * hp.embed_dim));
    GGC_TRY(dalloc(m, &m->pf_y, (size_t)PF_CHUNK * m->pf_ldy));
    GGC_TRY(dalloc(m, &m->pf_q, (size_t)PF_CHUNK * m->qdim));
    GGC_TRY(dalloc(m, &m->pf_o, (size_t)PF_CHUNK * m->qdim));
    GGC_TRY(dalloc(m, &m->pf_tok, PF_CHUNK));
    GGC_TRY(dalloc(m, &m->pf_pos, PF_CHUNK));
    return GGC_OK;
}

// y[:, 0:rows] (ldy) (+)= rmsnorm / swiglu / plain(x) . W^T for a raw weight
// X of a batch split into the product's bf16 hi / lo tiles once, for every
// weight that multiplies the same input (q, k, v; up, gate)
struct SplitX {
    uint8_t* xh = nullptr;
    uint8_t* xl = nullptr;
    uint32_t kpad = 0;
    uint32_t cols = 0;
};
// nan_val != 0 (RMSNorm only): the split is the NaN guard of x as well
int mm_split_x(ggc_model* m, const float* x, const float* x2, uint32_t n, uint32_t cols, uint32_t ldx, int pro,
               SplitX* sx, int nan_slot = 0, int nan_val = 0) {
    sx->cols = cols;
    return split_rows(m->ctx, x, x2, n, cols, ldx, pro, &sx->xh, &sx->xl, &sx->kpad, m->errf, nan_slot, nan_val);
}
int mm_split_w(ggc_model* m, const RawMat& w, const SplitX& sx, uint32_t n, float* y, uint32_t ldy, const float* resid) {
    if (w.cols != sx.cols) return set_error(GGC_ERR_INVALID_ARG, "prefill product: %u columns, split input %u", w.cols, sx.cols);
    cudaError_t err = cudaSuccess;
    if (!dispatch_dtype<RunMM>(w.dtype, m->ctx, (const uint8_t*)w.p, w.rows, w.cols, (const uint8_t*)sx.xh,
                               (const uint8_t*)sx.xl, n, sx.kpad, y, ldy, resid, m->errf, &err))
        return set_dequant_error(w.dtype, 0, 0, "prefill dtype");
    GGC_CUDA_TRY(err);
    return GGC_OK;
}
int mm_raw(ggc_model* m, const RawMat& w, const float* x, const float* x2, uint32_t n, uint32_t ldx, int pro, float* y,
           uint32_t ldy, const float* resid) {
    SplitX sx;
    GGC_TRY(mm_split_x(m, x, x2, n, w.cols, ldx, pro, &sx));
    return mm_split_w(m, w, sx, n, y, ldy, resid);
}

// K/V of `count` prompt tokens at cache slots [cache_len, cache_len + count)
// through every layer in passes of PF_CHUNK tokens: embed, then per layer
// RMSNorm -> q/k/v (k_mm_tc) -> bias + RoPE + cache append -> causal attention
// -> attn_output (+ residual) -> RMSNorm -> up, gate -> silu(gate) * up -> down
// (+ residual), with the NaN guards (llama.rs:266-350).  The last layer stops
// after its K/V: nothing of these tokens but the cache is used later (the last
// prompt token runs through the decode step for its logits).  Tensor parallel:
// the attn_output / ffn_down partials are all-reduced with NCCL (rank 0 adds
// the residual).
int prefill_batch(ggc_model* m, const uint32_t* tokens, const int64_t* positions, uint64_t count) {
    ggc_ctx* ctx = m->ctx;
    const ggc_hparams& hp = m->hp;
    const uint32_t d = hp.embed_dim, hd = m->hd;
    const bool tp = ctx->world > 1;
    const bool lead = !tp || ctx->rank == 0;
    GGC_TRY(ensure_prefill_buffers(m));
    std::vector<uint32_t> htok(count);
    std::vector<int64_t> hpos(count);
    GGC_CUDA_TRY(cudaMemcpy(htok.data(), tokens, count * sizeof(uint32_t), cudaMemcpyDefault));
    GGC_CUDA_TRY(cudaMemcpy(hpos.data(), positions, count * sizeof(int64_t), cudaMemcpyDefault));
    for (uint64_t i = 0; i < count; ++i)
        if (hpos[i] < 0 || hpos[i] >= (int64_t)hp.max_ctx)
            return set_error(GGC_ERR_INFERENCE, "position outside [0, %u)", hp.max_ctx);
    GGC_CUDA_TRY(cudaMemsetAsync(m->errf, 0, sizeof(int) * ERRF_COUNT, ctx->stream));
    const uint64_t base = m->cache_len;
    const size_t layer_kv = (size_t)hp.max_ctx * m->kvdim * m->kv_elem;
    const float inv = 1.0f / sqrtf((float)hd);
    auto allreduce_h = [&](uint32_t n) -> int {
        if (!tp) return GGC_OK;
        const ncclResult_t r = nccl().AllReduce(m->pf_h, m->pf_h, (size_t)n * d, ncclFloat, ncclSum, ctx->comm, ctx->stream);
        return r == ncclSuccess ? GGC_OK : nccl_error("ncclAllReduce", r);
    };
    for (uint64_t done = 0; done < count; done += PF_CHUNK) {
        const uint32_t n = (uint32_t)std::min<uint64_t>(PF_CHUNK, count - done);
        const uint32_t slot0 = (uint32_t)(base + done);
        GGC_CUDA_TRY(cudaMemcpyAsync(m->pf_tok, htok.data() + done, n * sizeof(uint32_t), cudaMemcpyHostToDevice,
                                     ctx->stream));
        GGC_CUDA_TRY(cudaMemcpyAsync(m->pf_pos, hpos.data() + done, n * sizeof(int64_t), cudaMemcpyHostToDevice,
                                     ctx->stream));
        cudaError_t err = cudaSuccess;
        dispatch_dtype<RunEmbedRows>(m->embd_dtype, ctx, (const uint8_t*)m->embd, m->embd_rows, d,
                                     (const uint32_t*)m->pf_tok, n, m->pf_h, m->errf, &err);
        GGC_CUDA_TRY(err);
        for (uint32_t l = 0; l < hp.n_layers; ++l) {
            ModelLayer& L = m->layers[l];
            const bool last = l + 1 == hp.n_layers;
            void* kc = (uint8_t*)m->kcache + l * layer_kv;
            void* vc = (uint8_t*)m->vcache + l * layer_kv;
            float* yq = m->pf_y;
            float* yk = m->pf_y + m->qdim;
            float* yv = yk + m->kvdim;
            const uint32_t ldy = m->qdim + 2 * m->kvdim;
            SplitX sx;   // RMSNorm(h) split once for q, k, v; the NaN guard after layer l - 1's ffn
            GGC_TRY(mm_split_x(m, m->pf_h, L.attn_norm, n, d, d, MMP_RMSNORM, &sx, ERRF_NAN_FFN, (int)l));
            if (!last) GGC_TRY(mm_split_w(m, L.rq, sx, n, yq, ldy, nullptr));
            GGC_TRY(mm_split_w(m, L.rk, sx, n, yk, ldy, nullptr));
            GGC_TRY(mm_split_w(m, L.rv, sx, n, yv, ldy, nullptr));
            GGC_CUDA_TRY(launch(ctx, k_qkv_post, dim3(n), dim3(256), 0, (const float*)m->pf_y, ldy, m->qdim, m->kvdim, hd,
                                (const float*)L.bq, (const float*)L.bk, (const float*)L.bv, (const int64_t*)m->pf_pos,
                                (const float2*)m->rope, slot0, last ? (float*)nullptr : m->pf_q, kc, vc, hp.max_ctx,
                                hp.kv_f16 ? 1 : 0));
            if (last) break;
            const dim3 ag(m->heads_l, cdiv<uint32_t>(n, PA_Q));
            if (hd == 64)
                GGC_CUDA_TRY(launch(ctx, k_attn_prefill<64>, ag, dim3(PA_WARPS * 32), pa_smem<64>(), (const float*)m->pf_q,
                                    (const void*)kc, (const void*)vc, (const int64_t*)m->pf_pos, slot0, n, m->heads_l,
                                    m->kv_heads_l, hp.max_ctx, hp.kv_f16 ? 1 : 0, inv, m->pf_o));
            else
                GGC_CUDA_TRY(launch(ctx, k_attn_prefill<128>, ag, dim3(PA_WARPS * 32), pa_smem<128>(), (const float*)m->pf_q,
                                    (const void*)kc, (const void*)vc, (const int64_t*)m->pf_pos, slot0, n, m->heads_l,
                                    m->kv_heads_l, hp.max_ctx, hp.kv_f16 ? 1 : 0, inv, m->pf_o));
            // attn_output + residual (rank 0 alone under tensor parallelism), all-reduce
            GGC_TRY(mm_raw(m, L.ro, m->pf_o, nullptr, n, m->qdim, MMP_PLAIN, m->pf_h, d, lead ? m->pf_h : nullptr));
            GGC_TRY(allreduce_h(n));
            // ffn: up | gate side by side in pf_y, then down (+ residual); the split
            // (once for up and gate) is the NaN guard after this layer's attention
            const uint32_t fl = L.f_l, ldu = 2 * fl;
            GGC_TRY(mm_split_x(m, m->pf_h, L.ffn_norm, n, d, d, MMP_RMSNORM, &sx, ERRF_NAN_ATTN, (int)l + 1));
            GGC_TRY(mm_split_w(m, L.rup, sx, n, m->pf_y, ldu, nullptr));
            GGC_TRY(mm_split_w(m, L.rgate, sx, n, m->pf_y + fl, ldu, nullptr));
            GGC_TRY(mm_raw(m, L.rdown, m->pf_y + fl, m->pf_y, n, ldu, MMP_SWIGLU, m->pf_h, d, lead ? m->pf_h : nullptr));
            GGC_TRY(allreduce_h(n));   // its NaN guard: the next layer's q/k/v split
        }
    }
    int hf[ERRF_COUNT];
    GGC_CUDA_TRY(cudaMemcpyAsync(hf, m->errf, sizeof(hf), cudaMemcpyDeviceToHost, ctx->stream));
    GGC_TRY(ctx_sync(ctx));
    const int status = errf_status(m, hf);
    if (status != GGC_OK) {
        cudaMemsetAsync(m->errf, 0, sizeof(int) * ERRF_COUNT, ctx->stream);
        cudaStreamSynchronize(ctx->stream);
        return status;
    }
    const uint32_t slot = (uint32_t)(base + count);
    GGC_CUDA_TRY(cudaMemcpyAsync(&m->st->slot, &slot, sizeof(slot), cudaMemcpyHostToDevice, ctx->stream));
    GGC_TRY(ctx_sync(ctx));
    m->cache_len = base + count;
    return GGC_OK;
}

}  // namespace

// LlamaModel::forward (llama.rs:214-224, :266-350)
extern "C" int ggc_model_forward(ggc_model* m, const uint32_t* tokens, const int64_t* positions, uint64_t n, float* logits,
                                 uint32_t* argmax) {
    if (!m) return set_error(GGC_ERR_INVALID_ARG, "null model");
    if (n == 0) return set_error(GGC_ERR_INFERENCE, "empty input");
    if (!tokens || !positions) return set_error(GGC_ERR_INVALID_ARG, "null tokens/positions");
    ggc_ctx* ctx = m->ctx;
    DeviceGuard g(ctx->device);
    if (m->cache_len + n > m->hp.max_ctx)
        return set_error(GGC_ERR_KV_CACHE_OVERFLOW, "KvCacheOverflow { seq_len: %llu, max_seq: %u }",
                         (unsigned long long)(m->cache_len + n), m->hp.max_ctx);
    // a long prompt prefix goes through the batched tensor-core path; the last
    // token (whose logits are returned) through the decode step
    uint64_t first = 0;
    if (m->prefill && n > PREFILL_MIN) {
        GGC_TRY(prefill_batch(m, tokens, positions, n - 1));
        first = n - 1;
    }
    const cudaMemcpyKind k1 = is_device_ptr(tokens) ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    const cudaMemcpyKind k2 = is_device_ptr(positions) ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    GGC_CUDA_TRY(cudaMemcpyAsync(m->in_tok, tokens + first, (n - first) * sizeof(uint32_t), k1, ctx->stream));
    GGC_CUDA_TRY(cudaMemcpyAsync(m->in_pos, positions + first, (n - first) * sizeof(int64_t), k2, ctx->stream));
    GGC_TRY(run_steps(m, n - first, 0, -1, n - first));
    // host logits go through the model's pinned buffer: a copy into pageable memory
    // would block the host until the stream drains, past ctx_sync's deadline
    const size_t lbytes = (size_t)m->hp.vocab_size * sizeof(float);
    const bool dev_logits = logits && is_device_ptr(logits);
    if (logits)
        GGC_CUDA_TRY(cudaMemcpyAsync(dev_logits ? (void*)logits : (void*)m->logits_host, m->logits, lbytes,
                                     dev_logits ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, ctx->stream));
    GGC_TRY(ctx_sync(ctx));
    if (logits && !dev_logits) memcpy(logits, m->logits_host, lbytes);
    GGC_TRY(check_run(m));
    if (argmax) {
        const uint32_t id = (uint32_t)(m->rb->key & 0xFFFFFFFFull);
        if (is_device_ptr(argmax)) {
            GGC_CUDA_TRY(cudaMemcpyAsync(argmax, &id, sizeof(id), cudaMemcpyHostToDevice, ctx->stream));
            GGC_TRY(ctx_sync(ctx));
        }
        else *argmax = id;
    }
    return GGC_OK;
}

extern "C" int ggc_model_generate_greedy(ggc_model* m, const uint32_t* prompt, uint64_t n_prompt, int64_t start_pos,
                                         uint64_t max_tokens, int64_t eos, uint32_t* out_ids, uint64_t* n_out) {
    if (!m || !n_out) return set_error(GGC_ERR_INVALID_ARG, "null argument");
    *n_out = 0;
    if (n_prompt == 0) return set_error(GGC_ERR_INFERENCE, "prompt tokenize empty");
    if (!prompt || (max_tokens && !out_ids)) return set_error(GGC_ERR_INVALID_ARG, "null buffer");
    ggc_ctx* ctx = m->ctx;
    DeviceGuard g(ctx->device);
    if (m->cache_len + n_prompt + max_tokens > m->hp.max_ctx)
        return set_error(GGC_ERR_KV_CACHE_OVERFLOW, "KvCacheOverflow { seq_len: %llu, max_seq: %u }",
                         (unsigned long long)(m->cache_len + n_prompt + max_tokens), m->hp.max_ctx);
    std::vector<int64_t> pos(n_prompt);
    for (uint64_t i = 0; i < n_prompt; ++i) pos[i] = start_pos + (int64_t)i;
    uint64_t first = 0;   // prompt prefix through the batched path (as ggc_model_forward)
    if (m->prefill && n_prompt > PREFILL_MIN) {
        GGC_TRY(prefill_batch(m, prompt, pos.data(), n_prompt - 1));
        first = n_prompt - 1;
    }
    const uint64_t rest = n_prompt - first;
    const cudaMemcpyKind k1 = is_device_ptr(prompt) ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    GGC_CUDA_TRY(cudaMemcpyAsync(m->in_tok, prompt + first, rest * sizeof(uint32_t), k1, ctx->stream));
    GGC_CUDA_TRY(cudaMemcpyAsync(m->in_pos, pos.data() + first, rest * sizeof(int64_t), cudaMemcpyHostToDevice,
                                 ctx->stream));
    GGC_TRY(run_steps(m, rest, max_tokens, eos, rest + max_tokens));
    GGC_TRY(ctx_sync(ctx));
    const uint64_t got = (uint64_t)m->rb->st.n_out;
    if (got) {
        GGC_CUDA_TRY(cudaMemcpyAsync(out_ids, m->out_ids, got * sizeof(uint32_t), cudaMemcpyDefault, ctx->stream));
        GGC_TRY(ctx_sync(ctx));
    }
    *n_out = got;
    return check_run(m);
}

extern "C" int ggc_model_wait(ggc_model* m, uint32_t* out_ids, uint64_t* n_out);

// Continues greedy decoding from the last forward's logits: `steps` iterations of
// sample -> forward(1 token), all on the device (no host round trip per token).
extern "C" int ggc_model_decode(ggc_model* m, uint64_t steps, int64_t eos, int sync, uint32_t* out_ids, uint64_t* n_out) {
    if (!m) return set_error(GGC_ERR_INVALID_ARG, "null model");
    if (n_out) *n_out = 0;
    if (m->cache_len == 0) return set_error(GGC_ERR_INFERENCE, "decode needs a previous forward");
    if (m->cache_len + steps > m->hp.max_ctx)
        return set_error(GGC_ERR_KV_CACHE_OVERFLOW, "KvCacheOverflow { seq_len: %llu, max_seq: %u }",
                         (unsigned long long)(m->cache_len + steps), m->hp.max_ctx);
    if (steps == 0) return GGC_OK;
    ggc_ctx* ctx = m->ctx;
    DeviceGuard g(ctx->device);
    int32_t ctl[6] = {0, 0, (int32_t)steps, (int32_t)(eos < 0 ? -1 : eos), 0, 0};
    GGC_TRY(put_ctl(m, ctl));
    GGC_CUDA_TRY(launch(ctx, k_decode_start, dim3(1), dim3(32), 0, m->st, (const unsigned long long*)m->argmax_key,
                        m->out_ids, m->errf));
    for (uint64_t i = 0; i < steps; ++i) {
        GGC_CUDA_TRY(cudaGraphLaunch(m->graph, ctx->stream));
        ctx->launches += m->launches_per_step;
    }
    m->cache_len += steps;   // provisional; corrected by the readback below / ggc_model_wait
    if (!sync) return GGC_OK;
    return ggc_model_wait(m, out_ids, n_out);
}

// Waits for the model's queued work, validates it and returns the generated ids.
extern "C" int ggc_model_wait(ggc_model* m, uint32_t* out_ids, uint64_t* n_out) {
    if (!m) return set_error(GGC_ERR_INVALID_ARG, "null model");
    ggc_ctx* ctx = m->ctx;
    DeviceGuard g(ctx->device);
    GGC_CUDA_TRY(cudaMemcpyAsync(&m->rb->st, m->st, sizeof(StepState), cudaMemcpyDeviceToHost, ctx->stream));
    GGC_CUDA_TRY(cudaMemcpyAsync(m->rb->errf, m->errf, sizeof(int) * ERRF_COUNT, cudaMemcpyDeviceToHost, ctx->stream));
    GGC_CUDA_TRY(cudaMemcpyAsync(&m->rb->key, m->argmax_key, sizeof(unsigned long long), cudaMemcpyDeviceToHost, ctx->stream));
    GGC_TRY(ctx_sync(ctx));
    const uint64_t got = (uint64_t)m->rb->st.n_out;
    if (out_ids && got) {
        GGC_CUDA_TRY(cudaMemcpyAsync(out_ids, m->out_ids, got * sizeof(uint32_t), cudaMemcpyDefault, m->ctx->stream));
        GGC_TRY(ctx_sync(m->ctx));
    }
    if (n_out) *n_out = got;
    return check_run(m);
}

extern "C" uint64_t ggc_model_cache_len(const ggc_model* m) { return m ? m->cache_len : 0; }

// Sampler::sample (sampler.rs:86-186) on the device (k_sample, sample.cuh)
extern "C" int ggc_sample(ggc_ctx* ctx, const float* logits, uint64_t vocab, const ggc_sampler_config* cfg,
                          const uint32_t* seen, uint64_t n_seen, float u, uint32_t* out_id) {
    if (!ctx || !logits || !cfg || !out_id || (n_seen && !seen)) return set_error(GGC_ERR_INVALID_ARG, "null argument");
    if (vocab == 0) return set_error(GGC_ERR_INFERENCE, "logits empty");
    if (vocab > 0xFFFFFFFFull) return set_error(GGC_ERR_INVALID_ARG, "vocabulary too large");
    if (!(u >= 0.0f && u < 1.0f)) return set_error(GGC_ERR_INVALID_ARG, "u must lie in [0, 1)");
    if (cfg->temperature > 1e-6f) {
        const bool use_k = cfg->top_k > 0 && cfg->top_k < vocab;
        if ((use_k ? (uint64_t)cfg->top_k : vocab) > (uint64_t)SAMPLE_MAX_K)
            return set_error(GGC_ERR_INVALID_ARG, "device sampling keeps at most %d candidates: set top_k in [1, %d]",
                             SAMPLE_MAX_K, SAMPLE_MAX_K);
    }
    DeviceGuard g(ctx->device);
    std::vector<uint32_t> ids(seen, seen + n_seen);   // the reference's seen map: distinct keys
    std::sort(ids.begin(), ids.end());
    ids.erase(std::unique(ids.begin(), ids.end()), ids.end());
    const void* dl;
    GGC_TRY(dev_in(ctx, 0, logits, vocab * sizeof(float), &dl));
    GGC_TRY(ensure_stage(ctx, 6, vocab * sizeof(float)));
    GGC_TRY(ensure_stage(ctx, 7, (ids.size() + 2) * sizeof(uint32_t)));
    uint32_t* io = (uint32_t*)ctx->stage[7];   // [0] id, [1] error flag, [2..] seen ids
    GGC_CUDA_TRY(cudaMemsetAsync(io, 0, 2 * sizeof(uint32_t), ctx->stream));
    if (!ids.empty())
        GGC_CUDA_TRY(cudaMemcpyAsync(io + 2, ids.data(), ids.size() * sizeof(uint32_t), cudaMemcpyHostToDevice,
                                     ctx->stream));
    const SampleCfg c{cfg->temperature, cfg->top_k, cfg->top_p, cfg->min_p, cfg->repeat_penalty};
    GGC_CUDA_TRY(launch(ctx, k_sample, dim3(1), dim3(SAMPLE_THREADS), 0, (const float*)dl, (uint32_t)vocab,
                        (const uint32_t*)(io + 2), (uint32_t)ids.size(), c, u, (float*)ctx->stage[6], io,
                        (int*)(io + 1)));
    uint32_t res[2] = {0, 0};
    GGC_CUDA_TRY(cudaMemcpyAsync(res, io, sizeof(res), cudaMemcpyDeviceToHost, ctx->stream));
    GGC_TRY(ctx_sync(ctx));
    if (res[1]) return set_error(GGC_ERR_INFERENCE, "NaN in logits");
    *out_id = res[0];
    return GGC_OK;
}

// the same over the logits of the model's last forward / decode step (device)
extern "C" int ggc_model_sample(ggc_model* m, const ggc_sampler_config* cfg, const uint32_t* seen, uint64_t n_seen,
                                float u, uint32_t* out_id) {
    if (!m) return set_error(GGC_ERR_INVALID_ARG, "null model");
    return ggc_sample(m->ctx, m->logits, m->hp.vocab_size, cfg, seen, n_seen, u, out_id);
}

extern "C" int ggc_allreduce_probe(ggc_ctx* ctx, uint32_t rows, int peer_writes, const float* part0,
                                   const float* part1, float* out) {
    if (!ctx || !part0 || !part1 || !out || rows == 0) return set_error(GGC_ERR_INVALID_ARG, "null argument or no rows");
    DeviceGuard g(ctx->device);
    // the group's buffers: rank 0's receive words [2 phases][2 ranks][rows], a
    // second buffer standing in for the peer's, the step counter, partials, result
    const size_t words = 2u * 2u * rows;
    unsigned long long* buf = nullptr;
    float* d = nullptr;
    uint32_t* step = nullptr;
    ArGroup* dg = nullptr;
    int* errf = nullptr;
    int st = ctx_errf(ctx, &errf);
    cudaError_t e = st == GGC_OK ? cudaMalloc(&buf, 2 * words * sizeof(unsigned long long)) : cudaErrorUnknown;
    if (e == cudaSuccess) e = cudaMalloc(&d, 3u * rows * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&step, sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMalloc(&dg, sizeof(ArGroup));
    if (e == cudaSuccess) e = cudaMemsetAsync(buf, 0, 2 * words * sizeof(unsigned long long), ctx->stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(errf, 0, sizeof(int) * ERRF_COUNT, ctx->stream);
    ArGroup hg{};
    hg.buf[0] = buf;
    hg.buf[1] = buf + words;
    hg.world = 2;
    hg.rank = 0;
    hg.stride = rows;
    hg.step = step;
    hg.per_step = 2;
    const uint32_t one = 1;
    if (e == cudaSuccess) e = cudaMemcpyAsync(step, &one, sizeof(one), cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dg, &hg, sizeof(hg), cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d, part0, rows * sizeof(float), cudaMemcpyDefault, ctx->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d + rows, part1, rows * sizeof(float), cudaMemcpyDefault, ctx->stream);
    if (e == cudaSuccess) {
        k_ar_probe<<<1, 32, 0, ctx->stream>>>(dg, rows, d, d + rows, peer_writes, d + 2 * rows, errf);
        e = cudaGetLastError();
    }
    int flags[ERRF_COUNT] = {0};
    if (e == cudaSuccess) e = cudaMemcpyAsync(flags, errf, sizeof(flags), cudaMemcpyDeviceToHost, ctx->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(out, d + 2 * rows, rows * sizeof(float), cudaMemcpyDefault, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    cudaFree(buf);
    cudaFree(d);
    cudaFree(step);
    cudaFree(dg);
    if (st != GGC_OK) return st;
    if (e != cudaSuccess) return set_error(GGC_ERR_CUDA, "allreduce probe: %s", cudaGetErrorString(e));
    if (flags[ERRF_TIMEOUT])
        return set_error(GGC_ERR_TIMEOUT, "all-reduce: the peer's partials did not arrive within the bounded poll");
    return GGC_OK;
}

extern "C" int ggc_model_allreduce_kind(const ggc_model* m) {
    if (!m || m->ctx->world < 2) return 0;
    return m->ar_p2p ? 2 : 1;
}

extern "C" int ggc_model_truncate(ggc_model* m, uint64_t new_len) {
    if (!m) return set_error(GGC_ERR_INVALID_ARG, "null model");
    if (new_len >= m->cache_len) return GGC_OK;   // cache.rs:86-93 only shrinks
    DeviceGuard g(m->ctx->device);
    const uint32_t slot = (uint32_t)new_len;
    GGC_CUDA_TRY(cudaMemcpyAsync(&m->st->slot, &slot, sizeof(slot), cudaMemcpyHostToDevice, m->ctx->stream));
    GGC_TRY(ctx_sync(m->ctx));
    m->cache_len = new_len;
    return GGC_OK;
}

extern "C" int ggc_model_reset_cache(ggc_model* m) { return ggc_model_truncate(m, 0); }

namespace {
// Copies `seq` rows of [seq][kvh * hd] (element size esz, host or device memory)
// into / out of the head-major cache rows [h][base .. base + seq) of one layer.
int kv_rows_to_cache(ggc_model* m, uint8_t* layer, const void* src, uint64_t base, uint64_t seq, size_t esz) {
    const size_t hd = m->hd, kvdim = m->kvdim;
    for (uint32_t h = 0; h < m->kv_heads_l; ++h)
        GGC_CUDA_TRY(cudaMemcpy2DAsync(layer + ((size_t)h * m->hp.max_ctx + base) * hd * esz, hd * esz,
                                       (const uint8_t*)src + h * hd * esz, kvdim * esz, hd * esz, seq, cudaMemcpyDefault,
                                       m->ctx->stream));
    GGC_TRY(ctx_sync(m->ctx));
    return GGC_OK;
}
int kv_cache_to_rows(ggc_model* m, const uint8_t* layer, void* dst, uint64_t seq, size_t esz) {
    const size_t hd = m->hd, kvdim = m->kvdim;
    for (uint32_t h = 0; h < m->kv_heads_l; ++h)
        GGC_CUDA_TRY(cudaMemcpy2DAsync((uint8_t*)dst + h * hd * esz, kvdim * esz,
                                       layer + (size_t)h * m->hp.max_ctx * hd * esz, hd * esz, hd * esz, seq,
                                       cudaMemcpyDefault, m->ctx->stream));
    GGC_TRY(ctx_sync(m->ctx));
    return GGC_OK;
}
}  // namespace

extern "C" int ggc_model_cache_append(ggc_model* m, uint32_t layer, const float* k, const float* v, uint64_t seq) {
    if (!m || !k || !v) return set_error(GGC_ERR_INVALID_ARG, "null argument");
    if (layer >= m->hp.n_layers) return set_error(GGC_ERR_INVALID_ARG, "layer %u out of range", layer);
    // every layer must hold the same number of tokens; the slot advances when the last layer is appended
    const uint64_t base = m->cache_len;
    if (base + seq > m->hp.max_ctx)
        return set_error(GGC_ERR_KV_CACHE_OVERFLOW, "KvCacheOverflow { seq_len: %llu, max_seq: %u }",
                         (unsigned long long)(base + seq), m->hp.max_ctx);
    DeviceGuard g(m->ctx->device);
    GGC_TRY(ctx_sync(m->ctx));
    const size_t layer_kv = (size_t)m->hp.max_ctx * m->kvdim * m->kv_elem;
    const size_t n = (size_t)seq * m->kvdim;
    uint8_t* kd = (uint8_t*)m->kcache + layer * layer_kv;
    uint8_t* vd = (uint8_t*)m->vcache + layer * layer_kv;
    if (seq) {
        if (m->hp.kv_f16) {
            std::vector<__half> hk(n), hv(n);
            std::vector<float> fk(n), fv(n);
            GGC_CUDA_TRY(cudaMemcpy(fk.data(), k, n * 4, cudaMemcpyDefault));
            GGC_CUDA_TRY(cudaMemcpy(fv.data(), v, n * 4, cudaMemcpyDefault));
            for (size_t i = 0; i < n; ++i) { hk[i] = __float2half_rn(fk[i]); hv[i] = __float2half_rn(fv[i]); }
            GGC_TRY(kv_rows_to_cache(m, kd, hk.data(), base, seq, 2));
            GGC_TRY(kv_rows_to_cache(m, vd, hv.data(), base, seq, 2));
        } else {
            GGC_TRY(kv_rows_to_cache(m, kd, k, base, seq, 4));
            GGC_TRY(kv_rows_to_cache(m, vd, v, base, seq, 4));
        }
    }
    if (layer == m->hp.n_layers - 1) {
        const uint32_t slot = (uint32_t)(base + seq);
        GGC_CUDA_TRY(cudaMemcpyAsync(&m->st->slot, &slot, sizeof(slot), cudaMemcpyHostToDevice, m->ctx->stream));
        GGC_TRY(ctx_sync(m->ctx));
        m->cache_len = base + seq;
    }
    return GGC_OK;
}

extern "C" int ggc_model_cache_read(ggc_model* m, uint32_t layer, float* k, float* v) {
    if (!m || !k || !v) return set_error(GGC_ERR_INVALID_ARG, "null argument");
    if (layer >= m->hp.n_layers) return set_error(GGC_ERR_INVALID_ARG, "layer %u out of range", layer);
    DeviceGuard g(m->ctx->device);
    GGC_TRY(ctx_sync(m->ctx));
    const size_t layer_kv = (size_t)m->hp.max_ctx * m->kvdim * m->kv_elem;
    const uint64_t len = m->cache_len;
    const size_t n = (size_t)len * m->kvdim;
    if (n == 0) return GGC_OK;
    const uint8_t* kd = (const uint8_t*)m->kcache + layer * layer_kv;
    const uint8_t* vd = (const uint8_t*)m->vcache + layer * layer_kv;
    if (m->hp.kv_f16) {
        std::vector<__half> hk(n), hv(n);
        GGC_TRY(kv_cache_to_rows(m, kd, hk.data(), len, 2));
        GGC_TRY(kv_cache_to_rows(m, vd, hv.data(), len, 2));
        std::vector<float> fk(n), fv(n);
        for (size_t i = 0; i < n; ++i) { fk[i] = __half2float(hk[i]); fv[i] = __half2float(hv[i]); }
        GGC_CUDA_TRY(cudaMemcpyAsync(k, fk.data(), n * 4, cudaMemcpyDefault, m->ctx->stream));
        GGC_CUDA_TRY(cudaMemcpyAsync(v, fv.data(), n * 4, cudaMemcpyDefault, m->ctx->stream));
        GGC_TRY(ctx_sync(m->ctx));
    } else {
        GGC_TRY(kv_cache_to_rows(m, kd, k, len, 4));
        GGC_TRY(kv_cache_to_rows(m, vd, v, len, 4));
    }
    return GGC_OK;
}
