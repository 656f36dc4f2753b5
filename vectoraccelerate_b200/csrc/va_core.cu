// va_core.cu -- errors, contexts, buffers, bounded waits and seeded data generation.
//
// Replaces the reference's core runtime on the hot path: Metal4Context (device, queue,
// executeAndWait; Core/Metal4Context.swift:97-488) and BufferPool (Core/BufferPool.swift:89-221).
// A context is one CUDA device plus one stream; stream order replaces Metal barriers.
#include <chrono>
#include <cmath>
#include <cstring>
#include <thread>

#include "va_internal.cuh"

#include <nvtx3/nvToolsExt.h>

static thread_local char g_last_error[1024] = "";

int va_log_level() {
    static const int level = [] {
        const char* e = getenv("VA_LOG_LEVEL");
        return e ? atoi(e) : 0;
    }();
    return level;
}

int va_set_error(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    if (va_log_level() >= 1) fprintf(stderr, "[libva_cuda] error %d: %s\n", code, g_last_error);
    return code;
}

void va_log_info(const char* fmt, ...) {
    if (va_log_level() < 2) return;
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    fprintf(stderr, "[libva_cuda] %s\n", buf);
}

VaRange::VaRange(const char* name) { nvtxRangePushA(name); }
VaRange::~VaRange() { nvtxRangePop(); }

int va_check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return va_set_error(VA_ERR_CUDA, "launch of %s failed: %s", what, cudaGetErrorString(e));
    return VA_OK;
}

int va_workspace(va_context* ctx, size_t bytes, void** out) {
    if (bytes == 0) bytes = 256;
    if (ctx->ws_bytes < bytes) {
        // Grow: the old scratch may still be in use by enqueued work, so wait first.
        if (ctx->ws) {
            VA_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
            VA_CUDA_TRY(cudaFree(ctx->ws));
            ctx->ws = nullptr;
            ctx->ws_bytes = 0;
        }
        size_t sz = bytes + bytes / 8;
        cudaError_t e = cudaMalloc(&ctx->ws, sz);
        if (e != cudaSuccess) {
            ctx->ws = nullptr;
            return va_set_error(VA_ERR_OOM, "workspace allocation of %zu bytes failed: %s", sz, cudaGetErrorString(e));
        }
        ctx->ws_bytes = sz;
    }
    *out = ctx->ws;
    return VA_OK;
}

static void prof_free(va_context* ctx);

static int grow_buffer(va_context* ctx, void** buf, size_t* have, size_t bytes, const char* what) {
    if (bytes == 0) bytes = 256;
    if (*have < bytes) {
        if (*buf) {
            VA_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
            VA_CUDA_TRY(cudaFree(*buf));
            *buf = nullptr;
            *have = 0;
        }
        cudaError_t e = cudaMalloc(buf, bytes);
        if (e != cudaSuccess) {
            *buf = nullptr;
            return va_set_error(VA_ERR_OOM, "%s allocation of %zu bytes failed: %s", what, bytes, cudaGetErrorString(e));
        }
        *have = bytes;
    }
    return VA_OK;
}

int va_io_buffer(va_context* ctx, size_t bytes, void** out) {
    VA_TRY(grow_buffer(ctx, &ctx->io, &ctx->io_bytes, bytes, "staging"));
    *out = ctx->io;
    return VA_OK;
}

int va_aux_buffer(va_context* ctx, size_t bytes, void** out) {
    VA_TRY(grow_buffer(ctx, &ctx->aux, &ctx->aux_bytes, bytes, "auxiliary scratch"));
    *out = ctx->aux;
    return VA_OK;
}

extern "C" {

const char* va_last_error(void) { return g_last_error; }
int va_abi_version(void) { return VA_ABI_VERSION; }

int va_device_count(int* count) {
    VA_REQUIRE(count, "count must not be NULL");
    int c = 0;
    VA_CUDA_TRY(cudaGetDeviceCount(&c));
    *count = c;
    return VA_OK;
}

int va_context_create(const va_config* cfg, va_context** out) {
    VA_REQUIRE(out, "out must not be NULL");
    *out = nullptr;
    int ndev = 0;
    VA_CUDA_TRY(cudaGetDeviceCount(&ndev));
    int dev = cfg ? cfg->device : 0;
    VA_REQUIRE(dev >= 0 && dev < ndev, "device %d out of range (device count %d)", dev, ndev);
    VA_CUDA_TRY(cudaSetDevice(dev));
    cudaDeviceProp prop;
    VA_CUDA_TRY(cudaGetDeviceProperties(&prop, dev));
    if (prop.major != 10)
        return va_set_error(VA_ERR_UNSUPPORTED, "device %d is sm_%d%d; this build targets sm_100a (B200)", dev,
                            prop.major, prop.minor);
    va_context* c = new va_context();
    c->device = dev;
    c->sm_count = prop.multiProcessorCount;
    c->timeout_ms = (cfg && cfg->timeout_ms) ? cfg->timeout_ms : 120000u;
    if (cfg && cfg->stream) {
        c->stream = (cudaStream_t)cfg->stream;
        c->own_stream = false;
    } else {
        cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
        if (e != cudaSuccess) {
            delete c;
            return va_set_error(VA_ERR_CUDA, "cudaStreamCreate failed: %s", cudaGetErrorString(e));
        }
        c->own_stream = true;
    }
    if (cudaMalloc(&c->d_error, sizeof(int)) != cudaSuccess || cudaMemset(c->d_error, 0, sizeof(int)) != cudaSuccess ||
        cudaEventCreate(&c->ev_start) != cudaSuccess || cudaEventCreate(&c->ev_stop) != cudaSuccess ||
        cudaEventCreate(&c->ev_k0) != cudaSuccess || cudaEventCreate(&c->ev_k1) != cudaSuccess ||
        cudaEventCreateWithFlags(&c->ev_sync, cudaEventDisableTiming) != cudaSuccess) {
        va_context_destroy(c);
        return va_set_error(VA_ERR_CUDA, "context resource creation failed: %s", cudaGetErrorString(cudaGetLastError()));
    }
    *out = c;
    return VA_OK;
}

int va_context_destroy(va_context* ctx) {
    if (!ctx) return VA_OK;
    if (ctx->group) va_group_destroy(ctx);  // the group's other members and its communicators
    cudaSetDevice(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    if (ctx->ws) cudaFree(ctx->ws);
    if (ctx->gbuf) cudaFree(ctx->gbuf);
    if (ctx->io) cudaFree(ctx->io);
    if (ctx->aux) cudaFree(ctx->aux);
    if (ctx->d_error) cudaFree(ctx->d_error);
    if (ctx->ev_start) cudaEventDestroy(ctx->ev_start);
    if (ctx->ev_stop) cudaEventDestroy(ctx->ev_stop);
    if (ctx->ev_sync) cudaEventDestroy(ctx->ev_sync);
    if (ctx->ev_k0) cudaEventDestroy(ctx->ev_k0);
    if (ctx->ev_k1) cudaEventDestroy(ctx->ev_k1);
    prof_free(ctx);
    if (ctx->own_stream && ctx->stream) cudaStreamDestroy(ctx->stream);
    delete ctx;
    return VA_OK;
}

int va_context_stream(va_context* ctx, void** stream) {
    VA_REQUIRE(ctx && stream, "ctx and stream must not be NULL");
    *stream = (void*)ctx->stream;
    return VA_OK;
}

int va_synchronize(va_context* ctx) {
    VA_REQUIRE(ctx, "ctx must not be NULL");
    if (ctx->group) return va_group_synchronize(ctx);
    return va_sync_one(ctx);
}

}  // extern "C"

// Bounded wait for this context's stream, then its device error word (the internal form: a
// member of a group waits for its own work only).
int va_sync_one(va_context* ctx) {
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    VA_CUDA_TRY(cudaEventRecord(ctx->ev_sync, ctx->stream));
    auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        cudaError_t e = cudaEventQuery(ctx->ev_sync);
        if (e == cudaSuccess) break;
        if (e != cudaErrorNotReady) return va_set_error(VA_ERR_CUDA, "device work failed: %s", cudaGetErrorString(e));
        auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
        if ((unsigned)ms > ctx->timeout_ms)
            return va_set_error(VA_ERR_TIMEOUT, "va_synchronize: work not finished after %u ms", ctx->timeout_ms);
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
    int derr = 0;
    VA_CUDA_TRY(cudaMemcpy(&derr, ctx->d_error, sizeof(int), cudaMemcpyDeviceToHost));
    if (derr) {
        VA_CUDA_TRY(cudaMemset(ctx->d_error, 0, sizeof(int)));
        return va_set_error(VA_ERR_TIMEOUT, "a bounded device-side wait expired (device error %d)", derr);
    }
    return VA_OK;
}

bool va_host_pinned(const void* p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeHost;
}

int va_copy_to_device(va_context* ctx, void* dst_dev, const void* src_host, size_t bytes) {
    if (!va_host_pinned(src_host)) VA_TRY(va_synchronize(ctx));
    VA_CUDA_TRY(cudaMemcpyAsync(dst_dev, src_host, bytes, cudaMemcpyHostToDevice, ctx->stream));
    return VA_OK;
}

int va_copy_to_host(va_context* ctx, void* dst_host, const void* src_dev, size_t bytes) {
    if (!va_host_pinned(dst_host)) VA_TRY(va_synchronize(ctx));
    VA_CUDA_TRY(cudaMemcpyAsync(dst_host, src_dev, bytes, cudaMemcpyDeviceToHost, ctx->stream));
    return VA_OK;
}

int va_read_u32(va_context* ctx, const uint32_t* src_dev, uint32_t* out) {
    VA_TRY(va_sync_one(ctx));
    VA_CUDA_TRY(cudaMemcpyAsync(out, src_dev, 4, cudaMemcpyDeviceToHost, ctx->stream));
    return va_sync_one(ctx);
}

extern "C" {

int va_last_gpu_time_ms(va_context* ctx, float* ms) {
    VA_REQUIRE(ctx && ms, "ctx and ms must not be NULL");
    *ms = ctx->last_ms;
    return VA_OK;
}

}  // extern "C"

static void prof_free(va_context* ctx) {
    for (int i = 0; i < 2 * ctx->prof_cap; ++i) cudaEventDestroy(ctx->prof_ev[i]);
    delete[] ctx->prof_ev;
    ctx->prof_ev = nullptr;
    ctx->prof_cap = ctx->prof_n = 0;
}

extern "C" {

int va_profile_start(va_context* ctx, int capacity) {
    VA_REQUIRE(ctx, "ctx must not be NULL");
    VA_REQUIRE(capacity > 0 && capacity <= 100000, "capacity must be in 1..100000, got %d", capacity);
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    prof_free(ctx);
    ctx->prof_ev = new cudaEvent_t[2 * capacity];
    for (int i = 0; i < 2 * capacity; ++i) {
        cudaError_t e = cudaEventCreate(&ctx->prof_ev[i]);
        if (e != cudaSuccess) {
            ctx->prof_cap = i / 2;
            prof_free(ctx);
            return va_set_error(VA_ERR_CUDA, "cudaEventCreate failed: %s", cudaGetErrorString(e));
        }
    }
    ctx->prof_cap = capacity;
    ctx->prof_n = 0;
    return VA_OK;
}

int va_profile_stop(va_context* ctx, float* kernel_ms_total, int* calls) {
    VA_REQUIRE(ctx && kernel_ms_total && calls, "ctx, kernel_ms_total and calls must not be NULL");
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    VA_TRY(va_synchronize(ctx));
    float tot = 0.f;
    for (int i = 0; i < ctx->prof_n; ++i) {
        float ms = 0.f;
        VA_CUDA_TRY(cudaEventElapsedTime(&ms, ctx->prof_ev[2 * i], ctx->prof_ev[2 * i + 1]));
        tot += ms;
    }
    *kernel_ms_total = tot;
    *calls = ctx->prof_n;
    prof_free(ctx);
    return VA_OK;
}

int va_last_search_times(va_context* ctx, float* total_ms, float* kernel_ms) {
    VA_REQUIRE(ctx && total_ms && kernel_ms, "ctx, total_ms and kernel_ms must not be NULL");
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    VA_CUDA_TRY(cudaEventElapsedTime(total_ms, ctx->ev_start, ctx->ev_stop));
    *kernel_ms = 0.f;
    if (ctx->k_recorded) VA_CUDA_TRY(cudaEventElapsedTime(kernel_ms, ctx->ev_k0, ctx->ev_k1));
    return VA_OK;
}

// ------------------------------------------------------------------------------------------------
// Buffers
// ------------------------------------------------------------------------------------------------
int va_buffer_alloc(va_context* ctx, size_t bytes, void** dptr) {
    VA_REQUIRE(ctx && dptr, "ctx and dptr must not be NULL");
    VA_REQUIRE(bytes > 0, "bytes must be positive, got %zu", bytes);
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    cudaError_t e = cudaMalloc(dptr, bytes);
    if (e != cudaSuccess) {
        *dptr = nullptr;
        cudaGetLastError();
        return va_set_error(VA_ERR_OOM, "device allocation of %zu bytes failed: %s", bytes, cudaGetErrorString(e));
    }
    return VA_OK;
}

int va_buffer_free(va_context* ctx, void* dptr) {
    VA_REQUIRE(ctx, "ctx must not be NULL");
    if (!dptr) return VA_OK;
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    VA_TRY(va_synchronize(ctx));  // bounded: the stream's work may still use the buffer
    VA_CUDA_TRY(cudaFree(dptr));
    return VA_OK;
}

int va_host_alloc(va_context* ctx, size_t bytes, void** hptr) {
    VA_REQUIRE(ctx && hptr, "ctx and hptr must not be NULL");
    VA_REQUIRE(bytes > 0, "bytes must be positive, got %zu", bytes);
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    cudaError_t e = cudaMallocHost(hptr, bytes);
    if (e != cudaSuccess) {
        *hptr = nullptr;
        cudaGetLastError();
        return va_set_error(VA_ERR_OOM, "pinned host allocation of %zu bytes failed: %s", bytes, cudaGetErrorString(e));
    }
    return VA_OK;
}

int va_host_free(va_context* ctx, void* hptr) {
    VA_REQUIRE(ctx, "ctx must not be NULL");
    if (!hptr) return VA_OK;
    VA_CUDA_TRY(cudaFreeHost(hptr));
    return VA_OK;
}

int va_buffer_upload(va_context* ctx, void* dst, const void* src, size_t bytes) {
    VA_REQUIRE(ctx && dst && src, "ctx, dst and src must not be NULL");
    if (!bytes) return VA_OK;
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    return va_copy_to_device(ctx, dst, src, bytes);
}

int va_buffer_download(va_context* ctx, void* dst, const void* src, size_t bytes) {
    VA_REQUIRE(ctx && dst && src, "ctx, dst and src must not be NULL");
    if (!bytes) return VA_OK;
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    return va_copy_to_host(ctx, dst, src, bytes);
}

int va_buffer_copy(va_context* ctx, void* dst, const void* src, size_t bytes) {
    VA_REQUIRE(ctx && dst && src, "ctx, dst and src must not be NULL");
    if (!bytes) return VA_OK;
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    VA_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, ctx->stream));
    return VA_OK;
}

}  // extern "C"

// ------------------------------------------------------------------------------------------------
// Seeded generation: TestRNG restated on the device (Tests/VectorAccelerateTests/Utilities/
// TestRNG.swift:57-161). One thread per row; stream = row0 + row. The Box-Muller step runs in
// double and rounds once to float, identically to the CPU oracle's generator.
// ------------------------------------------------------------------------------------------------
namespace {

struct DevRng {
    uint64_t s;
    bool has;
    float cached;
};

__device__ __forceinline__ uint64_t rng_next(DevRng& r) {
    r.s = 2862933555777941757ULL * r.s + 3037000493ULL;
    return r.s;
}
__device__ __forceinline__ void rng_init(DevRng& r, uint64_t seed, uint64_t stream) {
    uint64_t base = seed == 0 ? 1 : seed;
    r.s = base ^ (stream << 32);
    r.has = false;
    r.cached = 0.f;
    for (int i = 0; i < 10; ++i) rng_next(r);
}
__device__ __forceinline__ float rng_f01(DevRng& r) { return (float)(rng_next(r) >> 40) / 16777216.0f; }
__device__ __forceinline__ float rng_gauss(DevRng& r) {
    if (r.has) {
        r.has = false;
        return r.cached;
    }
    float u1 = fmaxf(rng_f01(r), 1.1920928955078125e-07f);
    float u2 = rng_f01(r);
    double rr = sqrt(-2.0 * log((double)u1));
    double th = 6.283185307179586 * (double)u2;
    double sn, cs;
    sincos(th, &sn, &cs);
    r.cached = (float)(rr * sn);
    r.has = true;
    return (float)(rr * cs);
}

__global__ void k_gen_gaussian(float* out, int64_t rows, int dim, uint64_t seed, int64_t row0) {
    int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    DevRng g;
    rng_init(g, seed, (uint64_t)(row0 + r));
    float* o = out + r * dim;
    for (int j = 0; j < dim; ++j) o[j] = rng_gauss(g);
}

__global__ void k_gen_mixture(float* out, int64_t rows, int dim, uint64_t seed, int64_t row0, int nc, float sigma,
                              int normalize) {
    int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    DevRng g, gc;
    rng_init(g, seed, (uint64_t)(row0 + r));
    uint64_t c = (rng_next(g) >> 33) % (uint64_t)nc;
    rng_init(gc, seed ^ 0xC3A5C85C97CB3127ULL, c);
    float* o = out + r * dim;
    double ss = 0;
    for (int j = 0; j < dim; ++j) {
        float cj = rng_gauss(gc);
        float v = cj + sigma * rng_gauss(g);
        o[j] = v;
        ss += (double)v * v;
    }
    if (normalize && ss > 0) {
        double inv = 1.0 / sqrt(ss);
        for (int j = 0; j < dim; ++j) o[j] = (float)(o[j] * inv);
    }
}

__global__ void k_f32_to_bf16(const float* x, int64_t n, uint16_t* out) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        uint32_t u = __float_as_uint(x[i]);
        if ((u & 0x7FFFFFFFu) > 0x7F800000u) {
            out[i] = (uint16_t)((u >> 16) | 0x40);
            continue;
        }
        u += 0x7FFFu + ((u >> 16) & 1u);
        out[i] = (uint16_t)(u >> 16);
    }
}

}  // namespace

extern "C" {

int va_gen_gaussian(va_context* ctx, float* out, int64_t rows, int dim, uint64_t seed, int64_t row0) {
    VA_REQUIRE(ctx && out, "ctx and out must not be NULL");
    VA_REQUIRE(rows >= 0 && dim > 0, "rows must be >= 0 and dim > 0 (rows %lld, dim %d)", (long long)rows, dim);
    if (!rows) return VA_OK;
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    k_gen_gaussian<<<(unsigned)((rows + 127) / 128), 128, 0, ctx->stream>>>(out, rows, dim, seed, row0);
    return va_check_launch("k_gen_gaussian");
}

int va_gen_mixture(va_context* ctx, float* out, int64_t rows, int dim, uint64_t seed, int64_t row0, int n_centroids,
                   float sigma, int normalize) {
    VA_REQUIRE(ctx && out, "ctx and out must not be NULL");
    VA_REQUIRE(rows >= 0 && dim > 0 && n_centroids > 0, "rows >= 0, dim > 0 and n_centroids > 0 required");
    if (!rows) return VA_OK;
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    k_gen_mixture<<<(unsigned)((rows + 127) / 128), 128, 0, ctx->stream>>>(out, rows, dim, seed, row0, n_centroids,
                                                                           sigma, normalize);
    return va_check_launch("k_gen_mixture");
}

int va_f32_to_bf16(va_context* ctx, const float* x, int64_t n, uint16_t* out) {
    VA_REQUIRE(ctx && x && out, "ctx, x and out must not be NULL");
    if (n <= 0) return VA_OK;
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    int blocks = (int)std::min<int64_t>((n + 255) / 256, (int64_t)ctx->sm_count * 16);
    k_f32_to_bf16<<<blocks, 256, 0, ctx->stream>>>(x, n, out);
    return va_check_launch("k_f32_to_bf16");
}

}  // extern "C"
