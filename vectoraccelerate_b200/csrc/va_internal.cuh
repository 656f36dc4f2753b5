// va_internal.cuh -- shared host/device helpers of libva_cuda (not part of the public ABI).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "../../include/va_cuda.h"

// ------------------------------------------------------------------------------------------------
// Host-side error plumbing: every ABI function returns a status and records a thread-local message.
// ------------------------------------------------------------------------------------------------
int va_set_error(int code, const char* fmt, ...);

// Diagnostics (the reference's Logger, Core/Logger.swift:71, as an environment switch):
// VA_LOG_LEVEL=1 prints every error status with its message to stderr, 2 also prints
// informational lines (group set-up, per-search certificate counts). Off by default.
int va_log_level();
void va_log_info(const char* fmt, ...);

// NVTX range around a public entry point (visible in Nsight Systems / Compute; free otherwise).
struct VaRange {
    explicit VaRange(const char* name);
    ~VaRange();
};

#define VA_CUDA_TRY(expr)                                                                          \
    do {                                                                                           \
        cudaError_t _e = (expr);                                                                   \
        if (_e != cudaSuccess)                                                                     \
            return va_set_error(_e == cudaErrorMemoryAllocation ? VA_ERR_OOM : VA_ERR_CUDA,        \
                                "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(_e), __FILE__,  \
                                __LINE__);                                                         \
    } while (0)

#define VA_TRY(expr)                 \
    do {                             \
        int _s = (expr);             \
        if (_s != VA_OK) return _s;  \
    } while (0)

#define VA_REQUIRE(cond, ...)                                       \
    do {                                                            \
        if (!(cond)) return va_set_error(VA_ERR_INVALID_ARG, __VA_ARGS__); \
    } while (0)

// Device-side error codes written to the context's error word.
#define VA_DEVERR_WAIT_TIMEOUT 1

struct va_context {
    int device = 0;
    cudaStream_t stream = nullptr;
    bool own_stream = false;
    unsigned timeout_ms = 120000;
    int sm_count = 148;
    int* d_error = nullptr;  // device error word (bounded waits write it)
    cudaEvent_t ev_start = nullptr, ev_stop = nullptr, ev_sync = nullptr;
    cudaEvent_t ev_k0 = nullptr, ev_k1 = nullptr;  // bracket the dominant kernel of the last search
    bool k_recorded = false;
    // Optional per-call profile: event pairs around the dominant kernel of each search.
    cudaEvent_t* prof_ev = nullptr;  // 2 * prof_cap events
    int prof_cap = 0, prof_n = 0;
    float last_ms = 0.f;
    // Scratch cache: one growing device allocation reused in stream order.
    void* ws = nullptr;
    size_t ws_bytes = 0;
    // Staging for the host-buffer entry points (queries in, results out).
    void* io = nullptr;
    size_t io_bytes = 0;
    // Third scratch for results that must outlive the workspace within one call (gathered
    // queries and results of the exact fallback, the Hamming merge output).
    void* aux = nullptr;
    size_t aux_bytes = 0;
    // Counts of the last va_knn_search: queries the first tensor-core pass could not certify exact,
    // and queries that took the exact route.
    int64_t stat_uncertified = 0;
    int64_t stat_exact = 0;
    // Multi-GPU (va_group.cu): set on the front context of a group only (a process-per-GPU rank
    // context, or the first device of a multi-device context); member contexts stay plain.
    struct va_group* group = nullptr;
    // Scratch of the sharded search's exchange (local lists, gathered records, merge inputs).
    void* gbuf = nullptr;
    size_t gbuf_bytes = 0;
};

// Bounded wait for one context's own stream and device error word (internal waits of a search).
int va_sync_one(va_context* ctx);
// Group synchronisation and NCCL error polling behind va_synchronize (va_group.cu).
int va_group_synchronize(va_context* ctx);
void va_group_destroy(va_context* ctx);

// Host <-> device copies of the host-buffer entry points. With page-locked host memory
// (cudaHostAlloc / cudaHostRegister, e.g. torch's pin_memory) the copy is queued asynchronously.
// A copy from or to pageable memory blocks the calling thread until the stream reaches it, so it
// is issued only after a bounded wait for the stream (va_synchronize): work held up on the stream
// (a collective whose peer has gone) then ends the call with VA_ERR_TIMEOUT or VA_ERR_NCCL
// instead of blocking it for good. A pageable download has landed when the call returns.
bool va_host_pinned(const void* p);
int va_copy_to_device(va_context* ctx, void* dst_dev, const void* src_host, size_t bytes);
int va_copy_to_host(va_context* ctx, void* dst_host, const void* src_dev, size_t bytes);
// A 32-bit count written by device work on this context's stream (bounded wait, then the copy).
int va_read_u32(va_context* ctx, const uint32_t* src_dev, uint32_t* out);

// Device staging buffer of at least `bytes` for host-buffer calls.
int va_io_buffer(va_context* ctx, size_t bytes, void** out);
// Auxiliary device scratch of at least `bytes` (stream-ordered reuse across calls).
int va_aux_buffer(va_context* ctx, size_t bytes, void** out);

// Returns a device scratch pointer of at least `bytes` (stream-ordered reuse across calls).
int va_workspace(va_context* ctx, size_t bytes, void** out);
// Launch-error check right after a kernel launch.
int va_check_launch(const char* what);

struct va_database {
    va_context* ctx = nullptr;
    int64_t n = 0;
    int dim = 0;
    int dtype = VA_DTYPE_F32;
    uint32_t id_base = 0;
    void* rows = nullptr;        // original rows [n x dim] (fp32 or bf16)
    uint16_t* op = nullptr;      // bf16 tensor-core operand [n x dpad], zero padded (lazily built)
    uint16_t* op_cos = nullptr;  // bf16 unit-norm operand for cosine [n x dpad] (lazily built)
    float* op_f32 = nullptr;     // fp32 operand for tf32 [n x dpad] (lazily built)
    float* op_f32_cos = nullptr; // fp32 unit-norm operand for tf32 cosine (lazily built)
    float* norms2 = nullptr;     // |x|^2 fp32 per row (fp64 accumulated); +inf pad to 256 rows
    float* zbias = nullptr;      // 0 per row; +inf pad to 256 rows (filter bias of IP / cosine)
    int dpad = 0;                // dim rounded up to the tensor-core K block (64)
    bool op_alias = false;       // op aliases rows (bf16 rows with dim % 64 == 0)
    bool op_f32_alias = false;   // op_f32 aliases rows (fp32 rows with dim % 64 == 0)
    // Integer databases (int8 per-dimension codes, or 0/1 bytes of binary codes).
    int kind = 0;                // 0 float rows, 1 int8 codes of fp32 rows, 2 binary codes
    int8_t* codes = nullptr;     // [n x cpad] int8 tensor-core operand, zero padded
    int* code_norms = nullptr;   // |code|^2 (int8) or popcount (binary); padded to 256 rows
    float* sq_mins = nullptr;    // int8: per-dimension minimum
    float* sq_scales = nullptr;  // int8: per-dimension scale
    int cpad = 0;                // code row length (multiple of 128)
    int words = 0;               // binary: 32-bit words per code
    // Binary databases whose 0/1 expansion does not fit: one chunk of rows is expanded at a time.
    int8_t* stage = nullptr;     // [stage_rows x cpad] 0/1 bytes of the current chunk
    int* stage_norms = nullptr;  // popcounts of the current chunk (padded to 256 rows)
    int64_t stage_rows = 0;      // rows per chunk (0: not chunked)
    int64_t chunk_request = 0;   // rows per chunk set by the caller (0: automatic)
    int64_t cap = 0;             // rows allocated in every per-row array (0: exactly n)
    // Exactness certificate of the reduced-precision filter: maxima over all rows ever held, as
    // float bit patterns (non-negative floats order like their bits, so atomicMax applies):
    // cert[0] = max |x|, cert[1 + kind] = max |operand - exact operand-space row| of operand kind
    // `kind` (VA_CERT_*). Maxima only grow (a compaction keeps them: still valid upper bounds).
    uint32_t* cert = nullptr;
    unsigned cert_ready = 0;     // bit kind set once cert[1 + kind] covers every row
    // Learned per metric: candidate pool of later tensor-core searches, as a multiple of k, once a
    // batch showed neighbourhoods too dense for the first pool to certify (0: no hint).
    int pool_hint[3] = {0, 0, 0};
    // Row-sharded database (va_group.cu): a multi-device context's database holds one shard per
    // device in `shards` (this object then holds no rows); a rank context's database is its own
    // shard with `group_shard` set. n_total = rows of the whole database.
    va_database** shards = nullptr;
    int nshards = 0;
    bool group_shard = false;
    int64_t n_total = 0;
};

// True when a search over db runs per shard and merges across the group.
inline bool va_is_sharded(const va_database* db) { return db->shards != nullptr || db->group_shard; }
int va_sharded_knn(va_context* ctx, const va_database* db, const float* queries, int64_t nq, int k, int metric,
                   int precision, int rerank, float* out_vals, uint32_t* out_ids);
int va_sharded_int8(va_context* ctx, const va_database* db, const float* queries, int64_t nq, int k, int candidates,
                    float* out_vals, uint32_t* out_ids);
int va_sharded_hamming(va_context* ctx, const va_database* db, const uint32_t* queries, int64_t nq, int k,
                       uint32_t* out_dists, uint32_t* out_ids);
// Plain (one-device) searches, called per shard by the sharded ones.
int va_knn_search_local(va_context* ctx, const va_database* db, const float* queries, int64_t nq, int k, int metric,
                        int precision, int rerank, float* out_vals, uint32_t* out_ids);
int va_int8_knn_local(va_context* ctx, const va_database* db, const float* queries, int64_t nq, int k, int candidates,
                      float* out_vals, uint32_t* out_ids);
int va_hamming_knn_local(va_context* ctx, const va_database* db, const uint32_t* queries, int64_t nq, int k,
                         uint32_t* out_dists, uint32_t* out_ids);

// Operand kinds of the certificate (which reduced-precision copy of a row the filter reads).
#define VA_CERT_BF16 0     // bf16(x)
#define VA_CERT_BF16_COS 1 // bf16(x / |x|)
#define VA_CERT_TF32 2     // x read as tf32 by the tensor core
#define VA_CERT_TF32_COS 3 // (x / |x|) read as tf32
#define VA_CERT_WORDS 8

#define VA_DB_FLOAT 0
#define VA_DB_INT8 1
#define VA_DB_BINARY 2

// ------------------------------------------------------------------------------------------------
// Device helpers
// ------------------------------------------------------------------------------------------------
namespace va {

constexpr uint32_t kInvalidId = 0xFFFFFFFFu;

// Monotone map float -> uint32 (ascending floats give ascending keys); NaN maps to the worst key.
__device__ __forceinline__ uint32_t f2key(float v) {
    uint32_t u = __float_as_uint(v);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0xFFFFFFFFu;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
    uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
    return __uint_as_float(u);
}
// Key in selection order for a value under mode (0 = min, 1 = max).
__device__ __forceinline__ uint32_t mode_key(float v, int mode) {
    uint32_t k = f2key(v);
    if (k == 0xFFFFFFFFu) return k;  // NaN is worst in both modes
    return mode ? ~k : k;
}
__device__ __forceinline__ float mode_val(uint32_t k, int mode) { return mode ? key2f(~k) : key2f(k); }

__device__ __forceinline__ uint64_t composite(uint32_t key, uint32_t id) {
    return ((uint64_t)key << 32) | (uint64_t)id;
}

// In-place ascending bitonic sort of n (power of two) uint64 values in shared memory.
__device__ __forceinline__ void block_bitonic_sort(uint64_t* s, int n) {
    for (int size = 2; size <= n; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            __syncthreads();
            for (int i = threadIdx.x; i < (n >> 1); i += blockDim.x) {
                int lo = 2 * i - (i & (stride - 1));
                int hi = lo + stride;
                bool up = ((lo & size) == 0);
                uint64_t a = s[lo], b = s[hi];
                if ((a > b) == up) {
                    s[lo] = b;
                    s[hi] = a;
                }
            }
        }
    }
    __syncthreads();
}

__host__ __device__ __forceinline__ int next_pow2(int v) {
    int p = 1;
    while (p < v) p <<= 1;
    return p;
}

// Shared state of block_select_radix.
struct SelectShared {
    unsigned hist[256];
    unsigned long long prefix, mask;
    int need;
    int done;
    int count;
    int count_eq;
};

// Block-wide exact selection of the `want` smallest 64-bit composite keys among n candidates
// given by get(i), i < n; the selection has exactly min(want, n) elements, written unsorted to
// out[0 .. min(want,n)). Radix passes of 8 bits from the top; a pass stops early once every
// element with the current prefix is needed. Composites are unique (the low 32 bits carry the
// id) except the padding value ~0, which may repeat: the elements below the final prefix are all
// taken and the ones equal to it only fill the remaining slots.
template <class Get>
__device__ int block_select_radix(int64_t n, int want, Get get, uint64_t* out, SelectShared& sh) {
    if (n <= want) {
        if (threadIdx.x == 0) sh.count = 0;
        __syncthreads();
        for (int64_t i = threadIdx.x; i < n; i += blockDim.x) out[i] = get(i);
        __syncthreads();
        return (int)n;
    }
    if (threadIdx.x == 0) {
        sh.prefix = 0;
        sh.mask = 0;
        sh.need = want;
        sh.done = 0;
        sh.count = 0;
        sh.count_eq = 0;
    }
    __syncthreads();
    for (int shift = 56; shift >= 0; shift -= 8) {
        for (int b = threadIdx.x; b < 256; b += blockDim.x) sh.hist[b] = 0;
        __syncthreads();
        const unsigned long long prefix = sh.prefix, mask = sh.mask;
        for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
            uint64_t c = get(i);
            if ((c & mask) == prefix) atomicAdd(&sh.hist[(c >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (threadIdx.x < 32) {
            // Warp 0 finds the digit where the running count reaches `need`.
            const int lane = threadIdx.x;
            unsigned local[8];
            unsigned tot = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                local[j] = sh.hist[lane * 8 + j];
                tot += local[j];
            }
            unsigned incl = tot;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                unsigned t = __shfl_up_sync(0xFFFFFFFFu, incl, o);
                if (lane >= o) incl += t;
            }
            unsigned excl = incl - tot;
            const unsigned need = (unsigned)sh.need;
            if (excl < need && need <= incl) {
                unsigned run = excl;
                int digit = 0;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    if (run + local[j] >= need) {
                        digit = j;
                        break;
                    }
                    run += local[j];
                }
                int d = lane * 8 + digit;
                unsigned cnt = sh.hist[d];
                sh.prefix = prefix | ((unsigned long long)d << shift);
                sh.mask = mask | (0xFFull << shift);
                sh.need = (int)(need - run);
                sh.done = (cnt == need - run) ? 1 : 0;
            }
        }
        __syncthreads();
        if (sh.done) break;
    }
    const unsigned long long prefix = sh.prefix, mask = sh.mask;
    // want - need elements lie below the prefix (front slots); `need` of those equal to it fill
    // the back slots.
    const int need = sh.need;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
        uint64_t c = get(i);
        const unsigned long long m = c & mask;
        if (m < prefix) {
            int slot = atomicAdd(&sh.count, 1);
            if (slot < want) out[slot] = c;
        } else if (m == prefix) {
            int slot = atomicAdd(&sh.count_eq, 1);
            if (slot < need) out[want - 1 - slot] = c;
        }
    }
    __syncthreads();
    return want;
}

// bf16 round to nearest even (NaN kept quiet), as the tensor-core operands are built.
__device__ __forceinline__ uint16_t f2bf_rn(float f) {
    uint32_t u = __float_as_uint(f);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x40);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
__device__ __forceinline__ float bf2f(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

// Bound of |tf32(v) - v| whatever the tensor core's fp32 -> tf32 conversion does (truncation or
// rounding of the low 13 mantissa bits, flushing of subnormals): one tf32 unit in the last place,
// or |v| itself below the normal range.
__device__ __forceinline__ double tf32_err_bound(float v) {
    const uint32_t u = __float_as_uint(v) & 0x7FFFFFFFu;
    if (u < 0x00800000u) return (double)__uint_as_float(u);
    if ((u & 0x1FFFu) == 0) return 0.0;  // exactly representable (bf16 values among them)
    return ldexp(1.0, (int)(u >> 23) - 127 - 10);
}

// One element of a certificate operand: t = the exact operand-space value (v, or v * scale for
// the unit-norm cosine operands, scale = 1/|x| in fp64) and a bound of |operand - t|, where the
// operand is what the filter's tensor core multiplies (bf16 built by f2bf_rn from the fp32 value,
// or the fp32 value read as tf32).
__device__ __forceinline__ void cert_elem(float v, double scale, int kind, double& t, double& err) {
    const bool cos = kind == VA_CERT_BF16_COS || kind == VA_CERT_TF32_COS;
    t = cos ? (double)v * scale : (double)v;
    const float vf = cos ? (float)t : v;  // the fp32 value the operand is made from
    if (kind == VA_CERT_BF16 || kind == VA_CERT_BF16_COS)
        err = fabs((double)bf2f(f2bf_rn(vf)) - t);
    else
        err = fabs((double)vf - t) + tf32_err_bound(vf);
}

// Bounded mbarrier / flag waits: the limit is measured on the global nanosecond timer.
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

}  // namespace va
