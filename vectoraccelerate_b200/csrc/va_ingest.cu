// va_ingest.cu -- growing, updating and compacting resident databases on the device.
//
// Replaces the storage side of the reference index: GPUVectorStorage's write / ensureCapacity /
// compact (Index/Internal/GPUVectorStorage.swift:75-260), with the derived data (row norms,
// tensor-core operands, int8 codes, 0/1 bit expansions) written at insert time as
// IVFQuantizedStorage does for its codes (Index/Internal/IVFQuantizedStorage.swift:158-260).
// Capacity grows geometrically (at least doubling, in multiples of 256 rows), so appends are
// amortized O(rows written); a compaction gathers the kept rows of every per-row array in order.
#include <algorithm>
#include <vector>

#include "va_internal.cuh"

int va_db_derive_rows(va_context* ctx, va_database* db, int64_t r0, int64_t count);
int va_db_derive_codes(va_context* ctx, va_database* db, int64_t r0, int64_t count);

namespace {

int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

// One per-row array of a database: its pointer slot, bytes per row, and whether the filter reads
// it padded to a multiple of 256 rows.
struct RowArray {
    void** ptr;
    size_t row_bytes;
    bool pad256;
};

size_t row_bytes_of_rows(const va_database* db) {
    if (db->kind == VA_DB_BINARY) return (size_t)db->words * 4;
    return (size_t)db->dim * (db->dtype == VA_DTYPE_BF16 ? 2 : 4);
}

int list_arrays(va_database* db, RowArray* a) {
    int n = 0;
    a[n++] = {&db->rows, row_bytes_of_rows(db), false};
    if (db->op && !db->op_alias) a[n++] = {(void**)&db->op, (size_t)db->dpad * 2, false};
    if (db->op_cos) a[n++] = {(void**)&db->op_cos, (size_t)db->dpad * 2, false};
    if (db->op_f32 && !db->op_f32_alias) a[n++] = {(void**)&db->op_f32, (size_t)db->dpad * 4, false};
    if (db->op_f32_cos) a[n++] = {(void**)&db->op_f32_cos, (size_t)db->dpad * 4, false};
    if (db->norms2) a[n++] = {(void**)&db->norms2, 4, true};
    if (db->zbias) a[n++] = {(void**)&db->zbias, 4, true};
    if (db->codes) a[n++] = {(void**)&db->codes, (size_t)db->cpad, false};
    if (db->code_norms) a[n++] = {(void**)&db->code_norms, 4, true};
    return n;
}

size_t array_bytes(const RowArray& a, int64_t rows) {
    return (size_t)(a.pad256 ? round_up(rows, 256) : rows) * a.row_bytes;
}

void repoint_aliases(va_database* db) {
    if (db->op_alias) db->op = (uint16_t*)db->rows;
    if (db->op_f32_alias) db->op_f32 = (float*)db->rows;
}

int64_t capacity(const va_database* db) { return db->cap ? db->cap : db->n; }

// Make room for `need` rows in every per-row array (existing rows copied, old arrays freed).
int grow(va_context* ctx, va_database* db, int64_t need) {
    if (need <= capacity(db)) return VA_OK;
    const int64_t cap = round_up(std::max<int64_t>(need, 2 * capacity(db)), 256);
    RowArray arr[16];
    const int na = list_arrays(db, arr);
    std::vector<void*> fresh((size_t)na, nullptr);
    for (int i = 0; i < na; ++i) {
        cudaError_t e = cudaMalloc(&fresh[(size_t)i], array_bytes(arr[i], cap));
        if (e != cudaSuccess) {
            cudaGetLastError();
            for (int j = 0; j < i; ++j) cudaFree(fresh[(size_t)j]);
            return va_set_error(VA_ERR_OOM, "growing the database to %lld rows failed: %s", (long long)cap,
                                cudaGetErrorString(e));
        }
        VA_CUDA_TRY(cudaMemcpyAsync(fresh[(size_t)i], *arr[i].ptr, (size_t)db->n * arr[i].row_bytes,
                                    cudaMemcpyDeviceToDevice, ctx->stream));
    }
    VA_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    for (int i = 0; i < na; ++i) {
        cudaFree(*arr[i].ptr);
        *arr[i].ptr = fresh[(size_t)i];
    }
    repoint_aliases(db);
    db->cap = cap;
    return VA_OK;
}

// Rows [r0, r0 + count) were written: recompute what is derived from them.
int derive(va_context* ctx, va_database* db, int64_t r0, int64_t count) {
    if (db->kind != VA_DB_BINARY) VA_TRY(va_db_derive_rows(ctx, db, r0, count));
    if (db->kind != VA_DB_FLOAT) VA_TRY(va_db_derive_codes(ctx, db, r0, count));
    return VA_OK;
}

template <class T>
__global__ void k_gather_rows(const T* __restrict__ src, T* __restrict__ dst, const int64_t* __restrict__ idx,
                              int64_t m, int64_t words) {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < m * words;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = e / words;
        dst[e] = src[idx[r] * words + (e - r * words)];
    }
}

__global__ void k_fill_f32(float* p, int64_t n, float v) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        p[i] = v;
}

int gather(va_context* ctx, const void* src, void* dst, const int64_t* idx, int64_t m, size_t row_bytes) {
    if (m <= 0) return VA_OK;
    const int blocks = (int)std::min<int64_t>((m * (int64_t)row_bytes / 4 + 255) / 256 + 1, (int64_t)ctx->sm_count * 16);
    if (row_bytes % 16 == 0)
        k_gather_rows<uint4><<<blocks, 256, 0, ctx->stream>>>((const uint4*)src, (uint4*)dst, idx, m, row_bytes / 16);
    else if (row_bytes % 4 == 0)
        k_gather_rows<uint32_t><<<blocks, 256, 0, ctx->stream>>>((const uint32_t*)src, (uint32_t*)dst, idx, m,
                                                                 row_bytes / 4);
    else if (row_bytes % 2 == 0)
        k_gather_rows<uint16_t><<<blocks, 256, 0, ctx->stream>>>((const uint16_t*)src, (uint16_t*)dst, idx, m,
                                                                 row_bytes / 2);
    else
        k_gather_rows<uint8_t><<<blocks, 256, 0, ctx->stream>>>((const uint8_t*)src, (uint8_t*)dst, idx, m, row_bytes);
    return va_check_launch("k_gather_rows");
}

}  // namespace

extern "C" {

int va_db_append(va_context* ctx, va_database* db, const void* rows, int on_device, int64_t count) {
    VA_REQUIRE(ctx && db && rows, "ctx, db and rows must not be NULL");
    VA_REQUIRE(!va_is_sharded(db), "a sharded database is not grown, updated or compacted in place (rebuild it)");
    VA_REQUIRE(count >= 0, "count must be >= 0, got %lld", (long long)count);
    VA_REQUIRE(db->ctx->device == ctx->device, "database lives on device %d, context on device %d", db->ctx->device,
               ctx->device);
    VA_REQUIRE((uint64_t)db->n + (uint64_t)count + db->id_base <= 0xFFFFFFFFull,
               "numDataset %lld + %lld + id_base exceeds the uint32 id range", (long long)db->n, (long long)count);
    if (!count) return VA_OK;
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    const int64_t r0 = db->n;
    VA_TRY(grow(ctx, db, r0 + count));
    const size_t rb = row_bytes_of_rows(db);
    VA_CUDA_TRY(cudaMemcpyAsync((uint8_t*)db->rows + (size_t)r0 * rb, rows, (size_t)count * rb,
                                on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, ctx->stream));
    db->n = r0 + count;
    return derive(ctx, db, r0, count);
}

int va_db_update(va_context* ctx, va_database* db, int64_t slot0, const void* rows, int on_device, int64_t count) {
    VA_REQUIRE(ctx && db && rows, "ctx, db and rows must not be NULL");
    VA_REQUIRE(!va_is_sharded(db), "a sharded database is not grown, updated or compacted in place (rebuild it)");
    VA_REQUIRE(slot0 >= 0 && count >= 0 && slot0 + count <= db->n,
               "slots [%lld, %lld) outside the database's %lld rows", (long long)slot0, (long long)(slot0 + count),
               (long long)db->n);
    if (!count) return VA_OK;
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    const size_t rb = row_bytes_of_rows(db);
    VA_CUDA_TRY(cudaMemcpyAsync((uint8_t*)db->rows + (size_t)slot0 * rb, rows, (size_t)count * rb,
                                on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, ctx->stream));
    return derive(ctx, db, slot0, count);
}

int va_db_compact(va_context* ctx, va_database* db, const uint8_t* keep, int64_t* new_slot) {
    VA_REQUIRE(ctx && db && keep, "ctx, db and keep must not be NULL");
    VA_REQUIRE(!va_is_sharded(db), "a sharded database is not grown, updated or compacted in place (rebuild it)");
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    const int64_t n = db->n;
    std::vector<int64_t> kept;
    kept.reserve((size_t)n);
    for (int64_t i = 0; i < n; ++i) {
        if (new_slot) new_slot[i] = keep[i] ? (int64_t)kept.size() : -1;
        if (keep[i]) kept.push_back(i);
    }
    const int64_t m = (int64_t)kept.size();
    if (m == n) return VA_OK;
    VA_REQUIRE(m > 0, "compaction would leave the database empty (create a new one instead)");
    const int64_t cap = capacity(db);
    void* didx = nullptr;
    VA_CUDA_TRY(cudaMalloc(&didx, (size_t)m * sizeof(int64_t)));
    int s = VA_OK;
    cudaError_t e = cudaMemcpyAsync(didx, kept.data(), (size_t)m * sizeof(int64_t), cudaMemcpyHostToDevice, ctx->stream);
    if (e != cudaSuccess) s = va_set_error(VA_ERR_CUDA, "index upload failed: %s", cudaGetErrorString(e));
    RowArray arr[16];
    const int na = list_arrays(db, arr);
    std::vector<void*> fresh((size_t)na, nullptr);
    for (int i = 0; i < na && s == VA_OK; ++i) {
        e = cudaMalloc(&fresh[(size_t)i], array_bytes(arr[i], cap));
        if (e != cudaSuccess) {
            cudaGetLastError();
            s = va_set_error(VA_ERR_OOM, "compaction buffers failed: %s", cudaGetErrorString(e));
            break;
        }
        s = gather(ctx, *arr[i].ptr, fresh[(size_t)i], (const int64_t*)didx, m, arr[i].row_bytes);
    }
    if (s == VA_OK) s = cudaStreamSynchronize(ctx->stream) == cudaSuccess ? VA_OK : va_set_error(VA_ERR_CUDA, "sync failed");
    if (s != VA_OK) {
        for (void* p : fresh)
            if (p) cudaFree(p);
        cudaFree(didx);
        return s;
    }
    for (int i = 0; i < na; ++i) {
        cudaFree(*arr[i].ptr);
        *arr[i].ptr = fresh[(size_t)i];
    }
    cudaFree(didx);
    repoint_aliases(db);
    db->n = m;
    db->cap = cap;
    // The filter reads row biases up to a multiple of 256 rows: the rows past the end are +inf.
    const int64_t pad = round_up(m, 256) - m;
    if (pad > 0 && db->norms2) {
        k_fill_f32<<<1, 256, 0, ctx->stream>>>(db->norms2 + m, pad, INFINITY);
        k_fill_f32<<<1, 256, 0, ctx->stream>>>(db->zbias + m, pad, INFINITY);
        VA_TRY(va_check_launch("k_fill_f32"));
    }
    return VA_OK;
}

}  // extern "C"
