// va_select.cu -- top-k selection and merges on the device.
//
// Replaces TopKSelectionKernel / WarpOptimizedSelectionKernel (Kernels/Metal4/
// TopKSelectionKernel.swift:228-411, WarpOptimizedSelectionKernel.swift:250-863, shaders
// SearchAndRetrieval.metal:88-156 and AdvancedTopK.metal:518-817) and TopKMergeKernel
// (TopKMergeKernel.swift:18-127, SearchAndRetrieval.metal:320-385).
//
// One block per row. Candidates become unique 64-bit composites (orderable key << 32 | id), an
// exact block-wide radix select keeps the k smallest, and a shared-memory bitonic sort orders
// them. The (key, id) composite is the reference's tie rule (AdvancedTopK.metal:48-52): equal
// values keep the smaller index. The reference's per-thread heap (K <= 128) is replaced by a
// selection whose cost is a few streaming passes over the row, independent of k.
#include <algorithm>

#include "va_internal.cuh"

namespace {

constexpr int kSelThreads = 512;

// Row-wise top-k of a dense value matrix.
__global__ void __launch_bounds__(kSelThreads) k_topk_rows(const float* __restrict__ in, int64_t n, int64_t in_stride,
                                                           int k, int mode, float* __restrict__ out_vals,
                                                           uint32_t* __restrict__ out_ids, int64_t out_stride) {
    extern __shared__ uint64_t s_sel[];
    __shared__ va::SelectShared sh;
    const float* row = in + (int64_t)blockIdx.x * in_stride;
    auto get = [&](int64_t i) -> uint64_t { return va::composite(va::mode_key(__ldg(row + i), mode), (uint32_t)i); };
    int m = va::block_select_radix(n, k, get, s_sel, sh);
    int p2 = va::next_pow2(m > 0 ? m : 1);
    for (int i = m + threadIdx.x; i < p2; i += blockDim.x) s_sel[i] = ~0ull;
    va::block_bitonic_sort(s_sel, p2);
    const float pad = mode ? -INFINITY : INFINITY;
    for (int i = threadIdx.x; i < k; i += blockDim.x) {
        float v = pad;
        uint32_t id = va::kInvalidId;
        if (i < m) {
            uint64_t c = s_sel[i];
            id = (uint32_t)c;
            v = __ldg(row + id);
        }
        if (out_vals) out_vals[(int64_t)blockIdx.x * out_stride + i] = v;
        if (out_ids) out_ids[(int64_t)blockIdx.x * out_stride + i] = id;
    }
}

// Generic merge: row r has `lists` sorted lists of length `len` each, element (l, i) at
// vals[(l*lstride) + r*len + i] (lstride = rows*len for the sharded layout); ids may carry an
// added base per list. Invalid ids are ignored.
struct ListSource {
    const float* vals;
    const uint32_t* ids;
    int64_t list_stride;  // elements between consecutive lists
    int len;
    uint32_t base;        // added to ids of this source
};

__global__ void __launch_bounds__(kSelThreads) k_merge(ListSource a, int a_lists, ListSource b, int b_lists, int k,
                                                       int mode, float* __restrict__ out_vals,
                                                       uint32_t* __restrict__ out_ids) {
    extern __shared__ uint64_t s_sel[];
    __shared__ va::SelectShared sh;
    // Candidates are indexed 0 .. a_lists*a.len + b_lists*b.len; the composite carries the
    // original value's key and the (based) id; values are re-read through a side table so the
    // output can alias the inputs: copy values to shared first.
    const int64_t r = blockIdx.x;
    const int64_t na = (int64_t)a_lists * a.len, nb = (int64_t)b_lists * b.len;
    auto get = [&](int64_t i) -> uint64_t {
        uint32_t id;
        float v;
        if (i < na) {
            int l = (int)(i / a.len), j = (int)(i % a.len);
            int64_t off = l * a.list_stride + r * a.len + j;
            id = a.ids[off];
            v = a.vals[off];
            if (id != va::kInvalidId) id += a.base;
        } else {
            int64_t t = i - na;
            int l = (int)(t / b.len), j = (int)(t % b.len);
            int64_t off = l * b.list_stride + r * b.len + j;
            id = b.ids[off];
            v = b.vals[off];
            if (id != va::kInvalidId) id += b.base;
        }
        if (id == va::kInvalidId) return ~0ull;  // sorts last, never reported
        return va::composite(va::mode_key(v, mode), id);
    };
    int m = va::block_select_radix(na + nb, k, get, s_sel, sh);
    int p2 = va::next_pow2(m > 0 ? m : 1);
    for (int i = m + threadIdx.x; i < p2; i += blockDim.x) s_sel[i] = ~0ull;
    va::block_bitonic_sort(s_sel, p2);
    __syncthreads();
    const float pad = mode ? -INFINITY : INFINITY;
    for (int i = threadIdx.x; i < k; i += blockDim.x) {
        uint64_t c = i < m ? s_sel[i] : ~0ull;
        float v = pad;
        uint32_t id = va::kInvalidId;
        if (c != ~0ull) {
            id = (uint32_t)c;
            v = va::mode_val((uint32_t)(c >> 32), mode);
        }
        out_vals[r * k + i] = v;
        out_ids[r * k + i] = id;
    }
}

}  // namespace

extern "C" {

int va_topk_select(va_context* ctx, const float* in, int64_t batch, int64_t n, int64_t in_stride, int k, int mode,
                   float* out_vals, uint32_t* out_ids, int64_t out_stride) {
    VaRange nvtx_range("va_topk_select");
    VA_REQUIRE(ctx && in, "ctx and in must not be NULL");
    VA_REQUIRE(out_vals || out_ids, "at least one of out_vals / out_ids is required");
    VA_REQUIRE(k > 0 && k <= VA_MAX_SELECT_K, "k must be between 1 and %d, got %d", VA_MAX_SELECT_K, k);
    VA_REQUIRE(mode == VA_SELECT_MIN || mode == VA_SELECT_MAX, "mode must be 0 (minimum) or 1 (maximum), got %d", mode);
    VA_REQUIRE(batch >= 0 && n >= 0, "batch and n must be >= 0");
    VA_REQUIRE(n <= 0xFFFFFFFFll, "n %lld exceeds the uint32 id range", (long long)n);
    VA_REQUIRE(in_stride >= n, "in_stride %lld must be >= n %lld", (long long)in_stride, (long long)n);
    VA_REQUIRE(out_stride >= k, "out_stride %lld must be >= k %d", (long long)out_stride, k);
    if (!batch) return VA_OK;
    VA_REQUIRE(batch <= 0x7FFFFFFF, "batch %lld too large", (long long)batch);
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    size_t smem = (size_t)va::next_pow2(k) * sizeof(uint64_t);
    if (smem > 48 * 1024) VA_CUDA_TRY(cudaFuncSetAttribute(k_topk_rows, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    k_topk_rows<<<(unsigned)batch, kSelThreads, smem, ctx->stream>>>(in, n, in_stride, k, mode, out_vals, out_ids,
                                                                      out_stride);
    return va_check_launch("k_topk_rows");
}

int va_topk_merge(va_context* ctx, const float* run_vals, const uint32_t* run_ids, int k, const float* chunk_vals,
                  const uint32_t* chunk_ids, int kc, uint32_t chunk_base, int64_t nq, int mode, float* out_vals,
                  uint32_t* out_ids) {
    VA_REQUIRE(ctx && run_vals && run_ids && chunk_vals && chunk_ids && out_vals && out_ids,
               "all buffers must be non-NULL");
    VA_REQUIRE(k > 0 && k <= VA_MAX_SELECT_K, "k must be between 1 and %d, got %d", VA_MAX_SELECT_K, k);
    VA_REQUIRE(kc > 0 && kc <= VA_MAX_SELECT_K, "kc must be between 1 and %d, got %d", VA_MAX_SELECT_K, kc);
    VA_REQUIRE(mode == VA_SELECT_MIN || mode == VA_SELECT_MAX, "mode must be 0 or 1, got %d", mode);
    if (nq <= 0) return VA_OK;
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    ListSource a{run_vals, run_ids, 0, k, 0u};
    ListSource b{chunk_vals, chunk_ids, 0, kc, chunk_base};
    size_t smem = (size_t)va::next_pow2(k) * sizeof(uint64_t);
    if (smem > 48 * 1024) VA_CUDA_TRY(cudaFuncSetAttribute(k_merge, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    // Outputs may alias the running lists: a row's outputs are written only after its block has
    // read every input of that row (the selection and sort complete before the writes).
    k_merge<<<(unsigned)nq, kSelThreads, smem, ctx->stream>>>(a, 1, b, 1, k, mode, out_vals, out_ids);
    return va_check_launch("k_merge");
}

// Internal: merge `nlists` lists of `len` sorted entries per row (list l of row r at
// vals[l*list_stride + r*len]) into the best k per row.
int va_merge_lists_internal(va_context* ctx, const float* vals, const uint32_t* ids, int nlists, int64_t list_stride,
                            int len, int64_t nq, int k, int mode, float* out_vals, uint32_t* out_ids) {
    if (nq <= 0) return VA_OK;
    VA_REQUIRE(k > 0 && k <= VA_MAX_SELECT_K, "k must be between 1 and %d, got %d", VA_MAX_SELECT_K, k);
    ListSource a{vals, ids, list_stride, len, 0u};
    ListSource b{vals, ids, 0, 1, 0u};
    size_t smem = (size_t)va::next_pow2(k) * sizeof(uint64_t);
    if (smem > 48 * 1024) VA_CUDA_TRY(cudaFuncSetAttribute(k_merge, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    k_merge<<<(unsigned)nq, kSelThreads, smem, ctx->stream>>>(a, nlists, b, 0, k, mode, out_vals, out_ids);
    return va_check_launch("k_merge(lists)");
}

int va_merge_shards(va_context* ctx, const float* vals, const uint32_t* ids, int nshards, int64_t nq, int k, int mode,
                    float* out_vals, uint32_t* out_ids) {
    VaRange nvtx_range("va_merge_shards");
    VA_REQUIRE(ctx && vals && ids && out_vals && out_ids, "all buffers must be non-NULL");
    VA_REQUIRE(nshards > 0, "nshards must be positive, got %d", nshards);
    VA_REQUIRE(k > 0 && k <= VA_MAX_SELECT_K, "k must be between 1 and %d, got %d", VA_MAX_SELECT_K, k);
    VA_REQUIRE(mode == VA_SELECT_MIN || mode == VA_SELECT_MAX, "mode must be 0 or 1, got %d", mode);
    if (nq <= 0) return VA_OK;
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    ListSource a{vals, ids, nq * (int64_t)k, k, 0u};
    ListSource b{vals, ids, 0, 1, 0u};
    size_t smem = (size_t)va::next_pow2(k) * sizeof(uint64_t);
    if (smem > 48 * 1024) VA_CUDA_TRY(cudaFuncSetAttribute(k_merge, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    k_merge<<<(unsigned)nq, kSelThreads, smem, ctx->stream>>>(a, nshards, b, 0, k, mode, out_vals, out_ids);
    return va_check_launch("k_merge(shards)");
}

}  // extern "C"
