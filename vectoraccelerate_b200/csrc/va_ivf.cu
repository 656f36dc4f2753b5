// va_ivf.cu -- inverted-file (IVF) search on the same kernels as the flat path.
//
// Replaces the reference's IVF pipeline (Index/Kernels/IVF/IVFSearchPipeline.swift:197-600:
// coarse quantization to the nprobe nearest centroids, then a search of the probed lists) and its
// k-means training (Index/Kernels/Clustering/KMeansPipeline.swift; assign / update / convergence
// kernels). Differences of layout, on purpose:
//   * the lists are materialised as one row-major copy of the database in list order (offsets per
//     list), so each probed list is one contiguous range streamed once per (query, probe);
//   * the coarse quantizer is the fused exact k-NN of the queries against the centroids
//     (tensor-core filter + exact rerank), and k-means assignment is the same search with k = 1;
//   * k-means starts from `nlist` distinct rows drawn with a seeded generator (the reference seeds
//     with k-means++) and runs Lloyd iterations until the largest centroid movement is below
//     `tol` (KMeansConvergenceKernel.swift:78-110), as the reference does.
// The list scan computes exact squared L2 (fp32 rows, fp64 accumulation) and keeps, per (query,
// probe), the k best (distance, id) composites; the probes' lists are merged by (distance, id).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "va_internal.cuh"

extern "C" int va_merge_lists_internal(va_context* ctx, const float* vals, const uint32_t* ids, int nlists,
                                       int64_t list_stride, int len, int64_t nq, int k, int mode, float* out_vals,
                                       uint32_t* out_ids);

struct va_ivf {
    va_context* ctx = nullptr;
    int nlist = 0;
    int dim = 0;
    int64_t n = 0;
    float* centroids = nullptr;    // [nlist x dim]
    va_database* cdb = nullptr;    // centroids as a database (coarse quantizer)
    float* rows = nullptr;         // [n x dim] rows in list order
    uint32_t* ids = nullptr;       // [n] original id of each row in list order
    int64_t* offsets = nullptr;    // [nlist + 1] device
    std::vector<int64_t> h_offsets;
};

namespace {

int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }
int grid_for(int64_t n) { return (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 16384)); }

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

// ---------------------------------------------------------------------------------- k-means
__global__ void k_gather_rows_f32(const float* __restrict__ src, int dim, const int64_t* __restrict__ rows, int64_t n,
                                  float* __restrict__ dst) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n * dim; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / dim;
        dst[i] = src[rows[r] * dim + (i - r * dim)];
    }
}

// sums[c] += row, counts[c] += 1 for every row's list c (fp64 sums: the mean does not depend on
// the order of the atomics beyond fp64 rounding).
__global__ void k_accumulate(const float* __restrict__ x, int64_t n, int dim, const uint32_t* __restrict__ assign,
                             double* __restrict__ sums, unsigned long long* __restrict__ counts) {
    const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (r >= n) return;
    const uint32_t c = assign[r];
    for (int j = lane; j < dim; j += 32) atomicAdd(sums + (int64_t)c * dim + j, (double)x[r * dim + j]);
    if (lane == 0) atomicAdd(counts + c, 1ull);
}

// New centroid = mean of its rows; a list without rows keeps its centroid.
__global__ void k_centroid_update(const double* __restrict__ sums, const unsigned long long* __restrict__ counts,
                                  int nlist, int dim, float* __restrict__ centroids) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (int64_t)nlist * dim;
         i += (int64_t)gridDim.x * blockDim.x) {
        const unsigned long long cnt = counts[i / dim];
        if (cnt) centroids[i] = (float)(sums[i] / (double)cnt);
    }
}

// move_bits = max over centroids of the squared Euclidean movement (float bits; non-negative
// floats order as unsigned integers).
__global__ void k_max_movement(const float* __restrict__ a, const float* __restrict__ b, int nlist, int dim,
                               unsigned* __restrict__ move_bits) {
    const int c = (int)(((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (c >= nlist) return;
    double s = 0;
    for (int j = lane; j < dim; j += 32) {
        const double t = (double)a[(int64_t)c * dim + j] - (double)b[(int64_t)c * dim + j];
        s += t * t;
    }
    s = warp_sum_d(s);
    if (lane == 0) atomicMax(move_bits, __float_as_uint((float)s));
}

// ---------------------------------------------------------------------------------- lists
__global__ void k_histogram(const uint32_t* __restrict__ assign, int64_t n, unsigned long long* __restrict__ counts) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        atomicAdd(counts + assign[i], 1ull);
}

// Stable positions in list order: one block per list walks the assignments in row order, so the
// rows of a list keep their relative order (ties in the scan then resolve by the original id as
// in a flat search). pos[r] = the row's index in list order; ids_out[pos] = r + id_base.
__global__ void k_list_positions(int64_t n, const uint32_t* __restrict__ assign, const int64_t* __restrict__ offsets,
                                 int64_t* __restrict__ pos, uint32_t* __restrict__ ids_out, uint32_t id_base) {
    const uint32_t c = blockIdx.x;
    __shared__ int64_t s_pos;
    __shared__ int s_warp[32];
    __shared__ int s_cnt;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) s_pos = offsets[c];
    __syncthreads();
    for (int64_t base = 0; base < n; base += blockDim.x) {
        const int64_t r = base + threadIdx.x;
        const bool mine = r < n && assign[r] == c;
        const unsigned bal = __ballot_sync(0xFFFFFFFFu, mine);
        if (lane == 0) s_warp[warp] = __popc(bal);
        __syncthreads();
        if (threadIdx.x == 0) {
            int acc = 0;
            for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
                const int t = s_warp[w];
                s_warp[w] = acc;
                acc += t;
            }
            s_cnt = acc;
        }
        __syncthreads();
        if (mine) {
            const int64_t at = s_pos + s_warp[warp] + __popc(bal & ((1u << lane) - 1u));
            pos[r] = at;
            ids_out[at] = (uint32_t)r + id_base;
        }
        __syncthreads();
        if (threadIdx.x == 0) s_pos += s_cnt;
        __syncthreads();
    }
}

// rows_out[pos[r]] = x[r], one warp per row.
__global__ void k_place_rows(const float* __restrict__ x, int64_t n, int dim, const int64_t* __restrict__ pos,
                             float* __restrict__ rows_out) {
    const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (r >= n) return;
    const int64_t o = pos[r];
    for (int j = lane; j < dim; j += 32) rows_out[o * dim + j] = x[r * dim + j];
}

// ---------------------------------------------------------------------------------- list scan
constexpr int LS_THREADS = 256;
constexpr int LS_BUF = 1024;

// One block per (probe, query): exact squared L2 of the query to every row of its probe-th list
// (a warp per row, fp64 accumulation), the k best (distance, id) composites kept through a
// shared-memory buffer compacted by radix selection; output lists [probe][query][k].
__global__ void __launch_bounds__(LS_THREADS) k_ivf_scan(const float* __restrict__ q, int64_t nq, int dim,
                                                         const uint32_t* __restrict__ probes, int nprobe,
                                                         const float* __restrict__ rows,
                                                         const uint32_t* __restrict__ ids,
                                                         const int64_t* __restrict__ offsets, int k,
                                                         float* __restrict__ out_v, uint32_t* __restrict__ out_i) {
    extern __shared__ float s_q[];                 // [dim]
    __shared__ uint64_t s_buf[LS_BUF];
    __shared__ uint64_t s_tmp[128];
    __shared__ unsigned long long s_thr;
    __shared__ int s_cnt;
    __shared__ va::SelectShared sh;
    const int64_t qi = blockIdx.y;
    const int p = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    for (int j = threadIdx.x; j < dim; j += blockDim.x) s_q[j] = q[qi * dim + j];
    if (threadIdx.x == 0) {
        s_thr = ~0ull;
        s_cnt = 0;
    }
    __syncthreads();
    const uint32_t list = probes[qi * nprobe + p];
    const int64_t r0 = list == va::kInvalidId ? 0 : offsets[list];
    const int64_t r1 = list == va::kInvalidId ? 0 : offsets[list + 1];
    auto compact = [&]() {
        const int c = min(s_cnt, LS_BUF);
        const int m = va::block_select_radix((int64_t)c, k, [&](int64_t i) -> uint64_t { return s_buf[i]; }, s_tmp, sh);
        __syncthreads();
        for (int i = threadIdx.x; i < m; i += blockDim.x) s_buf[i] = s_tmp[i];
        __syncthreads();
        if (threadIdx.x == 0) {
            s_cnt = m;
            if (m == k) {
                unsigned long long t = 0;
                for (int i = 0; i < m; ++i) t = s_buf[i] > t ? s_buf[i] : t;
                s_thr = t;
            }
        }
        __syncthreads();
    };
    for (int64_t base = r0; base < r1; base += nwarps) {
        const int64_t r = base + warp;
        if (r < r1) {
            double s = 0;
            for (int j = lane; j < dim; j += 32) {
                const double t = (double)s_q[j] - (double)rows[r * dim + j];
                s += t * t;
            }
            s = warp_sum_d(s);
            if (lane == 0) {
                const uint64_t comp = va::composite(va::f2key((float)s), ids[r]);
                if (comp < s_thr) {
                    const int slot = atomicAdd(&s_cnt, 1);
                    if (slot < LS_BUF) s_buf[slot] = comp;
                }
            }
        }
        __syncthreads();
        // Every thread reads the count before any warp of the next round adds to it.
        const bool full = s_cnt > LS_BUF - nwarps;
        __syncthreads();
        if (full) compact();
    }
    compact();
    const int m = s_cnt;
    const int64_t o = ((int64_t)p * nq + qi) * k;
    for (int i = threadIdx.x; i < k; i += blockDim.x) {
        const uint64_t c = i < m ? s_buf[i] : ~0ull;
        out_v[o + i] = c == ~0ull ? INFINITY : va::key2f((uint32_t)(c >> 32));
        out_i[o + i] = c == ~0ull ? va::kInvalidId : (uint32_t)c;
    }
}

// Assignment of every row to its nearest centroid (the fused search with k = 1).
int assign_rows(va_context* ctx, va_database* cdb, const float* x, int64_t n, uint32_t* assign, float* scratch_v) {
    return va_knn_search(ctx, cdb, x, n, 1, VA_METRIC_L2SQ, VA_PREC_AUTO, 0, scratch_v, assign);
}

}  // namespace

extern "C" {

int va_ivf_train(va_context* ctx, const float* x, int64_t n, int dim, int nlist, int max_iters, float tol,
                 uint64_t seed, int init_given, float* out_centroids, int* out_iters) {
    VA_REQUIRE(ctx && x && out_centroids, "ctx, x and out_centroids must not be NULL");
    VA_REQUIRE(dim > 0 && dim <= VA_MAX_DIM, "dimension must be in 1..%d, got %d", VA_MAX_DIM, dim);
    VA_REQUIRE(nlist > 0 && nlist <= n, "nlist must be in 1..numVectors (%lld), got %d", (long long)n, nlist);
    VA_REQUIRE(max_iters >= 0, "max_iters must be >= 0");
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    // Initial centroids: nlist distinct rows, a seeded partial Fisher-Yates shuffle on the host.
    std::vector<int64_t> pick((size_t)nlist);
    {
        uint64_t s = seed * 6364136223846793005ull + 1442695040888963407ull;
        std::vector<int64_t> perm;
        const bool dense = n <= (int64_t)nlist * 8;
        if (dense) {
            perm.resize((size_t)n);
            for (int64_t i = 0; i < n; ++i) perm[(size_t)i] = i;
        }
        std::vector<int64_t> chosen;
        for (int i = 0; i < nlist; ++i) {
            s = s * 6364136223846793005ull + 1442695040888963407ull;
            if (dense) {
                const int64_t j = i + (int64_t)((s >> 17) % (uint64_t)(n - i));
                std::swap(perm[(size_t)i], perm[(size_t)j]);
                pick[(size_t)i] = perm[(size_t)i];
            } else {
                int64_t r;
                do {
                    s = s * 6364136223846793005ull + 1442695040888963407ull;
                    r = (int64_t)((s >> 17) % (uint64_t)n);
                } while (std::find(chosen.begin(), chosen.end(), r) != chosen.end());
                chosen.push_back(r);
                pick[(size_t)i] = r;
            }
        }
    }
    const size_t cb = (size_t)nlist * dim;
    void* ws = nullptr;
    const size_t bytes = round_up((int64_t)nlist * 8, 256) + round_up((int64_t)cb * 8, 256) +
                         round_up((int64_t)cb * 4, 256) + round_up((int64_t)nlist * 8, 256) +
                         2 * round_up(n * 4, 256) + 256;
    VA_CUDA_TRY(cudaMalloc(&ws, bytes));
    uint8_t* p = (uint8_t*)ws;
    int64_t* d_pick = (int64_t*)p;
    p += round_up((int64_t)nlist * 8, 256);
    double* sums = (double*)p;
    p += round_up((int64_t)cb * 8, 256);
    float* prev = (float*)p;
    p += round_up((int64_t)cb * 4, 256);
    unsigned long long* counts = (unsigned long long*)p;
    p += round_up((int64_t)nlist * 8, 256);
    uint32_t* assign = (uint32_t*)p;
    p += round_up(n * 4, 256);
    float* vals = (float*)p;
    p += round_up(n * 4, 256);
    unsigned* move_bits = (unsigned*)p;
    int st = VA_OK;
    va_database* cdb = nullptr;
    int it = 0;
    auto fail = [&](int s) {
        if (cdb) va_db_destroy(cdb);
        cudaFree(ws);
        return s;
    };
    if (cudaMemcpyAsync(d_pick, pick.data(), (size_t)nlist * 8, cudaMemcpyHostToDevice, ctx->stream) != cudaSuccess)
        return fail(va_set_error(VA_ERR_CUDA, "upload failed"));
    if (!init_given) {
        k_gather_rows_f32<<<grid_for((int64_t)cb), 256, 0, ctx->stream>>>(x, dim, d_pick, nlist, out_centroids);
        if ((st = va_check_launch("k_gather_rows_f32")) != VA_OK) return fail(st);
    }
    // Lloyd iterations (KMeansPipeline.fit, KMeansPipeline.swift:165-230): assign, update, stop
    // once the largest centroid movement (Euclidean) is below tol.
    while (it < max_iters) {
        if (cdb) va_db_destroy(cdb);
        cdb = nullptr;
        if ((st = va_db_create(ctx, out_centroids, 1, nlist, dim, VA_DTYPE_F32, 0, &cdb)) != VA_OK) return fail(st);
        if ((st = assign_rows(ctx, cdb, x, n, assign, vals)) != VA_OK) return fail(st);
        cudaMemcpyAsync(prev, out_centroids, cb * 4, cudaMemcpyDeviceToDevice, ctx->stream);
        cudaMemsetAsync(sums, 0, cb * 8, ctx->stream);
        cudaMemsetAsync(counts, 0, (size_t)nlist * 8, ctx->stream);
        cudaMemsetAsync(move_bits, 0, 4, ctx->stream);
        k_accumulate<<<(unsigned)((n * 32 + 255) / 256), 256, 0, ctx->stream>>>(x, n, dim, assign, sums, counts);
        k_centroid_update<<<grid_for((int64_t)cb), 256, 0, ctx->stream>>>(sums, counts, nlist, dim, out_centroids);
        k_max_movement<<<(unsigned)(((int64_t)nlist * 32 + 255) / 256), 256, 0, ctx->stream>>>(prev, out_centroids,
                                                                                             nlist, dim, move_bits);
        if ((st = va_check_launch("k_max_movement")) != VA_OK) return fail(st);
        unsigned h = 0;
        cudaMemcpyAsync(&h, move_bits, 4, cudaMemcpyDeviceToHost, ctx->stream);
        if ((st = va_synchronize(ctx)) != VA_OK) return fail(st);
        ++it;
        float mv;
        std::memcpy(&mv, &h, 4);
        if (std::sqrt((double)mv) < (double)tol) break;
    }
    if (out_iters) *out_iters = it;
    st = va_synchronize(ctx);
    return fail(st);
}

int va_ivf_create(va_context* ctx, const float* rows, int64_t n, int dim, const float* centroids, int nlist,
                  uint32_t id_base, va_ivf** out) {
    VA_REQUIRE(ctx && rows && centroids && out, "ctx, rows, centroids and out must not be NULL");
    VA_REQUIRE(n > 0 && dim > 0 && dim <= VA_MAX_DIM && nlist > 0, "n, dim (<= %d) and nlist must be positive",
               VA_MAX_DIM);
    VA_REQUIRE((uint64_t)n + id_base <= 0xFFFFFFFFull, "numVectors + id_base exceeds the uint32 id range");
    *out = nullptr;
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    va_ivf* ivf = new va_ivf();
    ivf->ctx = ctx;
    ivf->nlist = nlist;
    ivf->dim = dim;
    ivf->n = n;
    auto fail = [&](int s) {
        va_ivf_destroy(ivf);
        return s;
    };
    cudaError_t e = cudaMalloc((void**)&ivf->centroids, (size_t)nlist * dim * 4);
    if (e == cudaSuccess) e = cudaMalloc((void**)&ivf->rows, (size_t)n * dim * 4);
    if (e == cudaSuccess) e = cudaMalloc((void**)&ivf->ids, (size_t)n * 4);
    if (e == cudaSuccess) e = cudaMalloc((void**)&ivf->offsets, (size_t)(nlist + 1) * 8);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(va_set_error(VA_ERR_OOM, "IVF allocation failed: %s", cudaGetErrorString(e)));
    }
    if (cudaMemcpyAsync(ivf->centroids, centroids, (size_t)nlist * dim * 4, cudaMemcpyDeviceToDevice, ctx->stream) !=
        cudaSuccess)
        return fail(va_set_error(VA_ERR_CUDA, "centroid copy failed"));
    int st = va_db_create(ctx, ivf->centroids, 1, nlist, dim, VA_DTYPE_F32, 0, &ivf->cdb);
    if (st != VA_OK) return fail(st);
    // Assign every row, count the lists, prefix-sum the offsets on the host, scatter in order.
    void* ws = nullptr;
    const size_t bytes = round_up(n * 4, 256) * 2 + round_up(n * 8, 256) + (size_t)nlist * 8 + 256;
    if (cudaMalloc(&ws, bytes) != cudaSuccess) {
        cudaGetLastError();
        return fail(va_set_error(VA_ERR_OOM, "IVF build scratch failed"));
    }
    uint32_t* assign = (uint32_t*)ws;
    float* vals = (float*)((uint8_t*)ws + round_up(n * 4, 256));
    int64_t* pos = (int64_t*)((uint8_t*)vals + round_up(n * 4, 256));
    unsigned long long* counts = (unsigned long long*)((uint8_t*)pos + round_up(n * 8, 256));
    st = assign_rows(ctx, ivf->cdb, rows, n, assign, vals);
    if (st == VA_OK) {
        cudaMemsetAsync(counts, 0, (size_t)nlist * 8, ctx->stream);
        k_histogram<<<grid_for(n), 256, 0, ctx->stream>>>(assign, n, counts);
        std::vector<unsigned long long> h((size_t)nlist);
        cudaMemcpyAsync(h.data(), counts, (size_t)nlist * 8, cudaMemcpyDeviceToHost, ctx->stream);
        st = va_synchronize(ctx);
        if (st == VA_OK) {
            ivf->h_offsets.assign((size_t)nlist + 1, 0);
            for (int c = 0; c < nlist; ++c) ivf->h_offsets[(size_t)c + 1] = ivf->h_offsets[(size_t)c] + (int64_t)h[(size_t)c];
            cudaMemcpyAsync(ivf->offsets, ivf->h_offsets.data(), (size_t)(nlist + 1) * 8, cudaMemcpyHostToDevice,
                            ctx->stream);
            k_list_positions<<<nlist, 1024, 0, ctx->stream>>>(n, assign, ivf->offsets, pos, ivf->ids, id_base);
            k_place_rows<<<(unsigned)((n * 32 + 255) / 256), 256, 0, ctx->stream>>>(rows, n, dim, pos, ivf->rows);
            st = va_check_launch("k_place_rows");
        }
    }
    if (st == VA_OK) st = va_synchronize(ctx);
    cudaFree(ws);
    if (st != VA_OK) return fail(st);
    *out = ivf;
    return VA_OK;
}

int va_ivf_create_lists(va_context* ctx, const float* centroids, int nlist, int dim, const float* rows,
                        const int64_t* offsets, const uint32_t* ids, int on_device, va_ivf** out) {
    VA_REQUIRE(ctx && centroids && offsets && out, "ctx, centroids, offsets and out must not be NULL");
    VA_REQUIRE(dim > 0 && dim <= VA_MAX_DIM && nlist > 0, "dim (<= %d) and nlist must be positive", VA_MAX_DIM);
    VA_REQUIRE(offsets[0] == 0, "offsets[0] must be 0");
    for (int c = 0; c < nlist; ++c)
        VA_REQUIRE(offsets[c + 1] >= offsets[c], "offsets must be non-decreasing (list %d)", c);
    const int64_t n = offsets[nlist];
    VA_REQUIRE(n == 0 || rows, "rows must not be NULL when the lists hold vectors");
    VA_REQUIRE(n <= 0xFFFFFFFFll, "total list length exceeds the uint32 id range");
    *out = nullptr;
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    va_ivf* ivf = new va_ivf();
    ivf->ctx = ctx;
    ivf->nlist = nlist;
    ivf->dim = dim;
    ivf->n = n;
    auto fail = [&](int s) {
        va_ivf_destroy(ivf);
        return s;
    };
    const cudaMemcpyKind kind = on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    cudaError_t e = cudaMalloc((void**)&ivf->centroids, (size_t)nlist * dim * 4);
    if (e == cudaSuccess) e = cudaMalloc((void**)&ivf->rows, (size_t)std::max<int64_t>(n, 1) * dim * 4);
    if (e == cudaSuccess) e = cudaMalloc((void**)&ivf->ids, (size_t)std::max<int64_t>(n, 1) * 4);
    if (e == cudaSuccess) e = cudaMalloc((void**)&ivf->offsets, (size_t)(nlist + 1) * 8);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(va_set_error(VA_ERR_OOM, "IVF allocation failed: %s", cudaGetErrorString(e)));
    }
    ivf->h_offsets.assign(offsets, offsets + nlist + 1);
    std::vector<uint32_t> flat;
    if (!ids) {
        // The reference's vector index is the position in the concatenated lists.
        flat.resize((size_t)n);
        for (int64_t i = 0; i < n; ++i) flat[(size_t)i] = (uint32_t)i;
    }
    e = cudaMemcpyAsync(ivf->centroids, centroids, (size_t)nlist * dim * 4, kind, ctx->stream);
    if (e == cudaSuccess && n)
        e = cudaMemcpyAsync(ivf->rows, rows, (size_t)n * dim * 4, kind, ctx->stream);
    if (e == cudaSuccess && n)
        e = ids ? cudaMemcpyAsync(ivf->ids, ids, (size_t)n * 4, kind, ctx->stream)
                : cudaMemcpyAsync(ivf->ids, flat.data(), (size_t)n * 4, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(ivf->offsets, ivf->h_offsets.data(), (size_t)(nlist + 1) * 8, cudaMemcpyHostToDevice,
                            ctx->stream);
    if (e != cudaSuccess) return fail(va_set_error(VA_ERR_CUDA, "IVF upload failed: %s", cudaGetErrorString(e)));
    int st = va_synchronize(ctx);
    if (st == VA_OK) st = va_db_create(ctx, ivf->centroids, 1, nlist, dim, VA_DTYPE_F32, 0, &ivf->cdb);
    if (st != VA_OK) return fail(st);
    *out = ivf;
    return VA_OK;
}

int va_ivf_destroy(va_ivf* ivf) {
    if (!ivf) return VA_OK;
    cudaSetDevice(ivf->ctx->device);
    cudaStreamSynchronize(ivf->ctx->stream);
    if (ivf->cdb) va_db_destroy(ivf->cdb);
    if (ivf->centroids) cudaFree(ivf->centroids);
    if (ivf->rows) cudaFree(ivf->rows);
    if (ivf->ids) cudaFree(ivf->ids);
    if (ivf->offsets) cudaFree(ivf->offsets);
    delete ivf;
    return VA_OK;
}

int va_ivf_list_sizes(const va_ivf* ivf, int64_t* sizes) {
    VA_REQUIRE(ivf && sizes, "ivf and sizes must not be NULL");
    for (int c = 0; c < ivf->nlist; ++c) sizes[c] = ivf->h_offsets[(size_t)c + 1] - ivf->h_offsets[(size_t)c];
    return VA_OK;
}

int va_ivf_search(va_context* ctx, const va_ivf* ivf, const float* queries, int64_t nq, int k, int nprobe,
                  float* out_vals, uint32_t* out_ids) {
    VA_REQUIRE(ctx && ivf && queries && out_vals && out_ids, "all pointers must be non-NULL");
    VA_REQUIRE(nq > 0, "numQueries must be positive, got %lld", (long long)nq);
    VA_REQUIRE(k > 0 && k <= 128, "k must be between 1 and 128 for the IVF search, got %d", k);
    VA_REQUIRE(nprobe > 0 && nprobe <= ivf->nlist, "nprobe must be in 1..nlist (%d), got %d", ivf->nlist, nprobe);
    VA_REQUIRE(nq <= 65535, "numQueries %lld exceeds 65535 per IVF call", (long long)nq);
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    void* aux;
    const size_t pb = round_up(nq * nprobe * 4, 256);
    const size_t lb = (size_t)nprobe * nq * k;
    VA_TRY(va_aux_buffer(ctx, 2 * pb + lb * 8 + 256, &aux));
    uint32_t* probes = (uint32_t*)aux;
    float* pv = (float*)((uint8_t*)aux + pb);
    float* cv = (float*)((uint8_t*)aux + 2 * pb);
    uint32_t* ci = (uint32_t*)(cv + lb);
    // Coarse quantization: the nprobe nearest centroids of every query (exact, (distance, id)).
    VA_TRY(va_knn_search(ctx, ivf->cdb, queries, nq, nprobe, VA_METRIC_L2SQ, VA_PREC_AUTO, 0, pv, probes));
    const size_t smem = (size_t)ivf->dim * 4;
    if (smem > 48 * 1024) VA_CUDA_TRY(cudaFuncSetAttribute(k_ivf_scan, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    dim3 grid((unsigned)nprobe, (unsigned)nq);
    k_ivf_scan<<<grid, LS_THREADS, smem, ctx->stream>>>(queries, nq, ivf->dim, probes, nprobe, ivf->rows, ivf->ids,
                                                       ivf->offsets, k, cv, ci);
    VA_TRY(va_check_launch("k_ivf_scan"));
    return va_merge_lists_internal(ctx, cv, ci, nprobe, nq * k, k, nq, k, VA_SELECT_MIN, out_vals, out_ids);
}

}  // extern "C"
