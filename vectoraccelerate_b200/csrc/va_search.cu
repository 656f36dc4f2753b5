// va_search.cu -- resident databases and the fused exact k-NN search.
//
// Replaces FusedL2TopKKernel.execute and its strategies (Kernels/Metal4/FusedL2TopKKernel.swift:
// 367-427, 581-1090) and the batch flat search AcceleratedVectorIndex.searchBatchGPU
// (Index/AcceleratedVectorIndex.swift:1278-1374), extended to cosine and inner product
// (AccelerateFallback.swift:27-60; MetalComputeProvider.swift:119-217).
//
// Tensor-core route (BF16 / TF32):
//   1. queries -> padded tensor-core operand (bf16 or fp32; unit-normalised for cosine)
//   2. va_tc_filter: per (query tile, row split) the KP best approximate candidates
//   3. k_merge_rerank: per query, exact radix selection of the KP best across splits, exact
//      distances of those KP candidates in fp64 from the ORIGINAL rows (the reference's
//      arithmetic: sum((q - x)^2), dot/(|q||x|) with 0 for a zero norm, dot), final sort by
//      (distance, id) and the top k.
// The exact rerank makes the reduced-precision pass a filter only: results equal the exact
// search whenever the true top k lie in the KP-candidate pool (KP >= 3k by default).
//
// FP32 route: the reference's chunked two-pass strategy (executeChunkedTwoPass,
// FusedL2TopKKernel.swift:765-1090) on exact fp32 SIMT distance tiles, with the device merge.
#include <algorithm>
#include <cfloat>
#include <cmath>
#include <mutex>

#include "va_internal.cuh"
#include "va_tc.cuh"

int va_distance_matrix_impl(va_context* ctx, const float* q, int64_t nq, const float* x, int64_t nx, int dim,
                            int metric, int flag, float* out, int64_t out_stride, float* norm_scratch);

extern "C" int va_merge_lists_internal(va_context* ctx, const float* vals, const uint32_t* ids, int nlists,
                                       int64_t list_stride, int len, int64_t nq, int k, int mode, float* out_vals,
                                       uint32_t* out_ids);

namespace {

constexpr int KBLOCK = 64;  // tensor-core K granularity of the padded operands (elements)

__device__ __forceinline__ float load_row(const void* rows, int dtype, int64_t idx) {
    if (dtype == VA_DTYPE_BF16) return __uint_as_float((uint32_t)((const uint16_t*)rows)[idx] << 16);
    return ((const float*)rows)[idx];
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

__device__ __forceinline__ uint16_t f2bf(float f) {
    uint32_t u = __float_as_uint(f);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x40);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

// Filter row biases: norms2[r] = |x_r|^2 (fp64 accumulation rounded once) and zbias[r] = 0 for
// real rows; both +inf for the pad rows up to n_pad so padded tile columns never pass the
// filter. One warp per row.
__global__ void k_row_bias(const void* rows, int dtype, int64_t n, int64_t n_pad, int dim, float* norms2,
                           float* zbias) {
    int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (r >= n_pad) return;
    double s = 0;
    if (r < n)
        for (int j = lane; j < dim; j += 32) {
            double v = load_row(rows, dtype, r * dim + j);
            s += v * v;
        }
    s = warp_sum_d(s);
    if (lane == 0) {
        norms2[r] = r < n ? (float)s : INFINITY;
        zbias[r] = r < n ? 0.f : INFINITY;
    }
}

// Padded tensor-core operand of rows [0, n_valid) of src (rows beyond n_valid up to n_out are
// zero). OUT = uint16_t (bf16) or float. normalize: scale each row to unit L2 norm (fp64 norm;
// zero rows stay zero). One warp per row.
template <class OUT>
__global__ void k_operand(const void* src, int dtype, int64_t n_valid, int64_t n_out, int dim, int dpad,
                          int normalize, OUT* out) {
    int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (r >= n_out) return;
    double scale = 1.0;
    if (normalize && r < n_valid) {
        double s = 0;
        for (int j = lane; j < dim; j += 32) {
            double v = load_row(src, dtype, r * dim + j);
            s += v * v;
        }
        s = warp_sum_d(s);
        scale = s > 0 ? 1.0 / sqrt(s) : 0.0;
    }
    OUT* o = out + r * dpad;
    for (int j = lane; j < dpad; j += 32) {
        float v = 0.f;
        if (r < n_valid && j < dim) v = (float)(load_row(src, dtype, r * dim + j) * scale);
        if constexpr (sizeof(OUT) == 2)
            o[j] = f2bf(v);
        else
            o[j] = v;
    }
}

// Per query: select the KP best approximate candidates over all splits, rerank exactly from the
// original rows, emit the top k sorted by (distance, id).
constexpr int MR_THREADS = 256;
constexpr int MR_POOL = 1024;  // candidates kept in shared memory after the bound test

__global__ void __launch_bounds__(MR_THREADS) k_merge_rerank(const float* __restrict__ part_keys,
                                                           const uint32_t* __restrict__ part_ids, int splits,
                                                           int64_t nq_pad, int kp, int pool_n,
                                                           const float* __restrict__ queries,
                                                           const void* __restrict__ rows, int dtype, int dim, int metric,
                                                           int k, uint32_t id_base, const uint32_t* __restrict__ gthr,
                                                           BoundLevels lv,
                                                           float* __restrict__ out_vals,
                                                           uint32_t* __restrict__ out_ids,
                                                           uint32_t* __restrict__ fail_list,
                                                           uint32_t* __restrict__ fail_cnt) {
    extern __shared__ uint8_t smem[];
    const int kp2 = va::next_pow2(max(kp, pool_n));
    uint64_t* sel = (uint64_t*)smem;       // [kp2]
    uint64_t* ex = sel + kp2;               // [kp2]
    uint64_t* pool = ex + kp2;              // [MR_POOL] candidates at or below the shared bound
    float* sq = (float*)(pool + MR_POOL);   // [dim]
    __shared__ va::SelectShared sh;
    __shared__ double s_qn;
    __shared__ int s_cnt;
    const int64_t qi = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;

    for (int j = threadIdx.x; j < dim; j += blockDim.x) sq[j] = queries[qi * dim + j];
    auto get = [&](int64_t i) -> uint64_t {
        const int s = (int)(i / kp), j = (int)(i - (int64_t)s * kp);
        const int64_t off = ((int64_t)s * nq_pad + qi) * kp + j;
        const uint32_t id = part_ids[off];
        if (id == va::kInvalidId) return ~0ull;
        return va::composite(va::f2key(part_keys[off]), id);
    };
    // The filter's shared bound (per level the largest slot, the smallest over levels) is at
    // least the global pool_n-th key, so candidates above it cannot be in the pool: one pass
    // keeps the rest in shared memory and the selection runs there. If more than MR_POOL
    // survive, the selection runs over all candidates instead.
    const int64_t n_all = (int64_t)splits * kp;
    uint32_t bound = 0xFFFFFFFFu;
    for (int l = 0; gthr && l < lv.n; ++l) {
        uint32_t m = 0;
        for (int sl = 0; sl < lv.slots[l]; ++sl) m = max(m, gthr[(int64_t)(lv.off[l] + sl) * nq_pad + qi]);
        bound = min(bound, m);
    }
    if (threadIdx.x == 0) s_cnt = 0;
    __syncthreads();
    // Lists are sorted by key: one thread walks each split's list and stops at the first key
    // above the bound or the first empty entry, so only the useful prefix is read.
    for (int s = threadIdx.x; s < splits; s += blockDim.x) {
        const int64_t off = ((int64_t)s * nq_pad + qi) * kp;
        for (int j = 0; j < kp; ++j) {
            const uint32_t key = va::f2key(part_keys[off + j]);
            const uint32_t id = part_ids[off + j];
            if (key > bound || id == va::kInvalidId) break;
            const int slot = atomicAdd(&s_cnt, 1);
            if (slot < MR_POOL) pool[slot] = va::composite(key, id);
        }
    }
    __syncthreads();
    const int n_pool = s_cnt;
    int m;
    // Exactly pool_n (<= kp) best candidates by (key, id) go to the rerank.
    if (n_pool <= MR_POOL)
        m = va::block_select_radix((int64_t)n_pool, pool_n, [&](int64_t i) -> uint64_t { return pool[i]; }, sel, sh);
    else
        m = va::block_select_radix(n_all, pool_n, get, sel, sh);
    if (fail_list) {
        // Pool wider than the lists (kp < pool_n, lists filled without a shared bound): the
        // selection is the exact top pool_n by (key, id) when every split's list holds all of its
        // candidates up to the selection's largest composite T, i.e. when no full list ends below
        // T. Otherwise the query is handed to the exact fallback.
        __shared__ unsigned long long s_t;
        if (threadIdx.x == 0) s_t = 0;
        __syncthreads();
        unsigned long long t = 0;
        for (int i = threadIdx.x; i < m; i += blockDim.x)
            if (sel[i] != ~0ull && sel[i] > t) t = sel[i];
        atomicMax(&s_t, t);
        __syncthreads();
        const unsigned long long T = s_t;
        int bad = 0;
        for (int s = threadIdx.x; s < splits; s += blockDim.x) {
            const uint64_t last = get((int64_t)s * kp + kp - 1);
            if (last != ~0ull && last < T) bad = 1;
        }
        if (__syncthreads_or(bad)) {
            if (threadIdx.x == 0) fail_list[atomicAdd(fail_cnt, 1u)] = (uint32_t)qi;
            return;
        }
    }
    if (metric == VA_METRIC_COSINE && warp == 0) {
        double s = 0;
        for (int j = lane; j < dim; j += 32) s += (double)sq[j] * sq[j];
        s = warp_sum_d(s);
        if (lane == 0) s_qn = sqrt(s);
    }
    __syncthreads();
    const int mode = metric == VA_METRIC_IP ? 1 : 0;
    for (int c = warp; c < kp2; c += nwarps) {
        uint64_t comp = c < m ? sel[c] : ~0ull;
        uint32_t id = (uint32_t)comp;
        if (comp == ~0ull || id == va::kInvalidId) {
            if (lane == 0) ex[c] = ~0ull;
            continue;
        }
        const int64_t base = (int64_t)id * dim;
        double s = 0, xx = 0;
        if ((dim & 127) == 0) {
            // 16-byte (fp32) or 8-byte (bf16) loads of four consecutive elements per lane: the
            // row's loads are independent and in flight together.
#pragma unroll 4
            for (int j0 = lane * 4; j0 < dim; j0 += 128) {
                const float4 qv = *(const float4*)(sq + j0);
                float4 xv;
                if (dtype == VA_DTYPE_BF16) {
                    const uint2 u = __ldg((const uint2*)((const uint16_t*)rows + base + j0));
                    xv = make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u),
                                     __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xFFFF0000u));
                } else {
                    xv = __ldg((const float4*)((const float*)rows + base + j0));
                }
                const float qa[4] = {qv.x, qv.y, qv.z, qv.w}, xa[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    if (metric == VA_METRIC_L2SQ) {
                        const double t = (double)qa[e] - (double)xa[e];
                        s += t * t;
                    } else {
                        s += (double)qa[e] * (double)xa[e];
                        xx += (double)xa[e] * (double)xa[e];
                    }
                }
            }
        } else if (metric == VA_METRIC_L2SQ) {
            for (int j = lane; j < dim; j += 32) {
                double t = (double)sq[j] - (double)load_row(rows, dtype, base + j);
                s += t * t;
            }
        } else {
            for (int j = lane; j < dim; j += 32) {
                double xv = load_row(rows, dtype, base + j);
                s += (double)sq[j] * xv;
                xx += xv * xv;
            }
        }
        if (metric == VA_METRIC_COSINE) xx = warp_sum_d(xx);
        s = warp_sum_d(s);
        if (lane == 0) {
            float v;
            if (metric == VA_METRIC_L2SQ || metric == VA_METRIC_IP) {
                v = (float)s;
            } else {
                double den = s_qn * sqrt(xx);
                double sim = den > 0 ? s / den : 0.0;
                sim = fmin(1.0, fmax(-1.0, sim));
                v = (float)(1.0 - sim);
            }
            ex[c] = va::composite(va::mode_key(v, mode), id);
        }
    }
    va::block_bitonic_sort(ex, kp2);
    const float pad = mode ? -INFINITY : INFINITY;
    for (int i = threadIdx.x; i < k; i += blockDim.x) {
        uint64_t comp = i < kp2 ? ex[i] : ~0ull;
        float v = pad;
        uint32_t id = va::kInvalidId;
        if (comp != ~0ull) {
            id = (uint32_t)comp + id_base;
            v = va::mode_val((uint32_t)(comp >> 32), mode);
        }
        out_vals[qi * k + i] = v;
        out_ids[qi * k + i] = id;
    }
}

__global__ void k_add_base(uint32_t* ids, int64_t n, uint32_t base) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        if (ids[i] != va::kInvalidId) ids[i] += base;
}

int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

int warps_grid(int64_t warps) { return (int)((warps * 32 + 255) / 256); }

// Build (once) the operand a precision/metric needs.
int ensure_operand(va_context* ctx, va_database* db, int elem, bool cosine, const void** out) {
    const int64_t n = db->n;
    if (elem == 2) {
        uint16_t** slot = cosine ? &db->op_cos : &db->op;
        if (!*slot) {
            if (!cosine && db->dtype == VA_DTYPE_BF16 && db->dim % KBLOCK == 0) {
                db->op = (uint16_t*)db->rows;
                db->op_alias = true;
            } else {
                VA_CUDA_TRY(cudaMalloc((void**)slot, (size_t)n * db->dpad * 2));
                k_operand<uint16_t><<<warps_grid(n), 256, 0, ctx->stream>>>(db->rows, db->dtype, n, n, db->dim,
                                                                            db->dpad, cosine ? 1 : 0, *slot);
                VA_TRY(va_check_launch("k_operand<bf16>"));
            }
        }
        *out = *slot;
    } else {
        float** slot = cosine ? &db->op_f32_cos : &db->op_f32;
        if (!*slot) {
            if (!cosine && db->dtype == VA_DTYPE_F32 && db->dim % KBLOCK == 0) {
                db->op_f32 = (float*)db->rows;
                db->op_f32_alias = true;
            } else {
                VA_CUDA_TRY(cudaMalloc((void**)slot, (size_t)n * db->dpad * 4));
                k_operand<float><<<warps_grid(n), 256, 0, ctx->stream>>>(db->rows, db->dtype, n, n, db->dim,
                                                                         db->dpad, cosine ? 1 : 0, *slot);
                VA_TRY(va_check_launch("k_operand<f32>"));
            }
        }
        *out = *slot;
    }
    return VA_OK;
}

// Candidate pool per query of the reduced-precision pass: rerank * k when the caller sets the
// factor, else k plus a margin of max(k / 4, 22) (32 for k = 10, 128 for k = 100); rounded up to
// a list size the filter supports (32, 64, 128), or 0 when none is large enough.
int choose_kp(int k, int rerank) {
    int want = rerank > 0 ? rerank * k : k + std::max(k / 4, 22);
    if (want < k) want = k;
    if (want <= 32) return 32;
    if (want <= 64) return 64;
    if (want <= 128) return 128;
    return 0;
}

// Pool of va_knn_search: as choose_kp up to 128; above it the wanted size itself (the filter then
// keeps 128-entry lists without a shared bound), up to VA_MAX_SELECT_K; 0 when larger.
int choose_pool(int k, int rerank) {
    const int kp = choose_kp(k, rerank);
    if (kp) return kp;
    const int64_t want = rerank > 0 ? (int64_t)rerank * k : (int64_t)k + std::max(k / 4, 22);
    return want <= VA_MAX_SELECT_K ? (int)want : 0;
}

int merge_rerank(va_context* ctx, va_database* db, const float* queries, int64_t nq, int k, int metric,
                 const TcPlan& plan, const float* part_keys, const uint32_t* part_ids, const uint32_t* gthr,
                 float* out_vals, uint32_t* out_ids, int pool_n = 0, uint32_t* fail_list = nullptr,
                 uint32_t* fail_cnt = nullptr);
int search_fp32(va_context* ctx, va_database* db, const float* queries, int64_t nq, int k, int metric, float* out_vals,
                uint32_t* out_ids);

__global__ void k_gather_rows(const float* __restrict__ src, int dim, const uint32_t* __restrict__ rows, int64_t n,
                              float* __restrict__ dst) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n * dim; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / dim;
        dst[i] = src[(int64_t)rows[r] * dim + (i - r * dim)];
    }
}

__global__ void k_scatter_results(const float* __restrict__ v, const uint32_t* __restrict__ ids,
                                  const uint32_t* __restrict__ rows, int64_t n, int k, float* __restrict__ out_v,
                                  uint32_t* __restrict__ out_i) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n * k; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / k;
        const int64_t o = (int64_t)rows[r] * k + (i - r * k);
        out_v[o] = v[i];
        out_i[o] = ids[i];
    }
}

int grid_for(int64_t n) { return (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 8192)); }

// Failed queries of a wide-pool merge (fail_cnt entries of fail_list): exact FP32 search of those
// queries, results written to their rows. Reads the count back, so the call waits for the stream.
int fallback_exact(va_context* ctx, va_database* db, const float* queries, int k, int metric,
                   const uint32_t* fail_list, const uint32_t* fail_cnt, float* gq, float* gv, uint32_t* gi,
                   float* out_vals, uint32_t* out_ids) {
    uint32_t nf = 0;
    VA_CUDA_TRY(cudaMemcpyAsync(&nf, fail_cnt, 4, cudaMemcpyDeviceToHost, ctx->stream));
    VA_TRY(va_synchronize(ctx));
    if (!nf) return VA_OK;
    k_gather_rows<<<grid_for((int64_t)nf * db->dim), 256, 0, ctx->stream>>>(queries, db->dim, fail_list, nf, gq);
    VA_TRY(va_check_launch("k_gather_rows"));
    VA_TRY(search_fp32(ctx, db, gq, nf, k, metric, gv, gi));
    k_scatter_results<<<grid_for((int64_t)nf * k), 256, 0, ctx->stream>>>(gv, gi, fail_list, nf, k, out_vals, out_ids);
    return va_check_launch("k_scatter_results");
}

// pool <= 128: lists of the pool's size sharing a per-query bound. pool > 128: 128-entry lists
// without a shared bound; the merge selects the pool from their union where that is provably the
// exact top pool (see k_merge_rerank) and the remaining queries take the exact FP32 route.
int search_tc(va_context* ctx, va_database* db, const float* queries, int64_t nq, int k, int metric, int elem,
              int pool, float* out_vals, uint32_t* out_ids) {
    const bool wide = pool > 128;
    TcPlan plan;
    VA_TRY(va_tc_plan_pool(ctx, nq, db->n, pool, &plan, (int64_t)db->dpad * elem));
    const int kp = plan.kp;  // list length (up to 128 the whole list is the pool)
    const bool cosine = metric == VA_METRIC_COSINE;
    const void* x_op = nullptr;
    VA_TRY(ensure_operand(ctx, db, elem, cosine, &x_op));
    // Scratch: query operand, partial lists, shared per-query bounds.
    const size_t q_bytes = (size_t)plan.nq_pad * db->dpad * elem;
    const size_t part = (size_t)plan.splits * plan.nq_pad * kp;
    const size_t bytes = round_up((int64_t)q_bytes, 256) + part * 8 + (size_t)plan.bound_slots * plan.nq_pad * 4 +
                         (size_t)plan.sync_words * 4 + 256;
    void* ws;
    VA_TRY(va_workspace(ctx, bytes, &ws));
    uint8_t* p = (uint8_t*)ws;
    void* q_op = p;
    p += round_up((int64_t)q_bytes, 256);
    float* part_keys = (float*)p;
    uint32_t* part_ids = (uint32_t*)(part_keys + part);
    uint32_t* gthr = part_ids + part;
    uint32_t* sync_cnt = gthr + (size_t)plan.bound_slots * plan.nq_pad;
    if (elem == 2)
        k_operand<uint16_t><<<warps_grid(plan.nq_pad), 256, 0, ctx->stream>>>(
            queries, VA_DTYPE_F32, nq, plan.nq_pad, db->dim, db->dpad, cosine ? 1 : 0, (uint16_t*)q_op);
    else
        k_operand<float><<<warps_grid(plan.nq_pad), 256, 0, ctx->stream>>>(
            queries, VA_DTYPE_F32, nq, plan.nq_pad, db->dim, db->dpad, cosine ? 1 : 0, (float*)q_op);
    VA_TRY(va_check_launch("k_operand(queries)"));

    TcFilterArgs a = {};
    a.q_op = q_op;
    a.x_op = x_op;
    a.elem_bytes = elem;
    a.dpad = db->dpad;
    a.n_rows = db->n;
    a.row_bias = metric == VA_METRIC_L2SQ ? db->norms2 : db->zbias;
    a.alpha = metric == VA_METRIC_L2SQ ? -2.f : -1.f;
    a.part_keys = part_keys;
    a.part_ids = part_ids;
    a.gthr = gthr;
    a.sync_cnt = sync_cnt;
    a.sync_words = plan.sync_words;
    // A single pipeline wait lasts microseconds; 2 s means the pipeline is stuck.
    a.limit_ms = 2000u;
    a.levels = plan.levels;
    // Wide pools: failure list and the fallback's gathered queries and results, sized before any
    // kernel writes them.
    uint32_t* fail_cnt = nullptr;
    uint32_t* fail_list = nullptr;
    float *gq = nullptr, *gv = nullptr;
    uint32_t* gi = nullptr;
    if (wide) {
        void* aux;
        const size_t lb = round_up(4 * (nq + 64), 256), qb = round_up(nq * db->dim * 4, 256),
                     rb = round_up(nq * k * 4, 256);
        VA_TRY(va_aux_buffer(ctx, lb + qb + 2 * rb, &aux));
        fail_cnt = (uint32_t*)aux;
        fail_list = fail_cnt + 64;
        gq = (float*)((uint8_t*)aux + lb);
        gv = (float*)((uint8_t*)gq + qb);
        gi = (uint32_t*)((uint8_t*)gv + rb);
        VA_CUDA_TRY(cudaMemsetAsync(fail_cnt, 0, 4, ctx->stream));
    }
    const bool prof = ctx->prof_ev && ctx->prof_n < ctx->prof_cap;
    VA_CUDA_TRY(cudaEventRecord(prof ? ctx->prof_ev[2 * ctx->prof_n] : ctx->ev_k0, ctx->stream));
    VA_TRY(va_tc_filter(ctx, a, plan));
    VA_CUDA_TRY(cudaEventRecord(prof ? ctx->prof_ev[2 * ctx->prof_n + 1] : ctx->ev_k1, ctx->stream));
    if (prof)
        ctx->prof_n++;
    else
        ctx->k_recorded = true;
    if (!wide) return merge_rerank(ctx, db, queries, nq, k, metric, plan, part_keys, part_ids, gthr, out_vals, out_ids);
    VA_TRY(merge_rerank(ctx, db, queries, nq, k, metric, plan, part_keys, part_ids, gthr, out_vals, out_ids, pool,
                        fail_list, fail_cnt));
    return fallback_exact(ctx, db, queries, k, metric, fail_list, fail_cnt, gq, gv, gi, out_vals, out_ids);
}

int merge_rerank(va_context* ctx, va_database* db, const float* queries, int64_t nq, int k, int metric,
                 const TcPlan& plan, const float* part_keys, const uint32_t* part_ids, const uint32_t* gthr,
                 float* out_vals, uint32_t* out_ids, int pool_n, uint32_t* fail_list, uint32_t* fail_cnt) {
    const int kp2 = va::next_pow2(std::max(plan.kp, pool_n));
    size_t smem = (size_t)kp2 * 16 + (size_t)MR_POOL * 8 + (size_t)db->dim * 4;
    if (smem > 48 * 1024)
        VA_CUDA_TRY(cudaFuncSetAttribute(k_merge_rerank, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    k_merge_rerank<<<(unsigned)nq, MR_THREADS, smem, ctx->stream>>>(part_keys, part_ids, plan.splits, plan.nq_pad,
                                                                    plan.kp, pool_n > 0 ? pool_n : plan.kp, queries,
                                                                    db->rows, db->dtype, db->dim,
                                                                    metric, k, db->id_base, gthr, plan.levels,
                                                                    out_vals, out_ids,
                                                                    fail_list, fail_cnt);
    return va_check_launch("k_merge_rerank");
}

int search_fp32(va_context* ctx, va_database* db, const float* queries, int64_t nq, int k, int metric, float* out_vals,
                uint32_t* out_ids) {
    if (db->dtype != VA_DTYPE_F32)
        return va_set_error(VA_ERR_UNSUPPORTED, "precision FP32 needs an fp32 database (this one is bf16)");
    const int mode = metric == VA_METRIC_IP ? VA_SELECT_MAX : VA_SELECT_MIN;
    const int flag = metric == VA_METRIC_COSINE ? 1 : 0;
    int64_t chunk = std::max<int64_t>(256, (int64_t)(256ll << 20) / (4 * std::max<int64_t>(nq, 1)));
    chunk = std::min<int64_t>(chunk, db->n);
    const size_t mat = (size_t)nq * chunk;
    const size_t lists = (size_t)nq * k;
    const size_t norms = (size_t)nq + chunk;
    void* ws;
    VA_TRY(va_workspace(ctx, (mat + norms) * 4 + lists * 8 + 512, &ws));
    float* dmat = (float*)ws;
    float* cv = dmat + mat;
    uint32_t* ci = (uint32_t*)(cv + lists);
    float* nscratch = (float*)(ci + lists);
    const float* rows = (const float*)db->rows;
    for (int64_t c0 = 0; c0 < db->n; c0 += chunk) {
        const int64_t cn = std::min<int64_t>(chunk, db->n - c0);
        VA_REQUIRE((nq + 63) / 64 <= 65535, "numQueries %lld too large for the FP32 route", (long long)nq);
        VA_TRY(va_distance_matrix_impl(ctx, queries, nq, rows + c0 * db->dim, cn, db->dim, metric, flag, dmat, cn,
                                       nscratch));
        if (c0 == 0) {
            VA_TRY(va_topk_select(ctx, dmat, nq, cn, cn, k, mode, out_vals, out_ids, k));
        } else {
            VA_TRY(va_topk_select(ctx, dmat, nq, cn, cn, k, mode, cv, ci, k));
            VA_TRY(va_topk_merge(ctx, out_vals, out_ids, k, cv, ci, k, (uint32_t)c0, nq, mode, out_vals, out_ids));
        }
    }
    if (db->id_base) {
        k_add_base<<<std::max(1, (int)std::min<int64_t>((nq * k + 255) / 256, 4096)), 256, 0, ctx->stream>>>(
            out_ids, nq * k, db->id_base);
        VA_TRY(va_check_launch("k_add_base"));
    }
    return VA_OK;
}

}  // namespace

// Database of original rows with norms; eager_operand also builds the bf16 tensor-core operand
// (integer databases skip it: they search their own codes).
int db_create_impl(va_context* ctx, const void* rows, int on_device, int64_t n, int dim, int dtype,
                   uint32_t id_base, va_database** out, bool eager_operand) {
    VA_REQUIRE(ctx && rows && out, "ctx, rows and out must not be NULL");
    VA_REQUIRE(n > 0, "numDataset must be positive, got %lld", (long long)n);
    VA_REQUIRE(dim > 0, "dimension must be positive, got %d", dim);
    VA_REQUIRE(dim <= VA_MAX_DIM, "dimension %d exceeds maximum supported dimension %d", dim, VA_MAX_DIM);
    VA_REQUIRE(dtype == VA_DTYPE_F32 || dtype == VA_DTYPE_BF16, "dtype must be VA_DTYPE_F32 or VA_DTYPE_BF16, got %d",
               dtype);
    VA_REQUIRE((uint64_t)n + id_base <= 0xFFFFFFFFull, "numDataset %lld + id_base %u exceeds the uint32 id range",
               (long long)n, id_base);
    *out = nullptr;
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    va_database* db = new va_database();
    db->ctx = ctx;
    db->n = n;
    db->dim = dim;
    db->dtype = dtype;
    db->id_base = id_base;
    db->dpad = (int)round_up(dim, KBLOCK);
    const size_t esz = dtype == VA_DTYPE_BF16 ? 2 : 4;
    const size_t bytes = (size_t)n * dim * esz;
    const int64_t n_pad = round_up(n, 256);
    cudaError_t e = cudaMalloc(&db->rows, bytes);
    if (e == cudaSuccess) e = cudaMalloc((void**)&db->norms2, (size_t)n_pad * 4);
    if (e == cudaSuccess) e = cudaMalloc((void**)&db->zbias, (size_t)n_pad * 4);
    if (e != cudaSuccess) {
        cudaGetLastError();
        va_db_destroy(db);
        return va_set_error(VA_ERR_OOM, "database allocation (%zu bytes) failed: %s", bytes, cudaGetErrorString(e));
    }
    e = cudaMemcpyAsync(db->rows, rows, bytes, on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                        ctx->stream);
    if (e != cudaSuccess) {
        va_db_destroy(db);
        return va_set_error(VA_ERR_CUDA, "database upload failed: %s", cudaGetErrorString(e));
    }
    k_row_bias<<<warps_grid(n_pad), 256, 0, ctx->stream>>>(db->rows, dtype, n, n_pad, dim, db->norms2, db->zbias);
    int s = va_check_launch("k_row_bias");
    if (s == VA_OK && eager_operand) {
        // The bf16 operand serves the default precision: build it now so searches only read.
        const void* op;
        s = ensure_operand(ctx, db, 2, false, &op);
    }
    if (s != VA_OK) {
        va_db_destroy(db);
        return s;
    }
    *out = db;
    return VA_OK;
}

extern "C" {

int va_db_create(va_context* ctx, const void* rows, int on_device, int64_t n, int dim, int dtype, uint32_t id_base,
                 va_database** out) {
    return db_create_impl(ctx, rows, on_device, n, dim, dtype, id_base, out, true);
}

int va_db_destroy(va_database* db) {
    if (!db) return VA_OK;
    cudaSetDevice(db->ctx->device);
    cudaStreamSynchronize(db->ctx->stream);
    if (db->op && !db->op_alias) cudaFree(db->op);
    if (db->stage) cudaFree(db->stage);
    if (db->stage_norms) cudaFree(db->stage_norms);
    if (db->op_cos) cudaFree(db->op_cos);
    if (db->op_f32 && !db->op_f32_alias) cudaFree(db->op_f32);
    if (db->op_f32_cos) cudaFree(db->op_f32_cos);
    if (db->norms2) cudaFree(db->norms2);
    if (db->zbias) cudaFree(db->zbias);
    if (db->codes) cudaFree(db->codes);
    if (db->code_norms) cudaFree(db->code_norms);
    if (db->sq_mins) cudaFree(db->sq_mins);
    if (db->sq_scales) cudaFree(db->sq_scales);
    if (db->rows) cudaFree(db->rows);
    delete db;
    return VA_OK;
}

int va_db_info(const va_database* db, int64_t* n, int* dim, int* dtype) {
    VA_REQUIRE(db, "db must not be NULL");
    if (n) *n = db->n;
    if (dim) *dim = db->dim;
    if (dtype) *dtype = db->dtype;
    return VA_OK;
}

int va_db_rows(const va_database* db, const void** rows) {
    VA_REQUIRE(db && rows, "db and rows must not be NULL");
    *rows = db->rows;
    return VA_OK;
}

int va_knn_search(va_context* ctx, const va_database* cdb, const float* queries, int64_t nq, int k, int metric,
                  int precision, int rerank, float* out_vals, uint32_t* out_ids) {
    VA_REQUIRE(ctx && cdb && out_vals && out_ids, "ctx, db, out_vals and out_ids must not be NULL");
    VA_REQUIRE(cdb->kind != VA_DB_BINARY, "a binary database is searched with va_hamming_knn_db");
    VA_REQUIRE(nq > 0, "numQueries must be positive, got %lld", (long long)nq);
    VA_REQUIRE(queries, "queries must not be NULL");
    VA_REQUIRE(k > 0, "k must be positive, got %d", k);
    VA_REQUIRE(k <= VA_MAX_K, "k %d exceeds maximum supported k %d", k, VA_MAX_K);
    VA_REQUIRE(metric >= 0 && metric <= 2, "metric must be 0 (L2SQ), 1 (COSINE) or 2 (IP), got %d", metric);
    VA_REQUIRE(precision >= VA_PREC_AUTO && precision <= VA_PREC_BF16, "precision must be 0..3, got %d", precision);
    VA_REQUIRE(rerank >= 0, "rerank must be >= 0, got %d", rerank);
    va_database* db = const_cast<va_database*>(cdb);
    VA_REQUIRE(db->ctx->device == ctx->device, "database lives on device %d, context on device %d", db->ctx->device,
               ctx->device);
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    VA_CUDA_TRY(cudaEventRecord(ctx->ev_start, ctx->stream));
    ctx->k_recorded = false;
    // Pools above 128 need fp32 rows: queries whose pool cannot be proven exact take the FP32 route.
    int pool = choose_pool(k, rerank);
    if (pool > 128 && db->dtype != VA_DTYPE_F32) pool = 0;
    int prec = precision;
    // AUTO: bf16 when the pool holds at least 3k candidates. Without a caller's factor, fp32 rows
    // take a 3k pool (wider than 128 from k = 43 on) to stay on bf16; otherwise (bf16 rows, a thin
    // caller-set pool) the 4x smaller tf32 error keeps the true top k inside the pool. No pool
    // size -> exact FP32 route. Rows of at most 16 dimensions (fp32) take the FP32 route too: few
    // dimensions give the reduced-precision keys no resolution between close neighbours (for
    // d = 1 a bf16 key cannot order points 1/N apart), and the SIMT route is cheap there.
    if (prec == VA_PREC_AUTO) {
        if (pool && pool < 3 * k && rerank == 0 && db->dtype == VA_DTYPE_F32 && 3 * k <= VA_MAX_SELECT_K)
            pool = 3 * k;
        prec = !pool ? VA_PREC_FP32 : (pool >= 3 * k ? VA_PREC_BF16 : VA_PREC_TF32);
        if (db->dim <= 16 && db->dtype == VA_DTYPE_F32) prec = VA_PREC_FP32;
    }
    if (prec == VA_PREC_FP32 && db->dtype != VA_DTYPE_F32) {
        if (!pool) return va_set_error(VA_ERR_UNSUPPORTED, "k %d needs the FP32 route, which needs fp32 rows", k);
        prec = VA_PREC_BF16;
    }
    if (prec == VA_PREC_FP32) {
        VA_TRY(search_fp32(ctx, db, queries, nq, k, metric, out_vals, out_ids));
    } else {
        if (!pool)
            return va_set_error(VA_ERR_UNSUPPORTED,
                                "candidate pool %lld of k %d is not supported by the tensor-core route (at most %d, "
                                "above 128 with fp32 rows); use precision FP32",
                                (long long)(rerank ? (int64_t)rerank * k : (int64_t)k + std::max(k / 4, 22)), k,
                                VA_MAX_SELECT_K);
        const int elem = prec == VA_PREC_TF32 ? 4 : 2;
        VA_TRY(search_tc(ctx, db, queries, nq, k, metric, elem, pool, out_vals, out_ids));
    }
    VA_CUDA_TRY(cudaEventRecord(ctx->ev_stop, ctx->stream));
    return VA_OK;
}

int va_knn_search_host(va_context* ctx, const va_database* db, const float* queries_host, int64_t nq, int k,
                       int metric, int precision, int rerank, float* out_vals_host, uint32_t* out_ids_host) {
    VA_REQUIRE(ctx && db && queries_host && out_vals_host && out_ids_host, "all pointers must be non-NULL");
    VA_REQUIRE(nq > 0, "numQueries must be positive, got %lld", (long long)nq);
    VA_REQUIRE(k > 0, "k must be positive, got %d", k);
    VA_REQUIRE(k <= VA_MAX_K, "k %d exceeds maximum supported k %d", k, VA_MAX_K);
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    const size_t qb = (size_t)nq * db->dim * 4, rb = (size_t)nq * k * 4;
    void* io;
    VA_TRY(va_io_buffer(ctx, round_up((int64_t)qb, 256) + 2 * round_up((int64_t)rb, 256), &io));
    float* dq = (float*)io;
    float* dv = (float*)((uint8_t*)io + round_up((int64_t)qb, 256));
    uint32_t* di = (uint32_t*)((uint8_t*)dv + round_up((int64_t)rb, 256));
    VA_CUDA_TRY(cudaMemcpyAsync(dq, queries_host, qb, cudaMemcpyHostToDevice, ctx->stream));
    VA_TRY(va_knn_search(ctx, db, dq, nq, k, metric, precision, rerank, dv, di));
    VA_CUDA_TRY(cudaMemcpyAsync(out_vals_host, dv, rb, cudaMemcpyDeviceToHost, ctx->stream));
    VA_CUDA_TRY(cudaMemcpyAsync(out_ids_host, di, rb, cudaMemcpyDeviceToHost, ctx->stream));
    VA_TRY(va_synchronize(ctx));
    cudaEventElapsedTime(&ctx->last_ms, ctx->ev_start, ctx->ev_stop);
    return VA_OK;
}

}  // extern "C"

// ------------------------------------------------------------------------------------------------
// Search without device allocation.
//
// Some callers cannot let a search call cudaMalloc: serving processes that hand all free device
// memory to their own pool at start-up (a later cudaMalloc would fail), callers whose device
// memory is owned by another allocator that forbids side allocations, and latency-bound paths
// where an allocation's implicit device synchronisation would stall other streams.
// va_knn_search_noalloc gives them the tensor-core search with its scratch (query operand,
// per-split candidate lists, per-query bounds) in one fixed device array of
// VA_NOALLOC_SCRATCH_BYTES, declared below; every GPU that loads the library holds that array
// until the process exits.
// ------------------------------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_noalloc_scratch[VA_NOALLOC_SCRATCH_BYTES];

namespace {

// Device address of g_noalloc_scratch on each device. In host code the array's name is only a
// host-side stand-in, so the address comes from cudaGetSymbolAddress, once per device, with that
// device current.
std::mutex g_noalloc_mu;
void* g_noalloc_addr[256] = {};

int noalloc_scratch(int device, void** out) {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (device < 0 || device >= 256) return va_set_error(VA_ERR_INVALID_ARG, "device %d out of range", device);
    if (!g_noalloc_addr[device]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p)
            return va_set_error(VA_ERR_CUDA, "cudaGetSymbolAddress of the fixed scratch failed on device %d: %s",
                                device, cudaGetErrorString(e));
        g_noalloc_addr[device] = p;
    }
    *out = g_noalloc_addr[device];
    return VA_OK;
}

// Same steps as search_tc, with the scratch carved from a caller-provided region.
int search_tc_fixed(va_context* ctx, va_database* db, const float* queries, int64_t nq, int k, int metric, int elem,
                    int kp, uint8_t* scratch, size_t scratch_bytes, float* out_vals, uint32_t* out_ids) {
    TcPlan plan;
    VA_TRY(va_tc_plan(ctx, nq, db->n, kp, &plan, (int64_t)db->dpad * elem));
    const bool cosine = metric == VA_METRIC_COSINE;
    const void* x_op = elem == 2 ? (cosine ? (const void*)db->op_cos : (const void*)db->op)
                                 : (cosine ? (const void*)db->op_f32_cos : (const void*)db->op_f32);
    if (!x_op)
        return va_set_error(VA_ERR_UNSUPPORTED,
                            "the %s operand of this database is not built yet and building it would allocate; run "
                            "one va_knn_search with this metric and precision first",
                            elem == 2 ? (cosine ? "unit-norm bf16" : "bf16") : (cosine ? "unit-norm fp32" : "fp32"));
    const size_t q_bytes = (size_t)plan.nq_pad * db->dpad * elem;
    const size_t part = (size_t)plan.splits * plan.nq_pad * kp;
    const size_t bytes =
        round_up((int64_t)q_bytes, 256) + part * 8 + (size_t)plan.nq_pad * 4 + (size_t)plan.sync_words * 4;
    if (bytes > scratch_bytes)
        return va_set_error(VA_ERR_INVALID_ARG,
                            "numQueries %lld at dimension %d needs %zu bytes of scratch; the allocation-free search "
                            "has %zu (split the batch)",
                            (long long)nq, db->dim, bytes, scratch_bytes);
    uint8_t* p = scratch;
    void* q_op = p;
    p += round_up((int64_t)q_bytes, 256);
    float* part_keys = (float*)p;
    uint32_t* part_ids = (uint32_t*)(part_keys + part);
    uint32_t* gthr = part_ids + part;
    uint32_t* sync_cnt = gthr + plan.nq_pad;
    if (elem == 2)
        k_operand<uint16_t><<<warps_grid(plan.nq_pad), 256, 0, ctx->stream>>>(
            queries, VA_DTYPE_F32, nq, plan.nq_pad, db->dim, db->dpad, cosine ? 1 : 0, (uint16_t*)q_op);
    else
        k_operand<float><<<warps_grid(plan.nq_pad), 256, 0, ctx->stream>>>(
            queries, VA_DTYPE_F32, nq, plan.nq_pad, db->dim, db->dpad, cosine ? 1 : 0, (float*)q_op);
    VA_TRY(va_check_launch("k_operand(queries)"));
    TcFilterArgs a = {};
    a.q_op = q_op;
    a.x_op = x_op;
    a.elem_bytes = elem;
    a.dpad = db->dpad;
    a.n_rows = db->n;
    a.row_bias = metric == VA_METRIC_L2SQ ? db->norms2 : db->zbias;
    a.alpha = metric == VA_METRIC_L2SQ ? -2.f : -1.f;
    a.part_keys = part_keys;
    a.part_ids = part_ids;
    a.gthr = gthr;          // va_tc_filter resets it before the launch
    a.sync_cnt = sync_cnt;  // likewise
    a.sync_words = plan.sync_words;
    a.limit_ms = 2000u;
    VA_TRY(va_tc_filter(ctx, a, plan));
    return merge_rerank(ctx, db, queries, nq, k, metric, plan, part_keys, part_ids, gthr, out_vals, out_ids);
}

}  // namespace

extern "C" int va_knn_search_noalloc(va_context* ctx, const va_database* cdb, const float* queries, int64_t nq, int k,
                                     int metric, int precision, int rerank, float* out_vals, uint32_t* out_ids) {
    VA_REQUIRE(ctx && cdb && out_vals && out_ids, "ctx, db, out_vals and out_ids must not be NULL");
    VA_REQUIRE(cdb->kind != VA_DB_BINARY, "a binary database is searched with va_hamming_knn_db");
    VA_REQUIRE(nq > 0, "numQueries must be positive, got %lld", (long long)nq);
    VA_REQUIRE(queries, "queries must not be NULL");
    VA_REQUIRE(k > 0, "k must be positive, got %d", k);
    VA_REQUIRE(k <= VA_MAX_K, "k %d exceeds maximum supported k %d", k, VA_MAX_K);
    VA_REQUIRE(metric >= 0 && metric <= 2, "metric must be 0 (L2SQ), 1 (COSINE) or 2 (IP), got %d", metric);
    VA_REQUIRE(precision == VA_PREC_AUTO || precision == VA_PREC_BF16 || precision == VA_PREC_TF32,
               "the allocation-free search runs the tensor-core route only (precision AUTO, BF16 or TF32), got %d",
               precision);
    VA_REQUIRE(rerank >= 0, "rerank must be >= 0, got %d", rerank);
    va_database* db = const_cast<va_database*>(cdb);
    VA_REQUIRE(db->ctx->device == ctx->device, "database lives on device %d, context on device %d", db->ctx->device,
               ctx->device);
    const int kp = choose_kp(k, rerank);
    VA_REQUIRE(kp > 0, "candidate pool of k %d exceeds the tensor-core filter's 128", k);
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    void* scratch = nullptr;
    VA_TRY(noalloc_scratch(ctx->device, &scratch));
    const int elem = precision == VA_PREC_TF32 ? 4 : 2;
    return search_tc_fixed(ctx, db, queries, nq, k, metric, elem, kp, (uint8_t*)scratch, VA_NOALLOC_SCRATCH_BYTES,
                           out_vals, out_ids);
}

// Derived per-row data of a float (or int8) database for rows [r0, r0 + count): row biases (and
// the +inf pad after them up to a multiple of 256 rows) and every tensor-core operand already
// built (aliases of the rows need nothing). Used by ingestion after rows were written.
int va_db_derive_rows(va_context* ctx, va_database* db, int64_t r0, int64_t count) {
    if (count <= 0) return VA_OK;
    const size_t esz = db->dtype == VA_DTYPE_BF16 ? 2 : 4;
    const void* src = (const uint8_t*)db->rows + (size_t)r0 * db->dim * esz;
    // Rows past the database's end (up to a multiple of 256) get the +inf pad; rows inside it
    // (an update in the middle) are left alone.
    const int64_t pad_end = r0 + count >= db->n ? round_up(db->n, 256) : r0 + count;
    if (db->norms2) {
        k_row_bias<<<warps_grid(pad_end - r0), 256, 0, ctx->stream>>>(src, db->dtype, count, pad_end - r0, db->dim,
                                                                      db->norms2 + r0, db->zbias + r0);
        VA_TRY(va_check_launch("k_row_bias(append)"));
    }
    const int64_t dp = db->dpad;
    if (db->op && !db->op_alias)
        k_operand<uint16_t><<<warps_grid(count), 256, 0, ctx->stream>>>(src, db->dtype, count, count, db->dim, db->dpad,
                                                                        0, db->op + r0 * dp);
    if (db->op_cos)
        k_operand<uint16_t><<<warps_grid(count), 256, 0, ctx->stream>>>(src, db->dtype, count, count, db->dim, db->dpad,
                                                                        1, db->op_cos + r0 * dp);
    if (db->op_f32 && !db->op_f32_alias)
        k_operand<float><<<warps_grid(count), 256, 0, ctx->stream>>>(src, db->dtype, count, count, db->dim, db->dpad,
                                                                     0, db->op_f32 + r0 * dp);
    if (db->op_f32_cos)
        k_operand<float><<<warps_grid(count), 256, 0, ctx->stream>>>(src, db->dtype, count, count, db->dim, db->dpad,
                                                                     1, db->op_f32_cos + r0 * dp);
    return va_check_launch("k_operand(append)");
}

// Internal entry of the merge + exact rerank step for other translation units (the int8 path).
int va_merge_rerank_internal(va_context* ctx, va_database* db, const float* queries, int64_t nq, int k, int metric,
                             const TcPlan& plan, const float* part_keys, const uint32_t* part_ids,
                             const uint32_t* gthr, float* out_vals, uint32_t* out_ids, int pool_n,
                             uint32_t* fail_list, uint32_t* fail_cnt) {
    return merge_rerank(ctx, db, queries, nq, k, metric, plan, part_keys, part_ids, gthr, out_vals, out_ids, pool_n,
                        fail_list, fail_cnt);
}
