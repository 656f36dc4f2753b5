// va_int.cu -- integer-code search paths on the int8 tensor cores (tcgen05.mma kind::i8, exact
// int32 accumulation).
//
// int8 scalar-quantized L2 (the benchmark's int8 configuration). The reference quantizes with
// global scales only (ScalarQuantizationKernel.swift:496-520, DataTransformations.metal:174-201);
// per-dimension codes are this build's definition, shared with the oracle: scale_j =
// max((max_j - min_j)/255, 1e-8), code = clamp(rint((x - min_j)/scale_j), 0, 255) - 128.
// L2 on codes is exact in int32 (|c_q|^2 + |c_x|^2 - 2 c_q.c_x <= 768 * 255^2), the top
// `candidates` codes by (integer distance, id) are reranked exactly against the fp32 rows.
//
// Hamming. popcount(q ^ x) of LSB-first packed codes (Metal4BinaryVector.hammingDistance,
// BinaryQuantizationKernel.swift:65-74) equals |q| + |x| - 2 q.x over the 0/1 expansion of the
// bits, so the binary database stores its codes as 0/1 bytes and the same integer contraction
// computes exact Hamming distances; results are ordered by (distance, id) with no rerank.
#include <algorithm>

#include "va_internal.cuh"
#include "va_tc.cuh"

extern "C" int va_merge_lists_internal(va_context* ctx, const float* vals, const uint32_t* ids, int nlists,
                                       int64_t list_stride, int len, int64_t nq, int k, int mode, float* out_vals,
                                       uint32_t* out_ids);
int db_create_impl(va_context* ctx, const void* rows, int on_device, int64_t n, int dim, int dtype,
                   uint32_t id_base, va_database** out, bool eager_operand);
int va_merge_rerank_internal(va_context* ctx, va_database* db, const float* queries, int64_t nq, int k, int metric,
                             const TcPlan& plan, const float* part_keys, const uint32_t* part_ids,
                             const uint32_t* gthr, float* out_vals, uint32_t* out_ids, int pool_n,
                             uint32_t* fail_list, uint32_t* fail_cnt);

namespace {

constexpr int CBLOCK = 128;  // int8 operand K granularity (one 128-byte swizzle row)

int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }
int warps_grid(int64_t warps) { return (int)((warps * 32 + 255) / 256); }

__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

// Per-column min / max (orderable keys, combined with atomics). Block: 8 rows x 32 columns.
__global__ void k_col_minmax(const float* __restrict__ x, int64_t n, int dim, unsigned* kmin, unsigned* kmax) {
    const int c = blockIdx.x * 32 + (threadIdx.x & 31);
    const int rr = threadIdx.x >> 5;
    float mn = INFINITY, mx = -INFINITY;
    if (c < dim)
        for (int64_t r = (int64_t)blockIdx.y * 8 + rr; r < n; r += (int64_t)gridDim.y * 8) {
            const float v = x[r * dim + c];
            mn = fminf(mn, v);
            mx = fmaxf(mx, v);
        }
    __shared__ float smn[8][32], smx[8][32];
    smn[rr][threadIdx.x & 31] = mn;
    smx[rr][threadIdx.x & 31] = mx;
    __syncthreads();
    if (rr == 0 && c < dim) {
        for (int j = 1; j < 8; ++j) {
            mn = fminf(mn, smn[j][threadIdx.x]);
            mx = fmaxf(mx, smx[j][threadIdx.x]);
        }
        atomicMin(kmin + c, va::f2key(mn));
        atomicMax(kmax + c, va::f2key(mx));
    }
}

__global__ void k_init_keys(unsigned* kmin, unsigned* kmax, int dim) {
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < dim; j += gridDim.x * blockDim.x) {
        kmin[j] = 0xFFFFFFFFu;
        kmax[j] = 0u;
    }
}

__global__ void k_keys_to_minmax(const unsigned* kmin, const unsigned* kmax, int dim, float* mins, float* maxs) {
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < dim; j += gridDim.x * blockDim.x) {
        mins[j] = va::key2f(kmin[j]);
        maxs[j] = va::key2f(kmax[j]);
    }
}

// Per-dimension parameters from min / max arrays (in place allowed: mins may alias mn_in, scales
// may alias mx_in).
__global__ void k_minmax_to_params(const float* mn_in, const float* mx_in, int dim, float* mins, float* scales) {
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < dim; j += gridDim.x * blockDim.x) {
        mins[j] = mn_in[j];
        scales[j] = fmaxf(__fdiv_rn(mx_in[j] - mn_in[j], 255.0f), 1e-8f);
    }
}

// Codes [n_out x cpad] (rows >= n_valid and columns >= dim are 0) and |code|^2 per row. One warp
// per row. code = clamp(rint((x - min)/scale), 0, 255) - 128 with IEEE division and round half
// to even, as the oracle computes it.
__global__ void k_perdim_codes(const float* __restrict__ x, int64_t n_valid, int64_t n_out, int dim, int cpad,
                               const float* __restrict__ mins, const float* __restrict__ scales, int8_t* __restrict__ out,
                               int* __restrict__ norms) {
    const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (r >= n_out) return;
    int acc = 0;
    for (int j = lane; j < cpad; j += 32) {
        int c = 0;
        if (r < n_valid && j < dim) {
            float u = rintf(__fdiv_rn(x[r * dim + j] - mins[j], scales[j]));
            u = fminf(255.f, fmaxf(0.f, u));
            c = (int)u - 128;
        }
        out[r * cpad + j] = (int8_t)c;
        acc += c * c;
    }
    acc = warp_sum_i(acc);
    if (lane == 0 && norms) norms[r] = acc;
}

// Four bits (LSB first) -> four 0/1 bytes of a little-endian word.
__device__ __forceinline__ uint32_t spread4(uint32_t x) {
    return (x & 1u) | ((x & 2u) << 7) | ((x & 4u) << 14) | ((x & 8u) << 21);
}

// 0/1 bytes of LSB-first packed codes [n_out x cpad] and popcounts. One warp per row; each lane
// expands whole 32-bit words into 32 bytes (two 16-byte stores).
__global__ void k_expand_bits(const uint32_t* __restrict__ codes, int64_t n_valid, int64_t n_out, int words, int cpad,
                              int8_t* __restrict__ out, int* __restrict__ pops) {
    const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (r >= n_out) return;
    int acc = 0;
    for (int w = lane; w < cpad / 32; w += 32) {
        const uint32_t x = (r < n_valid && w < words) ? __ldg(codes + r * words + w) : 0u;
        acc += __popc(x);
        uint4 lo, hi;
        lo.x = spread4(x);
        lo.y = spread4(x >> 4);
        lo.z = spread4(x >> 8);
        lo.w = spread4(x >> 12);
        hi.x = spread4(x >> 16);
        hi.y = spread4(x >> 20);
        hi.z = spread4(x >> 24);
        hi.w = spread4(x >> 28);
        uint4* o = (uint4*)(out + r * cpad + (int64_t)w * 32);
        o[0] = lo;
        o[1] = hi;
    }
    acc = warp_sum_i(acc);
    if (lane == 0) pops[r] = acc;
}

__global__ void k_bits_to_dists(const float* __restrict__ v, const uint32_t* __restrict__ ids, int64_t n,
                                uint32_t* __restrict__ out) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = ids[i] == va::kInvalidId ? 0xFFFFFFFFu : __float_as_uint(v[i]);
}

__global__ void k_add_base_ids(uint32_t* ids, int64_t n, uint32_t base) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        if (ids[i] != va::kInvalidId) ids[i] += base;
}

// Exact integer L2 of SCAN_Q queries (blockIdx.y tile) against every row, on the CUDA cores
// (dp4a): out[q * n + r] = bit pattern of |x_r|^2 + |q|^2 - 2 q.x_r as a float. The exact route
// for queries whose wide candidate pool the filter's lists could not prove.
constexpr int SCAN_Q = 8;

__global__ void __launch_bounds__(256) k_int8_scan(const int8_t* __restrict__ qc, const int* __restrict__ qn, int nqf,
                                                   const int8_t* __restrict__ xc, const int* __restrict__ xn, int64_t n,
                                                   int cpad, float* __restrict__ out) {
    extern __shared__ int4 s_q[];  // [SCAN_Q][cpad / 16]
    const int cw = cpad / 16;
    const int q0 = blockIdx.y * SCAN_Q;
    const int nqt = min(SCAN_Q, nqf - q0);
    for (int i = threadIdx.x; i < SCAN_Q * cw; i += blockDim.x) {
        const int qq = i / cw;
        s_q[i] = qq < nqt ? ((const int4*)(qc + (int64_t)(q0 + qq) * cpad))[i - qq * cw] : make_int4(0, 0, 0, 0);
    }
    __syncthreads();
    for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < n; r += (int64_t)gridDim.x * blockDim.x) {
        int acc[SCAN_Q];
#pragma unroll
        for (int j = 0; j < SCAN_Q; ++j) acc[j] = 0;
        const int4* xr = (const int4*)(xc + r * cpad);
        for (int c = 0; c < cw; ++c) {
            const int4 xv = __ldg(xr + c);
#pragma unroll
            for (int j = 0; j < SCAN_Q; ++j) {
                const int4 qv = s_q[j * cw + c];
                acc[j] = __dp4a(qv.x, xv.x, acc[j]);
                acc[j] = __dp4a(qv.y, xv.y, acc[j]);
                acc[j] = __dp4a(qv.z, xv.z, acc[j]);
                acc[j] = __dp4a(qv.w, xv.w, acc[j]);
            }
        }
        const int xnr = xn[r];
#pragma unroll
        for (int j = 0; j < SCAN_Q; ++j)
            if (j < nqt) out[(int64_t)(q0 + j) * n + r] = __int_as_float(xnr + qn[q0 + j] - 2 * acc[j]);
    }
}

__global__ void k_gather_f32_rows(const float* __restrict__ src, int dim, const uint32_t* __restrict__ rows, int64_t n,
                                  float* __restrict__ dst) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n * dim; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / dim;
        dst[i] = src[(int64_t)rows[r] * dim + (i - r * dim)];
    }
}

__global__ void k_scatter_rows(const float* __restrict__ v, const uint32_t* __restrict__ ids,
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

// ------------------------------------------------------------------------------------------------
// Small-batch Hamming scan (NQ <= 8 queries): one streaming pass over the PACKED codes, which is
// HBM-bound (128 B per 1024-bit row) where the tensor-core route would read the 8x larger 0/1
// expansion. LPR = WORDS/4 lanes hold one row (16 B each, coalesced); popcounts are reduced over
// those lanes. Each CTA keeps, per query, a shared-memory buffer of (distance << 32 | row)
// composites below its running threshold (the k-th best composite after the last compaction);
// when a buffer could overflow in the next iteration, a block-wide radix selection compacts it to
// the k best. Each CTA writes its k best per query; a merge over CTAs gives the result.
constexpr int HS_THREADS = 256;
constexpr int HS_BUF = 1024;  // composites per query buffer

template <int WORDS, int NQ>
__global__ void __launch_bounds__(HS_THREADS) k_hamming_scan(const uint32_t* __restrict__ x, int64_t n,
                                                             const uint32_t* __restrict__ q, int nq, int k,
                                                             int64_t rows_per_cta, float* __restrict__ part_vals,
                                                             uint32_t* __restrict__ part_ids) {
    constexpr int LPR = WORDS / 4;               // lanes per row
    constexpr int RPW = 32 / LPR;                // rows per warp load
    // Loads in flight per lane; an iteration covers at most 512 rows, so a buffer compacted to
    // <= 128 entries (or holding <= HS_BUF - IROWS) cannot overflow in the next one.
    constexpr int HS_UNROLL = WORDS / 2 < 8 ? WORDS / 2 : 8;
    constexpr int WROWS = RPW * HS_UNROLL;       // rows per warp per iteration
    constexpr int IROWS = WROWS * (HS_THREADS / 32);
    static_assert(IROWS + 128 <= HS_BUF && IROWS <= HS_BUF / 2, "buffer too small for one iteration");
    extern __shared__ uint64_t s_buf[];          // [NQ][HS_BUF]
    __shared__ uint64_t s_tmp[128];
    __shared__ unsigned long long s_thr[NQ];
    __shared__ int s_cnt[NQ];
    __shared__ va::SelectShared sh;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int sub = lane % LPR, rsub = lane / LPR;
    uint4 qv[NQ];
#pragma unroll
    for (int j = 0; j < NQ; ++j)
        qv[j] = j < nq ? ((const uint4*)(q + (int64_t)j * WORDS))[sub] : make_uint4(0, 0, 0, 0);
    if (threadIdx.x < NQ) {
        s_thr[threadIdx.x] = ~0ull;
        s_cnt[threadIdx.x] = 0;
    }
    __syncthreads();
    const int64_t r0 = (int64_t)blockIdx.x * rows_per_cta;
    const int64_t r1 = min(n, r0 + rows_per_cta);

    // Compact query j's buffer to its k best composites (block-wide; all threads call).
    auto compact = [&](int j) {
        const int c = min(s_cnt[j], HS_BUF);
        uint64_t* b = s_buf + (size_t)j * HS_BUF;
        const int m = va::block_select_radix((int64_t)c, k, [&](int64_t i) -> uint64_t { return b[i]; }, s_tmp, sh);
        __syncthreads();
        for (int i = threadIdx.x; i < m; i += blockDim.x) b[i] = s_tmp[i];
        __syncthreads();
        if (threadIdx.x == 0) {
            s_cnt[j] = m;
            if (m == k) {
                unsigned long long t = 0;
                for (int i = 0; i < m; ++i) t = b[i] > t ? b[i] : t;
                s_thr[j] = t;
            }
        }
        __syncthreads();
    };

    for (int64_t base = r0; base < r1; base += IROWS) {
        const int64_t wbase = base + (int64_t)warp * WROWS;
        uint4 v[HS_UNROLL];
#pragma unroll
        for (int u = 0; u < HS_UNROLL; ++u) {
            const int64_t row = wbase + u * RPW + rsub;
            v[u] = row < r1 ? __ldcs((const uint4*)(x + row * WORDS) + sub) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < HS_UNROLL; ++u) {
            const int64_t row = wbase + u * RPW + rsub;
#pragma unroll
            for (int j = 0; j < NQ; ++j) {
                uint32_t d = __popc(v[u].x ^ qv[j].x) + __popc(v[u].y ^ qv[j].y) + __popc(v[u].z ^ qv[j].z) +
                             __popc(v[u].w ^ qv[j].w);
#pragma unroll
                for (int o = 1; o < LPR; o <<= 1) d += __shfl_xor_sync(0xFFFFFFFFu, d, o);
                const uint64_t comp = ((uint64_t)d << 32) | (uint64_t)(uint32_t)row;
                if (sub == 0 && j < nq && row < r1 && comp < s_thr[j]) {
                    const int slot = atomicAdd(&s_cnt[j], 1);
                    if (slot < HS_BUF) s_buf[(size_t)j * HS_BUF + slot] = comp;
                }
            }
        }
        __syncthreads();
        // A buffer that the next iteration could overflow is compacted now (uniform decision).
        for (int j = 0; j < nq; ++j)
            if (s_cnt[j] > HS_BUF - IROWS) compact(j);
    }
    for (int j = 0; j < nq; ++j) {
        compact(j);
        const int m = s_cnt[j];
        float* pv = part_vals + ((int64_t)blockIdx.x * nq + j) * k;
        uint32_t* pi = part_ids + ((int64_t)blockIdx.x * nq + j) * k;
        for (int i = threadIdx.x; i < k; i += blockDim.x) {
            const uint64_t c = i < m ? s_buf[(size_t)j * HS_BUF + i] : ~0ull;
            pv[i] = c == ~0ull ? INFINITY : __uint_as_float((uint32_t)(c >> 32));
            pi[i] = c == ~0ull ? va::kInvalidId : (uint32_t)c;
        }
        __syncthreads();
    }
}

template <int WORDS, int NQ>
int launch_hscan(va_context* ctx, const uint32_t* x, int64_t n, const uint32_t* q, int nq, int k, int grid,
                 int64_t rows_per_cta, float* pv, uint32_t* pi) {
    const size_t smem = (size_t)NQ * HS_BUF * 8;
    if (smem > 48 * 1024)
        VA_CUDA_TRY(cudaFuncSetAttribute(k_hamming_scan<WORDS, NQ>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    k_hamming_scan<WORDS, NQ><<<grid, HS_THREADS, smem, ctx->stream>>>(x, n, q, nq, k, rows_per_cta, pv, pi);
    return va_check_launch("k_hamming_scan");
}

template <int WORDS>
int dispatch_hscan(va_context* ctx, const uint32_t* x, int64_t n, const uint32_t* q, int nq, int k, int grid,
                   int64_t rows_per_cta, float* pv, uint32_t* pi) {
    if (nq <= 1) return launch_hscan<WORDS, 1>(ctx, x, n, q, nq, k, grid, rows_per_cta, pv, pi);
    if (nq <= 2) return launch_hscan<WORDS, 2>(ctx, x, n, q, nq, k, grid, rows_per_cta, pv, pi);
    if (nq <= 4) return launch_hscan<WORDS, 4>(ctx, x, n, q, nq, k, grid, rows_per_cta, pv, pi);
    return launch_hscan<WORDS, 8>(ctx, x, n, q, nq, k, grid, rows_per_cta, pv, pi);
}

constexpr int HS_MAX_Q = 8;

bool hscan_supported(int words, int64_t nq) {
    return nq <= HS_MAX_Q && (words == 4 || words == 8 || words == 16 || words == 32);
}


// Filter over the database's integer codes for queries already encoded in q_codes / q_norms
// (both [plan.nq_pad]); partial lists land in the returned workspace pointers.
struct IntScratch {
    int8_t* q_codes;
    int* q_norms;
    float* part_keys;
    uint32_t* part_ids;
    uint32_t* gthr;
    uint32_t* sync;
};

int int_scratch(va_context* ctx, const va_database* db, const TcPlan& plan, IntScratch* s) {
    const size_t qb = (size_t)plan.nq_pad * db->cpad;
    const size_t part = (size_t)plan.splits * plan.nq_pad * plan.kp;
    const size_t bytes = round_up((int64_t)qb, 256) + (size_t)plan.nq_pad * 4 + part * 8 +
                         (size_t)plan.bound_slots * plan.nq_pad * 4 + (size_t)plan.sync_words * 4 + 512;
    void* ws;
    VA_TRY(va_workspace(ctx, bytes, &ws));
    uint8_t* p = (uint8_t*)ws;
    s->q_codes = (int8_t*)p;
    p += round_up((int64_t)qb, 256);
    s->q_norms = (int*)p;
    s->part_keys = (float*)(s->q_norms + plan.nq_pad);
    s->part_ids = (uint32_t*)(s->part_keys + part);
    s->gthr = s->part_ids + part;
    s->sync = s->gthr + (size_t)plan.bound_slots * plan.nq_pad;
    return VA_OK;
}

int run_int_filter(va_context* ctx, const va_database* db, const TcPlan& plan, const IntScratch& s) {
    TcFilterArgs a = {};
    a.levels = plan.levels;
    a.q_op = s.q_codes;
    a.x_op = db->codes;
    a.elem_bytes = 1;
    a.dpad = db->cpad;
    a.n_rows = db->n;
    a.row_bias = (const float*)db->code_norms;
    a.alpha = -2.f;
    a.row_qn = s.q_norms;
    a.part_keys = s.part_keys;
    a.part_ids = s.part_ids;
    a.gthr = s.gthr;
    a.sync_cnt = s.sync;
    a.sync_words = plan.sync_words;
    a.limit_ms = 2000u;
    return va_tc_filter(ctx, a, plan);
}

// Queries of an int8 search whose wide pool could not be proven from the filter's lists: exact
// integer distances to every row (k_int8_scan), the `pool` best by (distance, id), the same exact
// rerank, results written to their rows. Reads the failure count back (waits for the stream).
int int8_fallback(va_context* ctx, va_database* db, const float* queries, int k, int pool, const uint32_t* fail_list,
                  const uint32_t* fail_cnt, float* gq, float* gv, uint32_t* gi, float* out_vals, uint32_t* out_ids) {
    uint32_t nf = 0;
    VA_TRY(va_read_u32(ctx, fail_cnt, &nf));
    if (!nf) return VA_OK;
    const int dim = db->dim, cpad = db->cpad;
    const int64_t n = db->n;
    k_gather_f32_rows<<<grid_for((int64_t)nf * dim), 256, 0, ctx->stream>>>(queries, dim, fail_list, nf, gq);
    VA_TRY(va_check_launch("k_gather_f32_rows"));
    // Chunks of f queries: distances [f x n] fp32 bit patterns within 256 MiB.
    const int64_t f_max = std::max<int64_t>(1, std::min<int64_t>((int64_t)(256ll << 20) / (4 * n), 4096));
    const int64_t F = std::min<int64_t>(nf, f_max);
    const size_t cb = round_up(F * cpad, 256), nb = round_up(F * 4, 256), db_ = round_up(F * n * 4, 256),
                 lb = round_up(F * pool * 4, 256);
    void* ws;
    VA_TRY(va_workspace(ctx, cb + nb + db_ + 2 * lb, &ws));
    int8_t* qc = (int8_t*)ws;
    int* qn = (int*)((uint8_t*)ws + cb);
    float* dist = (float*)((uint8_t*)qn + nb);
    float* cv = (float*)((uint8_t*)dist + db_);
    uint32_t* ci = (uint32_t*)((uint8_t*)cv + lb);
    const size_t smem = (size_t)SCAN_Q * cpad;
    if (smem > 48 * 1024)
        VA_CUDA_TRY(cudaFuncSetAttribute(k_int8_scan, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    for (int64_t c0 = 0; c0 < nf; c0 += F) {
        const int f = (int)std::min<int64_t>(F, nf - c0);
        const float* q = gq + c0 * dim;
        k_perdim_codes<<<warps_grid(f), 256, 0, ctx->stream>>>(q, f, f, dim, cpad, db->sq_mins, db->sq_scales, qc, qn);
        VA_TRY(va_check_launch("k_perdim_codes(fallback)"));
        dim3 grid((unsigned)std::min<int64_t>((n + 255) / 256, (int64_t)ctx->sm_count * 8), (unsigned)((f + SCAN_Q - 1) / SCAN_Q));
        k_int8_scan<<<grid, 256, smem, ctx->stream>>>(qc, qn, f, db->codes, db->code_norms, n, cpad, dist);
        VA_TRY(va_check_launch("k_int8_scan"));
        VA_TRY(va_topk_select(ctx, dist, f, n, n, pool, VA_SELECT_MIN, cv, ci, pool));
        TcPlan one = {};
        one.splits = 1;
        one.nq_pad = f;
        one.kp = pool;
        VA_TRY(va_merge_rerank_internal(ctx, db, q, f, k, VA_METRIC_L2SQ, one, cv, ci, nullptr, gv + c0 * k,
                                        gi + c0 * k, pool, nullptr, nullptr));
    }
    k_scatter_rows<<<grid_for((int64_t)nf * k), 256, 0, ctx->stream>>>(gv, gi, fail_list, nf, k, out_vals, out_ids);
    return va_check_launch("k_scatter_rows");
}

int alloc_int_db(va_context* ctx, va_database* db, int64_t n, int cpad) {
    const int64_t n_pad = round_up(n, 256);
    cudaError_t e = cudaMalloc((void**)&db->codes, (size_t)n * cpad);
    if (e == cudaSuccess) e = cudaMalloc((void**)&db->code_norms, (size_t)n_pad * 4);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return va_set_error(VA_ERR_OOM, "code allocation (%zu bytes) failed: %s", (size_t)n * cpad,
                            cudaGetErrorString(e));
    }
    VA_CUDA_TRY(cudaMemsetAsync(db->code_norms, 0, (size_t)n_pad * 4, ctx->stream));
    return VA_OK;
}

}  // namespace

namespace {

// Filter + list merge of nq expanded queries over one database view; results [nq x k] as distance
// bit patterns and view-local ids.
int hamming_view(va_context* ctx, const va_database* view, const uint32_t* queries, int64_t nq, int k, float* out_v,
                 uint32_t* out_i) {
    TcPlan plan;
    VA_TRY(va_tc_plan_pool(ctx, nq, view->n, k, &plan, view->cpad));
    IntScratch s;
    VA_TRY(int_scratch(ctx, view, plan, &s));
    k_expand_bits<<<warps_grid(plan.nq_pad), 256, 0, ctx->stream>>>(queries, nq, plan.nq_pad, view->words, view->cpad,
                                                                    s.q_codes, s.q_norms);
    VA_TRY(va_check_launch("k_expand_bits(queries)"));
    VA_TRY(run_int_filter(ctx, view, plan, s));
    return va_merge_lists_internal(ctx, s.part_keys, s.part_ids, plan.splits, plan.nq_pad * plan.kp, plan.kp, nq, k,
                                   VA_SELECT_MIN, out_v, out_i);
}

// Chunked route: expand rows [r0, r0 + stage_rows) into the staging buffer, search them, keep
// each chunk's k best (global ids), merge the chunks' lists.
int hamming_chunked(va_context* ctx, va_database* db, const uint32_t* queries, int64_t nq, int k, uint32_t* out_dists,
                    uint32_t* out_ids) {
    const int64_t n = db->n, cr = db->stage_rows;
    const int64_t nch = (n + cr - 1) / cr;
    const size_t lb = (size_t)nch * nq * k;
    void* aux;
    VA_TRY(va_aux_buffer(ctx, lb * 8 + (size_t)nq * k * 4 + 512, &aux));
    float* cv = (float*)aux;
    uint32_t* ci = (uint32_t*)(cv + lb);
    float* mv = (float*)(ci + lb);
    const int blocks = std::max(1, (int)std::min<int64_t>((nq * k + 255) / 256, 4096));
    const bool prof = ctx->prof_ev && ctx->prof_n < ctx->prof_cap;
    VA_CUDA_TRY(cudaEventRecord(prof ? ctx->prof_ev[2 * ctx->prof_n] : ctx->ev_k0, ctx->stream));
    for (int64_t c = 0; c < nch; ++c) {
        const int64_t r0 = c * cr, rows = std::min(cr, n - r0);
        k_expand_bits<<<warps_grid(rows), 256, 0, ctx->stream>>>((const uint32_t*)db->rows + r0 * db->words, rows,
                                                                rows, db->words, db->cpad, db->stage, db->stage_norms);
        VA_TRY(va_check_launch("k_expand_bits(chunk)"));
        va_database view = *db;
        view.codes = db->stage;
        view.code_norms = db->stage_norms;
        view.n = rows;
        view.id_base = 0;
        float* v = cv + (size_t)c * nq * k;
        uint32_t* ids = ci + (size_t)c * nq * k;
        VA_TRY(hamming_view(ctx, &view, queries, nq, k, v, ids));
        if (r0) k_add_base_ids<<<blocks, 256, 0, ctx->stream>>>(ids, nq * k, (uint32_t)r0);
    }
    VA_CUDA_TRY(cudaEventRecord(prof ? ctx->prof_ev[2 * ctx->prof_n + 1] : ctx->ev_k1, ctx->stream));
    if (prof)
        ctx->prof_n++;
    else
        ctx->k_recorded = true;
    VA_TRY(va_merge_lists_internal(ctx, cv, ci, (int)nch, nq * k, k, nq, k, VA_SELECT_MIN, mv, out_ids));
    if (out_dists) k_bits_to_dists<<<blocks, 256, 0, ctx->stream>>>(mv, out_ids, nq * k, out_dists);
    if (db->id_base) k_add_base_ids<<<blocks, 256, 0, ctx->stream>>>(out_ids, nq * k, db->id_base);
    return va_check_launch("k_bits_to_dists");
}

}  // namespace

// Integer codes of rows [r0, r0 + count): per-dimension codes and |code|^2 of an int8 database,
// or the 0/1 expansion and popcounts of a binary database whose expansion is resident. Used by
// ingestion after rows were written.
int va_db_derive_codes(va_context* ctx, va_database* db, int64_t r0, int64_t count) {
    if (count <= 0) return VA_OK;
    if (db->kind == VA_DB_INT8) {
        k_perdim_codes<<<warps_grid(count), 256, 0, ctx->stream>>>((const float*)db->rows + r0 * db->dim, count, count,
                                                                  db->dim, db->cpad, db->sq_mins, db->sq_scales,
                                                                  db->codes + r0 * db->cpad, db->code_norms + r0);
        return va_check_launch("k_perdim_codes(append)");
    }
    if (db->kind == VA_DB_BINARY && db->codes) {
        k_expand_bits<<<warps_grid(count), 256, 0, ctx->stream>>>((const uint32_t*)db->rows + r0 * db->words, count,
                                                                 count, db->words, db->cpad, db->codes + r0 * db->cpad,
                                                                 db->code_norms + r0);
        return va_check_launch("k_expand_bits(append)");
    }
    return VA_OK;
}

extern "C" {

int va_sq_perdim_minmax(va_context* ctx, const float* x, int64_t n, int dim, float* out_min, float* out_max) {
    VA_REQUIRE(ctx && x && out_min && out_max, "ctx, x, out_min and out_max must not be NULL");
    VA_REQUIRE(n > 0 && dim > 0, "n and dim must be positive");
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    void* ws;
    VA_TRY(va_workspace(ctx, (size_t)dim * 8, &ws));
    unsigned* kmin = (unsigned*)ws;
    unsigned* kmax = kmin + dim;
    k_init_keys<<<std::max(1, (dim + 255) / 256), 256, 0, ctx->stream>>>(kmin, kmax, dim);
    dim3 grid((unsigned)((dim + 31) / 32), (unsigned)std::min<int64_t>((n + 7) / 8, 2048));
    k_col_minmax<<<grid, 256, 0, ctx->stream>>>(x, n, dim, kmin, kmax);
    k_keys_to_minmax<<<std::max(1, (dim + 255) / 256), 256, 0, ctx->stream>>>(kmin, kmax, dim, out_min, out_max);
    return va_check_launch("k_col_minmax");
}

int va_db_create_int8(va_context* ctx, const float* rows, int on_device, int64_t n, int dim, const float* mins,
                      const float* maxs, uint32_t id_base, va_database** out) {
    VaRange nvtx_range("va_db_create_int8");
    VA_REQUIRE(ctx && rows && out, "ctx, rows and out must not be NULL");
    VA_REQUIRE(n > 0, "numDataset must be positive, got %lld", (long long)n);
    VA_REQUIRE(dim > 0, "dimension must be positive, got %d", dim);
    VA_REQUIRE(dim <= VA_MAX_DIM, "dimension %d exceeds maximum supported dimension %d", dim, VA_MAX_DIM);
    VA_REQUIRE((mins == nullptr) == (maxs == nullptr), "mins and maxs must be both given or both NULL");
    VA_REQUIRE((uint64_t)n + id_base <= 0xFFFFFFFFull, "numDataset + id_base exceeds the uint32 id range");
    *out = nullptr;
    va_database* db = nullptr;
    VA_TRY(db_create_impl(ctx, rows, on_device, n, dim, VA_DTYPE_F32, id_base, &db, false));
    db->kind = VA_DB_INT8;
    db->cpad = (int)round_up(dim, CBLOCK);
    int s = alloc_int_db(ctx, db, n, db->cpad);
    if (s == VA_OK && (cudaMalloc((void**)&db->sq_mins, (size_t)dim * 4) != cudaSuccess ||
                       cudaMalloc((void**)&db->sq_scales, (size_t)dim * 4) != cudaSuccess)) {
        cudaGetLastError();
        s = va_set_error(VA_ERR_OOM, "parameter allocation failed");
    }
    if (s == VA_OK) {
        if (mins) {
            k_minmax_to_params<<<std::max(1, (dim + 255) / 256), 256, 0, ctx->stream>>>(mins, maxs, dim, db->sq_mins,
                                                                                       db->sq_scales);
            s = va_check_launch("k_minmax_to_params");
        } else {
            s = va_sq_perdim_minmax(ctx, (const float*)db->rows, n, dim, db->sq_mins, db->sq_scales);
            if (s == VA_OK) {
                k_minmax_to_params<<<std::max(1, (dim + 255) / 256), 256, 0, ctx->stream>>>(
                    db->sq_mins, db->sq_scales, dim, db->sq_mins, db->sq_scales);
                s = va_check_launch("k_minmax_to_params");
            }
        }
    }
    if (s == VA_OK) {
        k_perdim_codes<<<warps_grid(n), 256, 0, ctx->stream>>>((const float*)db->rows, n, n, dim, db->cpad,
                                                              db->sq_mins, db->sq_scales, db->codes, db->code_norms);
        s = va_check_launch("k_perdim_codes");
    }
    if (s != VA_OK) {
        va_db_destroy(db);
        return s;
    }
    *out = db;
    return VA_OK;
}

int va_db_int8_params(const va_database* db, const float** mins, const float** scales, const int8_t** codes,
                      int* code_stride) {
    VA_REQUIRE(db, "db must not be NULL");
    VA_REQUIRE(db->kind == VA_DB_INT8, "database is not an int8 database");
    if (mins) *mins = db->sq_mins;
    if (scales) *scales = db->sq_scales;
    if (codes) *codes = db->codes;
    if (code_stride) *code_stride = db->cpad;
    return VA_OK;
}

int va_int8_knn_search(va_context* ctx, const va_database* cdb, const float* queries, int64_t nq, int k, int candidates,
                       float* out_vals, uint32_t* out_ids) {
    VaRange nvtx_range("va_int8_knn_search");
    VA_REQUIRE(ctx && cdb && queries && out_vals && out_ids, "all pointers must be non-NULL");
    if (va_is_sharded(cdb)) return va_sharded_int8(ctx, cdb, queries, nq, k, candidates, out_vals, out_ids);
    return va_int8_knn_local(ctx, cdb, queries, nq, k, candidates, out_vals, out_ids);
}

}  // extern "C"

int va_int8_knn_local(va_context* ctx, const va_database* cdb, const float* queries, int64_t nq, int k, int candidates,
                      float* out_vals, uint32_t* out_ids) {
    VA_REQUIRE(ctx && cdb && queries && out_vals && out_ids, "all pointers must be non-NULL");
    VA_REQUIRE(cdb->kind == VA_DB_INT8, "database is not an int8 database (use va_db_create_int8)");
    VA_REQUIRE(nq > 0, "numQueries must be positive, got %lld", (long long)nq);
    VA_REQUIRE(k > 0, "k must be positive, got %d", k);
    VA_REQUIRE(candidates >= k, "candidates %d must be >= k %d", candidates, k);
    VA_REQUIRE(candidates <= VA_MAX_SELECT_K, "candidates %d exceeds the maximum of %d", candidates, VA_MAX_SELECT_K);
    VA_REQUIRE(k <= VA_MAX_K, "k %d exceeds maximum supported k %d", k, VA_MAX_K);
    // Up to 128 candidates: lists of that size sharing a per-query bound. More: 128-entry lists
    // without a shared bound, the pool proven from their union per query, the rest scanned exactly.
    const bool wide = candidates > 128;
    va_database* db = const_cast<va_database*>(cdb);
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    TcPlan plan;
    VA_TRY(va_tc_plan_pool(ctx, nq, db->n, candidates, &plan, db->cpad));
    IntScratch s;
    VA_TRY(int_scratch(ctx, db, plan, &s));
    uint32_t *fail_cnt = nullptr, *fail_list = nullptr, *gi = nullptr;
    float *gq = nullptr, *gv = nullptr;
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
    k_perdim_codes<<<warps_grid(plan.nq_pad), 256, 0, ctx->stream>>>(queries, nq, plan.nq_pad, db->dim, db->cpad,
                                                                     db->sq_mins, db->sq_scales, s.q_codes, s.q_norms);
    VA_TRY(va_check_launch("k_perdim_codes(queries)"));
    const bool prof = ctx->prof_ev && ctx->prof_n < ctx->prof_cap;
    VA_CUDA_TRY(cudaEventRecord(prof ? ctx->prof_ev[2 * ctx->prof_n] : ctx->ev_k0, ctx->stream));
    VA_TRY(run_int_filter(ctx, db, plan, s));
    VA_CUDA_TRY(cudaEventRecord(prof ? ctx->prof_ev[2 * ctx->prof_n + 1] : ctx->ev_k1, ctx->stream));
    if (prof)
        ctx->prof_n++;
    else
        ctx->k_recorded = true;
    VA_TRY(va_merge_rerank_internal(ctx, db, queries, nq, k, VA_METRIC_L2SQ, plan, s.part_keys, s.part_ids, s.gthr,
                                    out_vals, out_ids, candidates, fail_list, fail_cnt));
    if (!wide) return VA_OK;
    return int8_fallback(ctx, db, queries, k, candidates, fail_list, fail_cnt, gq, gv, gi, out_vals, out_ids);
}

extern "C" {

int va_db_create_binary(va_context* ctx, const uint32_t* codes, int on_device, int64_t n, int dim_bits,
                        uint32_t id_base, va_database** out) {
    VaRange nvtx_range("va_db_create_binary");
    VA_REQUIRE(ctx && codes && out, "ctx, codes and out must not be NULL");
    VA_REQUIRE(n > 0, "numDataset must be positive, got %lld", (long long)n);
    VA_REQUIRE(dim_bits > 0 && dim_bits <= 8192, "dimension must be in 1..8192 bits, got %d", dim_bits);
    VA_REQUIRE((uint64_t)n + id_base <= 0xFFFFFFFFull, "numDataset + id_base exceeds the uint32 id range");
    *out = nullptr;
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    va_database* db = new va_database();
    db->ctx = ctx;
    db->n = n;
    db->dim = dim_bits;
    db->dtype = VA_DTYPE_F32;
    db->id_base = id_base;
    db->kind = VA_DB_BINARY;
    db->words = (dim_bits + 31) / 32;
    db->cpad = (int)round_up((int64_t)db->words * 32, CBLOCK);
    const size_t pbytes = (size_t)n * db->words * 4;
    cudaError_t e = cudaMalloc(&db->rows, pbytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        delete db;
        return va_set_error(VA_ERR_OOM, "code allocation (%zu bytes) failed", pbytes);
    }
    int s = VA_OK;
    e = cudaMemcpyAsync(db->rows, codes, pbytes, on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                        ctx->stream);
    if (e != cudaSuccess) s = va_set_error(VA_ERR_CUDA, "code upload failed: %s", cudaGetErrorString(e));
    if (s != VA_OK) {
        va_db_destroy(db);
        return s;
    }
    *out = db;
    return VA_OK;
}

int va_db_binary_set_chunk_rows(va_database* db, int64_t rows) {
    VA_REQUIRE(db, "db must not be NULL");
    VA_REQUIRE(db->kind == VA_DB_BINARY, "database is not a binary database");
    VA_REQUIRE(rows >= 0, "rows must be >= 0, got %lld", (long long)rows);
    VA_REQUIRE(!db->codes && !db->stage, "the expansion of this database is already built");
    db->chunk_request = rows ? std::max<int64_t>(256, rows / 256 * 256) : 0;
    return VA_OK;
}

int va_hamming_knn_db(va_context* ctx, const va_database* cdb, const uint32_t* queries, int64_t nq, int k,
                      uint32_t* out_dists, uint32_t* out_ids) {
    VaRange nvtx_range("va_hamming_knn_db");
    VA_REQUIRE(ctx && cdb && queries && out_ids, "ctx, db, queries and out_ids must not be NULL");
    if (va_is_sharded(cdb)) return va_sharded_hamming(ctx, cdb, queries, nq, k, out_dists, out_ids);
    return va_hamming_knn_local(ctx, cdb, queries, nq, k, out_dists, out_ids);
}

}  // extern "C"

int va_hamming_knn_local(va_context* ctx, const va_database* cdb, const uint32_t* queries, int64_t nq, int k,
                         uint32_t* out_dists, uint32_t* out_ids) {
    VA_REQUIRE(ctx && cdb && queries && out_ids, "ctx, db, queries and out_ids must not be NULL");
    VA_REQUIRE(cdb->kind == VA_DB_BINARY, "database is not a binary database (use va_db_create_binary)");
    VA_REQUIRE(nq > 0, "numQueries must be positive, got %lld", (long long)nq);
    VA_REQUIRE(k > 0 && k <= 128, "k must be between 1 and 128 for the binary search, got %d", k);
    va_database* db = const_cast<va_database*>(cdb);
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    const int blocks = std::max(1, (int)std::min<int64_t>((nq * k + 255) / 256, 4096));
    if (hscan_supported(db->words, nq)) {
        // Small batch: one HBM-bound pass over the packed codes.
        const int64_t n = db->n;
        int grid = ctx->sm_count * 3;
        int64_t rpc = (n + grid - 1) / grid;
        rpc = round_up(rpc, 256);
        grid = (int)((n + rpc - 1) / rpc);
        const size_t part = (size_t)grid * nq * k;
        void* ws;
        VA_TRY(va_workspace(ctx, part * 8 + 256, &ws));
        float* pv = (float*)ws;
        uint32_t* pi = (uint32_t*)(pv + part);
        void* ws2;
        VA_TRY(va_aux_buffer(ctx, (size_t)nq * k * 4 + 256, &ws2));
        float* mv = (float*)ws2;
        const uint32_t* x = (const uint32_t*)db->rows;
        const int qn = (int)nq;
        const bool prof = ctx->prof_ev && ctx->prof_n < ctx->prof_cap;
        VA_CUDA_TRY(cudaEventRecord(prof ? ctx->prof_ev[2 * ctx->prof_n] : ctx->ev_k0, ctx->stream));
        int st;
        switch (db->words) {
            case 4: st = dispatch_hscan<4>(ctx, x, n, queries, qn, k, grid, rpc, pv, pi); break;
            case 8: st = dispatch_hscan<8>(ctx, x, n, queries, qn, k, grid, rpc, pv, pi); break;
            case 16: st = dispatch_hscan<16>(ctx, x, n, queries, qn, k, grid, rpc, pv, pi); break;
            default: st = dispatch_hscan<32>(ctx, x, n, queries, qn, k, grid, rpc, pv, pi); break;
        }
        VA_TRY(st);
        VA_CUDA_TRY(cudaEventRecord(prof ? ctx->prof_ev[2 * ctx->prof_n + 1] : ctx->ev_k1, ctx->stream));
        if (prof)
            ctx->prof_n++;
        else
            ctx->k_recorded = true;
        VA_TRY(va_merge_lists_internal(ctx, pv, pi, grid, nq * k, k, nq, k, VA_SELECT_MIN, mv, out_ids));
        if (out_dists) k_bits_to_dists<<<blocks, 256, 0, ctx->stream>>>(mv, out_ids, nq * k, out_dists);
        if (db->id_base) k_add_base_ids<<<blocks, 256, 0, ctx->stream>>>(out_ids, nq * k, db->id_base);
        return va_check_launch("k_bits_to_dists");
    }
    // Batches: the 0/1 expansion of the codes on the integer tensor cores. It is built once, on
    // first use, when it fits in 60% of the free device memory; otherwise (or when the caller set
    // a chunk size) chunks of rows are expanded and searched one at a time.
    if (!db->codes && !db->stage) {
        size_t free_b = 0, total_b = 0;
        VA_CUDA_TRY(cudaMemGetInfo(&free_b, &total_b));
        const double need = (double)db->n * db->cpad + (double)round_up(db->n, 256) * 4;
        if (!db->chunk_request && need <= 0.6 * (double)free_b) {
            VA_TRY(alloc_int_db(ctx, db, db->n, db->cpad));
            k_expand_bits<<<warps_grid(db->n), 256, 0, ctx->stream>>>((const uint32_t*)db->rows, db->n, db->n,
                                                                     db->words, db->cpad, db->codes, db->code_norms);
            VA_TRY(va_check_launch("k_expand_bits"));
        } else {
            int64_t rows = db->chunk_request ? db->chunk_request
                                             : (int64_t)(0.5 * (double)free_b / (double)(db->cpad + 4)) / 256 * 256;
            rows = std::min<int64_t>(std::max<int64_t>(rows, 256), db->n);
            cudaError_t e = cudaMalloc((void**)&db->stage, (size_t)rows * db->cpad);
            if (e == cudaSuccess) e = cudaMalloc((void**)&db->stage_norms, (size_t)round_up(rows, 256) * 4);
            if (e != cudaSuccess) {
                cudaGetLastError();
                if (db->stage) cudaFree(db->stage);
                db->stage = nullptr;
                return va_set_error(VA_ERR_OOM, "staging for %lld expanded rows failed: %s", (long long)rows,
                                    cudaGetErrorString(e));
            }
            VA_CUDA_TRY(cudaMemsetAsync(db->stage_norms, 0, (size_t)round_up(rows, 256) * 4, ctx->stream));
            db->stage_rows = rows;
        }
    }
    if (!db->codes) return hamming_chunked(ctx, db, queries, nq, k, out_dists, out_ids);
    TcPlan plan;
    VA_TRY(va_tc_plan_pool(ctx, nq, db->n, k, &plan, db->cpad));
    IntScratch s;
    VA_TRY(int_scratch(ctx, db, plan, &s));
    void* ws2;
    const size_t extra = (size_t)nq * k * 8;
    VA_TRY(va_aux_buffer(ctx, extra + 256, &ws2));
    float* mv = (float*)ws2;
    k_expand_bits<<<warps_grid(plan.nq_pad), 256, 0, ctx->stream>>>(queries, nq, plan.nq_pad, db->words, db->cpad,
                                                                    s.q_codes, s.q_norms);
    VA_TRY(va_check_launch("k_expand_bits(queries)"));
    const bool prof = ctx->prof_ev && ctx->prof_n < ctx->prof_cap;
    VA_CUDA_TRY(cudaEventRecord(prof ? ctx->prof_ev[2 * ctx->prof_n] : ctx->ev_k0, ctx->stream));
    VA_TRY(run_int_filter(ctx, db, plan, s));
    VA_CUDA_TRY(cudaEventRecord(prof ? ctx->prof_ev[2 * ctx->prof_n + 1] : ctx->ev_k1, ctx->stream));
    if (prof)
        ctx->prof_n++;
    else
        ctx->k_recorded = true;
    VA_TRY(va_merge_lists_internal(ctx, s.part_keys, s.part_ids, plan.splits, plan.nq_pad * plan.kp, plan.kp, nq, k,
                                   VA_SELECT_MIN, mv, out_ids));
    if (out_dists) k_bits_to_dists<<<blocks, 256, 0, ctx->stream>>>(mv, out_ids, nq * k, out_dists);
    if (db->id_base) k_add_base_ids<<<blocks, 256, 0, ctx->stream>>>(out_ids, nq * k, db->id_base);
    return va_check_launch("k_bits_to_dists");
}
