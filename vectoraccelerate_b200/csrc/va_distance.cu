// va_distance.cu -- fp32 distance primitives (exact SIMT arithmetic, no tensor cores).
//
// 1:1 pair kernels replace L2DistanceKernel / CosineSimilarityKernel (shaders l2_distance and
// cosine_similarity, DistanceShaders.metal:169-321). The all-pairs matrix replaces
// l2_distance_kernel (L2Distance.metal:34-91) and DotProductKernel (DotProduct.metal:29-432).
// L2 keeps the reference's direct form sum((q - x)^2) (L2Distance.metal:65-69), not the
// expanded |q|^2 + |x|^2 - 2 q.x, so near neighbours suffer no cancellation.
#include <cfloat>

#include "va_internal.cuh"

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

// One warp per pair.
__global__ void k_l2_pairs(const float* __restrict__ a, const float* __restrict__ b, int64_t pairs, int dim,
                           int compute_sqrt, float* __restrict__ out) {
    int64_t p = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (p >= pairs) return;
    const float* x = a + p * dim;
    const float* y = b + p * dim;
    float s = 0.f;
    for (int j = lane; j < dim; j += 32) {
        float t = x[j] - y[j];
        s = fmaf(t, t, s);
    }
    s = warp_sum(s);
    if (lane == 0) out[p] = compute_sqrt ? sqrtf(s) : s;
}

__global__ void k_cos_pairs(const float* __restrict__ a, const float* __restrict__ b, int64_t pairs, int dim,
                            int output_distance, float* __restrict__ out) {
    int64_t p = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (p >= pairs) return;
    const float* x = a + p * dim;
    const float* y = b + p * dim;
    float d = 0.f, aa = 0.f, bb = 0.f;
    for (int j = lane; j < dim; j += 32) {
        float u = x[j], v = y[j];
        d = fmaf(u, v, d);
        aa = fmaf(u, u, aa);
        bb = fmaf(v, v, bb);
    }
    d = warp_sum(d);
    aa = warp_sum(aa);
    bb = warp_sum(bb);
    if (lane == 0) {
        // DistanceShaders.metal:304-319: 0 below FLT_MIN, clamp to [-1, 1] keeping NaN.
        float den = sqrtf(aa) * sqrtf(bb);
        float sim = den < FLT_MIN ? 0.f : d / den;
        if (!(sim != sim)) sim = fminf(1.f, fmaxf(-1.f, sim));
        out[p] = output_distance ? 1.f - sim : sim;
    }
}

// Element of a row array: fp32, or bf16 bit patterns widened exactly.
__device__ __forceinline__ float ld_elem(const float* x, int64_t i) { return x[i]; }
__device__ __forceinline__ float ld_elem(const uint16_t* x, int64_t i) { return __uint_as_float((uint32_t)x[i] << 16); }

// Row norms |v| for the cosine matrix.
template <class XT>
__global__ void k_row_norms(const XT* __restrict__ x, int64_t rows, int dim, float* __restrict__ out) {
    int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (r >= rows) return;
    float s = 0.f;
    for (int j = lane; j < dim; j += 32) {
        float v = ld_elem(x, r * dim + j);
        s = fmaf(v, v, s);
    }
    s = warp_sum(s);
    if (lane == 0) out[r] = sqrtf(s);
}

// Tiled all-pairs matrix: 64 x 64 output tile per block, 256 threads, 4 x 4 outputs each,
// 32-wide dimension slices staged transposed in shared memory. Rows are fp32 or bf16 (XT).
constexpr int TM = 64, TN = 64, TK = 32;

template <int OP, class XT>  // OP 0 = squared L2 (direct form), 1 = dot
__global__ void __launch_bounds__(256) k_matrix(const float* __restrict__ q, int64_t nq, const XT* __restrict__ x,
                                                int64_t nx, int dim, int metric, int flag,
                                                const float* __restrict__ qn, const float* __restrict__ xn,
                                                float* __restrict__ out, int64_t out_stride) {
    __shared__ float sq[TK][TM + 4];
    __shared__ float sx[TK][TN + 4];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int64_t q0 = (int64_t)blockIdx.y * TM, x0 = (int64_t)blockIdx.x * TN;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < dim; k0 += TK) {
        for (int e = threadIdx.x; e < TM * TK; e += 256) {
            int r = e / TK, c = e % TK;
            int64_t gr = q0 + r;
            int gc = k0 + c;
            sq[c][r] = (gr < nq && gc < dim) ? q[gr * dim + gc] : 0.f;
            int64_t hr = x0 + r;
            sx[c][r] = (hr < nx && gc < dim) ? ld_elem(x, hr * dim + gc) : 0.f;
        }
        __syncthreads();
#pragma unroll 8
        for (int kk = 0; kk < TK; ++kk) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = sq[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = sx[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    if (OP == 0) {
                        float t = a[i] - b[j];
                        acc[i][j] = fmaf(t, t, acc[i][j]);
                    } else {
                        acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
                    }
                }
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        int64_t gr = q0 + ty * 4 + i;
        if (gr >= nq) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            int64_t gc = x0 + tx * 4 + j;
            if (gc >= nx) continue;
            float v = acc[i][j];
            if (metric == VA_METRIC_L2SQ) {
                if (flag) v = sqrtf(v);
            } else if (metric == VA_METRIC_IP) {
                if (flag) v = fabsf(v);
            } else {
                float den = qn[gr] * xn[gc];
                float sim = den < FLT_MIN ? 0.f : v / den;
                if (!(sim != sim)) sim = fminf(1.f, fmaxf(-1.f, sim));
                v = flag ? 1.f - sim : sim;
            }
            out[gr * out_stride + gc] = v;
        }
    }
}

}  // namespace

extern "C" {

int va_l2_distance_pairs(va_context* ctx, const float* a, const float* b, int64_t pairs, int dim, int compute_sqrt,
                         float* out) {
    VA_REQUIRE(ctx && a && b && out, "ctx, a, b and out must not be NULL");
    VA_REQUIRE(dim > 0, "dimension must be positive, got %d", dim);
    VA_REQUIRE(pairs >= 0, "pairs must be >= 0");
    if (!pairs) return VA_OK;
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    int64_t threads = pairs * 32;
    k_l2_pairs<<<(unsigned)((threads + 255) / 256), 256, 0, ctx->stream>>>(a, b, pairs, dim, compute_sqrt, out);
    return va_check_launch("k_l2_pairs");
}

int va_cosine_pairs(va_context* ctx, const float* a, const float* b, int64_t pairs, int dim, int output_distance,
                    float* out) {
    VA_REQUIRE(ctx && a && b && out, "ctx, a, b and out must not be NULL");
    VA_REQUIRE(dim > 0, "dimension must be positive, got %d", dim);
    VA_REQUIRE(pairs >= 0, "pairs must be >= 0");
    if (!pairs) return VA_OK;
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    int64_t threads = pairs * 32;
    k_cos_pairs<<<(unsigned)((threads + 255) / 256), 256, 0, ctx->stream>>>(a, b, pairs, dim, output_distance, out);
    return va_check_launch("k_cos_pairs");
}

}  // extern "C"

// Matrix with caller-provided norm scratch (nq + nx floats; used for cosine only), so internal
// callers can keep the context workspace for their own buffers. x_dtype: VA_DTYPE_F32 rows or
// VA_DTYPE_BF16 rows (widened exactly).
template <class XT>
int distance_matrix_t(va_context* ctx, const float* q, int64_t nq, const XT* x, int64_t nx, int dim, int metric,
                      int flag, float* out, int64_t out_stride, float* norm_scratch) {
    float *qn = nullptr, *xn = nullptr;
    if (metric == VA_METRIC_COSINE) {
        qn = norm_scratch;
        xn = qn + nq;
        k_row_norms<float><<<(unsigned)((nq * 32 + 255) / 256), 256, 0, ctx->stream>>>(q, nq, dim, qn);
        k_row_norms<XT><<<(unsigned)((nx * 32 + 255) / 256), 256, 0, ctx->stream>>>(x, nx, dim, xn);
        VA_TRY(va_check_launch("k_row_norms"));
    }
    dim3 grid((unsigned)((nx + TN - 1) / TN), (unsigned)((nq + TM - 1) / TM));
    if (metric == VA_METRIC_L2SQ)
        k_matrix<0, XT><<<grid, 256, 0, ctx->stream>>>(q, nq, x, nx, dim, metric, flag, qn, xn, out, out_stride);
    else
        k_matrix<1, XT><<<grid, 256, 0, ctx->stream>>>(q, nq, x, nx, dim, metric, flag, qn, xn, out, out_stride);
    return va_check_launch("k_matrix");
}

int va_distance_matrix_rows(va_context* ctx, const float* q, int64_t nq, const void* x, int x_dtype, int64_t nx,
                            int dim, int metric, int flag, float* out, int64_t out_stride, float* norm_scratch) {
    if (x_dtype == VA_DTYPE_BF16)
        return distance_matrix_t<uint16_t>(ctx, q, nq, (const uint16_t*)x, nx, dim, metric, flag, out, out_stride,
                                           norm_scratch);
    return distance_matrix_t<float>(ctx, q, nq, (const float*)x, nx, dim, metric, flag, out, out_stride,
                                    norm_scratch);
}

int va_distance_matrix_impl(va_context* ctx, const float* q, int64_t nq, const float* x, int64_t nx, int dim,
                            int metric, int flag, float* out, int64_t out_stride, float* norm_scratch) {
    return distance_matrix_t<float>(ctx, q, nq, x, nx, dim, metric, flag, out, out_stride, norm_scratch);
}

extern "C" {

int va_distance_matrix(va_context* ctx, const float* q, int64_t nq, const float* x, int64_t nx, int dim, int metric,
                       int flag, float* out, int64_t out_stride) {
    VaRange nvtx_range("va_distance_matrix");
    VA_REQUIRE(ctx && q && x && out, "ctx, q, x and out must not be NULL");
    VA_REQUIRE(dim > 0, "dimension must be positive, got %d", dim);
    VA_REQUIRE(metric >= 0 && metric <= 2, "metric must be 0 (L2SQ), 1 (COSINE) or 2 (IP), got %d", metric);
    VA_REQUIRE(nq >= 0 && nx >= 0, "nq and nx must be >= 0");
    VA_REQUIRE(out_stride >= nx, "out_stride %lld must be >= nx %lld", (long long)out_stride, (long long)nx);
    if (!nq || !nx) return VA_OK;
    VA_REQUIRE((nq + TM - 1) / TM <= 65535, "nq %lld too large for one matrix call", (long long)nq);
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    void* ws = nullptr;
    if (metric == VA_METRIC_COSINE) VA_TRY(va_workspace(ctx, (size_t)(nq + nx) * sizeof(float), &ws));
    return va_distance_matrix_impl(ctx, q, nq, x, nx, dim, metric, flag, out, out_stride, (float*)ws);
}

}  // extern "C"
