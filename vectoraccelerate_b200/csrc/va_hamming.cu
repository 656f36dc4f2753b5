// va_hamming.cu -- Hamming distance matrix and fused Hamming k-NN over LSB-first packed codes.
//
// Matrix: hamming_distance_batch / _normalized (Metal/Shaders/HammingDistance.metal:28-127,
// 242-321): popcount(q ^ x) per uint32 word. Fused k-NN: replaces the reference's route of a
// materialised Q x N matrix followed by a CPU sort (Metal4HammingResult.nearestNeighbors,
// Kernels/Metal4/HammingDistanceKernel.swift:114-120) -- distances never reach HBM.
//
// Fused layout: one thread per query with its code in registers; database codes stream through
// shared memory (16-byte loads, broadcast reads); each thread keeps a sorted (distance, id)
// list of its k best in shared memory and only touches it when a candidate beats the current
// k-th best. Candidates arrive in increasing id order, so the strict comparison keeps the
// smaller id among equal distances. Work items are (query tile, database split); per-split
// lists are merged by the shared list-merge kernel.
#include <algorithm>

#include "va_internal.cuh"

namespace {

__global__ void k_hamming_matrix(const uint32_t* __restrict__ q, int64_t nq, const uint32_t* __restrict__ x,
                                 int64_t nx, int words, uint32_t* __restrict__ out, float* __restrict__ outn,
                                 float inv_dim) {
    // 16 x 16 tile like the reference; each thread one (query, row) pair.
    __shared__ uint32_t sq[16][65];
    __shared__ uint32_t sx[16][65];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int64_t qi = (int64_t)blockIdx.y * 16 + ty, xi = (int64_t)blockIdx.x * 16 + tx;
    uint32_t acc = 0;
    for (int w0 = 0; w0 < words; w0 += 64) {
        for (int e = threadIdx.x; e < 16 * 64; e += 256) {
            int r = e / 64, c = e % 64;
            int64_t gq = (int64_t)blockIdx.y * 16 + r, gx = (int64_t)blockIdx.x * 16 + r;
            sq[r][c] = (gq < nq && w0 + c < words) ? q[gq * words + w0 + c] : 0u;
            sx[r][c] = (gx < nx && w0 + c < words) ? x[gx * words + w0 + c] : 0u;
        }
        __syncthreads();
        int lim = min(64, words - w0);
        for (int c = 0; c < lim; ++c) acc += __popc(sq[ty][c] ^ sx[tx][c]);
        __syncthreads();
    }
    if (qi < nq && xi < nx) {
        out[qi * nx + xi] = acc;
        if (outn) outn[qi * nx + xi] = (float)acc * inv_dim;
    }
}

constexpr int HQ = 128;   // queries per block (one per thread)
constexpr int HT = 128;   // database codes per shared-memory tile

template <int WORDS>
__global__ void __launch_bounds__(HQ) k_hamming_knn(const uint32_t* __restrict__ q, int64_t nq,
                                                    const uint32_t* __restrict__ x, int64_t nx, int k,
                                                    int n_qtiles, int64_t rows_per_split, float* __restrict__ part_vals,
                                                    uint32_t* __restrict__ part_ids, int64_t nq_pad) {
    extern __shared__ uint8_t smem[];
    uint32_t* s_codes = (uint32_t*)smem;                          // [HT][WORDS]
    uint32_t* s_lk = s_codes + HT * WORDS;                        // [k][HQ] distances
    uint32_t* s_li = s_lk + (size_t)k * HQ;                       // [k][HQ] ids
    const int item = blockIdx.x;
    const int qt = item % n_qtiles, split = item / n_qtiles;
    const int t = threadIdx.x;
    const int64_t qi = (int64_t)qt * HQ + t;
    uint32_t qc[WORDS];
#pragma unroll
    for (int w = 0; w < WORDS; ++w) qc[w] = qi < nq ? q[qi * WORDS + w] : 0u;
    for (int j = 0; j < k; ++j) {
        s_lk[j * HQ + t] = 0xFFFFFFFFu;
        s_li[j * HQ + t] = va::kInvalidId;
    }
    uint32_t thr = 0xFFFFFFFFu;
    const int64_t r0 = (int64_t)split * rows_per_split;
    const int64_t r1 = std::min<int64_t>(nx, r0 + rows_per_split);
    for (int64_t base = r0; base < r1; base += HT) {
        const int cnt = (int)std::min<int64_t>(HT, r1 - base);
        __syncthreads();
        const uint32_t* src = x + base * WORDS;
        const int nwords = cnt * WORDS;
        for (int e = t; e < nwords; e += HQ) s_codes[e] = __ldg(src + e);
        __syncthreads();
        for (int c = 0; c < cnt; ++c) {
            uint32_t d = 0;
            if constexpr (WORDS >= 4) {
                const uint4* code = (const uint4*)(s_codes + c * WORDS);
#pragma unroll
                for (int v = 0; v < WORDS / 4; ++v) {
                    uint4 u = code[v];
                    d += __popc(qc[4 * v] ^ u.x) + __popc(qc[4 * v + 1] ^ u.y) + __popc(qc[4 * v + 2] ^ u.z) +
                         __popc(qc[4 * v + 3] ^ u.w);
                }
            } else {
#pragma unroll
                for (int v = 0; v < WORDS; ++v) d += __popc(qc[v] ^ s_codes[c * WORDS + v]);
            }
            if (d < thr) {
                const uint32_t id = (uint32_t)(base + c);
                int p = k - 1;
                while (p > 0 && s_lk[(p - 1) * HQ + t] > d) {
                    s_lk[p * HQ + t] = s_lk[(p - 1) * HQ + t];
                    s_li[p * HQ + t] = s_li[(p - 1) * HQ + t];
                    --p;
                }
                s_lk[p * HQ + t] = d;
                s_li[p * HQ + t] = id;
                thr = s_lk[(k - 1) * HQ + t];
            }
        }
    }
    if (qi < nq) {
        float* pv = part_vals + ((int64_t)split * nq_pad + qi) * k;
        uint32_t* pi = part_ids + ((int64_t)split * nq_pad + qi) * k;
        for (int j = 0; j < k; ++j) {
            uint32_t id = s_li[j * HQ + t];
            pv[j] = id == va::kInvalidId ? INFINITY : (float)s_lk[j * HQ + t];
            pi[j] = id;
        }
    }
}

__global__ void k_vals_to_u32(const float* __restrict__ v, int64_t n, uint32_t* __restrict__ out) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        float f = v[i];
        out[i] = isinf(f) ? 0xFFFFFFFFu : (uint32_t)f;
    }
}

template <int W>
int launch_hknn(va_context* ctx, const uint32_t* q, int64_t nq, const uint32_t* x, int64_t nx, int k, int n_qtiles,
                int splits, int64_t rows_per_split, float* pv, uint32_t* pi, size_t smem) {
    VA_CUDA_TRY(cudaFuncSetAttribute(k_hamming_knn<W>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    k_hamming_knn<W><<<n_qtiles * splits, HQ, smem, ctx->stream>>>(q, nq, x, nx, k, n_qtiles, rows_per_split, pv, pi,
                                                                  nq);
    return va_check_launch("k_hamming_knn");
}

}  // namespace

extern "C" int va_merge_lists_internal(va_context* ctx, const float* vals, const uint32_t* ids, int nlists,
                                       int64_t list_stride, int len, int64_t nq, int k, int mode, float* out_vals,
                                       uint32_t* out_ids);

extern "C" {

int va_hamming_matrix(va_context* ctx, const uint32_t* q, int64_t nq, const uint32_t* x, int64_t nx, int words,
                      uint32_t* out, float* out_normalized, int dim) {
    VA_REQUIRE(ctx && q && x && out, "ctx, q, x and out must not be NULL");
    VA_REQUIRE(words > 0, "words must be positive, got %d", words);
    VA_REQUIRE(nq >= 0 && nx >= 0, "nq and nx must be >= 0");
    if (!nq || !nx) return VA_OK;
    VA_REQUIRE((nq + 15) / 16 <= 65535, "nq %lld too large for one matrix call", (long long)nq);
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    dim3 grid((unsigned)((nx + 15) / 16), (unsigned)((nq + 15) / 16));
    float inv = dim > 0 ? 1.0f / (float)dim : 1.0f / (float)(words * 32);
    k_hamming_matrix<<<grid, 256, 0, ctx->stream>>>(q, nq, x, nx, words, out, out_normalized, inv);
    return va_check_launch("k_hamming_matrix");
}

int va_hamming_knn(va_context* ctx, const uint32_t* q, int64_t nq, const uint32_t* x, int64_t nx, int words, int k,
                   uint32_t* out_dists, uint32_t* out_ids) {
    VA_REQUIRE(ctx && q && x && out_ids, "ctx, q, x and out_ids must not be NULL");
    VA_REQUIRE(words == 1 || words == 2 || words == 4 || words == 8 || words == 16 || words == 32,
               "words must be 1, 2, 4, 8, 16 or 32 (dimension 32..1024), got %d", words);
    VA_REQUIRE(k > 0 && k <= 128, "k must be between 1 and 128 for the fused Hamming search, got %d", k);
    VA_REQUIRE(nq >= 0 && nx > 0, "nq must be >= 0 and nx > 0");
    VA_REQUIRE(nx <= 0xFFFFFFFFll, "nx %lld exceeds the uint32 id range", (long long)nx);
    if (!nq) return VA_OK;
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    const int n_qtiles = (int)((nq + HQ - 1) / HQ);
    // Enough (query tile, split) items to fill the SMs twice over, splits of >= 4 tiles each.
    int64_t max_splits = std::max<int64_t>(1, nx / (4 * HT));
    int splits = (int)std::min<int64_t>(max_splits, std::max<int64_t>(1, (2LL * ctx->sm_count + n_qtiles - 1) / n_qtiles));
    int64_t rows_per_split = (nx + splits - 1) / splits;
    rows_per_split = (rows_per_split + HT - 1) / HT * HT;
    splits = (int)((nx + rows_per_split - 1) / rows_per_split);
    size_t part = (size_t)splits * nq * k;
    size_t smem = (size_t)HT * words * 4 + (size_t)k * HQ * 8;
    VA_REQUIRE(smem <= 227 * 1024, "k %d too large for the fused Hamming search at %d words", k, words);
    void* ws;
    VA_TRY(va_workspace(ctx, part * 8 + (size_t)nq * k * 4 + 256, &ws));
    float* pv = (float*)ws;
    uint32_t* pi = (uint32_t*)(pv + part);
    float* mv = (float*)(pi + part);
    int s;
    switch (words) {
        case 1: s = launch_hknn<1>(ctx, q, nq, x, nx, k, n_qtiles, splits, rows_per_split, pv, pi, smem); break;
        case 2: s = launch_hknn<2>(ctx, q, nq, x, nx, k, n_qtiles, splits, rows_per_split, pv, pi, smem); break;
        case 4: s = launch_hknn<4>(ctx, q, nq, x, nx, k, n_qtiles, splits, rows_per_split, pv, pi, smem); break;
        case 8: s = launch_hknn<8>(ctx, q, nq, x, nx, k, n_qtiles, splits, rows_per_split, pv, pi, smem); break;
        case 16: s = launch_hknn<16>(ctx, q, nq, x, nx, k, n_qtiles, splits, rows_per_split, pv, pi, smem); break;
        default: s = launch_hknn<32>(ctx, q, nq, x, nx, k, n_qtiles, splits, rows_per_split, pv, pi, smem); break;
    }
    VA_TRY(s);
    VA_TRY(va_merge_lists_internal(ctx, pv, pi, splits, (int64_t)nq * k, k, nq, k, VA_SELECT_MIN, mv, out_ids));
    if (out_dists) {
        k_vals_to_u32<<<std::max(1, (int)std::min<int64_t>((nq * k + 255) / 256, 4096)), 256, 0, ctx->stream>>>(
            mv, nq * k, out_dists);
        VA_TRY(va_check_launch("k_vals_to_u32"));
    }
    return VA_OK;
}

}  // extern "C"
