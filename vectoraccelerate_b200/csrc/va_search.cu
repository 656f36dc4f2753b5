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

int va_distance_matrix_rows(va_context* ctx, const float* q, int64_t nq, const void* x, int x_dtype, int64_t nx,
                            int dim, int metric, int flag, float* out, int64_t out_stride, float* norm_scratch);

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


// Filter row biases: norms2[r] = |x_r|^2 (fp64 accumulation rounded once) and zbias[r] = 0 for
// real rows; both +inf for the pad rows up to n_pad so padded tile columns never pass the
// filter. cert (optional) collects max |x_r| (rounded up) for the exactness certificate. One warp
// per row.
__global__ void k_row_bias(const void* rows, int dtype, int64_t n, int64_t n_pad, int dim, float* norms2,
                           float* zbias, uint32_t* cert) {
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
        if (cert && r < n) atomicMax(cert, __float_as_uint(__double2float_ru(sqrt(s))));
    }
}

// Certificate input of one operand kind: max over rows of |operand row - exact operand-space row|
// (rounded up), into cert[1 + kind]. Unit-norm kinds scale by 1/|x| in fp64 as k_operand does;
// zero rows stay zero (no error). One warp per row.
__global__ void k_operand_err(const void* rows, int dtype, int64_t n, int dim, int kind, uint32_t* cert) {
    int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (r >= n) return;
    double scale = 1.0;
    if (kind == VA_CERT_BF16_COS || kind == VA_CERT_TF32_COS) {
        double s = 0;
        for (int j = lane; j < dim; j += 32) {
            double v = load_row(rows, dtype, r * dim + j);
            s += v * v;
        }
        s = warp_sum_d(s);
        scale = s > 0 ? 1.0 / sqrt(s) : 0.0;
    }
    double e2 = 0;
    for (int j = lane; j < dim; j += 32) {
        double t, err;
        va::cert_elem(load_row(rows, dtype, r * dim + j), scale, kind, t, err);
        e2 += err * err;
    }
    e2 = warp_sum_d(e2);
    if (lane == 0) atomicMax(cert + 1 + kind, __float_as_uint(__double2float_ru(sqrt(e2) * (1.0 + 1e-12))));
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
            o[j] = va::f2bf_rn(v);
        else
            o[j] = v;
    }
}

// Per query: select the KP best approximate candidates over all splits, rerank exactly from the
// original rows, emit the top k sorted by (distance, id).
constexpr int MR_THREADS = 256;
constexpr int MR_POOL = 1024;  // candidates kept in shared memory after the bound test
constexpr int MR_VEC = 6;      // 16-byte row loads in flight per lane in the exact rerank

// Exactness certificate of one reduced-precision pass (see k_merge_rerank).
struct CertArgs {
    int on;                // 0: no certificate (exact integer keys)
    int kind;              // VA_CERT_* operand kind the filter multiplied
    int dpad;              // accumulated products per key (padded dimension)
    const uint32_t* cert;  // database maxima: [0] max |x|, [1 + kind] max operand error (float bits)
};

// The certificate. The filter orders rows by an approximate key K(y); the exact key is
//   D(y) = |y|^2 - 2 q.y (L2: distance - |q|^2),  -q.y (IP),  -cos(q, y) (cosine),
// which orders rows exactly as the reference's distance does. With a = q (or q/|q|), b = y (or
// y/|y|) and the tensor core's operands a~ = a + da, b~ = b + db:
//   a~.b~ - a.b = a~.db + da.b, so |a~.b~ - a.b| <= |a~| max|db| + |da| max|b|   (Cauchy-Schwarz)
//   |fp32 accumulation - a~.b~| <= g |a~| (max|b| + max|db|), g = dpad * 2^-22 (any summation
//       order, truncating adders: products of bf16 / tf32 values are exact in fp32)
//   plus the rounding of the key's fma and of the fp32 |y|^2 bias (2^-24 relative each).
// |da| and |a| come from this query; max|b| and max|db| are maxima over every row of the
// database (k_row_bias, k_operand_err). So |K(y) - D(y)| <= eps for every row y, including the
// rows the filter dropped. Every dropped row has K(y) >= T, the pool's largest approximate key
// (the pool is the exact top pool by (K, id): a list only drops keys at or above its last one,
// and the shared bound never cuts into the pool), hence D(y) >= T - eps. If the k-th exact key
// D_k (from the fp64 rerank, rounded up) satisfies D_k + eps < T, no dropped row can reach the
// top k: the result is the exact top k. Otherwise the query goes to the fail list.
__device__ __forceinline__ double cert_bound(const CertArgs& ca, int metric, float vk, double qn2, double a_norm,
                                            double a_err) {
    const double u24 = 5.9604644775390625e-08, u22 = 2.384185791015625e-07;
    double dk;  // upper bound of the k-th exact key
    if (metric == VA_METRIC_L2SQ)
        dk = (double)vk * (1.0 + 4.0 * u24) - qn2 * (1.0 - 1e-12);
    else if (metric == VA_METRIC_IP)
        dk = -(double)vk + fabs((double)vk) * 4.0 * u24 + 1e-30;
    else
        dk = (double)vk - 1.0 + 4.0 * u24;
    const double mx = (double)__uint_as_float(ca.cert[0]);
    const double md = (double)__uint_as_float(ca.cert[1 + ca.kind]);
    const double mb = metric == VA_METRIC_COSINE ? 1.0 : mx;
    const double A = a_norm + a_err;  // >= |a~|
    const double g = (double)ca.dpad * u22;
    double eps = A * md + a_err * mb + g * A * (mb + md);
    if (metric == VA_METRIC_L2SQ)
        eps = 2.0 * eps + u24 * (2.0 * A * (mb + md) * (1.0 + g) + mb * mb) + 2.0 * u24 * mb * mb;
    else
        eps += u24 * A * (mb + md) * (1.0 + g);
    eps = eps * (1.0 + 1e-6) + 1e-30;
    return dk + eps;
}

__global__ void __launch_bounds__(MR_THREADS, 3) k_merge_rerank(const float* __restrict__ part_keys,
                                                           const uint32_t* __restrict__ part_ids, int splits,
                                                           int64_t nq_pad, int kp, int pool_n,
                                                           const float* __restrict__ queries,
                                                           const void* __restrict__ rows, int dtype, int dim, int metric,
                                                           int k, uint32_t id_base, const uint32_t* __restrict__ gthr,
                                                           BoundLevels lv, int prove, CertArgs ca,
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
    __shared__ double s_qn, s_qn2, s_an, s_ae;
    __shared__ int s_cnt;
    __shared__ unsigned long long s_t;
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
    if (threadIdx.x == 0) {
        s_cnt = 0;
        s_t = 0;
    }
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
    // T: the pool's largest composite (~0 when the pool holds padding, i.e. every candidate).
    {
        unsigned long long t = 0;
        for (int i = threadIdx.x; i < m; i += blockDim.x) t = sel[i] > t ? sel[i] : t;
        if (m < pool_n) t = ~0ull;
        atomicMax(&s_t, t);
    }
    __syncthreads();
    const unsigned long long T = s_t;
    if (prove) {
        // Pool wider than the lists (kp < pool_n): the selection is the exact top pool_n by
        // (key, id) when every split's list holds all of its candidates up to T, i.e. when no full
        // list ends below T. Otherwise the query is handed to the fallback.
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
    if (warp == 0 && (metric == VA_METRIC_COSINE || ca.on)) {
        double s = 0;
        for (int j = lane; j < dim; j += 32) s += (double)sq[j] * sq[j];
        s = warp_sum_d(s);
        double an = 0, ae = 0;
        if (ca.on) {
            // |a| and a bound of |a~ - a| for this query's operand (same construction as k_operand)
            const double scale = metric == VA_METRIC_COSINE ? (s > 0 ? 1.0 / sqrt(s) : 0.0) : 1.0;
            for (int j = lane; j < dim; j += 32) {
                double t, err;
                va::cert_elem(sq[j], scale, ca.kind, t, err);
                an += t * t;
                ae += err * err;
            }
            an = warp_sum_d(an);
            ae = warp_sum_d(ae);
        }
        if (lane == 0) {
            s_qn2 = s;
            s_qn = sqrt(s);
            s_an = sqrt(an) * (1.0 + 1e-12);
            s_ae = sqrt(ae) * (1.0 + 1e-12);
        }
    }
    __syncthreads();
    const int mode = metric == VA_METRIC_IP ? 1 : 0;
    // Exact key of one candidate (warp-collective; every lane returns it).
    auto exact = [&](uint64_t comp) -> uint64_t {
        const uint32_t id = (uint32_t)comp;
        if (comp == ~0ull || id == va::kInvalidId) return ~0ull;
        const int64_t base = (int64_t)id * dim;
        double s = 0, xx = 0;
        if ((dim & 127) == 0) {
            // 16-byte (fp32) or 8-byte (bf16) loads of four consecutive elements per lane, issued
            // in batches of MR_VEC per lane before any of them is used: a row of up to
            // 128 * MR_VEC dimensions is one memory round trip (the gathered rows are
            // latency-bound, not bandwidth-bound).
            for (int j00 = 0; j00 < dim; j00 += 128 * MR_VEC) {
                float4 xv[MR_VEC];
#pragma unroll
                for (int v = 0; v < MR_VEC; ++v) {
                    const int j0 = j00 + 128 * v + lane * 4;
                    if (j0 < dim) {
                        if (dtype == VA_DTYPE_BF16) {
                            const uint2 u = __ldg((const uint2*)((const uint16_t*)rows + base + j0));
                            xv[v] = make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u),
                                                __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xFFFF0000u));
                        } else {
                            xv[v] = __ldg((const float4*)((const float*)rows + base + j0));
                        }
                    }
                }
#pragma unroll
                for (int v = 0; v < MR_VEC; ++v) {
                    const int j0 = j00 + 128 * v + lane * 4;
                    if (j0 >= dim) break;
                    const float4 qv = *(const float4*)(sq + j0);
                    const float qa[4] = {qv.x, qv.y, qv.z, qv.w}, xa[4] = {xv[v].x, xv[v].y, xv[v].z, xv[v].w};
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
        float v;
        if (metric == VA_METRIC_L2SQ || metric == VA_METRIC_IP) {
            v = (float)s;
        } else {
            double den = s_qn * sqrt(xx);
            double sim = den > 0 ? s / den : 0.0;
            sim = fmin(1.0, fmax(-1.0, sim));
            v = (float)(1.0 - sim);
        }
        return va::composite(va::mode_key(v, mode), id);
    };
    for (int c = warp; c < kp2; c += nwarps) {
        const uint64_t r = exact(c < m ? sel[c] : ~0ull);
        if (lane == 0) ex[c] = r;
    }
    va::block_bitonic_sort(ex, kp2);
    if (ca.on && T != ~0ull) {
        // The pool holds at least pool_n >= k valid candidates here, so ex[k - 1] is the k-th.
        __shared__ int s_ok, s_next;
        __shared__ double s_u;
        __shared__ unsigned s_lmin;
        if (threadIdx.x == 0) {
            const float vk = va::mode_val((uint32_t)(ex[k - 1] >> 32), mode);
            s_u = cert_bound(ca, metric, vk, s_qn2, s_an, s_ae);
            s_ok = s_u < (double)va::key2f((uint32_t)(T >> 32)) ? 1 : 0;
            s_lmin = 0xFFFFFFFFu;
            s_next = 0;
        }
        __syncthreads();
        if (!s_ok && n_pool <= MR_POOL) {
            // Extension. U = D_k (rounded up) + eps bounds the key of every row that can reach the
            // top k. Every row outside the collected candidates has a key of at least
            // B = min(next float above the shared bound, the last key of every full list): the
            // filter dropped it against the bound or a full list's threshold, or it sits in a list
            // above the bound. If U < B, the candidates with a key <= U (the pool plus the few
            // collected ones between T and U) contain every row with a key <= U, so their exact
            // top k is the exact answer: a row left out has D >= K - eps > U - eps = D_k, which is
            // >= the k-th exact distance of the larger set. No second filter pass is needed.
            for (int sp = threadIdx.x; sp < splits; sp += blockDim.x) {
                const int64_t off = ((int64_t)sp * nq_pad + qi) * kp + kp - 1;
                if (part_ids[off] != va::kInvalidId) atomicMin(&s_lmin, va::f2key(part_keys[off]));
            }
            __syncthreads();
            float B = s_lmin == 0xFFFFFFFFu ? INFINITY : va::key2f(s_lmin);
            if (bound != 0xFFFFFFFFu) B = fminf(B, nextafterf(va::key2f(bound), INFINITY));
            const double U = s_u;
            if (U < (double)B) {
                // the collected candidates above the pool with a key <= U, into sel (kp2 slots)
                for (int i = threadIdx.x; i < n_pool; i += blockDim.x)
                    if (pool[i] > T && (double)va::key2f((uint32_t)(pool[i] >> 32)) <= U) {
                        const int slot = atomicAdd(&s_next, 1);
                        if (slot < kp2) sel[slot] = pool[i];
                    }
                __syncthreads();
                const int m2 = s_next;
                if (m2 <= kp2) {
                    for (int c = warp; c < kp2; c += nwarps) {
                        const uint64_t r = exact(c < m2 ? sel[c] : ~0ull);
                        if (lane == 0) sel[c] = r;
                    }
                    va::block_bitonic_sort(sel, kp2);
                    __syncthreads();
                    if (threadIdx.x == 0) {
                        // the k smallest of the two sorted lists, into pool (no longer needed)
                        int a = 0, b = 0;
                        for (int i = 0; i < k; ++i) pool[i] = (b >= kp2 || (a < kp2 && ex[a] < sel[b])) ? ex[a++] : sel[b++];
                        for (int i = 0; i < k; ++i) ex[i] = pool[i];
                        s_ok = 1;
                    }
                    __syncthreads();
                }
            }
        }
        if (!s_ok) {
            if (threadIdx.x == 0) fail_list[atomicAdd(fail_cnt, 1u)] = (uint32_t)qi;
            return;
        }
    }
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

int cert_kind(int elem, bool cosine) {
    return elem == 2 ? (cosine ? VA_CERT_BF16_COS : VA_CERT_BF16) : (cosine ? VA_CERT_TF32_COS : VA_CERT_TF32);
}

// Certificate input of one operand kind over rows [r0, r0 + count): max operand error, into
// db->cert[1 + kind] (maxima only grow).
int operand_err(va_context* ctx, va_database* db, int kind, int64_t r0, int64_t count) {
    if (count <= 0) return VA_OK;
    const size_t esz = db->dtype == VA_DTYPE_BF16 ? 2 : 4;
    const void* src = (const uint8_t*)db->rows + (size_t)r0 * db->dim * esz;
    k_operand_err<<<warps_grid(count), 256, 0, ctx->stream>>>(src, db->dtype, count, db->dim, kind, db->cert);
    return va_check_launch("k_operand_err");
}

// Build (once) the operand a precision/metric needs, with its certificate input.
int ensure_operand(va_context* ctx, va_database* db, int elem, bool cosine, const void** out) {
    const int64_t n = db->n;
    if (elem == 2) {
        uint16_t** slot = cosine ? &db->op_cos : &db->op;
        if (!*slot) {
            if (!cosine && db->dtype == VA_DTYPE_BF16 && db->dim % KBLOCK == 0) {
                db->op = (uint16_t*)db->rows;
                db->op_alias = true;
            } else {
                VA_CUDA_TRY(cudaMalloc((void**)slot, (size_t)std::max<int64_t>(n, db->cap) * db->dpad * 2));
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
                VA_CUDA_TRY(cudaMalloc((void**)slot, (size_t)std::max<int64_t>(n, db->cap) * db->dpad * 4));
                k_operand<float><<<warps_grid(n), 256, 0, ctx->stream>>>(db->rows, db->dtype, n, n, db->dim,
                                                                         db->dpad, cosine ? 1 : 0, *slot);
                VA_TRY(va_check_launch("k_operand<f32>"));
            }
        }
        *out = *slot;
    }
    const int kind = cert_kind(elem, cosine);
    if (!(db->cert_ready & (1u << kind))) {
        VA_TRY(operand_err(ctx, db, kind, 0, n));
        db->cert_ready |= 1u << kind;
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
// keeps 64- or 128-entry lists and the merge proves the pool), up to VA_MAX_SELECT_K; 0 when larger.
int choose_pool(int k, int rerank) {
    const int kp = choose_kp(k, rerank);
    if (kp) return kp;
    const int64_t want = rerank > 0 ? (int64_t)rerank * k : (int64_t)k + std::max(k / 4, 22);
    return want <= VA_MAX_SELECT_K ? (int)want : 0;
}

// Pool of the second tensor-core pass over the queries the first pass could not certify: the next
// list size (32 -> 64 -> 128 entries: each doubling adds about ln 2 extreme-value spacings to the
// certificate's gap, and the pass over a few query tiles costs little), then four times wider
// (pools proven from 64/128-entry lists); 0 when no wider pool is supported (exact route next).
int wider_pool(int pool) {
    if (pool < 64) return 64;
    if (pool < 128) return 128;
    const int p = std::min(4 * pool, VA_MAX_SELECT_K);
    return p > pool ? p : 0;
}

int merge_rerank(va_context* ctx, va_database* db, const float* queries, int64_t nq, int k, int metric,
                 const TcPlan& plan, const float* part_keys, const uint32_t* part_ids, const uint32_t* gthr,
                 float* out_vals, uint32_t* out_ids, int pool_n, int prove, const CertArgs& ca,
                 uint32_t* fail_list, uint32_t* fail_cnt);

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

int gather_queries(va_context* ctx, const float* src, int dim, const uint32_t* list, int64_t n, float* dst) {
    k_gather_rows<<<grid_for(n * dim), 256, 0, ctx->stream>>>(src, dim, list, n, dst);
    return va_check_launch("k_gather_rows");
}

int scatter_results(va_context* ctx, const float* v, const uint32_t* ids, const uint32_t* list, int64_t n, int k,
                    float* out_v, uint32_t* out_i) {
    k_scatter_results<<<grid_for(n * k), 256, 0, ctx->stream>>>(v, ids, list, n, k, out_v, out_i);
    return va_check_launch("k_scatter_results");
}

// Count written by a merge (the call waits for the stream: the next passes depend on it).
int read_count(va_context* ctx, const uint32_t* dcnt, uint32_t* n) {
    return va_read_u32(ctx, dcnt, n);
}

// Exact route: the reference's chunked two-pass strategy (executeChunkedTwoPass,
// FusedL2TopKKernel.swift:765-1090) on fp32 SIMT distance tiles of the ORIGINAL rows (fp32 or
// bf16 widened exactly), per-chunk top-k and a running device merge. Scratch: `ws` of `ws_bytes`
// when given, else the context workspace.
int search_exact(va_context* ctx, va_database* db, const float* queries, int64_t nq, int k, int metric,
                 float* out_vals, uint32_t* out_ids, void* ws = nullptr, size_t ws_bytes = 0) {
    const int mode = metric == VA_METRIC_IP ? VA_SELECT_MAX : VA_SELECT_MIN;
    const int flag = metric == VA_METRIC_COSINE ? 1 : 0;
    VA_REQUIRE((nq + 63) / 64 <= 65535, "numQueries %lld too large for the exact route", (long long)nq);
    const size_t lists = (size_t)nq * k;
    int64_t chunk;
    if (ws) {
        // mat (nq x chunk) + norms (nq + chunk) + lists (8 B per entry) within ws_bytes
        const int64_t avail = (int64_t)ws_bytes - (int64_t)lists * 8 - (int64_t)nq * 4 - 512;
        chunk = avail / (4 * nq + 4);
        if (chunk < 64)
            return va_set_error(VA_ERR_INVALID_ARG,
                                "the exact route for %lld queries needs more than the %zu bytes of scratch available",
                                (long long)nq, ws_bytes);
    } else {
        chunk = std::max<int64_t>(256, (int64_t)(256ll << 20) / (4 * std::max<int64_t>(nq, 1)));
    }
    chunk = std::min<int64_t>(chunk, db->n);
    const size_t mat = (size_t)nq * chunk;
    const size_t norms = (size_t)nq + chunk;
    if (!ws) VA_TRY(va_workspace(ctx, (mat + norms) * 4 + lists * 8 + 512, &ws));
    float* dmat = (float*)ws;
    float* cv = dmat + mat;
    uint32_t* ci = (uint32_t*)(cv + lists);
    float* nscratch = (float*)(ci + lists);
    const size_t esz = db->dtype == VA_DTYPE_BF16 ? 2 : 4;
    for (int64_t c0 = 0; c0 < db->n; c0 += chunk) {
        const int64_t cn = std::min<int64_t>(chunk, db->n - c0);
        VA_TRY(va_distance_matrix_rows(ctx, queries, nq, (const uint8_t*)db->rows + (size_t)c0 * db->dim * esz,
                                       db->dtype, cn, db->dim, metric, flag, dmat, cn, nscratch));
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

// Filter arguments shared by the tensor-core passes.
TcFilterArgs filter_args(va_database* db, int metric, int elem, const void* q_op, const void* x_op,
                         const TcPlan& plan, float* part_keys, uint32_t* part_ids, uint32_t* gthr,
                         uint32_t* sync_cnt) {
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
    // A single pipeline wait lasts microseconds; 2 s means the pipeline is stuck.
    a.limit_ms = 2000u;
    a.levels = plan.levels;
    return a;
}

CertArgs cert_args(va_database* db, int elem, int metric) {
    CertArgs ca;
    ca.on = 1;
    ca.kind = cert_kind(elem, metric == VA_METRIC_COSINE);
    ca.dpad = db->dpad;
    ca.cert = db->cert;
    return ca;
}

// One tensor-core pass over queries[nq]: operand, filter, merge with exact rerank and the
// certificate. Queries that are not certified exact (and, for pools wider than the lists,
// queries whose pool is not proven) are appended to fail_list / fail_cnt (indices into
// `queries`) and get no output rows. `timed`: bracket the filter with the context's events.
int tc_pass(va_context* ctx, va_database* db, const float* queries, int64_t nq, int k, int metric, int elem, int pool,
            float* out_vals, uint32_t* out_ids, uint32_t* fail_list, uint32_t* fail_cnt, bool timed) {
    const bool wide = pool > 128;
    TcPlan plan;
    VA_TRY(va_tc_plan_pool(ctx, nq, db->n, pool, &plan, (int64_t)db->dpad * elem));
    const int kp = plan.kp;  // list length (up to 128 the whole list is the pool)
    const bool cosine = metric == VA_METRIC_COSINE;
    const void* x_op = nullptr;
    VA_TRY(ensure_operand(ctx, db, elem, cosine, &x_op));
    // Scratch: query operand, partial lists, shared per-query bounds, pacing counters.
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
    const TcFilterArgs a = filter_args(db, metric, elem, q_op, x_op, plan, part_keys, part_ids, gthr, sync_cnt);
    const bool prof = timed && ctx->prof_ev && ctx->prof_n < ctx->prof_cap;
    if (timed) VA_CUDA_TRY(cudaEventRecord(prof ? ctx->prof_ev[2 * ctx->prof_n] : ctx->ev_k0, ctx->stream));
    VA_TRY(va_tc_filter(ctx, a, plan));
    if (timed) {
        VA_CUDA_TRY(cudaEventRecord(prof ? ctx->prof_ev[2 * ctx->prof_n + 1] : ctx->ev_k1, ctx->stream));
        if (prof)
            ctx->prof_n++;
        else
            ctx->k_recorded = true;
    }
    return merge_rerank(ctx, db, queries, nq, k, metric, plan, part_keys, part_ids, gthr, out_vals, out_ids,
                        wide ? pool : 0, wide ? 1 : 0, cert_args(db, elem, metric), fail_list, fail_cnt);
}

// Tensor-core search with exactness guaranteed: pass 1 at `pool`; the queries it cannot certify
// take a second tensor-core pass with a wider pool; what that cannot certify takes the exact
// route. Each later pass reads back the count of the previous one (the call waits for the stream).
int search_tc(va_context* ctx, va_database* db, const float* queries, int64_t nq, int k, int metric, int elem,
              int pool, float* out_vals, uint32_t* out_ids) {
    // aux (sized before any kernel writes it): counters, two fail lists, gathered queries and
    // results of the second pass and of the exact route.
    const size_t cb = 256, lb = round_up(4 * nq, 256), qb = round_up(nq * db->dim * 4, 256),
                 rb = round_up(nq * k * 4, 256);
    void* aux;
    VA_TRY(va_aux_buffer(ctx, cb + 2 * lb + 2 * qb + 4 * rb, &aux));
    uint8_t* p = (uint8_t*)aux;
    uint32_t* cnt = (uint32_t*)p;  // [0] pass 1, [32] pass 2
    uint32_t* list1 = (uint32_t*)(p + cb);
    uint32_t* list2 = (uint32_t*)(p + cb + lb);
    float* gq1 = (float*)(p + cb + 2 * lb);
    float* gq2 = (float*)((uint8_t*)gq1 + qb);
    float* gv1 = (float*)((uint8_t*)gq2 + qb);
    uint32_t* gi1 = (uint32_t*)((uint8_t*)gv1 + rb);
    float* gv2 = (float*)((uint8_t*)gi1 + rb);
    uint32_t* gi2 = (uint32_t*)((uint8_t*)gv2 + rb);
    VA_CUDA_TRY(cudaMemsetAsync(cnt, 0, cb, ctx->stream));
    VA_TRY(tc_pass(ctx, db, queries, nq, k, metric, elem, pool, out_vals, out_ids, list1, cnt, true));
    uint32_t n1 = 0;
    VA_TRY(read_count(ctx, cnt, &n1));
    ctx->stat_uncertified = n1;
    va_log_info("va_knn_search: %lld queries, pool %d: %u not certified by the first pass", (long long)nq, pool, n1);
    if (!n1) return VA_OK;
    VA_TRY(gather_queries(ctx, queries, db->dim, list1, n1, gq1));
    // Few failures: the next list size. More than 1/32 of the batch: neighbourhoods denser than
    // the pool can separate at this precision (clustered data), so a much wider pool (at least 4x
    // and 512), which later searches of this metric then start with. (The second pass runs whole
    // query tiles over the whole database, so it costs about the failing fraction of the first;
    // a wider first pool costs a few percent of the filter: C3 with 20% failing spent 83 ms per
    // batch in second passes against 9 ms for the wider pool.)
    const bool dense = (int64_t)n1 * 32 > nq;
    int pool2 = wider_pool(pool);
    if (dense && pool < VA_MAX_SELECT_K) {
        pool2 = std::min(std::max(4 * pool, 512), VA_MAX_SELECT_K);
        if (nq >= 64) db->pool_hint[metric] = std::max(db->pool_hint[metric], (pool2 + k - 1) / k);
    }
    va_log_info("va_knn_search: second pass over %u queries with a pool of %d", n1, pool2);
    if (pool2) {
        VA_TRY(tc_pass(ctx, db, gq1, n1, k, metric, elem, pool2, gv1, gi1, list2, cnt + 32, false));
        uint32_t n2 = 0;
        VA_TRY(read_count(ctx, cnt + 32, &n2));
        ctx->stat_exact = n2;
        if (n2) {
            VA_TRY(gather_queries(ctx, gq1, db->dim, list2, n2, gq2));
            VA_TRY(search_exact(ctx, db, gq2, n2, k, metric, gv2, gi2));
            VA_TRY(scatter_results(ctx, gv2, gi2, list2, n2, k, gv1, gi1));
        }
    } else {
        ctx->stat_exact = n1;
        VA_TRY(search_exact(ctx, db, gq1, n1, k, metric, gv1, gi1));
    }
    return scatter_results(ctx, gv1, gi1, list1, n1, k, out_vals, out_ids);
}

int merge_rerank(va_context* ctx, va_database* db, const float* queries, int64_t nq, int k, int metric,
                 const TcPlan& plan, const float* part_keys, const uint32_t* part_ids, const uint32_t* gthr,
                 float* out_vals, uint32_t* out_ids, int pool_n, int prove, const CertArgs& ca,
                 uint32_t* fail_list, uint32_t* fail_cnt) {
    const int kp2 = va::next_pow2(std::max(plan.kp, pool_n));
    size_t smem = (size_t)kp2 * 16 + (size_t)MR_POOL * 8 + (size_t)db->dim * 4;
    if (smem > 48 * 1024)
        VA_CUDA_TRY(cudaFuncSetAttribute(k_merge_rerank, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    if ((prove || ca.on) && !(fail_list && fail_cnt))
        return va_set_error(VA_ERR_INVALID_ARG, "internal: a proving or certifying merge needs a fail list");
    k_merge_rerank<<<(unsigned)nq, MR_THREADS, smem, ctx->stream>>>(part_keys, part_ids, plan.splits, plan.nq_pad,
                                                                    plan.kp, pool_n > 0 ? pool_n : plan.kp, queries,
                                                                    db->rows, db->dtype, db->dim,
                                                                    metric, k, db->id_base, gthr, plan.levels,
                                                                    prove, ca, out_vals, out_ids,
                                                                    fail_list, fail_cnt);
    return va_check_launch("k_merge_rerank");
}

// Route of a float search after AUTO: the contraction precision and the candidate pool (pool 0
// with precision FP32: the exact route).
int plan_route(const va_database* db, int k, int precision, int rerank, int* prec_out, int* pool_out) {
    int pool = choose_pool(k, rerank);
    int prec = precision;
    // AUTO: bf16 when the pool holds at least 3k candidates. Without a caller's factor, fp32 rows
    // take a 3k pool (wider than 128 from k = 43 on) to stay on bf16; otherwise (bf16 rows, a thin
    // caller-set pool) the 4x smaller tf32 error keeps more queries certified in the first pass.
    // No pool size -> exact route. Rows of at most 16 dimensions (fp32) take the exact route too:
    // few dimensions give the reduced-precision keys no resolution between close neighbours (for
    // d = 1 a bf16 key cannot order points 1/N apart), so most queries would fail the
    // certificate, and the SIMT route is cheap there.
    if (prec == VA_PREC_AUTO) {
        if (pool && pool < 3 * k && rerank == 0 && db->dtype == VA_DTYPE_F32 && 3 * k <= VA_MAX_SELECT_K)
            pool = 3 * k;
        prec = !pool ? VA_PREC_FP32 : (pool >= 3 * k ? VA_PREC_BF16 : VA_PREC_TF32);
        if (db->dim <= 16 && db->dtype == VA_DTYPE_F32) prec = VA_PREC_FP32;
    }
    if (prec != VA_PREC_FP32 && !pool)
        return va_set_error(VA_ERR_UNSUPPORTED,
                            "candidate pool %lld of k %d is not supported by the tensor-core route (at most %d); "
                            "use precision FP32",
                            (long long)(rerank ? (int64_t)rerank * k : (int64_t)k + std::max(k / 4, 22)), k,
                            VA_MAX_SELECT_K);
    *prec_out = prec;
    *pool_out = pool;
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
    if (e == cudaSuccess) e = cudaMalloc((void**)&db->cert, VA_CERT_WORDS * sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMemsetAsync(db->cert, 0, VA_CERT_WORDS * sizeof(uint32_t), ctx->stream);
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
    k_row_bias<<<warps_grid(n_pad), 256, 0, ctx->stream>>>(db->rows, dtype, n, n_pad, dim, db->norms2, db->zbias,
                                                           db->cert);
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
    VaRange nvtx_range("va_db_create");
    return db_create_impl(ctx, rows, on_device, n, dim, dtype, id_base, out, true);
}

int va_db_destroy(va_database* db) {
    if (!db) return VA_OK;
    if (db->shards) {
        for (int m = 0; m < db->nshards; ++m) va_db_destroy(db->shards[m]);
        delete[] db->shards;
        delete db;
        return VA_OK;
    }
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
    if (db->cert) cudaFree(db->cert);
    if (db->rows) cudaFree(db->rows);
    delete db;
    return VA_OK;
}

int va_db_info(const va_database* db, int64_t* n, int* dim, int* dtype) {
    VA_REQUIRE(db, "db must not be NULL");
    if (n) *n = va_is_sharded(db) ? db->n_total : db->n;
    if (dim) *dim = db->dim;
    if (dtype) *dtype = db->dtype;
    return VA_OK;
}

int va_db_rows(const va_database* db, const void** rows) {
    VA_REQUIRE(db && rows, "db and rows must not be NULL");
    VA_REQUIRE(!db->shards, "a multi-device sharded database has one row array per device (va_db_shard)");
    *rows = db->rows;
    return VA_OK;
}

int va_knn_search(va_context* ctx, const va_database* cdb, const float* queries, int64_t nq, int k, int metric,
                  int precision, int rerank, float* out_vals, uint32_t* out_ids) {
    VaRange nvtx_range("va_knn_search");
    VA_REQUIRE(ctx && cdb && out_vals && out_ids, "ctx, db, out_vals and out_ids must not be NULL");
    if (va_is_sharded(cdb))
        return va_sharded_knn(ctx, cdb, queries, nq, k, metric, precision, rerank, out_vals, out_ids);
    return va_knn_search_local(ctx, cdb, queries, nq, k, metric, precision, rerank, out_vals, out_ids);
}

}  // extern "C"

int va_knn_search_local(va_context* ctx, const va_database* cdb, const float* queries, int64_t nq, int k, int metric,
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
    ctx->stat_uncertified = 0;
    ctx->stat_exact = 0;
    int prec = 0, pool = 0;
    VA_TRY(plan_route(db, k, precision, rerank, &prec, &pool));
    if (prec == VA_PREC_FP32) {
        ctx->stat_exact = nq;
        VA_TRY(search_exact(ctx, db, queries, nq, k, metric, out_vals, out_ids));
    } else {
        // A pool this database learned it needs for this metric (dense neighbourhoods).
        if (db->pool_hint[metric] > 0)
            pool = std::max(pool, (int)std::min<int64_t>((int64_t)db->pool_hint[metric] * k, VA_MAX_SELECT_K));
        const int elem = prec == VA_PREC_TF32 ? 4 : 2;
        VA_TRY(search_tc(ctx, db, queries, nq, k, metric, elem, pool, out_vals, out_ids));
    }
    VA_CUDA_TRY(cudaEventRecord(ctx->ev_stop, ctx->stream));
    return VA_OK;
}

extern "C" {

int va_last_search_stats(va_context* ctx, int64_t* uncertified, int64_t* exact) {
    VA_REQUIRE(ctx && uncertified && exact, "ctx, uncertified and exact must not be NULL");
    *uncertified = ctx->stat_uncertified;
    *exact = ctx->stat_exact;
    return VA_OK;
}

int va_knn_search_host(va_context* ctx, const va_database* db, const float* queries_host, int64_t nq, int k,
                       int metric, int precision, int rerank, float* out_vals_host, uint32_t* out_ids_host) {
    VaRange nvtx_range("va_knn_search_host");
    VA_REQUIRE(ctx && db && queries_host && out_vals_host && out_ids_host, "all pointers must be non-NULL");
    VA_REQUIRE(nq > 0, "numQueries must be positive, got %lld", (long long)nq);
    VA_REQUIRE(k > 0, "k must be positive, got %d", k);
    VA_REQUIRE(k <= VA_MAX_K, "k %d exceeds maximum supported k %d", k, VA_MAX_K);
    VA_REQUIRE(db->kind != VA_DB_BINARY, "a binary database is searched with va_hamming_knn_db");
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    const size_t qb = (size_t)nq * db->dim * 4, rb = (size_t)nq * k * 4;
    void* io;
    VA_TRY(va_io_buffer(ctx, round_up((int64_t)qb, 256) + 2 * round_up((int64_t)rb, 256), &io));
    float* dq = (float*)io;
    float* dv = (float*)((uint8_t*)io + round_up((int64_t)qb, 256));
    uint32_t* di = (uint32_t*)((uint8_t*)dv + round_up((int64_t)rb, 256));
    VA_TRY(va_copy_to_device(ctx, dq, queries_host, qb));
    VA_TRY(va_knn_search(ctx, db, dq, nq, k, metric, precision, rerank, dv, di));
    VA_TRY(va_copy_to_host(ctx, out_vals_host, dv, rb));
    VA_TRY(va_copy_to_host(ctx, out_ids_host, di, rb));
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

// Same steps as search_tc (pass 1 with the certificate), with the scratch carved from a
// caller-provided region; queries the pass cannot certify take the exact route inside the same
// region (the pass's lists are dead by then).
// Scratch bytes of search_tc_fixed's pass: fail count and list, query operand, lists, one bound
// slot per query, pacing counters.
int fixed_bytes(va_context* ctx, va_database* db, int64_t nq, int kp, int elem, TcPlan* plan, size_t* bytes) {
    VA_TRY(va_tc_plan(ctx, nq, db->n, kp, plan, (int64_t)db->dpad * elem));
    const size_t head = 256 + round_up(4 * nq, 256);
    const size_t q_bytes = (size_t)plan->nq_pad * db->dpad * elem;
    const size_t part = (size_t)plan->splits * plan->nq_pad * kp;
    *bytes = head + round_up((int64_t)q_bytes, 256) + part * 8 + (size_t)plan->nq_pad * 4 +
             (size_t)plan->sync_words * 4;
    return VA_OK;
}

int search_tc_fixed(va_context* ctx, va_database* db, const float* queries, int64_t nq, int k, int metric, int elem,
                    int kp, uint8_t* scratch, size_t scratch_bytes, float* out_vals, uint32_t* out_ids) {
    TcPlan plan;
    size_t bytes = 0;
    VA_TRY(fixed_bytes(ctx, db, nq, kp, elem, &plan, &bytes));
    const bool cosine = metric == VA_METRIC_COSINE;
    const void* x_op = elem == 2 ? (cosine ? (const void*)db->op_cos : (const void*)db->op)
                                 : (cosine ? (const void*)db->op_f32_cos : (const void*)db->op_f32);
    const int kind = cert_kind(elem, cosine);
    if (!x_op || !(db->cert_ready & (1u << kind)))
        return va_set_error(VA_ERR_UNSUPPORTED,
                            "the %s operand of this database is not built yet and building it would allocate; run "
                            "one va_knn_search with this metric and precision first",
                            elem == 2 ? (cosine ? "unit-norm bf16" : "bf16") : (cosine ? "unit-norm fp32" : "fp32"));
    const size_t head = 256 + round_up(4 * nq, 256);  // fail count + fail list
    const size_t q_bytes = (size_t)plan.nq_pad * db->dpad * elem;
    const size_t part = (size_t)plan.splits * plan.nq_pad * kp;
    if (bytes > scratch_bytes)
        return va_set_error(VA_ERR_INVALID_ARG,
                            "numQueries %lld at dimension %d with a pool of %d needs %zu bytes of scratch; the "
                            "allocation-free search has %zu (split the batch)",
                            (long long)nq, db->dim, kp, bytes, scratch_bytes);
    uint32_t* fail_cnt = (uint32_t*)scratch;
    uint32_t* fail_list = (uint32_t*)(scratch + 256);
    uint8_t* p = scratch + head;
    void* q_op = p;
    p += round_up((int64_t)q_bytes, 256);
    float* part_keys = (float*)p;
    uint32_t* part_ids = (uint32_t*)(part_keys + part);
    uint32_t* gthr = part_ids + part;
    uint32_t* sync_cnt = gthr + plan.nq_pad;
    VA_CUDA_TRY(cudaMemsetAsync(fail_cnt, 0, 4, ctx->stream));
    if (elem == 2)
        k_operand<uint16_t><<<warps_grid(plan.nq_pad), 256, 0, ctx->stream>>>(
            queries, VA_DTYPE_F32, nq, plan.nq_pad, db->dim, db->dpad, cosine ? 1 : 0, (uint16_t*)q_op);
    else
        k_operand<float><<<warps_grid(plan.nq_pad), 256, 0, ctx->stream>>>(
            queries, VA_DTYPE_F32, nq, plan.nq_pad, db->dim, db->dpad, cosine ? 1 : 0, (float*)q_op);
    VA_TRY(va_check_launch("k_operand(queries)"));
    const TcFilterArgs a = filter_args(db, metric, elem, q_op, x_op, plan, part_keys, part_ids, gthr, sync_cnt);
    VA_TRY(va_tc_filter(ctx, a, plan));
    VA_TRY(merge_rerank(ctx, db, queries, nq, k, metric, plan, part_keys, part_ids, gthr, out_vals, out_ids, 0, 0,
                        cert_args(db, elem, metric), fail_list, fail_cnt));
    uint32_t nf = 0;
    VA_TRY(read_count(ctx, fail_cnt, &nf));
    ctx->stat_uncertified = nf;
    ctx->stat_exact = nf;
    if (!nf) return VA_OK;
    // Exact route for the uncertified queries: gathered queries, their results, then the route's
    // own scratch, all after the fail list.
    uint8_t* r = scratch + head;
    float* gq = (float*)r;
    r += round_up((int64_t)nf * db->dim * 4, 256);
    float* gv = (float*)r;
    r += round_up((int64_t)nf * k * 4, 256);
    uint32_t* gi = (uint32_t*)r;
    r += round_up((int64_t)nf * k * 4, 256);
    if (r >= scratch + scratch_bytes)
        return va_set_error(VA_ERR_INVALID_ARG, "%u uncertified queries do not fit the allocation-free scratch", nf);
    VA_TRY(gather_queries(ctx, queries, db->dim, fail_list, nf, gq));
    VA_TRY(search_exact(ctx, db, gq, nf, k, metric, gv, gi, r, (size_t)(scratch + scratch_bytes - r)));
    return scatter_results(ctx, gv, gi, fail_list, nf, k, out_vals, out_ids);
}

}  // namespace

extern "C" int va_knn_search_noalloc(va_context* ctx, const va_database* cdb, const float* queries, int64_t nq, int k,
                                     int metric, int precision, int rerank, float* out_vals, uint32_t* out_ids) {
    VA_REQUIRE(ctx && cdb && out_vals && out_ids, "ctx, db, out_vals and out_ids must not be NULL");
    VA_REQUIRE(cdb->kind != VA_DB_BINARY, "a binary database is searched with va_hamming_knn_db");
    VA_REQUIRE(!va_is_sharded(cdb), "the allocation-free search takes a single-device database, not a sharded one");
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
    // The same route as va_knn_search (AUTO resolved identically); only its tensor-core form with
    // pools of at most 128 candidates runs here.
    int prec = 0, pool = 0;
    VA_TRY(plan_route(db, k, precision, rerank, &prec, &pool));
    if (prec == VA_PREC_FP32)
        return va_set_error(VA_ERR_UNSUPPORTED,
                            "k %d at dimension %d takes the exact FP32 route under AUTO, which allocates; pass "
                            "precision BF16 or TF32, or use va_knn_search",
                            k, db->dim);
    if (k > 128)
        return va_set_error(VA_ERR_UNSUPPORTED,
                            "k %d exceeds the allocation-free search's lists of at most 128 entries; use "
                            "va_knn_search",
                            k);
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    const int elem = prec == VA_PREC_TF32 ? 4 : 2;
    // Lists of the route's pool (at most 128 entries), halved while the batch does not fit the
    // array but never below k: the results stay exact, since the certificate sends every query
    // a thinner pool cannot prove to the exact route.
    int kp = choose_kp(std::min(pool, 128), 1);
    for (;;) {
        TcPlan plan;
        size_t bytes = 0;
        VA_TRY(fixed_bytes(ctx, db, nq, kp, elem, &plan, &bytes));
        if (bytes <= VA_NOALLOC_SCRATCH_BYTES || kp == 32 || kp / 2 < k) break;
        kp /= 2;
    }
    ctx->stat_uncertified = 0;
    ctx->stat_exact = 0;
    void* scratch = nullptr;
    VA_TRY(noalloc_scratch(ctx->device, &scratch));
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
                                                                      db->norms2 + r0, db->zbias + r0, db->cert);
        VA_TRY(va_check_launch("k_row_bias(append)"));
    }
    for (int kind = 0; kind < 4; ++kind)
        if (db->cert_ready & (1u << kind)) VA_TRY(operand_err(ctx, db, kind, r0, count));
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
// Internal entry of the merge + exact rerank step for other translation units (the int8 path,
// whose integer keys are exact: no certificate; fail_list set = prove a pool wider than the lists).
int va_merge_rerank_internal(va_context* ctx, va_database* db, const float* queries, int64_t nq, int k, int metric,
                             const TcPlan& plan, const float* part_keys, const uint32_t* part_ids,
                             const uint32_t* gthr, float* out_vals, uint32_t* out_ids, int pool_n,
                             uint32_t* fail_list, uint32_t* fail_cnt) {
    CertArgs off = {};
    return merge_rerank(ctx, db, queries, nq, k, metric, plan, part_keys, part_ids, gthr, out_vals, out_ids, pool_n,
                        fail_list ? 1 : 0, off, fail_list, fail_cnt);
}
