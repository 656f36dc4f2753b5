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
//   * k-means starts from k-means++ seeds, as the reference (KMeansPlusPlusKernel.swift), drawn
//     with a seeded generator (or from given centroids, or distinct random rows), and runs Lloyd
//     iterations until the largest centroid movement is below `tol`
//     (KMeansConvergenceKernel.swift:78-110), as the reference does.
// The list scan computes exact squared L2 (fp32 rows, fp64 accumulation) and keeps, per (query,
// probe), the k best (distance, id) composites; the probes' lists are merged by (distance, id).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <unordered_set>
#include <vector>

#include <cuda_bf16.h>

#include <cub/device/device_radix_sort.cuh>

#include "va_internal.cuh"
#include "va_tc.cuh"

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
    // Tensor-core operand of the rows in list order: bf16 [n x dpad] (zero padded), and the row
    // biases |x|^2 for n + 512 rows (+inf past n: a list's last tile may reach 255 rows beyond it).
    int dpad = 0;
    uint16_t* op = nullptr;
    float* op32 = nullptr;        // fp32 operand [n x dpad] for the tf32 route: the rows when dim = dpad
    bool op32_owned = false;
    float* bias = nullptr;
    // Search scratch, grown on demand (one search at a time per index), and pinned host memory
    // for the tile plan (the count read-back and one upload).
    void* scratch = nullptr;
    size_t scratch_bytes = 0;
    int* h_plan = nullptr;
    size_t h_plan_ints = 0;
    // Certificate inputs of the list scan (as a flat database's, va_internal.cuh): max |x| and the
    // max operand error of the bf16 and the tf32 operands over the rows.
    uint32_t* cert = nullptr;
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

// k-means++ seeding (KMeansPlusPlusKernel.swift:94-210: first centroid uniform, then each next
// one drawn with probability proportional to the squared distance to the nearest chosen one).
// d2[r] = min(d2[r], |x_r - c|^2) for the newest centroid c (first: d2[r] = |x_r - c|^2), and
// bsum[b] = the fp64 sum of d2 over block b's KPP_ROWS rows, in a fixed order (deterministic).
constexpr int KPP_ROWS = 1024;
__global__ void __launch_bounds__(256) k_kpp_update(const float* __restrict__ x, int64_t n, int dim,
                                                    const float* __restrict__ c, int first, float* __restrict__ d2,
                                                    double* __restrict__ bsum) {
    __shared__ double s_w[8];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t r0 = (int64_t)blockIdx.x * KPP_ROWS;
    double acc = 0;
    for (int64_t r = r0 + warp; r < n && r < r0 + KPP_ROWS; r += 8) {
        double s = 0;
        for (int j = lane; j < dim; j += 32) {
            const double t = (double)x[r * dim + j] - (double)c[j];
            s += t * t;
        }
        s = warp_sum_d(s);
        const float v = first ? (float)s : fminf(d2[r], (float)s);
        if (lane == 0) {
            d2[r] = v;
            acc += (double)v;
        }
    }
    if (lane == 0) s_w[warp] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0;
        for (int w = 0; w < 8; ++w) t += s_w[w];
        bsum[blockIdx.x] = t;
    }
}

// One warp: the first row r in [r0, r1) whose running fp64 sum of d2 from r0 reaches target
// (the last row with d2 > 0 when rounding leaves the target just out of reach).
__global__ void k_kpp_pick(const float* __restrict__ d2, int64_t r0, int64_t r1, double target,
                           int64_t* __restrict__ out) {
    const int lane = threadIdx.x;
    double run = 0;
    int64_t last_pos = -1;
    for (int64_t b = r0; b < r1; b += 32) {
        const int64_t r = b + lane;
        const double v = r < r1 ? (double)d2[r] : 0.0;
        double incl = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const double t = __shfl_up_sync(0xFFFFFFFFu, incl, o);
            if (lane >= o) incl += t;
        }
        const unsigned hit = __ballot_sync(0xFFFFFFFFu, v > 0 && run + incl >= target);
        const unsigned pos = __ballot_sync(0xFFFFFFFFu, v > 0);
        if (pos) last_pos = b + 31 - __clz(pos);
        if (hit) {
            if (lane == 0) *out = b + __ffs(hit) - 1;
            return;
        }
        run += __shfl_sync(0xFFFFFFFFu, incl, 31);
    }
    if (lane == 0) *out = last_pos >= 0 ? last_pos : r0;
}

// ---------------------------------------------------------------------------------- lists
__global__ void k_histogram(const uint32_t* __restrict__ assign, int64_t n, unsigned long long* __restrict__ counts) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        atomicAdd(counts + assign[i], 1ull);
}

__global__ void k_iota(uint32_t* __restrict__ v, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        v[i] = (uint32_t)i;
}

// Position p of the list-ordered copy takes row src[p] (rows sorted stably by list): a warp per
// position copies the row; ids_out[p] = src[p] + id_base.
__global__ void k_place_sorted(const float* __restrict__ x, const uint32_t* __restrict__ src, int64_t n, int dim,
                               uint32_t id_base, float* __restrict__ rows_out, uint32_t* __restrict__ ids_out) {
    const int64_t p = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (p >= n) return;
    const int64_t r = src[p];
    for (int j = lane; j < dim; j += 32) rows_out[p * dim + j] = x[r * dim + j];
    if (lane == 0) ids_out[p] = (uint32_t)r + id_base;
}

__device__ __forceinline__ void store_op(uint16_t* p, float v) { *p = __bfloat16_as_ushort(__float2bfloat16_rn(v)); }
__device__ __forceinline__ void store_op(float* p, float v) { *p = v; }

// out[r] = src row map(r) zero padded to dpad, as bf16 (T = uint16_t) or fp32 (a zero row when
// map(r) < 0). map = null: row r; else row map[r] / map_div (gathered (query, probe) pairs -> their
// query).
template <class T>
__global__ void k_rows_op(const float* __restrict__ src, int64_t n_out, int dim, int dpad,
                          const int* __restrict__ map, int map_div, T* __restrict__ out) {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n_out * dpad;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = e / dpad;
        const int j = (int)(e - r * dpad);
        int64_t sr = r;
        if (map) sr = map[r] >= 0 ? map[r] / map_div : -1;
        const float v = (sr >= 0 && j < dim) ? src[sr * dim + j] : 0.f;
        store_op(out + e, v);
    }
}

// bias[r] = |x_r|^2 (fp64 sum, rounded) for r < n; +inf for n <= r < n_alloc. A warp per row.
__global__ void k_row_norms(const float* __restrict__ x, int64_t n, int dim, int64_t n_alloc, float* __restrict__ bias) {
    const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (r >= n_alloc) return;
    if (r >= n) {
        if (lane == 0) bias[r] = INFINITY;
        return;
    }
    double s = 0;
    for (int j = lane; j < dim; j += 32) {
        const double v = x[r * dim + j];
        s += v * v;
    }
    s = warp_sum_d(s);
    if (lane == 0) bias[r] = (float)s;
}

// Certificate inputs over the rows: cert[0] = max |x|, cert[1 + kind] = max |operand - x| for the
// bf16 and tf32 operands (rounded up). A warp per row.
__global__ void k_ivf_row_cert(const float* __restrict__ x, int64_t n, int dim, uint32_t* __restrict__ cert) {
    const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (r >= n) return;
    double s = 0, eb = 0, et = 0;
    for (int j = lane; j < dim; j += 32) {
        const float v = x[r * dim + j];
        double t, e;
        s += (double)v * v;
        va::cert_elem(v, 1.0, VA_CERT_BF16, t, e);
        eb += e * e;
        va::cert_elem(v, 1.0, VA_CERT_TF32, t, e);
        et += e * e;
    }
    s = warp_sum_d(s);
    eb = warp_sum_d(eb);
    et = warp_sum_d(et);
    if (lane == 0) {
        atomicMax(cert, __float_as_uint(__double2float_ru(sqrt(s))));
        atomicMax(cert + 1 + VA_CERT_BF16, __float_as_uint(__double2float_ru(sqrt(eb) * (1.0 + 1e-12))));
        atomicMax(cert + 1 + VA_CERT_TF32, __float_as_uint(__double2float_ru(sqrt(et) * (1.0 + 1e-12))));
    }
}

template <class T>
__global__ void k_gather_rows_t(const T* __restrict__ src, int width, const uint32_t* __restrict__ rows, int64_t n,
                                T* __restrict__ dst) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n * width; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / width;
        dst[i] = src[(int64_t)rows[r] * width + (i - r * width)];
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

// Probe-rank bucket of pair i: its rank (the rank-th nearest centroid), ranks >= nb - 1 together.
__device__ __forceinline__ int rank_bucket(int64_t i, int nprobe, int nb) { return min((int)(i % nprobe), nb - 1); }

// cnt[L * nb + b] = pairs of rank bucket b that fall on list L.
__global__ void k_probe_hist(const uint32_t* __restrict__ probes, int64_t m, int nprobe, int nb, int* __restrict__ cnt) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < m; i += (int64_t)gridDim.x * blockDim.x)
        atomicAdd(cnt + (int64_t)probes[i] * nb + rank_bucket(i, nprobe, nb), 1);
}

// Every (query, probe) pair takes a row of its list's query tiles, the list's pairs ordered by
// rank bucket: position p = base[L, b] + arrival within (L, b), in tile tile_of[lt0[L] + p / 128]
// at row p % 128. gmap[g] = pair, ginv[pair] = g.
__global__ void k_probe_scatter(const uint32_t* __restrict__ probes, int64_t m, int nprobe, int nb,
                                const int* __restrict__ base, int* __restrict__ cursor, const int* __restrict__ lt0,
                                const int* __restrict__ tile_of, int* __restrict__ gmap, int64_t* __restrict__ ginv) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < m; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t ls = (int64_t)probes[i] * nb + rank_bucket(i, nprobe, nb);
        const int p = base[ls] + atomicAdd(cursor + ls, 1);
        const int64_t g = (int64_t)tile_of[lt0[probes[i]] + p / 128] * 128 + p % 128;
        gmap[g] = (int)i;
        ginv[i] = g;
    }
}

// One block per query: the `pool` best approximate keys among its nprobe lists of kp candidates
// (positions in list order), their exact squared L2 (fp64 of the fp32 rows), the k best by
// (distance, original id), sorted. Certificate (the flat search's, va_search.cu certify): every
// row of the probed lists outside the pool has an approximate key >= T, the pool's largest
// (a (query, probe) list drops only keys at or above its last, and the per-query bound never cuts
// into the pool), and |key - (|x|^2 - 2 q.x)| <= eps for every row; when the k-th exact key plus
// eps stays below T the k best of the probed lists are exact. Otherwise the query is appended to
// fail_list (no output) and rescanned exactly.
constexpr int MR_THREADS = 256;
__global__ void __launch_bounds__(MR_THREADS) k_ivf_merge_rerank(const float* __restrict__ q, int dim,
                                                                 const int64_t* __restrict__ ginv, int nprobe,
                                                                 const float* __restrict__ pk,
                                                                 const uint32_t* __restrict__ pi, int kp, int pool,
                                                                 int k, const float* __restrict__ rows,
                                                                 const uint32_t* __restrict__ ids,
                                                                 const uint32_t* __restrict__ cert, int cert_kind,
                                                                 int dpad, float* __restrict__ out_v,
                                                                 uint32_t* __restrict__ out_i,
                                                                 uint32_t* __restrict__ fail_list,
                                                                 uint32_t* __restrict__ fail_cnt,
                                                                 const uint32_t* __restrict__ gthr) {
    __shared__ uint64_t s_sel[128];
    __shared__ uint64_t s_ex[128];
    __shared__ va::SelectShared sh;
    __shared__ unsigned long long s_t;
    __shared__ double s_qn2, s_an, s_ae;
    __shared__ int s_ok;
    const int64_t qi = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    auto get = [&](int64_t i) -> uint64_t {
        const int s = (int)(i / kp), j = (int)(i - (int64_t)s * kp);
        const int64_t o = ginv[qi * nprobe + s] * kp + j;
        const uint32_t id = pi[o];
        if (id == va::kInvalidId) return ~0ull;
        return va::composite(va::f2key(pk[o]), id);
    };
    if (threadIdx.x == 0) s_t = 0;
    const int m = va::block_select_radix((int64_t)nprobe * kp, pool, get, s_sel, sh);
    __syncthreads();
    {
        unsigned long long t = 0;
        for (int i = threadIdx.x; i < m; i += blockDim.x) t = s_sel[i] > t ? s_sel[i] : t;
        if (m < pool) t = ~0ull;
        atomicMax(&s_t, t);
    }
    if (warp == 0 && cert) {
        double a = 0, e2 = 0;
        for (int j = lane; j < dim; j += 32) {
            double t, err;
            va::cert_elem(q[qi * dim + j], 1.0, cert_kind, t, err);
            a += t * t;
            e2 += err * err;
        }
        a = warp_sum_d(a);
        e2 = warp_sum_d(e2);
        if (lane == 0) {
            s_qn2 = a;
            s_an = sqrt(a) * (1.0 + 1e-12);
            s_ae = sqrt(e2) * (1.0 + 1e-12);
        }
    }
    // Exact key of one candidate (list position in the low word; warp-collective).
    auto exact = [&](uint64_t sc) -> uint64_t {
        if (sc == ~0ull) return ~0ull;
        const uint32_t pos = (uint32_t)sc;
        double acc = 0;
        for (int j = lane; j < dim; j += 32) {
            const double t = (double)q[qi * dim + j] - (double)rows[(int64_t)pos * dim + j];
            acc += t * t;
        }
        acc = warp_sum_d(acc);
        return va::composite(va::f2key((float)acc), ids[pos]);
    };
    for (int c = warp; c < m; c += MR_THREADS / 32) {
        const uint64_t comp = exact(s_sel[c]);
        if (lane == 0) s_ex[c] = comp;
    }
    const int p2 = va::next_pow2(m > 0 ? m : 1);
    for (int i = m + threadIdx.x; i < p2; i += blockDim.x) s_ex[i] = ~0ull;
    va::block_bitonic_sort(s_ex, p2);
    if (cert && s_t != ~0ull) {
        __shared__ double s_u;
        __shared__ unsigned s_lmin;
        __shared__ int s_next;
        if (threadIdx.x == 0) {
            const double u24 = 5.9604644775390625e-08, u22 = 2.384185791015625e-07;
            const double vk = (double)va::key2f((uint32_t)(s_ex[k - 1] >> 32));
            const double dk = vk * (1.0 + 4.0 * u24) - s_qn2 * (1.0 - 1e-12);
            const double mb = (double)__uint_as_float(cert[0]), md = (double)__uint_as_float(cert[1 + cert_kind]);
            const double A = s_an + s_ae, g = (double)dpad * u22;
            double eps = 2.0 * (A * md + s_ae * mb + g * A * (mb + md)) +
                         u24 * (2.0 * A * (mb + md) * (1.0 + g) + mb * mb) + 2.0 * u24 * mb * mb;
            eps = eps * (1.0 + 1e-6) + 1e-30;
            s_u = dk + eps;
            s_ok = s_u < (double)va::key2f((uint32_t)(s_t >> 32)) ? 1 : 0;
            s_lmin = 0xFFFFFFFFu;
            s_next = 0;
        }
        __syncthreads();
        if (!s_ok) {
            // Extension (as the flat merge's): every row outside the probed lists' entries was
            // dropped against the query's bound or a full list's last key, so its key is at least
            // B = min(next float above the bound, the last key of every full list). If U = D_k
            // (rounded up) + eps < B, the entries with a key <= U hold every row that can reach
            // the top k: rerank the ones above the pool too and take the exact top k.
            for (int sp = threadIdx.x; sp < nprobe; sp += blockDim.x) {
                const int64_t o = ginv[qi * nprobe + sp] * kp + kp - 1;
                if (pi[o] != va::kInvalidId) atomicMin(&s_lmin, va::f2key(pk[o]));
            }
            __syncthreads();
            float B = s_lmin == 0xFFFFFFFFu ? INFINITY : va::key2f(s_lmin);
            const uint32_t bnd = gthr ? gthr[qi] : 0xFFFFFFFFu;
            if (bnd != 0xFFFFFFFFu) B = fminf(B, nextafterf(va::key2f(bnd), INFINITY));
            const double U = s_u;
            if (U < (double)B) {
                __syncthreads();  // s_sel (the pool) is read no more: it takes the extension
                for (int64_t i = threadIdx.x; i < (int64_t)nprobe * kp; i += blockDim.x) {
                    const uint64_t c = get(i);
                    if (c != ~0ull && c > s_t && (double)va::key2f((uint32_t)(c >> 32)) <= U) {
                        const int slot = atomicAdd(&s_next, 1);
                        if (slot < 128) s_sel[slot] = c;
                    }
                }
                __syncthreads();
                const int m2 = s_next;
                if (m2 <= 128) {
                    for (int c = warp; c < 128; c += MR_THREADS / 32) {
                        const uint64_t comp = exact(c < m2 ? s_sel[c] : ~0ull);
                        if (lane == 0) s_sel[c] = comp;
                    }
                    va::block_bitonic_sort(s_sel, 128);
                    __syncthreads();
                    if (threadIdx.x == 0) {
                        // the k smallest of the two sorted lists (s_ex: p2 entries, s_sel: 128)
                        int a = 0, b = 0;
                        uint64_t outk[128];
                        for (int i = 0; i < k; ++i)
                            outk[i] = (b >= 128 || (a < p2 && s_ex[a] < s_sel[b])) ? s_ex[a++] : s_sel[b++];
                        for (int i = 0; i < k; ++i) s_ex[i] = outk[i];
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
    for (int i = threadIdx.x; i < k; i += blockDim.x) {
        const uint64_t c = i < m ? s_ex[i] : ~0ull;
        out_v[qi * k + i] = c == ~0ull ? INFINITY : va::key2f((uint32_t)(c >> 32));
        out_i[qi * k + i] = c == ~0ull ? va::kInvalidId : (uint32_t)c;
    }
}

// ---------------------------------------------------------------------------------- list scan
constexpr int LS_THREADS = 256;
constexpr int LS_BUF = 1024;
constexpr int LS_ROWS = 4;  // rows per warp and pass of the exact list scan

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
    // Each warp takes LS_ROWS rows per pass (rows base + warp + nwarps * u) and issues all of
    // their loads before using any: the scan is latency-bound on the row reads.
    const bool vec = (dim & 3) == 0;  // 16-byte loads: rows and the query start on 16 bytes
    for (int64_t base = r0; base < r1; base += (int64_t)nwarps * LS_ROWS) {
        double acc[LS_ROWS];
#pragma unroll
        for (int u = 0; u < LS_ROWS; ++u) acc[u] = 0;
        if (vec) {
            for (int j0 = lane * 4; j0 < dim; j0 += 128) {
                float4 xv[LS_ROWS];
#pragma unroll
                for (int u = 0; u < LS_ROWS; ++u) {
                    const int64_t r = base + warp + (int64_t)nwarps * u;
                    xv[u] = r < r1 ? __ldg((const float4*)(rows + r * dim + j0)) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
                const float4 qv = *(const float4*)(s_q + j0);
#pragma unroll
                for (int u = 0; u < LS_ROWS; ++u) {
                    const double t0 = (double)qv.x - (double)xv[u].x, t1 = (double)qv.y - (double)xv[u].y;
                    const double t2 = (double)qv.z - (double)xv[u].z, t3 = (double)qv.w - (double)xv[u].w;
                    acc[u] += t0 * t0 + t1 * t1 + t2 * t2 + t3 * t3;
                }
            }
        } else {
#pragma unroll
            for (int u = 0; u < LS_ROWS; ++u) {
                const int64_t r = base + warp + (int64_t)nwarps * u;
                double a = 0;
                if (r < r1)
                    for (int j = lane; j < dim; j += 32) {
                        const double t = (double)s_q[j] - (double)rows[r * dim + j];
                        a += t * t;
                    }
                acc[u] = a;
            }
        }
#pragma unroll
        for (int u = 0; u < LS_ROWS; ++u) acc[u] = warp_sum_d(acc[u]);
        if (lane == 0) {
#pragma unroll
            for (int u = 0; u < LS_ROWS; ++u) {
                const int64_t r = base + warp + (int64_t)nwarps * u;
                if (r < r1) {
                    const uint64_t comp = va::composite(va::f2key((float)acc[u]), ids[r]);
                    if (comp < s_thr) {
                        const int slot = atomicAdd(&s_cnt, 1);
                        if (slot < LS_BUF) s_buf[slot] = comp;
                    }
                }
            }
        }
        __syncthreads();
        // Every thread reads the count before any warp of the next pass over rows adds to it.
        const bool full = s_cnt > LS_BUF - nwarps * LS_ROWS;
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

// The bf16 operand and row biases of the rows in list order.
int prepare_operand(va_context* ctx, va_ivf* ivf) {
    ivf->dpad = (int)round_up(ivf->dim, 64);
    const int64_t n = ivf->n;
    cudaError_t e = cudaMalloc((void**)&ivf->op, (size_t)std::max<int64_t>(n, 1) * ivf->dpad * 2);
    if (e == cudaSuccess) e = cudaMalloc((void**)&ivf->bias, (size_t)(n + 512) * 4);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return va_set_error(VA_ERR_OOM, "IVF operand allocation failed: %s", cudaGetErrorString(e));
    }
    if (n) {
        k_rows_op<uint16_t><<<grid_for(n * ivf->dpad), 256, 0, ctx->stream>>>(ivf->rows, n, ivf->dim, ivf->dpad,
                                                                               nullptr, 1, ivf->op);
        VA_TRY(va_check_launch("k_rows_op"));
    }
    k_row_norms<<<(unsigned)(((n + 512) * 32 + 255) / 256), 256, 0, ctx->stream>>>(ivf->rows, n, ivf->dim, n + 512,
                                                                                  ivf->bias);
    VA_TRY(va_check_launch("k_row_norms"));
    if (cudaMalloc((void**)&ivf->cert, VA_CERT_WORDS * 4) != cudaSuccess) {
        cudaGetLastError();
        return va_set_error(VA_ERR_OOM, "IVF certificate buffer allocation failed");
    }
    VA_CUDA_TRY(cudaMemsetAsync(ivf->cert, 0, VA_CERT_WORDS * 4, ctx->stream));
    if (n) {
        k_ivf_row_cert<<<(unsigned)((n * 32 + 255) / 256), 256, 0, ctx->stream>>>(ivf->rows, n, ivf->dim, ivf->cert);
        VA_TRY(va_check_launch("k_ivf_row_cert"));
    }
    return va_synchronize(ctx);
}

// The index's search scratch, at least `bytes`; when it grows, its first `keep` bytes move along.
int scratch(va_context* ctx, va_ivf* ivf, size_t bytes, size_t keep, void** out) {
    if (bytes > ivf->scratch_bytes) {
        const size_t want = std::max(bytes, (size_t)1 << 20);
        void* fresh = nullptr;
        if (cudaMalloc(&fresh, want) != cudaSuccess) {
            cudaGetLastError();
            return va_set_error(VA_ERR_OOM, "IVF search scratch of %zu bytes failed", want);
        }
        if (ivf->scratch) {
            if (keep) VA_CUDA_TRY(cudaMemcpyAsync(fresh, ivf->scratch, keep, cudaMemcpyDeviceToDevice, ctx->stream));
            VA_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
            cudaFree(ivf->scratch);
        }
        ivf->scratch = fresh;
        ivf->scratch_bytes = want;
    }
    *out = ivf->scratch;
    return VA_OK;
}

// Seeded generator of the initial centroids (64-bit LCG; uniform doubles from its top 53 bits).
struct Lcg {
    uint64_t s;
    explicit Lcg(uint64_t seed) : s(seed * 6364136223846793005ull + 1442695040888963407ull) {}
    uint64_t next() {
        s = s * 6364136223846793005ull + 1442695040888963407ull;
        return s;
    }
    double uniform() { return (double)(next() >> 11) * (1.0 / 9007199254740992.0); }
};

// k-means++ seeding into cent[nlist x dim]: per centroid one update of the squared distances
// with a block-sum read back, the draw on the host (fp64 running sums over the blocks), and the
// row picked inside the drawn block by one warp.
int kmeanspp(va_context* ctx, const float* x, int64_t n, int dim, int nlist, Lcg& rng, float* cent) {
    const int64_t nblocks = (n + KPP_ROWS - 1) / KPP_ROWS;
    void* ws = nullptr;
    const size_t bytes = round_up(n * 4, 256) + round_up(nblocks * 8, 256) + 256;
    VA_CUDA_TRY(cudaMalloc(&ws, bytes));
    float* d2 = (float*)ws;
    double* bsum = (double*)((uint8_t*)ws + round_up(n * 4, 256));
    int64_t* d_idx = (int64_t*)((uint8_t*)bsum + round_up(nblocks * 8, 256));
    std::vector<double> h((size_t)nblocks);
    int st = VA_OK;
    int64_t idx = (int64_t)(rng.next() % (uint64_t)n);
    for (int c = 0; c < nlist && st == VA_OK; ++c) {
        if (c > 0) {
            k_kpp_update<<<(unsigned)nblocks, 256, 0, ctx->stream>>>(x, n, dim, cent + (size_t)(c - 1) * dim, c == 1,
                                                                     d2, bsum);
            if ((st = va_check_launch("k_kpp_update")) != VA_OK) break;
            if (cudaMemcpyAsync(h.data(), bsum, (size_t)nblocks * 8, cudaMemcpyDeviceToHost, ctx->stream) !=
                cudaSuccess) {
                st = va_set_error(VA_ERR_CUDA, "k-means++ read-back failed");
                break;
            }
            if ((st = va_synchronize(ctx)) != VA_OK) break;
            double total = 0;
            for (double v : h) total += v;
            if (!(total > 0)) {
                idx = (int64_t)(rng.next() % (uint64_t)n);  // every row sits on a centroid
            } else {
                const double target = rng.uniform() * total;
                double run = 0;
                int64_t b = 0;
                while (b + 1 < nblocks && run + h[(size_t)b] < target) run += h[(size_t)b++];
                const int64_t r0 = b * KPP_ROWS, r1 = std::min<int64_t>(n, r0 + KPP_ROWS);
                k_kpp_pick<<<1, 32, 0, ctx->stream>>>(d2, r0, r1, target - run, d_idx);
                if ((st = va_check_launch("k_kpp_pick")) != VA_OK) break;
                if (cudaMemcpyAsync(&idx, d_idx, 8, cudaMemcpyDeviceToHost, ctx->stream) != cudaSuccess) {
                    st = va_set_error(VA_ERR_CUDA, "k-means++ read-back failed");
                    break;
                }
                if ((st = va_synchronize(ctx)) != VA_OK) break;
            }
        }
        if (cudaMemcpyAsync(cent + (size_t)c * dim, x + idx * dim, (size_t)dim * 4, cudaMemcpyDeviceToDevice,
                            ctx->stream) != cudaSuccess)
            st = va_set_error(VA_ERR_CUDA, "k-means++ centroid copy failed");
    }
    if (st == VA_OK) st = va_synchronize(ctx);
    cudaFree(ws);
    return st;
}

// Assignment of every row to its nearest centroid (the fused search with k = 1).
int assign_rows(va_context* ctx, va_database* cdb, const float* x, int64_t n, uint32_t* assign, float* scratch_v) {
    return va_knn_search(ctx, cdb, x, n, 1, VA_METRIC_L2SQ, VA_PREC_AUTO, 0, scratch_v, assign);
}

}  // namespace

extern "C" {

int va_ivf_train(va_context* ctx, const float* x, int64_t n, int dim, int nlist, int max_iters, float tol,
                 uint64_t seed, int init, float* out_centroids, int* out_iters) {
    VaRange nvtx_range("va_ivf_train");
    VA_REQUIRE(ctx && x && out_centroids, "ctx, x and out_centroids must not be NULL");
    VA_REQUIRE(dim > 0 && dim <= VA_MAX_DIM, "dimension must be in 1..%d, got %d", VA_MAX_DIM, dim);
    VA_REQUIRE(nlist > 0 && nlist <= n, "nlist must be in 1..numVectors (%lld), got %d", (long long)n, nlist);
    VA_REQUIRE(max_iters >= 0, "max_iters must be >= 0");
    VA_REQUIRE(init == VA_IVF_INIT_KMEANSPP || init == VA_IVF_INIT_GIVEN || init == VA_IVF_INIT_RANDOM,
               "init must be VA_IVF_INIT_KMEANSPP, _GIVEN or _RANDOM, got %d", init);
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    Lcg rng(seed);
    if (init == VA_IVF_INIT_KMEANSPP) VA_TRY(kmeanspp(ctx, x, n, dim, nlist, rng, out_centroids));
    // Random initial centroids: nlist distinct rows (a partial Fisher-Yates shuffle when nlist is
    // a large share of n, else rejection of repeats).
    std::vector<int64_t> pick;
    if (init == VA_IVF_INIT_RANDOM) {
        pick.resize((size_t)nlist);
        if (n <= (int64_t)nlist * 8) {
            std::vector<int64_t> perm((size_t)n);
            for (int64_t i = 0; i < n; ++i) perm[(size_t)i] = i;
            for (int i = 0; i < nlist; ++i) {
                const int64_t j = i + (int64_t)(rng.next() % (uint64_t)(n - i));
                std::swap(perm[(size_t)i], perm[(size_t)j]);
                pick[(size_t)i] = perm[(size_t)i];
            }
        } else {
            std::unordered_set<int64_t> chosen;
            for (int i = 0; i < nlist; ++i) {
                int64_t r;
                do r = (int64_t)(rng.next() % (uint64_t)n);
                while (!chosen.insert(r).second);
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
    if (init == VA_IVF_INIT_RANDOM) {
        if (cudaMemcpyAsync(d_pick, pick.data(), (size_t)nlist * 8, cudaMemcpyHostToDevice, ctx->stream) !=
            cudaSuccess)
            return fail(va_set_error(VA_ERR_CUDA, "upload failed"));
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
    VaRange nvtx_range("va_ivf_create");
    VA_REQUIRE(ctx && rows && centroids && out, "ctx, rows, centroids and out must not be NULL");
    VA_REQUIRE(n > 0 && dim > 0 && dim <= VA_MAX_DIM && nlist > 0, "n, dim (<= %d) and nlist must be positive",
               VA_MAX_DIM);
    VA_REQUIRE((uint64_t)n + id_base <= 0xFFFFFFFFull, "numVectors + id_base exceeds the uint32 id range");
    VA_REQUIRE(n < ((int64_t)1 << 31), "numVectors must stay below 2^31 per IVF index, got %lld", (long long)n);
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
    // Assign every row, count the lists (offsets by a prefix sum on the host), sort the row
    // numbers by list with a stable radix sort (rows keep their order within a list), gather.
    int end_bit = 1;
    while (end_bit < 32 && ((uint64_t)1 << end_bit) < (uint64_t)nlist) ++end_bit;
    size_t temp_bytes = 0;
    if (cub::DeviceRadixSort::SortPairs(nullptr, temp_bytes, (const uint32_t*)nullptr, (uint32_t*)nullptr,
                                        (const uint32_t*)nullptr, (uint32_t*)nullptr, (int)n, 0, end_bit,
                                        ctx->stream) != cudaSuccess) {
        cudaGetLastError();
        return fail(va_set_error(VA_ERR_CUDA, "radix sort sizing failed"));
    }
    void* ws = nullptr;
    const size_t nb4 = round_up(n * 4, 256);
    const size_t bytes = nb4 * 5 + round_up((int64_t)nlist * 8, 256) + temp_bytes + 256;
    if (cudaMalloc(&ws, bytes) != cudaSuccess) {
        cudaGetLastError();
        return fail(va_set_error(VA_ERR_OOM, "IVF build scratch failed"));
    }
    uint8_t* w8 = (uint8_t*)ws;
    uint32_t* assign = (uint32_t*)w8;
    float* vals = (float*)(w8 + nb4);
    uint32_t* keys_out = (uint32_t*)(w8 + 2 * nb4);
    uint32_t* src_in = (uint32_t*)(w8 + 3 * nb4);
    uint32_t* src_out = (uint32_t*)(w8 + 4 * nb4);
    unsigned long long* counts = (unsigned long long*)(w8 + 5 * nb4);
    void* temp = w8 + 5 * nb4 + round_up((int64_t)nlist * 8, 256);
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
            k_iota<<<grid_for(n), 256, 0, ctx->stream>>>(src_in, n);
            if (cub::DeviceRadixSort::SortPairs(temp, temp_bytes, assign, keys_out, src_in, src_out, (int)n, 0, end_bit,
                                                ctx->stream) != cudaSuccess) {
                cudaGetLastError();
                st = va_set_error(VA_ERR_CUDA, "radix sort of the list assignment failed");
            } else {
                k_place_sorted<<<(unsigned)((n * 32 + 255) / 256), 256, 0, ctx->stream>>>(rows, src_out, n, dim,
                                                                                         id_base, ivf->rows, ivf->ids);
                st = va_check_launch("k_place_sorted");
            }
        }
    }
    if (st == VA_OK) st = va_synchronize(ctx);
    cudaFree(ws);
    if (st == VA_OK) st = prepare_operand(ctx, ivf);
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
    if (st == VA_OK) st = prepare_operand(ctx, ivf);
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
    if (ivf->op) cudaFree(ivf->op);
    if (ivf->op32 && ivf->op32_owned) cudaFree(ivf->op32);
    if (ivf->bias) cudaFree(ivf->bias);
    if (ivf->cert) cudaFree(ivf->cert);
    if (ivf->scratch) cudaFree(ivf->scratch);
    if (ivf->h_plan) cudaFreeHost(ivf->h_plan);
    delete ivf;
    return VA_OK;
}

int va_ivf_list_sizes(const va_ivf* ivf, int64_t* sizes) {
    VA_REQUIRE(ivf && sizes, "ivf and sizes must not be NULL");
    for (int c = 0; c < ivf->nlist; ++c) sizes[c] = ivf->h_offsets[(size_t)c + 1] - ivf->h_offsets[(size_t)c];
    return VA_OK;
}

int va_ivf_search(va_context* ctx, const va_ivf* civf, const float* queries, int64_t nq, int k, int nprobe,
                  float* out_vals, uint32_t* out_ids) {
    VaRange nvtx_range("va_ivf_search");
    VA_REQUIRE(ctx && civf && queries && out_vals && out_ids, "all pointers must be non-NULL");
    VA_REQUIRE(nq > 0, "numQueries must be positive, got %lld", (long long)nq);
    VA_REQUIRE(k > 0 && k <= 128, "k must be between 1 and 128 for the IVF search, got %d", k);
    VA_REQUIRE(nprobe > 0 && nprobe <= civf->nlist, "nprobe must be in 1..nlist (%d), got %d", civf->nlist, nprobe);
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    va_ivf* ivf = const_cast<va_ivf*>(civf);  // only its search scratch changes
    const int64_t m = nq * nprobe;
    VA_REQUIRE(m < ((int64_t)1 << 31) - 65536, "numQueries x nprobe (%lld) must stay below 2^31 per IVF call",
               (long long)m);
    // Pairs are ordered by probe rank in up to 8 buckets (ranks 7 and beyond together).
    const int nb = std::min(nprobe, 8);
    // Candidate pool of the tensor-core route, as the flat search's: bf16 keys with 3k (at least
    // k + max(k/4, 22)) while that fits one list of 128 per (query, probe) (k <= 42), then tf32
    // keys (4x smaller error) with k + max(k/4, 22) (k <= 103). Larger k: the exact scan.
    const int pool_bf = std::max(3 * k, k + std::max(k / 4, 22)), pool_tf = k + std::max(k / 4, 22);
    const int elem = pool_bf <= 128 ? 2 : 4;
    const int pool = elem == 2 ? pool_bf : pool_tf;
    const bool tc = pool <= 128 && ivf->n > 0;
    const int kp = pool <= 32 ? 32 : pool <= 64 ? 64 : 128;
    const int nlist = ivf->nlist;
    // Scratch: probes + their distances, then the route's arrays (sized after the plan).
    const size_t pb = round_up(m * 4, 256);
    void* ws;
    const size_t head = 2 * pb + round_up((int64_t)nlist * nb * 4, 256);
    VA_TRY(scratch(ctx, ivf, head, 0, &ws));
    uint32_t* probes = (uint32_t*)ws;
    float* pv = (float*)((uint8_t*)ws + pb);
    int* cnt = (int*)((uint8_t*)ws + 2 * pb);
    // Coarse quantization: the nprobe nearest centroids of every query (ties by list id). Up to
    // 16384 centroids the FP32 route (distance tiles + radix selection) is fastest (10K queries x
    // 1024 centroids x 128 dimensions: 0.33 ms, against 1.5 ms for the filter, whose cold lists
    // dominate at so few rows); beyond, TF32 with the default pool keeps lists of at most 128.
    const int cprec = nlist <= 16384 ? VA_PREC_FP32
                      : (ivf->dim > 16 && nprobe + std::max(nprobe / 4, 22) <= 128) ? VA_PREC_TF32
                                                                                     : VA_PREC_AUTO;
    VA_TRY(va_knn_search(ctx, ivf->cdb, queries, nq, nprobe, VA_METRIC_L2SQ, cprec, 0, pv, probes));
    if (!tc) {
        VA_REQUIRE(nq <= 65535, "numQueries %lld exceeds 65535 per IVF call for k > 103", (long long)nq);
        const size_t lb = (size_t)m * k;
        VA_TRY(scratch(ctx, ivf, pb + lb * 8 + 256, pb, &ws));  // the probes move along
        probes = (uint32_t*)ws;
        float* cv = (float*)((uint8_t*)ws + pb);
        uint32_t* ci = (uint32_t*)(cv + lb);
        const size_t smem = (size_t)ivf->dim * 4;
        if (smem > 48 * 1024)
            VA_CUDA_TRY(cudaFuncSetAttribute(k_ivf_scan, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        dim3 grid((unsigned)nprobe, (unsigned)nq);
        k_ivf_scan<<<grid, LS_THREADS, smem, ctx->stream>>>(queries, nq, ivf->dim, probes, nprobe, ivf->rows,
                                                           ivf->ids, ivf->offsets, k, cv, ci);
        VA_TRY(va_check_launch("k_ivf_scan"));
        return va_merge_lists_internal(ctx, cv, ci, nprobe, nq * k, k, nq, k, VA_SELECT_MIN, out_vals, out_ids);
    }
    // Pairs per (list, rank bucket), read back: the query tiles are laid out on the host.
    const int64_t nls = (int64_t)nlist * nb;
    VA_CUDA_TRY(cudaMemsetAsync(cnt, 0, (size_t)nls * 4, ctx->stream));
    k_probe_hist<<<grid_for(m), 256, 0, ctx->stream>>>(probes, m, nprobe, nb, cnt);
    VA_TRY(va_check_launch("k_probe_hist"));
    // Pinned plan buffer: [counts | base | lt0 | tile_of | tile_list], tiles at most m/128 + nlist.
    const int64_t nt_max = m / 128 + nlist + 1;
    const size_t plan_ints = (size_t)(2 * nls + nlist + 2 * nt_max);
    if (plan_ints > ivf->h_plan_ints) {
        if (ivf->h_plan) cudaFreeHost(ivf->h_plan);
        ivf->h_plan = nullptr;
        ivf->h_plan_ints = 0;
        if (cudaHostAlloc((void**)&ivf->h_plan, plan_ints * 4, cudaHostAllocDefault) != cudaSuccess) {
            cudaGetLastError();
            ivf->h_plan = nullptr;
            return va_set_error(VA_ERR_OOM, "pinned IVF plan buffer of %zu bytes failed", plan_ints * 4);
        }
        ivf->h_plan_ints = plan_ints;
    }
    int* h_cnt = ivf->h_plan;
    int* base = h_cnt + nls;
    int* lt0 = base + nls;
    int* tile_of = lt0 + nlist;
    int* tile_list = tile_of + nt_max;
    VA_CUDA_TRY(cudaMemcpyAsync(h_cnt, cnt, (size_t)nls * 4, cudaMemcpyDeviceToHost, ctx->stream));
    VA_TRY(va_synchronize(ctx));
    // A list's pairs in rank-bucket order, cut into query tiles of 128. Tiles run by the bucket of
    // their first pair, then longest list first: the first rounds of the persistent grid scan
    // the queries' nearest lists, whose candidates set the per-query bounds that prune the
    // farther lists' tiles. (Rank-0 pairs in tiles of their own, run in a first launch so that
    // every bound is set before the rest, measured slower: 30% more tiles, mostly padding.)
    struct TileKey {
        int rank;
        int64_t rows;
        int list, j;
    };
    std::vector<TileKey> keys;
    keys.reserve((size_t)nt_max);
    for (int L = 0; L < nlist; ++L) {
        int acc = 0;
        for (int r = 0; r < nb; ++r) {
            base[(size_t)L * nb + r] = acc;
            acc += h_cnt[(size_t)L * nb + r];
        }
        lt0[L] = (int)keys.size();
        const int64_t rows = ivf->h_offsets[(size_t)L + 1] - ivf->h_offsets[(size_t)L];
        int r = 0;
        for (int j = 0; j * 128 < acc; ++j) {
            while (r + 1 < nb && base[(size_t)L * nb + r + 1] <= j * 128) ++r;
            keys.push_back({r, rows, L, j});
        }
    }
    const int n_qtiles = (int)keys.size();
    std::vector<int> ord((size_t)n_qtiles);
    for (int i = 0; i < n_qtiles; ++i) ord[(size_t)i] = i;
    std::stable_sort(ord.begin(), ord.end(), [&](int x, int y) {
        const TileKey &a = keys[(size_t)x], &b = keys[(size_t)y];
        return a.rank != b.rank ? a.rank < b.rank : a.rows > b.rows;
    });
    for (int t = 0; t < n_qtiles; ++t) {
        const TileKey& kt = keys[(size_t)ord[(size_t)t]];
        tile_list[t] = kt.list;
        tile_of[lt0[kt.list] + kt.j] = t;
    }
    const int64_t G = (int64_t)n_qtiles * 128;
    // Scratch layout after the probes and counts; the plan keeps the pinned buffer's layout.
    size_t off = head;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off += round_up((int64_t)bytes, 256);
        return o;
    };
    const size_t plan_up = (size_t)(nls + nlist + 2 * nt_max) * 4;
    const size_t o_plan = take(plan_up), o_cur = take((size_t)nls * 4), o_gmap = take((size_t)G * 4),
                 o_ginv = take((size_t)m * 8), o_qop = take((size_t)G * ivf->dpad * elem),
                 o_pk = take((size_t)G * kp * 4), o_pi = take((size_t)G * kp * 4);
    // (Bound levels fed by the probes, a probe's rank picking its slot, measured 4% slower: the
    // nearest list's kp-th key already prunes most of the farther lists.)
    const size_t o_thr = take((size_t)G * 4);
    VA_TRY(scratch(ctx, ivf, off, pb, &ws));  // the probes move along
    uint8_t* sb = (uint8_t*)ws;
    probes = (uint32_t*)sb;
    int* d_base = (int*)(sb + o_plan);
    int* d_lt0 = d_base + nls;
    int* d_tof = d_lt0 + nlist;
    int* d_tiles = d_tof + nt_max;
    int* cursor = (int*)(sb + o_cur);
    int* gmap = (int*)(sb + o_gmap);
    int64_t* ginv = (int64_t*)(sb + o_ginv);
    void* qop = sb + o_qop;
    float* pk = (float*)(sb + o_pk);
    uint32_t* pi = (uint32_t*)(sb + o_pi);
    uint32_t* gthr = (uint32_t*)(sb + o_thr);
    VA_CUDA_TRY(cudaMemcpyAsync(d_base, base, plan_up, cudaMemcpyHostToDevice, ctx->stream));
    VA_CUDA_TRY(cudaMemsetAsync(cursor, 0, (size_t)nls * 4, ctx->stream));
    VA_CUDA_TRY(cudaMemsetAsync(gmap, 0xFF, (size_t)G * 4, ctx->stream));
    k_probe_scatter<<<grid_for(m), 256, 0, ctx->stream>>>(probes, m, nprobe, nb, d_base, cursor, d_lt0, d_tof,
                                                          gmap, ginv);
    VA_TRY(va_check_launch("k_probe_scatter"));
    if (elem == 2)
        k_rows_op<uint16_t><<<grid_for(G * ivf->dpad), 256, 0, ctx->stream>>>(queries, G, ivf->dim, ivf->dpad, gmap,
                                                                               nprobe, (uint16_t*)qop);
    else
        k_rows_op<float><<<grid_for(G * ivf->dpad), 256, 0, ctx->stream>>>(queries, G, ivf->dim, ivf->dpad, gmap,
                                                                            nprobe, (float*)qop);
    VA_TRY(va_check_launch("k_rows_op"));
    if (elem == 4 && !ivf->op32) {
        // The fp32 operand, on first use: the rows themselves when they need no padding.
        if (ivf->dim == ivf->dpad) {
            ivf->op32 = ivf->rows;
        } else {
            if (cudaMalloc((void**)&ivf->op32, (size_t)ivf->n * ivf->dpad * 4) != cudaSuccess) {
                cudaGetLastError();
                ivf->op32 = nullptr;
                return va_set_error(VA_ERR_OOM, "IVF fp32 operand allocation failed");
            }
            ivf->op32_owned = true;
            k_rows_op<float><<<grid_for(ivf->n * ivf->dpad), 256, 0, ctx->stream>>>(ivf->rows, ivf->n, ivf->dim,
                                                                                     ivf->dpad, nullptr, 1, ivf->op32);
            VA_TRY(va_check_launch("k_rows_op"));
        }
    }
    TcFilterArgs a = {};
    a.q_op = qop;
    a.x_op = elem == 2 ? (const void*)ivf->op : (const void*)ivf->op32;
    a.elem_bytes = elem;
    a.dpad = ivf->dpad;
    a.n_rows = ivf->n;
    a.row_bias = ivf->bias;
    a.alpha = -2.f;
    a.row_qn = nullptr;
    a.part_keys = pk;
    a.part_ids = pi;
    a.gthr = gthr;
    a.sync_cnt = nullptr;
    a.sync_words = 0;
    a.limit_ms = 2000u;
    // Fail count and list of the certificate (context aux buffer: the coarse step is done with it).
    void* aux;
    VA_TRY(va_aux_buffer(ctx, 256 + round_up(nq * 4, 256), &aux));
    uint32_t* fail_cnt = (uint32_t*)aux;
    uint32_t* fail_list = (uint32_t*)((uint8_t*)aux + 256);
    VA_CUDA_TRY(cudaMemsetAsync(fail_cnt, 0, 4, ctx->stream));
    VA_TRY(va_tc_filter_lists(ctx, a, n_qtiles, 0, n_qtiles, d_tiles, ivf->offsets, gmap, nprobe, kp, true));
    k_ivf_merge_rerank<<<(unsigned)nq, MR_THREADS, 0, ctx->stream>>>(
        queries, ivf->dim, ginv, nprobe, pk, pi, kp, pool, k, ivf->rows, ivf->ids, ivf->cert,
        elem == 2 ? VA_CERT_BF16 : VA_CERT_TF32, ivf->dpad, out_vals, out_ids, fail_list, fail_cnt, gthr);
    VA_TRY(va_check_launch("k_ivf_merge_rerank"));
    // Queries the certificate could not prove: an exact fp64 scan of their probed lists.
    uint32_t nf = 0;
    VA_TRY(va_read_u32(ctx, fail_cnt, &nf));
    ctx->stat_uncertified = nf;
    ctx->stat_exact = nf;
    if (!nf) return VA_OK;
    VA_REQUIRE(nf <= 65535, "%u uncertified IVF queries exceed one exact rescan (65535)", nf);
    const size_t gq = round_up((int64_t)nf * ivf->dim * 4, 256), gp = round_up((int64_t)nf * nprobe * 4, 256),
                 lb = (size_t)nprobe * nf * k, rb = round_up((int64_t)nf * k * 4, 256);
    void* ws2;
    VA_TRY(va_workspace(ctx, gq + gp + lb * 8 + 2 * rb + 256, &ws2));
    float* fq = (float*)ws2;
    uint32_t* fp = (uint32_t*)((uint8_t*)ws2 + gq);
    float* cv = (float*)((uint8_t*)fp + gp);
    uint32_t* ci = (uint32_t*)(cv + lb);
    float* fv = (float*)(ci + lb);
    uint32_t* fi = (uint32_t*)((uint8_t*)fv + rb);
    k_gather_rows_t<float><<<grid_for((int64_t)nf * ivf->dim), 256, 0, ctx->stream>>>(queries, ivf->dim, fail_list,
                                                                                      nf, fq);
    k_gather_rows_t<uint32_t><<<grid_for((int64_t)nf * nprobe), 256, 0, ctx->stream>>>(probes, nprobe, fail_list, nf,
                                                                                       fp);
    VA_TRY(va_check_launch("k_gather_rows_t"));
    const size_t smem = (size_t)ivf->dim * 4;
    if (smem > 48 * 1024)
        VA_CUDA_TRY(cudaFuncSetAttribute(k_ivf_scan, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    k_ivf_scan<<<dim3((unsigned)nprobe, nf), LS_THREADS, smem, ctx->stream>>>(fq, nf, ivf->dim, fp, nprobe, ivf->rows,
                                                                              ivf->ids, ivf->offsets, k, cv, ci);
    VA_TRY(va_check_launch("k_ivf_scan"));
    VA_TRY(va_merge_lists_internal(ctx, cv, ci, nprobe, (int64_t)nf * k, k, nf, k, VA_SELECT_MIN, fv, fi));
    k_scatter_rows<<<grid_for((int64_t)nf * k), 256, 0, ctx->stream>>>(fv, fi, fail_list, nf, k, out_vals, out_ids);
    return va_check_launch("k_scatter_rows");
}

int va_ivf_search_host(va_context* ctx, const va_ivf* ivf, const float* queries_host, int64_t nq, int k, int nprobe,
                       float* out_vals_host, uint32_t* out_ids_host) {
    VA_REQUIRE(ctx && ivf && queries_host && out_vals_host && out_ids_host, "all pointers must be non-NULL");
    VA_REQUIRE(nq > 0 && k > 0, "numQueries and k must be positive");
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    const size_t qb = (size_t)nq * ivf->dim * 4, rb = (size_t)nq * k * 4;
    void* io;
    VA_TRY(va_io_buffer(ctx, round_up((int64_t)qb, 256) + 2 * round_up((int64_t)rb, 256), &io));
    float* dq = (float*)io;
    float* dv = (float*)((uint8_t*)io + round_up((int64_t)qb, 256));
    uint32_t* di = (uint32_t*)((uint8_t*)dv + round_up((int64_t)rb, 256));
    VA_TRY(va_copy_to_device(ctx, dq, queries_host, qb));
    VA_TRY(va_ivf_search(ctx, ivf, dq, nq, k, nprobe, dv, di));
    VA_TRY(va_copy_to_host(ctx, out_vals_host, dv, rb));
    VA_TRY(va_copy_to_host(ctx, out_ids_host, di, rb));
    return va_synchronize(ctx);
}

}  // extern "C"
