// va_tc.cu -- tensor-core fused distance + top-k' candidate filter (sm_100a, tcgen05/TMEM/TMA).
//
// Replaces the contraction inside FusedL2TopKKernel (fused_l2_topk, AdvancedTopK.metal:204-314;
// l2_distance_kernel, L2Distance.metal:34-91; dot_product_kernel, DotProduct.metal:29-96):
// instead of one threadgroup per query re-reading every database row, a persistent CTA per SM
// runs 128 queries x 256 rows x K tiles on the 5th-generation tensor cores.
//
//   warp 0        TMA producer: query tile (A, 128 x 128 B) and row tile (B, 256 x 128 B) per
//                 K block into a STAGES-deep ring of 128B-swizzled shared-memory slots
//   warp 1        TMEM owner (allocates 2 x 256 fp32 columns) and single-thread MMA issuer:
//                 4 tcgen05.mma per K block into the current accumulator, tcgen05.commit frees
//                 the slot; a final commit hands the accumulator to the epilogue
//   warps 2..5    epilogue: tcgen05.ld 32 columns at a time (one query row per thread), forms
//                 key = alpha * (q.x) + |x|^2 term, and keeps a per-query sorted list of the KP
//                 best (key, id) in shared memory, touched only when a key beats the KP-th best
//
// Every (query tile, row split) item starts its lists empty, so without help each item would
// re-insert its first KP candidates and ~KP*ln(rows/KP) more. Items therefore share one bound per
// query in global memory: a finished item publishes its KP-th key (atomicMin on the orderable
// key); others drop keys above the smallest published bound. The bound is the KP-th key of a
// subset of rows, never below the global KP-th key, so no candidate of the final pool is lost.
//
// Two accumulators let the epilogue of tile t overlap the MMAs of tile t+1. The distance
// matrix never reaches HBM: per (query tile, row split) work item each query's KP best
// approximate candidates are written out, merged across splits and exactly reranked in fp64
// by va_search.cu. Every wait is bounded on the global timer; on expiry the kernel sets the
// context's device error word, stops issuing work and still frees its TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>

#include "va_internal.cuh"
#include "va_tc.cuh"

namespace {

constexpr int BM = 128;           // queries per tile (TMEM lanes)
constexpr int BN = 256;           // database rows per tile (TMEM columns per accumulator)
constexpr int BKB = 128;          // bytes of K per stage (one 128B swizzle row)
constexpr int A_BYTES = BM * BKB; // 16 KB
constexpr int B_BYTES = BN * BKB; // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int NUM_THREADS = 192;
constexpr int TMEM_COLS = 512;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: returns false (after flagging) when the limit expires or another role aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err,
                                          uint64_t limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = va::globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 255u) == 0) {
            if (*abort_flag) return false;
            if (va::globaltimer_ns() - t0 > limit_ns) {
                *abort_flag = 1;
                atomicExch(err, VA_DEVERR_WAIT_TIMEOUT);
                return false;
            }
        }
    }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::
            "r"(smem_u32(dst)),
        "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// UMMA shared-memory descriptor: K-major, 128B swizzle, 8-row atoms 1024 B apart (SBO),
// descriptor version 1 (sm_100).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFFu);
    d |= (uint64_t)1u << 16;             // LBO (unused for swizzled K-major), 16 B
    d |= (uint64_t)(1024u >> 4) << 32;   // SBO = 1024 B
    d |= (uint64_t)1u << 46;             // version 1
    d |= (uint64_t)2u << 61;             // SWIZZLE_128B
    return d;
}

template <int ELEM>
struct Kind;
template <>
struct Kind<2> {  // bf16 x bf16 -> fp32
    static constexpr uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                      ((uint32_t)(BM >> 4) << 24);
    __device__ static __forceinline__ void mma(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t acc) {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
            "l"(a), "l"(b), "r"(idesc), "r"(acc));
    }
};
template <>
struct Kind<4> {  // tf32 x tf32 -> fp32
    static constexpr uint32_t idesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                      ((uint32_t)(BM >> 4) << 24);
    __device__ static __forceinline__ void mma(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t acc) {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
            "l"(a), "l"(b), "r"(idesc), "r"(acc));
    }
};

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t addr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(addr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Insert (key, id) into the sorted list of query `row` (entries [j*BM + row], j < KP) and return
// the list's new KP-th key. Called only when key beats the current threshold, so it is kept out
// of line to keep the hot loop small. Candidates arrive in increasing id order: a key equal to an
// entry goes after it, which is the (key, id) order.
template <int KP>
__device__ __noinline__ float list_insert(float* lk, uint32_t* li, int row, float key, uint32_t id) {
    int p = KP - 1;
    while (p > 0) {
        const float prev = lk[(p - 1) * BM + row];
        if (prev <= key) break;
        lk[p * BM + row] = prev;
        li[p * BM + row] = li[(p - 1) * BM + row];
        --p;
    }
    lk[p * BM + row] = key;
    li[p * BM + row] = id;
    return lk[(KP - 1) * BM + row];
}

// Smallest float strictly above v (v finite or +inf).
__device__ __forceinline__ float next_up(float v) {
    if (v == INFINITY) return v;
    return nextafterf(v, INFINITY);
}

// Filter bound from the shared per-query key (0xFFFFFFFF = nothing published yet): the next
// float above the published key, so keys equal to it still pass.
__device__ __forceinline__ float load_bound(const uint32_t* g) {
    const uint32_t k = __ldcg(g);
    return k == 0xFFFFFFFFu ? INFINITY : next_up(va::key2f(k));
}

struct Work {
    int n_qtiles;
    int splits;
    int n_tiles;      // database tiles of BN rows
    int k_blocks;     // K blocks of BKB bytes
    int64_t n_rows;   // database rows
    int64_t nq_pad;   // n_qtiles * BM
};

__device__ __forceinline__ void item_range(const Work& w, int item, int& qt, int& t0, int& t1) {
    const int s = item / w.n_qtiles;
    qt = item - s * w.n_qtiles;
    t0 = (int)(((int64_t)w.n_tiles * s) / w.splits);
    t1 = (int)(((int64_t)w.n_tiles * (s + 1)) / w.splits);
}

template <int ELEM, int KP>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    k_tc_filter(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_x, Work w,
                const float* __restrict__ row_bias, float alpha, float* __restrict__ part_keys,
                uint32_t* __restrict__ part_ids, uint32_t* __restrict__ gthr, int* err, uint64_t limit_ns,
                int stages) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte alignment for the 128B-swizzled operand slots.
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* sA = smem;
    uint8_t* sB = smem + (size_t)stages * A_BYTES;
    float* l_key = (float*)(sB + (size_t)stages * B_BYTES);       // [KP][BM]
    uint32_t* l_id = (uint32_t*)(l_key + KP * BM);                 // [KP][BM]
    uint64_t* bars = (uint64_t*)(l_id + KP * BM);                  // full[stages], empty[stages], tfull[2], tempty[2]
    uint64_t* full = bars;
    uint64_t* empty = bars + stages;
    uint64_t* tfull = bars + 2 * stages;
    uint64_t* tempty = tfull + 2;
    uint32_t* s_tmem = (uint32_t*)(tempty + 2);
    volatile int* s_abort = (volatile int*)(s_tmem + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_items = w.n_qtiles * w.splits;

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 4);
        }
        *s_abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_q) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_x) : "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(s_tmem)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *s_tmem;

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producer
        if (lane == 0) {
            uint32_t it = 0;
            for (int item = blockIdx.x; item < n_items && !*s_abort; item += gridDim.x) {
                int qt, t0, t1;
                item_range(w, item, qt, t0, t1);
                for (int t = t0; t < t1; ++t) {
                    for (int kb = 0; kb < w.k_blocks; ++kb, ++it) {
                        const int s = it % stages;
                        const uint32_t ph = (it / stages) & 1u;
                        if (!mbar_wait(&empty[s], ph ^ 1u, s_abort, err, limit_ns)) goto producer_done;
                        mbar_expect_tx(&full[s], STAGE_BYTES);
                        const int kc = kb * (BKB / ELEM);
                        tma_load_2d(sA + (size_t)s * A_BYTES, &tmap_q, &full[s], kc, qt * BM);
                        tma_load_2d(sB + (size_t)s * B_BYTES, &tmap_x, &full[s], kc, t * BN);
                    }
                }
            }
        producer_done:;
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            uint32_t it = 0, tile = 0;
            for (int item = blockIdx.x; item < n_items && !*s_abort; item += gridDim.x) {
                int qt, t0, t1;
                item_range(w, item, qt, t0, t1);
                for (int t = t0; t < t1; ++t, ++tile) {
                    const uint32_t buf = tile & 1u;
                    const uint32_t tph = (tile >> 1) & 1u;
                    if (!mbar_wait(&tempty[buf], tph ^ 1u, s_abort, err, limit_ns)) goto mma_done;
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + buf * BN;
                    for (int kb = 0; kb < w.k_blocks; ++kb, ++it) {
                        const int s = it % stages;
                        const uint32_t ph = (it / stages) & 1u;
                        if (!mbar_wait(&full[s], ph, s_abort, err, limit_ns)) goto mma_done;
                        tc_fence_after();
                        const uint32_t a0 = smem_u32(sA + (size_t)s * A_BYTES);
                        const uint32_t b0 = smem_u32(sB + (size_t)s * B_BYTES);
#pragma unroll
                        for (int j = 0; j < BKB / 32; ++j) {
                            Kind<ELEM>::mma(d_tmem, smem_desc(a0 + 32 * j), smem_desc(b0 + 32 * j),
                                            (kb | j) ? 1u : 0u);
                        }
                        mma_commit(&empty[s]);
                    }
                    mma_commit(&tfull[buf]);
                }
            }
        mma_done:;
        }
    } else {
        // ---------------------------------------------------------------- epilogue (warps 2..5)
        // Thresholds: thr_own = this item's KP-th best key; thr_g = the smallest KP-th key any
        // finished item published for this query (an upper bound of the global KP-th key, so a
        // key above it can never reach the final pool). A candidate is inserted when
        // key < min(thr_own, next_up(thr_g)).
        const int quarter = warp & 3;             // TMEM lane quarter this warp may access
        const int row = quarter * 32 + lane;      // query row within the tile
        uint32_t tile = 0;
        for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
            int qt, t0, t1;
            item_range(w, item, qt, t0, t1);
            const int64_t q = (int64_t)qt * BM + row;
            for (int j = 0; j < KP; ++j) {
                l_key[j * BM + row] = INFINITY;
                l_id[j * BM + row] = va::kInvalidId;
            }
            float thr_own = INFINITY;
            float thr_g = load_bound(gthr + q);
            float thr = thr_g;
            for (int t = t0; t < t1; ++t, ++tile) {
                if (((t - t0) & 7) == 7) {
                    thr_g = load_bound(gthr + q);
                    thr = fminf(thr_own, thr_g);
                }
                const uint32_t buf = tile & 1u;
                const uint32_t tph = (tile >> 1) & 1u;
                // One lane waits; the warp follows its verdict so tcgen05.ld stays warp-uniform.
                int ok = 1;
                if (lane == 0) ok = mbar_wait(&tfull[buf], tph, s_abort, err, limit_ns) ? 1 : 0;
                ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
                if (!ok) goto epi_done;
                tc_fence_after();
                const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + buf * BN;
                const int64_t col0 = (int64_t)t * BN;
                // The tile's 256 row biases (|x|^2 for L2, 0 otherwise; +inf past the last row)
                // live 8 per lane and are broadcast by shuffles.
                const float4* bp = (const float4*)(row_bias + col0) + lane * 2;
                const float4 b0 = __ldg(bp), b1 = __ldg(bp + 1);
                const float bias[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll 1
                for (int c = 0; c < BN / 32; ++c) {
                    __syncwarp();
                    float v[32];
                    tmem_ld32(taddr + c * 32, v);
                    const uint32_t cb = (uint32_t)(col0 + c * 32);
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const float nb = __shfl_sync(0xFFFFFFFFu, bias[i & 7], c * 4 + (i >> 3));
                        const float key = fmaf(alpha, v[i], nb);
                        if (key < thr) {
                            thr_own = list_insert<KP>(l_key, l_id, row, key, cb + i);
                            thr = fminf(thr_own, thr_g);
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[buf]);
            }
            {
                // Publish this item's KP-th key (finite once the list is full) as a bound.
                if (thr_own < INFINITY) atomicMin(gthr + q, va::f2key(thr_own));
                const int s = item / w.n_qtiles;
                float* pk = part_keys + ((int64_t)s * w.nq_pad + q) * KP;
                uint32_t* pi = part_ids + ((int64_t)s * w.nq_pad + q) * KP;
#pragma unroll 4
                for (int j = 0; j < KP; ++j) {
                    pk[j] = l_key[j * BM + row];
                    pi[j] = l_id[j * BM + row];
                }
            }
        }
    epi_done:;
    }
    // Single-lane roles (producer, MMA issuer) rejoin their warps before the block barrier.
    __syncwarp();

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS));
    }
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void* p = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
    }
    return fn;
}

int make_tmap(CUtensorMap* map, const void* base, int64_t rows, int64_t cols_elems, int elem_bytes, int box_rows) {
    auto enc = get_encode_fn();
    if (!enc) return va_set_error(VA_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
    cuuint64_t dims[2] = {(cuuint64_t)cols_elems, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(cols_elems * elem_bytes)};
    cuuint32_t box[2] = {(cuuint32_t)(BKB / elem_bytes), (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                     const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return va_set_error(VA_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
    return VA_OK;
}

template <int ELEM, int KP>
int launch_filter(va_context* ctx, const TcFilterArgs& a, int stages, size_t smem, const CUtensorMap& mq,
                  const CUtensorMap& mx, const Work& w, int grid) {
    auto kern = k_tc_filter<ELEM, KP>;
    VA_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    VA_CUDA_TRY(cudaMemsetAsync(a.gthr, 0xFF, (size_t)w.nq_pad * sizeof(uint32_t), ctx->stream));
    kern<<<grid, NUM_THREADS, smem, ctx->stream>>>(mq, mx, w, a.row_bias, a.alpha, a.part_keys, a.part_ids, a.gthr,
                                                   ctx->d_error, (uint64_t)a.limit_ms * 1000000ull, stages);
    return va_check_launch("k_tc_filter");
}

}  // namespace

// Plan of a filter launch (host side, shared with va_search.cu).
int va_tc_plan(va_context* ctx, int64_t nq, int64_t n_rows, int kp, TcPlan* plan) {
    plan->n_qtiles = (int)((nq + BM - 1) / BM);
    plan->n_tiles = (int)((n_rows + BN - 1) / BN);
    plan->nq_pad = (int64_t)plan->n_qtiles * BM;
    // Splits: make (query tiles x splits) a multiple of the SM count so every CTA gets the same
    // number of equally sized items, but never split finer than one row tile.
    int g = ctx->sm_count;
    int a = plan->n_qtiles, b = g;
    while (b) {
        int t = a % b;
        a = b;
        b = t;
    }
    int splits = g / a;
    splits = std::max(1, std::min(splits, plan->n_tiles));
    plan->splits = splits;
    plan->kp = kp;
    plan->grid = std::min(plan->n_qtiles * splits, g);
    return VA_OK;
}

size_t va_tc_smem_bytes(int kp, int stages) {
    return 1024 + (size_t)stages * STAGE_BYTES + (size_t)kp * BM * 8 + (2 * stages + 4) * 8 + 16;
}

int va_tc_stages(int kp) {
    for (int s = 6; s >= 2; --s)
        if (va_tc_smem_bytes(kp, s) <= 227 * 1024) return s;
    return 0;
}

int va_tc_filter(va_context* ctx, const TcFilterArgs& a, const TcPlan& p) {
    const int elem = a.elem_bytes;
    CUtensorMap mq, mx;
    VA_TRY(make_tmap(&mq, a.q_op, p.nq_pad, a.dpad, elem, BM));
    VA_TRY(make_tmap(&mx, a.x_op, a.n_rows, a.dpad, elem, BN));
    Work w;
    w.n_qtiles = p.n_qtiles;
    w.splits = p.splits;
    w.n_tiles = p.n_tiles;
    w.k_blocks = (int)((a.dpad * elem + BKB - 1) / BKB);
    w.n_rows = a.n_rows;
    w.nq_pad = p.nq_pad;
    const int stages = va_tc_stages(p.kp);
    if (stages < 2) return va_set_error(VA_ERR_UNSUPPORTED, "candidate pool %d too large for shared memory", p.kp);
    const size_t smem = va_tc_smem_bytes(p.kp, stages);
    if (elem == 2) {
        if (p.kp == 32) return launch_filter<2, 32>(ctx, a, stages, smem, mq, mx, w, p.grid);
        if (p.kp == 64) return launch_filter<2, 64>(ctx, a, stages, smem, mq, mx, w, p.grid);
    } else {
        if (p.kp == 32) return launch_filter<4, 32>(ctx, a, stages, smem, mq, mx, w, p.grid);
        if (p.kp == 64) return launch_filter<4, 64>(ctx, a, stages, smem, mq, mx, w, p.grid);
    }
    return va_set_error(VA_ERR_UNSUPPORTED, "candidate pool %d not supported by the tensor-core filter", p.kp);
}
