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
//   warps 2..5    epilogue: tcgen05.ld 64 columns at a time (one query row per thread, loads
//                 double-buffered), forms key = alpha * (q.x) + row bias (|x|^2 for L2; the
//                 exact integer distance for int8 / bit codes) with the biases broadcast by
//                 shuffles, and keeps a sorted list of each query's KP best (key, id) in shared
//                 memory. A warp-uniform test per 64-column chunk skips the lists; otherwise the
//                 candidates are inserted one at a time by the whole warp (few candidates) or by
//                 every lane into its own row at once (many; lists of every size)
//
// Every (query tile, row split) item starts its lists empty, so without help each item would
// re-insert its first KP candidates and ~KP*ln(rows/KP) more. Items therefore share a bound per
// query in global memory, in levels of slots fed with list keys of several ranks (see
// Work::lv); keys above it are dropped, and it never cuts into the final candidate pool.
//
// The producers of all CTAs advance through row chunks in loose lockstep (each CTA at most two
// 16-tile chunks ahead of the slowest), so the 2-3 row splits in flight stay in L2 and each row is
// read from HBM about once per launch (measured 24 GB of DRAM reads for the 15.4 GB operand).
//
// Two accumulators let the epilogue of tile t overlap the MMAs of tile t+1. The distance
// matrix never reaches HBM: per (query tile, row split) work item each query's KP best
// approximate candidates are written out, merged across splits and exactly reranked in fp64
// by va_search.cu. Every wait is bounded on the global timer; on expiry the kernel sets the
// context's device error word, stops issuing work and still frees its TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>

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

// Teardown after an abort: wait (bounded by limit_ns, ignoring the abort flag) for a phase that
// work already in flight will complete: a TMA load's bytes landing, or a tcgen05.commit.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
    if (mbar_try_wait(bar, parity)) return;
    const uint64_t t0 = va::globaltimer_ns();
    while (!mbar_try_wait(bar, parity))
        if (va::globaltimer_ns() - t0 > limit_ns) return;
}

// Bound of each teardown wait: in-flight copies and MMAs finish within microseconds.
constexpr uint64_t kDrainLimitNs = 1000000000ull;

// The producer's teardown after an abort: every TMA load it issued into the stage ring (the last
// min(stages, issued) iterations) has landed before the CTA may exit.
__device__ __forceinline__ void drain_loads(uint64_t* full, int stages, uint32_t issued) {
    const uint32_t first = issued > (uint32_t)stages ? issued - (uint32_t)stages : 0u;
    for (uint32_t i = first; i < issued; ++i) mbar_drain(&full[i % stages], (i / stages) & 1u, kDrainLimitNs);
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
struct Kind<1> {  // s8 x s8 -> s32 (exact)
    static constexpr uint32_t idesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                      ((uint32_t)(BM >> 4) << 24);
    __device__ static __forceinline__ void mma(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t acc) {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
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

// Issue a 64-column TMEM load (one accumulator row per thread); the registers are valid only
// after tmem_wait64 on the same array.
__device__ __forceinline__ void tmem_ld64(uint32_t addr, uint32_t (&r)[64]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x64.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,"
        "%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
        "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
          "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
          "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
          "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
          "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
        : "r"(addr));
}

// Wait for every outstanding TMEM load of this thread. The array is an in/out operand so the
// compiler cannot move any use of its registers above the wait.
__device__ __forceinline__ void tmem_wait64(uint32_t (&r)[64]) {
    asm volatile(
        "tcgen05.wait::ld.sync.aligned;"
        : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
          "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]),
          "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
          "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31]),
          "+r"(r[32]), "+r"(r[33]), "+r"(r[34]), "+r"(r[35]), "+r"(r[36]), "+r"(r[37]), "+r"(r[38]), "+r"(r[39]),
          "+r"(r[40]), "+r"(r[41]), "+r"(r[42]), "+r"(r[43]), "+r"(r[44]), "+r"(r[45]), "+r"(r[46]), "+r"(r[47]),
          "+r"(r[48]), "+r"(r[49]), "+r"(r[50]), "+r"(r[51]), "+r"(r[52]), "+r"(r[53]), "+r"(r[54]), "+r"(r[55]),
          "+r"(r[56]), "+r"(r[57]), "+r"(r[58]), "+r"(r[59]), "+r"(r[60]), "+r"(r[61]), "+r"(r[62]), "+r"(r[63])
        :
        : "memory");
}

// Candidate lists live in shared memory row-contiguous: query row r owns keys lk[r*KP + j] and
// ids li[r*KP + j], j < KP, sorted by (key, id). The 32 lanes of a warp update one row's list
// together: lane l holds entries l, l + 32, ... (E = KP / 32 per lane).
//
// Row stride of the candidate lists in shared memory: KP + 1, so that both one row read by the
// whole warp (warp-cooperative insertion) and 32 rows read one entry each (per-lane insertion) touch
// 32 different banks. (128-entry lists with stride 129 still leave room for the stages the
// kernels had with stride 128: 2 single-CTA stages, 3 pair stages.)
template <int KP>
constexpr int list_stride() { return KP + 1; }

// Insert (key, id) into row r's list (warp-uniform arguments) and return the new KP-th key.
// The position is the number of entries <= key (candidates arrive in increasing id order, so an
// equal key goes after the entries already there: the (key, id) order); entries from the position
// on move up one slot with a shuffle. No loop over KP, no serial shared-memory chain.
template <int KP>
__device__ __forceinline__ float warp_list_insert(float* lk, uint32_t* li, int r, float key, uint32_t id, int lane) {
    constexpr int E = KP / 32;
    float ek[E];
    uint32_t ei[E];
#pragma unroll
    for (int k = 0; k < E; ++k) {
        ek[k] = lk[r * list_stride<KP>() + k * 32 + lane];
        ei[k] = li[r * list_stride<KP>() + k * 32 + lane];
    }
    int pos = 0;
#pragma unroll
    for (int k = 0; k < E; ++k) pos += __popc(__ballot_sync(0xFFFFFFFFu, ek[k] <= key));
    float last = 0.f;
#pragma unroll
    for (int k = E - 1; k >= 0; --k) {
        // previous entry (position p - 1) of this lane's slot p = 32k + lane
        float pk = __shfl_up_sync(0xFFFFFFFFu, ek[k], 1);
        uint32_t pi = __shfl_up_sync(0xFFFFFFFFu, ei[k], 1);
        if (k > 0) {
            const float wk = __shfl_sync(0xFFFFFFFFu, ek[k - 1], 31);
            const uint32_t wi = __shfl_sync(0xFFFFFFFFu, ei[k - 1], 31);
            if (lane == 0) {
                pk = wk;
                pi = wi;
            }
        }
        const int p = 32 * k + lane;
        if (p >= pos) {
            const float nk = p == pos ? key : pk;
            const uint32_t ni = p == pos ? id : pi;
            lk[r * list_stride<KP>() + p] = nk;
            li[r * list_stride<KP>() + p] = ni;
            if (k == E - 1) last = nk;
        } else if (k == E - 1) {
            last = ek[k];
        }
    }
    return __shfl_sync(0xFFFFFFFFu, last, 31);
}

// Insert (key, id) into this lane's own row list (key below the row's KP-th key): entries
// greater than key move up one slot from the end (the KP-th drops out), an equal key goes after
// the entries already there. Returns the new KP-th key.
template <int KP>
__device__ __forceinline__ float lane_list_insert(float* lk, uint32_t* li, int r, float key, uint32_t id) {
    float* k = lk + r * list_stride<KP>();
    uint32_t* d = li + r * list_stride<KP>();
    int p = KP - 1;
    for (; p > 0; --p) {
        const float prev = k[p - 1];
        if (!(prev > key)) break;
        k[p] = prev;
        d[p] = d[p - 1];
    }
    k[p] = key;
    d[p] = id;
    return k[KP - 1];
}

// One 64-column chunk C (compile-time, so every shuffle reads a fixed register of a fixed lane).
// Fast path: key = alpha * acc + bias (bias of column 64C + i sits in lane i % 32, register
// 2C + i / 32) kept in place in r, eight partial minima, and one warp-uniform branch. Cold path,
// when some lane's minimum beats its threshold: each lane marks its passing columns; the warp
// then inserts the marked candidates one at a time (lowest lane first, each lane in column
// order), re-checking each against the owning lane's current threshold.
//
// Integer mode (INTK, int8 codes with int32 accumulation): the key is the exact integer distance
// bias - 2 * acc + qn (bias = |x|^2 of the codes, or |x| of 0/1 codes; qn the same for the
// query), stored as the bit pattern of a non-negative float, which orders like the integer. Rows
// past n_rows are excluded by id in the cold path.
template <int C, int KP, bool INTK>
__device__ __forceinline__ void filter_chunk(uint32_t (&r)[64], const float (&bias)[8], float alpha, int qn,
                                             uint32_t id0, uint32_t n_rows, float* lk, uint32_t* li, int row0,
                                             int lane, float thr_g, float& thr_own, float& thr) {
    float mn[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) mn[j] = INFINITY;
#pragma unroll
    for (int i = 0; i < 64; ++i) {
        const float b = __shfl_sync(0xFFFFFFFFu, bias[2 * C + (i >> 5)], i & 31);
        float key;
        if constexpr (INTK)
            key = __int_as_float(__float_as_int(b) - 2 * (int)r[i] + qn);
        else
            key = fmaf(alpha, __uint_as_float(r[i]), b);
        r[i] = __float_as_uint(key);
        mn[i & 7] = fminf(mn[i & 7], key);
    }
    const float m = fminf(fminf(fminf(mn[0], mn[1]), fminf(mn[2], mn[3])), fminf(fminf(mn[4], mn[5]), fminf(mn[6], mn[7])));
    if (!__any_sync(0xFFFFFFFFu, m < thr)) return;
    uint64_t pass = 0;
#pragma unroll
    for (int i = 0; i < 64; ++i) pass |= (uint64_t)(__uint_as_float(r[i]) < thr) << i;
    // Lanes with marked columns park their keys in thread-local memory for indexed reads.
    float kk[64];
    if (pass) {
#pragma unroll
        for (int i = 0; i < 64; ++i) kk[i] = __uint_as_float(r[i]);
    }
    {
        // Many candidates in the chunk (a cold list, or a dense pool): each lane inserts its own
        // candidates into its own row in column order, all lanes at once.
        const unsigned total = __reduce_add_sync(0xFFFFFFFFu, (unsigned)__popcll(pass));
        if (total >= 8u) {
            while (__any_sync(0xFFFFFFFFu, pass != 0)) {
                if (pass) {
                    const int i = __ffsll((long long)pass) - 1;
                    pass &= pass - 1;
                    const float key = kk[i];
                    if (key < thr && id0 + (uint32_t)i < n_rows) {
                        thr_own = lane_list_insert<KP>(lk, li, row0 + lane, key, id0 + (uint32_t)i);
                        thr = fminf(thr_own, thr_g);
                    }
                }
            }
            return;
        }
    }
    for (;;) {
        const uint32_t lanes = __ballot_sync(0xFFFFFFFFu, pass != 0);
        if (!lanes) break;
        const int L = __ffs(lanes) - 1;
        // the leader's lowest marked column and its key, broadcast to the warp
        int i = 0;
        float key = 0.f;
        if (lane == L) {
            i = __ffsll((long long)pass) - 1;
            pass &= pass - 1;
            key = kk[i];
        }
        i = __shfl_sync(0xFFFFFFFFu, i, L);
        key = __shfl_sync(0xFFFFFFFFu, key, L);
        const float thrL = __shfl_sync(0xFFFFFFFFu, thr, L);
        if (key < thrL && id0 + (uint32_t)i < n_rows) {
            const float kth = warp_list_insert<KP>(lk, li, row0 + L, key, id0 + (uint32_t)i, lane);
            if (lane == L) {
                thr_own = kth;
                thr = fminf(thr_own, thr_g);
            }
        }
    }
}

// Smallest float strictly above v (v finite or +inf).
__device__ __forceinline__ float next_up(float v) {
    if (v == INFINITY) return v;
    return nextafterf(v, INFINITY);
}

// Filter bound from the shared per-query slots (0xFFFFFFFF = nothing published yet): per level
// the largest slot (infinite while one is empty), the smallest over levels, then the next float
// above it so keys equal to it still pass. g points at this query's column of slot 0.
__device__ __forceinline__ float load_bound(const uint32_t* g, int64_t stride, const BoundLevels& lv) {
    float best = INFINITY;
    for (int l = 0; l < lv.n; ++l) {
        const uint32_t* gl = g + (int64_t)lv.off[l] * stride;
        const int ns = lv.slots[l];
        uint32_t m = 0;
        bool empty = false;
        // Eight independent loads in flight per batch (the slots sit in L2).
        for (int s0 = 0; s0 < ns; s0 += 8) {
            uint32_t v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = s0 + j < ns ? __ldcg(gl + (s0 + j) * stride) : 0u;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                empty |= v[j] == 0xFFFFFFFFu;
                m = v[j] > m ? v[j] : m;
            }
        }
        if (!empty) best = fminf(best, next_up(va::key2f(m)));
    }
    return best;
}

// Publish a list's keys at each level's rank into the item's slot of that level.
__device__ __forceinline__ void publish_bound(uint32_t* g, int64_t stride, const BoundLevels& lv, int split,
                                              const float* row_keys) {
    for (int l = 0; l < lv.n; ++l) {
        const float v = row_keys[lv.rank[l] - 1];
        if (v < INFINITY) atomicMin(g + (int64_t)(lv.off[l] + split % lv.slots[l]) * stride, va::f2key(v));
    }
}

struct Work {
    int n_qtiles;
    int splits;
    int n_tiles;      // database tiles of BN rows
    int k_blocks;     // K blocks of BKB bytes
    int64_t n_rows;   // database rows
    int64_t nq_pad;   // n_qtiles * BM
    // Lockstep over row chunks (see the producer): chunk_tiles tiles per chunk, cpr chunk slots
    // per round, lag = how many chunks a CTA may run ahead of the slowest CTA of the grid.
    int chunk_tiles;
    int cpr;
    int lag;
    uint32_t* sync_cnt;  // [rounds * cpr] arrivals per chunk slot, zeroed before the launch
    // Shared per-query bound ([total slots][nq_pad] keys) in levels: while it runs (every 4
    // tiles) and at its end, an item publishes, for each level, the key at the level's list rank
    // (once the list holds that many) into slot (split % slots) of the level with atomicMin. A
    // level's bound is its largest slot (infinite while a slot is empty): the slot minima come
    // from `slots` DISTINCT items, each holding `rank` real candidates at or below its key, so
    // at least slots * rank candidates lie at or below it, and with slots * rank >= the final
    // pool it never cuts into the pool. Every level is valid, so the filter uses the smallest.
    // One slot at a high rank is available after the first item's first tiles; many slots at a
    // low rank are tighter once items of every split class have run.
    BoundLevels lv;
    // List mode (single-CTA kernel only; null in a flat search): item i is query tile i, whose
    // 128 queries are matched against list tile_list[i] alone, rows [list_off[L], list_off[L+1])
    // of the operand. No row splits and no pacing.
    const int* tile_list;
    const int64_t* list_off;
    // List mode: query tile row r holds (query, probe) pair row_pair[r] (-1: padding), of query
    // row_pair[r] / pair_div. The bound slot is per query, shared by all of its probes' items
    // (any item's KP-th key bounds the query's pool); padding rows neither read nor publish.
    const int* row_pair;
    int pair_div;
    int item_base;  // list mode: item i is query tile item_base + i
    // Test hook (VA_TC_TEST_STALL_TILES): the MMA issuer stops after this many tiles, so the
    // epilogue's bounded wait for the next accumulator expires; -1 in every real launch.
    int stall_tiles;
};

__device__ __forceinline__ uint32_t ld_relaxed(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Soft wait for a chunk slot to collect `target` arrivals. It only paces the producer for L2
// locality: on expiry it returns false and the caller stops pacing (no error).
__device__ __forceinline__ bool wait_arrivals(const uint32_t* p, uint32_t target, uint64_t limit_ns) {
    if (ld_relaxed(p) >= target) return true;
    const uint64_t t0 = va::globaltimer_ns();
    while (ld_relaxed(p) < target) {
        __nanosleep(128);
        if (va::globaltimer_ns() - t0 > limit_ns) return false;
    }
    return true;
}

BoundLevels one_level(int kp) {
    BoundLevels lv = {};
    lv.n = 1;
    lv.slots[0] = 1;
    lv.rank[0] = kp;
    lv.off[0] = 0;
    return lv;
}

__device__ __forceinline__ void item_range(const Work& w, int item, int& qt, int& t0, int& t1) {
    const int s = item / w.n_qtiles;
    qt = item - s * w.n_qtiles;
    t0 = (int)(((int64_t)w.n_tiles * s) / w.splits);
    t1 = (int)(((int64_t)w.n_tiles * (s + 1)) / w.splits);
}

// An item's query tile, its row tiles [t0, t1) counted from row `rb`, and the end of its rows
// (rows at or past `re` never pass). Flat search: rb = 0, re = n_rows.
__device__ __forceinline__ void item_rows(const Work& w, int item, int& qt, int& t0, int& t1, int64_t& rb,
                                          uint32_t& re) {
    if (w.tile_list) {
        qt = w.item_base + item;
        const int L = w.tile_list[qt];
        rb = w.list_off[L];
        const int64_t e = w.list_off[L + 1];
        re = (uint32_t)e;
        t0 = 0;
        t1 = (int)((e - rb + BN - 1) / BN);
    } else {
        item_range(w, item, qt, t0, t1);
        rb = 0;
        re = (uint32_t)w.n_rows;
    }
}

template <int ELEM, int KP>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    k_tc_filter(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_x, Work w,
                const float* __restrict__ row_bias, float alpha, const int* __restrict__ row_qn,
                float* __restrict__ part_keys,
                uint32_t* __restrict__ part_ids, uint32_t* __restrict__ gthr, int* err, uint64_t limit_ns,
                int stages) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte alignment for the 128B-swizzled operand slots.
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* sA = smem;
    uint8_t* sB = smem + (size_t)stages * A_BYTES;
    float* l_key = (float*)(sB + (size_t)stages * B_BYTES);       // [BM][stride]
    uint32_t* l_id = (uint32_t*)(l_key + list_stride<KP>() * BM);  // [BM][stride]
    uint64_t* bars = (uint64_t*)(l_id + list_stride<KP>() * BM);                  // full[stages], empty[stages], tfull[2], tempty[2]
    uint64_t* full = bars;
    uint64_t* empty = bars + stages;
    uint64_t* tfull = bars + 2 * stages;
    uint64_t* tempty = tfull + 2;
    uint64_t* dbar = tempty + 2;  // teardown: the MMA issuer's final commit
    uint32_t* s_tmem = (uint32_t*)(dbar + 1);
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
        mbar_init(dbar, 1);
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
        // Lockstep for L2 reuse: all CTAs of a round stream the same 2-3 row splits; each split
        // is read by up to one CTA per query tile. Before starting chunk slot g (round * cpr +
        // local chunk) a CTA waits until every CTA of the grid has started slot g - lag, so the
        // rows in flight stay within ~lag chunks per split and are fetched from HBM about once.
        if (lane == 0) {
            uint32_t it = 0;
            int round = 0;
            bool pace = true;
            for (int item = blockIdx.x; item < n_items && !*s_abort; item += gridDim.x, ++round) {
                int qt, t0, t1;
                int64_t rb;
                uint32_t re;
                item_rows(w, item, qt, t0, t1, rb, re);
                int next_slot = 0;
                for (int t = t0; t < t1; ++t) {
                    const int j = t - t0;
                    if (w.sync_cnt && j % w.chunk_tiles == 0) {
                        const int g = round * w.cpr + j / w.chunk_tiles;
                        if (pace && g >= w.lag) {
                            const int gr = (g - w.lag) / w.cpr;
                            const uint32_t target = (uint32_t)min((int)gridDim.x, n_items - gr * (int)gridDim.x);
                            pace = wait_arrivals(w.sync_cnt + (g - w.lag), target, 200000000ull);
                        }
                        atomicAdd(w.sync_cnt + g, 1u);
                        next_slot = j / w.chunk_tiles + 1;
                    }
                    for (int kb = 0; kb < w.k_blocks; ++kb, ++it) {
                        const int s = it % stages;
                        const uint32_t ph = (it / stages) & 1u;
                        if (!mbar_wait(&empty[s], ph ^ 1u, s_abort, err, limit_ns)) goto producer_done;
                        mbar_expect_tx(&full[s], STAGE_BYTES);
                        const int kc = kb * (BKB / ELEM);
                        tma_load_2d(sA + (size_t)s * A_BYTES, &tmap_q, &full[s], kc, qt * BM);
                        tma_load_2d(sB + (size_t)s * B_BYTES, &tmap_x, &full[s], kc, (int)(rb + (int64_t)t * BN));
                    }
                }
                // A shorter item still arrives at every slot of its round.
                if (w.sync_cnt)
                    for (int c = next_slot; c < w.cpr; ++c) atomicAdd(w.sync_cnt + round * w.cpr + c, 1u);
            }
        producer_done:
            // After an abort, loads still in flight write this CTA's shared memory: wait for them.
            if (*s_abort) drain_loads(full, stages, it);
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            uint32_t it = 0, tile = 0;
            for (int item = blockIdx.x; item < n_items && !*s_abort; item += gridDim.x) {
                int qt, t0, t1;
                int64_t rb;
                uint32_t re;
                item_rows(w, item, qt, t0, t1, rb, re);
                for (int t = t0; t < t1; ++t, ++tile) {
                    if ((int)tile == w.stall_tiles) goto mma_done;
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
        mma_done:
            // After an abort (or a stall), MMAs already issued may still write TMEM: one more
            // commit tracks all of them; wait for it before TMEM is freed.
            if (*s_abort || w.stall_tiles >= 0) {
                mma_commit(dbar);
                mbar_drain(dbar, 0u, kDrainLimitNs);
            }
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
            int64_t rb;
            uint32_t re;
            item_rows(w, item, qt, t0, t1, rb, re);
            const int64_t q = (int64_t)qt * BM + row;
            uint32_t* gq = gthr + q;
            if (w.row_pair) {
                const int pr = w.row_pair[q];
                gq = pr >= 0 ? gthr + pr / w.pair_div : nullptr;
            }
            const int split = item / w.n_qtiles;
            // Reset this warp's 32 row lists (row-contiguous, KP entries each; coalesced).
            for (int e = lane; e < 32 * list_stride<KP>(); e += 32) {
                l_key[quarter * 32 * list_stride<KP>() + e] = INFINITY;
                l_id[quarter * 32 * list_stride<KP>() + e] = va::kInvalidId;
            }
            __syncwarp();
            const int qn = row_qn ? row_qn[q] : 0;
            const uint32_t n_rows32 = re;
            float thr_own = INFINITY;
            // Padding rows of a list-mode tile insert nothing (their lists are never read).
            float thr_g = gq ? load_bound(gq, w.nq_pad, w.lv) : -INFINITY;
            float thr = thr_g;
            // The tile's 256 row biases (|x|^2 for L2, 0 otherwise; +inf past the last row): lane j
            // holds columns j + 32r, r < 8; the next tile's are prefetched while this one runs.
            float bias[8], nbias[8];
#pragma unroll
            for (int r = 0; r < 8; ++r) bias[r] = __ldg(row_bias + rb + (int64_t)t0 * BN + lane + 32 * r);
            const float* const row_keys = l_key + (size_t)row * list_stride<KP>();
            for (int t = t0; t < t1; ++t, ++tile) {
                if (((t - t0) & 3) == 3) {
                    if (gq) {
                        publish_bound(gq, w.nq_pad, w.lv, split, row_keys);
                        thr_g = load_bound(gq, w.nq_pad, w.lv);
                    }
                    thr = fminf(thr_own, thr_g);
                }
                const int64_t col0 = rb + (int64_t)t * BN;
                if (t + 1 < t1) {
#pragma unroll
                    for (int r = 0; r < 8; ++r) nbias[r] = __ldg(row_bias + col0 + BN + lane + 32 * r);
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
                const uint32_t id0 = (uint32_t)col0;
                // Four 64-column chunks, TMEM loads double-buffered against the filtering.
                uint32_t ra[64], rb[64];
                tmem_ld64(taddr, ra);
                tmem_wait64(ra);
                tmem_ld64(taddr + 64, rb);
                filter_chunk<0, KP, (ELEM == 1)>(ra, bias, alpha, qn, id0, n_rows32, l_key, l_id, quarter * 32, lane, thr_g, thr_own, thr);
                __syncwarp();
                tmem_wait64(rb);
                tmem_ld64(taddr + 128, ra);
                filter_chunk<1, KP, (ELEM == 1)>(rb, bias, alpha, qn, id0 + 64, n_rows32, l_key, l_id, quarter * 32, lane, thr_g, thr_own, thr);
                __syncwarp();
                tmem_wait64(ra);
                tmem_ld64(taddr + 192, rb);
                filter_chunk<2, KP, (ELEM == 1)>(ra, bias, alpha, qn, id0 + 128, n_rows32, l_key, l_id, quarter * 32, lane, thr_g, thr_own, thr);
                __syncwarp();
                tmem_wait64(rb);
                // Every TMEM read of this tile is done: hand the accumulator back to the MMA warp.
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[buf]);
                filter_chunk<3, KP, (ELEM == 1)>(rb, bias, alpha, qn, id0 + 192, n_rows32, l_key, l_id, quarter * 32, lane, thr_g, thr_own, thr);
                __syncwarp();
#pragma unroll
                for (int r = 0; r < 8; ++r) bias[r] = nbias[r];
            }
            {
                // Publish this item's final rank keys as bounds.
                const int s = split;
                if (gq) publish_bound(gq, w.nq_pad, w.lv, split, row_keys);
                // The warp's 32 lists are contiguous in shared memory and in the output
                // ([split][query][KP]): copy them with coalesced stores.
                const int64_t out0 = ((int64_t)s * w.nq_pad + (int64_t)qt * BM + quarter * 32) * KP;
                for (int e = lane; e < 32 * KP; e += 32) {
                    const int src = (quarter * 32 + e / KP) * list_stride<KP>() + e % KP;
                    part_keys[out0 + e] = l_key[src];
                    part_ids[out0 + e] = l_id[src];
                }
                __syncwarp();
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

// ================================================================================================
// Pair kernel. Two CTAs of a cluster issue cta_group::2 MMAs of M = 256 queries (128 per CTA) by
// N = 256 rows (128 loaded per CTA), so each SM moves 32 KB of operands per K block instead of
// 48 KB. The 1-CTA tile's 48 KB of TMA writes plus its tensor-core operand reads per K block
// oversubscribe the SM's shared-memory and L2 feed (measured: ~54% of the MMA rate with the
// epilogue removed); the pair halves the B traffic per SM.
//
// Protocol (rank 0 = leader, rank 1 = peer; same shared-memory offsets in both CTAs):
//   producer (both CTAs)  waits its own empty[s]; loads its 128 query rows and 128 tile rows with
//                         cta_group::2 TMA whose completion counts on the LEADER's full[s]; the
//                         leader also posts expect_tx for both CTAs' bytes
//   MMA (leader only)     waits full[s], issues the pair MMAs, commits empty[s] in both CTAs; after
//                         a tile's last K block commits tfull[buf] in both CTAs; waits the
//                         leader's tempty[buf], which both CTAs' epilogue warps (8) arrive on
//   epilogue (both CTAs)  as in the 1-CTA kernel, on its own 128 queries and TMEM
// No commit or load uses a multicast form: the leader commits twice (own and peer address).
// ================================================================================================
constexpr int P_ROWS = 128;                  // rows per CTA of each operand tile
constexpr int PA_BYTES = P_ROWS * BKB;       // 16 KB of queries
constexpr int PB_BYTES = P_ROWS * BKB;       // 16 KB of database rows
constexpr int PSTAGE_BYTES = PA_BYTES + PB_BYTES;
constexpr int PBM = 256;                     // queries per pair tile

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_index() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_count() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}
// Address of the same shared-memory location in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t map_rank(uint32_t smem_addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster_addr, int c0,
                                                 int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
        "[%2];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(bar_cluster_addr), "r"(c0), "r"(c1)
        : "memory");
}
__device__ __forceinline__ void mma_commit_pair(uint32_t bar_cluster_addr) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster_addr)
                 : "memory");
}
// An abort in one CTA of a pair stops both: its flag is also set in the peer CTA.
__device__ __forceinline__ void abort_peer(volatile int* s_abort, uint32_t rank) {
    *s_abort = 1;
    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(map_rank(smem_u32((const void*)s_abort), rank ^ 1u)), "r"(1)
                 : "memory");
}
// Teardown of a pair after an abort: a CTA's TMA loads signal the leader's barriers, so the peer
// cannot wait for its own loads; both CTAs let in-flight copies land (a fixed settle time, far
// above a copy's latency) before the cluster barrier that precedes TMEM release and exit.
__device__ __forceinline__ void settle_ns(uint64_t ns) {
    const uint64_t t0 = va::globaltimer_ns();
    while (va::globaltimer_ns() - t0 < ns) __nanosleep(1000);
}

template <int ELEM>
struct PairKind;
template <>
struct PairKind<2> {  // bf16 x bf16 -> fp32, M = 256 across the pair
    static constexpr uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                      ((uint32_t)(PBM >> 4) << 24);
    __device__ static __forceinline__ void mma(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t acc) {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
            "l"(a), "l"(b), "r"(idesc), "r"(acc));
    }
};
template <>
struct PairKind<1> {  // s8 x s8 -> s32, M = 256 across the pair
    static constexpr uint32_t idesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                      ((uint32_t)(PBM >> 4) << 24);
    __device__ static __forceinline__ void mma(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t acc) {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
            "l"(a), "l"(b), "r"(idesc), "r"(acc));
    }
};
template <>
struct PairKind<4> {  // tf32 x tf32 -> fp32, M = 256 across the pair
    static constexpr uint32_t idesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                      ((uint32_t)(PBM >> 4) << 24);
    __device__ static __forceinline__ void mma(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t acc) {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
            "l"(a), "l"(b), "r"(idesc), "r"(acc));
    }
};

template <int ELEM, int KP>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    k_tc_filter_pair(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_x, Work w,
                     const float* __restrict__ row_bias, float alpha, const int* __restrict__ row_qn,
                float* __restrict__ part_keys,
                     uint32_t* __restrict__ part_ids, uint32_t* __restrict__ gthr, int* err, uint64_t limit_ns,
                     int stages) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* sA = smem;
    uint8_t* sB = smem + (size_t)stages * PA_BYTES;
    float* l_key = (float*)(sB + (size_t)stages * PB_BYTES);  // [128][stride]
    uint32_t* l_id = (uint32_t*)(l_key + list_stride<KP>() * P_ROWS);  // [128][stride]
    uint64_t* bars = (uint64_t*)(l_id + list_stride<KP>() * P_ROWS);
    uint64_t* full = bars;
    uint64_t* empty = bars + stages;
    uint64_t* tfull = bars + 2 * stages;
    uint64_t* tempty = tfull + 2;
    uint64_t* dbar = tempty + 2;  // teardown: the leader's final pair commit
    uint32_t* s_tmem = (uint32_t*)(dbar + 1);
    volatile int* s_abort = (volatile int*)(s_tmem + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const int cid = (int)cluster_index(), ncl = (int)cluster_count();
    const int n_items = w.n_qtiles * w.splits;

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 8);
        }
        mbar_init(dbar, 1);
        *s_abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_q) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_x) : "memory");
    }
    // Both CTAs' barriers exist before either CTA signals the other's.
    cluster_sync();
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(s_tmem)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *s_tmem;

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producer (both CTAs)
        if (lane == 0) {
            uint32_t it = 0;
            int round = 0;
            bool pace = true;
            for (int item = cid; item < n_items && !*s_abort; item += ncl, ++round) {
                int qt, t0, t1;
                item_range(w, item, qt, t0, t1);
                int next_slot = 0;
                for (int t = t0; t < t1; ++t) {
                    const int j = t - t0;
                    if (j % w.chunk_tiles == 0) {
                        const int g = round * w.cpr + j / w.chunk_tiles;
                        if (pace && g >= w.lag) {
                            const int gr = (g - w.lag) / w.cpr;
                            const uint32_t target = 2u * (uint32_t)min(ncl, n_items - gr * ncl);
                            pace = wait_arrivals(w.sync_cnt + (g - w.lag), target, 200000000ull);
                        }
                        atomicAdd(w.sync_cnt + g, 1u);
                        next_slot = j / w.chunk_tiles + 1;
                    }
                    for (int kb = 0; kb < w.k_blocks; ++kb, ++it) {
                        const int s = it % stages;
                        const uint32_t ph = (it / stages) & 1u;
                        if (!mbar_wait(&empty[s], ph ^ 1u, s_abort, err, limit_ns)) {
                            abort_peer(s_abort, rank);
                            goto producer_done;
                        }
                        const uint32_t full_leader = map_rank(smem_u32(&full[s]), 0);
                        if (leader) mbar_expect_tx(&full[s], 2 * PSTAGE_BYTES);
                        const int kc = kb * (BKB / ELEM);
                        tma_load_2d_pair(sA + (size_t)s * PA_BYTES, &tmap_q, full_leader, kc,
                                         qt * PBM + (int)rank * P_ROWS);
                        tma_load_2d_pair(sB + (size_t)s * PB_BYTES, &tmap_x, full_leader, kc,
                                         t * BN + (int)rank * P_ROWS);
                    }
                }
                for (int c = next_slot; c < w.cpr; ++c) atomicAdd(w.sync_cnt + round * w.cpr + c, 1u);
            }
        producer_done:
            if (*s_abort) {
                // The leader's full barriers count both CTAs' bytes of every stage it armed.
                if (leader) drain_loads(full, stages, it);
                settle_ns(1000000ull);
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer (leader only)
        if (leader && lane == 0) {
            uint32_t it = 0, tile = 0;
            for (int item = cid; item < n_items && !*s_abort; item += ncl) {
                int qt, t0, t1;
                item_range(w, item, qt, t0, t1);
                for (int t = t0; t < t1; ++t, ++tile) {
                    const uint32_t buf = tile & 1u;
                    const uint32_t tph = (tile >> 1) & 1u;
                    if (!mbar_wait(&tempty[buf], tph ^ 1u, s_abort, err, limit_ns)) {
                        abort_peer(s_abort, rank);
                        goto mma_done;
                    }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + buf * BN;
                    for (int kb = 0; kb < w.k_blocks; ++kb, ++it) {
                        const int s = it % stages;
                        const uint32_t ph = (it / stages) & 1u;
                        if (!mbar_wait(&full[s], ph, s_abort, err, limit_ns)) {
                            abort_peer(s_abort, rank);
                            goto mma_done;
                        }
                        tc_fence_after();
                        const uint32_t a0 = smem_u32(sA + (size_t)s * PA_BYTES);
                        const uint32_t b0 = smem_u32(sB + (size_t)s * PB_BYTES);
#pragma unroll
                        for (int j = 0; j < BKB / 32; ++j)
                            PairKind<ELEM>::mma(d_tmem, smem_desc(a0 + 32 * j), smem_desc(b0 + 32 * j),
                                                (kb | j) ? 1u : 0u);
                        const uint32_t e = smem_u32(&empty[s]);
                        mma_commit_pair(map_rank(e, 0));
                        mma_commit_pair(map_rank(e, 1));
                    }
                    const uint32_t f = smem_u32(&tfull[buf]);
                    mma_commit_pair(map_rank(f, 0));
                    mma_commit_pair(map_rank(f, 1));
                }
            }
        mma_done:
            if (*s_abort) {
                // pair MMAs already issued write both CTAs' TMEM: wait for all of them
                mma_commit_pair(map_rank(smem_u32(dbar), 0));
                mbar_drain(dbar, 0u, kDrainLimitNs);
            }
        }
    } else {
        // ---------------------------------------------------------------- epilogue (both CTAs)
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        uint32_t tile = 0;
        for (int item = cid; item < n_items; item += ncl) {
            int qt, t0, t1;
            item_range(w, item, qt, t0, t1);
            const int64_t qbase = (int64_t)qt * PBM + (int64_t)rank * P_ROWS;
            const int64_t q = qbase + row;
            for (int e = lane; e < 32 * list_stride<KP>(); e += 32) {
                l_key[quarter * 32 * list_stride<KP>() + e] = INFINITY;
                l_id[quarter * 32 * list_stride<KP>() + e] = va::kInvalidId;
            }
            __syncwarp();
            const int qn = row_qn ? row_qn[q] : 0;
            const uint32_t n_rows32 = (uint32_t)w.n_rows;
            float thr_own = INFINITY;
            float thr_g = load_bound(gthr + q, w.nq_pad, w.lv);
            float thr = thr_g;
            float bias[8], nbias[8];
#pragma unroll
            for (int r = 0; r < 8; ++r) bias[r] = __ldg(row_bias + (int64_t)t0 * BN + lane + 32 * r);
            const int split = item / w.n_qtiles;
            const float* const row_keys = l_key + (size_t)row * list_stride<KP>();
            for (int t = t0; t < t1; ++t, ++tile) {
                if (((t - t0) & 3) == 3) {
                    publish_bound(gthr + q, w.nq_pad, w.lv, split, row_keys);
                    thr_g = load_bound(gthr + q, w.nq_pad, w.lv);
                    thr = fminf(thr_own, thr_g);
                }
                const int64_t col0 = (int64_t)t * BN;
                if (t + 1 < t1) {
#pragma unroll
                    for (int r = 0; r < 8; ++r) nbias[r] = __ldg(row_bias + col0 + BN + lane + 32 * r);
                }
                const uint32_t buf = tile & 1u;
                const uint32_t tph = (tile >> 1) & 1u;
                int ok = 1;
                if (lane == 0) {
                    ok = mbar_wait(&tfull[buf], tph, s_abort, err, limit_ns) ? 1 : 0;
                    if (!ok) abort_peer(s_abort, rank);
                }
                ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
                if (!ok) goto epi_done;
                tc_fence_after();
                const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + buf * BN;
                const uint32_t id0 = (uint32_t)col0;
                uint32_t ra[64], rb[64];
                tmem_ld64(taddr, ra);
                tmem_wait64(ra);
                tmem_ld64(taddr + 64, rb);
                filter_chunk<0, KP, (ELEM == 1)>(ra, bias, alpha, qn, id0, n_rows32, l_key, l_id, quarter * 32, lane, thr_g, thr_own, thr);
                __syncwarp();
                tmem_wait64(rb);
                tmem_ld64(taddr + 128, ra);
                filter_chunk<1, KP, (ELEM == 1)>(rb, bias, alpha, qn, id0 + 64, n_rows32, l_key, l_id, quarter * 32, lane, thr_g, thr_own, thr);
                __syncwarp();
                tmem_wait64(ra);
                tmem_ld64(taddr + 192, rb);
                filter_chunk<2, KP, (ELEM == 1)>(ra, bias, alpha, qn, id0 + 128, n_rows32, l_key, l_id, quarter * 32, lane, thr_g, thr_own, thr);
                __syncwarp();
                tmem_wait64(rb);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_remote(map_rank(smem_u32(&tempty[buf]), 0));
                filter_chunk<3, KP, (ELEM == 1)>(rb, bias, alpha, qn, id0 + 192, n_rows32, l_key, l_id, quarter * 32, lane, thr_g, thr_own, thr);
                __syncwarp();
#pragma unroll
                for (int r = 0; r < 8; ++r) bias[r] = nbias[r];
            }
            {
                const int s = split;
                publish_bound(gthr + q, w.nq_pad, w.lv, split, row_keys);
                const int64_t out0 = ((int64_t)s * w.nq_pad + qbase + quarter * 32) * KP;
                for (int e = lane; e < 32 * KP; e += 32) {
                    const int src = (quarter * 32 + e / KP) * list_stride<KP>() + e % KP;
                    part_keys[out0 + e] = l_key[src];
                    part_ids[out0 + e] = l_id[src];
                }
                __syncwarp();
            }
        }
    epi_done:;
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    // The peer's last remote arrivals and the pair MMAs are done before either CTA frees TMEM
    // or exits.
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS));
    }
}

// Test hooks of the bounded-wait path, read at every launch: VA_TC_WAIT_LIMIT_MS replaces the
// device waits' limit; VA_TC_TEST_STALL_TILES makes the single-CTA kernel's MMA issuer stop after
// that many tiles (the pair kernel ignores it), so a bounded wait expires and the launch reports
// VA_ERR_TIMEOUT through va_synchronize. Unset in normal use.
uint64_t wait_limit_ns(unsigned limit_ms) {
    const char* e = getenv("VA_TC_WAIT_LIMIT_MS");
    const long v = e ? atol(e) : 0;
    return (uint64_t)(v > 0 ? (unsigned long)v : limit_ms) * 1000000ull;
}

int test_stall_tiles() {
    const char* e = getenv("VA_TC_TEST_STALL_TILES");
    return e && e[0] ? std::max(0, atoi(e)) : -1;
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
    const CUtensorMapDataType dt = elem_bytes == 1   ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                   : elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                     : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    CUresult r = enc(map, dt, 2,
                     const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return va_set_error(VA_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
    return VA_OK;
}

template <int ELEM, int KP>
int launch_filter(va_context* ctx, const TcFilterArgs& a, int stages, size_t smem, const CUtensorMap& mq,
                  const CUtensorMap& mx, const Work& w, int grid, bool pair, bool reset_bounds = true) {
    auto kern = pair ? k_tc_filter_pair<ELEM, KP> : k_tc_filter<ELEM, KP>;
    VA_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int total_slots = 0;
    for (int l = 0; l < w.lv.n; ++l) total_slots += w.lv.slots[l];
    if (reset_bounds)
        VA_CUDA_TRY(cudaMemsetAsync(a.gthr, 0xFF, (size_t)total_slots * w.nq_pad * sizeof(uint32_t), ctx->stream));
    if (w.sync_cnt)
        VA_CUDA_TRY(cudaMemsetAsync(w.sync_cnt, 0, (size_t)a.sync_words * sizeof(uint32_t), ctx->stream));
    // Cooperative launch: the CTAs pace each other, so all of them must be resident at once.
    // The pair kernel also runs as clusters of two CTAs.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(NUM_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 2;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pair ? 2 : 1;
    VA_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, mq, mx, w, a.row_bias, a.alpha, a.row_qn, a.part_keys, a.part_ids,
                                   a.gthr, ctx->d_error, wait_limit_ns(a.limit_ms), stages));
    return va_check_launch(pair ? "k_tc_filter_pair" : "k_tc_filter");
}

size_t smem_bytes(int kp, int stages, bool pair) {
    const int stride = kp + 1;  // list_stride<KP>()
    return 1024 + (size_t)stages * (pair ? PSTAGE_BYTES : STAGE_BYTES) + (size_t)stride * BM * 8 +
           (2 * stages + 5) * 8 + 16;
}

}  // namespace

// The single-CTA kernel is the default; VA_TC_PAIR=1 selects the cta_group::2 pair kernel. At
// the 10M x 768 headline both run at the same rate, held by the 1 kW power cap (measured: 151.6
// vs 151.7 ms per launch, sw_power_cap active throughout).
bool va_tc_use_pair() {
    static const int v = [] {
        const char* e = getenv("VA_TC_PAIR");
        return (e && e[0] == '1') ? 1 : 0;
    }();
    return v != 0;
}

// Plan of a filter launch (host side, shared with va_search.cu).
int va_tc_plan(va_context* ctx, int64_t nq, int64_t n_rows, int kp, TcPlan* plan, int64_t row_bytes) {
    // A 128-entry list takes 128 KB of shared memory; the pair kernel's 32 KB stages still leave
    // room for three of them (the single-CTA kernel would have two).
    const bool pair = (va_tc_use_pair() || kp >= 128) && ctx->sm_count >= 2;
    const int qrows = pair ? PBM : BM;
    plan->pair = pair;
    plan->n_qtiles = (int)((nq + qrows - 1) / qrows);
    plan->n_tiles = (int)((n_rows + BN - 1) / BN);
    plan->nq_pad = (int64_t)plan->n_qtiles * qrows;
    // Splits: the number of row splits that minimizes the modelled time rounds x (tiles per item
    // + c), where rounds = ceil(query tiles x splits / workers) and c is the fixed cost of a work
    // item (list reset and copy-out, bound refresh, the pipeline bubble at its boundary) in tiles:
    // measured at ~16 us, 5.3 bf16 tiles of 768 dimensions, so c = 8192 / row bytes. Equal splits
    // per worker (query tiles x splits a multiple of the workers) remain the start; fewer, longer
    // items win when the tile count leaves items short (1.25M rows per GPU: 37 instead of 148
    // splits, 9% faster). Never finer than one row tile.
    const int g = pair ? ctx->sm_count / 2 : ctx->sm_count;
    int a = plan->n_qtiles, b = g;
    while (b) {
        int t = a % b;
        a = b;
        b = t;
    }
    const double c_item = 8192.0 / (double)std::max<int64_t>(row_bytes, 128);
    auto cost = [&](int sp) {
        const int64_t rounds = ((int64_t)plan->n_qtiles * sp + g - 1) / g;
        return (double)rounds * ((double)plan->n_tiles / sp + c_item);
    };
    int splits = std::max(1, std::min(g / a, plan->n_tiles));
    double best = cost(splits);
    // At least 32 splits (or the balanced count if smaller): the shared bound's levels need items
    // from up to 8 split classes, and each round of the grid should stream few splits at once.
    for (int sp = std::min(32, splits); sp <= std::min(g, plan->n_tiles); ++sp) {
        const double cst = cost(sp);
        if (cst < best * 0.995) {
            best = cst;
            splits = sp;
        }
    }
    plan->splits = splits;
    plan->kp = kp;
    const int workers = std::min(plan->n_qtiles * splits, g);
    plan->grid = pair ? 2 * workers : workers;
    // Lockstep pacing: chunks of 16 row tiles, a CTA at most 2 chunks ahead of the slowest.
    plan->chunk_tiles = 16;
    plan->lag = 2;
    const int max_item_tiles = (plan->n_tiles + splits - 1) / splits;
    plan->cpr = (max_item_tiles + plan->chunk_tiles - 1) / plan->chunk_tiles;
    const int rounds = (plan->n_qtiles * splits + workers - 1) / workers;
    plan->sync_words = (int64_t)rounds * plan->cpr;
    plan->levels = one_level(kp);
    plan->bound_slots = 1;
    return VA_OK;
}

// Plan for a final pool of `pool` candidates per query. Up to 128: one list of the pool's size
// (32/64/128) per item and one bound slot. Wider: 64-entry lists (the single-CTA kernel) when the
// row splits give at least twice the pool in list entries, else 128-entry lists, with
// ceil(pool / kp) bound slots.
int va_tc_plan_pool(va_context* ctx, int64_t nq, int64_t n_rows, int pool, TcPlan* plan, int64_t row_bytes) {
    if (pool <= 128) {
        VA_TRY(va_tc_plan(ctx, nq, n_rows, pool <= 32 ? 32 : pool <= 64 ? 64 : 128, plan, row_bytes));
    } else {
        VA_TRY(va_tc_plan(ctx, nq, n_rows, 64, plan, row_bytes));
        if ((int64_t)plan->splits * 64 < 2 * (int64_t)pool)
            VA_TRY(va_tc_plan(ctx, nq, n_rows, 128, plan, row_bytes));
    }
    // Bound levels: the pool (at least the list length) must stay at or below each. Ranks kp,
    // kp/2, kp/4, kp/8 with slots = ceil(target / rank), while the slots have items to feed them
    // (slots <= splits) and the total stays within 32 loads per refresh.
    const int target = std::max(pool, plan->kp);
    BoundLevels lv = {};
    int total = 0;
    for (int r = plan->kp; r >= 1 && lv.n < 4 && r * 8 >= plan->kp; r /= 2) {
        const int ns = (target + r - 1) / r;
        if (ns > plan->splits || total + ns > 32) break;
        lv.slots[lv.n] = ns;
        lv.rank[lv.n] = r;
        lv.off[lv.n] = total;
        total += ns;
        ++lv.n;
    }
    if (!lv.n) {
        lv = one_level(plan->kp);
        lv.slots[0] = (target + plan->kp - 1) / plan->kp;
        total = lv.slots[0];
    }
    plan->levels = lv;
    plan->bound_slots = total;
    return VA_OK;
}

int va_tc_stages(int kp, bool pair) {
    for (int s = pair ? 8 : 6; s >= 2; --s)
        if (smem_bytes(kp, s, pair) <= 227 * 1024) return s;
    return 0;
}

int va_tc_filter(va_context* ctx, const TcFilterArgs& a, const TcPlan& p) {
    const int elem = a.elem_bytes;
    CUtensorMap mq, mx;
    VA_TRY(make_tmap(&mq, a.q_op, p.nq_pad, a.dpad, elem, p.pair ? P_ROWS : BM));
    VA_TRY(make_tmap(&mx, a.x_op, a.n_rows, a.dpad, elem, p.pair ? P_ROWS : BN));
    Work w;
    w.n_qtiles = p.n_qtiles;
    w.splits = p.splits;
    w.n_tiles = p.n_tiles;
    w.k_blocks = (int)((a.dpad * elem + BKB - 1) / BKB);
    w.n_rows = a.n_rows;
    w.nq_pad = p.nq_pad;
    w.chunk_tiles = p.chunk_tiles;
    w.cpr = p.cpr;
    w.lag = p.lag;
    w.sync_cnt = a.sync_cnt;
    w.tile_list = nullptr;
    w.list_off = nullptr;
    w.row_pair = nullptr;
    w.pair_div = 1;
    w.item_base = 0;
    w.lv = a.levels.n > 0 ? a.levels : one_level(p.kp);
    w.stall_tiles = test_stall_tiles();
    for (int l = 0; l < w.lv.n; ++l)
        if (w.lv.rank[l] < 1 || w.lv.rank[l] > p.kp || w.lv.slots[l] < 1)
            return va_set_error(VA_ERR_INVALID_ARG, "bound level %d: rank %d / slots %d invalid for lists of %d", l,
                                w.lv.rank[l], w.lv.slots[l], p.kp);
    if (a.sync_words < p.sync_words) return va_set_error(VA_ERR_INVALID_ARG, "sync buffer too small");
    const int stages = va_tc_stages(p.kp, p.pair);
    if (stages < 2) return va_set_error(VA_ERR_UNSUPPORTED, "candidate pool %d too large for shared memory", p.kp);
    const size_t smem = smem_bytes(p.kp, stages, p.pair);
    if (elem == 1) {
        if (p.kp == 32) return launch_filter<1, 32>(ctx, a, stages, smem, mq, mx, w, p.grid, p.pair);
        if (p.kp == 64) return launch_filter<1, 64>(ctx, a, stages, smem, mq, mx, w, p.grid, p.pair);
        if (p.kp == 128) return launch_filter<1, 128>(ctx, a, stages, smem, mq, mx, w, p.grid, p.pair);
    } else if (elem == 2) {
        if (p.kp == 32) return launch_filter<2, 32>(ctx, a, stages, smem, mq, mx, w, p.grid, p.pair);
        if (p.kp == 64) return launch_filter<2, 64>(ctx, a, stages, smem, mq, mx, w, p.grid, p.pair);
        if (p.kp == 128) return launch_filter<2, 128>(ctx, a, stages, smem, mq, mx, w, p.grid, p.pair);
    } else {
        if (p.kp == 32) return launch_filter<4, 32>(ctx, a, stages, smem, mq, mx, w, p.grid, p.pair);
        if (p.kp == 64) return launch_filter<4, 64>(ctx, a, stages, smem, mq, mx, w, p.grid, p.pair);
        if (p.kp == 128) return launch_filter<4, 128>(ctx, a, stages, smem, mq, mx, w, p.grid, p.pair);
    }
    return va_set_error(VA_ERR_UNSUPPORTED, "candidate pool %d not supported by the tensor-core filter", p.kp);
}

// List mode: query tile i (128 gathered queries) against the rows of list tile_list[i] only. One
// item per query tile (no row splits, no pacing), at most one CTA per SM, the single-CTA kernel.
// This launch runs tiles [tile0, tile0 + tiles) of n_qtiles; lists go out as [n_qtiles * 128][kp].
// The bound is per query (row_pair[r] / pair_div for query tile row r; -1 = padding), one slot at
// rank kp: a.gthr needs n_qtiles * 128 words, reset (to "none") when reset_bounds, else kept from
// the previous launch.
int va_tc_filter_lists(va_context* ctx, const TcFilterArgs& a, int n_qtiles, int tile0, int tiles,
                       const int* tile_list, const int64_t* list_off, const int* row_pair, int pair_div, int kp,
                       bool reset_bounds) {
    if (tiles <= 0) return VA_OK;
    VA_REQUIRE(kp == 32 || kp == 64 || kp == 128, "list length %d not supported", kp);
    VA_REQUIRE(a.elem_bytes == 2 || a.elem_bytes == 4, "list mode takes bf16 or fp32 (tf32) operands");
    const int elem = a.elem_bytes;
    VA_REQUIRE(tile0 >= 0 && tile0 + tiles <= n_qtiles, "tile range [%d, %d) outside %d tiles", tile0, tile0 + tiles,
               n_qtiles);
    CUtensorMap mq, mx;
    const int64_t nq_pad = (int64_t)n_qtiles * BM;
    VA_TRY(make_tmap(&mq, a.q_op, nq_pad, a.dpad, elem, BM));
    VA_TRY(make_tmap(&mx, a.x_op, a.n_rows, a.dpad, elem, BN));
    Work w = {};
    w.n_qtiles = tiles;
    w.splits = 1;
    w.n_tiles = 0;
    w.k_blocks = (int)((a.dpad * elem + BKB - 1) / BKB);
    w.n_rows = a.n_rows;
    w.nq_pad = nq_pad;
    w.chunk_tiles = 1;
    w.cpr = 1;
    w.lag = 0;
    w.sync_cnt = nullptr;
    w.lv = one_level(kp);
    w.tile_list = tile_list;
    w.list_off = list_off;
    w.row_pair = row_pair;
    w.pair_div = pair_div;
    w.item_base = tile0;
    w.stall_tiles = -1;
    const int stages = va_tc_stages(kp, false);
    if (stages < 2) return va_set_error(VA_ERR_UNSUPPORTED, "list length %d too large for shared memory", kp);
    const size_t smem = smem_bytes(kp, stages, false);
    const int grid = std::min(tiles, ctx->sm_count);
    if (elem == 4) {
        if (kp == 32) return launch_filter<4, 32>(ctx, a, stages, smem, mq, mx, w, grid, false, reset_bounds);
        if (kp == 64) return launch_filter<4, 64>(ctx, a, stages, smem, mq, mx, w, grid, false, reset_bounds);
        return launch_filter<4, 128>(ctx, a, stages, smem, mq, mx, w, grid, false, reset_bounds);
    }
    if (kp == 32) return launch_filter<2, 32>(ctx, a, stages, smem, mq, mx, w, grid, false, reset_bounds);
    if (kp == 64) return launch_filter<2, 64>(ctx, a, stages, smem, mq, mx, w, grid, false, reset_bounds);
    return launch_filter<2, 128>(ctx, a, stages, smem, mq, mx, w, grid, false, reset_bounds);
}
