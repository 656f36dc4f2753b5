// va_oracle.cpp -- TEST INFRASTRUCTURE ONLY.
//
// CPU restatement of VectorAccelerate's exact-search arithmetic. It is the checker for the
// CUDA library (tests/, __graft_entry__.smoke()) and the timed CPU baseline in bench.py.
// The product library (libva_cuda.so) never links, loads or calls this code.
//
// The reference is Swift + Metal + Apple Accelerate and cannot be built on Linux, so every
// function below restates the reference's algorithm from its source (file:line cited, paths
// relative to the VectorAccelerate project root). Parity pins: the known-answer cases in
// tests/golden/ are transcribed from the reference's own XCTest files and checked against this
// oracle by tests/test_oracle_golden.py. The VectorCore flat-search code named by the project
// brief is an un-vendored dependency (github.com/gifton/VectorCore, "from: 0.3.0", no lockfile);
// its arithmetic order is unpinned, so truth distances here accumulate in fp64 and round once.
//
// Conventions shared with the CUDA library:
//   * ids are uint32; 0xFFFFFFFF pads results when fewer than k candidates exist
//   * every selection uses the total order (key, id) ascending; "max" modes order by
//     (-value, id), i.e. larger value first and the smaller id on equal values
//   * L2 results are squared distances (computeSqrt = false)

#include <algorithm>
#include <atomic>
#include <cfloat>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

namespace {

// ---------------------------------------------------------------------------------------------
// TestRNG restatement (Tests/VectorAccelerateTests/Utilities/TestRNG.swift).
//   init:  state = max(seed,1) ^ (stream << 32), then 10 warm-up draws      (:57-69)
//   step:  state = 2862933555777941757 * state + 3037000493 (mod 2^64)      (:79)
//   float: (state >> 40) / 2^24                                              (:100-104)
//   gauss: Box-Muller pairs, u1 floored at Float.ulpOfOne, second value cached (:139-161)
// Deviation (stated): the Box-Muller transcendental step runs in double and rounds once to
// float, so this generator and the device generator in libva_cuda agree bit-for-bit except
// for rare last-ulp differences of the double-precision libm versus CUDA's.
// ---------------------------------------------------------------------------------------------
struct Rng {
    uint64_t s;
    bool has;
    float cached;
};

inline uint64_t rng_next(Rng& r) {
    r.s = 2862933555777941757ULL * r.s + 3037000493ULL;
    return r.s;
}

inline void rng_init(Rng& r, uint64_t seed, uint64_t stream) {
    uint64_t base = seed == 0 ? 1 : seed;
    r.s = base ^ (stream << 32);
    r.has = false;
    r.cached = 0.f;
    for (int i = 0; i < 10; ++i) rng_next(r);
}

inline float rng_f01(Rng& r) { return (float)(rng_next(r) >> 40) / 16777216.0f; }

inline float rng_gauss(Rng& r) {
    if (r.has) {
        r.has = false;
        return r.cached;
    }
    float u1 = std::max(rng_f01(r), FLT_EPSILON);
    float u2 = rng_f01(r);
    double rr = std::sqrt(-2.0 * std::log((double)u1));
    double th = 6.283185307179586 * (double)u2;
    r.cached = (float)(rr * std::sin(th));
    r.has = true;
    return (float)(rr * std::cos(th));
}

template <class F>
void parallel_for(int64_t n, int threads, F&& f) {
    if (threads <= 0) threads = (int)std::max(1u, std::thread::hardware_concurrency());
    if (n <= 0) return;
    if (threads == 1 || n == 1) {
        for (int64_t i = 0; i < n; ++i) f(i);
        return;
    }
    std::atomic<int64_t> next{0};
    std::vector<std::thread> pool;
    int t = (int)std::min<int64_t>(threads, n);
    for (int w = 0; w < t; ++w)
        pool.emplace_back([&] {
            for (;;) {
                int64_t i = next.fetch_add(1);
                if (i >= n) break;
                f(i);
            }
        });
    for (auto& th : pool) th.join();
}

// Orderable key of a float: monotone map float -> uint32. NaN maps to the worst key.
inline uint32_t f2key(float v) {
    if (std::isnan(v)) return 0xFFFFFFFFu;
    uint32_t u;
    std::memcpy(&u, &v, 4);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

struct Cand {
    uint32_t key;  // orderable key (already inverted for max mode)
    uint32_t id;
    float val;     // value reported to the caller
};
inline bool cand_less(const Cand& a, const Cand& b) {
    return a.key < b.key || (a.key == b.key && a.id < b.id);
}

// Bounded max-heap of the k best candidates under the (key, id) order.
// Restates CPUTopK.search (CPU/CPUTopK.swift:49-79): fill to k, heapify, then replace the root
// only when the newcomer is strictly better; the final array is sorted ascending. Because the
// (key, id) order is total, "strictly better" also settles equal distances by the smaller id,
// the rule of AdvancedTopK.metal:48-52 and SearchAndRetrieval.metal:313-317.
struct TopK {
    std::vector<Cand> h;
    int k;
    explicit TopK(int kk) : k(kk) { h.reserve(kk); }
    void sift_down(size_t i) {
        size_t n = h.size();
        for (;;) {
            size_t l = 2 * i + 1, r = l + 1, m = i;
            if (l < n && cand_less(h[m], h[l])) m = l;
            if (r < n && cand_less(h[m], h[r])) m = r;
            if (m == i) return;
            std::swap(h[i], h[m]);
            i = m;
        }
    }
    void push(const Cand& c) {
        if ((int)h.size() < k) {
            h.push_back(c);
            if ((int)h.size() == k)
                for (int i = k / 2 - 1; i >= 0; --i) sift_down((size_t)i);
        } else if (k > 0 && cand_less(c, h[0])) {
            h[0] = c;
            sift_down(0);
        }
    }
    bool would_accept(uint32_t key, uint32_t id) const {
        if ((int)h.size() < k) return true;
        return key < h[0].key || (key == h[0].key && id < h[0].id);
    }
    void emit(int kout, float pad, uint32_t* ids, float* vals) {
        std::sort(h.begin(), h.end(), cand_less);
        for (int i = 0; i < kout; ++i) {
            if (i < (int)h.size()) {
                if (ids) ids[i] = h[i].id;
                if (vals) vals[i] = h[i].val;
            } else {
                if (ids) ids[i] = 0xFFFFFFFFu;
                if (vals) vals[i] = pad;
            }
        }
    }
};

inline float bf16_to_f32(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

inline float load_x(const void* x, int dtype, int64_t idx) {
    if (dtype == 1) return bf16_to_f32(((const uint16_t*)x)[idx]);
    return ((const float*)x)[idx];
}

// fp32 sum of squared differences with 16 independent partial sums (vectorisable without
// reassociation flags). Used for the timed CPU baseline: the reference's vDSP_distancesq
// (CPU/CPUTopK.swift:62) also accumulates in fp32 in an unspecified lane order.
inline float l2sq_f32(const float* a, const float* b, int d) {
    float acc[16] = {0};
    int i = 0;
    for (; i + 16 <= d; i += 16)
        for (int j = 0; j < 16; ++j) {
            float t = a[i + j] - b[i + j];
            acc[j] += t * t;
        }
    float s = 0;
    for (int j = 0; j < 16; ++j) s += acc[j];
    for (; i < d; ++i) {
        float t = a[i] - b[i];
        s += t * t;
    }
    return s;
}

inline float dot_f32(const float* a, const float* b, int d) {
    float acc[16] = {0};
    int i = 0;
    for (; i + 16 <= d; i += 16)
        for (int j = 0; j < 16; ++j) acc[j] += a[i + j] * b[i + j];
    float s = 0;
    for (int j = 0; j < 16; ++j) s += acc[j];
    for (; i < d; ++i) s += a[i] * b[i];
    return s;
}

// fp64 sum of squared differences / of products with 8 independent partial sums (vectorisable
// without reassociation flags): the truth accumulation of knn_truth_rows. The summation order
// differs from a sequential fp64 sum only at the 1e-16 level, before the single rounding to fp32.
inline double l2sq_f64(const double* a, const double* b, int d) {
    double acc[8] = {0};
    int i = 0;
    for (; i + 8 <= d; i += 8)
        for (int j = 0; j < 8; ++j) {
            double t = a[i + j] - b[i + j];
            acc[j] += t * t;
        }
    double s = 0;
    for (int j = 0; j < 8; ++j) s += acc[j];
    for (; i < d; ++i) {
        double t = a[i] - b[i];
        s += t * t;
    }
    return s;
}

inline double dot_f64(const double* a, const double* b, int d) {
    double acc[8] = {0};
    int i = 0;
    for (; i + 8 <= d; i += 8)
        for (int j = 0; j < 8; ++j) acc[j] += a[i + j] * b[i + j];
    double s = 0;
    for (int j = 0; j < 8; ++j) s += acc[j];
    for (; i < d; ++i) s += a[i] * b[i];
    return s;
}

// Truth-mode k-NN split over row chunks (every host thread busy even for a few queries): each
// chunk keeps a bounded heap per query over its rows (rows widened to fp64 once per block and
// reused by every query), then the chunk heaps are merged per query under the same (key, id)
// order. Same selection and values as the per-query scan of CPUTopK.search.
void knn_truth_rows(const float* q, int64_t Q, const void* x, int x_dtype, int64_t N, int d, int k, int metric,
                    int threads, uint32_t* out_ids, float* out_vals) {
    if (threads <= 0) threads = (int)std::max(1u, std::thread::hardware_concurrency());
    const float pad = metric == 2 ? -INFINITY : INFINITY;
    std::vector<double> qd((size_t)Q * d), qn((size_t)Q);
    for (int64_t i = 0; i < Q; ++i) {
        double s = 0;
        for (int j = 0; j < d; ++j) {
            qd[(size_t)i * d + j] = q[i * d + j];
            s += (double)q[i * d + j] * q[i * d + j];
        }
        qn[(size_t)i] = std::sqrt(s);
    }
    const int64_t chunk = std::max<int64_t>(2048, (N + threads * 8 - 1) / ((int64_t)threads * 8));
    const int64_t nchunks = (N + chunk - 1) / chunk;
    std::vector<std::vector<TopK>> tops((size_t)nchunks);
    parallel_for(nchunks, threads, [&](int64_t c) {
        const int64_t r0 = c * chunk, r1 = std::min(N, r0 + chunk);
        std::vector<TopK> t;
        t.reserve((size_t)Q);
        for (int64_t i = 0; i < Q; ++i) t.emplace_back(k);
        constexpr int RB = 16;
        std::vector<double> xd((size_t)RB * d);
        double xn[RB];
        for (int64_t b0 = r0; b0 < r1; b0 += RB) {
            const int nb = (int)std::min<int64_t>(RB, r1 - b0);
            for (int r = 0; r < nb; ++r) {
                double s = 0;
                for (int j = 0; j < d; ++j) {
                    const double v = load_x(x, x_dtype, (b0 + r) * d + j);
                    xd[(size_t)r * d + j] = v;
                    s += v * v;
                }
                xn[r] = std::sqrt(s);
            }
            for (int64_t i = 0; i < Q; ++i) {
                const double* qq = qd.data() + (size_t)i * d;
                for (int r = 0; r < nb; ++r) {
                    const double* xx = xd.data() + (size_t)r * d;
                    float val;
                    if (metric == 0) {
                        val = (float)l2sq_f64(qq, xx, d);
                    } else {
                        const double s = dot_f64(qq, xx, d);
                        if (metric == 2) {
                            val = (float)s;
                        } else {
                            const double den = qn[(size_t)i] * xn[r];
                            double sim = den > 0 ? s / den : 0.0;
                            sim = std::min(1.0, std::max(-1.0, sim));
                            val = (float)(1.0 - sim);
                        }
                    }
                    uint32_t key = metric == 2 ? ~f2key(val) : f2key(val);
                    if (std::isnan(val)) key = 0xFFFFFFFFu;
                    const uint32_t id = (uint32_t)(b0 + r);
                    if (t[(size_t)i].would_accept(key, id)) t[(size_t)i].push(Cand{key, id, val});
                }
            }
        }
        tops[(size_t)c] = std::move(t);
    });
    parallel_for(Q, threads, [&](int64_t i) {
        TopK fin(k);
        for (int64_t c = 0; c < nchunks; ++c)
            for (const Cand& cd : tops[(size_t)c][(size_t)i].h) fin.push(cd);
        fin.emit(k, pad, out_ids ? out_ids + i * k : nullptr, out_vals ? out_vals + i * k : nullptr);
    });
}

}  // namespace

extern "C" {

int orc_version(void) { return 1; }

// ---------------------------------------------------------------------------------------------
// Data generation (seeded; stream = global row index, TestRNG.swift:62).
// ---------------------------------------------------------------------------------------------

// rows x dim i.i.d. N(0,1); row r uses stream (row0 + r).
void orc_gen_gaussian(float* out, int64_t rows, int dim, uint64_t seed, int64_t row0, int threads) {
    parallel_for(rows, threads, [&](int64_t r) {
        Rng g;
        rng_init(g, seed, (uint64_t)(row0 + r));
        float* o = out + r * dim;
        for (int j = 0; j < dim; ++j) o[j] = rng_gauss(g);
    });
}

// Gaussian-mixture rows: centroid c is N(0,1) from stream c of (seed ^ 0xC3A5C85C97CB3127);
// row r draws its cluster as (next() >> 33) % n_centroids from stream (row0 + r) of `seed`,
// then adds sigma * N(0,1) noise; optionally L2-normalises (norm in double, zero rows kept).
// Follows TestDataGenerator.gaussianClusters (Utilities/TestDataGenerator.swift:106-140) with
// the centroid law and sigma of the benchmark configurations.
void orc_gen_mixture(float* out, int64_t rows, int dim, uint64_t seed, int64_t row0, int n_centroids,
                     float sigma, int normalize, int threads) {
    const uint64_t cseed = seed ^ 0xC3A5C85C97CB3127ULL;
    parallel_for(rows, threads, [&](int64_t r) {
        Rng g;
        rng_init(g, seed, (uint64_t)(row0 + r));
        uint64_t c = (rng_next(g) >> 33) % (uint64_t)n_centroids;
        Rng gc;
        rng_init(gc, cseed, c);
        float* o = out + r * dim;
        for (int j = 0; j < dim; ++j) {
            float cj = rng_gauss(gc);
            o[j] = cj + sigma * rng_gauss(g);
        }
        if (normalize) {
            double ss = 0;
            for (int j = 0; j < dim; ++j) ss += (double)o[j] * o[j];
            if (ss > 0) {
                double inv = 1.0 / std::sqrt(ss);
                for (int j = 0; j < dim; ++j) o[j] = (float)(o[j] * inv);
            }
        }
    });
}

// ---------------------------------------------------------------------------------------------
// Exact flat k-NN.
//   metric 0 = squared L2   (CPU/CPUTopK.swift:34-112; L2Distance.metal:65-69)
//   metric 1 = cosine distance 1 - sim, sim = dot/(|q||x|), 0 when a norm is 0, clamped to
//              [-1, 1]        (Operations/AccelerateFallback.swift:27-49,209-243;
//                              Integration/MetalComputeProvider.swift:136;
//                              Metal/Shaders/DistanceShaders.metal:304-319)
//   metric 2 = inner product, larger is closer (AccelerateFallback.swift:52-60,240-248;
//              MetalComputeProvider.swift:212-217)
// x_dtype 0 = fp32 rows, 1 = bf16 rows (upcast exactly to fp32).
// acc 1 = truth mode: fp64 accumulation, one rounding to fp32.
// acc 0 = baseline mode: fp32 accumulation like vDSP (fp32 rows only).
// Output per query: k ids + k values sorted best-first; padding id 0xFFFFFFFF with +inf
// (min modes) or -inf (inner product).
// ---------------------------------------------------------------------------------------------
void orc_knn(const float* q, int64_t Q, const void* x, int x_dtype, int64_t N, int d, int k, int metric,
             int acc, int threads, uint32_t* out_ids, float* out_vals) {
    if (acc == 1) {
        knn_truth_rows(q, Q, x, x_dtype, N, d, k, metric, threads, out_ids, out_vals);
        return;
    }
    const float pad = metric == 2 ? -INFINITY : INFINITY;
    std::vector<double> xnorm;
    if (metric == 1) {
        xnorm.resize((size_t)N);
        parallel_for(N, threads, [&](int64_t i) {
            double s = 0;
            for (int j = 0; j < d; ++j) {
                double v = load_x(x, x_dtype, i * d + j);
                s += v * v;
            }
            xnorm[(size_t)i] = std::sqrt(s);
        });
    }
    // Queries are processed in blocks of QB so each database row is reused from cache.
    const int QB = 8;
    int64_t nblocks = (Q + QB - 1) / QB;
    parallel_for(nblocks, threads, [&](int64_t b) {
        int64_t q0 = b * QB, q1 = std::min<int64_t>(Q, q0 + QB);
        int nq = (int)(q1 - q0);
        std::vector<TopK> tops;
        for (int i = 0; i < nq; ++i) tops.emplace_back(k);
        double qn[QB];
        for (int i = 0; i < nq; ++i) {
            double s = 0;
            for (int j = 0; j < d; ++j) s += (double)q[(q0 + i) * d + j] * q[(q0 + i) * d + j];
            qn[i] = std::sqrt(s);
        }
        for (int64_t n = 0; n < N; ++n) {
            for (int i = 0; i < nq; ++i) {
                const float* qq = q + (q0 + i) * d;
                float val;
                if (acc == 0 && x_dtype == 0) {
                    const float* xx = (const float*)x + n * d;
                    if (metric == 0) val = l2sq_f32(qq, xx, d);
                    else if (metric == 2) val = dot_f32(qq, xx, d);
                    else {
                        float dt = dot_f32(qq, xx, d);
                        double den = qn[i] * xnorm[(size_t)n];
                        double sim = den > 0 ? (double)dt / den : 0.0;
                        sim = std::min(1.0, std::max(-1.0, sim));
                        val = (float)(1.0 - sim);
                    }
                } else {
                    double s = 0;
                    if (metric == 0) {
                        for (int j = 0; j < d; ++j) {
                            double t = (double)qq[j] - (double)load_x(x, x_dtype, n * d + j);
                            s += t * t;
                        }
                        val = (float)s;
                    } else {
                        for (int j = 0; j < d; ++j) s += (double)qq[j] * (double)load_x(x, x_dtype, n * d + j);
                        if (metric == 2) val = (float)s;
                        else {
                            double den = qn[i] * xnorm[(size_t)n];
                            double sim = den > 0 ? s / den : 0.0;
                            sim = std::min(1.0, std::max(-1.0, sim));
                            val = (float)(1.0 - sim);
                        }
                    }
                }
                uint32_t key = metric == 2 ? ~f2key(val) : f2key(val);
                if (std::isnan(val)) key = 0xFFFFFFFFu;
                if (tops[i].would_accept(key, (uint32_t)n)) tops[i].push(Cand{key, (uint32_t)n, val});
            }
        }
        for (int i = 0; i < nq; ++i)
            tops[i].emit(k, pad, out_ids ? out_ids + (q0 + i) * k : nullptr,
                         out_vals ? out_vals + (q0 + i) * k : nullptr);
    });
}

// Exact distances of explicit (query, candidate) pairs, in truth mode (fp64, one rounding).
// cand_ids is Q x kc; ids equal to 0xFFFFFFFF produce the pad value. Used to check reranks.
void orc_rerank(const float* q, int64_t Q, const void* x, int x_dtype, int d, const uint32_t* cand_ids,
                int kc, int k, int metric, int threads, uint32_t* out_ids, float* out_vals) {
    const float pad = metric == 2 ? -INFINITY : INFINITY;
    parallel_for(Q, threads, [&](int64_t qi) {
        TopK top(k);
        const float* qq = q + qi * d;
        double qn = 0;
        for (int j = 0; j < d; ++j) qn += (double)qq[j] * qq[j];
        qn = std::sqrt(qn);
        for (int c = 0; c < kc; ++c) {
            uint32_t id = cand_ids[qi * kc + c];
            if (id == 0xFFFFFFFFu) continue;
            double s = 0, xn = 0;
            for (int j = 0; j < d; ++j) {
                double xv = load_x(x, x_dtype, (int64_t)id * d + j);
                if (metric == 0) {
                    double t = (double)qq[j] - xv;
                    s += t * t;
                } else {
                    s += (double)qq[j] * xv;
                    xn += xv * xv;
                }
            }
            float val;
            if (metric == 0 || metric == 2) val = (float)s;
            else {
                double den = qn * std::sqrt(xn);
                double sim = den > 0 ? s / den : 0.0;
                sim = std::min(1.0, std::max(-1.0, sim));
                val = (float)(1.0 - sim);
            }
            uint32_t key = metric == 2 ? ~f2key(val) : f2key(val);
            top.push(Cand{key, id, val});
        }
        top.emit(k, pad, out_ids + qi * k, out_vals + qi * k);
    });
}

// ---------------------------------------------------------------------------------------------
// Batch top-K over a value matrix (TopKSelectionKernel.select, Kernels/Metal4/
// TopKSelectionKernel.swift:369-411; topk_select_batch_kernel SearchAndRetrieval.metal:88-156).
// mode 0 = minimum, 1 = maximum. Row r holds n values at in + r*in_stride. Output sorted
// best-first; padding +inf / -inf with id 0xFFFFFFFF (SearchAndRetrieval.metal:151-155).
// ---------------------------------------------------------------------------------------------
void orc_topk_select(const float* in, int64_t batch, int64_t n, int64_t in_stride, int k, int mode,
                     int threads, float* out_vals, uint32_t* out_ids) {
    const float pad = mode == 1 ? -INFINITY : INFINITY;
    parallel_for(batch, threads, [&](int64_t r) {
        TopK top(k);
        const float* row = in + r * in_stride;
        for (int64_t i = 0; i < n; ++i) {
            float v = row[i];
            uint32_t key = mode == 1 ? ~f2key(v) : f2key(v);
            if (std::isnan(v)) key = 0xFFFFFFFFu;
            if (top.would_accept(key, (uint32_t)i)) top.push(Cand{key, (uint32_t)i, v});
        }
        top.emit(k, pad, out_ids + r * k, out_vals + r * k);
    });
}

// Merge of a running sorted top-k with a chunk's sorted top-kc whose ids are chunk-local
// (merge_topk_sorted_kernel, SearchAndRetrieval.metal:320-385; TopKMergeKernel.swift:18-127):
// chunk ids get chunk_base added; the result is the best k of the union under (key, id).
void orc_topk_merge(const float* run_vals, const uint32_t* run_ids, int k, const float* chunk_vals,
                    const uint32_t* chunk_ids, int kc, uint32_t chunk_base, int64_t Q, int mode,
                    float* out_vals, uint32_t* out_ids) {
    const float pad = mode == 1 ? -INFINITY : INFINITY;
    for (int64_t qi = 0; qi < Q; ++qi) {
        TopK top(k);
        for (int i = 0; i < k; ++i) {
            uint32_t id = run_ids[qi * k + i];
            if (id == 0xFFFFFFFFu) continue;
            float v = run_vals[qi * k + i];
            top.push(Cand{mode == 1 ? ~f2key(v) : f2key(v), id, v});
        }
        for (int i = 0; i < kc; ++i) {
            uint32_t id = chunk_ids[qi * kc + i];
            if (id == 0xFFFFFFFFu) continue;
            float v = chunk_vals[qi * kc + i];
            top.push(Cand{mode == 1 ? ~f2key(v) : f2key(v), id + chunk_base, v});
        }
        top.emit(k, pad, out_ids + qi * k, out_vals + qi * k);
    }
}

// ---------------------------------------------------------------------------------------------
// Pair and matrix distances (truth mode: fp64 accumulation, one rounding).
// ---------------------------------------------------------------------------------------------

// 1:1 pairs, L2 (l2_distance, DistanceShaders.metal:169-226): squared unless compute_sqrt.
void orc_l2_pairs(const float* a, const float* b, int64_t pairs, int d, int compute_sqrt, float* out) {
    for (int64_t p = 0; p < pairs; ++p) {
        double s = 0;
        for (int j = 0; j < d; ++j) {
            double t = (double)a[p * d + j] - b[p * d + j];
            s += t * t;
        }
        out[p] = compute_sqrt ? (float)std::sqrt(s) : (float)s;
    }
}

// 1:1 pairs, cosine (cosine_similarity, DistanceShaders.metal:239-321): sim = dot/(|a||b|),
// 0 when the denominator is below FLT_MIN, clamped to [-1,1]; distance output 1 - sim.
void orc_cosine_pairs(const float* a, const float* b, int64_t pairs, int d, int output_distance, float* out) {
    for (int64_t p = 0; p < pairs; ++p) {
        double dt = 0, aa = 0, bb = 0;
        for (int j = 0; j < d; ++j) {
            double x = a[p * d + j], y = b[p * d + j];
            dt += x * y;
            aa += x * x;
            bb += y * y;
        }
        double den = std::sqrt(aa) * std::sqrt(bb);
        double sim = den < (double)FLT_MIN ? 0.0 : dt / den;
        sim = std::min(1.0, std::max(-1.0, sim));
        out[p] = output_distance ? (float)(1.0 - sim) : (float)sim;
    }
}

// All-pairs matrices Q x N: metric 0 = squared L2 (l2_distance_kernel, L2Distance.metal:34-91,
// optional sqrt), 2 = dot (dot_product_kernel, DotProduct.metal:29-96, optional abs),
// 1 = cosine similarity (or 1 - sim when flag set). flag: sqrt / abs / distance.
void orc_matrix(const float* q, int64_t Q, const float* x, int64_t N, int d, int metric, int flag,
                int threads, float* out, int64_t out_stride) {
    parallel_for(Q, threads, [&](int64_t i) {
        double qn = 0;
        for (int j = 0; j < d; ++j) qn += (double)q[i * d + j] * q[i * d + j];
        for (int64_t n = 0; n < N; ++n) {
            double s = 0, xn = 0;
            for (int j = 0; j < d; ++j) {
                double a = q[i * d + j], b = x[n * d + j];
                if (metric == 0) {
                    s += (a - b) * (a - b);
                } else {
                    s += a * b;
                    xn += b * b;
                }
            }
            float v;
            if (metric == 0) v = flag ? (float)std::sqrt(s) : (float)s;
            else if (metric == 2) v = flag ? (float)std::fabs(s) : (float)s;
            else {
                double den = std::sqrt(qn) * std::sqrt(xn);
                double sim = den < (double)FLT_MIN ? 0.0 : s / den;
                sim = std::min(1.0, std::max(-1.0, sim));
                v = flag ? (float)(1.0 - sim) : (float)sim;
            }
            out[i * out_stride + n] = v;
        }
    });
}

// ---------------------------------------------------------------------------------------------
// Scalar quantization.
// ---------------------------------------------------------------------------------------------

// Global parameters (ScalarQuantizationKernel.computeQuantizationParams,
// Kernels/Metal4/ScalarQuantizationKernel.swift:496-520). type 0 symmetric, 1 asymmetric.
// bits 8 or 4. Returns scale; *zero_point set (0 for symmetric).
float orc_sq_params(const float* x, int64_t n, int type, int bits, int8_t* zero_point) {
    float mn = 0, mx = 0;
    if (n > 0) {
        mn = x[0];
        mx = x[0];
        for (int64_t i = 1; i < n; ++i) {
            mn = std::min(mn, x[i]);
            mx = std::max(mx, x[i]);
        }
    }
    float smax = bits == 4 ? 7.0f : 127.0f, amax = bits == 4 ? 15.0f : 255.0f;
    if (type == 1) {
        float scale = std::max((mx - mn) / amax, 1e-8f);
        // Int8(clamping: Int(-round(min/scale))) -- Swift round() is half away from zero.
        double zr = -std::round((double)(mn / scale));
        if (zr < -128) zr = -128;
        if (zr > 127) zr = 127;
        *zero_point = (int8_t)zr;
        return scale;
    }
    float absmax = std::max(std::fabs(mn), std::fabs(mx));
    *zero_point = 0;
    return std::max(absmax / smax, 1e-8f);
}

// quantize_int8_kernel (Metal/Shaders/DataTransformations.metal:174-201): q = clamp(rint(x/scale
// + zp), -128, 127); per-channel parameters use contiguous blocks channel = i / per_channel
// (:142-171). scales/zps may be null (global). rint = round half to even.
void orc_quantize_int8(const float* x, int64_t n, float gscale, int8_t gzp, const float* scales,
                       const int8_t* zps, int64_t per_channel, int64_t n_channels, int8_t* out) {
    for (int64_t i = 0; i < n; ++i) {
        float s = gscale;
        int8_t z = gzp;
        if (scales && per_channel > 0) {
            int64_t c = i / per_channel;
            if (c < n_channels) {
                s = scales[c];
                z = zps ? zps[c] : 0;
            }
        }
        if (std::fabs(s) < 1e-9f) {
            out[i] = z;
            continue;
        }
        float v = x[i] / s + (float)z;
        float r = std::nearbyint(v);
        r = std::min(127.0f, std::max(-128.0f, r));
        out[i] = (int8_t)r;
    }
}

// dequantize_int8_kernel (DataTransformations.metal:203-221): x = (q - zp) * scale.
void orc_dequantize_int8(const int8_t* in, int64_t n, float gscale, int8_t gzp, const float* scales,
                         const int8_t* zps, int64_t per_channel, int64_t n_channels, float* out) {
    for (int64_t i = 0; i < n; ++i) {
        float s = gscale;
        int8_t z = gzp;
        if (scales && per_channel > 0) {
            int64_t c = i / per_channel;
            if (c < n_channels) {
                s = scales[c];
                z = zps ? zps[c] : 0;
            }
        }
        out[i] = ((float)in[i] - (float)z) * s;
    }
}

// int4 (DataTransformations.metal:224-306): q = clamp(rint(x/scale + zp), -8, 7), two codes per
// byte, element 2i in the low nibble, 2i+1 in the high nibble. For an odd count the high nibble
// of the last byte holds the code of 0.0 (the shader loads 0.0f past the end, :249).
void orc_quantize_int4(const float* x, int64_t n, float gscale, int8_t gzp, uint8_t* out) {
    const int64_t nb = (n + 1) / 2;
    for (int64_t i = 0; i < nb; ++i) out[i] = 0;
    for (int64_t i = 0; i < 2 * nb; ++i) {
        const float v = i < n ? x[i] : 0.0f;
        float r = std::fabs(gscale) < 1e-9f ? (float)gzp : std::nearbyint(v / gscale + (float)gzp);
        int q = (int)std::min(7.0f, std::max(-8.0f, r));
        uint8_t nib = (uint8_t)(q & 0xF);
        out[i / 2] |= (i & 1) ? (uint8_t)(nib << 4) : nib;
    }
}

void orc_dequantize_int4(const uint8_t* in, int64_t n, float gscale, int8_t gzp, float* out) {
    for (int64_t i = 0; i < n; ++i) {
        uint8_t nib = (i & 1) ? (uint8_t)(in[i / 2] >> 4) : (uint8_t)(in[i / 2] & 0xF);
        int q = (nib & 0x8) ? (int)nib - 16 : (int)nib;
        out[i] = ((float)q - (float)gzp) * gscale;
    }
}

// Per-dimension int8 codes for the int8 search path. The reference has only global scales and
// block-contiguous channels, so the per-dimension definition is this build's own (stated):
// scale_j = max((max_j - min_j)/255, 1e-8); u = clamp(rint((x - min_j)/scale_j), 0, 255);
// code = u - 128. L2 on codes is invariant to the -128 shift.
void orc_sq_perdim_params(const float* x, int64_t n, int d, float* mins, float* scales) {
    for (int j = 0; j < d; ++j) {
        float mn = INFINITY, mx = -INFINITY;
        for (int64_t i = 0; i < n; ++i) {
            mn = std::min(mn, x[i * d + j]);
            mx = std::max(mx, x[i * d + j]);
        }
        if (n == 0) mn = mx = 0;
        mins[j] = mn;
        scales[j] = std::max((mx - mn) / 255.0f, 1e-8f);
    }
}

void orc_sq_perdim_quantize(const float* x, int64_t n, int d, const float* mins, const float* scales,
                            int8_t* codes) {
    for (int64_t i = 0; i < n; ++i)
        for (int j = 0; j < d; ++j) {
            float u = std::nearbyint((x[i * d + j] - mins[j]) / scales[j]);
            u = std::min(255.0f, std::max(0.0f, u));
            codes[i * d + j] = (int8_t)((int)u - 128);
        }
}

// Integer L2 top-kc on codes (exact int32 sum of squared code differences), then exact rerank
// of those kc candidates against the original fp32 rows, final top-k by (distance, id).
// Writes the integer candidate lists too when cand_ids/cand_dists are non-null.
void orc_int8_knn(const int8_t* qc, const float* qf, int64_t Q, const int8_t* xc, const float* xf, int64_t N,
                  int d, int kc, int k, int threads, uint32_t* cand_ids, int32_t* cand_dists, uint32_t* out_ids,
                  float* out_vals) {
    parallel_for(Q, threads, [&](int64_t qi) {
        TopK top(kc);
        const int8_t* a = qc + qi * d;
        for (int64_t n = 0; n < N; ++n) {
            const int8_t* b = xc + n * d;
            int32_t s = 0;
            for (int j = 0; j < d; ++j) {
                int32_t t = (int32_t)a[j] - (int32_t)b[j];
                s += t * t;
            }
            uint32_t key = (uint32_t)s;
            if (top.would_accept(key, (uint32_t)n)) top.push(Cand{key, (uint32_t)n, (float)s});
        }
        std::vector<uint32_t> ids((size_t)kc);
        std::vector<float> vals((size_t)kc);
        top.emit(kc, INFINITY, ids.data(), vals.data());
        if (cand_ids)
            for (int i = 0; i < kc; ++i) cand_ids[qi * kc + i] = ids[(size_t)i];
        if (cand_dists)
            for (int i = 0; i < kc; ++i)
                cand_dists[qi * kc + i] = ids[(size_t)i] == 0xFFFFFFFFu ? -1 : (int32_t)vals[(size_t)i];
        TopK fin(k);
        const float* qq = qf + qi * d;
        for (int i = 0; i < kc; ++i) {
            uint32_t id = ids[(size_t)i];
            if (id == 0xFFFFFFFFu) continue;
            double s = 0;
            for (int j = 0; j < d; ++j) {
                double t = (double)qq[j] - (double)xf[(int64_t)id * d + j];
                s += t * t;
            }
            float v = (float)s;
            fin.push(Cand{f2key(v), id, v});
        }
        fin.emit(k, INFINITY, out_ids + qi * k, out_vals + qi * k);
    });
}

// ---------------------------------------------------------------------------------------------
// Binary quantization and Hamming distance.
// ---------------------------------------------------------------------------------------------

// binaryQuantize (Metal/Shaders/QuantizationShaders.metal:132-160): bit b of word w is dimension
// 32w+b (LSB first), set when value > threshold (the shader compares with 0.0 and ignores the
// host's threshold; pass 0 for the reference behaviour).
void orc_binary_quantize(const float* x, int64_t n, int d, float threshold, uint32_t* out) {
    int words = (d + 31) / 32;
    for (int64_t i = 0; i < n; ++i)
        for (int w = 0; w < words; ++w) {
            uint32_t word = 0;
            for (int b = 0; b < 32 && w * 32 + b < d; ++b)
                if (x[i * d + w * 32 + b] > threshold) word |= 1u << b;
            out[i * words + w] = word;
        }
}

// Hamming Q x N (hamming_distance_batch, Metal/Shaders/HammingDistance.metal:28-127;
// Metal4BinaryVector.hammingDistance, Kernels/Metal4/BinaryQuantizationKernel.swift:65-74).
void orc_hamming_matrix(const uint32_t* q, int64_t Q, const uint32_t* x, int64_t N, int words, uint32_t* out) {
    for (int64_t i = 0; i < Q; ++i)
        for (int64_t n = 0; n < N; ++n) {
            uint32_t s = 0;
            for (int w = 0; w < words; ++w) s += (uint32_t)__builtin_popcount(q[i * words + w] ^ x[n * words + w]);
            out[i * N + n] = s;
        }
}

// Hamming k-NN by (distance, id) ascending. The reference's only route is a full CPU sort of the
// materialised Q x N matrix (Metal4HammingResult.nearestNeighbors, HammingDistanceKernel.swift:
// 114-120); this returns the same ordered prefix without materialising it.
void orc_hamming_knn(const uint32_t* q, int64_t Q, const uint32_t* x, int64_t N, int words, int k, int threads,
                     uint32_t* out_ids, uint32_t* out_dists) {
    parallel_for(Q, threads, [&](int64_t i) {
        TopK top(k);
        const uint32_t* a = q + i * words;
        for (int64_t n = 0; n < N; ++n) {
            const uint32_t* b = x + n * words;
            uint32_t s = 0;
            for (int w = 0; w < words; ++w) s += (uint32_t)__builtin_popcount(a[w] ^ b[w]);
            if (top.would_accept(s, (uint32_t)n)) top.push(Cand{s, (uint32_t)n, (float)s});
        }
        std::sort(top.h.begin(), top.h.end(), cand_less);
        for (int j = 0; j < k; ++j) {
            if (j < (int)top.h.size()) {
                out_ids[i * k + j] = top.h[(size_t)j].id;
                out_dists[i * k + j] = top.h[(size_t)j].key;
            } else {
                out_ids[i * k + j] = 0xFFFFFFFFu;
                out_dists[i * k + j] = 0xFFFFFFFFu;
            }
        }
    });
}

// Round fp32 -> bf16 (round to nearest even; NaN kept quiet). Used to build bf16 databases on
// the host side of tests the same way the device conversion does.
void orc_f32_to_bf16(const float* x, int64_t n, uint16_t* out) {
    for (int64_t i = 0; i < n; ++i) {
        uint32_t u;
        std::memcpy(&u, &x[i], 4);
        if ((u & 0x7FFFFFFFu) > 0x7F800000u) {
            out[i] = (uint16_t)((u >> 16) | 0x40);
            continue;
        }
        uint32_t lsb = (u >> 16) & 1u;
        u += 0x7FFFu + lsb;
        out[i] = (uint16_t)(u >> 16);
    }
}

}  // extern "C"
