/*
 * va_cuda.h -- C ABI of libva_cuda, the B200 (sm_100a) exact-search library.
 *
 * This is the drop-in boundary for VectorAccelerate's exact flat k-NN path. Every entry point
 * replaces one reference interface (Swift class/method; file:line relative to the
 * VectorAccelerate project root) and keeps its argument meaning, result conventions and error
 * behaviour:
 *   - ids are uint32; 0xFFFFFFFF pads a result row when fewer than k candidates exist
 *     (FusedL2TopKKernel.swift:155-172, SearchAndRetrieval.metal:151-155);
 *   - squared L2 is returned (computeSqrt = false), ascending; inner product is returned
 *     descending; cosine distance is 1 - similarity, ascending;
 *   - every selection orders by (distance, id): equal distances keep the smaller id
 *     (AdvancedTopK.metal:48-52, SearchAndRetrieval.metal:313-317);
 *   - distance pads are +inf (minimum modes) and -inf (maximum modes).
 *
 * Conventions of this ABI:
 *   - plain pointers and sizes only; device pointers are CUDA device addresses on the
 *     context's device, host pointers are ordinary (pageable or pinned) memory;
 *   - every function returns an int status: VA_OK (0) or a negative VA_ERR_* code, and never
 *     aborts; va_last_error() returns a thread-local message naming the offending parameter and
 *     its limit (IndexError.invalidInput messages, FusedL2TopKKernel.swift:52-85);
 *   - work is enqueued on the context's stream (stream order replaces Metal's memoryBarrier);
 *     va_synchronize() is the bounded wait that replaces Metal4Context.executeAndWait
 *     (Core/Metal4Context.swift:342-410);
 *   - there is no CPU fallback: without a usable GPU every call fails with VA_ERR_CUDA.
 */
#ifndef VA_CUDA_H
#define VA_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#define VA_ABI_VERSION 1

/* ------------------------------------------------------------------------------------------ */
/* Status codes                                                                                */
/* ------------------------------------------------------------------------------------------ */
#define VA_OK 0
#define VA_ERR_INVALID_ARG (-1) /* VectorError.invalidInput / IndexError.invalidInput           */
#define VA_ERR_OOM (-2)         /* VectorError.bufferAllocationFailed                            */
#define VA_ERR_CUDA (-3)        /* VectorError.computeFailed (commandBuffer.error)               */
#define VA_ERR_NCCL (-4)        /* collective failure (no reference counterpart: single GPU)     */
#define VA_ERR_TIMEOUT (-5)     /* a bounded host wait or a bounded device wait expired          */
#define VA_ERR_UNSUPPORTED (-6) /* combination not supported by this build                       */

/* Metrics (SupportedDistanceMetric subset on the flat path). */
#define VA_METRIC_L2SQ 0   /* squared Euclidean, smaller is closer                                */
#define VA_METRIC_COSINE 1 /* 1 - cos(q, x), smaller is closer                                    */
#define VA_METRIC_IP 2     /* inner product, larger is closer                                      */

/* Contraction precision of the fused search. Reduced-precision passes are always followed by an
 * exact rerank of the candidates, so results equal the exact search's apart from stated ties. */
#define VA_PREC_AUTO 0 /* BF16 with a pool of >= 3k candidates (TF32 for bf16 rows at large k,
                          FP32 when no pool fits or d <= 16)                                  */
#define VA_PREC_FP32 1 /* exact fp32 SIMT contraction, chunked, no rerank needed             */
#define VA_PREC_TF32 2 /* tcgen05 kind::tf32 on the fp32 rows + exact rerank                 */
#define VA_PREC_BF16 3 /* tcgen05 kind::f16 (bf16) + exact rerank                            */

/* Row element types of a database. */
#define VA_DTYPE_F32 0
#define VA_DTYPE_BF16 1

/* Selection modes (Metal4SelectionMode, TopKSelectionKernel.swift:23-29). */
#define VA_SELECT_MIN 0
#define VA_SELECT_MAX 1

/* Limits of this build (the reference caps d <= 768 and k <= 128:
 * FusedL2TopKKernel.swift:39-42; TopKSelectionKernel.swift:60). */
#define VA_MAX_DIM 4096
#define VA_MAX_K 1024
#define VA_MAX_SELECT_K 4096

typedef struct va_context va_context;
typedef struct va_database va_database;
typedef struct va_ivf va_ivf;

/* Context configuration (Metal4Configuration, Core/Metal4Context.swift:13-44). */
typedef struct va_config {
    int device;              /* CUDA device ordinal                                            */
    unsigned int timeout_ms; /* limit of every bounded wait; 0 selects 120000                  */
    void* stream;            /* optional cudaStream_t to enqueue on; NULL creates one          */
} va_config;

/* ------------------------------------------------------------------------------------------ */
/* Errors, devices, contexts                                                                   */
/* ------------------------------------------------------------------------------------------ */
const char* va_last_error(void);
int va_abi_version(void);
int va_device_count(int* count);

/* Replaces Metal4Context.init(configuration:) (Core/Metal4Context.swift:175-183). */
int va_context_create(const va_config* cfg, va_context** out);
int va_context_destroy(va_context* ctx);
/* The cudaStream_t the context enqueues on. */
int va_context_stream(va_context* ctx, void** stream);
/* Bounded wait for all enqueued work, then a check of the device error word written by bounded
 * device-side waits. Replaces executeAndWait's commit/wait/error check
 * (Core/Metal4Context.swift:377-409). */
int va_synchronize(va_context* ctx);
/* Device time in ms of the last call that timed itself (GPUTimingInfo, Metal4Context.swift:48-65). */
int va_last_gpu_time_ms(va_context* ctx, float* ms);
/* Device times of the last va_knn_search on this context, measured with CUDA events on the
 * context stream: the whole search and its dominant kernel (the tensor-core filter; 0 on the
 * FP32 route). Valid once the search has completed (after va_synchronize). */
int va_last_search_times(va_context* ctx, float* total_ms, float* kernel_ms);
/* Profile the dominant kernel of the next `capacity` searches (a CUDA event pair per call on
 * the context stream, no synchronisation between calls); va_profile_stop waits (bounded) and
 * returns the summed kernel time and the number of profiled calls. */
int va_profile_start(va_context* ctx, int capacity);
int va_profile_stop(va_context* ctx, float* kernel_ms_total, int* calls);

/* ------------------------------------------------------------------------------------------ */
/* Buffers: replace MTLBuffer / BufferToken (Core/BufferPool.swift:89-221,                     */
/* Core/Metal4Context.swift:471-488). Caller-owned; free with va_buffer_free.                  */
/* ------------------------------------------------------------------------------------------ */
int va_buffer_alloc(va_context* ctx, size_t bytes, void** dptr);
int va_buffer_free(va_context* ctx, void* dptr);
int va_host_alloc(va_context* ctx, size_t bytes, void** hptr); /* pinned host memory */
int va_host_free(va_context* ctx, void* hptr);
/* Stream-ordered copies (host<->device or device<->device); asynchronous for page-locked host
 * memory. With pageable host memory the call first waits (bounded, as va_synchronize) for the
 * stream, then copies: it returns when the copy is done, or with VA_ERR_TIMEOUT / VA_ERR_NCCL. */
int va_buffer_upload(va_context* ctx, void* dst_dev, const void* src_host, size_t bytes);
int va_buffer_download(va_context* ctx, void* dst_host, const void* src_dev, size_t bytes);
int va_buffer_copy(va_context* ctx, void* dst_dev, const void* src_dev, size_t bytes);

/* ------------------------------------------------------------------------------------------ */
/* Distance primitives (device pointers, fp32, stream-ordered)                                 */
/* ------------------------------------------------------------------------------------------ */
/* 1:1 pairs: out[p] = |a_p - b_p|^2 (or |a_p - b_p| when compute_sqrt).
 * Replaces L2DistanceKernel.encode (Kernels/Metal4/L2DistanceKernel.swift:49-86). */
int va_l2_distance_pairs(va_context* ctx, const float* a, const float* b, int64_t pairs, int dim,
                         int compute_sqrt, float* out);
/* 1:1 pairs: cosine similarity, or 1 - similarity when output_distance; 0 when a norm is 0.
 * Replaces CosineSimilarityKernel.encode (Kernels/Metal4/CosineSimilarityKernel.swift:50-87). */
int va_cosine_pairs(va_context* ctx, const float* a, const float* b, int64_t pairs, int dim,
                    int output_distance, float* out);
/* All-pairs matrix out[i*out_stride + j] for queries q[nq x dim], rows x[nx x dim]:
 *   VA_METRIC_L2SQ: squared L2 (sqrt when flag)      -- l2_distance_kernel, L2Distance.metal:34-91
 *   VA_METRIC_IP:   dot product (abs when flag)      -- DotProductKernel.encode,
 *                                                       Kernels/Metal4/DotProductKernel.swift:226-275
 *   VA_METRIC_COSINE: similarity (1 - sim when flag) -- cosine all-pairs, CosineSimilarity.metal */
int va_distance_matrix(va_context* ctx, const float* q, int64_t nq, const float* x, int64_t nx, int dim,
                       int metric, int flag, float* out, int64_t out_stride);

/* ------------------------------------------------------------------------------------------ */
/* Selection                                                                                   */
/* ------------------------------------------------------------------------------------------ */
/* Batch top-k of rows in[r*in_stride + i], i < n: sorted best-first by (value, index).
 * Replaces TopKSelectionKernel.execute/select (Kernels/Metal4/TopKSelectionKernel.swift:228-411)
 * and WarpOptimizedSelectionKernel (WarpOptimizedSelectionKernel.swift:250-863).
 * k <= VA_MAX_SELECT_K. out rows have stride out_stride (>= k). */
int va_topk_select(va_context* ctx, const float* in, int64_t batch, int64_t n, int64_t in_stride, int k,
                   int mode, float* out_vals, uint32_t* out_ids, int64_t out_stride);
/* Merge a running sorted top-k with a chunk's sorted top-kc whose ids are chunk-local (chunk_base
 * is added). Replaces TopKMergeKernel (Kernels/Metal4/TopKMergeKernel.swift:18-127). Output may
 * alias the running buffers. */
int va_topk_merge(va_context* ctx, const float* run_vals, const uint32_t* run_ids, int k, const float* chunk_vals,
                  const uint32_t* chunk_ids, int kc, uint32_t chunk_base, int64_t nq, int mode, float* out_vals,
                  uint32_t* out_ids);
/* Merge per-shard results gathered as [nshards][nq][k] (global ids) into the global top-k.
 * The device merge after the NCCL allgather of a row-sharded search (no reference counterpart:
 * the reference is single-GPU; its chunk merge is SearchAndRetrieval.metal:320-385). */
int va_merge_shards(va_context* ctx, const float* vals, const uint32_t* ids, int nshards, int64_t nq, int k,
                    int mode, float* out_vals, uint32_t* out_ids);

/* ------------------------------------------------------------------------------------------ */
/* Database and fused search                                                                   */
/* ------------------------------------------------------------------------------------------ */
/* Create a resident database of n rows x dim (row-major, dtype VA_DTYPE_F32 or VA_DTYPE_BF16),
 * copied from host (on_device = 0) or device memory. Replaces the storage buffer of
 * GPUVectorStorage (Index/Internal/GPUVectorStorage.swift:52-100). id_base is added to every
 * returned id (global ids of a row shard). At build time the library derives the tensor-core
 * operand copy (bf16, normalised for cosine) and the row norms. */
int va_db_create(va_context* ctx, const void* rows, int on_device, int64_t n, int dim, int dtype,
                 uint32_t id_base, va_database** out);
int va_db_destroy(va_database* db);
int va_db_info(const va_database* db, int64_t* n, int* dim, int* dtype);
/* Device pointer of the database's original rows (fp32 or bf16 per dtype). */
int va_db_rows(const va_database* db, const void** rows);

/* Ingestion (GPUVectorStorage write / ensureCapacity / compact, Index/Internal/
 * GPUVectorStorage.swift:75-260): append `count` rows (the database's row format: dtype rows,
 * or packed uint32 codes for a binary database) from host or device memory, growing capacity
 * geometrically; overwrite rows [slot0, slot0 + count); keep only the rows whose keep[i] != 0
 * (host array of the current row count), in order. Norms, tensor-core operands, int8 codes and a
 * resident bit expansion are updated for the written rows. new_slot (optional, host, one per old
 * row) receives each row's new index or -1. Stream-ordered; compaction waits for the stream. */
int va_db_append(va_context* ctx, va_database* db, const void* rows, int on_device, int64_t count);
int va_db_update(va_context* ctx, va_database* db, int64_t slot0, const void* rows, int on_device, int64_t count);
int va_db_compact(va_context* ctx, va_database* db, const uint8_t* keep, int64_t* new_slot);

/* Fused exact k-NN over the database: queries[nq x dim] fp32 (device), results sorted
 * best-first into out_vals/out_ids [nq x k] (device). Replaces FusedL2TopKKernel.execute
 * (Kernels/Metal4/FusedL2TopKKernel.swift:367-427) and the batch flat search
 * AcceleratedVectorIndex.searchBatchGPU (Index/AcceleratedVectorIndex.swift:1278-1374), extended
 * to cosine and inner product. rerank = candidate-pool factor of the reduced-precision pass
 * (pool = rerank * k; 0 = automatic: k + max(k/4, 22), widened to 3k for bf16).
 * Exactness: the reduced-precision keys only choose a candidate pool, which is reranked exactly;
 * a per-query certificate (a rigorous bound of the keys' rounding error against the gap between
 * the k-th exact distance and the pool's last key) proves that no row outside the pool can enter
 * the top k; where the pool's last key is too close, the candidates the filter kept beyond the
 * pool (below the last key of every full list and the shared bound) are reranked too. Queries
 * that still fail take a second tensor-core pass with a wider pool (the next list size, or at
 * least 4x and 512 when more than 1/32 of the batch fails; the database then keeps that pool for
 * the metric), and what that cannot certify takes the exact SIMT route, so every result is the
 * exact top k.
 * The tensor-core route reads back the count of uncertified queries, so the call waits for the
 * stream once (twice when a second pass runs). A context serves one host thread at a time (its
 * scratch buffers are shared by its calls). */
int va_knn_search(va_context* ctx, const va_database* db, const float* queries, int64_t nq, int k, int metric,
                  int precision, int rerank, float* out_vals, uint32_t* out_ids);
/* Counts of the last va_knn_search (or va_knn_search_noalloc) on this context: queries whose first
 * tensor-core pass was not certified exact, and queries that took the exact SIMT route (all of
 * them on the FP32 route). No reference counterpart (the reference's fused kernel is fp32). */
int va_last_search_stats(va_context* ctx, int64_t* uncertified, int64_t* exact);
/* Same, with HOST query and result buffers: copies in, searches, copies out and waits (bounded).
 * This is the whole reference call (findNearestNeighbors, FusedL2TopKKernel.swift:439-529). */
int va_knn_search_host(va_context* ctx, const va_database* db, const float* queries_host, int64_t nq, int k,
                       int metric, int precision, int rerank, float* out_vals_host, uint32_t* out_ids_host);

/* Size of the fixed device scratch of va_knn_search_noalloc (16 MiB per GPU). */
#define VA_NOALLOC_SCRATCH_BYTES (16u << 20)
/* va_knn_search without any device allocation; this entry point has no counterpart in the
 * reference. For callers that must not allocate at search time: processes that give all free
 * device memory to their own pool at start-up, callers whose device memory belongs to another
 * allocator, and latency-bound paths that cannot take an allocation's implicit synchronisation.
 * Inputs, outputs and the database are the caller's, as for va_knn_search; the search's scratch
 * lives in one fixed device array of VA_NOALLOC_SCRATCH_BYTES that every GPU loading this
 * library holds until exit. It resolves AUTO exactly as va_knn_search does and returns the same
 * exact results (certificate included; uncertified queries take the exact SIMT route inside the
 * same array). Limits: the tensor-core route only, k <= 128; AUTO resolving to the FP32 route
 * (d <= 16 with fp32 rows) or k > 128 is rejected with VA_ERR_UNSUPPORTED. The candidate lists
 * take the route's pool (at most 128 entries) and are halved, never below k, while the batch does
 * not fit the array (results stay exact: the certificate sends what a thinner pool cannot prove
 * to the exact route). A batch that fits no list size is rejected with VA_ERR_INVALID_ARG naming
 * the bytes needed. At d = 768 and millions of rows, 32-entry lists fit about 1,400 queries per
 * call and 64-entry lists about 500; 128-entry lists (query tiles of 256 on 74 row splits) do not
 * fit, so k in 65..128 is rejected at that size. The database must
 * already hold the operand the metric/precision needs (bf16 for L2/IP is built by va_db_create;
 * others by a first va_knn_search), else VA_ERR_UNSUPPORTED. The first call on a device looks up
 * the array's device address (make it before any stream capture). Every call shares the array,
 * so calls that overlap on the GPU (other streams or contexts of the same device) race;
 * serialise them. The call waits for the stream once (the count of uncertified queries). */
int va_knn_search_noalloc(va_context* ctx, const va_database* db, const float* queries, int64_t nq, int k,
                          int metric, int precision, int rerank, float* out_vals, uint32_t* out_ids);

/* ------------------------------------------------------------------------------------------ */
/* Multi-GPU: row-sharded search over a group of devices (no reference counterpart: the        */
/* reference's Metal4Context, Core/Metal4Context.swift:175,183, owns one device).              */
/* ------------------------------------------------------------------------------------------ */
/* A group joins several devices with an NCCL communicator (loaded at run time: libnccl.so.2, or
 * the path in VA_NCCL_LIBRARY; VA_ERR_NCCL when absent). Its front context is an ordinary
 * va_context on the group's first local device: every call that takes a context accepts it.
 * A database sharded over the group holds rows [row0, row0 + rows) of the whole database on
 * each rank (N / ranks rows each, the last rank also the remainder: va_shard_range), with global
 * ids row0 + local row. va_knn_search, va_knn_search_host, va_int8_knn_search and
 * va_hamming_knn_db over a sharded database search every shard exactly (each shard's own local
 * top k, certified as on one device), exchange them in ONE ncclAllGather of packed 8-byte
 * (value, id) records per rank and merge by (distance, id) on the front context's device, so the
 * result equals the single-device search of the whole database. The communicators are
 * non-blocking: NCCL steps and va_synchronize poll ncclCommGetAsyncError against the context's
 * timeout and abort the communicators on expiry (VA_ERR_TIMEOUT) or error (VA_ERR_NCCL); an
 * aborted group refuses further collectives. A sharded database is not grown in place. */
#define VA_NCCL_ID_BYTES 128
/* An NCCL unique id for va_context_create_rank (made by one rank, shared with the others out of
 * band, e.g. through the launcher's store). */
int va_nccl_unique_id(void* id);
/* All listed devices in this process: one context and stream per device (cfg->stream, if set,
 * belongs to devices[0]), one communicator per device. The returned context is devices[0]'s;
 * queries and results of the sharded searches live there (queries reach the other devices by
 * ncclBroadcast; each device's search runs in its own host thread). Destroying it destroys
 * the group. */
int va_context_create_multi(const int* devices, int ndev, const va_config* cfg, va_context** out);
/* One rank of a group spread over processes (one process per GPU): cfg->device is this process's
 * device, nranks the group size, rank this process's rank, nccl_id the shared unique id. Every
 * rank calls it (NCCL initialisation is collective); the call waits, bounded by the timeout. */
int va_context_create_rank(const va_config* cfg, int nranks, int rank, const void* nccl_id, va_context** out);
/* Group size, the global rank of the context's first local device, and local devices (1, 0, 1
 * for a single-device context). */
int va_context_group(const va_context* ctx, int* nranks, int* rank, int* local_devices);
/* Rows [row0, row0 + rows) of an n-row database that local device `member` holds. */
int va_shard_range(const va_context* ctx, int64_t n, int member, int64_t* row0, int64_t* rows);
/* Row-sharded databases. `rows` holds the rows this process owns, in global order: all n rows
 * for a multi-device context, this rank's shard (va_shard_range) for a rank context; host memory
 * (on_device = 0) or device memory (on_device = 1; for a multi-device context, on devices[0]).
 * n is the row count of the WHOLE database. The int8 form codes every shard with the
 * per-dimension range of the whole database (min / max all-reduced over the group). */
int va_db_create_sharded(va_context* ctx, const void* rows, int on_device, int64_t n, int dim, int dtype,
                         va_database** out);
int va_db_create_int8_sharded(va_context* ctx, const float* rows, int on_device, int64_t n, int dim,
                              va_database** out);
int va_db_create_binary_sharded(va_context* ctx, const uint32_t* codes, int on_device, int64_t n, int dim_bits,
                                va_database** out);
/* The shard of local device `member` (a multi-device database), or the database itself (member 0
 * of a rank's shard or of an unsharded database). */
int va_db_shard(const va_database* db, int member, va_database** shard);

/* ------------------------------------------------------------------------------------------ */
/* Scalar quantization (ScalarQuantizationKernel, Kernels/Metal4/ScalarQuantizationKernel.swift;  */
/* quantize_int8_kernel / dequantize_int8_kernel / int4, DataTransformations.metal:142-306)      */
/* ------------------------------------------------------------------------------------------ */
/* q = clamp(rint(x/scale + zp), -128, 127). When scales != NULL, channel c = i / (n/n_channels)
 * uses scales[c] and zps[c] (zps may be NULL: 0). */
int va_sq_quantize_int8(va_context* ctx, const float* x, int64_t n, float scale, int8_t zero_point,
                        const float* scales, const int8_t* zps, int64_t n_channels, int8_t* out);
int va_sq_dequantize_int8(va_context* ctx, const int8_t* in, int64_t n, float scale, int8_t zero_point,
                          const float* scales, const int8_t* zps, int64_t n_channels, float* out);
/* int4: two codes per byte, element 2i in the low nibble; range [-8, 7]. */
int va_sq_quantize_int4(va_context* ctx, const float* x, int64_t n, float scale, int8_t zero_point, uint8_t* out);
int va_sq_dequantize_int4(va_context* ctx, const uint8_t* in, int64_t n, float scale, int8_t zero_point,
                          float* out);
/* Global min and max of x (device reduction); out_minmax[2] is a device pointer. */
int va_minmax(va_context* ctx, const float* x, int64_t n, float* out_minmax);
/* Per-dimension min and max of x[n x dim] (device): the statistics the reference's asymmetric
 * parameters take over the whole array (ScalarQuantizationKernel.swift:509-520), per column. */
int va_sq_perdim_minmax(va_context* ctx, const float* x, int64_t n, int dim, float* out_min, float* out_max);

/* ------------------------------------------------------------------------------------------ */
/* int8 scalar-quantized search                                                                */
/* ------------------------------------------------------------------------------------------ */
/* Resident int8 database: per-dimension codes of the fp32 rows[n x dim] (host or device), with
 * scale_j = max((max_j - min_j) / 255, 1e-8) and code = clamp(rint((x - min_j) / scale_j), 0, 255)
 * - 128 (the asymmetric uint8 mapping of ScalarQuantizationKernel.swift:509-520 applied per
 * dimension and shifted into int8). mins / maxs (device, [dim]) give the range, e.g. the global
 * range of a row-sharded database; NULL computes it over these rows. The fp32 rows stay resident
 * for the exact rerank. */
int va_db_create_int8(va_context* ctx, const float* rows, int on_device, int64_t n, int dim, const float* mins,
                      const float* maxs, uint32_t id_base, va_database** out);
/* Device pointers of an int8 database's parameters and codes (codes row stride in bytes). */
int va_db_int8_params(const va_database* db, const float** mins, const float** scales, const int8_t** codes,
                      int* code_stride);
/* int8 L2 k-NN: queries[nq x dim] fp32 (device) are quantized with the database's parameters;
 * squared L2 between codes in exact int32 arithmetic (tensor cores) selects the `candidates`
 * best rows per query by (integer distance, id); those are reranked by exact squared L2 against
 * the fp32 rows (fp64 accumulation); out_vals/out_ids [nq x k] sorted by (distance, id). No
 * reference counterpart (the reference has quantizers only, DataTransformations.metal:142-221);
 * this is the search its int8 storage would feed (IVFQuantizedStorage.swift). candidates <= 4096;
 * above 128 the call waits for the stream once (queries whose candidate set could not be proven
 * from the filter's lists are recomputed by an exact integer scan). */
int va_int8_knn_search(va_context* ctx, const va_database* db, const float* queries, int64_t nq, int k, int candidates,
                       float* out_vals, uint32_t* out_ids);

/* ------------------------------------------------------------------------------------------ */
/* Binary quantization and Hamming (BinaryQuantizationKernel, HammingDistanceKernel)           */
/* ------------------------------------------------------------------------------------------ */
/* Pack bit b of word w = (x[i][32w+b] > threshold), LSB first (binaryQuantize,
 * QuantizationShaders.metal:132-160; the shader fixes threshold = 0). out: n x ceil(dim/32). */
int va_binary_quantize(va_context* ctx, const float* x, int64_t n, int dim, float threshold, uint32_t* out);
/* Hamming matrix out[i*nx + j] = popcount(q_i ^ x_j) over `words` uint32 words
 * (hamming_distance_batch, HammingDistance.metal:28-127). out_normalized (optional, may be
 * NULL) receives distance / dim (hamming_distance_normalized, :242-321). */
int va_hamming_matrix(va_context* ctx, const uint32_t* q, int64_t nq, const uint32_t* x, int64_t nx, int words,
                      uint32_t* out, float* out_normalized, int dim);
/* Fused Hamming k-NN: distances never materialised; results sorted by (distance, id)
 * (replaces computeBitPacked + Metal4HammingResult.nearestNeighbors' CPU sort,
 * HammingDistanceKernel.swift:114-120,313-363). */
int va_hamming_knn(va_context* ctx, const uint32_t* q, int64_t nq, const uint32_t* x, int64_t nx, int words, int k,
                   uint32_t* out_dists, uint32_t* out_ids);
/* Resident binary database of n codes of dim_bits bits (LSB-first uint32 words, as
 * Metal4BinaryVector, BinaryQuantizationKernel.swift:23-74), host or device. */
int va_db_create_binary(va_context* ctx, const uint32_t* codes, int on_device, int64_t n, int dim_bits,
                        uint32_t id_base, va_database** out);
/* Rows expanded per pass of the batched search (rounded down to a multiple of 256; 0 =
 * automatic: the whole 0/1 expansion (dim_bits bytes per row) is kept resident when it fits in 60%
 * of the free device memory, otherwise chunks of half the free memory are expanded per pass).
 * Must be called before the first batched search. No counterpart in the reference. */
int va_db_binary_set_chunk_rows(va_database* db, int64_t rows);
/* Batched Hamming k-NN over a binary database on the integer tensor cores: popcount(q ^ x) =
 * |q| + |x| - 2 q.x over the 0/1 bits, exact; results sorted by (distance, id), k <= 128. Same
 * results as va_hamming_knn (HammingDistanceKernel.computeBitPacked + nearestNeighbors,
 * HammingDistanceKernel.swift:114-120,313-363). out_dists may be NULL. */
int va_hamming_knn_db(va_context* ctx, const va_database* db, const uint32_t* queries, int64_t nq, int k,
                      uint32_t* out_dists, uint32_t* out_ids);

/* ------------------------------------------------------------------------------------------ */
/* IVF index (IVFSearchPipeline, Index/Kernels/IVF/IVFSearchPipeline.swift:110-600; k-means      */
/* training, Index/Kernels/Clustering/KMeansPipeline.swift:102-240). Squared L2, fp32 rows.     */
/* ------------------------------------------------------------------------------------------ */
/* Initial centroids of va_ivf_train. */
#define VA_IVF_INIT_KMEANSPP 0 /* k-means++ (KMeansPlusPlusKernel.swift:94-210), draws from `seed` */
#define VA_IVF_INIT_GIVEN 1    /* the centroids out_centroids holds on entry */
#define VA_IVF_INIT_RANDOM 2   /* nlist distinct rows drawn from `seed` */
/* k-means over x[n x dim] (device): initial centroids per `init`, then Lloyd iterations (exact
 * assignment, mean update; an empty list keeps its centroid) until the largest centroid movement
 * is below tol or max_iters iterations ran. out_centroids [nlist x dim] (device); out_iters
 * (host, optional) = iterations run. Deterministic for a given seed. */
int va_ivf_train(va_context* ctx, const float* x, int64_t n, int dim, int nlist, int max_iters, float tol,
                 uint64_t seed, int init, float* out_centroids, int* out_iters);
/* Build the inverted lists: every row of rows[n x dim] (device) goes to its nearest centroid
 * (ties to the lower list), rows are copied in list order (stable within a list), ids are
 * row + id_base (IVFSearchPipeline.prepareIndexStructure, :110-195). */
int va_ivf_create(va_context* ctx, const float* rows, int64_t n, int dim, const float* centroids, int nlist,
                  uint32_t id_base, va_ivf** out);
/* The same from lists the caller has already formed (IVFSearchPipeline.prepareIndexStructure
 * with explicit lists, :110-185): centroids [nlist x dim], rows [offsets[nlist] x dim] in list
 * order, offsets [nlist + 1] (HOST, offsets[0] = 0), ids [offsets[nlist]] or NULL for the
 * position in the concatenated lists (the reference's vector index). centroids, rows and ids are
 * host (on_device = 0) or device (1) memory. */
int va_ivf_create_lists(va_context* ctx, const float* centroids, int nlist, int dim, const float* rows,
                        const int64_t* offsets, const uint32_t* ids, int on_device, va_ivf** out);
int va_ivf_destroy(va_ivf* ivf);
/* Rows per list (host array of nlist). */
int va_ivf_list_sizes(const va_ivf* ivf, int64_t* sizes);
/* Approximate k-NN (IVFSearchPipeline.search, :197-570): each query's nprobe nearest centroids
 * (ties by list id), then the k best rows of those lists by exact squared L2 and (distance, id),
 * sorted best-first; missing results are (+inf, 0xFFFFFFFF). queries [nq x dim], outputs
 * [nq x k], all device; k <= 128. For k <= 103 the lists are scanned on the tensor cores (the
 * queries of each list gathered into tiles of 128, a per-query bound shared by its probes) and a
 * candidate pool is reranked exactly: bf16 keys and max(3k, k + 22) candidates up to k = 42, tf32
 * keys and k + max(k/4, 22) candidates beyond; the tile layout is read back (the call waits for
 * the coarse step). Larger k: an exact fp64 scan, nq <= 65535. The index keeps one search
 * scratch: one search at a time per index. */
int va_ivf_search(va_context* ctx, const va_ivf* ivf, const float* queries, int64_t nq, int k, int nprobe,
                  float* out_vals, uint32_t* out_ids);
/* Same with HOST query and result buffers (copies in, searches, copies out, waits). The whole
 * reference call IVFSearchPipeline.search(queries:structure:k:). */
int va_ivf_search_host(va_context* ctx, const va_ivf* ivf, const float* queries_host, int64_t nq, int k, int nprobe,
                       float* out_vals_host, uint32_t* out_ids_host);

/* ------------------------------------------------------------------------------------------ */
/* Seeded synthetic data on the device (restates Tests/.../Utilities/TestRNG.swift:57-161;     */
/* stream = row0 + row).                                                                       */
/* ------------------------------------------------------------------------------------------ */
int va_gen_gaussian(va_context* ctx, float* out, int64_t rows, int dim, uint64_t seed, int64_t row0);
int va_gen_mixture(va_context* ctx, float* out, int64_t rows, int dim, uint64_t seed, int64_t row0,
                   int n_centroids, float sigma, int normalize);
/* fp32 -> bf16 (round to nearest even). */
int va_f32_to_bf16(va_context* ctx, const float* x, int64_t n, uint16_t* out);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif
#endif /* VA_CUDA_H */
