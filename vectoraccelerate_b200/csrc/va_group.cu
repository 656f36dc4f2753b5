// va_group.cu -- several GPUs behind one handle: a group of devices joined by an NCCL
// communicator, row-sharded databases, and the sharded search.
//
// The reference runs on one GPU (Core/Metal4Context.swift:175,183 creates the single device
// context that wraps every search, Index/AcceleratedVectorIndex.swift:1278-1374). The sharded
// search is this build's: every device holds a contiguous range of rows (N / ranks each, the
// last rank also the remainder; global id = first row of the shard + local row), searches it
// exactly (its local top k, certified like a one-device search), and the per-device lists travel
// as ONE all-gather of packed 8-byte (value bits, id) records per device, merged on the device by
// (value, id). Everything crosses NVLink inside NCCL into local buffers; no kernel reads a
// peer's memory.
//
// Two kinds of group:
//   va_context_create_multi   all listed devices in this process (one context and stream per
//                             device, one host thread per device during a search)
//   va_context_create_rank    one rank of a group spread over processes (one process per GPU);
//                             the ranks share an NCCL unique id made by va_nccl_unique_id
// NCCL is loaded at run time (libnccl.so.2, or VA_NCCL_LIBRARY): a process that already loaded it
// (PyTorch does) shares that copy, and the library still loads where NCCL is absent. The
// communicators are non-blocking: every NCCL step and every synchronisation polls
// ncclCommGetAsyncError against the context's timeout, and aborts the communicators when it
// expires (VA_ERR_TIMEOUT) or NCCL reports an error (VA_ERR_NCCL).
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "va_internal.cuh"

int db_create_impl(va_context* ctx, const void* rows, int on_device, int64_t n, int dim, int dtype,
                   uint32_t id_base, va_database** out, bool eager_operand);

namespace {

constexpr int kMaxLocal = 16;

// NCCL entry points, resolved from the shared library at run time.
struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*);
    ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*);
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*);
    ncclResult_t (*CommFinalize)(ncclComm_t);
    ncclResult_t (*CommDestroy)(ncclComm_t);
    ncclResult_t (*CommAbort)(ncclComm_t);
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*Broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*GroupStart)();
    ncclResult_t (*GroupEnd)();
    const char* (*GetErrorString)(ncclResult_t);
};

std::mutex g_nccl_mu;
NcclApi g_nccl;
int g_nccl_state = 0;  // 0 untried, 1 loaded, -1 unavailable
std::string g_nccl_why;

int nccl(const NcclApi** out) {
    std::lock_guard<std::mutex> lock(g_nccl_mu);
    if (g_nccl_state == 0) {
        const char* path = getenv("VA_NCCL_LIBRARY");
        void* h = dlopen(path && path[0] ? path : "libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        g_nccl_state = -1;
        if (!h) {
            const char* e = dlerror();
            g_nccl_why = e ? e : "dlopen failed";
        } else {
            bool ok = true;
            auto sym = [&](const char* name) {
                void* p = dlsym(h, name);
                if (!p) {
                    ok = false;
                    g_nccl_why = std::string("missing symbol ") + name;
                }
                return p;
            };
            g_nccl.GetUniqueId = (decltype(g_nccl.GetUniqueId))sym("ncclGetUniqueId");
            g_nccl.CommInitRankConfig = (decltype(g_nccl.CommInitRankConfig))sym("ncclCommInitRankConfig");
            g_nccl.CommGetAsyncError = (decltype(g_nccl.CommGetAsyncError))sym("ncclCommGetAsyncError");
            g_nccl.CommFinalize = (decltype(g_nccl.CommFinalize))sym("ncclCommFinalize");
            g_nccl.CommDestroy = (decltype(g_nccl.CommDestroy))sym("ncclCommDestroy");
            g_nccl.CommAbort = (decltype(g_nccl.CommAbort))sym("ncclCommAbort");
            g_nccl.AllGather = (decltype(g_nccl.AllGather))sym("ncclAllGather");
            g_nccl.AllReduce = (decltype(g_nccl.AllReduce))sym("ncclAllReduce");
            g_nccl.Broadcast = (decltype(g_nccl.Broadcast))sym("ncclBroadcast");
            g_nccl.GroupStart = (decltype(g_nccl.GroupStart))sym("ncclGroupStart");
            g_nccl.GroupEnd = (decltype(g_nccl.GroupEnd))sym("ncclGroupEnd");
            g_nccl.GetErrorString = (decltype(g_nccl.GetErrorString))sym("ncclGetErrorString");
            if (ok) g_nccl_state = 1;
        }
    }
    if (g_nccl_state != 1)
        return va_set_error(VA_ERR_NCCL, "NCCL is unavailable (%s); set VA_NCCL_LIBRARY to libnccl.so.2",
                            g_nccl_why.c_str());
    *out = &g_nccl;
    return VA_OK;
}

int64_t shard_rows(int64_t n, int nranks, int rank, int64_t* row0) {
    const int64_t per = n / nranks;
    *row0 = (int64_t)rank * per;
    return rank == nranks - 1 ? n - *row0 : per;
}

}  // namespace

struct va_group {
    int nranks = 1;                 // ranks (devices) of the whole group
    int nlocal = 1;                 // members in this process
    int rank0 = 0;                  // global rank of members[0]
    va_context* members[kMaxLocal] = {};  // members[0] is the front context (owns the group)
    ncclComm_t comms[kMaxLocal] = {};
    bool aborted = false;
    unsigned timeout_ms = 120000;
};

namespace {

void abort_group(va_group* g) {
    const NcclApi* api = nullptr;
    if (nccl(&api) != VA_OK) return;
    for (int m = 0; m < g->nlocal; ++m)
        if (g->comms[m]) {
            api->CommAbort(g->comms[m]);
            g->comms[m] = nullptr;
        }
    g->aborted = true;
}

// Poll every communicator of the group until no operation is in progress (bounded).
int wait_comms(va_group* g, const char* what) {
    const NcclApi* api = nullptr;
    VA_TRY(nccl(&api));
    const auto t0 = std::chrono::steady_clock::now();
    for (int m = 0; m < g->nlocal; ++m) {
        for (;;) {
            ncclResult_t st = ncclSuccess;
            ncclResult_t r = api->CommGetAsyncError(g->comms[m], &st);
            if (r != ncclSuccess) st = r;
            if (st == ncclSuccess) break;
            if (st != ncclInProgress) {
                const std::string msg = api->GetErrorString(st);
                abort_group(g);
                return va_set_error(VA_ERR_NCCL, "%s: NCCL error on member %d: %s (communicators aborted)", what, m,
                                    msg.c_str());
            }
            const auto ms =
                std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
            if ((unsigned)ms > g->timeout_ms) {
                abort_group(g);
                return va_set_error(VA_ERR_TIMEOUT, "%s: NCCL step not finished after %u ms (communicators aborted)",
                                    what, g->timeout_ms);
            }
            std::this_thread::sleep_for(std::chrono::microseconds(50));
        }
    }
    return VA_OK;
}

int check_nccl(va_group* g, ncclResult_t r, const char* what) {
    if (r == ncclSuccess || r == ncclInProgress) return wait_comms(g, what);
    const NcclApi* api = nullptr;
    VA_TRY(nccl(&api));
    const std::string msg = api->GetErrorString(r);
    abort_group(g);
    return va_set_error(VA_ERR_NCCL, "%s failed: %s (communicators aborted)", what, msg.c_str());
}

// ncclGroupStart only opens a group on this thread: a status check, no communicator to poll.
int group_start(const NcclApi* api) {
    const ncclResult_t r = api->GroupStart();
    if (r != ncclSuccess) return va_set_error(VA_ERR_NCCL, "ncclGroupStart failed: %s", api->GetErrorString(r));
    return VA_OK;
}

int usable(va_group* g) {
    if (!g) return va_set_error(VA_ERR_INVALID_ARG, "the context is not a multi-GPU group (va_context_create_multi "
                                                   "or va_context_create_rank)");
    if (g->aborted) return va_set_error(VA_ERR_NCCL, "the group's communicators were aborted after an earlier error");
    return VA_OK;
}

// Group-level scratch on one member context (grown in stream order).
int gbuf(va_context* c, size_t bytes, void** out) {
    if (c->gbuf_bytes < bytes) {
        if (c->gbuf) {
            VA_CUDA_TRY(cudaStreamSynchronize(c->stream));
            VA_CUDA_TRY(cudaFree(c->gbuf));
            c->gbuf = nullptr;
            c->gbuf_bytes = 0;
        }
        cudaError_t e = cudaMalloc(&c->gbuf, bytes);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return va_set_error(VA_ERR_OOM, "exchange scratch of %zu bytes failed: %s", bytes, cudaGetErrorString(e));
        }
        c->gbuf_bytes = bytes;
    }
    *out = c->gbuf;
    return VA_OK;
}

int64_t ru256(int64_t v) { return (v + 255) / 256 * 256; }

__global__ void k_pack(const float* __restrict__ v, const uint32_t* __restrict__ ids, int64_t n,
                       unsigned long long* __restrict__ rec) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        rec[i] = ((unsigned long long)__float_as_uint(v[i]) << 32) | ids[i];
}

__global__ void k_unpack(const unsigned long long* __restrict__ rec, int64_t n, float* __restrict__ v,
                         uint32_t* __restrict__ ids) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        v[i] = __uint_as_float((uint32_t)(rec[i] >> 32));
        ids[i] = (uint32_t)rec[i];
    }
}

__global__ void k_bits_to_u32(const float* __restrict__ v, const uint32_t* __restrict__ ids, int64_t n,
                              uint32_t* __restrict__ out) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = ids[i] == va::kInvalidId ? 0xFFFFFFFFu : __float_as_uint(v[i]);
}

int grid_of(int64_t n) { return (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 4096)); }

// Runs f(m) for every member, one host thread per member when there are several (each member's
// search waits for its own stream); the first failure's status and message are returned.
template <class F>
int for_members(va_group* g, F&& f) {
    if (g->nlocal == 1) return f(0);
    std::vector<int> st((size_t)g->nlocal, VA_OK);
    std::vector<std::string> msg((size_t)g->nlocal);
    std::vector<std::thread> th;
    for (int m = 0; m < g->nlocal; ++m)
        th.emplace_back([&, m] {
            cudaSetDevice(g->members[m]->device);
            st[(size_t)m] = f(m);
            if (st[(size_t)m] != VA_OK) msg[(size_t)m] = va_last_error();
        });
    for (auto& t : th) t.join();
    for (int m = 0; m < g->nlocal; ++m)
        if (st[(size_t)m] != VA_OK)
            return va_set_error(st[(size_t)m], "member %d (device %d): %s", m, g->members[m]->device,
                                msg[(size_t)m].c_str());
    return VA_OK;
}

// The shard database member m searches.
const va_database* shard_of(const va_database* db, int m) { return db->shards ? db->shards[m] : db; }

// Sharded search: queries (device, on the front's device) reach every member (NCCL broadcast in a
// multi-device context), each member searches its shard into its local top k (local(m, ctx,
// shard, queries, vals, ids)), one all-gather of packed records, the merge on the front.
template <class Local>
int sharded_run(va_context* ctx, const va_database* db, const void* queries, size_t qrow_bytes, int64_t nq, int k,
                int mode, Local&& local, float* out_vals, uint32_t* out_ids) {
    va_group* g = ctx->group;
    VA_TRY(usable(g));
    VA_REQUIRE(db->shards ? db->nshards == g->nlocal : g->nlocal == 1,
               "the database was sharded for a different group (%d shards, %d local devices)", db->nshards, g->nlocal);
    VA_REQUIRE(shard_of(db, 0)->ctx == ctx, "the database belongs to another context");
    VA_REQUIRE(nq > 0 && k > 0, "numQueries and k must be positive");
    const NcclApi* api = nullptr;
    VA_TRY(nccl(&api));
    const int R = g->nranks;
    const int64_t nk = nq * k;
    const size_t qb = (size_t)ru256((int64_t)nq * qrow_bytes), lb = (size_t)ru256(nk * 4),
                 rb = (size_t)ru256(nk * 8), gb = (size_t)ru256((int64_t)R * nk * 8),
                 mb = (size_t)ru256((int64_t)R * nk * 4);
    struct Bufs {
        uint8_t* q;
        float* lv;
        uint32_t* li;
        unsigned long long* rec;
        unsigned long long* all;
        float* gv;
        uint32_t* gi;
    } b[kMaxLocal];
    for (int m = 0; m < g->nlocal; ++m) {
        va_context* c = g->members[m];
        VA_CUDA_TRY(cudaSetDevice(c->device));
        void* p;
        VA_TRY(gbuf(c, qb + 2 * lb + rb + gb + 2 * mb, &p));
        uint8_t* u = (uint8_t*)p;
        b[m].q = u;
        b[m].lv = (float*)(u + qb);
        b[m].li = (uint32_t*)(u + qb + lb);
        b[m].rec = (unsigned long long*)(u + qb + 2 * lb);
        b[m].all = (unsigned long long*)(u + qb + 2 * lb + rb);
        b[m].gv = (float*)(u + qb + 2 * lb + rb + gb);
        b[m].gi = (uint32_t*)(u + qb + 2 * lb + rb + gb + mb);
    }
    // 1. queries to every member of this process
    if (g->nlocal > 1) {
        VA_TRY(group_start(api));
        for (int m = 0; m < g->nlocal; ++m) {
            cudaSetDevice(g->members[m]->device);
            api->Broadcast(queries, b[m].q, (size_t)nq * qrow_bytes, ncclUint8, 0, g->comms[m], g->members[m]->stream);
        }
        VA_TRY(check_nccl(g, api->GroupEnd(), "ncclBroadcast(queries)"));
    }
    // 2. local searches (one host thread per member), packed into records
    VA_TRY(for_members(g, [&](int m) -> int {
        va_context* c = g->members[m];
        const void* q = g->nlocal > 1 ? (const void*)b[m].q : queries;
        VA_TRY(local(m, c, shard_of(db, m), q, b[m].lv, b[m].li));
        k_pack<<<grid_of(nk), 256, 0, c->stream>>>(b[m].lv, b[m].li, nk, b[m].rec);
        return va_check_launch("k_pack");
    }));
    // 3. one all-gather of the packed (value, id) records
    if (g->nlocal > 1) VA_TRY(group_start(api));
    for (int m = 0; m < g->nlocal; ++m) {
        cudaSetDevice(g->members[m]->device);
        ncclResult_t r = api->AllGather(b[m].rec, b[m].all, (size_t)nk, ncclUint64, g->comms[m], g->members[m]->stream);
        if (g->nlocal == 1) VA_TRY(check_nccl(g, r, "ncclAllGather(records)"));
    }
    if (g->nlocal > 1) VA_TRY(check_nccl(g, api->GroupEnd(), "ncclAllGather(records)"));
    // 4. the merge on the front context, by (value, id)
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    k_unpack<<<grid_of((int64_t)R * nk), 256, 0, ctx->stream>>>(b[0].all, (int64_t)R * nk, b[0].gv, b[0].gi);
    VA_TRY(va_check_launch("k_unpack"));
    return va_merge_shards(ctx, b[0].gv, b[0].gi, R, nq, k, mode, out_vals, out_ids);
}

// Certificate counts of a multi-device search: the members' sums on the front context.
void sum_stats(va_group* g) {
    int64_t u = 0, e = 0;
    for (int m = 0; m < g->nlocal; ++m) {
        u += g->members[m]->stat_uncertified;
        e += g->members[m]->stat_exact;
    }
    g->members[0]->stat_uncertified = u;
    g->members[0]->stat_exact = e;
}

int init_comms(va_group* g, const ncclUniqueId& id) {
    const NcclApi* api = nullptr;
    VA_TRY(nccl(&api));
    if (g->nlocal > 1) VA_TRY(group_start(api));
    for (int m = 0; m < g->nlocal; ++m) {
        VA_CUDA_TRY(cudaSetDevice(g->members[m]->device));
        ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
        cfg.blocking = 0;
        ncclResult_t r = api->CommInitRankConfig(&g->comms[m], g->nranks, id, g->rank0 + m, &cfg);
        if (r != ncclSuccess && r != ncclInProgress) {
            if (g->nlocal > 1) api->GroupEnd();
            return va_set_error(VA_ERR_NCCL, "ncclCommInitRankConfig (rank %d of %d) failed: %s", g->rank0 + m,
                                g->nranks, api->GetErrorString(r));
        }
    }
    if (g->nlocal > 1) return check_nccl(g, api->GroupEnd(), "NCCL communicator initialisation");
    return wait_comms(g, "NCCL communicator initialisation");
}

// Sharded database over the context's group: member m gets the rows of its shard from `rows`
// (all n rows for a multi-device context; this rank's shard for a rank context), built by
// make(member ctx, shard rows, shard n, first global row, &shard db).
template <class Make>
int create_sharded(va_context* ctx, const void* rows, size_t row_bytes, int64_t n, Make&& make, va_database** out) {
    VA_REQUIRE(ctx && rows && out, "ctx, rows and out must not be NULL");
    va_group* g = ctx->group;
    VA_TRY(usable(g));
    VA_REQUIRE(n >= g->nranks, "numDataset %lld is smaller than the group's %d ranks", (long long)n, g->nranks);
    VA_REQUIRE((uint64_t)n <= 0xFFFFFFFFull, "numDataset %lld exceeds the uint32 id range", (long long)n);
    *out = nullptr;
    std::vector<va_database*> sh((size_t)g->nlocal, nullptr);
    int s = VA_OK;
    for (int m = 0; m < g->nlocal && s == VA_OK; ++m) {
        int64_t row0 = 0;
        const int64_t cnt = shard_rows(n, g->nranks, g->rank0 + m, &row0);
        const uint8_t* src = (const uint8_t*)rows + (g->nlocal > 1 ? (size_t)row0 * row_bytes : 0);
        s = make(g->members[m], (const void*)src, cnt, row0, &sh[(size_t)m]);
    }
    if (s != VA_OK) {
        for (auto* d : sh) va_db_destroy(d);
        return s;
    }
    if (g->nlocal == 1) {
        sh[0]->group_shard = true;
        sh[0]->n_total = n;
        *out = sh[0];
        return VA_OK;
    }
    va_database* db = new va_database();
    db->ctx = ctx;
    db->n = 0;
    db->n_total = n;
    db->dim = sh[0]->dim;
    db->dtype = sh[0]->dtype;
    db->kind = sh[0]->kind;
    db->words = sh[0]->words;
    db->shards = new va_database*[(size_t)g->nlocal];
    db->nshards = g->nlocal;
    for (int m = 0; m < g->nlocal; ++m) db->shards[m] = sh[(size_t)m];
    *out = db;
    return VA_OK;
}

}  // namespace

// ------------------------------------------------------------------------------------------------
// Internal entry points used by va_core.cu and the search files.
// ------------------------------------------------------------------------------------------------
int va_group_synchronize(va_context* ctx) {
    va_group* g = ctx->group;
    const NcclApi* api = nullptr;
    VA_TRY(nccl(&api));
    std::vector<cudaEvent_t> ev((size_t)g->nlocal, nullptr);
    for (int m = 0; m < g->nlocal; ++m) {
        va_context* c = g->members[m];
        VA_CUDA_TRY(cudaSetDevice(c->device));
        VA_CUDA_TRY(cudaEventRecord(c->ev_sync, c->stream));
    }
    const auto t0 = std::chrono::steady_clock::now();
    for (int m = 0; m < g->nlocal; ++m) {
        va_context* c = g->members[m];
        cudaSetDevice(c->device);
        for (;;) {
            cudaError_t e = cudaEventQuery(c->ev_sync);
            if (e == cudaSuccess) break;
            if (e != cudaErrorNotReady)
                return va_set_error(VA_ERR_CUDA, "device work failed on device %d: %s", c->device, cudaGetErrorString(e));
            for (int j = 0; !g->aborted && j < g->nlocal; ++j) {
                ncclResult_t st = ncclSuccess;
                if (api->CommGetAsyncError(g->comms[j], &st) == ncclSuccess && st != ncclSuccess && st != ncclInProgress) {
                    const std::string msg = api->GetErrorString(st);
                    abort_group(g);
                    return va_set_error(VA_ERR_NCCL, "NCCL error on member %d: %s (communicators aborted)", j,
                                        msg.c_str());
                }
            }
            const auto ms =
                std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
            if ((unsigned)ms > g->timeout_ms) {
                abort_group(g);
                return va_set_error(VA_ERR_TIMEOUT, "va_synchronize: group work not finished after %u ms "
                                                    "(communicators aborted)", g->timeout_ms);
            }
            std::this_thread::sleep_for(std::chrono::microseconds(20));
        }
    }
    for (int m = 0; m < g->nlocal; ++m) {
        va_context* c = g->members[m];
        cudaSetDevice(c->device);
        int derr = 0;
        VA_CUDA_TRY(cudaMemcpy(&derr, c->d_error, sizeof(int), cudaMemcpyDeviceToHost));
        if (derr) {
            VA_CUDA_TRY(cudaMemset(c->d_error, 0, sizeof(int)));
            return va_set_error(VA_ERR_TIMEOUT, "a bounded device-side wait expired on device %d (device error %d)",
                                c->device, derr);
        }
    }
    cudaSetDevice(ctx->device);
    return VA_OK;
}

void va_group_destroy(va_context* ctx) {
    va_group* g = ctx->group;
    if (!g) return;
    ctx->group = nullptr;  // members are plain contexts from here on
    const NcclApi* api = nullptr;
    if (nccl(&api) == VA_OK && !g->aborted) {
        // Bounded wait for the members' streams: a collective still waiting for a peer that has
        // gone is aborted rather than finalized (finalizing would wait for it).
        bool idle = true;
        for (int m = 0; m < g->nlocal; ++m)
            if (va_sync_one(g->members[m]) != VA_OK) idle = false;
        if (!idle) {
            abort_group(g);
        } else {
            for (int m = 0; m < g->nlocal; ++m) {
                if (!g->comms[m]) continue;
                cudaSetDevice(g->members[m]->device);
                api->CommFinalize(g->comms[m]);
            }
            if (wait_comms(g, "ncclCommFinalize") == VA_OK)
                for (int m = 0; m < g->nlocal; ++m)
                    if (g->comms[m]) api->CommDestroy(g->comms[m]);
        }
    }
    for (int m = 1; m < g->nlocal; ++m) va_context_destroy(g->members[m]);
    delete g;
}

int va_sharded_knn(va_context* ctx, const va_database* db, const float* queries, int64_t nq, int k, int metric,
                   int precision, int rerank, float* out_vals, uint32_t* out_ids) {
    VA_REQUIRE(queries, "queries must not be NULL");
    VA_REQUIRE(db->kind == VA_DB_FLOAT, "a sharded %s database is searched with its own entry point",
               db->kind == VA_DB_INT8 ? "int8" : "binary");
    VA_REQUIRE(metric >= 0 && metric <= 2, "metric must be 0 (L2SQ), 1 (COSINE) or 2 (IP), got %d", metric);
    const int mode = metric == VA_METRIC_IP ? VA_SELECT_MAX : VA_SELECT_MIN;
    const int s = sharded_run(
        ctx, db, queries, (size_t)db->dim * 4, nq, k, mode,
        [&](int, va_context* c, const va_database* sd, const void* q, float* lv, uint32_t* li) {
            return va_knn_search_local(c, sd, (const float*)q, nq, k, metric, precision, rerank, lv, li);
        },
        out_vals, out_ids);
    sum_stats(ctx->group);
    return s;
}

int va_sharded_int8(va_context* ctx, const va_database* db, const float* queries, int64_t nq, int k, int candidates,
                    float* out_vals, uint32_t* out_ids) {
    VA_REQUIRE(db->kind == VA_DB_INT8, "database is not an int8 database (use va_db_create_int8_sharded)");
    return sharded_run(
        ctx, db, queries, (size_t)db->dim * 4, nq, k, VA_SELECT_MIN,
        [&](int, va_context* c, const va_database* sd, const void* q, float* lv, uint32_t* li) {
            return va_int8_knn_local(c, sd, (const float*)q, nq, k, candidates, lv, li);
        },
        out_vals, out_ids);
}

int va_sharded_hamming(va_context* ctx, const va_database* db, const uint32_t* queries, int64_t nq, int k,
                       uint32_t* out_dists, uint32_t* out_ids) {
    VA_REQUIRE(db->kind == VA_DB_BINARY, "database is not a binary database (use va_db_create_binary_sharded)");
    // Distances travel as their uint32 bit patterns in the float records (non-negative integers
    // order like their bits) and come back as integers.
    void* tmp;
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    VA_TRY(va_aux_buffer(ctx, (size_t)ru256(nq * k * 4), &tmp));
    float* mv = (float*)tmp;
    VA_TRY(sharded_run(
        ctx, db, queries, (size_t)db->words * 4, nq, k, VA_SELECT_MIN,
        [&](int, va_context* c, const va_database* sd, const void* q, float* lv, uint32_t* li) {
            return va_hamming_knn_local(c, sd, (const uint32_t*)q, nq, k, (uint32_t*)lv, li);
        },
        mv, out_ids));
    if (out_dists) {
        k_bits_to_u32<<<grid_of(nq * k), 256, 0, ctx->stream>>>(mv, out_ids, nq * k, out_dists);
        VA_TRY(va_check_launch("k_bits_to_u32"));
    }
    return VA_OK;
}

// ------------------------------------------------------------------------------------------------
// Public ABI
// ------------------------------------------------------------------------------------------------
extern "C" {

int va_nccl_unique_id(void* id) {
    VA_REQUIRE(id, "id must not be NULL");
    const NcclApi* api = nullptr;
    VA_TRY(nccl(&api));
    ncclUniqueId u;
    ncclResult_t r = api->GetUniqueId(&u);
    if (r != ncclSuccess) return va_set_error(VA_ERR_NCCL, "ncclGetUniqueId failed: %s", api->GetErrorString(r));
    static_assert(sizeof(ncclUniqueId) == VA_NCCL_ID_BYTES, "NCCL unique id size");
    memcpy(id, &u, sizeof(u));
    return VA_OK;
}

int va_context_create_rank(const va_config* cfg, int nranks, int rank, const void* nccl_id, va_context** out) {
    VaRange nvtx_range("va_context_create_rank");
    VA_REQUIRE(out && nccl_id, "out and nccl_id must not be NULL");
    VA_REQUIRE(nranks >= 1 && rank >= 0 && rank < nranks, "rank %d outside a group of %d ranks", rank, nranks);
    *out = nullptr;
    const NcclApi* api = nullptr;
    VA_TRY(nccl(&api));
    va_context* c = nullptr;
    VA_TRY(va_context_create(cfg, &c));
    va_group* g = new va_group();
    g->nranks = nranks;
    g->nlocal = 1;
    g->rank0 = rank;
    g->members[0] = c;
    g->timeout_ms = c->timeout_ms;
    ncclUniqueId id;
    memcpy(&id, nccl_id, sizeof(id));
    const int s = init_comms(g, id);
    if (s != VA_OK) {
        abort_group(g);
        delete g;
        va_context_destroy(c);
        return s;
    }
    c->group = g;
    va_log_info("rank %d of %d on device %d: NCCL communicator ready", rank, nranks, c->device);
    *out = c;
    return VA_OK;
}

int va_context_create_multi(const int* devices, int ndev, const va_config* cfg, va_context** out) {
    VaRange nvtx_range("va_context_create_multi");
    VA_REQUIRE(out && devices, "out and devices must not be NULL");
    VA_REQUIRE(ndev >= 1 && ndev <= kMaxLocal, "ndev must be in 1..%d, got %d", kMaxLocal, ndev);
    for (int i = 0; i < ndev; ++i)
        for (int j = i + 1; j < ndev; ++j)
            VA_REQUIRE(devices[i] != devices[j], "device %d is listed twice", devices[i]);
    *out = nullptr;
    const NcclApi* api = nullptr;
    VA_TRY(nccl(&api));
    va_group* g = new va_group();
    g->nranks = ndev;
    g->nlocal = ndev;
    g->rank0 = 0;
    int s = VA_OK;
    for (int m = 0; m < ndev && s == VA_OK; ++m) {
        va_config c = {};
        c.device = devices[m];
        c.timeout_ms = cfg ? cfg->timeout_ms : 0;
        c.stream = (m == 0 && cfg) ? cfg->stream : nullptr;  // a caller's stream belongs to the first device
        s = va_context_create(&c, &g->members[m]);
    }
    if (s == VA_OK) {
        g->timeout_ms = g->members[0]->timeout_ms;
        ncclUniqueId id;
        ncclResult_t r = api->GetUniqueId(&id);
        s = r == ncclSuccess ? init_comms(g, id)
                             : va_set_error(VA_ERR_NCCL, "ncclGetUniqueId failed: %s", api->GetErrorString(r));
    }
    if (s != VA_OK) {
        abort_group(g);
        for (int m = 0; m < ndev; ++m) va_context_destroy(g->members[m]);
        delete g;
        return s;
    }
    g->members[0]->group = g;
    *out = g->members[0];
    return VA_OK;
}

int va_context_group(const va_context* ctx, int* nranks, int* rank, int* local_devices) {
    VA_REQUIRE(ctx, "ctx must not be NULL");
    const va_group* g = ctx->group;
    if (nranks) *nranks = g ? g->nranks : 1;
    if (rank) *rank = g ? g->rank0 : 0;
    if (local_devices) *local_devices = g ? g->nlocal : 1;
    return VA_OK;
}

int va_shard_range(const va_context* ctx, int64_t n, int member, int64_t* row0, int64_t* rows) {
    VA_REQUIRE(ctx && row0 && rows, "ctx, row0 and rows must not be NULL");
    const va_group* g = ctx->group;
    const int nr = g ? g->nranks : 1, nl = g ? g->nlocal : 1, r0 = g ? g->rank0 : 0;
    VA_REQUIRE(member >= 0 && member < nl, "member %d outside the context's %d local devices", member, nl);
    VA_REQUIRE(n >= nr, "numDataset %lld is smaller than the group's %d ranks", (long long)n, nr);
    *rows = shard_rows(n, nr, r0 + member, row0);
    return VA_OK;
}

int va_db_shard(const va_database* db, int member, va_database** shard) {
    VA_REQUIRE(db && shard, "db and shard must not be NULL");
    if (!db->shards) {
        VA_REQUIRE(member == 0, "member %d of an unsharded (or rank) database", member);
        *shard = const_cast<va_database*>(db);
        return VA_OK;
    }
    VA_REQUIRE(member >= 0 && member < db->nshards, "member %d outside %d shards", member, db->nshards);
    *shard = db->shards[member];
    return VA_OK;
}

int va_db_create_sharded(va_context* ctx, const void* rows, int on_device, int64_t n, int dim, int dtype,
                         va_database** out) {
    VaRange nvtx_range("va_db_create_sharded");
    VA_REQUIRE(dtype == VA_DTYPE_F32 || dtype == VA_DTYPE_BF16, "dtype must be VA_DTYPE_F32 or VA_DTYPE_BF16");
    VA_REQUIRE(dim > 0 && dim <= VA_MAX_DIM, "dimension %d outside 1..%d", dim, VA_MAX_DIM);
    const size_t rb = (size_t)dim * (dtype == VA_DTYPE_BF16 ? 2 : 4);
    return create_sharded(
        ctx, rows, rb, n,
        [&](va_context* c, const void* src, int64_t cnt, int64_t row0, va_database** sd) {
            return db_create_impl(c, src, on_device, cnt, dim, dtype, (uint32_t)row0, sd, true);
        },
        out);
}

int va_db_create_binary_sharded(va_context* ctx, const uint32_t* codes, int on_device, int64_t n, int dim_bits,
                                va_database** out) {
    VaRange nvtx_range("va_db_create_binary_sharded");
    VA_REQUIRE(dim_bits > 0 && dim_bits <= 8192, "dimension must be in 1..8192 bits, got %d", dim_bits);
    const size_t rb = (size_t)((dim_bits + 31) / 32) * 4;
    return create_sharded(
        ctx, codes, rb, n,
        [&](va_context* c, const void* src, int64_t cnt, int64_t row0, va_database** sd) {
            return va_db_create_binary(c, (const uint32_t*)src, on_device, cnt, dim_bits, (uint32_t)row0, sd);
        },
        out);
}

int va_db_create_int8_sharded(va_context* ctx, const float* rows, int on_device, int64_t n, int dim,
                              va_database** out) {
    VaRange nvtx_range("va_db_create_int8_sharded");
    VA_REQUIRE(ctx && rows && out, "ctx, rows and out must not be NULL");
    va_group* g = ctx->group;
    VA_TRY(usable(g));
    VA_REQUIRE(dim > 0 && dim <= VA_MAX_DIM, "dimension %d outside 1..%d", dim, VA_MAX_DIM);
    VA_REQUIRE(n >= g->nranks, "numDataset %lld is smaller than the group's %d ranks", (long long)n, g->nranks);
    const NcclApi* api = nullptr;
    VA_TRY(nccl(&api));
    // Every member's rows on its device (a staged copy unless they already live there), the
    // per-dimension min / max of each shard, then MIN / MAX over the group: every shard is coded
    // with the range of the WHOLE database.
    float* stage[kMaxLocal] = {};
    float* mm[kMaxLocal] = {};
    int s = VA_OK;
    auto cleanup = [&] {
        // bounded: an exchange still waiting for a peer that has gone is aborted before the frees
        for (int m = 0; m < g->nlocal; ++m)
            if (!g->aborted && va_sync_one(g->members[m]) != VA_OK) abort_group(g);
        for (int m = 0; m < g->nlocal; ++m) {
            cudaSetDevice(g->members[m]->device);
            if (stage[m]) cudaFree(stage[m]);
            if (mm[m]) cudaFree(mm[m]);
        }
        cudaSetDevice(ctx->device);
    };
    for (int m = 0; m < g->nlocal && s == VA_OK; ++m) {
        va_context* c = g->members[m];
        int64_t row0 = 0;
        const int64_t cnt = shard_rows(n, g->nranks, g->rank0 + m, &row0);
        const float* src = rows + (g->nlocal > 1 ? row0 * dim : 0);
        cudaSetDevice(c->device);
        cudaPointerAttributes at = {};
        const bool local = on_device && cudaPointerGetAttributes(&at, src) == cudaSuccess &&
                           at.type == cudaMemoryTypeDevice && at.device == c->device;
        const float* dev = src;
        if (!local) {
            if (cudaMalloc((void**)&stage[m], (size_t)cnt * dim * 4) != cudaSuccess) {
                cudaGetLastError();
                s = va_set_error(VA_ERR_OOM, "staging %lld rows on device %d failed", (long long)cnt, c->device);
                break;
            }
            cudaMemcpyAsync(stage[m], src, (size_t)cnt * dim * 4, on_device ? cudaMemcpyDeviceToDevice
                                                                                : cudaMemcpyHostToDevice,
                            c->stream);
            dev = stage[m];
        }
        if (cudaMalloc((void**)&mm[m], (size_t)dim * 8) != cudaSuccess) {
            cudaGetLastError();
            s = va_set_error(VA_ERR_OOM, "range buffers failed");
            break;
        }
        s = va_sq_perdim_minmax(c, dev, cnt, dim, mm[m], mm[m] + dim);
    }
    if (s == VA_OK && g->nranks > 1) {
        // Both reductions in one group, also with one local member: a non-blocking communicator
        // takes no second call while the first is still being enqueued.
        s = group_start(api);
        for (int m = 0; m < g->nlocal && s == VA_OK; ++m) {
            cudaSetDevice(g->members[m]->device);
            api->AllReduce(mm[m], mm[m], (size_t)dim, ncclFloat32, ncclMin, g->comms[m], g->members[m]->stream);
            api->AllReduce(mm[m] + dim, mm[m] + dim, (size_t)dim, ncclFloat32, ncclMax, g->comms[m],
                           g->members[m]->stream);
        }
        if (s == VA_OK) s = check_nccl(g, api->GroupEnd(), "ncclAllReduce(range)");
    }
    std::vector<va_database*> sh((size_t)g->nlocal, nullptr);
    for (int m = 0; m < g->nlocal && s == VA_OK; ++m) {
        va_context* c = g->members[m];
        int64_t row0 = 0;
        const int64_t cnt = shard_rows(n, g->nranks, g->rank0 + m, &row0);
        const float* dev = stage[m] ? stage[m] : rows + (g->nlocal > 1 ? row0 * dim : 0);
        s = va_db_create_int8(c, dev, 1, cnt, dim, mm[m], mm[m] + dim, (uint32_t)row0, &sh[(size_t)m]);
    }
    cleanup();
    if (s != VA_OK) {
        for (auto* d : sh) va_db_destroy(d);
        return s;
    }
    if (g->nlocal == 1) {
        sh[0]->group_shard = true;
        sh[0]->n_total = n;
        *out = sh[0];
        return VA_OK;
    }
    va_database* db = new va_database();
    db->ctx = ctx;
    db->n_total = n;
    db->dim = dim;
    db->kind = VA_DB_INT8;
    db->shards = new va_database*[(size_t)g->nlocal];
    db->nshards = g->nlocal;
    for (int m = 0; m < g->nlocal; ++m) db->shards[m] = sh[(size_t)m];
    *out = db;
    return VA_OK;
}

}  // extern "C"
