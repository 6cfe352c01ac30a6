// mars_shard.cu -- row-sharded batched top-K across GPUs (one process per
// GPU), with the exchange steps done by NCCL inside the library.
//
// The reference runs on one GPU; its only multi-GPU plan is a note
// (NEXT_STEPS.md:31).  Here a corpus larger than one GPU, or a batch that
// should finish faster, is split by rows: rank r holds rows
// [offset_r, offset_r + n_r) in its own store and every rank answers the same
// B queries.  One call of mars_shard_query_batch_topk on every rank:
//
//  1. the local batched pipeline (mars_batch.cu): fp16 tensor-core short
//     list with proven margins, then rescore pass 1, which writes each
//     query's certified K-th lower bound on this shard (K rows of the shard
//     score at least that much);
//  2. NCCL all-reduce (max) of the B bounds: the largest is a lower bound of
//     the global K-th score, valid on every shard;
//  3. rescore pass 2 against that bound: only rows that can still enter the
//     global top-K are scored exactly (about K / world + a few per shard);
//     uncertified queries are rescanned exactly on the device;
//  4. the local lists become 64-bit rank keys (score, then id, in one
//     integer; 0 = no entry) and ONE ncclAllGather moves them, B x K x 8
//     bytes per rank;
//  5. every rank selects each query's top-K of the world x K keys.
//
// The results equal a single-GPU mars_query_batch_topk over the whole
// corpus bit for bit: every shard's exact scores are the fp32 scan's, the
// pruning only drops rows that cannot place, and keys rank by (score desc,
// id asc).  Every rank takes the same collective steps in the same order in
// every path: a rank whose local work fails still joins both collectives
// with neutral data (bounds -inf, no keys) and returns its error after them.
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <algorithm>
#include <cmath>
#include <cstddef>
#include <cstring>
#include <mutex>
#include <type_traits>
#include <string>

#include "mars_b200.h"
#include "mars_common.cuh"
#include "mars_internal.h"
#include "mars_kernels.cuh"
#include "mars_nccl.h"
#include "mars_scan_body.cuh"
#include "mars_select.cuh"
#include "mars_shard_internal.h"

namespace mars {

// ---- NCCL at run time ------------------------------------------------------
const NcclApi* nccl_api(const char** why) {
    static NcclApi api{};
    static const char* reason = nullptr;
    static bool ok = false;
    static std::once_flag once;
    std::call_once(once, [] {
        // a copy already in the process (same soname) first, else the search path
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (h == nullptr) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (h == nullptr) { reason = "libnccl.so.2 could not be loaded"; return; }
        bool all = true;
        auto get = [&](auto& fn, const char* name) {
            fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
            all = all && fn != nullptr;
        };
        get(api.GetUniqueId, "ncclGetUniqueId");
        get(api.CommInitRank, "ncclCommInitRank");
        get(api.CommDestroy, "ncclCommDestroy");
        get(api.CommAbort, "ncclCommAbort");
        get(api.CommGetAsyncError, "ncclCommGetAsyncError");
        get(api.AllReduce, "ncclAllReduce");
        get(api.AllGather, "ncclAllGather");
        get(api.GetErrorString, "ncclGetErrorString");
        get(api.GetVersion, "ncclGetVersion");
        if (!all) { reason = "libnccl.so.2 lacks an entry point this library needs"; return; }
        ok = true;
    });
    if (why != nullptr) *why = reason;
    return ok ? &api : nullptr;
}

namespace shard {

constexpr int kThreads = 256;

// [n] (id, score) -> rank keys; id < 0 (no entry) -> 0, below every key.
__global__ void pack_keys_kernel(const int32_t* __restrict__ ids, const float* __restrict__ vals, int64_t n,
                                 unsigned long long* __restrict__ keys) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int32_t id = ids[i];
        keys[i] = id >= 0 ? rank_key(vals[i], id) : 0ull;
    }
}

// Query qi's top-K of the world x K gathered keys ([rank][B][K] layout): the
// non-empty keys go to shared memory and the block's radix selection takes
// the K largest.  world x K <= kMergeKeys.  failed (> 0 when some shard's
// call failed): no result is served, counts are -1.
__global__ void __launch_bounds__(kThreads) merge_keys_kernel(const unsigned long long* __restrict__ keys, int world,
                                                              int K, int B, const float* __restrict__ failed,
                                                              int32_t* __restrict__ ids_out,
                                                              float* __restrict__ vals_out,
                                                              int32_t* __restrict__ cnt_out) {
    __shared__ unsigned long long s_keys[kMergeKeys];
    __shared__ int s_hist[2048];
    __shared__ int s_misc[16];
    const int qi = blockIdx.x;
    if (__ldcg(failed) > 0.0f) {
        for (int p = threadIdx.x; p < K; p += kThreads) {
            vals_out[(int64_t)qi * K + p] = -INFINITY;
            ids_out[(int64_t)qi * K + p] = -1;
        }
        if (threadIdx.x == 0 && cnt_out != nullptr) cnt_out[qi] = -1;
        return;
    }
    const int total = world * K;
    if (threadIdx.x == 0) s_misc[15] = 0;
    __syncthreads();
    for (int j0 = 0; j0 < total; j0 += kThreads) {
        const int j = j0 + threadIdx.x;
        unsigned long long k = 0ull;
        if (j < total) {
            const int r = j / K, e = j - r * K;
            k = __ldg(keys + ((int64_t)r * B + qi) * K + e);
        }
        warp_append(k != 0ull, k, s_keys, &s_misc[15], kMergeKeys);
    }
    __syncthreads();
    const int M = s_misc[15];
    __syncthreads();
    const int cnt = block_select_topk<kThreads>(s_keys, M, K, s_hist, s_misc);
    for (int p = threadIdx.x; p < K; p += kThreads) {
        const bool valid = p < cnt;
        vals_out[(int64_t)qi * K + p] = valid ? key_score(s_keys[p]) : -INFINITY;
        ids_out[(int64_t)qi * K + p] = valid ? key_id(s_keys[p]) : -1;
    }
    if (threadIdx.x == 0 && cnt_out != nullptr) cnt_out[qi] = cnt;
}

// Merge for the sharded query's seeds: as merge_keys_kernel, but a rank
// that failed sends all-ones keys (kFailedKey, never a rank key of a
// finite score); any such key marks the merge failed (count -1).
constexpr unsigned long long kFailedKey = ~0ull;
__global__ void __launch_bounds__(kThreads) merge_keys_flagged_kernel(const unsigned long long* __restrict__ keys,
                                                                      int world, int K, int B,
                                                                      int32_t* __restrict__ ids_out,
                                                                      float* __restrict__ vals_out,
                                                                      int32_t* __restrict__ cnt_out) {
    __shared__ unsigned long long s_keys[kMergeKeys];
    __shared__ int s_hist[2048];
    __shared__ int s_misc[16];
    __shared__ int s_failed;
    const int qi = blockIdx.x;
    const int total = world * K;
    if (threadIdx.x == 0) { s_misc[15] = 0; s_failed = 0; }
    __syncthreads();
    for (int j0 = 0; j0 < total; j0 += kThreads) {
        const int j = j0 + threadIdx.x;
        unsigned long long k = 0ull;
        if (j < total) {
            const int r = j / K, e = j - r * K;
            k = __ldg(keys + ((int64_t)r * B + qi) * K + e);
            if (k == kFailedKey) { s_failed = 1; k = 0ull; }
        }
        warp_append(k != 0ull, k, s_keys, &s_misc[15], kMergeKeys);
    }
    __syncthreads();
    const int M = s_misc[15];
    const bool failed = s_failed != 0;
    __syncthreads();
    const int cnt = failed ? 0 : block_select_topk<kThreads>(s_keys, M, K, s_hist, s_misc);
    for (int p = threadIdx.x; p < K; p += kThreads) {
        const bool valid = p < cnt;
        vals_out[(int64_t)qi * K + p] = valid ? key_score(s_keys[p]) : -INFINITY;
        ids_out[(int64_t)qi * K + p] = valid ? key_id(s_keys[p]) : -1;
    }
    if (threadIdx.x == 0 && cnt_out != nullptr) cnt_out[qi] = failed ? -1 : cnt;
}

// A shard whose call ended before its exchange: bounds -inf, flag = failed.
__global__ void neutral_bounds_kernel(float* p, int n, float failed) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) p[i] = -INFINITY;
    if (i == n) p[n] = failed;
}

}  // namespace shard
}  // namespace mars

using namespace mars;

struct mars_shard_comm {
    int32_t device = 0;
    int32_t rank = 0;
    int32_t world = 1;
    int32_t max_batch = 0;
    int32_t max_k = 0;
    const NcclApi* nccl = nullptr;
    ncclComm_t comm = nullptr;
    unsigned long long* d_send = nullptr;   // max_batch x max_k keys
    unsigned long long* d_recv = nullptr;   // world x max_batch x max_k keys
    float* d_bound = nullptr;               // max_batch + 1: bounds and flag when the batched call failed early
    const float* last_bound = nullptr;      // the exchanged array of the current call
    cudaEvent_t ev[4] = {nullptr, nullptr, nullptr, nullptr};   // local / exchange / merge boundaries
    bool timed = false;
    void* bfs_state = nullptr;              // mars_shard_query's scratch (made on first use)
};

namespace {

int nccl_fail(const NcclApi* api, ncclResult_t r, const char* what) {
    return fail(MARS_ERR_CUDA, std::string(what) + ": NCCL error " + std::to_string((int)r) + " (" +
                                   (api ? api->GetErrorString(r) : "?") + ")");
}

// max over the shards of the B certified bounds and the failure flag, in
// place, on st
int exchange_bounds(void* arg, float* d_bound, int32_t B, cudaStream_t st) {
    auto* c = static_cast<mars_shard_comm*>(arg);
    c->last_bound = d_bound;
    const ncclResult_t r = c->nccl->AllReduce(d_bound, d_bound, (size_t)B + 1, ncclFloat32, ncclMax, c->comm, st);
    if (r != ncclSuccess) return nccl_fail(c->nccl, r, "mars_shard_query_batch_topk: bound all-reduce");
    return MARS_OK;
}

}  // namespace

int mars::shard_comm_view(mars_shard_comm* c, ShardCommView* v) {
    if (c == nullptr || c->comm == nullptr) return fail(MARS_ERR_INVALID, "NULL or aborted shard communicator");
    v->device = c->device;
    v->rank = c->rank;
    v->world = c->world;
    v->max_k = c->max_k;
    v->bfs_state = &c->bfs_state;
    return MARS_OK;
}

static mars_shard_comm* comm_of(const ShardCommView& v) {
    return reinterpret_cast<mars_shard_comm*>(reinterpret_cast<char*>(v.bfs_state) -
                                              offsetof(mars_shard_comm, bfs_state));
}

int mars::shard_gather_merge(const ShardCommView& v, const int32_t* d_ids, const float* d_vals, int32_t B, int32_t K,
                             int32_t* d_ids_out, float* d_vals_out, int32_t* d_counts, bool neutral,
                             cudaStream_t st) {
    mars_shard_comm* c = comm_of(v);
    if (B > c->max_batch || K > c->max_k) return fail(MARS_ERR_INVALID, "shard merge: B or K beyond the communicator");
    const int64_t n = (int64_t)B * K;
    if (!neutral && d_ids != nullptr) {
        shard::pack_keys_kernel<<<(int)std::min<int64_t>((n + 255) / 256, 1024), 256, 0, st>>>(d_ids, d_vals, n,
                                                                                             c->d_send);
        MARS_CUDA_TRY(cudaGetLastError());
    } else {
        MARS_CUDA_TRY(cudaMemsetAsync(c->d_send, 0xff, (size_t)n * 8, st));   // kFailedKey
    }
    const ncclResult_t r = c->nccl->AllGather(c->d_send, c->d_recv, (size_t)n, ncclUint64, c->comm, st);
    if (r != ncclSuccess) return nccl_fail(c->nccl, r, "shard merge: all-gather");
    shard::merge_keys_flagged_kernel<<<B, shard::kThreads, 0, st>>>(c->d_recv, c->world, K, B, d_ids_out, d_vals_out,
                                                                    d_counts);
    MARS_CUDA_TRY(cudaGetLastError());
    return MARS_OK;
}

int mars::shard_allreduce_max_f32(const ShardCommView& v, float* d, int32_t n, cudaStream_t st) {
    mars_shard_comm* c = comm_of(v);
    const ncclResult_t r = c->nccl->AllReduce(d, d, (size_t)n, ncclFloat32, ncclMax, c->comm, st);
    if (r != ncclSuccess) return nccl_fail(c->nccl, r, "shard all-reduce");
    return MARS_OK;
}

int mars::shard_allreduce_max_i32(const ShardCommView& v, int32_t* d, int32_t n, cudaStream_t st) {
    mars_shard_comm* c = comm_of(v);
    const ncclResult_t r = c->nccl->AllReduce(d, d, (size_t)n, ncclInt32, ncclMax, c->comm, st);
    if (r != ncclSuccess) return nccl_fail(c->nccl, r, "shard all-reduce");
    return MARS_OK;
}

extern "C" {

int mars_shard_unique_id(void* id_out) {
    if (id_out == nullptr) return fail(MARS_ERR_INVALID, "mars_shard_unique_id: NULL output");
    const char* why = nullptr;
    const NcclApi* api = nccl_api(&why);
    if (api == nullptr) return fail(MARS_ERR_UNSUPPORTED, std::string("mars_shard_unique_id: ") + why);
    ncclUniqueId id;
    const ncclResult_t r = api->GetUniqueId(&id);
    if (r != ncclSuccess) return nccl_fail(api, r, "mars_shard_unique_id");
    std::memcpy(id_out, &id, sizeof(id));
    return MARS_OK;
}

int mars_shard_comm_create(int32_t device, int32_t rank, int32_t world, const void* unique_id, int32_t max_batch,
                           int32_t max_k, mars_shard_comm** out) {
    if (out == nullptr || unique_id == nullptr) return fail(MARS_ERR_INVALID, "mars_shard_comm_create: NULL argument");
    *out = nullptr;
    if (world <= 0 || rank < 0 || rank >= world || max_batch <= 0 || max_k <= 0 || max_k > MARS_MAX_TOP_K ||
        (int64_t)world * max_k > kMergeKeys)
        return fail(MARS_ERR_INVALID, "mars_shard_comm_create: need 0 <= rank < world, max_k <= " +
                                          std::to_string(MARS_MAX_TOP_K) + " and world x max_k <= " +
                                          std::to_string(kMergeKeys));
    const char* why = nullptr;
    const NcclApi* api = nccl_api(&why);
    if (api == nullptr) return fail(MARS_ERR_UNSUPPORTED, std::string("mars_shard_comm_create: ") + why);
    MarsDeviceGuard g(device);
    if (!g.ok) return fail(MARS_ERR_NO_DEVICE, "mars_shard_comm_create: cudaSetDevice failed");
    auto* c = new mars_shard_comm();
    c->device = device;
    c->rank = rank;
    c->world = world;
    c->max_batch = max_batch;
    c->max_k = max_k;
    c->nccl = api;
    int rc = MARS_OK;
    auto T = [&](cudaError_t e, const char* w) {
        if (rc == MARS_OK && e != cudaSuccess) rc = cuda_fail(e, w, __FILE__, __LINE__);
    };
    const size_t keys = (size_t)max_batch * max_k;
    T(cudaMalloc(&c->d_send, keys * 8), "shard send keys");
    T(cudaMalloc(&c->d_recv, keys * 8 * world), "shard gathered keys");
    T(cudaMalloc(&c->d_bound, ((size_t)max_batch + 1) * 4), "shard bounds + failure flag");
    for (auto& e : c->ev) T(cudaEventCreate(&e), "event");
    if (rc == MARS_OK) {
        ncclUniqueId id;
        std::memcpy(&id, unique_id, sizeof(id));
        const ncclResult_t r = api->CommInitRank(&c->comm, world, id, rank);
        if (r != ncclSuccess) { c->comm = nullptr; rc = nccl_fail(api, r, "mars_shard_comm_create: ncclCommInitRank"); }
    }
    if (rc != MARS_OK) { mars_shard_comm_destroy(c); return rc; }
    *out = c;
    return MARS_OK;
}

int mars_shard_comm_destroy(mars_shard_comm* c) {
    if (c == nullptr) return MARS_OK;
    MarsDeviceGuard g(c->device);
    cudaDeviceSynchronize();
    if (c->bfs_state != nullptr) shard_bfs_state_free(c->bfs_state);
    if (c->comm != nullptr) c->nccl->CommDestroy(c->comm);
    cudaFree(c->d_send);
    cudaFree(c->d_recv);
    cudaFree(c->d_bound);
    for (cudaEvent_t e : c->ev)
        if (e) cudaEventDestroy(e);
    delete c;
    return MARS_OK;
}

int mars_shard_comm_status(mars_shard_comm* c) {
    if (c == nullptr || c->comm == nullptr) return fail(MARS_ERR_INVALID, "mars_shard_comm_status: NULL communicator");
    ncclResult_t async = ncclSuccess;
    const ncclResult_t r = c->nccl->CommGetAsyncError(c->comm, &async);
    if (r != ncclSuccess) return nccl_fail(c->nccl, r, "mars_shard_comm_status");
    if (async != ncclSuccess) return nccl_fail(c->nccl, async, "mars_shard_comm_status: asynchronous error");
    return MARS_OK;
}

int mars_shard_comm_abort(mars_shard_comm* c) {
    if (c == nullptr) return MARS_OK;
    if (c->comm != nullptr) {
        c->nccl->CommAbort(c->comm);
        c->comm = nullptr;
    }
    return MARS_OK;
}

int mars_shard_comm_set_timing(mars_shard_comm* c, int32_t enable) {
    if (c == nullptr) return fail(MARS_ERR_INVALID, "mars_shard_comm_set_timing: NULL communicator");
    c->timed = enable != 0;
    return MARS_OK;
}

int mars_shard_last_times(mars_shard_comm* c, float* local_ms, float* gather_ms, float* merge_ms) {
    if (c == nullptr) return fail(MARS_ERR_INVALID, "mars_shard_last_times: NULL communicator");
    if (!c->timed) return fail(MARS_ERR_INVALID, "mars_shard_last_times: timing is off (mars_shard_comm_set_timing)");
    MarsDeviceGuard g(c->device);
    MARS_CUDA_TRY(cudaEventSynchronize(c->ev[3]));
    float a = 0.f, b = 0.f, m = 0.f;
    MARS_CUDA_TRY(cudaEventElapsedTime(&a, c->ev[0], c->ev[1]));
    MARS_CUDA_TRY(cudaEventElapsedTime(&b, c->ev[1], c->ev[2]));
    MARS_CUDA_TRY(cudaEventElapsedTime(&m, c->ev[2], c->ev[3]));
    if (local_ms) *local_ms = a;
    if (gather_ms) *gather_ms = b;
    if (merge_ms) *merge_ms = m;
    return MARS_OK;
}

int mars_shard_query_batch_topk(const mars_store* s, mars_batch_ctx* ctx, mars_shard_comm* c,
                                const float* d_queries, int32_t query_pitch, int32_t B, float query_timestamp,
                                float lambda, int32_t modality_filter, int32_t use_importance, int32_t K,
                                int32_t row_offset, int32_t* d_ids, float* d_vals, int32_t* d_counts,
                                void* stream) {
    // B and K are the same on every rank (the call is collective): checks on
    // them reject on every rank alike, before any collective
    if (c == nullptr || c->comm == nullptr)
        return fail(MARS_ERR_INVALID, "mars_shard_query_batch_topk: NULL or aborted communicator");
    if (B < 0 || B > c->max_batch || K <= 0 || K > c->max_k)
        return fail(MARS_ERR_INVALID, "mars_shard_query_batch_topk: B or K beyond the communicator's limits");
    if (B == 0) return MARS_OK;
    if (d_ids == nullptr || d_vals == nullptr)
        return fail(MARS_ERR_INVALID, "mars_shard_query_batch_topk: NULL output");
    MarsDeviceGuard g(c->device);
    if (!g.ok) return fail(MARS_ERR_NO_DEVICE, "mars_shard_query_batch_topk: cudaSetDevice failed");
    // NULL: the batch context's own stream, as mars_query_batch_topk
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream)
                             : (ctx != nullptr ? batch_ctx_stream(ctx) : static_cast<cudaStream_t>(nullptr));
    if (c->timed) MARS_CUDA_TRY(cudaEventRecord(c->ev[0], st));
    c->last_bound = nullptr;

    // 1-3: the local pipeline with the bound exchange between the rescore passes
    BoundExchange xchg{&exchange_bounds, c, false};
    int local_rc = MARS_OK;
    if (s == nullptr || ctx == nullptr || s->device != c->device)
        local_rc = fail(MARS_ERR_INVALID, "mars_shard_query_batch_topk: store and context must be on the "
                                          "communicator's device");
    else
        local_rc = batch_topk_sharded(s, ctx, d_queries, query_pitch, B, query_timestamp, lambda, modality_filter,
                                      use_importance, K, row_offset, d_ids, d_vals, d_counts, st, &xchg);
    const std::string local_msg = local_rc != MARS_OK ? std::string(mars_last_error()) : std::string();
    if (!xchg.done) {
        // the local call ended before its exchange (an error, or the exact
        // per-query scans of a small shard): join it with no bound
        shard::neutral_bounds_kernel<<<(B + 256) / 256, 256, 0, st>>>(c->d_bound, B,
                                                                      local_rc != MARS_OK ? 1.0f : 0.0f);
        MARS_CUDA_TRY(cudaGetLastError());
        MARS_TRY(exchange_bounds(c, c->d_bound, B, st));
    }
    if (c->timed) MARS_CUDA_TRY(cudaEventRecord(c->ev[1], st));

    // 4: one all-gather of the packed local lists
    const int64_t n = (int64_t)B * K;
    if (local_rc == MARS_OK) {
        shard::pack_keys_kernel<<<(int)std::min<int64_t>((n + 255) / 256, 1024), 256, 0, st>>>(d_ids, d_vals, n,
                                                                                             c->d_send);
        MARS_CUDA_TRY(cudaGetLastError());
    } else {
        MARS_CUDA_TRY(cudaMemsetAsync(c->d_send, 0, (size_t)n * 8, st));
    }
    const ncclResult_t r = c->nccl->AllGather(c->d_send, c->d_recv, (size_t)n, ncclUint64, c->comm, st);
    if (r != ncclSuccess) return nccl_fail(c->nccl, r, "mars_shard_query_batch_topk: all-gather");
    if (c->timed) MARS_CUDA_TRY(cudaEventRecord(c->ev[2], st));

    // 5: every rank merges
    shard::merge_keys_kernel<<<B, shard::kThreads, 0, st>>>(c->d_recv, c->world, K, B, c->last_bound + B, d_ids,
                                                            d_vals, d_counts);
    MARS_CUDA_TRY(cudaGetLastError());
    if (c->timed) MARS_CUDA_TRY(cudaEventRecord(c->ev[3], st));
    if (local_rc != MARS_OK) return fail(local_rc, local_msg);
    return MARS_OK;
}

}  // extern "C"
