// mars_shard.cu -- row-sharded batched top-K across GPUs (one process per
// GPU), with the exchange steps done by NCCL inside the library.
//
// The reference runs on one GPU; its only multi-GPU plan is a note
// (NEXT_STEPS.md:31).  Here a corpus larger than one GPU, or a batch that
// should finish faster, is split by rows: rank r holds rows
// [offset_r, offset_r + n_r) in its own store and every rank answers the same
// B queries.  One call of mars_shard_query_batch_topk on every rank:
//
//  1. the local batched pipeline (mars_batch.cu) on the shard's rows: the
//     sample pass, then ONE ncclAllGather of every shard's best sampled
//     lower bounds per query (B x 16 floats per rank), from which every
//     shard takes the same short-list threshold -- the level a sample of the
//     whole corpus gives, so a shard short-lists about 1 / world of what its
//     own sample would let through;
//  2. the fp16 tensor-core candidates pass against that threshold, then
//     rescore pass 1, which writes each query's record: the candidates whose
//     lower bound reaches the threshold, the K-th and the ceil(K / world)-th
//     largest lower bounds;
//  3. ONE ncclAllGather of the records (3 B + 1 floats per rank): the counts
//     add up to the completeness check (K of them over all shards certify
//     every shard's short list), and the largest K-th bound, the smallest
//     ceil(K / world)-th bound and the threshold are lower bounds of the
//     global K-th score, valid on every shard;
//  4. rescore pass 2 against the largest of them: only rows that can still
//     enter the global top-K are scored exactly (about K / world + a few per
//     shard); uncertified queries are rescanned exactly on every shard;
//  5. the local lists become 64-bit rank keys (score, then id, in one
//     integer; 0 = no entry) and ONE ncclAllGather moves them, B x K x 8
//     bytes per rank;
//  6. every rank selects each query's top-K of the world x K keys.
//
// The results equal a single-GPU mars_query_batch_topk over the whole
// corpus bit for bit: every shard's exact scores are the fp32 scan's, the
// pruning only drops rows that cannot place, and keys rank by (score desc,
// id asc).  Every rank takes the same collective steps in the same order in
// every path: a rank whose local work fails still joins all three
// collectives with neutral data (no samples, bounds -inf, no keys) and
// returns its error after them.
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <algorithm>
#include <cmath>
#include <cstddef>
#include <chrono>
#include <condition_variable>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <type_traits>
#include <vector>

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
        get(api.CommInitRankConfig, "ncclCommInitRankConfig");
        get(api.CommFinalize, "ncclCommFinalize");
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

// Query qi's top-K of the world x K gathered keys ([rank][B][K] layout).
// Every rank's K keys of a query are sorted (largest first, 0 = no entry,
// after the real keys), as every path of the batched pipeline writes them,
// so a key's place in the answer is its place in its own list plus, for
// every other list, the number of keys above it (a binary search; keys are
// unique: global ids differ).  One pass over the world x K keys in shared
// memory, no selection passes.  recs: every shard's bound record
// (rank-major, 3 B + 1 floats each, the last the shard's failure flag); when
// some shard's call failed no result is served and counts are -1.
constexpr int kSortedMergeThreads = 128;
__global__ void __launch_bounds__(kSortedMergeThreads) merge_sorted_keys_kernel(
    const unsigned long long* __restrict__ keys, int world, int K, int B, const float* __restrict__ recs,
    int32_t* __restrict__ ids_out, float* __restrict__ vals_out, int32_t* __restrict__ cnt_out) {
    extern __shared__ unsigned long long s_lists[];   // world x K
    __shared__ int s_n;
    const int qi = blockIdx.x;
    bool failed = false;
    for (int r = 0; r < world; ++r) failed = failed || __ldcg(recs + (int64_t)r * (3 * (int64_t)B + 1) + 3 * B) > 0.0f;
    if (threadIdx.x == 0) s_n = 0;
    const int total = world * K;
    for (int j = threadIdx.x; j < total; j += kSortedMergeThreads) {
        const int r = j / K, e = j - r * K;
        s_lists[j] = __ldg(keys + ((int64_t)r * B + qi) * K + e);
    }
    __syncthreads();
    if (!failed) {
        int n = 0;
        for (int j = threadIdx.x; j < total; j += kSortedMergeThreads) {
            const unsigned long long x = s_lists[j];
            if (x == 0ull) continue;
            ++n;
            const int r0 = j / K;
            int rank = j - r0 * K;                     // keys above x in its own list
            for (int r = 0; r < world && rank < K; ++r) {
                if (r == r0) continue;
                const unsigned long long* l = s_lists + r * K;
                int lo = 0, hi = K;                    // first position whose key is below x
                while (lo < hi) {
                    const int mid = (lo + hi) >> 1;
                    if (l[mid] > x) lo = mid + 1; else hi = mid;
                }
                rank += lo;
            }
            if (rank < K) {
                vals_out[(int64_t)qi * K + rank] = key_score(x);
                ids_out[(int64_t)qi * K + rank] = key_id(x);
            }
        }
        n = warp_reduce_sum_int(n);
        if ((threadIdx.x & 31) == 0) atomicAdd(&s_n, n);
    }
    __syncthreads();
    const int cnt = failed ? 0 : min(s_n, K);
    for (int p = cnt + threadIdx.x; p < K; p += kSortedMergeThreads) {
        vals_out[(int64_t)qi * K + p] = -INFINITY;
        ids_out[(int64_t)qi * K + p] = -1;
    }
    if (threadIdx.x == 0 && cnt_out != nullptr) cnt_out[qi] = failed ? -1 : cnt;
}

// Merge for the sharded query's seeds (lists in any order): the non-empty
// keys go to shared memory and the block's radix selection takes the K
// largest; a rank that failed sends all-ones keys (kFailedKey, never a rank key of a
// finite score); any such key marks the merge failed (count -1).
constexpr unsigned long long kFailedKey = ~0ull;
__global__ void __launch_bounds__(kThreads) merge_keys_flagged_kernel(const unsigned long long* __restrict__ keys,
                                                                      int world, int K, int B,
                                                                      int32_t* __restrict__ ids_out,
                                                                      float* __restrict__ vals_out,
                                                                      int32_t* __restrict__ cnt_out) {
    __shared__ unsigned long long s_keys[kMergeKeys];
    __shared__ __align__(16) int s_hist[2048];   // also read as 64-bit keys
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
    float* d_xsend[2] = {nullptr, nullptr};  // this rank's threshold / bound record
    float* d_xrecv[2] = {nullptr, nullptr};  // every rank's, rank-major
    cudaEvent_t ev[4] = {nullptr, nullptr, nullptr, nullptr};   // local / exchange / merge boundaries
    bool timed = false;
    bool exchange_single = false;           // test hook: world 1 runs the whole exchange protocol
    int32_t timeout_ms = 0;                 // deadline of NCCL's set-up work (creation, first use, teardown)
    void* bfs_state = nullptr;              // mars_shard_query's scratch (made on first use)
};

namespace {

int nccl_fail(const NcclApi* api, ncclResult_t r, const char* what) {
    return fail(MARS_ERR_CUDA, std::string(what) + ": NCCL error " + std::to_string((int)r) + " (" +
                                   (api ? api->GetErrorString(r) : "?") + ")");
}

// The communicator is non-blocking: a call returns once its work is
// enqueued, or ncclInProgress while NCCL still sets something up in the
// background (the communicator itself, a connection on first use, the
// teardown).  The next NCCL call may only follow once the communicator has
// left that state, polled here up to the communicator's deadline: a peer
// that never arrives ends the wait with MARS_ERR_TIMEOUT instead of a hang.
int nccl_settle(const NcclApi* api, ncclComm_t comm, ncclResult_t r, int32_t timeout_ms, const char* what) {
    if (r != ncclSuccess && r != ncclInProgress) return nccl_fail(api, r, what);
    if (r == ncclSuccess) return MARS_OK;
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        ncclResult_t state = ncclSuccess;
        const ncclResult_t q = api->CommGetAsyncError(comm, &state);
        if (q != ncclSuccess) return nccl_fail(api, q, what);
        if (state == ncclSuccess) return MARS_OK;
        if (state != ncclInProgress) return nccl_fail(api, state, what);
        const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0);
        if (timeout_ms > 0 && ms.count() >= timeout_ms)
            return fail(MARS_ERR_TIMEOUT, std::string(what) + ": NCCL still in progress after " +
                                              std::to_string(timeout_ms) + " ms (a peer that did not join?)");
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

// all-gather of one record (`which`: 0 threshold, 1 bound) of `count`
// floats per rank, on st
int exchange_records(void* arg, int which, int32_t count, cudaStream_t st) {
    auto* c = static_cast<mars_shard_comm*>(arg);
    const ncclResult_t r = c->nccl->AllGather(c->d_xsend[which], c->d_xrecv[which], (size_t)count, ncclFloat32,
                                              c->comm, st);
    return nccl_settle(c->nccl, c->comm, r, c->timeout_ms,
                       which == 0 ? "mars_shard_query_batch_topk: threshold all-gather"
                                  : "mars_shard_query_batch_topk: bound all-gather");
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
    MARS_TRY(nccl_settle(c->nccl, c->comm, r, c->timeout_ms, "shard merge: all-gather"));
    shard::merge_keys_flagged_kernel<<<B, shard::kThreads, 0, st>>>(c->d_recv, c->world, K, B, d_ids_out, d_vals_out,
                                                                    d_counts);
    MARS_CUDA_TRY(cudaGetLastError());
    return MARS_OK;
}

int mars::shard_allreduce_max_f32(const ShardCommView& v, float* d, int32_t n, cudaStream_t st) {
    mars_shard_comm* c = comm_of(v);
    const ncclResult_t r = c->nccl->AllReduce(d, d, (size_t)n, ncclFloat32, ncclMax, c->comm, st);
    return nccl_settle(c->nccl, c->comm, r, c->timeout_ms, "shard all-reduce");
}

int mars::shard_allreduce_max_i32(const ShardCommView& v, int32_t* d, int32_t n, cudaStream_t st) {
    mars_shard_comm* c = comm_of(v);
    const ncclResult_t r = c->nccl->AllReduce(d, d, (size_t)n, ncclInt32, ncclMax, c->comm, st);
    return nccl_settle(c->nccl, c->comm, r, c->timeout_ms, "shard all-reduce");
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
    return mars_shard_comm_create_timeout(device, rank, world, unique_id, max_batch, max_k,
                                          MARS_SHARD_DEFAULT_TIMEOUT_MS, out);
}

int mars_shard_comm_create_timeout(int32_t device, int32_t rank, int32_t world, const void* unique_id,
                                   int32_t max_batch, int32_t max_k, int32_t timeout_ms, mars_shard_comm** out) {
    if (out == nullptr || unique_id == nullptr) return fail(MARS_ERR_INVALID, "mars_shard_comm_create: NULL argument");
    *out = nullptr;
    if (world <= 0 || rank < 0 || rank >= world || max_batch <= 0 || max_k <= 0 || max_k > MARS_MAX_TOP_K ||
        (int64_t)world * max_k > kMergeKeys || timeout_ms < 0)
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
    c->timeout_ms = timeout_ms;
    int rc = MARS_OK;
    auto T = [&](cudaError_t e, const char* w) {
        if (e == cudaSuccess) return;
        if (rc == MARS_OK) rc = cuda_fail(e, w, __FILE__, __LINE__);   // records the first failure
        else (void)cudaGetLastError();                                 // later ones only clear the state
    };
    const size_t keys = (size_t)max_batch * max_k;
    T(cudaMalloc(&c->d_send, keys * 8), "shard send keys");
    T(cudaMalloc(&c->d_recv, keys * 8 * world), "shard gathered keys");
    const size_t rec[2] = {(size_t)shard_thr_floats(max_batch), (size_t)shard_rec_floats(max_batch)};
    for (int w = 0; w < 2; ++w) {
        T(cudaMalloc(&c->d_xsend[w], rec[w] * 4), "shard record");
        T(cudaMalloc(&c->d_xrecv[w], rec[w] * 4 * world), "shard records of every rank");
    }
    for (auto& e : c->ev) T(cudaEventCreate(&e), "event");
    if (rc == MARS_OK) {
        ncclUniqueId id;
        std::memcpy(&id, unique_id, sizeof(id));
        // non-blocking: creation runs in the background and is polled
        // against the deadline (a rank that never joins ends it with
        // MARS_ERR_TIMEOUT, and the half-made communicator is aborted)
        ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
        cfg.blocking = 0;
        const ncclResult_t r = api->CommInitRankConfig(&c->comm, world, id, rank, &cfg);
        if (r != ncclSuccess && r != ncclInProgress) {
            c->comm = nullptr;
            rc = nccl_fail(api, r, "mars_shard_comm_create: ncclCommInitRankConfig");
        } else {
            rc = nccl_settle(api, c->comm, r, timeout_ms, "mars_shard_comm_create");
            if (rc != MARS_OK) {
                api->CommAbort(c->comm);
                c->comm = nullptr;
            }
        }
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
    if (c->comm != nullptr) {
        // flush and quiesce (polled against the deadline), then free; a
        // teardown that does not settle is aborted instead
        if (nccl_settle(c->nccl, c->comm, c->nccl->CommFinalize(c->comm), c->timeout_ms,
                        "mars_shard_comm_destroy") == MARS_OK)
            c->nccl->CommDestroy(c->comm);
        else
            c->nccl->CommAbort(c->comm);
    }
    cudaFree(c->d_send);
    cudaFree(c->d_recv);
    for (int w = 0; w < 2; ++w) {
        cudaFree(c->d_xsend[w]);
        cudaFree(c->d_xrecv[w]);
    }
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
    // ncclInProgress: NCCL is still setting up an operation (not an error)
    if (async != ncclSuccess && async != ncclInProgress)
        return nccl_fail(c->nccl, async, "mars_shard_comm_status: asynchronous error");
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

int mars_shard_comm_set_exchange_at_world1(mars_shard_comm* c, int32_t enable) {
    if (c == nullptr) return fail(MARS_ERR_INVALID, "mars_shard_comm_set_exchange_at_world1: NULL communicator");
    c->exchange_single = enable != 0;
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
    if (c->world == 1 && !c->exchange_single) {
        // one shard holds every row: its local answer is the merged one, so
        // the call is the single-store pipeline (no records, no exchange,
        // no merge)
        const int rc = (s == nullptr || ctx == nullptr || s->device != c->device)
                           ? fail(MARS_ERR_INVALID, "mars_shard_query_batch_topk: store and context must be on "
                                                    "the communicator's device")
                           : batch_topk_sharded(s, ctx, d_queries, query_pitch, B, query_timestamp, lambda,
                                                modality_filter, use_importance, K, row_offset, d_ids, d_vals,
                                                d_counts, st, nullptr);
        if (c->timed)
            for (int e = 1; e < 4; ++e) MARS_CUDA_TRY(cudaEventRecord(c->ev[e], st));
        return rc;
    }

    // 1-4: the local pipeline with the two record exchanges
    BoundExchange xchg{&exchange_records, c, c->world, {c->d_xsend[0], c->d_xsend[1]},
                       {c->d_xrecv[0], c->d_xrecv[1]}, false, false};
    int local_rc = MARS_OK;
    if (s == nullptr || ctx == nullptr || s->device != c->device)
        local_rc = fail(MARS_ERR_INVALID, "mars_shard_query_batch_topk: store and context must be on the "
                                          "communicator's device");
    else
        local_rc = batch_topk_sharded(s, ctx, d_queries, query_pitch, B, query_timestamp, lambda, modality_filter,
                                      use_importance, K, row_offset, d_ids, d_vals, d_counts, st, &xchg);
    const std::string local_msg = local_rc != MARS_OK ? std::string(mars_last_error()) : std::string();
    // the local call ended before an exchange (an error, or the exact
    // per-query scans of a small shard): join it with a neutral record
    if (!xchg.theta_done) {
        MARS_TRY(shard_neutral_thr(c->d_xsend[0], B, st));
        MARS_TRY(exchange_records(c, 0, shard_thr_floats(B), st));
    }
    if (!xchg.done) {
        MARS_TRY(shard_neutral_rec(c->d_xsend[1], B, local_rc != MARS_OK, st));
        MARS_TRY(exchange_records(c, 1, shard_rec_floats(B), st));
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
    MARS_TRY(nccl_settle(c->nccl, c->comm, r, c->timeout_ms, "mars_shard_query_batch_topk: all-gather"));
    if (c->timed) MARS_CUDA_TRY(cudaEventRecord(c->ev[2], st));

    // 5: every rank merges
    shard::merge_sorted_keys_kernel<<<B, shard::kSortedMergeThreads, (size_t)c->world * K * 8, st>>>(
        c->d_recv, c->world, K, B, c->d_xrecv[1], d_ids, d_vals, d_counts);
    MARS_CUDA_TRY(cudaGetLastError());
    if (c->timed) MARS_CUDA_TRY(cudaEventRecord(c->ev[3], st));
    if (local_rc != MARS_OK) return fail(local_rc, local_msg);
    return MARS_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// One-GPU emulation of the sharded call (test hook).  Every shard runs
// batch_topk_sharded on its own host thread and stream; an exchange is two
// host barriers: after the first every shard's record is ready (its event
// recorded), and each shard copies all records into its own receive buffer;
// after the second every copy is enqueued, and each stream waits for all of
// them before it may write a send buffer again.  No kernel waits on another.
namespace {

struct EmuShared {
    int world = 0;
    std::mutex mu;
    std::condition_variable cv;
    int arrived = 0;
    long generation = 0;
    std::vector<cudaEvent_t> ready, copied;
    std::vector<float*> send[2], recv[2];

    void barrier() {
        std::unique_lock<std::mutex> lock(mu);
        const long g = generation;
        if (++arrived == world) {
            arrived = 0;
            ++generation;
            cv.notify_all();
        } else {
            cv.wait(lock, [&] { return generation != g; });
        }
    }
};

struct EmuArg {
    EmuShared* sh;
    int rank;
};

int emu_gather(void* arg, int which, int32_t count, cudaStream_t st) {
    auto* a = static_cast<EmuArg*>(arg);
    EmuShared& sh = *a->sh;
    const int r = a->rank;
    // both barriers are reached whatever fails, so no shard is left waiting
    cudaError_t e = cudaEventRecord(sh.ready[r], st);
    sh.barrier();
    for (int q = 0; q < sh.world && e == cudaSuccess; ++q) {
        e = cudaStreamWaitEvent(st, sh.ready[q], 0);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(sh.recv[which][r] + (size_t)q * count, sh.send[which][q], (size_t)count * 4,
                                cudaMemcpyDeviceToDevice, st);
    }
    const cudaError_t e2 = cudaEventRecord(sh.copied[r], st);
    sh.barrier();
    cudaError_t e3 = cudaSuccess;
    for (int q = 0; q < sh.world && e3 == cudaSuccess; ++q) e3 = cudaStreamWaitEvent(st, sh.copied[q], 0);
    if (e != cudaSuccess) return cuda_fail(e, "shard emulation: record copy", __FILE__, __LINE__);
    if (e2 != cudaSuccess) return cuda_fail(e2, "shard emulation: event", __FILE__, __LINE__);
    if (e3 != cudaSuccess) return cuda_fail(e3, "shard emulation: event wait", __FILE__, __LINE__);
    return MARS_OK;
}

}  // namespace

extern "C" int mars_shard_emulate_query_batch_topk(int32_t world, const mars_store* const* stores,
                                                   mars_batch_ctx* const* ctxs, const int32_t* row_offsets,
                                                   const float* d_queries, int32_t query_pitch, int32_t B,
                                                   float query_timestamp, float lambda, int32_t modality_filter,
                                                   int32_t use_importance, int32_t K, int32_t* d_ids,
                                                   float* d_vals, int32_t* d_counts) {
    if (world <= 0 || world > 16 || stores == nullptr || ctxs == nullptr || row_offsets == nullptr ||
        d_ids == nullptr || d_vals == nullptr || d_counts == nullptr)
        return fail(MARS_ERR_INVALID, "mars_shard_emulate_query_batch_topk: bad arguments");
    if (B <= 0 || K <= 0 || K > MARS_MAX_TOP_K || (int64_t)world * K > kMergeKeys)
        return fail(MARS_ERR_INVALID, "mars_shard_emulate_query_batch_topk: need B > 0, 0 < K <= 256, world x K <= 4096");
    for (int r = 0; r < world; ++r)
        if (stores[r] == nullptr || ctxs[r] == nullptr || stores[r]->device != stores[0]->device)
            return fail(MARS_ERR_INVALID, "mars_shard_emulate_query_batch_topk: every shard on one device");
    const int dev = stores[0]->device;
    MarsDeviceGuard g(dev);
    if (!g.ok) return fail(MARS_ERR_NO_DEVICE, "mars_shard_emulate_query_batch_topk: cudaSetDevice failed");
    EmuShared sh;
    sh.world = world;
    const size_t n = (size_t)B * K;
    const int32_t cnt[2] = {shard_thr_floats(B), shard_rec_floats(B)};
    std::vector<int32_t*> l_ids(world, nullptr), l_cnt(world, nullptr);
    std::vector<float*> l_vals(world, nullptr);
    std::vector<unsigned long long*> keys(world, nullptr);
    std::vector<cudaEvent_t> keys_ready(world, nullptr);
    unsigned long long* all_keys = nullptr;
    sh.ready.assign(world, nullptr);
    sh.copied.assign(world, nullptr);
    for (int w = 0; w < 2; ++w) {
        sh.send[w].assign(world, nullptr);
        sh.recv[w].assign(world, nullptr);
    }
    int rc = MARS_OK;
    auto T = [&](cudaError_t e, const char* what) {
        if (e == cudaSuccess) return;
        if (rc == MARS_OK) rc = cuda_fail(e, what, __FILE__, __LINE__);   // records the first failure
        else (void)cudaGetLastError();                                 // later ones only clear the state
    };
    for (int r = 0; r < world; ++r) {
        T(cudaMalloc(&l_ids[r], n * 4), "emulation buffers");
        T(cudaMalloc(&l_vals[r], n * 4), "emulation buffers");
        T(cudaMalloc(&l_cnt[r], (size_t)B * 4), "emulation buffers");
        T(cudaMalloc(&keys[r], n * 8), "emulation buffers");
        for (int w = 0; w < 2; ++w) {
            T(cudaMalloc(&sh.send[w][r], (size_t)cnt[w] * 4), "emulation buffers");
            T(cudaMalloc(&sh.recv[w][r], (size_t)cnt[w] * 4 * world), "emulation buffers");
        }
        T(cudaEventCreateWithFlags(&sh.ready[r], cudaEventDisableTiming), "event");
        T(cudaEventCreateWithFlags(&sh.copied[r], cudaEventDisableTiming), "event");
        T(cudaEventCreateWithFlags(&keys_ready[r], cudaEventDisableTiming), "event");
    }
    T(cudaMalloc(&all_keys, n * 8 * world), "emulation buffers");
    T(cudaDeviceSynchronize(), "emulation set-up");
    std::vector<int> rcs(world, MARS_OK);
    std::vector<std::string> msgs(world);
    if (rc == MARS_OK) {
        std::vector<EmuArg> args(world);
        std::vector<std::thread> th;
        for (int r = 0; r < world; ++r) {
            args[r] = EmuArg{&sh, r};
            th.emplace_back([&, r] {
                MarsDeviceGuard tg(dev);
                cudaStream_t st = batch_ctx_stream(ctxs[r]);
                BoundExchange x{&emu_gather, &args[r], world, {sh.send[0][r], sh.send[1][r]},
                                {sh.recv[0][r], sh.recv[1][r]}, false, false};
                int lrc = tg.ok ? batch_topk_sharded(stores[r], ctxs[r], d_queries, query_pitch, B, query_timestamp,
                                                     lambda, modality_filter, use_importance, K, row_offsets[r],
                                                     l_ids[r], l_vals[r], l_cnt[r], st, &x)
                                : fail(MARS_ERR_NO_DEVICE, "shard emulation: cudaSetDevice failed");
                if (lrc != MARS_OK) msgs[r] = mars_last_error();
                // every shard takes both exchanges exactly once
                if (!x.theta_done) {
                    shard_neutral_thr(sh.send[0][r], B, st);
                    emu_gather(&args[r], 0, cnt[0], st);
                }
                if (!x.done) {
                    shard_neutral_rec(sh.send[1][r], B, lrc != MARS_OK, st);
                    emu_gather(&args[r], 1, cnt[1], st);
                }
                if (lrc == MARS_OK)
                    shard::pack_keys_kernel<<<(int)std::min<size_t>((n + 255) / 256, 1024), 256, 0, st>>>(
                        l_ids[r], l_vals[r], (int64_t)n, keys[r]);
                else
                    cudaMemsetAsync(keys[r], 0, n * 8, st);
                cudaEventRecord(keys_ready[r], st);
                rcs[r] = lrc;
            });
        }
        for (auto& t : th) t.join();
        // the key "all-gather" and the merge, on shard 0's stream
        cudaStream_t st0 = batch_ctx_stream(ctxs[0]);
        for (int r = 0; r < world; ++r) {
            T(cudaStreamWaitEvent(st0, keys_ready[r], 0), "event wait");
            T(cudaMemcpyAsync(all_keys + (size_t)r * n, keys[r], n * 8, cudaMemcpyDeviceToDevice, st0), "key copy");
        }
        if (rc == MARS_OK) {
            shard::merge_sorted_keys_kernel<<<B, shard::kSortedMergeThreads, (size_t)world * K * 8, st0>>>(
                all_keys, world, K, B, sh.recv[1][0], d_ids, d_vals, d_counts);
            T(cudaGetLastError(), "merge");
        }
        T(cudaStreamSynchronize(st0), "emulation");
    }
    cudaDeviceSynchronize();
    for (int r = 0; r < world; ++r) {
        cudaFree(l_ids[r]); cudaFree(l_vals[r]); cudaFree(l_cnt[r]); cudaFree(keys[r]);
        for (int w = 0; w < 2; ++w) { cudaFree(sh.send[w][r]); cudaFree(sh.recv[w][r]); }
        if (sh.ready[r]) cudaEventDestroy(sh.ready[r]);
        if (sh.copied[r]) cudaEventDestroy(sh.copied[r]);
        if (keys_ready[r]) cudaEventDestroy(keys_ready[r]);
    }
    cudaFree(all_keys);
    if (rc != MARS_OK) return rc;
    for (int r = 0; r < world; ++r)
        if (rcs[r] != MARS_OK) return fail(rcs[r], msgs[r]);
    return MARS_OK;
}
