// mars_shard_bfs.cu -- query_memory_fast (scan -> top-K seeds -> BFS ->
// top-K of the visited set) over a row-sharded corpus, one process per GPU.
//
// Reference: query_memory_fast (src/memory_cuda.cu:1069-1158) with its BFS
// (bfs_init_seeds_kernel / bfs_expand_device_driven_kernel, :450-514) on one
// GPU; the reference has no multi-GPU path.  The semantics are this
// library's canonical BFS (the same answer as mars_query on one GPU holding
// every row): a node first reached at level h scores
// max over its level h-1 parents p of fmaxf(score_p * decay, own * 0.8f),
// own = the node's fused score (-FLT_MAX when the modality filter rejects
// it), and the answer is the top-K of every visited node by (score desc, id
// asc).
//
// The graph (a CSR over global row ids) is small next to the rows and is
// replicated on every rank; rank r holds rows [row_offset, row_offset + n_r).
// Expanding a level needs only the graph and the previous level's scores,
// so every rank expands every level itself and all ranks hold the same
// level (the same set; sorted by id so that positions agree).  Only a
// node's own score needs its row, held by one rank: per level, each rank
// scores the nodes it owns, writes -inf for the others, and one NCCL
// all-reduce (max) gives every rank every own score.  Collectives per query:
// one all-gather of the K local seed keys, one all-reduce per hop
// (kLevelCap floats), one all-reduce of the K result modalities.
//
// Visited marks are the 64-bit words of the single-GPU BFS: (stamp << 32 |
// score key), stamp = (epoch << 4) | (15 - level); one atomicMax per edge
// claims a node for a level and keeps its best parent, and nothing is
// cleared between queries.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <string>

#include "mars_b200.h"
#include "mars_common.cuh"
#include "mars_internal.h"
#include "mars_kernels.cuh"
#include "mars_nccl.h"
#include "mars_select.cuh"
#include "mars_shard_internal.h"

namespace mars {
namespace sbfs {

constexpr int kLevelCap = 16384;     // nodes of one level
constexpr int kVisitCap = 16384;     // visited nodes of one query (all levels)
constexpr int kSortThreads = 1024;
constexpr uint32_t kMaxEpoch = (1u << 28) - 1;

// lvl[0..15]: start of level h in the visited list (lvl[h + 1] = its end);
// lvl[16]: nodes claimed by the running expansion; lvl[17]: overflow flag;
// lvl[18]: size of the level being scored.
constexpr int kClaimed = 16, kOverflow = 17, kLevelSize = 18, kLvlWords = 20;

struct Params {
    StoreView s;                 // this rank's rows (local ids)
    const int32_t* ro;           // global CSR
    const int32_t* ci;
    int32_t n_global;
    int32_t row_offset;          // first global row of this rank
    const float4* q;
    float t_q, lambda, decay;
    int32_t filter, use_imp;
    unsigned long long* stamp;   // n_global words
    uint32_t epoch_base;         // epoch << 4
    int32_t* vis_ids;            // kVisitCap
    float* vis_score;
    int32_t* lvl;
    int32_t* level;              // kLevelCap: the level being built, then sorted
    float* own;                  // kLevelCap own scores (-inf where not owned)
};

__device__ __forceinline__ unsigned long long stamp_word(uint32_t epoch_base, int level, float key_score) {
    return ((unsigned long long)(epoch_base | (uint32_t)(15 - level)) << 32) | f2key(key_score);
}

// The seeds: level 0 of the visited list (count -1: some rank failed).
__global__ void seed_kernel(Params p, const int32_t* __restrict__ ids, const float* __restrict__ vals,
                            const int32_t* __restrict__ cnt) {
    const int n = max(*cnt, 0);
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int32_t u = ids[i];
        atomicMax(p.stamp + u, stamp_word(p.epoch_base, 0, vals[i]));
        p.vis_ids[i] = u;
        p.vis_score[i] = vals[i];
    }
    if (threadIdx.x == 0) {
        p.lvl[0] = 0;
        p.lvl[1] = n;
        p.lvl[kClaimed] = 0;
        p.lvl[kOverflow] = *cnt < 0 ? 2 : 0;
    }
}

// Level hop - 1 -> the unordered list of nodes first reached at level hop.
__global__ void expand_kernel(Params p, int hop) {
    const int lane = threadIdx.x & 31;
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nw = (gridDim.x * blockDim.x) >> 5;
    const int32_t beg = p.lvl[hop - 1], end = p.lvl[hop];
    for (int32_t idx = beg + gw; idx < end; idx += nw) {
        const int32_t u = p.vis_ids[idx];
        const unsigned long long word = stamp_word(p.epoch_base, hop, p.vis_score[idx] * p.decay);
        const int32_t e0 = __ldg(p.ro + u), e1 = __ldg(p.ro + u + 1);
        for (int32_t e = e0 + lane; e < e1; e += 32) {
            const int32_t v = __ldg(p.ci + e);
            if (v < 0 || v >= p.n_global) continue;
            const unsigned long long old = atomicMax(p.stamp + v, word);
            if ((uint32_t)(old >> 32) < p.epoch_base) {      // first claim in this query
                const int pos = atomicAdd(p.lvl + kClaimed, 1);
                if (pos < kLevelCap) p.level[pos] = v;
                else atomicMax(p.lvl + kOverflow, 1);
            }
        }
    }
}

// One CTA: the level sorted by id (the same order on every rank), its size
// published, the claim counter reset for the next expansion.
__global__ void __launch_bounds__(kSortThreads) sort_kernel(Params p, int hop) {
    extern __shared__ int32_t s_ids[];
    const int claimed = p.lvl[kClaimed];
    const int total = p.lvl[hop];                 // visited before this level
    int n = min(claimed, kLevelCap);
    if (total + n > kVisitCap) n = max(0, kVisitCap - total);
    int P = 1;
    while (P < n) P <<= 1;
    for (int i = threadIdx.x; i < P; i += kSortThreads) s_ids[i] = i < n ? p.level[i] : INT32_MAX;
    __syncthreads();
    for (int k = 2; k <= P; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int t = threadIdx.x; t < (P >> 1); t += kSortThreads) {
                const int i = ((t & ~(j - 1)) << 1) | (t & (j - 1));
                const int l = i | j;
                const int32_t a = s_ids[i], b = s_ids[l];
                const bool asc = (i & k) == 0;
                if (asc ? (a > b) : (a < b)) { s_ids[i] = b; s_ids[l] = a; }
            }
            __syncthreads();
        }
    }
    for (int i = threadIdx.x; i < n; i += kSortThreads) p.level[i] = s_ids[i];
    if (threadIdx.x == 0) {
        if (claimed > n) atomicMax(p.lvl + kOverflow, 1);
        p.lvl[kLevelSize] = n;
        p.lvl[kClaimed] = 0;
    }
}

// Own scores of the level's nodes that this rank holds (one warp per node,
// the scan's canonical dot); -inf for the others and past the level.
__global__ void own_kernel(Params p) {
    const int lane = threadIdx.x & 31;
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nw = (gridDim.x * blockDim.x) >> 5;
    const int n = p.lvl[kLevelSize];
    const int32_t n_local = p.s.d_n != nullptr ? *p.s.d_n : 0;   // 0: no rows here (this rank failed)
    for (int i = gw; i < kLevelCap; i += nw) {
        float own = -INFINITY;
        if (i < n) {
            const int32_t u = p.level[i] - p.row_offset;
            if (u >= 0 && u < n_local) {
                if (p.filter >= 0 && __ldg(p.s.mod + u) != p.filter) {
                    own = -FLT_MAX;
                } else {
                    const float4* row = reinterpret_cast<const float4*>(p.s.E) + (int64_t)u * p.s.pitch4;
                    const float dot = warp_dot_canonical(row, p.q, p.s.nc, lane);
                    own = fused_weight_apply(dot, __ldg(p.s.ts + u), p.t_q, p.lambda);
                    if (p.use_imp != 0 && p.s.imp != nullptr) own = own * __ldg(p.s.imp + u);
                }
            }
        }
        if (lane == 0) p.own[i] = own;
    }
}

// After the all-reduce: the level's scores, appended to the visited list.
__global__ void score_kernel(Params p, int hop) {
    const int n = p.lvl[kLevelSize];
    const int base = p.lvl[hop];
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const int32_t u = p.level[i];
        const float best_parent = key2f((uint32_t)(__ldcg(p.stamp + u) & 0xffffffffull));
        p.vis_ids[base + i] = u;
        p.vis_score[base + i] = fmaxf(best_parent, p.own[i] * 0.8f);
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) p.lvl[hop + 1] = base + n;
}

// One CTA: the top-K of every visited node by (score desc, id asc); the
// modality of each result that this rank holds (-1 otherwise) goes to mods
// for the exchange.
__global__ void __launch_bounds__(kSortThreads) final_kernel(Params p, int hops, int K, mars_query_result* out,
                                                             int32_t* out_cnt, int32_t* mods) {
    extern __shared__ unsigned long long s_keys[];
    const int total = p.lvl[hops + 1];
    int P = 1;
    while (P < total) P <<= 1;
    for (int i = threadIdx.x; i < P; i += kSortThreads)
        s_keys[i] = i < total ? rank_key(p.vis_score[i], p.vis_ids[i]) : 0ull;
    block_bitonic_desc<kSortThreads>(s_keys, P);
    const int n = min(K, total);
    const int32_t n_local = p.s.d_n != nullptr ? *p.s.d_n : 0;
    for (int i = threadIdx.x; i < n; i += kSortThreads) {
        const int32_t u = key_id(s_keys[i]);
        // the level of u: the visited list is the concatenation of the levels
        // and u appears once; find its position's level by searching the list
        int hop_of_u = 0;
        for (int lv = 0; lv <= hops; ++lv) {
            bool found = false;
            for (int j = p.lvl[lv]; j < p.lvl[lv + 1]; ++j)
                if (p.vis_ids[j] == u) { found = true; break; }
            if (found) { hop_of_u = lv; break; }
        }
        mars_query_result r;
        r.node_id = u;
        r.score = key_score(s_keys[i]);
        r.hops_from_seed = hop_of_u;
        const int32_t lu = u - p.row_offset;
        r.modality = (lu >= 0 && lu < n_local) ? __ldg(p.s.mod + lu) : -1;
        out[i] = r;
        mods[i] = r.modality;
    }
    if (threadIdx.x == 0) *out_cnt = p.lvl[kOverflow] != 0 ? -p.lvl[kOverflow] : n;
}

}  // namespace sbfs
}  // namespace mars

using namespace mars;
using namespace mars::sbfs;

// Per-communicator state of the sharded query (made on first use).
struct ShardBfsState {
    int32_t n_global = 0;
    int32_t pitch = 0;
    int32_t max_k = 0;
    uint32_t epoch = 0;
    unsigned long long* d_stamp = nullptr;
    float* d_q = nullptr;
    int32_t* d_lvl = nullptr;
    int32_t* d_vis_ids = nullptr;
    float* d_vis_score = nullptr;
    int32_t* d_level = nullptr;
    float* d_own = nullptr;
    int32_t* d_seed_ids = nullptr;      // local top-K, then the merged seeds
    float* d_seed_vals = nullptr;
    int32_t* d_seed_cnt = nullptr;
    mars_query_result* d_res = nullptr;
    int32_t* d_res_cnt = nullptr;
    int32_t* d_mods = nullptr;
    mars_query_result* h_res = nullptr;  // pinned
    int32_t* h_res_cnt = nullptr;
    int32_t* h_mods = nullptr;
    ~ShardBfsState() {
        cudaFree(d_stamp); cudaFree(d_q); cudaFree(d_lvl); cudaFree(d_vis_ids); cudaFree(d_vis_score);
        cudaFree(d_level); cudaFree(d_own); cudaFree(d_seed_ids); cudaFree(d_seed_vals); cudaFree(d_seed_cnt);
        cudaFree(d_res); cudaFree(d_res_cnt); cudaFree(d_mods);
        cudaFreeHost(h_res); cudaFreeHost(h_res_cnt); cudaFreeHost(h_mods);
    }
};

void shard_bfs_state_free(void* st) { delete static_cast<ShardBfsState*>(st); }

namespace {

int prepare(ShardCommView& v, int32_t n_global, int32_t pitch, int32_t K, ShardBfsState** out) {
    auto* b = static_cast<ShardBfsState*>(*v.bfs_state);
    if (b != nullptr && (b->n_global < n_global || b->pitch < pitch || b->max_k < K)) {
        cudaDeviceSynchronize();
        delete b;
        b = nullptr;
        *v.bfs_state = nullptr;
    }
    if (b == nullptr) {
        b = new ShardBfsState();
        b->n_global = n_global;
        b->pitch = pitch;
        b->max_k = std::max(K, 64);
        int rc = MARS_OK;
        auto T = [&](cudaError_t e, const char* w) {
            if (e == cudaSuccess) return;
            if (rc == MARS_OK) rc = cuda_fail(e, w, __FILE__, __LINE__);   // records the first failure
            else (void)cudaGetLastError();                                 // later ones only clear the state
        };
        T(cudaMalloc(&b->d_stamp, (size_t)n_global * 8), "shard BFS marks");
        if (rc == MARS_OK) T(cudaMemset(b->d_stamp, 0, (size_t)n_global * 8), "memset");
        T(cudaMalloc(&b->d_q, (size_t)pitch * 4), "query");
        if (rc == MARS_OK) T(cudaMemset(b->d_q, 0, (size_t)pitch * 4), "memset");
        T(cudaMalloc(&b->d_lvl, kLvlWords * 4), "levels");
        T(cudaMalloc(&b->d_vis_ids, (size_t)kVisitCap * 4), "visited");
        T(cudaMalloc(&b->d_vis_score, (size_t)kVisitCap * 4), "visited");
        T(cudaMalloc(&b->d_level, (size_t)kLevelCap * 4), "level");
        T(cudaMalloc(&b->d_own, (size_t)kLevelCap * 4), "own scores");
        T(cudaMalloc(&b->d_seed_ids, (size_t)b->max_k * 4), "seeds");
        T(cudaMalloc(&b->d_seed_vals, (size_t)b->max_k * 4), "seeds");
        T(cudaMalloc(&b->d_seed_cnt, 4), "seeds");
        T(cudaMalloc(&b->d_res, (size_t)b->max_k * sizeof(mars_query_result)), "results");
        T(cudaMalloc(&b->d_res_cnt, 4), "results");
        T(cudaMalloc(&b->d_mods, (size_t)b->max_k * 4), "modalities");
        T(cudaMallocHost(&b->h_res, (size_t)b->max_k * sizeof(mars_query_result)), "pinned results");
        T(cudaMallocHost(&b->h_res_cnt, 4), "pinned results");
        T(cudaMallocHost(&b->h_mods, (size_t)b->max_k * 4), "pinned modalities");
        static bool attr_done[64] = {};
        int dev = 0;
        cudaGetDevice(&dev);
        if (rc == MARS_OK && dev < 64 && !attr_done[dev]) {
            T(cudaFuncSetAttribute(final_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kVisitCap * 8), "smem");
            T(cudaFuncSetAttribute(sort_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kLevelCap * 4), "smem");
            attr_done[dev] = rc == MARS_OK;
        }
        if (rc != MARS_OK) { delete b; return rc; }
        *v.bfs_state = b;
    }
    *out = b;
    return MARS_OK;
}

}  // namespace

extern "C" int mars_shard_query(const mars_store* s, mars_query_ctx* ctx, mars_shard_comm* comm,
                                const int32_t* d_row_offsets, const int32_t* d_col_indices, int32_t n_global,
                                const float* query, float t_q, const mars_retrieval_config* cfg,
                                int32_t row_offset, mars_query_result* out, int32_t* n_out) {
    // cfg (top_k, hops) and n_global are the same on every rank: checks on
    // them reject on every rank alike, before any collective
    if (comm == nullptr || cfg == nullptr || out == nullptr || n_out == nullptr || query == nullptr)
        return fail(MARS_ERR_INVALID, "mars_shard_query: NULL argument");
    ShardCommView v;
    MARS_TRY(shard_comm_view(comm, &v));
    const int K = cfg->top_k, hops = cfg->bfs_max_hops;
    if (K <= 0 || K > v.max_k || K > MARS_MAX_TOP_K || hops < 0 || hops > MARS_MAX_BFS_HOPS || n_global <= 0)
        return fail(MARS_ERR_INVALID, "mars_shard_query: top_k must be in [1, the communicator's max_k], "
                                      "bfs_max_hops in [0, 14], n_global > 0");
    if (hops > 0 && (d_row_offsets == nullptr || d_col_indices == nullptr))
        return fail(MARS_ERR_INVALID, "mars_shard_query: BFS hops need the global CSR");
    *n_out = 0;
    MarsDeviceGuard g(v.device);
    if (!g.ok) return fail(MARS_ERR_NO_DEVICE, "mars_shard_query: cudaSetDevice failed");
    int local_rc = MARS_OK;
    if (s == nullptr || ctx == nullptr || s->device != v.device)
        local_rc = fail(MARS_ERR_INVALID, "mars_shard_query: store and context must be on the communicator's device");
    else if ((s->dim & 3) != 0)
        local_rc = fail(MARS_ERR_UNSUPPORTED, "mars_shard_query: needs dim % 4 == 0");
    else if (row_offset < 0 || (int64_t)row_offset + s->n > n_global)
        local_rc = fail(MARS_ERR_INVALID, "mars_shard_query: the shard's rows must lie in [0, n_global)");
    ShardBfsState* b = nullptr;
    const int32_t pitch = s != nullptr ? s->pitch : 4;
    MARS_TRY(prepare(v, n_global, pitch, K, &b));
    cudaStream_t st = ctx != nullptr ? static_cast<cudaStream_t>(mars_query_ctx_stream(ctx)) : nullptr;
    if (local_rc == MARS_OK) MARS_CUDA_TRY(cudaStreamWaitEvent(st, s->written, 0));
    if (b->epoch >= kMaxEpoch) {
        MARS_CUDA_TRY(cudaMemsetAsync(b->d_stamp, 0, (size_t)b->n_global * 8, st));
        b->epoch = 0;
    }
    const uint32_t epoch = ++b->epoch;

    // 1. seeds: the local top-K, one all-gather of their keys, the merge
    const int32_t dim = s != nullptr ? s->dim : 0;
    if (local_rc == MARS_OK) {
        MARS_CUDA_TRY(cudaMemcpyAsync(b->d_q, query, (size_t)dim * 4, cudaMemcpyDefault, st));
        local_rc = mars_scan_topk(s, ctx, b->d_q, t_q, cfg->time_decay_lambda, cfg->modality_filter,
                                  cfg->use_importance, K, row_offset, b->d_seed_ids, b->d_seed_vals, nullptr, st);
    }
    MARS_TRY(shard_gather_merge(v, local_rc == MARS_OK ? b->d_seed_ids : nullptr, b->d_seed_vals, 1, K,
                                b->d_seed_ids, b->d_seed_vals, b->d_seed_cnt, local_rc != MARS_OK, st));

    Params p{};
    if (s != nullptr && local_rc == MARS_OK) {
        p.s.E = s->d_E; p.s.ts = s->d_ts; p.s.imp = s->d_imp; p.s.mod = s->d_mod; p.s.d_n = s->d_n;
        p.s.pitch4 = s->pitch / 4; p.s.nc = (s->dim + 3) / 4;
    }
    p.ro = d_row_offsets;
    p.ci = d_col_indices;
    p.n_global = n_global;
    p.row_offset = row_offset;
    p.q = reinterpret_cast<const float4*>(b->d_q);
    p.t_q = t_q;
    p.lambda = cfg->time_decay_lambda;
    p.decay = cfg->bfs_score_decay;
    p.filter = cfg->modality_filter;
    p.use_imp = cfg->use_importance;
    p.stamp = b->d_stamp;
    p.epoch_base = epoch << 4;
    p.vis_ids = b->d_vis_ids;
    p.vis_score = b->d_vis_score;
    p.lvl = b->d_lvl;
    p.level = b->d_level;
    p.own = b->d_own;
    const bool run = local_rc == MARS_OK;
    seed_kernel<<<1, 256, 0, st>>>(p, b->d_seed_ids, b->d_seed_vals, b->d_seed_cnt);
    MARS_CUDA_TRY(cudaGetLastError());

    // 2. per hop: expand (every rank), own scores (owners), all-reduce, scores
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, v.device);
    for (int h = 1; h <= hops; ++h) {
        expand_kernel<<<sms, 256, 0, st>>>(p, h);
        MARS_CUDA_TRY(cudaGetLastError());
        sort_kernel<<<1, kSortThreads, kLevelCap * 4, st>>>(p, h);
        MARS_CUDA_TRY(cudaGetLastError());
        // a rank whose part failed scores nothing (its view has no rows)
        Params po = p;
        if (!run) po.s = StoreView{};
        own_kernel<<<2 * sms, 256, 0, st>>>(po);
        MARS_CUDA_TRY(cudaGetLastError());
        MARS_TRY(shard_allreduce_max_f32(v, b->d_own, kLevelCap, st));
        score_kernel<<<(kLevelCap + 255) / 256, 256, 0, st>>>(p, h);
        MARS_CUDA_TRY(cudaGetLastError());
    }

    // 3. the top-K of the visited set, and the results' modalities from their owners
    Params pf = p;
    if (!run) pf.s = StoreView{};
    final_kernel<<<1, kSortThreads, kVisitCap * 8, st>>>(pf, hops, K, b->d_res, b->d_res_cnt, b->d_mods);
    MARS_CUDA_TRY(cudaGetLastError());
    MARS_TRY(shard_allreduce_max_i32(v, b->d_mods, K, st));
    MARS_CUDA_TRY(cudaMemcpyAsync(b->h_res, b->d_res, (size_t)K * sizeof(mars_query_result), cudaMemcpyDeviceToHost, st));
    MARS_CUDA_TRY(cudaMemcpyAsync(b->h_res_cnt, b->d_res_cnt, 4, cudaMemcpyDeviceToHost, st));
    MARS_CUDA_TRY(cudaMemcpyAsync(b->h_mods, b->d_mods, (size_t)K * 4, cudaMemcpyDeviceToHost, st));
    MARS_CUDA_TRY(cudaStreamSynchronize(st));
    if (local_rc != MARS_OK) return fail(local_rc, "mars_shard_query: local failure on this rank");
    if (*b->h_res_cnt == -2)
        return fail(MARS_ERR_INVALID, "mars_shard_query: another rank's part of the call failed");
    if (*b->h_res_cnt < 0)
        return fail(MARS_ERR_CAPACITY, "mars_shard_query: the BFS outgrew its level or visited capacity (16384)");
    const int n = *b->h_res_cnt;
    for (int i = 0; i < n; ++i) {
        out[i] = b->h_res[i];
        out[i].modality = b->h_mods[i];
    }
    *n_out = n;
    return MARS_OK;
}
