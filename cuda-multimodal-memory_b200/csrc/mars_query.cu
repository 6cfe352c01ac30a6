// mars_query.cu -- query context and the query pipeline
// (create_query_context / query_memory_fast / query_memory of
// include/memory_cuda.cuh:113-194, src/memory_cuda.cu:651-1158).
//
// One query is: [copy query + per-query descriptor] -> fused scan + top-K
// (one kernel) -> one BFS kernel per hop -> finalize + top-K of the visited
// set (one kernel) -> [copy K results back].  No pass over N other than the
// scan itself: no score array, no N-sized memset, no compaction scan.  The
// host-facing call replays the whole sequence as one CUDA graph.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstring>
#include <string>

#include "mars_b200.h"
#include "mars_internal.h"
#include "mars_kernels.cuh"

using namespace mars;

namespace {

constexpr int kTickets = 8;   // scan, hop, finalize, merge, spare
constexpr int kMultiMax = 256; // queries per launch of the multi-query scan
constexpr uint32_t kMaxEpoch = (1u << 28) - 1;

StoreView make_view(const mars_store* s) {
    StoreView v{};
    v.E = s->d_E;
    v.ts = s->d_ts;
    v.imp = s->d_imp;
    v.mod = s->d_mod;
    v.d_n = s->d_n;
    v.pitch4 = s->pitch / 4;
    v.nc = (s->dim + 3) / 4;
    v.row_offsets = s->csr_n > 0 ? s->d_row_offsets : nullptr;
    v.col_indices = s->d_col_indices;
    v.csr_n = s->csr_n;
    v.extra = s->edge_slack > 0 ? s->d_extra : nullptr;
    v.extra_cnt = s->d_extra_cnt;
    v.slack = s->edge_slack;
    return v;
}

int check_store_ctx(const mars_store* s, const mars_query_ctx* c, const char* fn) {
    if (s == nullptr || c == nullptr) return fail(MARS_ERR_INVALID, std::string(fn) + ": NULL store or context");
    if (s->device != c->device) return fail(MARS_ERR_INVALID, std::string(fn) + ": store and context on different devices");
    if (s->dim != c->dim) return fail(MARS_ERR_INVALID, std::string(fn) + ": store and context dimensions differ");
    if (s->n > c->max_nodes)
        return fail(MARS_ERR_CAPACITY, std::string(fn) + ": store has " + std::to_string(s->n) +
                                           " rows, context was created for " + std::to_string(c->max_nodes));
    return MARS_OK;
}

int check_cfg(const mars_query_ctx* c, int K, int hops, const char* fn) {
    if (K <= 0 || K > c->max_k)
        return fail(MARS_ERR_INVALID, std::string(fn) + ": top_k must be in [1, " + std::to_string(c->max_k) + "]");
    if (hops < 0 || hops > MARS_MAX_BFS_HOPS)
        return fail(MARS_ERR_INVALID, std::string(fn) + ": bfs_max_hops must be in [0, 14]");
    return MARS_OK;
}

int kpl_class(int K) { return K <= 32 ? 32 : (K <= 64 ? 64 : (K <= 128 ? 128 : 256)); }

uint32_t next_epoch(mars_query_ctx* c, cudaStream_t st, int* status) {
    *status = MARS_OK;
    if (c->epoch >= kMaxEpoch) {
        if (cudaMemsetAsync(c->d_stamp, 0, (size_t)c->max_nodes * 8, st) != cudaSuccess)
            *status = fail(MARS_ERR_CUDA, "epoch wrap: stamp reset failed");
        c->epoch = 0;
    }
    return ++c->epoch;
}

// Enqueue scan -> hops -> finalize.  q / dyn: device query and optional
// device descriptor (graph path).
int enqueue_pipeline(const mars_store* s, mars_query_ctx* c, const MarsQueryDesc& d,
                     const MarsQueryDesc* dyn, const float* q, cudaStream_t st, bool timing) {
    ScanArgs sa{};
    sa.s = make_view(s);
    sa.d = d;
    sa.dyn = dyn;
    sa.q = reinterpret_cast<const float4*>(q);
    sa.part_val = c->d_part_val;
    sa.part_idx = c->d_part_idx;
    sa.ticket = c->d_ticket + 0;
    sa.cursor = c->d_ticket + kTickets + 0;
    sa.out_val = c->d_seed_val;
    sa.out_idx = c->d_seed_idx;
    sa.out_cnt = c->d_seed_cnt;
    sa.stamp = c->d_stamp;
    sa.vis_ids = c->d_vis_ids;
    sa.vis_score = c->d_vis_score;
    sa.lvl = c->d_lvl;
    if (timing) MARS_CUDA_TRY(cudaEventRecord(c->ev[0], st));
    MARS_CUDA_TRY(launch_scan_topk(sa, d.K, c->scan_blocks, st));
    if (timing) MARS_CUDA_TRY(cudaEventRecord(c->ev[1], st));

    BfsArgs ba{};
    ba.s = sa.s;
    ba.d = d;
    ba.dyn = dyn;
    ba.q = sa.q;
    ba.stamp = c->d_stamp;
    ba.vis_ids = c->d_vis_ids;
    ba.vis_score = c->d_vis_score;
    ba.lvl = c->d_lvl;
    ba.ticket = c->d_ticket + 1;
    ba.results = c->d_results;
    ba.result_cnt = c->d_result_cnt;
    for (int h = 0; h < d.hops; ++h) MARS_CUDA_TRY(launch_bfs_hop(ba, h, c->bfs_blocks, st));
    ba.ticket = c->d_ticket + 2;
    MARS_CUDA_TRY(launch_bfs_finalize(ba, d.hops, d.K, c->bfs_blocks, st));
    if (timing) MARS_CUDA_TRY(cudaEventRecord(c->ev[2], st));
    return MARS_OK;
}

MarsQueryDesc make_desc(const mars_retrieval_config* cfg, float t_q, uint32_t epoch) {
    MarsQueryDesc d{};
    d.t_q = t_q;
    d.lambda = cfg->time_decay_lambda;
    d.hop_decay = cfg->bfs_score_decay;
    d.filter = cfg->modality_filter;
    d.use_imp = cfg->use_importance;
    d.K = cfg->top_k;
    d.hops = cfg->bfs_max_hops;
    d.epoch = epoch;
    d.row_offset = 0;
    return d;
}

uint64_t graph_key(const mars_store* s, const mars_retrieval_config* cfg) {
    uint64_t h = 1469598103934665603ull;
    auto mix = [&](uint64_t v) { h = (h ^ v) * 1099511628211ull; };
    mix((uint64_t)(uintptr_t)s);
    mix((uint64_t)(uintptr_t)s->d_E);
    mix((uint64_t)(uintptr_t)s->d_row_offsets);
    mix((uint64_t)(uintptr_t)s->d_col_indices);
    mix((uint64_t)s->csr_n);
    mix((uint64_t)cfg->top_k);
    mix((uint64_t)cfg->bfs_max_hops);
    mix((uint64_t)(uint32_t)cfg->modality_filter);
    mix((uint64_t)cfg->use_importance);
    uint32_t lb, db;
    std::memcpy(&lb, &cfg->time_decay_lambda, 4);
    std::memcpy(&db, &cfg->bfs_score_decay, 4);
    mix(lb);
    mix(db);
    return h | 1ull;   // never 0 (0 = no graph)
}

constexpr int kFusedMaxK = 64;
constexpr int kFusedTicket = 4;
constexpr int32_t kCountPending = -2;
constexpr int kPollMs = 200;

// One query as a single kernel launch (mars_fastq.cu).  *done = 0 when the
// kernel reported that the BFS outgrew its last CTA (nothing written to out).
int query_single_launch(const mars_store* s, mars_query_ctx* c, const float* query, float t_q,
                        uint32_t epoch, const mars_retrieval_config* cfg, mars_query_result* out,
                        int32_t* n_out, mars_retrieval_stats* stats, int* done) {
    *done = 0;
    cudaStream_t st = c->stream;
    FusedQueryArgs p{};
    ScanArgs& a = p.a;
    a.s = make_view(s);
    a.d = make_desc(cfg, t_q, epoch);
    a.dyn = nullptr;
    a.part_val = c->d_part_val;
    a.part_idx = c->d_part_idx;
    a.ticket = c->d_ticket + kFusedTicket;
    a.cursor = c->d_ticket + kTickets + kFusedTicket;
    a.all_scores = cfg->bfs_max_hops > 0 ? c->d_all_scores : nullptr;
    a.stamp = c->d_stamp;
    p.out = c->dm_results;
    p.out_cnt = c->dm_result_cnt;
    // the query rides in the parameter block; a device-resident query is
    // read in place when its layout allows float4 loads
    cudaPointerAttributes pa{};
    const bool on_device = cudaPointerGetAttributes(&pa, query) == cudaSuccess &&
                           pa.type == cudaMemoryTypeDevice;
    (void)cudaGetLastError();
    if (on_device) {
        if ((s->dim & 3) != 0 || (reinterpret_cast<uintptr_t>(query) & 15u) != 0) {
            MARS_CUDA_TRY(cudaMemcpy(p.qbuf, query, (size_t)s->dim * sizeof(float), cudaMemcpyDeviceToHost));
        } else {
            a.q = reinterpret_cast<const float4*>(query);
        }
    } else {
        std::memcpy(p.qbuf, query, (size_t)s->dim * sizeof(float));
    }
    volatile int32_t* flag = c->h_result_cnt;
    flag[0] = kCountPending;
    if (stats) MARS_CUDA_TRY(cudaEventRecord(c->ev[0], st));
    MARS_CUDA_TRY(launch_query_fused(p, c->scan_blocks, st));
    if (stats) {
        MARS_CUDA_TRY(cudaEventRecord(c->ev[2], st));
        MARS_CUDA_TRY(cudaStreamSynchronize(st));
    } else {
        // the kernel writes the count last (after a system-scope fence), so
        // the results can be taken as soon as it changes, without waiting
        // for the kernel to retire; a bounded spin, then the stream's own
        // synchronisation (which also reports any launch failure)
        const auto t0 = std::chrono::steady_clock::now();
        for (uint32_t i = 0; flag[0] == kCountPending; ++i) {
            if ((i & 1023u) == 1023u &&
                std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(kPollMs)) break;
        }
        if (flag[0] == kCountPending) MARS_CUDA_TRY(cudaStreamSynchronize(st));
        std::atomic_thread_fence(std::memory_order_acquire);
    }
    const int32_t got = flag[0];
    if (got == kCountPending) return fail(MARS_ERR_DEVICE, "mars_query: the query kernel did not report");
    if (got < 0) return MARS_OK;
    const int32_t cnt = std::min(got, cfg->top_k);
    std::memcpy(out, c->h_results, (size_t)cnt * sizeof(mars_query_result));
    *n_out = cnt;
    if (stats) {
        float ms = 0.f;
        cudaEventElapsedTime(&ms, c->ev[0], c->ev[2]);
        stats->gpu_ms_similarity = ms;   // one kernel: scan, selection and BFS together
        stats->gpu_ms_topk = 0.f;
        stats->gpu_ms_rerank = 0.f;
        stats->gpu_ms_bfs = 0.f;
        stats->gpu_ms_total = ms;
        stats->nodes_scanned = s->n;
        stats->bfs_waves = cfg->bfs_max_hops;
        stats->nodes_visited = flag[1];
    }
    ++c->fused_queries;
    *done = 1;
    return MARS_OK;
}

}  // namespace

extern "C" {

int mars_query_ctx_create(int32_t device, int32_t max_nodes, int32_t dim, int32_t max_k,
                          mars_query_ctx** out) {
    if (out == nullptr) return fail(MARS_ERR_INVALID, "mars_query_ctx_create: out is NULL");
    *out = nullptr;
    if (max_nodes < 0 || dim <= 0 || dim > 1024 || max_k <= 0)
        return fail(MARS_ERR_INVALID, "mars_query_ctx_create: need max_nodes >= 0, 0 < dim <= 1024, max_k > 0");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev)
        return fail(MARS_ERR_NO_DEVICE, "mars_query_ctx_create: no such CUDA device");
    MarsDeviceGuard g(device);
    if (!g.ok) return fail(MARS_ERR_CUDA, "mars_query_ctx_create: cudaSetDevice failed");
    cudaDeviceProp prop;
    MARS_CUDA_TRY(cudaGetDeviceProperties(&prop, device));
    if (prop.major < 10)
        return fail(MARS_ERR_NO_DEVICE, "mars_query_ctx_create: this library is built for sm_100a (B200)");

    mars_query_ctx* c = new mars_query_ctx();
    c->device = device;
    c->max_nodes = max_nodes;
    c->dim = dim;
    c->pitch = (dim + 3) & ~3;
    c->max_k = std::min(max_k, (int32_t)MARS_MAX_TOP_K);
    c->num_sms = prop.multiProcessorCount;
    const int nc = (dim + 3) / 4;
    c->scan_blocks = c->num_sms * scan_blocks_per_sm(nc, kpl_class(c->max_k));
    c->bfs_blocks = c->num_sms * 2;
    const size_t nmax = (size_t)std::max(max_nodes, 1);
    int rc = MARS_OK;
    auto T = [&](cudaError_t e, const char* what) {
        if (e == cudaSuccess) return;
        if (rc == MARS_OK) rc = cuda_fail(e, what, __FILE__, __LINE__);   // records the first failure
        else (void)cudaGetLastError();                                 // later ones only clear the state
    };
    T(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking), "stream");
    for (int i = 0; i < 5; ++i) T(cudaEventCreate(&c->ev[i]), "event");
    c->desc_bytes = kDescQueryOffset + (size_t)c->pitch * sizeof(float);
    T(cudaMallocHost(&c->h_desc, c->desc_bytes), "pinned desc");
    T(cudaMalloc(&c->d_desc, c->desc_bytes), "desc");
    T(cudaMalloc(&c->d_part_val, (size_t)c->scan_blocks * MARS_MAX_TOP_K * sizeof(float)), "partials");
    T(cudaMalloc(&c->d_part_idx, (size_t)c->scan_blocks * MARS_MAX_TOP_K * sizeof(int32_t)), "partials");
    // [0, kTickets) completion tickets, [kTickets, 2 kTickets) row counters
    T(cudaMalloc(&c->d_ticket, 2 * kTickets * sizeof(unsigned int)), "tickets");
    T(cudaMalloc(&c->d_multi, 2 * kMultiMax * sizeof(unsigned int)), "multi-query tickets");
    T(cudaMalloc(&c->d_stamp, nmax * sizeof(unsigned long long)), "stamps");
    T(cudaMalloc(&c->d_vis_ids, nmax * sizeof(int32_t)), "visited");
    T(cudaMalloc(&c->d_vis_score, nmax * sizeof(float)), "visited");
    T(cudaMalloc(&c->d_lvl, 32 * sizeof(int32_t)), "levels");
    T(cudaMalloc(&c->d_seed_val, MARS_MAX_TOP_K * sizeof(float)), "seeds");
    T(cudaMalloc(&c->d_seed_idx, MARS_MAX_TOP_K * sizeof(int32_t)), "seeds");
    T(cudaMalloc(&c->d_seed_cnt, sizeof(int32_t)), "seeds");
    T(cudaMalloc(&c->d_results, MARS_MAX_TOP_K * sizeof(mars_query_result)), "results");
    T(cudaMalloc(&c->d_result_cnt, 2 * sizeof(int32_t)), "results");
    T(cudaMalloc(&c->d_all_scores, nmax * sizeof(float)), "row scores");
    // results land in mapped pinned memory: the single-launch path writes
    // them from the kernel, the pipeline copies them there
    T(cudaHostAlloc(&c->h_results, MARS_MAX_TOP_K * sizeof(mars_query_result), cudaHostAllocMapped),
      "pinned results");
    T(cudaHostAlloc(&c->h_result_cnt, 2 * sizeof(int32_t), cudaHostAllocMapped), "pinned results");
    if (rc == MARS_OK) {
        T(cudaHostGetDevicePointer(reinterpret_cast<void**>(&c->dm_results), c->h_results, 0), "mapped results");
        T(cudaHostGetDevicePointer(reinterpret_cast<void**>(&c->dm_result_cnt), c->h_result_cnt, 0),
          "mapped results");
    }
    if (rc == MARS_OK) {
        T(cudaMemsetAsync(c->d_ticket, 0, 2 * kTickets * sizeof(unsigned int), c->stream), "memset");
        T(cudaMemsetAsync(c->d_multi, 0, 2 * kMultiMax * sizeof(unsigned int), c->stream), "memset");
        T(cudaMemsetAsync(c->d_stamp, 0, nmax * sizeof(unsigned long long), c->stream), "memset");
        T(cudaMemsetAsync(c->d_desc, 0, c->desc_bytes, c->stream), "memset");
        std::memset(c->h_desc, 0, c->desc_bytes);
        T(cudaStreamSynchronize(c->stream), "init");
    }
    if (rc != MARS_OK) {
        mars_query_ctx_destroy(c);
        return rc;
    }
    *out = c;
    return MARS_OK;
}

int mars_query_ctx_destroy(mars_query_ctx* c) {
    if (c == nullptr) return MARS_OK;
    MarsDeviceGuard g(c->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    if (c->graph) cudaGraphExecDestroy(c->graph);
    cudaFree(c->d_desc);
    cudaFreeHost(c->h_desc);
    cudaFree(c->d_part_val);
    cudaFree(c->d_part_idx);
    cudaFree(c->d_ticket);
    cudaFree(c->d_multi);
    cudaFree(c->d_f16_ticket);
    cudaFree(c->d_f16_cnt);
    cudaFree(c->d_f16_overflow);
    cudaFree(c->d_f16_cand);
    cudaFreeHost(c->h_f16_overflow);
    cudaFree(c->d_f16_qout);
    cudaFreeHost(c->h_f16_qout);
    cudaFree(c->d_stamp);
    cudaFree(c->d_vis_ids);
    cudaFree(c->d_vis_score);
    cudaFree(c->d_lvl);
    cudaFree(c->d_seed_val);
    cudaFree(c->d_seed_idx);
    cudaFree(c->d_seed_cnt);
    cudaFree(c->d_results);
    cudaFree(c->d_result_cnt);
    cudaFree(c->d_all_scores);
    cudaFreeHost(c->h_results);
    cudaFreeHost(c->h_result_cnt);
    for (int i = 0; i < 5; ++i)
        if (c->ev[i]) cudaEventDestroy(c->ev[i]);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
    return MARS_OK;
}

void* mars_query_ctx_stream(mars_query_ctx* c) { return c ? (void*)c->stream : nullptr; }

int mars_query_ctx_use_graph(mars_query_ctx* c, int32_t enable) {
    if (c == nullptr) return fail(MARS_ERR_INVALID, "mars_query_ctx_use_graph: NULL context");
    c->use_graph = enable != 0;
    return MARS_OK;
}

int mars_query_ctx_use_fused(mars_query_ctx* c, int32_t enable) {
    if (c == nullptr) return fail(MARS_ERR_INVALID, "mars_query_ctx_use_fused: NULL context");
    c->use_fused = enable != 0;
    return MARS_OK;
}

int mars_query_ctx_path_counts(const mars_query_ctx* c, uint64_t* fused, uint64_t* reruns) {
    if (c == nullptr) return fail(MARS_ERR_INVALID, "mars_query_ctx_path_counts: NULL context");
    if (fused) *fused = c->fused_queries;
    if (reruns) *reruns = c->fused_reruns;
    return MARS_OK;
}

int mars_query(const mars_store* s, mars_query_ctx* c, const float* query, float t_q,
               const mars_retrieval_config* cfg, mars_query_result* out, int32_t* n_out,
               mars_retrieval_stats* stats) {
    MARS_TRY(check_store_ctx(s, c, "mars_query"));
    if (query == nullptr || cfg == nullptr || out == nullptr || n_out == nullptr)
        return fail(MARS_ERR_INVALID, "mars_query: NULL argument");
    MARS_TRY(check_cfg(c, cfg->top_k, cfg->bfs_max_hops, "mars_query"));
    *n_out = 0;
    MarsDeviceGuard g(c->device);
    cudaStream_t st = c->stream;
    MARS_CUDA_TRY(cudaStreamWaitEvent(st, s->written, 0));
    if (s->n == 0) {
        if (stats) *stats = mars_retrieval_stats{};
        return MARS_OK;
    }
    int rc = MARS_OK;
    uint32_t epoch = next_epoch(c, st, &rc);
    MARS_TRY(rc);

    if (c->use_fused && cfg->bfs_max_hops == 0 && s->n >= kF16QueryRows && cfg->top_k <= 64 &&
        (s->dim & 3) == 0) {
        // a hop-free query over a large store: streaming the fp16 copy halves
        // the bytes, with the same results
        int done = 0;
        MARS_TRY(query_f16(s, c, query, t_q, cfg, out, n_out, stats, &done));
        if (done) return MARS_OK;
    }
    if (c->use_fused && cfg->top_k <= kFusedMaxK && (s->dim + 3) / 4 <= kFusedMaxChunks) {
        int done = 0;
        MARS_TRY(query_single_launch(s, c, query, t_q, epoch, cfg, out, n_out, stats, &done));
        if (done) return MARS_OK;
        // the BFS outgrew the last CTA: answer with the multi-kernel pipeline
        ++c->fused_reruns;
        epoch = next_epoch(c, st, &rc);
        MARS_TRY(rc);
    }

    // stage descriptor + query in pinned memory (the previous query has
    // completed: this call is synchronous)
    MarsQueryDesc d = make_desc(cfg, t_q, epoch);
    std::memcpy(c->h_desc, &d, sizeof(d));
    MARS_CUDA_TRY(cudaMemcpy(static_cast<char*>(c->h_desc) + kDescQueryOffset, query,
                             (size_t)s->dim * sizeof(float), cudaMemcpyDefault));
    const auto* dyn = static_cast<const MarsQueryDesc*>(c->d_desc);
    const float* dq = reinterpret_cast<const float*>(static_cast<const char*>(c->d_desc) + kDescQueryOffset);
    const size_t res_bytes = (size_t)cfg->top_k * sizeof(mars_query_result);

    if (c->use_graph && stats == nullptr) {
        const uint64_t key = graph_key(s, cfg);
        if (c->graph == nullptr || c->graph_key != key) {
            if (c->graph) { cudaGraphExecDestroy(c->graph); c->graph = nullptr; c->graph_key = 0; }
            cudaGraph_t gr = nullptr;
            MARS_CUDA_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
            int crc = MARS_OK;
            if (cudaMemcpyAsync(c->d_desc, c->h_desc, c->desc_bytes, cudaMemcpyHostToDevice, st) != cudaSuccess)
                crc = fail(MARS_ERR_CUDA, "mars_query: capture of descriptor copy failed");
            if (crc == MARS_OK) crc = enqueue_pipeline(s, c, d, dyn, dq, st, false);
            if (crc == MARS_OK &&
                (cudaMemcpyAsync(c->h_results, c->d_results, res_bytes, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
                 cudaMemcpyAsync(c->h_result_cnt, c->d_result_cnt, 2 * sizeof(int32_t),
                                 cudaMemcpyDeviceToHost, st) != cudaSuccess))
                crc = fail(MARS_ERR_CUDA, "mars_query: capture of result copy failed");
            const cudaError_t ce = cudaStreamEndCapture(st, &gr);
            if (crc != MARS_OK) { if (gr) cudaGraphDestroy(gr); return crc; }
            if (ce != cudaSuccess) return cuda_fail(ce, "cudaStreamEndCapture", __FILE__, __LINE__);
            const cudaError_t ie = cudaGraphInstantiate(&c->graph, gr, 0);
            cudaGraphDestroy(gr);
            if (ie != cudaSuccess) { c->graph = nullptr; return cuda_fail(ie, "cudaGraphInstantiate", __FILE__, __LINE__); }
            c->graph_key = key;
        }
        MARS_CUDA_TRY(cudaGraphLaunch(c->graph, st));
        MARS_CUDA_TRY(cudaStreamSynchronize(st));
    } else {
        MARS_CUDA_TRY(cudaMemcpyAsync(c->d_desc, c->h_desc, c->desc_bytes, cudaMemcpyHostToDevice, st));
        MARS_TRY(enqueue_pipeline(s, c, d, dyn, dq, st, stats != nullptr));
        MARS_CUDA_TRY(cudaMemcpyAsync(c->h_results, c->d_results, res_bytes, cudaMemcpyDeviceToHost, st));
        MARS_CUDA_TRY(cudaMemcpyAsync(c->h_result_cnt, c->d_result_cnt, 2 * sizeof(int32_t),
                                      cudaMemcpyDeviceToHost, st));
        MARS_CUDA_TRY(cudaStreamSynchronize(st));
        if (stats) {
            float a = 0.f, b = 0.f;
            cudaEventElapsedTime(&a, c->ev[0], c->ev[1]);
            cudaEventElapsedTime(&b, c->ev[1], c->ev[2]);
            stats->gpu_ms_similarity = a;
            stats->gpu_ms_topk = 0.f;
            stats->gpu_ms_rerank = 0.f;
            stats->gpu_ms_bfs = b;
            stats->gpu_ms_total = a + b;
        }
    }
    const int32_t cnt = std::min(c->h_result_cnt[0], cfg->top_k);
    std::memcpy(out, c->h_results, (size_t)cnt * sizeof(mars_query_result));
    *n_out = cnt;
    if (stats) {
        stats->nodes_scanned = s->n;
        stats->bfs_waves = cfg->bfs_max_hops;
        stats->nodes_visited = c->h_result_cnt[1];
    }
    return MARS_OK;
}

int mars_query_device(const mars_store* s, mars_query_ctx* c, const float* d_query, float t_q,
                      const mars_retrieval_config* cfg, mars_query_result* d_out, int32_t* d_count,
                      void* stream) {
    MARS_TRY(check_store_ctx(s, c, "mars_query_device"));
    if (d_query == nullptr || cfg == nullptr || d_out == nullptr || d_count == nullptr)
        return fail(MARS_ERR_INVALID, "mars_query_device: NULL argument");
    if ((reinterpret_cast<uintptr_t>(d_query) & 15u) != 0)
        return fail(MARS_ERR_INVALID, "mars_query_device: d_query must be 16-byte aligned");
    if ((s->dim & 3) != 0)
        return fail(MARS_ERR_UNSUPPORTED, "mars_query_device: device queries need dim % 4 == 0 (use mars_query)");
    MARS_TRY(check_cfg(c, cfg->top_k, cfg->bfs_max_hops, "mars_query_device"));
    MarsDeviceGuard g(c->device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    MARS_CUDA_TRY(cudaStreamWaitEvent(st, s->written, 0));
    int rc = MARS_OK;
    const uint32_t epoch = next_epoch(c, st, &rc);
    MARS_TRY(rc);
    const MarsQueryDesc d = make_desc(cfg, t_q, epoch);
    MARS_TRY(enqueue_pipeline(s, c, d, nullptr, d_query, st, false));
    MARS_CUDA_TRY(cudaMemcpyAsync(d_out, c->d_results, (size_t)cfg->top_k * sizeof(mars_query_result),
                                  cudaMemcpyDeviceToDevice, st));
    MARS_CUDA_TRY(cudaMemcpyAsync(d_count, c->d_result_cnt, sizeof(int32_t), cudaMemcpyDeviceToDevice, st));
    return MARS_OK;
}

int mars_query_once(const mars_store* s, const float* query, float t_q,
                    const mars_retrieval_config* cfg, mars_query_result* out, int32_t* n_out,
                    mars_retrieval_stats* stats) {
    if (s == nullptr || cfg == nullptr) return fail(MARS_ERR_INVALID, "mars_query_once: NULL argument");
    mars_query_ctx* c = nullptr;
    MARS_TRY(mars_query_ctx_create(s->device, std::max(s->n, 1), s->dim, std::max(cfg->top_k, 1), &c));
    c->use_graph = false;
    const int rc = mars_query(s, c, query, t_q, cfg, out, n_out, stats);
    mars_query_ctx_destroy(c);
    return rc;
}

int mars_scan_topk(const mars_store* s, mars_query_ctx* c, const float* d_query, float t_q, float lambda,
                   int32_t modality_filter, int32_t use_importance, int32_t K, int32_t row_offset,
                   int32_t* d_ids, float* d_vals, int32_t* d_count, void* stream) {
    return mars::scan_topk_excluding(s, c, d_query, t_q, lambda, modality_filter, use_importance, K,
                                     row_offset, -1, d_ids, d_vals, d_count, stream);
}

}  // extern "C"

int mars::query_ctx_f16_buffers(mars_query_ctx* c) {
    if (c->d_f16_cand != nullptr) return MARS_OK;
    MARS_CUDA_TRY(cudaMalloc(&c->d_f16_ticket, kF16Slots * sizeof(unsigned int)));
    MARS_CUDA_TRY(cudaMalloc(&c->d_f16_cnt, kF16Slots * sizeof(int32_t)));
    MARS_CUDA_TRY(cudaMalloc(&c->d_f16_overflow, 3 * kF16Slots * sizeof(int32_t)));
    MARS_CUDA_TRY(cudaMallocHost(&c->h_f16_overflow, 3 * kF16Slots * sizeof(int32_t)));
    MARS_CUDA_TRY(cudaMemset(c->d_f16_ticket, 0, kF16Slots * sizeof(unsigned int)));
    MARS_CUDA_TRY(cudaMemset(c->d_f16_cnt, 0, kF16Slots * sizeof(int32_t)));
    MARS_CUDA_TRY(cudaMemset(c->d_f16_overflow, 0, 3 * kF16Slots * sizeof(int32_t)));
    MARS_CUDA_TRY(cudaMalloc(&c->d_f16_cand, (size_t)kF16Slots * kF16CandCap * sizeof(unsigned long long)));
    MARS_CUDA_TRY(cudaMalloc(&c->d_f16_qout, (4 + 3 * (size_t)c->max_k) * sizeof(int32_t)));
    MARS_CUDA_TRY(cudaMallocHost(&c->h_f16_qout, (4 + 3 * (size_t)c->max_k) * sizeof(int32_t)));
    return MARS_OK;
}

extern "C" int mars_scan_topk_multi(const mars_store* s, mars_query_ctx* c, const float* d_queries,
                                    int32_t query_pitch, int32_t nq, float t_q, float lambda,
                                    int32_t modality_filter, int32_t use_importance, int32_t K,
                                    int32_t row_offset, int32_t* d_ids, float* d_vals, int32_t* d_counts,
                                    void* stream) {
    MARS_TRY(check_store_ctx(s, c, "mars_scan_topk_multi"));
    if (d_queries == nullptr || d_ids == nullptr || d_vals == nullptr || nq < 0)
        return fail(MARS_ERR_INVALID, "mars_scan_topk_multi: NULL argument or nq < 0");
    if ((reinterpret_cast<uintptr_t>(d_queries) & 15u) != 0 || query_pitch < s->pitch || (query_pitch & 3) != 0)
        return fail(MARS_ERR_INVALID, "mars_scan_topk_multi: queries must be 16-byte aligned rows, pitch >= the store's");
    if ((s->dim & 3) != 0)
        return fail(MARS_ERR_UNSUPPORTED, "mars_scan_topk_multi: device queries need dim % 4 == 0");
    MARS_TRY(check_cfg(c, K, 0, "mars_scan_topk_multi"));
    if (nq == 0) return MARS_OK;
    MarsDeviceGuard g(c->device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    MARS_CUDA_TRY(cudaStreamWaitEvent(st, s->written, 0));
    ScanArgs sa{};
    sa.s = make_view(s);
    sa.d.t_q = t_q;
    sa.d.lambda = lambda;
    sa.d.filter = modality_filter;
    sa.d.use_imp = use_importance;
    sa.d.K = K;
    sa.d.row_offset = row_offset;
    sa.dyn = nullptr;
    sa.part_val = c->d_part_val;
    sa.part_idx = c->d_part_idx;
    sa.ticket = c->d_multi;
    sa.cursor = c->d_multi + kMultiMax;
    // the partial buffers hold MARS_MAX_TOP_K entries per CTA: that many
    // entries' worth of queries per launch
    const int32_t per = std::max(1, std::min(kMultiMax, (int)MARS_MAX_TOP_K / K));
    for (int32_t q0 = 0; q0 < nq; q0 += per) {
        const int32_t n = std::min(per, nq - q0);
        sa.out_val = d_vals + (size_t)q0 * K;
        sa.out_idx = d_ids + (size_t)q0 * K;
        sa.out_cnt = d_counts ? d_counts + q0 : nullptr;
        // one wave for the whole launch: the queries' CTAs are all resident
        // and walk the same rows in step, so each row comes from HBM about
        // once and the other queries read it from L2
        const int gx = std::max(1, c->scan_blocks / n);
        MARS_CUDA_TRY(launch_scan_multi(sa, d_queries + (size_t)q0 * query_pitch, query_pitch, n, gx, st));
    }
    return MARS_OK;
}

int mars::scan_topk_excluding(const mars_store* s, mars_query_ctx* c, const float* d_query, float t_q,
                              float lambda, int32_t modality_filter, int32_t use_importance, int32_t K,
                              int32_t row_offset, int32_t exclude_row, int32_t* d_ids, float* d_vals,
                              int32_t* d_count, void* stream) {
    MARS_TRY(check_store_ctx(s, c, "mars_scan_topk"));
    if (d_query == nullptr || d_ids == nullptr || d_vals == nullptr)
        return fail(MARS_ERR_INVALID, "mars_scan_topk: NULL argument");
    if ((reinterpret_cast<uintptr_t>(d_query) & 15u) != 0)
        return fail(MARS_ERR_INVALID, "mars_scan_topk: d_query must be 16-byte aligned");
    if ((s->dim & 3) != 0)
        return fail(MARS_ERR_UNSUPPORTED, "mars_scan_topk: device queries need dim % 4 == 0");
    MARS_TRY(check_cfg(c, K, 0, "mars_scan_topk"));
    MarsDeviceGuard g(c->device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    MARS_CUDA_TRY(cudaStreamWaitEvent(st, s->written, 0));
    ScanArgs sa{};
    sa.s = make_view(s);
    sa.d.t_q = t_q;
    sa.d.lambda = lambda;
    sa.d.filter = modality_filter;
    sa.d.use_imp = use_importance;
    sa.d.K = K;
    sa.d.row_offset = row_offset;
    sa.d.exclude_plus1 = exclude_row + 1;
    sa.dyn = nullptr;
    sa.q = reinterpret_cast<const float4*>(d_query);
    sa.part_val = c->d_part_val;
    sa.part_idx = c->d_part_idx;
    sa.ticket = c->d_ticket + 3;
    sa.cursor = c->d_ticket + kTickets + 3;
    sa.out_val = d_vals;
    sa.out_idx = d_ids;
    sa.out_cnt = d_count ? d_count : c->d_seed_cnt;
    MARS_CUDA_TRY(launch_scan_topk(sa, K, c->scan_blocks, st));
    return MARS_OK;
}

extern "C" {

int mars_topk_merge(mars_query_ctx* c, const int32_t* d_ids_in, const float* d_vals_in, int32_t n_lists,
                    int32_t K, int32_t* d_ids_out, float* d_vals_out, int32_t* d_count, void* stream) {
    return mars_topk_merge_batch(c, d_ids_in, d_vals_in, n_lists, K, 1, d_ids_out, d_vals_out, d_count,
                                 stream);
}

int mars_topk_merge_batch(mars_query_ctx* c, const int32_t* d_ids_in, const float* d_vals_in,
                          int32_t n_lists, int32_t K, int32_t Q, int32_t* d_ids_out, float* d_vals_out,
                          int32_t* d_counts, void* stream) {
    if (c == nullptr || d_ids_in == nullptr || d_vals_in == nullptr || d_ids_out == nullptr ||
        d_vals_out == nullptr || n_lists < 0 || Q < 0)
        return fail(MARS_ERR_INVALID, "mars_topk_merge: bad arguments");
    if (K <= 0 || K > MARS_MAX_TOP_K) return fail(MARS_ERR_INVALID, "mars_topk_merge: K out of range");
    if (Q == 0) return MARS_OK;
    MarsDeviceGuard g(c->device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    MARS_CUDA_TRY(launch_topk_merge(d_ids_in, d_vals_in, n_lists, K, Q, d_ids_out, d_vals_out, d_counts, st));
    return MARS_OK;
}

int mars_novelty(const mars_store* s, mars_query_ctx* c, const float* d_query, float* d_max,
                 void* stream) {
    MARS_TRY(check_store_ctx(s, c, "mars_novelty"));
    if (d_query == nullptr || d_max == nullptr) return fail(MARS_ERR_INVALID, "mars_novelty: NULL argument");
    if ((reinterpret_cast<uintptr_t>(d_query) & 15u) != 0 || (s->dim & 3) != 0)
        return fail(MARS_ERR_INVALID, "mars_novelty: aligned query and dim % 4 == 0 required");
    MarsDeviceGuard g(c->device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    MARS_CUDA_TRY(cudaStreamWaitEvent(st, s->written, 0));
    ScanArgs sa{};
    sa.s = make_view(s);
    sa.d.t_q = 0.0f;
    sa.d.lambda = 0.0f;     // weight exactly 1: the score is the dot product
    sa.d.filter = -1;
    sa.d.use_imp = 0;
    sa.d.K = 1;
    sa.q = reinterpret_cast<const float4*>(d_query);
    sa.part_val = c->d_part_val;
    sa.part_idx = c->d_part_idx;
    sa.ticket = c->d_ticket + 5;
    sa.cursor = c->d_ticket + kTickets + 5;
    sa.out_val = d_max;
    sa.out_idx = c->d_seed_idx;
    sa.out_cnt = c->d_seed_cnt;
    MARS_CUDA_TRY(launch_scan_topk(sa, 1, c->scan_blocks, st));
    return MARS_OK;
}

int mars_debug_fused_scores(const mars_store* s, mars_query_ctx* c, const float* d_query, float t_q,
                            float lambda, int32_t modality_filter, int32_t use_importance, float* d_out,
                            void* stream) {
    MARS_TRY(check_store_ctx(s, c, "mars_debug_fused_scores"));
    if (d_query == nullptr || d_out == nullptr) return fail(MARS_ERR_INVALID, "mars_debug_fused_scores: NULL argument");
    if ((reinterpret_cast<uintptr_t>(d_query) & 15u) != 0 || (s->dim & 3) != 0)
        return fail(MARS_ERR_INVALID, "mars_debug_fused_scores: aligned query and dim % 4 == 0 required");
    MarsDeviceGuard g(c->device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    MARS_CUDA_TRY(cudaStreamWaitEvent(st, s->written, 0));
    ScanArgs sa{};
    sa.s = make_view(s);
    sa.d.t_q = t_q;
    sa.d.lambda = lambda;
    sa.d.filter = modality_filter;
    sa.d.use_imp = use_importance;
    sa.d.K = 1;
    sa.q = reinterpret_cast<const float4*>(d_query);
    sa.part_val = c->d_part_val;
    sa.part_idx = c->d_part_idx;
    sa.ticket = c->d_ticket + 4;
    sa.cursor = c->d_ticket + kTickets + 4;
    sa.out_val = c->d_seed_val;
    sa.out_idx = c->d_seed_idx;
    sa.out_cnt = c->d_seed_cnt;
    sa.all_scores = d_out;
    MARS_CUDA_TRY(launch_scan_topk(sa, 1, c->scan_blocks, st));
    return MARS_OK;
}

}  // extern "C"
