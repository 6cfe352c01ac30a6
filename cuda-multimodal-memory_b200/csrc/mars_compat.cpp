// mars_compat.cpp -- the reference's C++ API (include/memory_cuda.cuh) on top
// of the C ABI, so reference callers relink unchanged.
//
// DeviceMemoryGraph is a value type holding raw device pointers; the store
// that owns those arrays is found again through a registry keyed by the
// embedding pointer.  A DeviceMemoryGraph that a caller assembled by hand
// (not returned by upload_to_device) is used through a non-owning view.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <cstdlib>
#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "mars_b200.h"
#include "mars_internal.h"
#include "cmng.cuh"
#include "memory_cuda.cuh"

namespace {

struct Registry {
    std::mutex mu;
    std::unordered_map<const void*, mars_store*> stores;        // d_embeddings -> store
    std::unordered_map<const void*, mars_query_ctx*> aux_ctx;   // store -> novelty context
    std::unordered_map<const void*, float*> dense;              // store -> dense N x D copy (D % 4 != 0)
};

Registry& reg() {
    static Registry r;
    return r;
}

[[noreturn]] void die(int status, const char* where) {
    const std::string msg = std::string(where) + ": " + mars_status_string(status) + " - " + mars_last_error();
    const char* t = std::getenv("MARS_COMPAT_THROW");
    if (t != nullptr && t[0] == '1') throw std::runtime_error(msg);
    std::fprintf(stderr, "MARS error %s\n", msg.c_str());
    std::exit(EXIT_FAILURE);
}

void check(int status, const char* where) {
    if (status != MARS_OK) die(status, where);
}

int current_device() {
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess) d = 0;
    return d;
}

mars_store* find_store(const DeviceMemoryGraph& dg) {
    Registry& r = reg();
    std::lock_guard<std::mutex> lk(r.mu);
    auto it = r.stores.find(dg.d_embeddings);
    return it == r.stores.end() ? nullptr : it->second;
}

// Non-owning view of a caller-assembled DeviceMemoryGraph.
mars_store* view_store(const DeviceMemoryGraph& dg) {
    if ((dg.embedding_dim & 3) != 0)
        die(MARS_ERR_UNSUPPORTED, "query on a hand-built DeviceMemoryGraph (embedding_dim % 4 != 0)");
    mars_store* s = new mars_store();
    s->device = current_device();
    s->capacity = dg.num_nodes;
    s->dim = dg.embedding_dim;
    s->pitch = dg.embedding_dim;
    s->n = dg.num_nodes;
    s->owns = false;
    s->d_E = dg.d_embeddings;
    s->d_ts = dg.d_timestamps;
    s->d_imp = dg.d_importance;
    s->d_mod = dg.d_modalities;
    s->csr_n = dg.d_row_offsets ? dg.num_nodes : 0;
    s->num_edges = dg.num_edges;
    s->d_row_offsets = dg.d_row_offsets;
    s->d_col_indices = dg.d_col_indices;
    if (cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&s->written, cudaEventDisableTiming) != cudaSuccess ||
        cudaMalloc(&s->d_n, sizeof(int32_t)) != cudaSuccess ||
        cudaMemcpy(s->d_n, &s->n, sizeof(int32_t), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaEventRecord(s->written, s->stream) != cudaSuccess)
        die(MARS_ERR_CUDA, "view of DeviceMemoryGraph");
    return s;
}

struct StoreRef {
    mars_store* s = nullptr;
    bool temp = false;
    explicit StoreRef(const DeviceMemoryGraph& dg) {
        s = find_store(dg);
        if (s == nullptr) { s = view_store(dg); temp = true; }
    }
    ~StoreRef() { if (temp) mars_store_destroy(s); }
};

mars_retrieval_config to_c(const RetrievalConfig& cfg, int32_t K) {
    mars_retrieval_config c{};
    c.top_k = K;
    c.bfs_max_hops = cfg.bfs_max_hops;
    c.time_decay_lambda = cfg.time_decay_lambda;
    c.bfs_score_decay = cfg.bfs_score_decay;
    c.modality_filter = cfg.modality_filter;
    c.use_importance = cfg.use_importance ? 1 : 0;
    return c;
}

std::vector<QueryResult> to_results(const std::vector<mars_query_result>& r, int32_t n) {
    std::vector<QueryResult> out;
    out.reserve((size_t)n);
    for (int32_t i = 0; i < n; ++i)
        out.push_back({r[i].node_id, r[i].score, r[i].modality, r[i].hops_from_seed});
    return out;
}

void fill_stats(RetrievalStats& st, const mars_retrieval_stats& m) {
    st.gpu_ms_similarity = m.gpu_ms_similarity;
    st.gpu_ms_topk = m.gpu_ms_topk;
    st.gpu_ms_bfs = m.gpu_ms_bfs;
    st.gpu_ms_rerank = m.gpu_ms_rerank;
    st.gpu_ms_total = m.gpu_ms_total;
    st.nodes_scanned = m.nodes_scanned;
    st.bfs_waves = m.bfs_waves;
}

__global__ void f32_to_f16_kernel(const float* __restrict__ in, int64_t pitch, half* __restrict__ out,
                                  int64_t n, int32_t dim) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n * dim) return;
    const int64_t r = i / dim, c = i % dim;
    out[i] = __float2half(in[r * pitch + c]);
}

// The embeddings a returned DeviceMemoryGraph / CMNGGraph points at: the
// reference's layout is dense N x D; the store keeps rows padded to a
// multiple of 4 floats for its 16-byte loads.  When D % 4 == 0 the two are
// the same memory; otherwise the caller gets a dense, read-only copy made at
// upload (the queries keep reading the store's padded rows).  The store is
// registered under the returned pointer.
float* expose_rows(mars_store* s, int32_t n, int32_t D) {
    float* rows = s->d_E;
    if ((D & 3) != 0 && n > 0) {
        CUDA_CHECK(cudaMalloc(&rows, (size_t)n * D * sizeof(float)));
        CUDA_CHECK(cudaMemcpy2D(rows, (size_t)D * sizeof(float), s->d_E, (size_t)s->pitch * sizeof(float),
                                (size_t)D * sizeof(float), (size_t)n, cudaMemcpyDeviceToDevice));
    }
    Registry& r = reg();
    std::lock_guard<std::mutex> lk(r.mu);
    r.stores[rows] = s;
    if (rows != s->d_E) r.dense[s] = rows;
    return rows;
}

}  // namespace

DeviceMemoryGraph upload_to_device(const MemoryGraph& h) {
    mars_store* s = nullptr;
    check(mars_store_create(current_device(), h.num_nodes, std::max(h.embedding_dim, 1), 0, &s),
          "upload_to_device");
    const bool has_graph = (int32_t)h.row_offsets.size() == h.num_nodes + 1;
    const int32_t ne = has_graph ? (int32_t)h.col_indices.size() : 0;
    check(mars_store_upload(s, h.num_nodes, h.embeddings.data(), h.modalities.data(), h.timestamps.data(),
                            nullptr, has_graph ? h.row_offsets.data() : nullptr,
                            has_graph ? h.col_indices.data() : nullptr, ne),
          "upload_to_device");
    DeviceMemoryGraph d;
    d.num_nodes = h.num_nodes;
    d.num_edges = h.num_edges;
    d.embedding_dim = h.embedding_dim;
    d.d_row_offsets = s->d_row_offsets;
    d.d_col_indices = s->d_col_indices;
    d.d_embeddings = expose_rows(s, h.num_nodes, h.embedding_dim);
    d.d_modalities = s->d_mod;
    d.d_timestamps = s->d_ts;
    return d;
}

void free_device(DeviceMemoryGraph& d) {
    mars_store* s = nullptr;
    mars_query_ctx* aux = nullptr;
    float* dense = nullptr;
    {
        Registry& r = reg();
        std::lock_guard<std::mutex> lk(r.mu);
        auto it = r.stores.find(d.d_embeddings);
        if (it != r.stores.end()) {
            s = it->second;
            r.stores.erase(it);
            auto jt = r.aux_ctx.find(s);
            if (jt != r.aux_ctx.end()) { aux = jt->second; r.aux_ctx.erase(jt); }
            auto kt = r.dense.find(s);
            if (kt != r.dense.end()) { dense = kt->second; r.dense.erase(kt); }
        }
    }
    mars_query_ctx_destroy(aux);
    if (dense) cudaFree(dense);
    if (d.d_embeddings_fp16) cudaFree(d.d_embeddings_fp16);
    if (d.d_edge_hits) cudaFree(d.d_edge_hits);
    mars_store_destroy(s);
    d = DeviceMemoryGraph{};
}

void upload_fp16_embeddings(DeviceMemoryGraph& dg) {
    const int64_t n = dg.num_nodes, D = dg.embedding_dim;
    if (n <= 0 || dg.d_embeddings == nullptr) return;
    StoreRef sr(dg);
    CUDA_CHECK(cudaMalloc(&dg.d_embeddings_fp16, n * D * sizeof(half)));
    const int64_t total = n * D;
    f32_to_f16_kernel<<<(unsigned)((total + 255) / 256), 256>>>(sr.s->d_E, sr.s->pitch,
                                                                dg.d_embeddings_fp16, n, (int32_t)D);
    CUDA_CHECK(cudaGetLastError());
    CUDA_CHECK(cudaDeviceSynchronize());
}

void free_fp16_embeddings(DeviceMemoryGraph& dg) {
    if (dg.d_embeddings_fp16) {
        cudaFree(dg.d_embeddings_fp16);
        dg.d_embeddings_fp16 = nullptr;
    }
}

QueryContext create_query_context(int32_t max_nodes, int32_t embedding_dim, int32_t max_k) {
    QueryContext ctx;
    mars_query_ctx* c = nullptr;
    check(mars_query_ctx_create(current_device(), max_nodes, embedding_dim, std::max(max_k, 1), &c),
          "create_query_context");
    ctx.max_nodes = max_nodes;
    ctx.embedding_dim = embedding_dim;
    ctx.max_k = c->max_k;
    ctx.stream = c->stream;
    ctx.valid = true;
    ctx.impl = c;
    return ctx;
}

void destroy_query_context(QueryContext& ctx) {
    if (!ctx.valid) return;
    mars_query_ctx_destroy(static_cast<mars_query_ctx*>(ctx.impl));
    ctx = QueryContext{};
}

std::vector<QueryResult> query_memory_fast(const DeviceMemoryGraph& dg, QueryContext& ctx,
                                           const float* h_query, float query_timestamp,
                                           const RetrievalConfig& cfg, RetrievalStats& stats) {
    if (!ctx.valid || ctx.impl == nullptr) die(MARS_ERR_INVALID, "query_memory_fast (invalid context)");
    auto* c = static_cast<mars_query_ctx*>(ctx.impl);
    StoreRef sr(dg);
    const int32_t K = std::min(cfg.top_k, ctx.max_k);
    if (K <= 0) return {};
    mars_query_ctx_use_graph(c, ctx.use_cuda_graph ? 1 : 0);
    mars_retrieval_config cc = to_c(cfg, K);
    std::vector<mars_query_result> res((size_t)K);
    int32_t n = 0;
    mars_retrieval_stats ms{};
    // stage timings are reported when the query is not replayed from a graph
    check(mars_query(sr.s, c, h_query, query_timestamp, &cc, res.data(), &n,
                     ctx.use_cuda_graph ? nullptr : &ms),
          "query_memory_fast");
    if (ctx.use_cuda_graph) {
        ms.nodes_scanned = dg.num_nodes;
        ms.bfs_waves = cfg.bfs_max_hops;
    }
    fill_stats(stats, ms);
    return to_results(res, n);
}

std::vector<QueryResult> query_memory(const DeviceMemoryGraph& dg, const float* h_query,
                                      float query_timestamp, const RetrievalConfig& cfg,
                                      RetrievalStats& stats) {
    StoreRef sr(dg);
    const int32_t K = std::min(cfg.top_k, (int32_t)MARS_MAX_TOP_K);
    if (K <= 0) return {};
    mars_retrieval_config cc = to_c(cfg, K);
    std::vector<mars_query_result> res((size_t)K);
    int32_t n = 0;
    mars_retrieval_stats ms{};
    check(mars_query_once(sr.s, h_query, query_timestamp, &cc, res.data(), &n, &ms), "query_memory");
    fill_stats(stats, ms);
    return to_results(res, n);
}

void init_importance(DeviceMemoryGraph& dg) {
    mars_store* s = find_store(dg);
    if (s == nullptr) {
        // caller-owned graph: allocate like the reference does
        if (dg.d_importance) cudaFree(dg.d_importance);
        CUDA_CHECK(cudaMalloc(&dg.d_importance, (size_t)std::max(dg.num_nodes, 1) * sizeof(float)));
        std::vector<float> ones((size_t)std::max(dg.num_nodes, 1), 1.0f);
        CUDA_CHECK(cudaMemcpy(dg.d_importance, ones.data(), ones.size() * 4, cudaMemcpyHostToDevice));
        return;
    }
    check(mars_importance_fill(s, 1.0f), "init_importance");
    dg.d_importance = s->d_imp;
}

void update_importance(DeviceMemoryGraph& dg, const int32_t* d_result_ids, int32_t n_results,
                       float boost, float decay_rate, float max_importance, cudaStream_t stream) {
    if (!dg.d_importance || dg.num_nodes <= 0) return;
    StoreRef sr(dg);
    check(mars_importance_update(sr.s, d_result_ids, d_result_ids ? n_results : 0, boost, decay_rate,
                                 max_importance, stream),
          "update_importance");
    if (sr.temp) CUDA_CHECK(cudaStreamSynchronize(stream ? stream : sr.s->stream));
}

float compute_novelty(const DeviceMemoryGraph& dg, const float* d_query, cudaStream_t stream) {
    if (dg.num_nodes <= 0) return 0.0f;
    StoreRef sr(dg);
    mars_query_ctx* c = nullptr;
    {
        Registry& r = reg();
        std::lock_guard<std::mutex> lk(r.mu);
        auto it = r.aux_ctx.find(sr.s);
        if (it != r.aux_ctx.end()) c = it->second;
    }
    if (c == nullptr || c->max_nodes < dg.num_nodes) {
        if (c) mars_query_ctx_destroy(c);
        check(mars_query_ctx_create(sr.s->device, std::max(sr.s->capacity, dg.num_nodes), dg.embedding_dim, 1, &c),
              "compute_novelty");
        if (!sr.temp) {
            Registry& r = reg();
            std::lock_guard<std::mutex> lk(r.mu);
            r.aux_ctx[sr.s] = c;
        }
    }
    float* d_max = nullptr;
    CUDA_CHECK(cudaMalloc(&d_max, sizeof(float)));
    cudaStream_t st = stream ? stream : c->stream;
    check(mars_novelty(sr.s, c, d_query, d_max, st), "compute_novelty");
    float v = 0.0f;
    CUDA_CHECK(cudaMemcpyAsync(&v, d_max, sizeof(float), cudaMemcpyDeviceToHost, st));
    CUDA_CHECK(cudaStreamSynchronize(st));
    cudaFree(d_max);
    if (sr.temp) mars_query_ctx_destroy(c);
    // the reference starts its host max at -1 (src/memory_cuda.cu:1278)
    return std::max(v, -1.0f);
}

void init_edge_hits(DeviceMemoryGraph& dg) {
    if (dg.d_edge_hits) cudaFree(dg.d_edge_hits);
    CUDA_CHECK(cudaMalloc(&dg.d_edge_hits, (size_t)std::max(dg.num_edges, 1) * sizeof(int32_t)));
    CUDA_CHECK(cudaMemset(dg.d_edge_hits, 0, (size_t)std::max(dg.num_edges, 1) * sizeof(int32_t)));
}

// The reference counts edges whose hit counter is <= min_hits and resets the
// counters (src/memory_cuda.cu:1330-1352); nothing increments the counters on
// its query path, so the count is of untouched edges.  Same contract here.
int32_t maintain_graph(DeviceMemoryGraph& dg, int32_t min_hits, int32_t window_queries,
                       cudaStream_t stream) {
    (void)window_queries;
    (void)stream;
    if (!dg.d_edge_hits || dg.num_edges <= 0) return 0;
    std::vector<int32_t> h((size_t)dg.num_edges);
    CUDA_CHECK(cudaMemcpy(h.data(), dg.d_edge_hits, h.size() * 4, cudaMemcpyDeviceToHost));
    int32_t low = 0;
    for (int32_t v : h) low += v <= min_hits ? 1 : 0;
    CUDA_CHECK(cudaMemset(dg.d_edge_hits, 0, h.size() * 4));
    return low;
}

// ===========================================================================
// include/cmng.cuh
CMNGGraph build_cmng(const float* h_embeddings, const int32_t* h_modalities, const float* h_timestamps,
                     int32_t N, int32_t D, int32_t degree, int32_t degree_cross) {
    mars_store* s = nullptr;
    check(mars_store_create(current_device(), N, std::max(D, 1), 0, &s), "build_cmng");
    check(mars_store_upload(s, N, h_embeddings, h_modalities, h_timestamps, nullptr, nullptr, nullptr, 0),
          "build_cmng");
    CMNGGraph g;
    g.N = N;
    g.D = D;
    g.degree = degree;
    g.degree_cross = degree_cross;
    CUDA_CHECK(cudaMalloc(&g.d_neighbors, (size_t)std::max(N, 1) * degree * sizeof(int32_t)));
    // the reference selects bridges for MOD_COUNT = 3 modalities (src/cmng_build.cu:234)
    check(mars_cmng_build(s, degree, degree_cross, 3, g.d_neighbors, &g.build_time_ms), "build_cmng");
    g.d_embeddings = expose_rows(s, N, D);
    g.d_modalities = s->d_mod;
    g.d_timestamps = s->d_ts;
    return g;
}

void cmng_upload_fp16(CMNGGraph& g) {
    if (g.N <= 0 || g.d_embeddings == nullptr) return;
    DeviceMemoryGraph dg;
    dg.num_nodes = g.N;
    dg.embedding_dim = g.D;
    dg.d_embeddings = g.d_embeddings;
    upload_fp16_embeddings(dg);
    g.d_embeddings_fp16 = dg.d_embeddings_fp16;
}

void free_cmng(CMNGGraph& g) {
    if (g.d_neighbors) cudaFree(g.d_neighbors);
    if (g.d_embeddings_fp16) cudaFree(g.d_embeddings_fp16);
    DeviceMemoryGraph dg;
    dg.d_embeddings = g.d_embeddings;
    free_device(dg);
    g = CMNGGraph{};
}

CMNGSearchContext create_cmng_context(int32_t D, int32_t max_beam, int32_t max_k) {
    CMNGSearchContext ctx;
    ctx.max_D = D;
    ctx.max_K = max_k;
    ctx.max_beam = max_beam;
    CUDA_CHECK(cudaMalloc(&ctx.d_result_ids, (size_t)std::max(max_k, 1) * sizeof(int32_t)));
    CUDA_CHECK(cudaMalloc(&ctx.d_result_scores, (size_t)std::max(max_k, 1) * sizeof(float)));
    CUDA_CHECK(cudaMalloc(&ctx.d_result_mods, (size_t)std::max(max_k, 1) * sizeof(int32_t)));
    CUDA_CHECK(cudaMalloc(&ctx.d_result_count, sizeof(int32_t)));
    CUDA_CHECK(cudaMalloc(&ctx.d_query, (size_t)((D + 3) & ~3) * sizeof(float)));
    CUDA_CHECK(cudaMemset(ctx.d_query, 0, (size_t)((D + 3) & ~3) * sizeof(float)));
    CUDA_CHECK(cudaMallocHost(&ctx.h_query_pinned, (size_t)std::max(D, 1) * sizeof(float)));
    CUDA_CHECK(cudaEventCreate(&ctx.e_start));
    CUDA_CHECK(cudaEventCreate(&ctx.e_end));
    CUDA_CHECK(cudaStreamCreateWithFlags(&ctx.stream, cudaStreamNonBlocking));
    ctx.valid = true;
    return ctx;
}

void destroy_cmng_context(CMNGSearchContext& ctx) {
    if (!ctx.valid) return;
    cudaStreamSynchronize(ctx.stream);
    cudaFree(ctx.d_result_ids);
    cudaFree(ctx.d_result_scores);
    cudaFree(ctx.d_result_mods);
    cudaFree(ctx.d_result_count);
    cudaFree(ctx.d_query);
    cudaFreeHost(ctx.h_query_pinned);
    cudaEventDestroy(ctx.e_start);
    cudaEventDestroy(ctx.e_end);
    cudaStreamDestroy(ctx.stream);
    ctx = CMNGSearchContext{};
}

std::vector<QueryResult> cmng_search(const CMNGGraph& g, CMNGSearchContext& ctx, const float* h_query,
                                     float query_timestamp, const CMNGSearchConfig& cfg,
                                     RetrievalStats& stats) {
    if (!ctx.valid) die(MARS_ERR_INVALID, "cmng_search (invalid context)");
    DeviceMemoryGraph dg;
    dg.num_nodes = g.N;
    dg.embedding_dim = g.D;
    dg.d_embeddings = g.d_embeddings;
    dg.d_modalities = g.d_modalities;
    dg.d_timestamps = g.d_timestamps;
    StoreRef sr(dg);
    const int32_t K = std::min(cfg.K, ctx.max_K);   // src/cmng_search.cu:355
    if (K <= 0) return {};
    std::memcpy(ctx.h_query_pinned, h_query, (size_t)g.D * sizeof(float));
    CUDA_CHECK(cudaMemcpyAsync(ctx.d_query, ctx.h_query_pinned, (size_t)g.D * sizeof(float),
                               cudaMemcpyHostToDevice, ctx.stream));
    mars_cmng_config c{};
    c.K = K;
    c.beam_width = cfg.beam_width;
    c.max_iterations = cfg.max_iterations;
    c.num_parents = cfg.num_parents;
    c.time_decay_lambda = cfg.time_decay_lambda;
    c.modality_filter = cfg.modality_filter;
    c.use_fp16 = cfg.use_fp16 ? 1 : 0;
    CUDA_CHECK(cudaEventRecord(ctx.e_start, ctx.stream));
    check(mars_cmng_search_batch(sr.s, g.d_neighbors, g.degree, ctx.d_query, (g.D + 3) & ~3, 1, query_timestamp,
                                 &c, ctx.d_result_ids, ctx.d_result_scores, ctx.d_result_mods,
                                 ctx.d_result_count, nullptr, nullptr, ctx.stream),
          "cmng_search");
    CUDA_CHECK(cudaEventRecord(ctx.e_end, ctx.stream));
    int32_t count = 0;
    CUDA_CHECK(cudaMemcpyAsync(&count, ctx.d_result_count, sizeof(int32_t), cudaMemcpyDeviceToHost, ctx.stream));
    CUDA_CHECK(cudaStreamSynchronize(ctx.stream));
    count = std::min(count, K);
    std::vector<int32_t> ids((size_t)std::max(count, 0)), mods((size_t)std::max(count, 0));
    std::vector<float> scores((size_t)std::max(count, 0));
    if (count > 0) {
        CUDA_CHECK(cudaMemcpy(ids.data(), ctx.d_result_ids, (size_t)count * 4, cudaMemcpyDeviceToHost));
        CUDA_CHECK(cudaMemcpy(scores.data(), ctx.d_result_scores, (size_t)count * 4, cudaMemcpyDeviceToHost));
        CUDA_CHECK(cudaMemcpy(mods.data(), ctx.d_result_mods, (size_t)count * 4, cudaMemcpyDeviceToHost));
    }
    std::vector<QueryResult> out;
    out.reserve((size_t)count);
    for (int32_t i = 0; i < count; ++i) out.push_back({ids[i], scores[i], mods[i], 0});
    cudaEventElapsedTime(&stats.gpu_ms_total, ctx.e_start, ctx.e_end);
    stats.gpu_ms_similarity = stats.gpu_ms_total;
    stats.gpu_ms_topk = 0;
    stats.gpu_ms_bfs = 0;
    stats.gpu_ms_rerank = 0;
    stats.nodes_scanned = 0;
    stats.bfs_waves = 0;
    return out;
}
