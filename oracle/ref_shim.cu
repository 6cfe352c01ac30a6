// ref_shim.cu -- C entry points over the REFERENCE's own GPU path.
//
// TEST INFRASTRUCTURE ONLY.  Compiled by oracle/Makefile.ref together with
// the reference's unmodified sources (src/memory_cuda.cu, src/cmng_build.cu,
// src/cmng_search.cu, src/memory_graph.cpp from the reference checkout) into
// oracle/_ref/libmars_ref_gpu.so, which tests on the GPU box load with ctypes
// to compare this repository's kernels with the reference's kernels on the
// same inputs.  Nothing in the product links it.
//
// The reference reports CUDA errors by exiting the process (its CUDA_CHECK);
// these wrappers add nothing to that.
#include <chrono>
#include <cstdint>
#include <cstring>
#include <vector>

#include "cmng.cuh"
#include "memory_cuda.cuh"
#include "memory_graph.h"

namespace {

MemoryGraph make_graph(const float* E, const int32_t* mod, const float* ts, int32_t N, int32_t D,
                       const int32_t* row_off, const int32_t* col, int32_t nnz) {
    MemoryGraph g;
    g.num_nodes = N;
    g.embedding_dim = D;
    g.embeddings.assign(E, E + (size_t)N * D);
    g.modalities.assign(mod, mod + N);
    g.timestamps.assign(ts, ts + N);
    if (row_off != nullptr) {
        g.row_offsets.assign(row_off, row_off + N + 1);
        g.col_indices.assign(col, col + nnz);
    } else {
        g.row_offsets.assign((size_t)N + 1, 0);
    }
    g.num_edges = (int32_t)g.col_indices.size();
    return g;
}

}  // namespace

extern "C" {

// query_memory_fast over nq queries (src/memory_cuda.cu:1069-1158).
// use_cublas / use_cub select the reference's "--mars" configuration
// (src/latency_bench.cu:336-337).  Outputs are [nq][K]; counts[nq];
// wall_us[nq] = host time around the call, gpu_ms[nq] = its gpu_ms_total.
int ref_query_batch(const float* E, const int32_t* mod, const float* ts, int32_t N, int32_t D,
                    const int32_t* row_off, const int32_t* col, int32_t nnz, const float* Q,
                    int32_t nq, float t_q, int32_t K, int32_t hops, float lambda, float decay,
                    int32_t filter, int32_t use_cublas, int32_t use_cub, int32_t use_graph,
                    int32_t* out_ids, float* out_scores, int32_t* out_mods, int32_t* out_hops,
                    int32_t* out_counts, float* wall_us, float* gpu_ms) {
    MemoryGraph g = make_graph(E, mod, ts, N, D, row_off, col, nnz);
    DeviceMemoryGraph dg = upload_to_device(g);
    QueryContext ctx = create_query_context(N, D, K);
    ctx.use_cublas = use_cublas != 0;
    ctx.use_cub_topk = use_cub != 0;
    ctx.use_cuda_graph = use_graph != 0;
    RetrievalConfig cfg;
    cfg.top_k = K;
    cfg.bfs_max_hops = hops;
    cfg.time_decay_lambda = lambda;
    cfg.bfs_score_decay = decay;
    cfg.modality_filter = filter;
    for (int32_t q = 0; q < nq; ++q) {
        RetrievalStats st;
        const auto t0 = std::chrono::steady_clock::now();
        std::vector<QueryResult> r = query_memory_fast(dg, ctx, Q + (size_t)q * D, t_q, cfg, st);
        const auto t1 = std::chrono::steady_clock::now();
        if (wall_us) wall_us[q] = std::chrono::duration<float, std::micro>(t1 - t0).count();
        if (gpu_ms) gpu_ms[q] = st.gpu_ms_total;
        const int32_t n = (int32_t)r.size() < K ? (int32_t)r.size() : K;
        out_counts[q] = n;
        for (int32_t i = 0; i < n; ++i) {
            out_ids[(size_t)q * K + i] = r[i].node_id;
            out_scores[(size_t)q * K + i] = r[i].score;
            out_mods[(size_t)q * K + i] = r[i].modality;
            out_hops[(size_t)q * K + i] = r[i].hops_from_seed;
        }
    }
    destroy_query_context(ctx);
    free_device(dg);
    return 0;
}

// build_cmng (src/cmng_build.cu:135-255): neighbour lists [N][degree].
int ref_build_cmng(const float* E, const int32_t* mod, const float* ts, int32_t N, int32_t D,
                   int32_t degree, int32_t degree_cross, int32_t* out_neighbors, float* build_ms) {
    CMNGGraph g = build_cmng(E, mod, ts, N, D, degree, degree_cross);
    cudaMemcpy(out_neighbors, g.d_neighbors, (size_t)N * degree * sizeof(int32_t),
               cudaMemcpyDeviceToHost);
    if (build_ms) *build_ms = g.build_time_ms;
    free_cmng(g);
    return 0;
}

// cmng_search (src/cmng_search.cu:347-422) over a given neighbour graph.
int ref_cmng_search(const float* E, const int32_t* mod, const float* ts, int32_t N, int32_t D,
                    const int32_t* neighbors, int32_t degree, const float* Q, int32_t nq,
                    float t_q, int32_t K, int32_t beam, int32_t iters, int32_t num_parents,
                    float lambda, int32_t* out_ids, float* out_scores, int32_t* out_counts,
                    float* gpu_ms) {
    CMNGGraph g;
    g.N = N;
    g.D = D;
    g.degree = degree;
    g.degree_cross = 0;
    cudaMalloc(&g.d_neighbors, (size_t)N * degree * sizeof(int32_t));
    cudaMalloc(&g.d_embeddings, (size_t)N * D * sizeof(float));
    cudaMalloc(&g.d_modalities, (size_t)N * sizeof(int32_t));
    cudaMalloc(&g.d_timestamps, (size_t)N * sizeof(float));
    cudaMemcpy(g.d_neighbors, neighbors, (size_t)N * degree * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(g.d_embeddings, E, (size_t)N * D * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(g.d_modalities, mod, (size_t)N * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(g.d_timestamps, ts, (size_t)N * 4, cudaMemcpyHostToDevice);
    CMNGSearchContext ctx = create_cmng_context(D, beam, K);
    CMNGSearchConfig cfg;
    cfg.K = K;
    cfg.beam_width = beam;
    cfg.max_iterations = iters;
    cfg.num_parents = num_parents;
    cfg.time_decay_lambda = lambda;
    for (int32_t q = 0; q < nq; ++q) {
        RetrievalStats st;
        std::vector<QueryResult> r = cmng_search(g, ctx, Q + (size_t)q * D, t_q, cfg, st);
        if (gpu_ms) gpu_ms[q] = st.gpu_ms_total;
        const int32_t n = (int32_t)r.size() < K ? (int32_t)r.size() : K;
        out_counts[q] = n;
        for (int32_t i = 0; i < n; ++i) {
            out_ids[(size_t)q * K + i] = r[i].node_id;
            out_scores[(size_t)q * K + i] = r[i].score;
        }
    }
    destroy_cmng_context(ctx);
    free_cmng(g);
    return 0;
}

}  // extern "C"
