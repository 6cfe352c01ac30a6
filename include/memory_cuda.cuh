// memory_cuda.cuh -- the reference's C++ retrieval API, served by the B200
// library.
//
// Same declarations as include/memory_cuda.cuh of
// antonellof/cuda-multimodal-memory, so reference callers (main.cu,
// validate.cu, latency_bench.cu, engine_server.cu, the demos) compile and link
// against libmars_b200 unchanged.  Every function forwards to the C ABI in
// mars_b200.h:
//
//   upload_to_device / free_device        -> mars_store_create/upload/destroy
//   create/destroy_query_context          -> mars_query_ctx_create/destroy
//   query_memory_fast / query_memory      -> mars_query / mars_query_once
//   init/update_importance                -> mars_importance_*
//   compute_novelty                       -> mars_novelty
//
// Differences a caller can observe:
//   * the pipeline is always the fused fp32 scan (ctx.use_cublas,
//     ctx.use_cub_topk and ctx.use_fp16 are accepted and have no effect; the
//     fp16 copy is still created by upload_fp16_embeddings for callers that
//     read it);
//   * top-K is exact for K up to 128 (the reference clamps to 64 and its
//     custom top-K kernels drop candidates for K > 8);
//   * BFS takes the best parent score deterministically and never truncates
//     the frontier; results are ranked (score desc, node id asc);
//   * on an error the call prints the message and exits, like the
//     reference's CUDA_CHECK; with MARS_COMPAT_THROW=1 in the environment it
//     throws std::runtime_error instead.
#ifndef MEMORY_CUDA_CUH
#define MEMORY_CUDA_CUH

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "memory_graph.h"

#define CUDA_CHECK(call)                                                    \
    do {                                                                    \
        cudaError_t err__ = (call);                                         \
        if (err__ != cudaSuccess) {                                         \
            std::fprintf(stderr, "CUDA error %s:%d - %s\n",                 \
                         __FILE__, __LINE__, cudaGetErrorString(err__));    \
            std::exit(EXIT_FAILURE);                                        \
        }                                                                   \
    } while (0)

// Device-resident graph: raw device pointers (the arrays belong to the store
// that upload_to_device created; free_device releases it).
struct DeviceMemoryGraph {
    int32_t  num_nodes     = 0;
    int32_t  num_edges     = 0;
    int32_t  embedding_dim = 0;
    int32_t* d_row_offsets = nullptr;
    int32_t* d_col_indices = nullptr;
    float*   d_embeddings  = nullptr;      // rows padded to a multiple of 4 floats
    half*    d_embeddings_fp16 = nullptr;
    int32_t* d_modalities  = nullptr;
    float*   d_timestamps  = nullptr;
    float*   d_importance  = nullptr;      // set by init_importance
    int32_t* d_edge_hits   = nullptr;      // set by init_edge_hits
};

DeviceMemoryGraph upload_to_device(const MemoryGraph& h);
void              free_device(DeviceMemoryGraph& d);

void upload_fp16_embeddings(DeviceMemoryGraph& dg);
void free_fp16_embeddings(DeviceMemoryGraph& dg);

struct QueryResult {
    int32_t node_id;
    float   score;
    int32_t modality;
    int32_t hops_from_seed;
};

struct RetrievalConfig {
    int32_t top_k             = 10;
    int32_t bfs_max_hops      = 2;
    float   time_decay_lambda = 1e-8f;
    float   bfs_score_decay   = 0.5f;
    int32_t modality_filter   = -1;
    bool    use_importance    = false;
};

struct RetrievalStats {
    float gpu_ms_similarity = 0.0f;
    float gpu_ms_topk       = 0.0f;
    float gpu_ms_bfs        = 0.0f;
    float gpu_ms_rerank     = 0.0f;
    float gpu_ms_total      = 0.0f;
    int32_t nodes_scanned   = 0;
    int32_t bfs_waves       = 0;
};

std::vector<QueryResult>
query_memory(const DeviceMemoryGraph& dg, const float* h_query, float query_timestamp,
             const RetrievalConfig& cfg, RetrievalStats& stats);

// Query scratch.  A value type like the reference's (include/memory_cuda.cuh
// of the reference, QueryContext): the same members in the same order, so
// code that names them compiles unchanged.  This library keeps its own state
// behind `impl` (appended after them) and leaves the reference's scratch
// pointers, events, graph and cuBLAS/CUB members null or zero: they describe
// the reference's pipeline, which is not run here.  `stream` is the
// context's stream, `valid` is set by create_query_context, and
// use_cuda_graph is honoured; use_fp16 / use_cublas / use_cub_topk are
// accepted and have no effect (the fused fp32 pipeline always runs).
struct QueryContext {
    int32_t max_nodes     = 0;
    int32_t embedding_dim = 0;
    int32_t max_k         = 0;

    float*   d_query      = nullptr;
    float*   d_sim        = nullptr;
    float*   d_final      = nullptr;
    float*   d_bfs_score  = nullptr;
    int32_t* d_hop_count  = nullptr;
    int32_t* d_top_idx    = nullptr;
    float*   d_top_val    = nullptr;
    int32_t* d_front_a    = nullptr;
    int32_t* d_front_b    = nullptr;
    int32_t* d_front_cnt  = nullptr;
    void*    d_compact_out   = nullptr;
    int32_t* d_compact_count = nullptr;
    int32_t  max_compact     = 0;
    int32_t* d_front_cnt_b   = nullptr;
    float*   h_query_pinned  = nullptr;

    cudaEvent_t e0 = nullptr, e1 = nullptr, e2 = nullptr, e3 = nullptr, e4 = nullptr;
    cudaStream_t stream   = nullptr;   // the context's stream
    bool valid            = false;

    cudaGraph_t      captured_graph   = nullptr;
    cudaGraphExec_t  graph_exec       = nullptr;
    bool             graph_captured   = false;
    int32_t          graph_N          = 0;
    int32_t          graph_K          = 0;
    int32_t          graph_bfs_hops   = 0;
    int32_t          graph_mod_filter = -1;
    bool             graph_fp16       = false;

    bool use_cuda_graph   = false;     // replay the query as one CUDA graph
    bool use_fp16         = false;     // accepted, no effect
    bool use_cublas       = false;     // accepted, no effect
    bool use_cub_topk     = false;     // accepted, no effect

    void*    cublas_handle    = nullptr;
    void*    d_sort_temp      = nullptr;
    size_t   sort_temp_bytes  = 0;
    float*   d_sort_keys_in   = nullptr;
    float*   d_sort_keys_out  = nullptr;
    int32_t* d_sort_vals_in   = nullptr;
    int32_t* d_sort_vals_out  = nullptr;

    void* impl            = nullptr;   // mars_query_ctx* (this library's state)
};

QueryContext create_query_context(int32_t max_nodes, int32_t embedding_dim, int32_t max_k = 64);
void         destroy_query_context(QueryContext& ctx);

std::vector<QueryResult>
query_memory_fast(const DeviceMemoryGraph& dg, QueryContext& ctx, const float* h_query,
                  float query_timestamp, const RetrievalConfig& cfg, RetrievalStats& stats);

// importance[i] = 1 for all rows.
void init_importance(DeviceMemoryGraph& dg);

// importance *= (1 - decay_rate) for all rows, then for every listed node
// importance = min(importance + boost, max_importance).  Asynchronous on
// `stream`.
void update_importance(DeviceMemoryGraph& dg, const int32_t* d_result_ids, int32_t n_results,
                       float boost = 0.1f, float decay_rate = 0.001f,
                       float max_importance = 5.0f, cudaStream_t stream = nullptr);

// Largest dot product of the device vector d_query with any stored row.
float compute_novelty(const DeviceMemoryGraph& dg, const float* d_query,
                      cudaStream_t stream = nullptr);

void    init_edge_hits(DeviceMemoryGraph& dg);
int32_t maintain_graph(DeviceMemoryGraph& dg, int32_t min_hits = 0,
                       int32_t window_queries = 1000, cudaStream_t stream = nullptr);

#endif  // MEMORY_CUDA_CUH
