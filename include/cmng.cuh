// cmng.cuh -- the reference's Cross-Modal Navigable Graph API, served by the
// B200 library.
//
// Same declarations as include/cmng.cuh of antonellof/cuda-multimodal-memory,
// forwarding to the C ABI in mars_b200.h:
//
//   build_cmng              -> mars_store_create/upload + mars_cmng_build
//                              (tensor-core kNN, exact fp32 lists)
//   cmng_search             -> mars_cmng_search_batch with one query
//   create/destroy_cmng_context, cmng_upload_fp16, free_cmng
//
// A fixed out-degree directed graph: node v's neighbours are
// d_neighbors[v * degree .. (v + 1) * degree - 1], the last degree_cross of
// them cross-modal bridges, -1 for empty slots.  Search is a greedy beam search
// with temporal decay applied to the final beam.
#ifndef CMNG_CUH
#define CMNG_CUH

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cstdint>
#include <cstdio>
#include <vector>

#include "memory_cuda.cuh"

#ifndef CMNG_CHECK
#define CMNG_CHECK(call) CUDA_CHECK(call)
#endif

struct CMNGGraph {
    int32_t N            = 0;
    int32_t D            = 0;
    int32_t degree       = 64;
    int32_t degree_cross = 4;

    int32_t* d_neighbors       = nullptr;   // N x degree
    float*   d_embeddings      = nullptr;   // N rows, padded to a multiple of 4 floats
    half*    d_embeddings_fp16 = nullptr;   // optional copy (cmng_upload_fp16)
    int32_t* d_modalities      = nullptr;
    float*   d_timestamps      = nullptr;

    float    build_time_ms     = 0.0f;
};

struct CMNGSearchConfig {
    int32_t K                 = 10;
    int32_t beam_width        = 128;
    int32_t max_iterations    = 64;
    int32_t num_parents       = 1;
    float   time_decay_lambda = 1e-8f;
    int32_t modality_filter   = -1;     // accepted, unused (as in the reference)
    bool    use_fp16          = false;  // accepted, unused: fp32 rows are scored
};

struct CMNGSearchContext {
    int32_t max_D    = 0;
    int32_t max_K    = 0;
    int32_t max_beam = 0;

    int32_t* d_result_ids    = nullptr;
    float*   d_result_scores = nullptr;
    int32_t* d_result_mods   = nullptr;
    int32_t* d_result_count  = nullptr;

    float*   h_query_pinned  = nullptr;
    float*   d_query         = nullptr;

    cudaEvent_t e_start, e_end;
    cudaStream_t stream      = nullptr;
    bool valid               = false;
};

CMNGGraph build_cmng(const float* h_embeddings, const int32_t* h_modalities, const float* h_timestamps,
                     int32_t N, int32_t D, int32_t degree = 64, int32_t degree_cross = 4);

void cmng_upload_fp16(CMNGGraph& g);
void free_cmng(CMNGGraph& g);

CMNGSearchContext create_cmng_context(int32_t D, int32_t max_beam = 128, int32_t max_k = 64);
void destroy_cmng_context(CMNGSearchContext& ctx);

std::vector<QueryResult> cmng_search(const CMNGGraph& g, CMNGSearchContext& ctx, const float* h_query,
                                     float query_timestamp, const CMNGSearchConfig& cfg,
                                     RetrievalStats& stats);

#endif  // CMNG_CUH
