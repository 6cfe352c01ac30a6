// mars_kernels.cuh -- kernel argument blocks and launchers shared by the
// host files of the library.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace mars {

constexpr int kScanThreads = 256;
constexpr int kScanWarps = kScanThreads / 32;
constexpr int kBfsThreads = 256;
constexpr int kBfsWarps = kBfsThreads / 32;

// Per-query parameters.  Kernels take them by value; when `dyn` is set the
// two fields that change on every query of a replayed CUDA graph (t_q and
// epoch) are read from that device copy instead, which the graph's first
// node refreshes together with the query vector (at kDescQueryOffset).
struct MarsQueryDesc {
    float    t_q;
    float    lambda;
    float    hop_decay;
    int32_t  filter;
    int32_t  use_imp;
    int32_t  K;
    int32_t  hops;
    uint32_t epoch;
    int32_t  row_offset;
    int32_t  exclude_plus1;   // 1 + local row to leave out (0: none)
    int32_t  reserved[6];
};
constexpr size_t kDescQueryOffset = 64;
static_assert(sizeof(MarsQueryDesc) <= kDescQueryOffset, "descriptor too large");

struct StoreView {
    const float*   E;         // rows x pitch
    const float*   ts;
    const float*   imp;
    const int32_t* mod;
    const int32_t* d_n;       // device N
    int64_t        pitch4;    // float4 per row
    int32_t        nc;        // float4 chunks holding the D values
    // graph
    const int32_t* row_offsets;
    const int32_t* col_indices;
    int32_t        csr_n;
    const int32_t* extra;
    const int32_t* extra_cnt;
    int32_t        slack;
};

struct ScanArgs {
    StoreView s;
    MarsQueryDesc d;
    const MarsQueryDesc* dyn;         // device copy for t_q / epoch (may be null)
    const float4* q;                  // device query, nc chunks
    float*   part_val;                // gridDim.x * K
    int32_t* part_idx;
    unsigned int* ticket;
    unsigned int* cursor;             // dynamic row hand-out (may be null: static split only)
    float*   out_val;                 // K
    int32_t* out_idx;
    int32_t* out_cnt;
    float*   all_scores;              // diagnostic: every row's score (may be null)
    // BFS seeding (when vis_ids != nullptr)
    unsigned long long* stamp;
    int32_t* vis_ids;
    float*   vis_score;
    int32_t* lvl;                     // [0..15] level offsets, [16] tail
    // multi-query launches
    const int32_t* only;              // only[qi] == 0: query qi is skipped (null: every query)
    int32_t  exclude_base1;           // 1 + the row query 0 leaves out; query qi leaves out
                                      // row exclude_base1 - 1 + qi (0: none)
};

struct BfsArgs {
    StoreView s;
    MarsQueryDesc d;
    const MarsQueryDesc* dyn;
    const float4* q;
    unsigned long long* stamp;
    int32_t* vis_ids;
    float*   vis_score;
    int32_t* lvl;
    unsigned int* ticket;
    // final selection output
    void*    results;                 // mars_query_result[K]
    int32_t* result_cnt;              // [0] count, [1] visited
};

// Single-launch query (mars_fastq.cu): the scan arguments, the result
// destination (device or host-mapped memory) and, when a.q is null, the query
// vector itself (nc <= kFusedMaxChunks float4 chunks, i.e. D <= 1024).
constexpr int kFusedMaxChunks = 256;
struct FusedQueryArgs {
    ScanArgs a;
    void*    out;        // mars_query_result[K]
    int32_t* out_cnt;    // [0] count (-1: the BFS outgrew the last CTA), [1] visited
    float4   qbuf[kFusedMaxChunks];
};

__device__ __forceinline__ float desc_tq(const MarsQueryDesc& d, const MarsQueryDesc* dyn) {
    return dyn != nullptr ? dyn->t_q : d.t_q;
}
__device__ __forceinline__ uint32_t desc_epoch(const MarsQueryDesc& d, const MarsQueryDesc* dyn) {
    return dyn != nullptr ? dyn->epoch : d.epoch;
}

// Launchers (return cudaGetLastError()).
cudaError_t launch_scan_topk(const ScanArgs& a, int k_max, int grid, cudaStream_t st);
cudaError_t launch_bfs_hop(const BfsArgs& a, int hop, int grid, cudaStream_t st);
cudaError_t launch_bfs_finalize(const BfsArgs& a, int last_level, int k_max, int grid,
                                cudaStream_t st);
cudaError_t launch_scan_multi(const ScanArgs& a, const float* Q, int64_t qpitch, int nq, int grid,
                              cudaStream_t st);
cudaError_t launch_query_fused(const FusedQueryArgs& p, int grid, cudaStream_t st);
cudaError_t launch_topk_merge(const int32_t* ids_in, const float* vals_in, int n_lists, int K, int Q,
                              int32_t* ids_out, float* vals_out, int32_t* cnt, cudaStream_t st);
int scan_blocks_per_sm(int nc, int k_max);
// Loads the scan_topk_kernel variants for K <= 128, D <= 1024 on the current
// device; returns 0 or the cudaError_t value.
int preload_scan_topk_kernels();

}  // namespace mars
