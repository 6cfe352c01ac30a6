// mars_internal.h -- host-side objects behind the C ABI handles.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "mars_b200.h"

struct mars_store;
struct mars_query_ctx;

// ---- error plumbing ------------------------------------------------------
namespace mars {

void set_error(const std::string& msg);

// mars_query_batch_topk where query b leaves out row self_base + b
// (self_base < 0: none); used by the kNN-graph build.
int batch_topk(const mars_store* s, struct mars_batch_ctx* c, const float* d_queries, int32_t query_pitch,
               int32_t B, float t_q, float lambda, int32_t modality_filter, int32_t use_importance,
               int32_t K, int32_t row_offset, int32_t self_base, int32_t* d_ids, float* d_vals,
               int32_t* d_counts, void* stream);

// Row shards: a batched call on one shard exchanges two small records with
// the other shards, each by one all-gather of the same number of floats per
// rank on `st` (gather(arg, which, count, st): send[which] -> recv[which],
// world records rank-major):
//  0. before the candidates pass, the threshold record (kShardThr*): each
//     query's kShardJ largest sampled lower bounds (descending, -inf padded)
//     and [sampled rows, rows, mode] as int bits after the B lists; every
//     shard of mode 1 takes the same short-list threshold from their union;
//  1. between the rescore passes, the bound record (kShardRec*): per query
//     the count of candidates whose lower bound reaches the threshold (int
//     bits), the K-th and the ceil(K / world)-th largest lower bounds, then
//     one failure flag (1: the shard's call failed; no result is served).
// theta_done / done record that the call reached each exchange: every rank
// runs each exactly once per call, with neutral records (mode 0, counts 0,
// bounds -inf) when its local call ended early.
constexpr int kShardJ = 16;
inline int32_t shard_thr_floats(int32_t B) { return B * kShardJ + 3; }
inline int32_t shard_rec_floats(int32_t B) { return 3 * B + 1; }
struct BoundExchange {
    int (*gather)(void* arg, int which, int32_t count, cudaStream_t st);
    void* arg;
    int32_t world;
    float* send[2];
    const float* recv[2];
    bool theta_done;
    bool done;
};
// Enqueue neutral records of B queries on st.
int shard_neutral_thr(float* d_rec, int32_t B, cudaStream_t st);
int shard_neutral_rec(float* d_rec, int32_t B, bool failed, cudaStream_t st);

// The stream a batched call with stream == NULL runs on.
cudaStream_t batch_ctx_stream(const struct mars_batch_ctx* c);

// mars_query_batch_topk over one row shard with the bound exchange above.
int batch_topk_sharded(const mars_store* s, struct mars_batch_ctx* c, const float* d_queries,
                       int32_t query_pitch, int32_t B, float t_q, float lambda, int32_t modality_filter,
                       int32_t use_importance, int32_t K, int32_t row_offset, int32_t* d_ids, float* d_vals,
                       int32_t* d_counts, void* stream, BoundExchange* xchg);

// mars_scan_topk that leaves out one local row (exclude_row < 0: none).
int scan_topk_excluding(const mars_store* s, mars_query_ctx* c, const float* d_query, float t_q,
                        float lambda, int32_t modality_filter, int32_t use_importance, int32_t K,
                        int32_t row_offset, int32_t exclude_row, int32_t* d_ids, float* d_vals,
                        int32_t* d_count, void* stream);
// Largest |component| the fp16 copies of rows and queries may hold: within
// it the fp16 rounding error bounds used by the batched short list and the
// fp16-filtered scan hold.
constexpr float kF16Max = 60000.0f;

// Bring the store's fp16 copy of the rows up to date on stream st; *ok says
// whether it may be used (every component within kF16Max).
int store_f16_rows(const mars_store* s, cudaStream_t st, bool* ok);

// fp16-filtered scan: queries per launch and candidate rows kept per query
constexpr int kF16Slots = 16;
constexpr int kF16CandCap = 65536;
int query_ctx_f16_buffers(mars_query_ctx* c);
// mars_query through the fp16-filtered scan (hop-free queries over large
// stores); *done = 0 when the caller must answer with the fp32 kernel.
constexpr int32_t kF16QueryRows = 1 << 18;
int query_f16(const mars_store* s, mars_query_ctx* c, const float* query, float t_q,
              const mars_retrieval_config* cfg, mars_query_result* out, int32_t* n_out,
              mars_retrieval_stats* stats, int* done);

int fail(int status, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what, const char* file, int line);

}  // namespace mars

#define MARS_CUDA_TRY(call)                                                  \
    do {                                                                     \
        cudaError_t mars_e__ = (call);                                       \
        if (mars_e__ != cudaSuccess)                                         \
            return mars::cuda_fail(mars_e__, #call, __FILE__, __LINE__);     \
    } while (0)

#define MARS_TRY(call)                                                       \
    do {                                                                     \
        int mars_s__ = (call);                                               \
        if (mars_s__ != MARS_OK) return mars_s__;                            \
    } while (0)

// Scoped device selection: restores the caller's current device.
struct MarsDeviceGuard {
    int prev = -1;
    bool ok = true;
    explicit MarsDeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
    }
    ~MarsDeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

// ---- store (DeviceMemoryGraph) -------------------------------------------
struct mars_store {
    int32_t device = 0;
    int32_t capacity = 0;
    int32_t dim = 0;
    int32_t pitch = 0;          // floats per row (dim rounded up to 4)
    int32_t n = 0;              // host mirror of *d_n
    int32_t edge_slack = 0;
    bool owns = true;           // false: wraps memory owned by a caller

    float* d_E = nullptr;       // capacity x pitch
    float* d_ts = nullptr;
    float* d_imp = nullptr;
    int32_t* d_mod = nullptr;
    int32_t* d_n = nullptr;     // device N

    // CSR over nodes [0, csr_n)
    int32_t csr_n = 0;
    int32_t num_edges = 0;
    int32_t csr_edge_cap = 0;
    int32_t* d_row_offsets = nullptr;
    int32_t* d_col_indices = nullptr;

    // append-only neighbour slack: node u's extras at d_extra[u*slack ...]
    int32_t* d_extra = nullptr;
    int32_t* d_extra_cnt = nullptr;
    std::vector<int32_t> h_extra_cnt;

    cudaStream_t stream = nullptr;
    cudaEvent_t written = nullptr;  // last write to the store

    // [0]: the largest row norm; [1]: the largest fp16 rounding error
    // ||e - fp16(e)|| of a row of the fp16 copy; both as the bits of
    // non-negative floats (they bound the error of the tensor-core short
    // list; kernels read them on the device)
    unsigned int* d_norm_bits = nullptr;

    // raw view of a caller-owned DeviceMemoryGraph (compat layer)
    void* compat_key = nullptr;

    // pinned, device-mapped staging for small appends: the caller's host
    // arrays are packed here and read by the append kernel directly, so an
    // append is one launch and returns without waiting for the device.  Two
    // buffers alternate; each is reused only after its last kernel finished.
    struct HostStage {
        char* h = nullptr;        // host address
        char* d = nullptr;        // device view of the same memory
        size_t cap = 0;
        cudaEvent_t done = nullptr;
    };
    HostStage stage[2];
    int stage_next = 0;

    // scratch of the kNN-graph build, kept between builds (freed with the
    // store): the batched top-K context and the per-row candidate lists
    struct BuildCache {
        struct mars_batch_ctx* bc = nullptr;
        int32_t bc_nodes = 0, bc_chunk = 0, bc_k = 0;
        int32_t* d_knn = nullptr;
        float* d_vals = nullptr;
        int32_t* d_cnt = nullptr;
        size_t entries = 0;           // capacity of d_knn / d_vals
        int32_t rows = 0;             // capacity of d_cnt
    };
    BuildCache build;

    // fp16 copy of the rows for the batched tensor-core short list (made on
    // the first batched query; rows [0, e16_rows) are current: appends extend
    // it, uploads and deletes reset it)
    void* d_E16 = nullptr;
    int32_t e16_pitch = 0;      // halves per row (dim rounded up to 8)
    int32_t e16_rows = 0;
    bool e16_in_range = false;  // every component within the fp16 range covered
    cudaEvent_t e16_ready = nullptr;   // the last conversion into d_E16
};

// ---- query context (QueryContext) ----------------------------------------

struct mars_query_ctx {
    int32_t device = 0;
    int32_t max_nodes = 0;
    int32_t dim = 0;
    int32_t pitch = 0;
    int32_t max_k = 0;
    int32_t num_sms = 0;
    int32_t scan_blocks = 0;
    int32_t bfs_blocks = 0;

    cudaStream_t stream = nullptr;
    cudaEvent_t ev[5] = {nullptr, nullptr, nullptr, nullptr, nullptr};

    // per-query descriptor: host pinned staging + device copy
    void* h_desc = nullptr;
    void* d_desc = nullptr;
    size_t desc_bytes = 0;

    // scan scratch
    float* d_part_val = nullptr;    // scan_blocks * kMaxTopK
    int32_t* d_part_idx = nullptr;
    unsigned int* d_ticket = nullptr;   // [4] tickets for scan / bfs / finalize / merge
    unsigned int* d_multi = nullptr;    // tickets + row counters of the multi-query scan

    // BFS scratch
    unsigned long long* d_stamp = nullptr;  // max_nodes
    uint32_t epoch = 0;
    int32_t* d_vis_ids = nullptr;           // max_nodes
    float* d_vis_score = nullptr;           // max_nodes
    int32_t* d_lvl = nullptr;               // [16] level offsets + [16] tail
    float* d_seed_val = nullptr;            // kMaxTopK
    int32_t* d_seed_idx = nullptr;
    int32_t* d_seed_cnt = nullptr;

    // results
    mars_query_result* d_results = nullptr;   // max_k
    int32_t* d_result_cnt = nullptr;
    mars_query_result* h_results = nullptr;    // pinned
    int32_t* h_result_cnt = nullptr;           // pinned [2]: count, visited

    // single-launch path (mars_fastq.cu): every row's fused score for the
    // in-kernel BFS, and device views of the host-mapped result buffers
    bool use_fused = true;
    float* d_all_scores = nullptr;              // max_nodes
    mars_query_result* dm_results = nullptr;    // = h_results, device view
    int32_t* dm_result_cnt = nullptr;           // = h_result_cnt, device view
    uint64_t fused_queries = 0;                 // answered by the single launch
    uint64_t fused_reruns = 0;                  // BFS outgrew the last CTA

    // fp16-filtered scan (mars_scan16.cu), allocated on first use
    unsigned int* d_f16_ticket = nullptr;       // kF16Slots
    unsigned long long* d_f16_cand = nullptr;   // kF16Slots x kF16CandCap
    int32_t* d_f16_cnt = nullptr;               // kF16Slots
    int32_t* d_f16_overflow = nullptr;          // kF16Slots flags, then kF16Slots x (candidates, survivors)
    int32_t* h_f16_overflow = nullptr;          // pinned copy
    uint64_t f16_reruns = 0;                    // queries re-run on the fp32 scan
    int32_t* d_f16_qout = nullptr;              // one query's packed results (mars_query):
    int32_t* h_f16_qout = nullptr;              //   [overflow, count, -, -, ids K, scores K, modalities K]
    int32_t f16_max_cand = 0;                   // largest candidate list of the last call
    int32_t f16_max_surv = 0;                   // largest survivor count of the last call (-1: overflow)

    // graph replay of the whole query (H2D desc -> kernels -> D2H)
    bool use_graph = true;
    cudaGraphExec_t graph = nullptr;
    uint64_t graph_key = 0;
};
