/*
 * mars_b200.h -- C ABI of the B200-native MARS retrieval path.
 *
 * This is the drop-in boundary.  Every entry point takes plain pointers and
 * sizes, returns an int status (MARS_OK or MARS_ERR_*), never exits the
 * process, and never falls back to CPU code.  Each declaration names the
 * reference interface it replaces (paths relative to the root of
 * antonellof/cuda-multimodal-memory).  The reference's C++ API
 * (memory_cuda.cuh, cmng.cuh) is provided on top of this ABI by the same
 * library, so reference callers relink unchanged.
 *
 * Pointer arguments documented as "host or device" may point to pageable or
 * pinned host memory or to device memory of the store's GPU (the library
 * copies with cudaMemcpyDefault).  Streams are passed as void* (a
 * cudaStream_t); NULL means the object's own stream.
 *
 * Threading: like the reference's QueryContext (include/memory_cuda.cuh:122),
 * a context or store must not be used by two host threads at once.
 */
#ifndef MARS_B200_H
#define MARS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MARS_B200_ABI_VERSION 1
#define MARS_MAX_TOP_K 256      /* reference: MAX_TOP_K = 64 (src/memory_cuda.cu:38) */
#define MARS_MAX_BFS_HOPS 14

/* ---- status ------------------------------------------------------------ */
enum {
    MARS_OK              = 0,
    MARS_ERR_INVALID     = 1,   /* bad argument                              */
    MARS_ERR_CUDA        = 2,   /* CUDA runtime error                        */
    MARS_ERR_OOM         = 3,   /* device or pinned allocation failed        */
    MARS_ERR_CAPACITY    = 4,   /* store / context / edge slack exhausted    */
    MARS_ERR_UNSUPPORTED = 5,   /* shape or option not supported             */
    MARS_ERR_TIMEOUT     = 6,   /* a bounded device-side wait gave up        */
    MARS_ERR_NO_DEVICE   = 7,   /* no usable sm_100 device                   */
    MARS_ERR_DEVICE      = 8    /* a device-side check set the error flag    */
};

/* Message of the last failure on the calling thread (never NULL). */
const char* mars_last_error(void);
const char* mars_status_string(int status);
int         mars_abi_version(void);

/* ---- value types (binary layout of the reference structs) ------------- */

/* QueryResult, include/memory_cuda.cuh:85-90 */
typedef struct mars_query_result {
    int32_t node_id;
    float   score;
    int32_t modality;
    int32_t hops_from_seed;
} mars_query_result;

/* RetrievalConfig, include/memory_cuda.cuh:92-99 (bool use_importance is
 * widened to int32 for a stable C layout). */
typedef struct mars_retrieval_config {
    int32_t top_k;
    int32_t bfs_max_hops;
    float   time_decay_lambda;
    float   bfs_score_decay;
    int32_t modality_filter;
    int32_t use_importance;
} mars_retrieval_config;

/* RetrievalStats, include/memory_cuda.cuh:101-109, plus the device counts
 * of this implementation. */
typedef struct mars_retrieval_stats {
    float   gpu_ms_similarity;   /* fused scan + top-K                      */
    float   gpu_ms_topk;         /* 0: top-K is fused into the scan          */
    float   gpu_ms_bfs;          /* BFS hops + final selection               */
    float   gpu_ms_rerank;       /* 0: decay is fused into the scan          */
    float   gpu_ms_total;
    int32_t nodes_scanned;
    int32_t bfs_waves;
    int32_t nodes_visited;       /* seeds + BFS-discovered nodes             */
} mars_retrieval_stats;

/* ---- device store: DeviceMemoryGraph (include/memory_cuda.cuh:60-75) --- */
typedef struct mars_store mars_store;

typedef struct mars_store_info {
    int32_t  device;
    int32_t  num_nodes;        /* current N                                   */
    int32_t  capacity;         /* rows allocated                              */
    int32_t  embedding_dim;    /* D                                           */
    int32_t  row_pitch;        /* floats between rows (D rounded up to 4)      */
    int32_t  num_edges;        /* CSR edges                                   */
    int32_t  csr_nodes;        /* nodes covered by the CSR                    */
    int32_t  edge_slack;       /* append-only neighbour slots per node        */
    float*   d_embeddings;     /* capacity x row_pitch, zero padded           */
    int32_t* d_modalities;
    float*   d_timestamps;
    float*   d_importance;     /* initialised to 1                            */
    int32_t* d_row_offsets;    /* csr_nodes + 1 (NULL without a graph)        */
    int32_t* d_col_indices;
    int32_t* d_num_nodes;      /* device copy of N read by every kernel       */
} mars_store_info;

/* Allocate an empty store with room for `capacity` rows of dimension `dim`
 * on `device`, and `edge_slack` append-only neighbour slots per node.
 * Replaces the allocation half of upload_to_device
 * (include/memory_cuda.cuh:77, src/memory_cuda.cu:593-616). */
int mars_store_create(int32_t device, int32_t capacity, int32_t dim,
                      int32_t edge_slack, mars_store** out);

/* Replace the contents with n rows (host or device pointers) and an
 * optional CSR graph over them (row_offsets may be NULL).  importance may be
 * NULL (all 1).  Embeddings are taken as given, like upload_to_device.
 * Replaces the copy half of upload_to_device (src/memory_cuda.cu:599-615). */
int mars_store_upload(mars_store* s, int32_t n, const float* embeddings,
                      const int32_t* modalities, const float* timestamps,
                      const float* importance, const int32_t* row_offsets,
                      const int32_t* col_indices, int32_t num_edges);

/* Streaming insert: append n rows in place (no rebuild, no re-upload).
 * With normalize != 0 each row is divided by (sqrt(sum x^2) + 1e-8), summed
 * sequentially in fp32 exactly as engine_server's add_node
 * (src/engine_server.cu:154-176); the reference instead grows host vectors
 * and re-uploads the whole corpus (src/engine_server.cu:188-213).
 * first_id (may be NULL) receives the id of the first appended row. */
int mars_store_append(mars_store* s, int32_t n, const float* embeddings,
                      const int32_t* modalities, const float* timestamps,
                      const float* importance, int32_t normalize,
                      int32_t* first_id);

/* Tombstone delete (engine_server DELETE, src/engine_server.cu:178-185):
 * each listed row's embedding becomes zero and its timestamp -1, as the
 * reference does; ids outside [0, N) are ignored.  ids: host array.  Like
 * the reference, the row keeps its id and its edges (its fused score is 0,
 * and a BFS can still reach it).  Asynchronous like mars_store_append. */
int mars_store_delete(mars_store* s, int32_t n, const int32_t* ids);

/* Append n directed edges src[i] -> dst[i] (host arrays) to the per-node
 * slack lists; MARS_ERR_CAPACITY if a node's slack is full (nothing is
 * written then).  Replaces the periodic NSN rebuild of
 * src/engine_server.cu:193-200 for incremental bridges. */
int mars_store_append_edges(mars_store* s, int32_t n, const int32_t* src,
                            const int32_t* dst);

/* Overwrite importance weights of rows [first, first+n) (host or device). */
int mars_store_set_importance(mars_store* s, int32_t first, int32_t n,
                              const float* importance);

/* init_importance (include/memory_cuda.cuh:203-205,
 * src/memory_cuda.cu:1165-1176): importance of every row = value. */
int mars_importance_fill(mars_store* s, float value);

/* update_importance (include/memory_cuda.cuh:207-215,
 * src/memory_cuda.cu:1179-1224): importance *= (1 - decay_rate) for all rows,
 * then importance[id] = min(importance[id] + boost, max_importance) for each
 * of the n device ids (ids < 0 or >= N are skipped).  A repeated id is
 * boosted once per occurrence (atomic update; the reference's plain
 * read-modify-write may lose repeats).  Asynchronous on `stream`. */
int mars_importance_update(mars_store* s, const int32_t* d_ids, int32_t n,
                           float boost, float decay_rate, float max_importance,
                           void* stream);

int mars_store_info_get(const mars_store* s, mars_store_info* out);

/* Copy rows [first, first+n) back to host arrays (any may be NULL): the
 * embeddings as stored (n x dim), modalities, timestamps, importance. */
int mars_store_read(const mars_store* s, int32_t first, int32_t n,
                    float* embeddings, int32_t* modalities, float* timestamps,
                    float* importance);

/* free_device (include/memory_cuda.cuh:78).  NULL is accepted. */
int mars_store_destroy(mars_store* s);

/* ---- query context: QueryContext (include/memory_cuda.cuh:122-181) ---- */
typedef struct mars_query_ctx mars_query_ctx;

/* create_query_context (include/memory_cuda.cuh:183-184,
 * src/memory_cuda.cu:789-854): scratch for stores of up to max_nodes rows,
 * top-K up to max_k (<= MARS_MAX_TOP_K). */
int mars_query_ctx_create(int32_t device, int32_t max_nodes, int32_t dim,
                          int32_t max_k, mars_query_ctx** out);

/* destroy_query_context (include/memory_cuda.cuh:185).  NULL is accepted. */
int mars_query_ctx_destroy(mars_query_ctx* ctx);

/* query_memory_fast (include/memory_cuda.cuh:188-194,
 * src/memory_cuda.cu:1069-1158): fused score x decay [x importance] ->
 * top-K seeds -> BFS over the store's graph -> best top_k visited nodes by
 * (score desc, id asc).  query: host or device, D floats.  out: host array
 * of cfg->top_k entries; *n_out receives the count.  stats may be NULL.
 * Blocks until the results are on the host (like the reference).  A query
 * without BFS hops over a store of at least 2^18 rows (top_k <= 64, D a
 * multiple of 4, values within the fp16 range) streams the store's fp16 copy
 * through the exact fp16-filtered scan (mars_scan_topk_f16): same results,
 * half the bytes. */
int mars_query(const mars_store* s, mars_query_ctx* ctx, const float* query,
               float query_timestamp, const mars_retrieval_config* cfg,
               mars_query_result* out, int32_t* n_out,
               mars_retrieval_stats* stats);

/* Same pipeline, device in / device out, asynchronous on `stream` (NULL:
 * the context's stream).  d_query: D floats on the device; d_out: top_k
 * results; d_count: one int32.  Capturable in a CUDA graph once the first
 * call with the same (store, top_k class, hops) has been made. */
int mars_query_device(const mars_store* s, mars_query_ctx* ctx,
                      const float* d_query, float query_timestamp,
                      const mars_retrieval_config* cfg,
                      mars_query_result* d_out, int32_t* d_count,
                      void* stream);

/* query_memory (include/memory_cuda.cuh:113-118): as mars_query with a
 * temporary context. */
int mars_query_once(const mars_store* s, const float* query,
                    float query_timestamp, const mars_retrieval_config* cfg,
                    mars_query_result* out, int32_t* n_out,
                    mars_retrieval_stats* stats);

/* Fused scan only (no BFS), device in / device out: top-K of
 * dot(E_i, q) * __expf(-lambda * max(0, t_q - ts_i)) [* imp_i] over rows
 * passing the modality filter, ranked (score desc, id asc), rows from
 * `row_offset` on reported as row_offset + i.  d_ids / d_vals: K entries,
 * unused tail = (-1, -inf); d_count: number found.  This is stages 1-3 of
 * src/memory_cuda.cu:936-1021 (cublasSgemv -> temporal_rerank_kernel ->
 * CUB radix sort) in one kernel. */
int mars_scan_topk(const mars_store* s, mars_query_ctx* ctx,
                   const float* d_query, float query_timestamp, float lambda,
                   int32_t modality_filter, int32_t use_importance, int32_t K,
                   int32_t row_offset, int32_t* d_ids, float* d_vals,
                   int32_t* d_count, void* stream);

/* nq queries of mars_scan_topk in one launch (results identical to nq
 * separate calls).  d_queries: nq rows of query_pitch floats on the device
 * (16-byte aligned, pitch >= the store's row pitch); d_ids / d_vals:
 * nq x K, d_counts: nq (may be NULL).  The queries are the rows of one 2-D
 * grid: while the last CTA of one query merges its partial lists, the CTAs
 * of the next query already stream, so the per-query selection tail and the
 * launch gaps overlap with streaming.  Every query still reads every row.
 * The reference answers one query per pipeline (src/memory_cuda.cu:924-1067);
 * this entry point has no counterpart there. */
int mars_scan_topk_multi(const mars_store* s, mars_query_ctx* ctx, const float* d_queries,
                         int32_t query_pitch, int32_t nq, float query_timestamp, float lambda,
                         int32_t modality_filter, int32_t use_importance, int32_t K,
                         int32_t row_offset, int32_t* d_ids, float* d_vals, int32_t* d_counts,
                         void* stream);

/* The same results as mars_scan_topk_multi, bit for bit, from the store's
 * fp16 copy of its rows (2 bytes per value instead of 4).  The fp16 pass only
 * filters: with a proven error margin it brackets every row's fused score,
 * keeps the rows whose upper bound reaches the K-th best lower bound, and
 * scores those exactly in fp32 with the scan's arithmetic.  The fp16 copy is
 * made on first use (2 bytes per value of the store) and kept current.
 * K <= 64, D <= 1024 with D % 4 == 0; otherwise, or when a value exceeds
 * 60000, it runs mars_scan_topk_multi.  Blocks until done: queries whose
 * candidate list overflows are answered again by the fp32 scan.  The
 * reference's FP16 path (src/memory_cuda.cu:113-156) changes the scores; this
 * one does not. */
int mars_scan_topk_f16(const mars_store* s, mars_query_ctx* ctx, const float* d_queries,
                       int32_t query_pitch, int32_t nq, float query_timestamp, float lambda,
                       int32_t modality_filter, int32_t use_importance, int32_t K,
                       int32_t row_offset, int32_t* d_ids, float* d_vals, int32_t* d_counts,
                       void* stream);
/* mars_scan_topk_f16's filter: *reruns = queries answered again with the
 * fp32 scan because their candidate list overflowed (heavy ties, or a query
 * too large for the bound), over the context's life; *max_candidates and
 * *max_survivors = the largest candidate list and the largest number of rows
 * rescored in fp32 for one query of the last call (-1: overflow).  Any
 * pointer may be NULL. */
int mars_query_ctx_f16_stats(const mars_query_ctx* ctx, uint64_t* reruns, int32_t* max_candidates,
                             int32_t* max_survivors);

/* Merge `n_lists` ranked lists of K (id, score) pairs that sit back to back
 * in device memory (e.g. the gather buffer of an all-gather of per-shard
 * mars_scan_topk results) into one ranked list of K.  Ties by id. */
int mars_topk_merge(mars_query_ctx* ctx, const int32_t* d_ids_in,
                    const float* d_vals_in, int32_t n_lists, int32_t K,
                    int32_t* d_ids_out, float* d_vals_out, int32_t* d_count,
                    void* stream);

/* Batched form for Q queries: list l of query q starts at (l*Q + q)*K (the
 * rank-major layout of an all-gather of per-rank [Q][K] buffers); outputs
 * are [Q][K] and d_counts[Q] (may be NULL). */
int mars_topk_merge_batch(mars_query_ctx* ctx, const int32_t* d_ids_in,
                          const float* d_vals_in, int32_t n_lists, int32_t K,
                          int32_t Q, int32_t* d_ids_out, float* d_vals_out,
                          int32_t* d_counts, void* stream);

/* compute_novelty (include/memory_cuda.cuh:217-222,
 * src/memory_cuda.cu:1232-1290): the largest dot(E_i, q) over all rows,
 * written to *d_max (device float) -- the fused scan with K = 1, no decay,
 * no filter; no N-sized buffer and no host round trip. */
int mars_novelty(const mars_store* s, mars_query_ctx* ctx, const float* d_query,
                 float* d_max, void* stream);

/* ---- batched queries on the tensor cores --------------------------------
 * No reference counterpart: the reference answers one query per call
 * (query_memory_fast, include/memory_cuda.cuh:188); a batch of B queries there
 * costs B full passes over the embeddings.  Here the scores of 128 queries x
 * 256 rows are formed per tcgen05 tile (TF32 inputs, fp32 accumulation), rows
 * that can still reach a query's top-K are short-listed with a proven error
 * margin, and the short list is rescored in exact fp32 with the arithmetic of
 * mars_scan_topk -- so each query's result equals mars_scan_topk's for it.
 * Queries whose short list cannot be proven complete are recomputed with
 * mars_scan_topk (counted in mars_batch_stats.fallbacks). */
typedef struct mars_batch_ctx mars_batch_ctx;

typedef struct mars_batch_stats {
    int32_t path;            /* 3: tensor cores, fp16 operands, small-batch tiles
                                (128 rows x B queries, B <= 64); 2: tensor cores,
                                fp16 operands (128 queries x 256 rows); 1: tensor
                                cores, TF32; 0: per-query scans (small N) */
    int32_t fallbacks;       /* queries recomputed exactly                         */
    int64_t candidates;      /* short-listed (query, row) pairs                    */
    int32_t max_candidates;  /* largest short list of one query                    */
    int32_t sample_tiles;    /* 256-row tiles in the threshold sample              */
    int32_t sample_rank;     /* rank of the sampled bound used as threshold        */
    int64_t rescored;        /* candidates rescored exactly after pruning          */
    float   gemm_ms;         /* device time of the candidates pass (CUDA events on
                                the call's stream; 0 on the scan path)             */
} mars_batch_stats;

int mars_batch_ctx_create(int32_t device, int32_t max_nodes, int32_t dim,
                          int32_t max_batch, int32_t max_k, mars_batch_ctx** out);
int mars_batch_ctx_destroy(mars_batch_ctx* ctx);

/* Operand precision of the batched tensor-core short list.  By default the
 * GEMM runs on fp16 copies of the rows and queries (kind::f16: twice the
 * TF32 rate and half the bytes, the same 10 mantissa bits, so the same
 * proven error margin plus an absolute term for values below the fp16
 * normal range); stores or queries with a component beyond 60000 use TF32.
 * tf32_only != 0 always uses TF32 operands.  Either way the final scores are
 * exact fp32 and the results identical.  The fp16 copy of a store is made on
 * its first batched query (2 bytes per value) and kept current. */
int mars_batch_ctx_set_precision(mars_batch_ctx* ctx, int32_t tf32_only);

/* Small batches (B <= 64 on fp16 operands): enable != 0 (the default on
 * devices with cooperative launch) runs the sample pass, the thresholds and
 * the candidates pass as one cooperative launch; 0 runs them as three
 * launches.  The results are the same. */
int mars_batch_ctx_set_single_launch(mars_batch_ctx* ctx, int32_t enable);

/* d_queries: B rows of query_pitch floats (16-byte aligned; values past dim
 * must be zero).  One query time t_q for the whole batch.  Outputs d_ids /
 * d_vals: [B][K] (ids offset by row_offset), d_counts: [B] (may be NULL).
 * Asynchronous on `stream`: a query whose short list cannot be proven
 * complete, or with a component outside the fp16 range, is rescanned exactly
 * on the device in the same stream (mars_batch_stats.fallbacks).  A
 * pipeline error of a call (a bounded device-side wait that gave up) is
 * returned as MARS_ERR_TIMEOUT by mars_batch_last_stats or by the next call;
 * the failed call's results are not served: every count is -1, every id -1
 * and every score -inf. */
int mars_query_batch_topk(const mars_store* s, mars_batch_ctx* ctx,
                          const float* d_queries, int32_t query_pitch, int32_t B,
                          float query_timestamp, float lambda,
                          int32_t modality_filter, int32_t use_importance,
                          int32_t K, int32_t row_offset, int32_t* d_ids,
                          float* d_vals, int32_t* d_counts, void* stream);

/* Statistics of the last mars_query_batch_topk call (waits for it). */
int mars_batch_last_stats(const mars_batch_ctx* ctx, mars_batch_stats* out);

/* Test hook for the bounded grid-wide wait of the single-launch small-batch
 * path (no reference counterpart).  spin_limit bounds the polls of that wait
 * (0: the default, about 2^26 polls of >= 128 ns); extra_arrivals > 0 makes
 * the next call wait for that many arrivals more than its CTAs make, so its
 * wait cannot end and gives up after spin_limit polls.  That call's results
 * are then marked invalid and its status is MARS_ERR_TIMEOUT; the call after
 * it runs normally. */
int mars_batch_ctx_debug_wait(mars_batch_ctx* ctx, uint32_t spin_limit, int32_t extra_arrivals);

/* ---- row shards across GPUs ---------------------------------------------
 * No reference counterpart: the reference runs on one GPU and lists
 * multi-GPU sharding as future work (NEXT_STEPS.md:31).  One process per GPU;
 * rank r holds rows [offset_r, offset_r + n_r) of the corpus in its own
 * store.  The library owns an NCCL communicator (libnccl.so.2, loaded at run
 * time: the copy already in the process, else the system's).  Rank 0 makes a
 * unique id with mars_shard_unique_id and the caller hands its
 * MARS_SHARD_ID_BYTES bytes to every rank (any channel), then every rank
 * creates its communicator. */
#define MARS_SHARD_ID_BYTES 128
typedef struct mars_shard_comm mars_shard_comm;

int mars_shard_unique_id(void* id_out);
/* Collective over the `world` ranks (blocks until all have joined).  Calls
 * on it take B <= max_batch queries and K <= max_k; world x max_k <= 4096.
 * The NCCL communicator is non-blocking: its creation, the set-up NCCL does
 * on a first use and its teardown are polled (ncclCommGetAsyncError)
 * against a deadline -- MARS_SHARD_DEFAULT_TIMEOUT_MS here, timeout_ms with
 * the _timeout form (0: none) -- and a rank that never joins ends the call
 * with MARS_ERR_TIMEOUT (the half-made communicator is aborted) instead of
 * waiting for ever. */
#define MARS_SHARD_DEFAULT_TIMEOUT_MS 600000
int mars_shard_comm_create(int32_t device, int32_t rank, int32_t world, const void* unique_id,
                           int32_t max_batch, int32_t max_k, mars_shard_comm** out);
int mars_shard_comm_create_timeout(int32_t device, int32_t rank, int32_t world, const void* unique_id,
                                   int32_t max_batch, int32_t max_k, int32_t timeout_ms,
                                   mars_shard_comm** out);
/* Waits for the device, then frees the communicator.  NULL is accepted. */
int mars_shard_comm_destroy(mars_shard_comm* comm);
/* MARS_OK, or the communicator's asynchronous NCCL error (a peer that failed
 * or left); after an error, mars_shard_comm_abort ends the communicator so
 * that no rank waits for the others any longer, then destroy it. */
int mars_shard_comm_status(mars_shard_comm* comm);
int mars_shard_comm_abort(mars_shard_comm* comm);
/* Optional: record events around the call's three phases (local pipeline
 * with the bound exchange / all-gather / merge); mars_shard_last_times waits
 * for the last call and returns their device times in ms. */
int mars_shard_comm_set_timing(mars_shard_comm* comm, int32_t enable);
int mars_shard_last_times(mars_shard_comm* comm, float* local_ms, float* gather_ms, float* merge_ms);
/* A communicator of one rank answers mars_shard_query_batch_topk with the
 * single-store pipeline (its local answer is the merged one).  Test hook:
 * enable = 1 makes it run the whole exchange protocol instead (records,
 * NCCL all-gathers, merge), so one GPU can check that path against the
 * single-store call. */
int mars_shard_comm_set_exchange_at_world1(mars_shard_comm* comm, int32_t enable);

/* mars_query_batch_topk over a row-sharded corpus, called by every rank with
 * the same queries, B, K, t_q, lambda, filter and use_importance (a
 * collective).  s: this rank's shard; row_offset: its first global row.
 * Outputs on every rank: the global top-K [B][K] (global ids), d_counts [B].
 * Each shard runs the batched tensor-core pipeline with three NCCL
 * all-gathers: after the sample pass, every shard's best sampled lower
 * bounds per query (B x 16 floats per rank), from which all shards take one
 * short-list threshold (the level a sample of the whole corpus gives);
 * between the two rescore passes, per query the count of candidates whose
 * lower bound reaches it and two lower-bound order statistics (3 B + 1
 * floats per rank), which certify the short lists over all shards and give
 * every shard a bound of the global K-th score, so a shard rescores only
 * rows that can still place; and B x K packed 64-bit keys (score, then id),
 * followed by a per-query selection on every rank.  The
 * results equal mars_query_batch_topk over the whole corpus on one GPU, bit
 * for bit.  Asynchronous on `stream` (NULL: the batch context's stream).  If
 * any rank's call fails (an argument, or a bounded device wait that gave
 * up), every rank's results of that call are marked invalid (counts -1, ids
 * -1) and the failing rank returns the error; ranks still take every
 * collective step. */
int mars_shard_query_batch_topk(const mars_store* s, mars_batch_ctx* ctx, mars_shard_comm* comm,
                                const float* d_queries, int32_t query_pitch, int32_t B,
                                float query_timestamp, float lambda, int32_t modality_filter,
                                int32_t use_importance, int32_t K, int32_t row_offset,
                                int32_t* d_ids, float* d_vals, int32_t* d_counts, void* stream);

/* Test hook, no reference counterpart: mars_shard_query_batch_topk over
 * `world` row shards that all live on ONE GPU (stores[r] holds global rows
 * [row_offsets[r], row_offsets[r] + n_r), ctxs[r] is its batch context),
 * each shard's pipeline on its own host thread and its context's stream,
 * with the three all-gathers replaced by device copies between the shards'
 * buffers (host barriers order them; no kernel waits on another).  The same
 * code runs for every shard as under NCCL, so the merged answer in d_ids /
 * d_vals / d_counts ([B][K], [B]) shows what `world` GPUs would return.
 * Blocks until the answer is written.  world <= 16. */
int mars_shard_emulate_query_batch_topk(int32_t world, const mars_store* const* stores,
                                        mars_batch_ctx* const* ctxs, const int32_t* row_offsets,
                                        const float* d_queries, int32_t query_pitch, int32_t B,
                                        float query_timestamp, float lambda, int32_t modality_filter,
                                        int32_t use_importance, int32_t K, int32_t* d_ids, float* d_vals,
                                        int32_t* d_counts);

/* query_memory_fast (include/memory_cuda.cuh:188-194, src/memory_cuda.cu:
 * 1069-1158) over a row-sharded corpus, one process per GPU (a collective:
 * every rank calls it with the same query, t_q and cfg).  s: this rank's rows,
 * global ids [row_offset, row_offset + N_r); d_row_offsets / d_col_indices:
 * the CSR over all n_global rows in global ids (device arrays replicated on
 * every rank; NULL allowed without BFS hops).  The answer -- the same as
 * mars_query on one GPU holding every row and that graph -- lands in `out`
 * (host, cfg->top_k entries) on every rank: the local top-K seeds merged with
 * one all-gather; per BFS level, every rank expands the level over the
 * replicated graph and one all-reduce gives every node's own score from the
 * rank that holds its row; the results' modalities come from their owners.
 * Limits: 16384 nodes per level and in total (MARS_ERR_CAPACITY beyond),
 * top_k <= the communicator's max_k, D % 4 == 0.  Blocks until the results
 * are on the host.  A rank whose part fails still takes every collective
 * step; every rank then returns an error. */
int mars_shard_query(const mars_store* s, mars_query_ctx* ctx, mars_shard_comm* comm,
                     const int32_t* d_row_offsets, const int32_t* d_col_indices, int32_t n_global,
                     const float* query, float query_timestamp, const mars_retrieval_config* cfg,
                     int32_t row_offset, mars_query_result* out, int32_t* n_out);

/* ---- CMNG kNN graph (include/cmng.cuh) --------------------------------- */

/* CMNGSearchConfig, include/cmng.cuh:54-62 (bools widened to int32). */
typedef struct mars_cmng_config {
    int32_t K;
    int32_t beam_width;
    int32_t max_iterations;
    int32_t num_parents;
    float   time_decay_lambda;
    int32_t modality_filter;   /* accepted, unused (as in the reference) */
    int32_t use_fp16;          /* accepted, unused: fp32 rows are scored */
} mars_cmng_config;

/* build_cmng (include/cmng.cuh:91-96, src/cmng_build.cu:135-255) over the
 * store's rows: for every row the k_init = 2*degree nearest other rows by
 * dot product (exact fp32, ties by id), then the first degree-degree_cross of
 * them and, for every modality m < num_modalities other than the row's own,
 * the nearest kNN entry of modality m (or -1); -1 padding.  The reference
 * fixes num_modalities = 3 (src/cmng_build.cu:234).  d_neighbors: device
 * N x degree int32.  build_ms (may be NULL) receives the device time. */
int mars_cmng_build(const mars_store* s, int32_t degree, int32_t degree_cross,
                    int32_t num_modalities, int32_t* d_neighbors, float* build_ms);

/* The same neighbour lists for rows first .. first + count - 1 only (each
 * still searched against every row of the store), written to d_neighbors as
 * count x degree.  Row blocks built on several GPUs that each hold the whole
 * store, then gathered, equal mars_cmng_build: the N x N product of
 * src/cmng_build.cu:203-246 split by row blocks. */
int mars_cmng_build_rows(const mars_store* s, int32_t first, int32_t count, int32_t degree,
                         int32_t degree_cross, int32_t num_modalities, int32_t* d_neighbors,
                         float* build_ms);

/* The exact k nearest other rows of every row (the kNN lists of the build):
 * d_ids / d_vals: N x k (dot desc, id asc), d_counts: N (may be NULL). */
int mars_cmng_knn(const mars_store* s, int32_t k, int32_t* d_ids, float* d_vals,
                  int32_t* d_counts);

/* cmng_search (include/cmng.cuh:112-118, src/cmng_search.cu:110-308) for nq
 * queries at once (the reference answers one per launch).  d_queries: nq
 * rows of query_pitch floats; outputs [nq][K] ids, decayed scores, modalities
 * (d_mods may be NULL), d_counts[nq]; d_iters / d_scored (may be NULL)
 * receive the expansions and distinct rows scored per query. */
int mars_cmng_search_batch(const mars_store* s, const int32_t* d_neighbors,
                           int32_t degree, const float* d_queries,
                           int32_t query_pitch, int32_t nq, float query_timestamp,
                           const mars_cmng_config* cfg, int32_t* d_ids,
                           float* d_scores, int32_t* d_mods, int32_t* d_counts,
                           int32_t* d_iters, int32_t* d_scored, void* stream);

/* cmng_search followed by a cross-modal BFS (no reference counterpart: the
 * reference's cmng_search stops at the beam, src/cmng_search.cu:110-308).
 * The beam's top-K (decayed scores) seed a BFS of bfs_hops levels over the
 * CMNG adjacency with the canonical rule of mars_query: a node's score is the
 * best fmaxf(parent * bfs_score_decay, own * 0.8f) over its parents one level
 * up, own = dot x __expf(-lambda * age) [x importance]; the result is the
 * top-K of all visited nodes by (score desc, id asc).  The context holds the
 * per-block visited tables (sized for K x (1 + degree + ... + degree^hops)). */
typedef struct mars_cmng_ctx mars_cmng_ctx;

int mars_cmng_ctx_create(int32_t device, int32_t max_queries, int32_t K, int32_t degree,
                         int32_t bfs_hops, int32_t max_nodes, mars_cmng_ctx** out);
int mars_cmng_ctx_destroy(mars_cmng_ctx* ctx);
/* The BFS keeps each query's visited set in shared memory while it holds at
 * most max_nodes nodes (default and limit 2048); a query that visits more is
 * answered again with the context's global-memory tables, with the same
 * result.  0: global tables only.  Tests use it to compare the two. */
int mars_cmng_ctx_set_bfs_smem_nodes(mars_cmng_ctx* ctx, int32_t max_nodes);

int mars_cmng_search_bfs_batch(const mars_store* s, mars_cmng_ctx* ctx,
                               const int32_t* d_neighbors, int32_t degree,
                               const float* d_queries, int32_t query_pitch, int32_t nq,
                               float query_timestamp, const mars_cmng_config* cfg,
                               int32_t bfs_hops, float bfs_score_decay,
                               int32_t use_importance, int32_t* d_ids, float* d_scores,
                               int32_t* d_mods, int32_t* d_hops, int32_t* d_counts,
                               int32_t* d_visited, void* stream);

/* Fused scan top-K that allocates nothing.  No counterpart in the reference:
 * it exists for callers that may not call cudaMalloc -- processes that
 * reserve all GPU memory up front (for example a real-time loop whose memory
 * budget is fixed before its deadline-bound phase) or hosts that forbid a
 * library from growing their footprint.  The caller passes its own device
 * arrays (embeddings with a row pitch in floats, timestamps, optional
 * importance and modalities, the query; all 16-byte aligned rows) and the
 * outputs (d_ids / d_vals: K entries, d_count may be NULL); results equal
 * mars_scan_topk's.  Working memory is a library-owned device array of
 * MARS_NOALLOC_SCRATCH_BYTES that every GPU loading the library holds until
 * exit; K above MARS_NOALLOC_MAX_K is rejected with MARS_ERR_CAPACITY.  The
 * first call on a device sets it up: it looks the array up
 * (cudaGetSymbolAddress) and loads every kernel this entry point can launch,
 * which is when the library's code and the array take their place in device
 * memory under lazy module loading (the CUDA default).  Make that first call
 * (any K, any D) before reserving the rest of the device memory and before
 * any stream capture, or run with CUDA_MODULE_LOADING=EAGER; later calls
 * load nothing.  All calls share the array, so calls that overlap on the
 * GPU race; serialise them.  Works on the current device. */
#define MARS_NOALLOC_MAX_K 128
#define MARS_NOALLOC_SCRATCH_BYTES 524548
int mars_scan_topk_noalloc(const float* d_embeddings, int32_t row_pitch,
                           const float* d_timestamps, const float* d_importance,
                           const int32_t* d_modalities, int32_t n, int32_t dim,
                           const float* d_query, float query_timestamp,
                           float lambda, int32_t modality_filter,
                           int32_t use_importance, int32_t K,
                           int32_t row_offset, int32_t* d_ids, float* d_vals,
                           int32_t* d_count, void* stream);

/* Diagnostic: the fused score of every row (same arithmetic as the scan),
 * d_out: N floats, -FLT_MAX for rows rejected by the filter. */
int mars_debug_fused_scores(const mars_store* s, mars_query_ctx* ctx,
                            const float* d_query, float query_timestamp,
                            float lambda, int32_t modality_filter,
                            int32_t use_importance, float* d_out,
                            void* stream);

/* Replay the host-facing mars_query as one CUDA graph (default on; the
 * reference's QueryContext::use_cuda_graph, include/memory_cuda.cuh:163).
 * Calls that request stats always run the kernels directly so the stage
 * timings are real. */
int mars_query_ctx_use_graph(mars_query_ctx* ctx, int32_t enable);

/* Answer mars_query with one kernel launch when top_k <= 64 and dim <= 1024
 * (default on): the query vector travels in the launch's parameter block,
 * the last CTA of the scan also runs the BFS and ranks the visited set, and
 * the results are written straight into mapped host memory.  This replaces
 * the 6-9 launches and copies of src/memory_cuda.cu:1069-1158 for one query.
 * A query whose BFS outgrows that CTA (more than 3072 visited nodes or 1024
 * nodes in one level) is answered again by the multi-kernel pipeline; the
 * results are the same either way.  enable = 0 always uses the pipeline. */
int mars_query_ctx_use_fused(mars_query_ctx* ctx, int32_t enable);

/* Number of mars_query calls answered by a single launch (the fused query
 * kernel, or the fp16-filtered scan for large hop-free queries), and of those
 * that had to be answered again by the pipeline.  Either pointer may be NULL. */
int mars_query_ctx_path_counts(const mars_query_ctx* ctx, uint64_t* fused, uint64_t* reruns);

/* The context's CUDA stream (cudaStream_t as void*). */
void* mars_query_ctx_stream(mars_query_ctx* ctx);

#ifdef __cplusplus
}
#endif
#endif /* MARS_B200_H */
