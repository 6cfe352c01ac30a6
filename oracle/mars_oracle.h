/*
 * mars_oracle.h -- CPU restatement of the MARS retrieval path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (the CUDA library under
 * cuda-multimodal-memory_b200/) links, calls or falls back to this code.  It is
 * used by tests/ as the parity checker, by __graft_entry__.smoke() as the
 * checker of one small GPU call, and by bench.py's cpu_baseline / reference arm
 * as the timed CPU implementation of the path.
 *
 * Every function restates the algorithm of a reference function; the
 * reference file:line is given beside each declaration (paths are relative to
 * the root of antonellof/cuda-multimodal-memory).
 *
 * Parity pin: the restatement is checked against golden vectors produced by
 * the reference's own CPU pipeline (scripts/bench_cpu.py:91-146, imported and
 * run by tests/golden/make_golden.py) and against outputs of the reference's
 * GPU path rebuilt from its sources (oracle/ref_shim.cu, run on the GPU box).
 */
#ifndef MARS_ORACLE_H
#define MARS_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- dot-product summation orders ------------------------------------
 * fp32 dot products are not associative, so every order used anywhere in
 * the build is named and restated exactly here.                          */
enum {
    /* The order of the B200 kernels in this repository: lane l (0..31) of a
     * warp owns float4 chunks c = l, l+32, ... of the row and accumulates them
     * with fmaf in component order x,y,z,w; the 32 lane sums are then
     * combined by an xor butterfly with offsets 16,8,4,2,1.                   */
    ORC_DOT_CANONICAL = 0,
    /* Plain sequential fp32 multiply-then-add (src/latency_bench.cu:146-160). */
    ORC_DOT_SEQ = 1,
    /* Double accumulation rounded once (src/validate.cu:124-139).            */
    ORC_DOT_F64 = 2,
    /* cosine_similarity_kernel: 256 threads, thread t sums d = t, t+256, ...
     * with FMA, shfl_down tree inside each warp, then a shfl_down tree over
     * the 8 warp sums (src/memory_cuda.cu:50-93).                            */
    ORC_DOT_REF_BLOCK256 = 3,
    /* warp_dot_product: lane-strided FMA then a shfl_down tree
     * (src/cmng_search.cu:59-70).                                            */
    ORC_DOT_REF_WARP = 4,
    /* Vectorised fp32 (AVX2 FMA, 4x8 partial sums) for timed CPU baselines. */
    ORC_DOT_FAST = 5
};

float orc_dot(const float* a, const float* b, int32_t D, int32_t order);

/* L2 normalisation exactly as engine_server's add_node
 * (src/engine_server.cu:165-171): sequential fp32 sum of squares,
 * sqrtf, + 1e-8f, element-wise division.                                  */
void orc_l2_normalize(float* v, int32_t D);

/* ---- corpus ----------------------------------------------------------- */
typedef struct orc_corpus {
    int32_t        N;            /* rows                                          */
    int32_t        D;            /* embedding dimension                           */
    int64_t        pitch;        /* floats between consecutive rows (>= D)        */
    const float*   E;            /* N * pitch, row-major                          */
    const float*   ts;           /* N timestamps (seconds)                        */
    const float*   imp;          /* N importance weights, or NULL (= 1)           */
    const int32_t* mod;          /* N modality ids                                */
    /* CSR graph (may be NULL when no BFS is run)                                 */
    const int32_t* row_offsets;  /* N + 1                                          */
    const int32_t* col_indices;  /* row_offsets[N]                                 */
    /* optional per-node append-only adjacency used by streaming inserts:
     * node u's extra neighbours are extra_nbrs[u*extra_stride + 0..extra_cnt[u]-1] */
    const int32_t* extra_nbrs;
    const int32_t* extra_cnt;
    int32_t        extra_stride;
    /* optional fixed-degree adjacency (CMNG layout, -1 = empty slot); used by
     * the BFS that follows cmng_search when row_offsets is NULL              */
    const int32_t* fixed_nbrs;
    int32_t        fixed_degree;
} orc_corpus;

typedef struct orc_config {
    int32_t top_k;             /* RetrievalConfig::top_k            */
    int32_t bfs_max_hops;      /* RetrievalConfig::bfs_max_hops     */
    float   lambda;            /* RetrievalConfig::time_decay_lambda */
    float   bfs_score_decay;   /* RetrievalConfig::bfs_score_decay  */
    int32_t modality_filter;   /* RetrievalConfig::modality_filter  */
    int32_t use_importance;    /* multiply by importance (north-star extension) */
    int32_t dot_order;         /* ORC_DOT_*                          */
} orc_config;

/* QueryResult (include/memory_cuda.cuh:85-90) */
typedef struct orc_result {
    int32_t node_id;
    float   score;
    int32_t modality;
    int32_t hops;
} orc_result;

/* Fused per-row score: dot(E_i, q) * __expf(-lambda * max(0, t_q - ts_i))
 * [* imp_i]; rows rejected by the modality filter get -FLT_MAX
 * (src/memory_cuda.cu:50-93 and :292-310).                                */
void orc_fused_scores(const orc_corpus* c, const float* q, float t_q,
                      float lambda, int32_t modality_filter,
                      int32_t use_importance, int32_t dot_order,
                      float* out_final);

/* Top-K by (score desc, id asc) over the rows that pass the modality filter
 * (the CUB path, src/memory_cuda.cu:972-1000, sorts -score stably so equal
 * scores come out in ascending id).  Returns min(K, eligible rows).        */
int32_t orc_topk(const float* scores, const int32_t* mod,
                 int32_t modality_filter, int32_t N, int32_t K,
                 int32_t* out_ids, float* out_vals);

/* Canonical level-synchronous BFS (src/memory_cuda.cu:450-469 seeds,
 * :478-514 expansion): hop[u] = BFS distance <= hops from the seed set;
 * score[u] = max over parents p one level up of
 * fmaxf(score[p] * hop_decay, final[u] * 0.8f); seeds keep their seed value.
 * The reference resolves concurrent parents with atomicCAS (first claimer
 * wins); the canonical rule takes the best parent and does not cap the
 * frontier.  final[u] comes from final_scores when it is not NULL, else it
 * is computed for the visited nodes only from sp.  Writes visited nodes
 * ordered by (hop, id) and returns their count (-1 if max_visited is too
 * small).                                                                  */
typedef struct orc_score_params {   /* how final[u] is computed on demand */
    const float* q;
    float        t_q;
    float        lambda;
    int32_t      modality_filter;
    int32_t      use_importance;
    int32_t      dot_order;
} orc_score_params;

int32_t orc_bfs(const orc_corpus* c, const int32_t* seed_ids,
                const float* seed_vals, int32_t n_seeds,
                const float* final_scores, const orc_score_params* sp,
                int32_t hops, float hop_decay,
                orc_result* out_visited, int32_t max_visited);

/* Final ordering (src/memory_cuda.cu:1127-1146): sort by (score desc,
 * id asc), keep the first K.  Returns the kept count.                     */
int32_t orc_finalize(orc_result* visited, int32_t n, int32_t K);

/* Whole query_memory_fast pipeline (src/memory_cuda.cu:924-1158):
 * fused scores -> top-K -> BFS -> finalize.  out must hold cfg->top_k.
 * Returns the number of results.                                          */
int32_t orc_query(const orc_corpus* c, const float* q, float t_q,
                  const orc_config* cfg, orc_result* out);

/* Batched top-K without BFS (multi-query scoring): for each of B queries the
 * top-K of the fused score.  Uses up to n_threads OpenMP threads.         */
void orc_query_batch_topk(const orc_corpus* c, const float* Q, int32_t B,
                          float t_q, float lambda, int32_t modality_filter,
                          int32_t use_importance, int32_t K,
                          int32_t dot_order, int32_t n_threads,
                          int32_t* out_ids, float* out_vals);

/* Fast multi-threaded fused scan + top-K used as the timed CPU baseline.
 * Same contract as orc_fused_scores + orc_topk, but the dot product uses
 * vectorised fp32 partial sums (ORC_DOT_FAST), so scores may differ from
 * the canonical order in the last bits.  Returns count.                   */
int32_t orc_scan_topk_fast(const orc_corpus* c, const float* q, float t_q,
                           float lambda, int32_t modality_filter,
                           int32_t use_importance, int32_t K,
                           int32_t n_threads, int32_t* out_ids,
                           float* out_vals);

/* Exact kNN (the intended result of build_cmng's SGEMM tiles + insertion
 * merge, src/cmng_build.cu:28-71 and :195-230): for each listed row i, the k
 * rows j != i with the largest dot(E_i, E_j), ties by ascending j.        */
void orc_knn(const orc_corpus* c, const int32_t* rows, int32_t n_rows,
             int32_t k, int32_t dot_order, int32_t n_threads,
             int32_t* out_ids, float* out_vals);

/* Neighbour selection with cross-modal bridges (src/cmng_build.cu:75-132):
 * first (degree - degree_cross) valid kNN ids, -1 padded, then for every
 * other modality m < num_modalities the first kNN entry of modality m
 * (or -1), then -1 padding.                                               */
void orc_cmng_select(const int32_t* knn_ids, int32_t k_init,
                     const int32_t* mod, int32_t N, const int32_t* rows,
                     int32_t n_rows, int32_t degree, int32_t degree_cross,
                     int32_t num_modalities, int32_t* out_neighbors);

/* cmng_search configuration (include/cmng.cuh:54-62) */
typedef struct orc_cmng_config {
    int32_t K;
    int32_t beam_width;
    int32_t max_iterations;
    int32_t num_parents;
    float   lambda;
    int32_t dot_order;
} orc_cmng_config;

typedef struct orc_cmng_stats {
    int32_t iterations;    /* expansions performed                 */
    int32_t rows_scored;   /* distinct rows whose dot was computed  */
} orc_cmng_stats;

/* Greedy beam search (src/cmng_search.cu:110-308), restated step by step:
 * seeds from the bits of q[0], q[1]; iteration t expands the node at beam
 * position t (the reference flags positions, not nodes); unvisited
 * neighbours are scored and merged into the beam; finally the beam is
 * decayed and the top K selected.  The visited set is exact: the
 * reference's 8192-slot hash gives up after 32 probes and then neither
 * records the node nor reports it as new, which only happens near overflow.
 * A duplicate id inside one neighbour list is scored once, at its first
 * occurrence (the reference's warps race on it).  Returns count.          */
int32_t orc_cmng_search(const orc_corpus* c, const int32_t* neighbors,
                        int32_t degree, const float* q, float t_q,
                        const orc_cmng_config* cfg, orc_result* out,
                        orc_cmng_stats* stats);

#ifdef __cplusplus
}
#endif
#endif /* MARS_ORACLE_H */
