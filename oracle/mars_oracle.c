/*
 * mars_oracle.c -- CPU restatement of the MARS retrieval path.
 *
 * TEST INFRASTRUCTURE ONLY (see mars_oracle.h).  Compiled with
 * -ffp-contract=off so that every multiply-add is exactly the one written:
 * fmaf() where the restated code fuses, a separate multiply and add where it
 * does not.
 */
#include "mars_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

#if defined(__AVX2__) && defined(__FMA__)
#include <immintrin.h>
#define ORC_HAVE_AVX2 1
#endif
#ifdef _OPENMP
#include <omp.h>
#endif

/* ======================================================================
 * Dot products
 * ====================================================================== */

/* Canonical order of this repository's kernels (mars_dot_canonical in
 * cuda-multimodal-memory_b200/csrc/mars_common.cuh).  Elements past D inside
 * the last float4 chunk are zero on the device (rows are zero padded), so
 * they are fused as fmaf(0, 0, acc) here too.                              */
static float dot_canonical(const float* a, const float* b, int32_t D)
{
    float lane[32], tmp[32];
    const int32_t nc = (D + 3) / 4;
    for (int l = 0; l < 32; ++l) {
        float acc = 0.0f;
        for (int32_t c = l; c < nc; c += 32) {
            for (int k = 0; k < 4; ++k) {
                const int32_t d = 4 * c + k;
                const float x = d < D ? a[d] : 0.0f;
                const float y = d < D ? b[d] : 0.0f;
                acc = fmaf(x, y, acc);
            }
        }
        lane[l] = acc;
    }
    for (int off = 16; off >= 1; off >>= 1) {
        for (int l = 0; l < 32; ++l) tmp[l] = lane[l] + lane[l ^ off];
        memcpy(lane, tmp, sizeof(lane));
    }
    return lane[0];
}

/* __shfl_down_sync tree over 32 lanes; lane 0's value is returned.  Lanes
 * whose source is out of range read their own value (CUDA semantics).     */
static float shfl_down_tree(float* v, int width_log2)
{
    float tmp[32];
    for (int off = 1 << (width_log2 - 1); off >= 1; off >>= 1) {
        for (int l = 0; l < 32; ++l) tmp[l] = v[l] + (l + off < 32 ? v[l + off] : v[l]);
        memcpy(v, tmp, sizeof(tmp));
    }
    return v[0];
}

/* src/memory_cuda.cu:50-93 (cosine_similarity_kernel, 256 threads). */
static float dot_ref_block256(const float* a, const float* b, int32_t D)
{
    float part[256];
    for (int t = 0; t < 256; ++t) {
        float p = 0.0f;
        for (int32_t d = t; d < D; d += 256) p = fmaf(a[d], b[d], p);
        part[t] = p;
    }
    float warp_sums[8];
    for (int w = 0; w < 8; ++w) {
        float v[32];
        memcpy(v, part + 32 * w, sizeof(v));
        warp_sums[w] = shfl_down_tree(v, 5);
    }
    /* warp 0: lanes 0..7 hold the warp sums, the rest 0; offsets 4, 2, 1 */
    float v[32];
    for (int l = 0; l < 32; ++l) v[l] = l < 8 ? warp_sums[l] : 0.0f;
    return shfl_down_tree(v, 3);
}

/* src/cmng_search.cu:59-70 (warp_dot_product). */
static float dot_ref_warp(const float* a, const float* b, int32_t D)
{
    float v[32];
    for (int l = 0; l < 32; ++l) {
        float s = 0.0f;
        for (int32_t d = l; d < D; d += 32) s = fmaf(a[d], b[d], s);
        v[l] = s;
    }
    return shfl_down_tree(v, 5);
}

/* src/latency_bench.cu:146-160 (cpu_topk): sequential multiply then add. */
static float dot_seq(const float* a, const float* b, int32_t D)
{
    float s = 0.0f;
    for (int32_t d = 0; d < D; ++d) {
        const float p = a[d] * b[d];
        s = s + p;
    }
    return s;
}

/* src/validate.cu:124-139 (cpu_top_k): double accumulation. */
static float dot_f64(const float* a, const float* b, int32_t D)
{
    double s = 0.0;
    for (int32_t d = 0; d < D; ++d) s += (double)a[d] * (double)b[d];
    return (float)s;
}

/* Vectorised fp32 dot for timed CPU baselines. */
static float dot_fast(const float* a, const float* b, int32_t D)
{
    int32_t d = 0;
    float s = 0.0f;
#ifdef ORC_HAVE_AVX2
    __m256 acc0 = _mm256_setzero_ps(), acc1 = _mm256_setzero_ps();
    __m256 acc2 = _mm256_setzero_ps(), acc3 = _mm256_setzero_ps();
    for (; d + 32 <= D; d += 32) {
        acc0 = _mm256_fmadd_ps(_mm256_loadu_ps(a + d), _mm256_loadu_ps(b + d), acc0);
        acc1 = _mm256_fmadd_ps(_mm256_loadu_ps(a + d + 8), _mm256_loadu_ps(b + d + 8), acc1);
        acc2 = _mm256_fmadd_ps(_mm256_loadu_ps(a + d + 16), _mm256_loadu_ps(b + d + 16), acc2);
        acc3 = _mm256_fmadd_ps(_mm256_loadu_ps(a + d + 24), _mm256_loadu_ps(b + d + 24), acc3);
    }
    __m256 acc = _mm256_add_ps(_mm256_add_ps(acc0, acc1), _mm256_add_ps(acc2, acc3));
    float lanes[8];
    _mm256_storeu_ps(lanes, acc);
    for (int k = 0; k < 8; ++k) s += lanes[k];
#endif
    for (; d < D; ++d) s = fmaf(a[d], b[d], s);
    return s;
}

float orc_dot(const float* a, const float* b, int32_t D, int32_t order)
{
    switch (order) {
    case ORC_DOT_CANONICAL:    return dot_canonical(a, b, D);
    case ORC_DOT_SEQ:          return dot_seq(a, b, D);
    case ORC_DOT_F64:          return dot_f64(a, b, D);
    case ORC_DOT_REF_BLOCK256: return dot_ref_block256(a, b, D);
    case ORC_DOT_REF_WARP:     return dot_ref_warp(a, b, D);
    case ORC_DOT_FAST:         return dot_fast(a, b, D);
    default:                   return dot_canonical(a, b, D);
    }
}

/* src/engine_server.cu:165-171 */
void orc_l2_normalize(float* v, int32_t D)
{
    float norm = 0.0f;
    for (int32_t d = 0; d < D; ++d) {
        const float p = v[d] * v[d];
        norm = norm + p;
    }
    norm = sqrtf(norm) + 1e-8f;
    for (int32_t d = 0; d < D; ++d) v[d] = v[d] / norm;
}

/* ======================================================================
 * Fused score, top-K
 * ====================================================================== */

static inline int eligible(const int32_t* mod, int32_t filter, int32_t i)
{
    return filter < 0 || (mod != NULL && mod[i] == filter);
}

/* One row's fused score: src/memory_cuda.cu:50-93 then :292-310. */
static inline float fused_one(const orc_corpus* c, int32_t i, const float* q,
                              float t_q, float lambda, int32_t filter,
                              int32_t use_imp, int32_t order)
{
    if (!eligible(c->mod, filter, i)) return -FLT_MAX;
    const float dot = orc_dot(c->E + (int64_t)i * c->pitch, q, c->D, order);
    const float age = fmaxf(0.0f, t_q - c->ts[i]);
    const float w = expf(-lambda * age);
    float f = dot * w;
    if (use_imp && c->imp != NULL) f = f * c->imp[i];
    return f;
}

void orc_fused_scores(const orc_corpus* c, const float* q, float t_q,
                      float lambda, int32_t modality_filter,
                      int32_t use_importance, int32_t dot_order,
                      float* out_final)
{
    for (int32_t i = 0; i < c->N; ++i)
        out_final[i] = fused_one(c, i, q, t_q, lambda, modality_filter,
                                 use_importance, dot_order);
}

static inline int better(float sa, int32_t ia, float sb, int32_t ib)
{
    return sa > sb || (sa == sb && ia < ib);
}

/* Sorted insertion into a (score desc, id asc) list of capacity K. */
static inline void topk_push(float* vals, int32_t* ids, int32_t* cnt,
                             int32_t K, float s, int32_t id)
{
    int32_t n = *cnt;
    if (n == K && !better(s, id, vals[K - 1], ids[K - 1])) return;
    int32_t pos = n < K ? n : K - 1;
    while (pos > 0 && better(s, id, vals[pos - 1], ids[pos - 1])) {
        vals[pos] = vals[pos - 1];
        ids[pos] = ids[pos - 1];
        --pos;
    }
    vals[pos] = s;
    ids[pos] = id;
    if (n < K) *cnt = n + 1;
}

int32_t orc_topk(const float* scores, const int32_t* mod,
                 int32_t modality_filter, int32_t N, int32_t K,
                 int32_t* out_ids, float* out_vals)
{
    int32_t cnt = 0;
    if (K <= 0) return 0;
    for (int32_t i = 0; i < N; ++i) {
        if (!eligible(mod, modality_filter, i)) continue;
        topk_push(out_vals, out_ids, &cnt, K, scores[i], i);
    }
    return cnt;
}

/* ======================================================================
 * BFS
 * ====================================================================== */

static int cmp_i32(const void* a, const void* b)
{
    const int32_t x = *(const int32_t*)a, y = *(const int32_t*)b;
    return (x > y) - (x < y);
}

typedef struct {
    const int32_t* p;
    int32_t n;
} nbr_span;

/* Neighbours of u: CSR row, then the streaming extra list; or the fixed
 * degree list when there is no CSR.                                       */
static int32_t gather_nbrs(const orc_corpus* c, int32_t u, nbr_span out[2])
{
    int32_t k = 0;
    if (c->row_offsets != NULL) {
        out[k].p = c->col_indices + c->row_offsets[u];
        out[k].n = c->row_offsets[u + 1] - c->row_offsets[u];
        ++k;
    } else if (c->fixed_nbrs != NULL) {
        out[k].p = c->fixed_nbrs + (int64_t)u * c->fixed_degree;
        out[k].n = c->fixed_degree;
        ++k;
    }
    if (c->extra_nbrs != NULL && c->extra_cnt != NULL) {
        out[k].p = c->extra_nbrs + (int64_t)u * c->extra_stride;
        out[k].n = c->extra_cnt[u] < c->extra_stride ? c->extra_cnt[u] : c->extra_stride;
        ++k;
    }
    return k;
}

int32_t orc_bfs(const orc_corpus* c, const int32_t* seed_ids,
                const float* seed_vals, int32_t n_seeds,
                const float* final_scores, const orc_score_params* sp,
                int32_t hops, float hop_decay,
                orc_result* out_visited, int32_t max_visited)
{
    const int32_t N = c->N;
    int32_t* hop = (int32_t*)malloc(sizeof(int32_t) * (size_t)(N > 0 ? N : 1));
    float* score = (float*)malloc(sizeof(float) * (size_t)(N > 0 ? N : 1));
    float* best = (float*)malloc(sizeof(float) * (size_t)(N > 0 ? N : 1));
    int32_t* front = (int32_t*)malloc(sizeof(int32_t) * (size_t)(N > 0 ? N : 1));
    int32_t* next = (int32_t*)malloc(sizeof(int32_t) * (size_t)(N > 0 ? N : 1));
    int32_t nv = 0, nf = 0, rc = 0;
    for (int32_t i = 0; i < N; ++i) hop[i] = -1;

    for (int32_t s = 0; s < n_seeds; ++s) {
        const int32_t u = seed_ids[s];
        if (u < 0 || u >= N || hop[u] != -1) continue;
        hop[u] = 0;
        score[u] = seed_vals[s];
        front[nf++] = u;
    }
    qsort(front, (size_t)nf, sizeof(int32_t), cmp_i32);
    for (int32_t i = 0; i < nf; ++i) {
        if (nv >= max_visited) { rc = -1; goto done; }
        out_visited[nv].node_id = front[i];
        out_visited[nv].score = score[front[i]];
        out_visited[nv].modality = c->mod ? c->mod[front[i]] : 0;
        out_visited[nv].hops = 0;
        ++nv;
    }

    for (int32_t h = 0; h < hops && nf > 0; ++h) {
        int32_t nn = 0;
        for (int32_t i = 0; i < nf; ++i) {
            const int32_t u = front[i];
            const float cand = score[u] * hop_decay;
            nbr_span sp2[2];
            const int32_t ns = gather_nbrs(c, u, sp2);
            for (int32_t k = 0; k < ns; ++k) {
                for (int32_t e = 0; e < sp2[k].n; ++e) {
                    const int32_t v = sp2[k].p[e];
                    if (v < 0 || v >= N) continue;
                    if (hop[v] == -1) {
                        hop[v] = h + 1;
                        best[v] = cand;
                        next[nn++] = v;
                    } else if (hop[v] == h + 1 && cand > best[v]) {
                        best[v] = cand;
                    }
                }
            }
        }
        qsort(next, (size_t)nn, sizeof(int32_t), cmp_i32);
        for (int32_t i = 0; i < nn; ++i) {
            const int32_t v = next[i];
            float fv;
            if (final_scores != NULL)
                fv = final_scores[v];
            else
                fv = fused_one(c, v, sp->q, sp->t_q, sp->lambda, sp->modality_filter,
                               sp->use_importance, sp->dot_order);
            score[v] = fmaxf(best[v], fv * 0.8f);
            if (nv >= max_visited) { rc = -1; goto done; }
            out_visited[nv].node_id = v;
            out_visited[nv].score = score[v];
            out_visited[nv].modality = c->mod ? c->mod[v] : 0;
            out_visited[nv].hops = h + 1;
            ++nv;
        }
        int32_t* t = front; front = next; next = t;
        nf = nn;
    }
    rc = nv;
done:
    free(hop); free(score); free(best); free(front); free(next);
    return rc;
}

static int cmp_result(const void* a, const void* b)
{
    const orc_result* x = (const orc_result*)a;
    const orc_result* y = (const orc_result*)b;
    if (x->score > y->score) return -1;
    if (x->score < y->score) return 1;
    return (x->node_id > y->node_id) - (x->node_id < y->node_id);
}

int32_t orc_finalize(orc_result* visited, int32_t n, int32_t K)
{
    qsort(visited, (size_t)n, sizeof(orc_result), cmp_result);
    return n < K ? n : K;
}

int32_t orc_query(const orc_corpus* c, const float* q, float t_q,
                  const orc_config* cfg, orc_result* out)
{
    const int32_t N = c->N;
    const int32_t K = cfg->top_k;
    if (N <= 0 || K <= 0) return 0;
    float* fin = (float*)malloc(sizeof(float) * (size_t)N);
    int32_t* ids = (int32_t*)malloc(sizeof(int32_t) * (size_t)K);
    float* vals = (float*)malloc(sizeof(float) * (size_t)K);
    orc_result* vis = (orc_result*)malloc(sizeof(orc_result) * (size_t)N);
    orc_fused_scores(c, q, t_q, cfg->lambda, cfg->modality_filter,
                     cfg->use_importance, cfg->dot_order, fin);
    const int32_t ns = orc_topk(fin, c->mod, cfg->modality_filter, N, K, ids, vals);
    int32_t nv = orc_bfs(c, ids, vals, ns, fin, NULL,
                         (c->row_offsets || c->fixed_nbrs) ? cfg->bfs_max_hops : 0,
                         cfg->bfs_score_decay, vis, N);
    int32_t nk = 0;
    if (nv > 0) {
        nk = orc_finalize(vis, nv, K);
        memcpy(out, vis, sizeof(orc_result) * (size_t)nk);
    }
    free(fin); free(ids); free(vals); free(vis);
    return nk;
}

/* ======================================================================
 * Batched scan, fast baseline
 * ====================================================================== */

void orc_query_batch_topk(const orc_corpus* c, const float* Q, int32_t B,
                          float t_q, float lambda, int32_t modality_filter,
                          int32_t use_importance, int32_t K,
                          int32_t dot_order, int32_t n_threads,
                          int32_t* out_ids, float* out_vals)
{
    const int64_t qpitch = c->pitch;
#ifdef _OPENMP
    if (n_threads <= 0) n_threads = omp_get_max_threads();
#pragma omp parallel for schedule(dynamic, 1) num_threads(n_threads)
#endif
    for (int32_t b = 0; b < B; ++b) {
        const float* q = Q + (int64_t)b * qpitch;
        int32_t* ids = out_ids + (int64_t)b * K;
        float* vals = out_vals + (int64_t)b * K;
        int32_t cnt = 0;
        for (int32_t k = 0; k < K; ++k) { ids[k] = -1; vals[k] = -FLT_MAX; }
        for (int32_t i = 0; i < c->N; ++i) {
            if (!eligible(c->mod, modality_filter, i)) continue;
            const float f = fused_one(c, i, q, t_q, lambda, modality_filter,
                                      use_importance, dot_order);
            topk_push(vals, ids, &cnt, K, f, i);
        }
    }
    (void)n_threads;
}

int32_t orc_scan_topk_fast(const orc_corpus* c, const float* q, float t_q,
                           float lambda, int32_t modality_filter,
                           int32_t use_importance, int32_t K,
                           int32_t n_threads, int32_t* out_ids,
                           float* out_vals)
{
    if (K <= 0) return 0;
#ifdef _OPENMP
    if (n_threads <= 0) n_threads = omp_get_max_threads();
#else
    n_threads = 1;
#endif
    float* tv = (float*)malloc(sizeof(float) * (size_t)K * (size_t)n_threads);
    int32_t* ti = (int32_t*)malloc(sizeof(int32_t) * (size_t)K * (size_t)n_threads);
    int32_t* tc = (int32_t*)calloc((size_t)n_threads, sizeof(int32_t));
#ifdef _OPENMP
#pragma omp parallel num_threads(n_threads)
#endif
    {
#ifdef _OPENMP
        const int t = omp_get_thread_num();
        const int nt = omp_get_num_threads();
#else
        const int t = 0, nt = 1;
#endif
        const int64_t lo = (int64_t)c->N * t / nt, hi = (int64_t)c->N * (t + 1) / nt;
        float* v = tv + (int64_t)t * K;
        int32_t* id = ti + (int64_t)t * K;
        int32_t cnt = 0;
        for (int64_t i = lo; i < hi; ++i) {
            if (!eligible(c->mod, modality_filter, (int32_t)i)) continue;
            const float f = fused_one(c, (int32_t)i, q, t_q, lambda, modality_filter,
                                      use_importance, ORC_DOT_FAST);
            if (cnt == K && !better(f, (int32_t)i, v[K - 1], id[K - 1])) continue;
            topk_push(v, id, &cnt, K, f, (int32_t)i);
        }
        tc[t] = cnt;
    }
    int32_t cnt = 0;
    for (int t = 0; t < n_threads; ++t)
        for (int32_t k = 0; k < tc[t]; ++k)
            topk_push(out_vals, out_ids, &cnt, K, tv[(int64_t)t * K + k], ti[(int64_t)t * K + k]);
    free(tv); free(ti); free(tc);
    return cnt;
}

/* ======================================================================
 * kNN graph (cmng_build)
 * ====================================================================== */

void orc_knn(const orc_corpus* c, const int32_t* rows, int32_t n_rows,
             int32_t k, int32_t dot_order, int32_t n_threads,
             int32_t* out_ids, float* out_vals)
{
#ifdef _OPENMP
    if (n_threads <= 0) n_threads = omp_get_max_threads();
#pragma omp parallel for schedule(dynamic, 4) num_threads(n_threads)
#endif
    for (int32_t r = 0; r < n_rows; ++r) {
        const int32_t i = rows[r];
        int32_t* ids = out_ids + (int64_t)r * k;
        float* vals = out_vals + (int64_t)r * k;
        int32_t cnt = 0;
        for (int32_t j = 0; j < k; ++j) { ids[j] = -1; vals[j] = -1e30f; }
        const float* ei = c->E + (int64_t)i * c->pitch;
        for (int32_t j = 0; j < c->N; ++j) {
            if (j == i) continue;   /* src/cmng_build.cu:50 */
            const float s = orc_dot(ei, c->E + (int64_t)j * c->pitch, c->D, dot_order);
            topk_push(vals, ids, &cnt, k, s, j);
        }
    }
    (void)n_threads;
}

void orc_cmng_select(const int32_t* knn_ids, int32_t k_init,
                     const int32_t* mod, int32_t N, const int32_t* rows,
                     int32_t n_rows, int32_t degree, int32_t degree_cross,
                     int32_t num_modalities, int32_t* out_neighbors)
{
    const int32_t intra = degree - degree_cross;
    for (int32_t r = 0; r < n_rows; ++r) {
        const int32_t node = rows[r];
        const int32_t* knn = knn_ids + (int64_t)r * k_init;
        int32_t* out = out_neighbors + (int64_t)r * degree;
        const int32_t my_mod = mod[node];
        int32_t filled = 0;
        for (int32_t i = 0; i < k_init && filled < intra; ++i) {
            const int32_t cand = knn[i];
            if (cand < 0 || cand >= N) continue;
            out[filled++] = cand;
        }
        for (int32_t i = filled; i < intra; ++i) out[i] = -1;
        int32_t b = intra;
        for (int32_t m = 0; m < num_modalities && b < degree; ++m) {
            if (m == my_mod) continue;
            int found = 0;
            for (int32_t i = 0; i < k_init; ++i) {
                const int32_t cand = knn[i];
                if (cand < 0 || cand >= N) continue;
                if (mod[cand] == m) { out[b++] = cand; found = 1; break; }
            }
            if (!found && b < degree) out[b++] = -1;
        }
        for (int32_t i = b; i < degree; ++i) out[i] = -1;
    }
}

/* ======================================================================
 * cmng_search (src/cmng_search.cu:110-308)
 * ====================================================================== */

/* src/cmng_search.cu:88-104: reject if not strictly better than the worst,
 * replace the worst, bubble up past strictly smaller scores.             */
static int beam_insert(float* bs, int32_t* bi, int32_t bw, float s, int32_t id)
{
    if (s <= bs[bw - 1]) return 0;
    bs[bw - 1] = s;
    bi[bw - 1] = id;
    for (int32_t j = bw - 2; j >= 0; --j) {
        if (bs[j] < bs[j + 1]) {
            float t = bs[j]; bs[j] = bs[j + 1]; bs[j + 1] = t;
            int32_t u = bi[j]; bi[j] = bi[j + 1]; bi[j + 1] = u;
        } else break;
    }
    return 1;
}

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

int32_t orc_cmng_search(const orc_corpus* c, const int32_t* neighbors,
                        int32_t degree, const float* q, float t_q,
                        const orc_cmng_config* cfg, orc_result* out,
                        orc_cmng_stats* stats)
{
    const int32_t N = c->N, D = c->D;
    const int32_t bw = cfg->beam_width;
    const int32_t K = cfg->K;
    const int32_t order = cfg->dot_order;
    if (N <= 0 || bw <= 0 || D < 2) return 0;
    float* bs = (float*)malloc(sizeof(float) * (size_t)bw);
    int32_t* bi = (int32_t*)malloc(sizeof(int32_t) * (size_t)bw);
    int32_t* bp = (int32_t*)malloc(sizeof(int32_t) * (size_t)bw);
    unsigned char* vis = (unsigned char*)calloc((size_t)N, 1);
    float* dist = (float*)malloc(sizeof(float) * (size_t)(degree > 0 ? degree : 1));
    int32_t iters = 0, scored = 0;
    for (int32_t i = 0; i < bw; ++i) { bs[i] = -FLT_MAX; bi[i] = -1; bp[i] = 0; }

    /* seeds: src/cmng_search.cu:158-180 */
    int32_t num_seeds = 8 * cfg->num_parents;
    if (num_seeds > bw) num_seeds = bw;
    const uint32_t h = f2u(q[0]) ^ f2u(q[1]);
    for (int32_t w = 0; w < 8; ++w) {
        if (w >= num_seeds) continue;
        const int32_t seed = (int32_t)((h + (uint32_t)w * 7919u) % (uint32_t)N);
        const float sim = orc_dot(c->E + (int64_t)seed * c->pitch, q, D, order);
        bs[w] = sim;
        bi[w] = seed;
        if (!vis[seed]) { vis[seed] = 1; ++scored; }
    }
    /* exchange sort of the initial beam: src/cmng_search.cu:184-193 */
    for (int32_t i = 0; i < bw - 1; ++i)
        for (int32_t j = i + 1; j < bw; ++j)
            if (bs[j] > bs[i]) {
                float t = bs[i]; bs[i] = bs[j]; bs[j] = t;
                int32_t u = bi[i]; bi[i] = bi[j]; bi[j] = u;
            }

    /* main loop: src/cmng_search.cu:196-272 */
    for (int32_t it = 0; it < cfg->max_iterations; ++it) {
        int32_t parent = -1;
        for (int32_t i = 0; i < bw; ++i)
            if (bi[i] >= 0 && bp[i] == 0) { parent = bi[i]; bp[i] = 1; break; }
        if (parent < 0) break;
        ++iters;
        const int32_t* nb = neighbors + (int64_t)parent * degree;
        for (int32_t i = 0; i < degree; ++i) {
            const int32_t v = nb[i];
            dist[i] = -FLT_MAX;
            if (v < 0 || v >= N || vis[v]) continue;
            dist[i] = orc_dot(c->E + (int64_t)v * c->pitch, q, D, order);
            vis[v] = 1;
            ++scored;
        }
        for (int32_t i = 0; i < degree; ++i) {
            if (nb[i] < 0 || dist[i] <= -FLT_MAX * 0.5f) continue;
            beam_insert(bs, bi, bw, dist[i], nb[i]);
        }
    }

    /* decay on the beam: src/cmng_search.cu:275-280 */
    for (int32_t t = 0; t < bw; ++t) {
        if (bi[t] < 0) continue;
        const float age = fmaxf(0.0f, t_q - c->ts[bi[t]]);
        bs[t] = bs[t] * expf(-cfg->lambda * age);
    }
    /* selection sort of the first K: src/cmng_search.cu:283-295 */
    const int32_t kk = K < bw ? K : bw;
    for (int32_t i = 0; i < kk - 1; ++i) {
        int32_t b = i;
        for (int32_t j = i + 1; j < bw; ++j)
            if (bs[j] > bs[b]) b = j;
        if (b != i) {
            float t = bs[i]; bs[i] = bs[b]; bs[b] = t;
            int32_t u = bi[i]; bi[i] = bi[b]; bi[b] = u;
        }
    }
    int32_t count = 0;
    for (int32_t i = 0; i < kk; ++i) {
        if (bi[i] < 0) break;
        out[i].node_id = bi[i];
        out[i].score = bs[i];
        out[i].modality = c->mod ? c->mod[bi[i]] : 0;
        out[i].hops = 0;
        ++count;
    }
    if (stats) { stats->iterations = iters; stats->rows_scored = scored; }
    free(bs); free(bi); free(bp); free(vis); free(dist);
    return count;
}
