// mars_cmng.cu -- CMNG: kNN-graph build (G1/G2) and greedy beam search (C1).
//
// Build (build_cmng, src/cmng_build.cu:135-255).  The reference forms every
// 4096 x 4096 tile of E*E^T with cuBLAS SGEMM and merges it into per-row
// sorted lists of k_init = 2*degree candidates with 256 threads doing
// unsynchronised read-modify-write on the same list (:28-71), then picks
// neighbours and cross-modal bridges with one thread per row (:75-132).
// Here the exact k_init nearest rows of every row come from the tensor-core
// batched top-K (mars_batch.cu) with the row itself left out -- candidates
// short-listed on TF32 tiles with a proven margin and rescored with the exact
// canonical dot, so the lists equal an exact fp32 kNN ranked (dot desc, id
// asc) -- and the selection runs one warp per row.
//
// Search (cmng_search, src/cmng_search.cu:110-308): one block of 256 threads
// per query, any number of queries per launch.  The reference's semantics are
// kept step by step, with its serial thread-0 phases replaced by parallel
// equivalents:
//  * seeds: warp w scores node (bits(q0) ^ bits(q1)) + 7919*w mod N;
//  * the initial exchange sort over the valid seeds (thread 0, <= 8 entries);
//  * iteration t expands the node at beam position t (the reference marks
//    positions, not nodes, as expanded: position t is the first unmarked one
//    while it holds a node, and the search ends when it does not);
//  * unvisited neighbours are scored with the reference's warp dot order
//    (lane-strided fma, shfl_down tree), so beams agree bit for bit;
//  * the reference inserts candidates one by one (reject if not better than
//    the worst, bubble up past strictly smaller scores); that equals keeping
//    the beam-width best of (beam + candidates) under (score desc, beam entries
//    before candidates, candidates in neighbour order), computed here as a
//    parallel rank merge;
//  * decay of the final beam, then the reference's selection sort (first
//    position wins among equal scores) as block argmax passes.
// The visited set is an exact open-addressing table in shared memory (the
// reference's 32-probe table can give up near overflow), and an id repeated
// inside one neighbour list is scored once, at its first slot (the reference's
// warps race on it).
#include <cuda_runtime.h>

#include <algorithm>
#include <cfloat>
#include <cstring>
#include <string>
#include <vector>

#include "mars_b200.h"
#include "mars_common.cuh"
#include "mars_internal.h"
#include "mars_kernels.cuh"

namespace mars {
namespace cmng {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxBeam = 256;      // reference MAX_BEAM (src/cmng_search.cu:25)
constexpr int kMaxDegree = 128;    // reference MAX_DEGREE (src/cmng_search.cu:26)

// ---------------------------------------------------------------------------
// Neighbour selection with cross-modal bridges (src/cmng_build.cu:75-132).
// Rows first .. first + count - 1; knn, knn_cnt and out are indexed from
// the first of them.
__global__ void select_kernel(const int32_t* __restrict__ knn, const int32_t* __restrict__ knn_cnt,
                              int32_t k_init, const int32_t* __restrict__ mod, int32_t first, int32_t count,
                              int32_t degree, int32_t degree_cross, int32_t num_modalities,
                              int32_t* __restrict__ out) {
    const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= count) return;
    const int32_t* kr = knn + row * k_init;
    const int32_t cnt = min(knn_cnt[row], k_init);
    int32_t* o = out + row * degree;
    const int32_t intra = degree - degree_cross;
    for (int j = lane; j < intra; j += 32) o[j] = j < cnt ? kr[j] : -1;
    const int32_t my_mod = mod[first + row];
    int32_t b = intra;
    for (int32_t m = 0; m < num_modalities && b < degree; ++m) {
        if (m == my_mod) continue;
        int32_t found = -1;
        for (int base = 0; base < cnt; base += 32) {
            const int i = base + lane;
            const bool hit = i < cnt && __ldg(mod + kr[i]) == m;
            const unsigned bal = __ballot_sync(0xffffffffu, hit);
            if (bal) { found = kr[base + __ffs(bal) - 1]; break; }
        }
        if (lane == 0) o[b] = found;
        ++b;
    }
    for (int j = b + lane; j < degree; j += 32) o[j] = -1;
}

// ---------------------------------------------------------------------------
// The reference's warp dot product (src/cmng_search.cu:59-70): lane-strided
// fused multiply-add, then a shfl_down tree; lane 0's value is the result.
__device__ __forceinline__ float warp_dot_ref(const float* __restrict__ a, const float* __restrict__ b,
                                              int D, int lane) {
    float s = 0.0f;
    for (int d = lane; d < D; d += 32) s = __fmaf_rn(__ldg(a + d), b[d], s);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s = __fadd_rn(s, __shfl_down_sync(0xffffffffu, s, off));
    return __shfl_sync(0xffffffffu, s, 0);
}

// The same arithmetic with a row's loads issued together: lane l holds
// elements l, l + 32, ... (at most C of them, D <= 32 C) in registers before
// the fused multiply-adds run in the reference's order, so a row costs one
// memory round trip instead of one per unrolled group of the loop.
template <int C>
__device__ __forceinline__ float warp_dot_ref_rows(const float* __restrict__ a, const float* __restrict__ b,
                                                   int D, int lane) {
    float v[C];
#pragma unroll
    for (int c = 0; c < C; ++c) {
        const int d = lane + 32 * c;
        v[c] = d < D ? __ldg(a + d) : 0.0f;
    }
    float s = 0.0f;
#pragma unroll
    for (int c = 0; c < C; ++c) {
        const int d = lane + 32 * c;
        if (d < D) s = __fmaf_rn(v[c], b[d], s);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s = __fadd_rn(s, __shfl_down_sync(0xffffffffu, s, off));
    return __shfl_sync(0xffffffffu, s, 0);
}

__device__ __forceinline__ float warp_dot_ref_fast(const float* __restrict__ a, const float* __restrict__ b, int D,
                                                   int lane) {
    if (D <= 256) return warp_dot_ref_rows<8>(a, b, D, lane);
    if (D <= 512) return warp_dot_ref_rows<16>(a, b, D, lane);
    if (D <= 768) return warp_dot_ref_rows<24>(a, b, D, lane);
    if (D <= 1024) return warp_dot_ref_rows<32>(a, b, D, lane);
    return warp_dot_ref(a, b, D, lane);
}

struct SearchArgs {
    const int32_t* nbrs;      // N x degree
    const float* E;           // N x pitch
    const float* ts;
    const int32_t* mod;
    int64_t pitch;
    int32_t N, D, degree;
    const float* Q;           // nq x qpitch
    int64_t qpitch;
    int32_t nq;
    float t_q, lambda;
    int32_t K, beam, max_iter, num_parents;
    int32_t hash_size;        // power of two
    int32_t* out_ids;         // nq x K
    float* out_scores;
    int32_t* out_mods;
    int32_t* out_cnt;         // nq
    int32_t* stat_iters;      // nq (may be null)
    int32_t* stat_scored;     // nq (may be null)
    int* ticket;              // zeroed counter handing out queries (NULL: block b takes b, b + grid, ...)
};

// The next query of a block.  With a ticket counter (zeroed before the
// launch) the blocks draw queries one at a time, so a block that drew quick
// queries takes more and the launch ends about one query after the last
// start, whatever the spread of the queries' costs; without one, block b
// takes b, b + grid, ...  Block-collective.
__device__ __forceinline__ int next_query(int* ticket, int* s_slot, int prev) {
    if (ticket == nullptr) return prev < 0 ? (int)blockIdx.x : prev + (int)gridDim.x;
    __syncthreads();                       // the previous query's slot has been read
    if (threadIdx.x == 0) *s_slot = atomicAdd(ticket, 1);
    __syncthreads();
    return *s_slot;
}

__device__ __forceinline__ uint32_t hash32(int32_t v) {
    uint32_t x = (uint32_t)v;
    x ^= x >> 16; x *= 0x7feb352dU; x ^= x >> 15; x *= 0x846ca68bU; x ^= x >> 16;
    return x;
}

// Exact set: returns true when `v` was newly inserted.
__device__ __forceinline__ bool set_insert(int32_t* table, uint32_t mask, int32_t v) {
    uint32_t s = hash32(v) & mask;
    for (uint32_t probe = 0; probe <= mask; ++probe) {
        const int32_t old = atomicCAS(table + s, -1, v);
        if (old == -1) return true;
        if (old == v) return false;
        s = (s + 1) & mask;
    }
    return false;   // unreachable: the table is sized to at most 2/3 full
}

__device__ __forceinline__ bool set_contains(const int32_t* table, uint32_t mask, int32_t v) {
    uint32_t s = hash32(v) & mask;
    for (uint32_t probe = 0; probe <= mask; ++probe) {
        const int32_t cur = table[s];
        if (cur == v) return true;
        if (cur == -1) return false;
        s = (s + 1) & mask;
    }
    return false;
}

// Four warps per query and up to eight queries per SM: a query's latency
// per iteration is mostly dependent loads (its neighbour list, then its rows,
// about degree / 4 per warp), so more queries in flight per SM raise the
// throughput more than more warps per query would.
constexpr int kSearchThreads = 128;
constexpr int kSearchWarps = kSearchThreads / 32;

__global__ void __launch_bounds__(kSearchThreads, 8) search_kernel(const SearchArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    float* s_q = reinterpret_cast<float*>(smem);                        // D (padded to 4)
    float* s_bs = s_q + ((a.D + 3) & ~3);                               // beam scores
    int32_t* s_bi = reinterpret_cast<int32_t*>(s_bs + kMaxBeam);       // beam ids
    float* s_nbs = reinterpret_cast<float*>(s_bi + kMaxBeam);          // merged beam scores
    int32_t* s_nbi = reinterpret_cast<int32_t*>(s_nbs + kMaxBeam);     // merged beam ids
    int32_t* s_nb = s_nbi + kMaxBeam;                                   // neighbour ids
    float* s_dist = reinterpret_cast<float*>(s_nb + kMaxDegree);       // neighbour scores
    int32_t* s_hash = reinterpret_cast<int32_t*>(s_dist + kMaxDegree);
    __shared__ int s_scored;
    __shared__ float s_red_v[kSearchWarps];
    __shared__ int s_red_i[kSearchWarps];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int bw = a.beam;
    const uint32_t mask = (uint32_t)a.hash_size - 1u;
    const uint32_t row_bytes = (uint32_t)((a.D + 3) & ~3) * 4u;   // rows are float4 aligned

    __shared__ int s_qslot;
    for (int qi = next_query(a.ticket, &s_qslot, -1); qi < a.nq; qi = next_query(a.ticket, &s_qslot, qi)) {
        // the beam and its merged successor swap roles every iteration
        float* bs = s_bs;
        int32_t* bi = s_bi;
        float* nbs = s_nbs;
        int32_t* nbi = s_nbi;
        const float* q = a.Q + (int64_t)qi * a.qpitch;
        for (int d = tid; d < a.D; d += kSearchThreads) s_q[d] = q[d];
        for (int i = tid; i < a.hash_size; i += kSearchThreads) s_hash[i] = -1;
        for (int i = tid; i < bw; i += kSearchThreads) { s_bs[i] = -FLT_MAX; s_bi[i] = -1; }
        if (tid == 0) s_scored = 0;
        __syncthreads();

        // ---- seeds (src/cmng_search.cu:158-180) ----
        const int num_seeds = min(8 * a.num_parents, bw);
        for (int w = warp; w < min(num_seeds, 8); w += kSearchWarps) {
            const uint32_t h = __float_as_uint(s_q[0]) ^ __float_as_uint(s_q[1]);
            const int32_t seed = (int32_t)((h + (uint32_t)w * 7919u) % (uint32_t)a.N);
            const float sim = warp_dot_ref_fast(a.E + (int64_t)seed * a.pitch, s_q, a.D, lane);
            if (lane == 0) {
                bs[w] = sim;
                bi[w] = seed;
                if (set_insert(s_hash, mask, seed)) atomicAdd(&s_scored, 1);
            }
        }
        __syncthreads();
        // exchange sort of the seeded positions (src/cmng_search.cu:184-193)
        if (tid == 0) {
            const int ns = min(min(num_seeds, 8), bw);
            for (int i = 0; i < ns - 1; ++i)
                for (int j = i + 1; j < ns; ++j)
                    if (bs[j] > bs[i]) {
                        const float t = bs[i]; bs[i] = bs[j]; bs[j] = t;
                        const int32_t u = bi[i]; bi[i] = bi[j]; bi[j] = u;
                    }
        }
        __syncthreads();

        // ---- main loop (src/cmng_search.cu:196-272) ----
        int iters = 0;
        for (int it = 0; it < a.max_iter; ++it) {
            if (it >= bw) break;
            const int32_t parent = bi[it];
            if (parent < 0) break;
            ++iters;
            const int32_t* nb = a.nbrs + (int64_t)parent * a.degree;
            // candidate slots: valid id, not visited, first occurrence in the
            // list.  A candidate's row is requested into L2 as soon as it is
            // known to be one, so the warps' dot products below (about
            // degree / 4 rows per warp, one after another) mostly wait on L2
            // instead of one DRAM trip per row; visited rows are not fetched.
            for (int j = tid; j < a.degree; j += kSearchThreads) s_nb[j] = __ldg(nb + j);
            __syncthreads();
            for (int j = tid; j < a.degree; j += kSearchThreads) {
                const int32_t v = s_nb[j];
                bool ok = v >= 0 && v < a.N && !set_contains(s_hash, mask, v);
                for (int k = 0; ok && k < j; ++k) ok = s_nb[k] != v;
                s_dist[j] = ok ? 0.0f : -FLT_MAX;
                if (ok) prefetch_l2_bulk(a.E + (int64_t)v * a.pitch, row_bytes);
            }
            __syncthreads();
            for (int j = warp; j < a.degree; j += kSearchWarps) {
                if (s_dist[j] == -FLT_MAX) continue;                    // warp-uniform
                const int32_t v = s_nb[j];
                const float sim = warp_dot_ref_fast(a.E + (int64_t)v * a.pitch, s_q, a.D, lane);
                if (lane == 0) s_dist[j] = sim;
            }
            __syncthreads();
            for (int j = tid; j < a.degree; j += kSearchThreads)
                if (s_dist[j] > -FLT_MAX * 0.5f) { set_insert(s_hash, mask, s_nb[j]); atomicAdd(&s_scored, 1); }
            // rank merge: beam entries keep their order and precede equal candidates
            for (int o = tid; o < bw; o += kSearchThreads) {
                const float so = bs[o];
                int pos = o;
                for (int j = 0; j < a.degree; ++j) pos += (s_dist[j] > -FLT_MAX * 0.5f && s_dist[j] > so) ? 1 : 0;
                if (pos < bw) { nbs[pos] = so; nbi[pos] = bi[o]; }
            }
            for (int j = tid; j < a.degree; j += kSearchThreads) {
                const float d = s_dist[j];
                if (!(d > -FLT_MAX * 0.5f)) continue;
                int pos = 0;
                for (int k = 0; k < a.degree; ++k) {
                    const float dk = s_dist[k];
                    pos += (dk > -FLT_MAX * 0.5f && (dk > d || (dk == d && k < j))) ? 1 : 0;
                }
                for (int o = 0; o < bw; ++o) pos += (bs[o] >= d) ? 1 : 0;
                if (pos < bw) {
                    nbs[pos] = d;
                    nbi[pos] = s_nb[j];
                    // a later iteration may expand this position: its
                    // neighbour list is requested into L2 now
                    if (pos > it && pos < a.max_iter)
                        prefetch_l2_span(a.nbrs + (int64_t)s_nb[j] * a.degree, (uint32_t)a.degree * 4u);
                }
            }
            __syncthreads();
            // the merged beam is the beam of the next iteration
            float* tf = bs; bs = nbs; nbs = tf;
            int32_t* ti = bi; bi = nbi; nbi = ti;
        }

        // ---- decay (src/cmng_search.cu:275-280) ----
        if (bs != s_bs) {   // the current beam sits in the second buffer: bring it home
            for (int o = tid; o < bw; o += kSearchThreads) { s_bs[o] = bs[o]; s_bi[o] = bi[o]; }
            __syncthreads();
        }
        for (int o = tid; o < bw; o += kSearchThreads) {
            const int32_t id = s_bi[o];
            if (id >= 0) {
                const float age = fmaxf(0.0f, a.t_q - __ldg(a.ts + id));
                s_bs[o] *= __expf(-a.lambda * age);
            }
        }
        __syncthreads();
        // ---- selection of the first K (src/cmng_search.cu:283-295) ----
        const int kk = min(a.K, bw);
        for (int i = 0; i < kk - 1; ++i) {
            float bv = -INFINITY;
            int bi = INT32_MAX;
            for (int o = i + tid; o < bw; o += kSearchThreads) {
                const float v = s_bs[o];
                if (v > bv || (v == bv && o < bi)) { bv = v; bi = o; }
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                const float ov = __shfl_down_sync(0xffffffffu, bv, off);
                const int oi = __shfl_down_sync(0xffffffffu, bi, off);
                if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
            }
            if (lane == 0) { s_red_v[warp] = bv; s_red_i[warp] = bi; }
            __syncthreads();
            if (tid == 0) {
                float v = s_red_v[0];
                int best = s_red_i[0];
                for (int w = 1; w < kSearchWarps; ++w)
                    if (s_red_v[w] > v || (s_red_v[w] == v && s_red_i[w] < best)) { v = s_red_v[w]; best = s_red_i[w]; }
                // (max score, lowest position) = the reference's strict '>' scan
                if (best != i && best != INT32_MAX) {
                    const float t = s_bs[i]; s_bs[i] = s_bs[best]; s_bs[best] = t;
                    const int32_t u = s_bi[i]; s_bi[i] = s_bi[best]; s_bi[best] = u;
                }
            }
            __syncthreads();
        }
        if (tid == 0) {
            int cnt = 0;
            for (int i = 0; i < kk; ++i) {
                if (s_bi[i] < 0) break;
                a.out_ids[(int64_t)qi * a.K + i] = s_bi[i];
                a.out_scores[(int64_t)qi * a.K + i] = s_bs[i];
                if (a.out_mods) a.out_mods[(int64_t)qi * a.K + i] = __ldg(a.mod + s_bi[i]);
                ++cnt;
            }
            for (int i = cnt; i < a.K; ++i) {
                a.out_ids[(int64_t)qi * a.K + i] = -1;
                a.out_scores[(int64_t)qi * a.K + i] = -INFINITY;
                if (a.out_mods) a.out_mods[(int64_t)qi * a.K + i] = -1;
            }
            a.out_cnt[qi] = cnt;
            if (a.stat_iters) a.stat_iters[qi] = iters;
            if (a.stat_scored) a.stat_scored[qi] = s_scored;
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------
// BFS from each query's beam-search results over the CMNG adjacency
// (the canonical BFS of the scan pipeline: level-synchronous, a node's score is
// the best fmaxf(parent * decay, own * 0.8f) over its parents one level up,
// seeds keep their beam score, no frontier cap), then the top-K of all visited
// nodes by (score desc, id asc).  One block per query; the visited set is a
// per-block open-addressing table in global memory whose entries carry the
// block's query epoch, so nothing is cleared between queries:
//   tag[slot]   = (epoch << 32) | node
//   state[slot] = ((epoch << 4 | (15 - level)) << 32) | key(best parent score)
// One atomicMax on state both claims the node for a level and keeps its best
// parent; the thread that sees an older state appends the node to the level.
struct BfsArgs2 {
    const int32_t* nbrs;
    int32_t degree;
    const float* E;
    const float* ts;
    const float* imp;
    const int32_t* mod;
    int64_t pitch4;
    int32_t nc, N;
    const float* Q;
    int64_t qpitch;
    int32_t nq;
    float t_q, lambda, hop_decay;
    int32_t use_imp, hops, K;
    const int32_t* seed_ids;      // nq x seed_stride
    const float* seed_scores;
    const int32_t* seed_cnt;
    int32_t seed_stride;
    unsigned long long* tags;     // gridDim x table
    unsigned long long* states;
    int32_t* lists;               // gridDim x vcap
    uint32_t* epochs;             // gridDim
    int32_t table, vcap;
    int32_t* out_ids;             // nq x K
    float* out_scores;
    int32_t* out_mods;
    int32_t* out_hops;
    int32_t* out_cnt;
    int32_t* out_visited;         // nq (may be null)
    int* err;
    // queries that the shared-memory kernel could not hold: it appends them,
    // the global-table kernel then answers only those (NULL: every query)
    int32_t* redo;
    int32_t* redo_cnt;
    int32_t smem_nodes;           // visited nodes the shared table takes per query
    int* ticket;                  // shared-memory kernel: zeroed counter handing out queries (NULL: static order)
};

__device__ __forceinline__ int table_find_or_claim(unsigned long long* tags, uint32_t mask, uint32_t epoch,
                                                   int32_t v) {
    const unsigned long long want = ((unsigned long long)epoch << 32) | (uint32_t)v;
    uint32_t s = hash32(v) & mask;
    for (uint32_t probe = 0; probe <= mask; ++probe) {
        unsigned long long cur = __ldcg(tags + s);
        while ((uint32_t)(cur >> 32) != epoch) {          // stale slot: try to take it
            const unsigned long long prev = atomicCAS(tags + s, cur, want);
            if (prev == cur) return (int)s;
            cur = prev;
        }
        if (cur == want) return (int)s;
        s = (s + 1) & mask;
    }
    return -1;   // unreachable: the table is sized to at most half full
}

__device__ __forceinline__ float bfs_own_score(const BfsArgs2& a, const float4* q4, int32_t u, int lane) {
    const float4* row = reinterpret_cast<const float4*>(a.E) + (int64_t)u * a.pitch4;
    const float dot = warp_dot_canonical(row, q4, a.nc, lane);
    float f = fused_weight_apply(dot, __ldg(a.ts + u), a.t_q, a.lambda);
    if (a.use_imp && a.imp != nullptr) f = f * __ldg(a.imp + u);
    return f;
}

// The top-K of a query's visited nodes (list / lscore, `total` of them) by
// (score desc, id asc) into the outputs: per-warp ranked lists merged by warp
// 0; hop_of(u) gives a listed node's level.
template <int KPL, class HopOf>
__device__ __forceinline__ void bfs_emit_topk(const BfsArgs2& a, int qi, const int32_t* list, const float* lscore,
                                              int total, float (*s_val)[kMaxTopK], int32_t (*s_idx)[kMaxTopK],
                                              HopOf hop_of) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    WarpTopK<KPL> top;
    top.init(a.K);
    for (int base = warp * 32; base < total; base += kThreads) {
        const int j = base + lane;
        float sv = -INFINITY;
        int32_t id = INT32_MAX;
        if (j < total) { sv = lscore[j]; id = list[j]; }
        top.offer_lanes(sv, id, j < total, lane);
    }
    top.store(s_val[warp], s_idx[warp], lane);
    __syncthreads();
    if (warp == 0) {
        for (int w = 1; w < kWarps; ++w) top.offer_sorted(s_val[w], s_idx[w], a.K, lane);
        int cnt = 0;
#pragma unroll
        for (int sl = 0; sl < KPL; ++sl) {
            const int p = sl * 32 + lane;
            const bool valid = p < a.K && top.i[sl] != INT32_MAX;
            cnt += __popc(__ballot_sync(0xffffffffu, valid));
            if (p < a.K) {
                const int64_t o = (int64_t)qi * a.K + p;
                if (valid) {
                    const int32_t u = top.i[sl];
                    a.out_ids[o] = u;
                    a.out_scores[o] = top.v[sl];
                    if (a.out_mods) a.out_mods[o] = __ldg(a.mod + u);
                    if (a.out_hops) a.out_hops[o] = hop_of(u);
                } else {
                    a.out_ids[o] = -1;
                    a.out_scores[o] = -INFINITY;
                    if (a.out_mods) a.out_mods[o] = -1;
                    if (a.out_hops) a.out_hops[o] = -1;
                }
            }
        }
        if (lane == 0) {
            a.out_cnt[qi] = cnt;
            if (a.out_visited) a.out_visited[qi] = total;
        }
    }
    __syncthreads();
}

template <int KPL>
__global__ void __launch_bounds__(kThreads, 3) bfs_kernel(const BfsArgs2 a) {
    __shared__ int s_lvl[16];       // level offsets; [15] = tail
    __shared__ float   s_val[kWarps][kMaxTopK];
    __shared__ int32_t s_idx[kWarps][kMaxTopK];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t mask = (uint32_t)a.table - 1u;
    unsigned long long* tags = a.tags + (int64_t)blockIdx.x * a.table;
    unsigned long long* states = a.states + (int64_t)blockIdx.x * a.table;
    int32_t* list = a.lists + (int64_t)blockIdx.x * a.vcap;
    float* lscore = reinterpret_cast<float*>(list + a.vcap / 2);   // second half: scores
    const int vcap = a.vcap / 2;

    const int nwork = a.redo != nullptr ? __ldcg(a.redo_cnt) : a.nq;
    for (int wi = blockIdx.x; wi < nwork; wi += gridDim.x) {
        const int qi = a.redo != nullptr ? __ldcg(a.redo + wi) : wi;
        uint32_t epoch = 0;
        if (tid == 0) {
            epoch = a.epochs[blockIdx.x] + 1;
            if (epoch >= (1u << 27)) epoch = 1;   // wraps after 2^27 queries per block (tables reset below)
            a.epochs[blockIdx.x] = epoch;
            s_lvl[0] = 0;
        }
        __syncthreads();
        epoch = a.epochs[blockIdx.x];
        if (epoch == 1) {   // first use or wrap: clear this block's table
            for (int i = tid; i < a.table; i += kThreads) { tags[i] = 0ull; states[i] = 0ull; }
            __syncthreads();
        }
        const float4* q4 = reinterpret_cast<const float4*>(a.Q + (int64_t)qi * a.qpitch);
        // ---- level 0: the seeds with their beam scores ----
        const int ns = min(a.seed_cnt[qi], a.seed_stride);
        const unsigned long long st0 = (unsigned long long)((epoch << 4) | 15u) << 32;
        if (tid == 0) {
            int n0 = 0;
            for (int i = 0; i < ns; ++i) {
                const int32_t u = a.seed_ids[(int64_t)qi * a.seed_stride + i];
                if (u < 0 || u >= a.N) continue;
                const int slot = table_find_or_claim(tags, mask, epoch, u);
                const unsigned long long old = atomicMax(states + slot,
                    st0 | f2key(a.seed_scores[(int64_t)qi * a.seed_stride + i]));
                if ((uint32_t)(old >> 32) < (epoch << 4)) {
                    list[n0] = u;
                    lscore[n0] = a.seed_scores[(int64_t)qi * a.seed_stride + i];
                    ++n0;
                }
            }
            s_lvl[1] = n0;
            s_lvl[15] = n0;
        }
        __syncthreads();
        bool overflow = false;
        for (int h = 0; h <= a.hops; ++h) {
            const int beg = s_lvl[h], end = s_lvl[h + 1];
            const unsigned long long nst = (unsigned long long)((epoch << 4) | (uint32_t)(15 - (h + 1))) << 32;
            for (int idx = beg + warp; idx < end; idx += kWarps) {
                const int32_t u = list[idx];
                float su;
                if (h == 0) {
                    su = lscore[idx];
                } else {
                    const float own = bfs_own_score(a, q4, u, lane);
                    const int slot = table_find_or_claim(tags, mask, epoch, u);
                    const float best = key2f((uint32_t)(__ldcg(states + slot) & 0xffffffffull));
                    su = fmaxf(best, own * 0.8f);
                    if (lane == 0) lscore[idx] = su;
                }
                if (h == a.hops) continue;           // last level: scored, not expanded
                const unsigned long long word = nst | f2key(su * a.hop_decay);
                const int32_t* nb = a.nbrs + (int64_t)u * a.degree;
                for (int e = lane; e < a.degree; e += 32) {
                    const int32_t v = __ldg(nb + e);
                    if (v < 0 || v >= a.N) continue;
                    const int slot = table_find_or_claim(tags, mask, epoch, v);
                    const unsigned long long old = atomicMax(states + slot, word);
                    if ((uint32_t)(old >> 32) < (epoch << 4)) {
                        const int pos = atomicAdd(&s_lvl[15], 1);
                        if (pos < vcap) list[pos] = v; else overflow = true;
                    }
                }
            }
            __syncthreads();
            if (tid == 0 && h + 2 < 15) s_lvl[h + 2] = min(s_lvl[15], vcap);
            __syncthreads();
        }
        if (overflow) atomicCAS(a.err, 0, 7);
        bfs_emit_topk<KPL>(a, qi, list, lscore, min(s_lvl[15], vcap), s_val, s_idx, [&](int32_t u) {
            const int slot = table_find_or_claim(tags, mask, epoch, u);
            return 15 - (int)((uint32_t)(__ldcg(states + slot) >> 32) & 15u);
        });
    }
}

// The same BFS with the visited set in shared memory: a table of kBfsSlots
// node ids and states per block (cleared per query), at most smem_nodes
// visited nodes per query (half the table or less).  The state word and the
// rule are the global kernel's -- ((1 << 4 | (15 - level)) << 32) | key(best
// parent score), one atomicMax both claims a node for a level and keeps its
// best parent -- and the answer does not depend on the order of the claims.
// Per level the own scores come first (a warp per node; the node's slot was
// kept when it was listed), then every (node, edge) pair of the level is
// handed to its own thread, so a level's claims are shared-memory atomics
// spread over the whole block.  A query that outgrows the table is appended
// to a.redo for the global-table kernel.
constexpr int kBfsSlots = 4096;
constexpr uint32_t kEmptyTag = 0xffffffffu;
constexpr size_t kBfsSmemBytes = (size_t)kBfsSlots * (4 + 8) + (size_t)(kBfsSlots / 2) * 2;

// The slot of v (claimed when absent), -1 when the table is full.
__device__ __forceinline__ int smem_claim(uint32_t* tag, int32_t v) {
    uint32_t s = hash32(v) & (uint32_t)(kBfsSlots - 1);
    for (int probe = 0; probe < kBfsSlots; ++probe) {
        const uint32_t cur = *reinterpret_cast<volatile uint32_t*>(tag + s);
        if (cur == (uint32_t)v) return (int)s;
        if (cur == kEmptyTag) {
            const uint32_t old = atomicCAS(tag + s, kEmptyTag, (uint32_t)v);
            if (old == kEmptyTag || old == (uint32_t)v) return (int)s;
        }
        s = (s + 1) & (uint32_t)(kBfsSlots - 1);
    }
    return -1;
}

__device__ __forceinline__ int smem_find(const uint32_t* tag, int32_t v) {
    uint32_t s = hash32(v) & (uint32_t)(kBfsSlots - 1);
    for (int probe = 0; probe < kBfsSlots; ++probe) {
        const uint32_t cur = tag[s];
        if (cur == (uint32_t)v) return (int)s;
        if (cur == kEmptyTag) return -1;
        s = (s + 1) & (uint32_t)(kBfsSlots - 1);
    }
    return -1;
}

template <int KPL>
__global__ void __launch_bounds__(kThreads, 3) bfs_smem_kernel(const BfsArgs2 a) {
    extern __shared__ __align__(16) uint8_t bfs_smem[];
    unsigned long long* s_state = reinterpret_cast<unsigned long long*>(bfs_smem);
    uint32_t* s_tag = reinterpret_cast<uint32_t*>(s_state + kBfsSlots);
    uint16_t* s_lslot = reinterpret_cast<uint16_t*>(s_tag + kBfsSlots);   // the slot of each listed node
    __shared__ int s_lvl[16];
    __shared__ int s_tail, s_ovf;
    __shared__ float   s_val[kWarps][kMaxTopK];
    __shared__ int32_t s_idx[kWarps][kMaxTopK];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int32_t* list = a.lists + (int64_t)blockIdx.x * a.vcap;
    float* lscore = reinterpret_cast<float*>(list + a.vcap / 2);
    const int limit = min(a.smem_nodes, a.vcap / 2);
    const uint32_t row_bytes = (uint32_t)a.nc * 16u;

    __shared__ int s_qslot;
    for (int qi = next_query(a.ticket, &s_qslot, -1); qi < a.nq; qi = next_query(a.ticket, &s_qslot, qi)) {
        for (int i = tid; i < kBfsSlots; i += kThreads) { s_tag[i] = kEmptyTag; s_state[i] = 0ull; }
        if (tid == 0) { s_tail = 0; s_ovf = 0; s_lvl[0] = 0; }
        __syncthreads();
        const float4* q4 = reinterpret_cast<const float4*>(a.Q + (int64_t)qi * a.qpitch);
        // ---- level 0: the seeds with their beam scores, one thread each ----
        const int ns = min(a.seed_cnt[qi], a.seed_stride);
        const unsigned long long st0 = (unsigned long long)((1u << 4) | 15u) << 32;
        for (int i = tid; i < ns; i += kThreads) {
            const int32_t u = a.seed_ids[(int64_t)qi * a.seed_stride + i];
            if (u < 0 || u >= a.N) continue;
            const int slot = smem_claim(s_tag, u);
            if (slot < 0) { s_ovf = 1; continue; }
            const unsigned long long old = atomicMax(s_state + slot,
                                                     st0 | f2key(a.seed_scores[(int64_t)qi * a.seed_stride + i]));
            if ((old >> 32) == 0ull) {
                const int pos = atomicAdd(&s_tail, 1);
                if (pos < limit) { list[pos] = u; s_lslot[pos] = (uint16_t)slot; } else { s_ovf = 1; }
            }
        }
        __syncthreads();
        if (tid == 0) s_lvl[1] = min(s_tail, limit);
        __syncthreads();
        for (int h = 0; h <= a.hops; ++h) {
            if (s_ovf != 0) break;                 // read after a barrier: the same on every thread
            const int beg = s_lvl[h], end = s_lvl[h + 1];
            // the level's scores: seeds keep their beam score (the state's
            // key), later levels max(best parent x decay, own x 0.8)
            if (h == 0) {
                for (int idx = beg + tid; idx < end; idx += kThreads)
                    lscore[idx] = key2f((uint32_t)(s_state[s_lslot[idx]] & 0xffffffffull));
            } else {
                // each warp requests its next two rows into L2 while it
                // scores the current one (three rows travel per warp)
                auto prefetch_node = [&](int idx) {
                    if (lane == 0 && idx < end)
                        prefetch_l2_bulk(reinterpret_cast<const float4*>(a.E) + (int64_t)list[idx] * a.pitch4,
                                         row_bytes);
                };
                prefetch_node(beg + warp + kWarps);
                for (int idx = beg + warp; idx < end; idx += kWarps) {
                    prefetch_node(idx + 2 * kWarps);
                    const float own = bfs_own_score(a, q4, list[idx], lane);
                    const float best = key2f((uint32_t)(s_state[s_lslot[idx]] & 0xffffffffull));
                    if (lane == 0) lscore[idx] = fmaxf(best, own * 0.8f);
                }
            }
            if (h == a.hops) break;                // last level: scored, not expanded
            __syncthreads();
            const unsigned long long nst = (unsigned long long)((1u << 4) | (uint32_t)(15 - (h + 1))) << 32;
            const int total = (end - beg) * a.degree;
            // two edges per thread at a time: both neighbour ids are loaded
            // before either is claimed
            for (int p0 = tid; p0 < total; p0 += 2 * kThreads) {
                int32_t v[2];
                int ix[2];
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const int p = p0 + u * kThreads;
                    v[u] = -1;
                    ix[u] = beg;
                    if (p < total) {
                        const int k = p / a.degree;
                        ix[u] = beg + k;
                        v[u] = __ldg(a.nbrs + (int64_t)list[ix[u]] * a.degree + (p - k * a.degree));
                    }
                }
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    if (v[u] < 0 || v[u] >= a.N) continue;
                    const int slot = smem_claim(s_tag, v[u]);
                    if (slot < 0) { s_ovf = 1; continue; }
                    const unsigned long long old =
                        atomicMax(s_state + slot, nst | f2key(lscore[ix[u]] * a.hop_decay));
                    if ((old >> 32) == 0ull) {
                        const int pos = atomicAdd(&s_tail, 1);
                        if (pos < limit) { list[pos] = v[u]; s_lslot[pos] = (uint16_t)slot; } else { s_ovf = 1; }
                    }
                }
            }
            __syncthreads();
            if (tid == 0 && h + 2 < 15) s_lvl[h + 2] = min(s_tail, limit);
            __syncthreads();
        }
        __syncthreads();
        const bool ovf = s_ovf != 0;
        const int visited = min(s_tail, limit);
        __syncthreads();                           // every thread has read the flag before the next query resets it
        if (ovf) {
            if (tid == 0) a.redo[atomicAdd(a.redo_cnt, 1)] = qi;
            continue;
        }
        bfs_emit_topk<KPL>(a, qi, list, lscore, visited, s_val, s_idx, [&](int32_t u) {
            const int slot = smem_find(s_tag, u);
            return slot < 0 ? -1 : 15 - (int)((uint32_t)(s_state[slot] >> 32) & 15u);
        });
    }
}

}  // namespace cmng
}  // namespace mars

// ===========================================================================
// Host side
using namespace mars;
using namespace mars::cmng;

namespace {

int hash_size_for(int32_t max_iter, int32_t degree) {
    // at most 8 seeds + max_iter x degree entries, the table at most 2/3 full
    int64_t need = (3 * (8 + (int64_t)max_iter * degree) + 1) / 2;
    int64_t h = 256;
    while (h < need) h <<= 1;
    return (int)h;
}

size_t search_smem(int32_t D, int hash_size) {
    return (size_t)((D + 3) & ~3) * 4 + 4 * kMaxBeam * 4 + 2 * kMaxDegree * 4 + (size_t)hash_size * 4;
}

}  // namespace

extern "C" {

int mars_cmng_build(const mars_store* s, int32_t degree, int32_t degree_cross, int32_t num_modalities,
                    int32_t* d_neighbors, float* build_ms) {
    if (s == nullptr) return fail(MARS_ERR_INVALID, "mars_cmng_build: NULL argument");
    return mars_cmng_build_rows(s, 0, s->n, degree, degree_cross, num_modalities, d_neighbors, build_ms);
}

int mars_cmng_build_rows(const mars_store* s, int32_t first, int32_t count, int32_t degree,
                         int32_t degree_cross, int32_t num_modalities, int32_t* d_neighbors,
                         float* build_ms) {
    if (s == nullptr || d_neighbors == nullptr) return fail(MARS_ERR_INVALID, "mars_cmng_build: NULL argument");
    if (degree <= 0 || degree > kMaxDegree || degree_cross < 0 || degree_cross > degree || num_modalities < 0)
        return fail(MARS_ERR_INVALID, "mars_cmng_build: need 0 < degree <= 128, 0 <= degree_cross <= degree");
    const int32_t N = s->n;
    if (N < 2) return fail(MARS_ERR_INVALID, "mars_cmng_build: need at least 2 rows");
    if (first < 0 || count < 0 || (int64_t)first + count > N)
        return fail(MARS_ERR_INVALID, "mars_cmng_build_rows: rows outside the store");
    if (build_ms) *build_ms = 0.f;
    if (count == 0) return MARS_OK;
    const int32_t k_init = std::min(2 * degree, std::min(N - 1, (int32_t)MARS_MAX_TOP_K));
    MarsDeviceGuard g(s->device);
    const int32_t chunk = std::min(count, 4096);
    // scratch kept on the store between builds (the store is used by one
    // host thread at a time)
    auto& bcache = const_cast<mars_store*>(s)->build;
    int rc = MARS_OK;
    if (bcache.bc == nullptr || bcache.bc_nodes < N || bcache.bc_chunk < chunk || bcache.bc_k < k_init) {
        if (bcache.bc) mars_batch_ctx_destroy(bcache.bc);
        bcache.bc = nullptr;
        rc = mars_batch_ctx_create(s->device, N, s->dim, chunk, k_init, &bcache.bc);
        if (rc != MARS_OK) return rc;
        bcache.bc_nodes = N;
        bcache.bc_chunk = chunk;
        bcache.bc_k = k_init;
    }
    const size_t entries = (size_t)count * k_init;
    if (bcache.entries < entries || bcache.rows < count) {
        cudaFree(bcache.d_knn);
        cudaFree(bcache.d_vals);
        cudaFree(bcache.d_cnt);
        bcache.d_knn = nullptr;
        bcache.d_vals = nullptr;
        bcache.d_cnt = nullptr;
        bcache.entries = 0;
        bcache.rows = 0;
        if (cudaMalloc(&bcache.d_knn, entries * 4) != cudaSuccess ||
            cudaMalloc(&bcache.d_vals, entries * 4) != cudaSuccess ||
            cudaMalloc(&bcache.d_cnt, (size_t)count * 4) != cudaSuccess) {
            (void)cudaGetLastError();   // the failed allocation's error is reported here, not by the next launch
            return fail(MARS_ERR_OOM, "mars_cmng_build: kNN buffers");
        }
        bcache.entries = entries;
        bcache.rows = count;
    }
    int32_t* d_knn = bcache.d_knn;
    int32_t* d_cnt = bcache.d_cnt;
    float* d_vals = bcache.d_vals;
    mars_batch_ctx* bc = bcache.bc;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    MARS_CUDA_TRY(cudaEventCreate(&e0));
    MARS_CUDA_TRY(cudaEventCreate(&e1));
    cudaStream_t st = s->stream;
    cudaEventRecord(e0, st);
    for (int32_t c0 = first; rc == MARS_OK && c0 < first + count; c0 += chunk) {
        const int32_t b = std::min(chunk, first + count - c0);
        const size_t o = (size_t)(c0 - first);
        // rows as queries, each leaving itself out; plain dot products
        // (lambda = 0: weight exactly 1)
        rc = mars::batch_topk(s, bc, s->d_E + (size_t)c0 * s->pitch, s->pitch, b, 0.0f, 0.0f, -1, 0, k_init, 0,
                              c0, d_knn + o * k_init, d_vals + o * k_init, d_cnt + o, st);
    }
    if (rc == MARS_OK) {
        select_kernel<<<(unsigned)(((int64_t)count * 32 + 255) / 256), 256, 0, st>>>(
            d_knn, d_cnt, k_init, s->d_mod, first, count, degree, degree_cross, num_modalities, d_neighbors);
        if (cudaGetLastError() != cudaSuccess) rc = fail(MARS_ERR_CUDA, "mars_cmng_build: select launch");
    }
    if (rc == MARS_OK) {
        cudaEventRecord(e1, st);
        if (cudaStreamSynchronize(st) != cudaSuccess) rc = fail(MARS_ERR_CUDA, "mars_cmng_build: sync");
        float ms = 0.f;
        cudaEventElapsedTime(&ms, e0, e1);
        if (build_ms) *build_ms = ms;
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    return rc;
}

int mars_cmng_knn(const mars_store* s, int32_t k, int32_t* d_ids, float* d_vals, int32_t* d_counts) {
    if (s == nullptr || d_ids == nullptr || d_vals == nullptr) return fail(MARS_ERR_INVALID, "mars_cmng_knn: NULL argument");
    const int32_t N = s->n;
    if (k <= 0 || k > MARS_MAX_TOP_K || k > N - 1) return fail(MARS_ERR_INVALID, "mars_cmng_knn: k out of range");
    MarsDeviceGuard g(s->device);
    const int32_t chunk = std::min(N, 4096);
    mars_batch_ctx* bc = nullptr;
    MARS_TRY(mars_batch_ctx_create(s->device, N, s->dim, chunk, k, &bc));
    int rc = MARS_OK;
    for (int32_t c0 = 0; rc == MARS_OK && c0 < N; c0 += chunk) {
        const int32_t b = std::min(chunk, N - c0);
        rc = mars::batch_topk(s, bc, s->d_E + (size_t)c0 * s->pitch, s->pitch, b, 0.0f, 0.0f, -1, 0, k, 0, c0,
                              d_ids + (size_t)c0 * k, d_vals + (size_t)c0 * k, d_counts ? d_counts + c0 : nullptr,
                              s->stream);
    }
    if (rc == MARS_OK && cudaStreamSynchronize(s->stream) != cudaSuccess) rc = fail(MARS_ERR_CUDA, "mars_cmng_knn: sync");
    mars_batch_ctx_destroy(bc);
    return rc;
}

static int cmng_search_launch(const mars_store* s, const int32_t* d_neighbors, int32_t degree,
                              const float* d_queries, int32_t query_pitch, int32_t nq, float t_q,
                              const mars_cmng_config* cfg, int32_t* d_ids, float* d_scores, int32_t* d_mods,
                              int32_t* d_counts, int32_t* d_iters, int32_t* d_scored, void* stream, int* ticket);

int mars_cmng_search_batch(const mars_store* s, const int32_t* d_neighbors, int32_t degree,
                           const float* d_queries, int32_t query_pitch, int32_t nq, float t_q,
                           const mars_cmng_config* cfg, int32_t* d_ids, float* d_scores, int32_t* d_mods,
                           int32_t* d_counts, int32_t* d_iters, int32_t* d_scored, void* stream) {
    return cmng_search_launch(s, d_neighbors, degree, d_queries, query_pitch, nq, t_q, cfg, d_ids, d_scores, d_mods,
                              d_counts, d_iters, d_scored, stream, nullptr);
}

// The beam-search launch; ticket (device int, may be NULL) hands the queries
// out dynamically and is zeroed here on the stream first.
static int cmng_search_launch(const mars_store* s, const int32_t* d_neighbors, int32_t degree,
                              const float* d_queries, int32_t query_pitch, int32_t nq, float t_q,
                              const mars_cmng_config* cfg, int32_t* d_ids, float* d_scores, int32_t* d_mods,
                              int32_t* d_counts, int32_t* d_iters, int32_t* d_scored, void* stream, int* ticket) {
    if (s == nullptr || d_neighbors == nullptr || d_queries == nullptr || cfg == nullptr || d_ids == nullptr ||
        d_scores == nullptr || d_counts == nullptr)
        return fail(MARS_ERR_INVALID, "mars_cmng_search_batch: NULL argument");
    if (degree <= 0 || degree > kMaxDegree) return fail(MARS_ERR_INVALID, "mars_cmng_search_batch: degree must be in [1, 128]");
    if (cfg->K <= 0 || cfg->max_iterations < 0 || cfg->num_parents < 0 || cfg->beam_width <= 0)
        return fail(MARS_ERR_INVALID, "mars_cmng_search_batch: bad configuration");
    if (query_pitch < s->dim || s->n <= 0 || s->dim < 2)
        return fail(MARS_ERR_INVALID, "mars_cmng_search_batch: query pitch, empty store or dim < 2");
    if (nq == 0) return MARS_OK;
    const int hs = hash_size_for(cfg->max_iterations, degree);
    if (hs > 32768) return fail(MARS_ERR_UNSUPPORTED, "mars_cmng_search_batch: max_iterations x degree too large");
    MarsDeviceGuard g(s->device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : s->stream;
    MARS_CUDA_TRY(cudaStreamWaitEvent(st, s->written, 0));
    SearchArgs a{};
    a.nbrs = d_neighbors;
    a.E = s->d_E;
    a.ts = s->d_ts;
    a.mod = s->d_mod;
    a.pitch = s->pitch;
    a.N = s->n;
    a.D = s->dim;
    a.degree = degree;
    a.Q = d_queries;
    a.qpitch = query_pitch;
    a.nq = nq;
    a.t_q = t_q;
    a.lambda = cfg->time_decay_lambda;
    a.K = cfg->K;
    a.beam = std::min(cfg->beam_width, (int32_t)kMaxBeam);   // src/cmng_search.cu:356
    a.max_iter = cfg->max_iterations;
    a.num_parents = cfg->num_parents;
    a.hash_size = hs;
    a.out_ids = d_ids;
    a.out_scores = d_scores;
    a.out_mods = d_mods;
    a.out_cnt = d_counts;
    a.stat_iters = d_iters;
    a.stat_scored = d_scored;
    a.ticket = ticket;
    if (ticket != nullptr) MARS_CUDA_TRY(cudaMemsetAsync(ticket, 0, sizeof(int), st));
    const size_t smem = search_smem(s->dim, hs);
    if (smem > 48 * 1024)
        MARS_CUDA_TRY(cudaFuncSetAttribute(search_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int nb = 0, dev = s->device, sms = 0;
    MARS_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, search_kernel, kSearchThreads, smem));
    MARS_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int grid = std::max(1, std::min(nq, std::max(nb, 1) * sms));
    search_kernel<<<grid, kSearchThreads, smem, st>>>(a);
    MARS_CUDA_TRY(cudaGetLastError());
    return MARS_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
struct mars_cmng_ctx {
    int32_t device = 0;
    int32_t max_queries = 0, K = 0, degree = 0, hops = 0;
    int32_t grid = 0, table = 0, vcap = 0;
    int32_t* d_seed_ids = nullptr;
    float* d_seed_scores = nullptr;
    int32_t* d_seed_cnt = nullptr;
    unsigned long long* d_tags = nullptr;
    unsigned long long* d_states = nullptr;
    int32_t* d_lists = nullptr;
    uint32_t* d_epochs = nullptr;
    int* d_err = nullptr;
    int32_t* d_redo = nullptr;           // max_queries + 3: queries for the global-table BFS, their count,
                                         // the search's and the shared-memory BFS's query tickets
    int32_t smem_nodes = kBfsSlots / 2;  // visited nodes per query in the shared-memory BFS (0: never)
};

extern "C" {

int mars_cmng_ctx_create(int32_t device, int32_t max_queries, int32_t K, int32_t degree, int32_t bfs_hops,
                         int32_t max_nodes, mars_cmng_ctx** out) {
    if (out == nullptr) return fail(MARS_ERR_INVALID, "mars_cmng_ctx_create: out is NULL");
    *out = nullptr;
    if (max_queries <= 0 || K <= 0 || K > MARS_MAX_TOP_K || degree <= 0 || degree > kMaxDegree ||
        bfs_hops < 0 || bfs_hops > 13 || max_nodes <= 0)
        return fail(MARS_ERR_INVALID, "mars_cmng_ctx_create: bad sizes");
    MarsDeviceGuard g(device);
    // visited nodes per query: K * (1 + d + d^2 + ...) capped at max_nodes
    int64_t v = K, lvl = K;
    for (int h = 0; h < bfs_hops; ++h) { lvl = std::min<int64_t>(lvl * degree, max_nodes); v += lvl; }
    v = std::min<int64_t>(v, (int64_t)max_nodes);
    if (v > (1 << 24)) return fail(MARS_ERR_UNSUPPORTED, "mars_cmng_ctx_create: BFS too large");
    int64_t t = 256;
    while (t < 2 * v) t <<= 1;
    auto* c = new mars_cmng_ctx();
    c->device = device;
    c->max_queries = max_queries;
    c->K = K;
    c->degree = degree;
    c->hops = bfs_hops;
    c->table = (int32_t)t;
    c->vcap = (int32_t)(2 * v);          // ids + scores
    int sms = 0, nb = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, bfs_kernel<1>, kThreads, 0);
    c->grid = std::max(1, std::min(max_queries, sms * std::max(1, std::min(nb, 4))));
    int rc = MARS_OK;
    auto T = [&](cudaError_t e, const char* w) {
        if (e == cudaSuccess) return;
        if (rc == MARS_OK) rc = cuda_fail(e, w, __FILE__, __LINE__);   // records the first failure
        else (void)cudaGetLastError();                                 // later ones only clear the state
    };
    T(cudaMalloc(&c->d_seed_ids, (size_t)max_queries * K * 4), "seeds");
    T(cudaMalloc(&c->d_seed_scores, (size_t)max_queries * K * 4), "seeds");
    T(cudaMalloc(&c->d_seed_cnt, (size_t)max_queries * 4), "seeds");
    T(cudaMalloc(&c->d_tags, (size_t)c->grid * t * 8), "visited tables");
    T(cudaMalloc(&c->d_states, (size_t)c->grid * t * 8), "visited tables");
    T(cudaMalloc(&c->d_lists, (size_t)c->grid * c->vcap * 4), "level lists");
    T(cudaMalloc(&c->d_epochs, (size_t)c->grid * 4), "epochs");
    T(cudaMalloc(&c->d_err, sizeof(int)), "error word");
    T(cudaMalloc(&c->d_redo, ((size_t)max_queries + 3) * 4), "BFS redo list and query tickets");
    if (rc == MARS_OK) {
        T(cudaFuncSetAttribute(bfs_smem_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kBfsSmemBytes), "attribute");
        T(cudaFuncSetAttribute(bfs_smem_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kBfsSmemBytes), "attribute");
        T(cudaFuncSetAttribute(bfs_smem_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kBfsSmemBytes), "attribute");
        T(cudaFuncSetAttribute(bfs_smem_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kBfsSmemBytes), "attribute");
    }
    if (rc == MARS_OK) T(cudaMemset(c->d_epochs, 0, (size_t)c->grid * 4), "memset");
    if (rc == MARS_OK) T(cudaMemset(c->d_err, 0, sizeof(int)), "memset");
    if (rc != MARS_OK) { mars_cmng_ctx_destroy(c); return rc; }
    *out = c;
    return MARS_OK;
}

int mars_cmng_ctx_set_bfs_smem_nodes(mars_cmng_ctx* c, int32_t max_nodes) {
    if (c == nullptr) return fail(MARS_ERR_INVALID, "mars_cmng_ctx_set_bfs_smem_nodes: NULL context");
    if (max_nodes < 0 || max_nodes > kBfsSlots / 2)
        return fail(MARS_ERR_INVALID, "mars_cmng_ctx_set_bfs_smem_nodes: need 0 <= max_nodes <= " +
                                          std::to_string(kBfsSlots / 2));
    c->smem_nodes = max_nodes;
    return MARS_OK;
}

int mars_cmng_ctx_destroy(mars_cmng_ctx* c) {
    if (c == nullptr) return MARS_OK;
    MarsDeviceGuard g(c->device);
    cudaFree(c->d_seed_ids); cudaFree(c->d_seed_scores); cudaFree(c->d_seed_cnt);
    cudaFree(c->d_tags); cudaFree(c->d_states); cudaFree(c->d_lists); cudaFree(c->d_epochs);
    cudaFree(c->d_err);
    cudaFree(c->d_redo);
    delete c;
    return MARS_OK;
}

int mars_cmng_search_bfs_batch(const mars_store* s, mars_cmng_ctx* c, const int32_t* d_neighbors, int32_t degree,
                               const float* d_queries, int32_t query_pitch, int32_t nq, float t_q,
                               const mars_cmng_config* cfg, int32_t bfs_hops, float bfs_score_decay,
                               int32_t use_importance, int32_t* d_ids, float* d_scores, int32_t* d_mods,
                               int32_t* d_hops, int32_t* d_counts, int32_t* d_visited, void* stream) {
    if (s == nullptr || c == nullptr || cfg == nullptr || d_ids == nullptr || d_scores == nullptr ||
        d_counts == nullptr)
        return fail(MARS_ERR_INVALID, "mars_cmng_search_bfs_batch: NULL argument");
    if (nq > c->max_queries || cfg->K != c->K || degree != c->degree || bfs_hops != c->hops)
        return fail(MARS_ERR_INVALID, "mars_cmng_search_bfs_batch: arguments do not match the context");
    if ((s->dim & 3) != 0 || (query_pitch & 3) != 0 || (reinterpret_cast<uintptr_t>(d_queries) & 15u) != 0)
        return fail(MARS_ERR_INVALID, "mars_cmng_search_bfs_batch: dim and query rows must be float4 aligned");
    if (nq == 0) return MARS_OK;
    MarsDeviceGuard g(s->device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : s->stream;
    // 1. beam search into the context's seed buffers
    int* tickets = reinterpret_cast<int*>(c->d_redo + c->max_queries + 1);
    MARS_TRY(cmng_search_launch(s, d_neighbors, degree, d_queries, query_pitch, nq, t_q, cfg, c->d_seed_ids,
                                c->d_seed_scores, nullptr, c->d_seed_cnt, nullptr, nullptr, st, tickets));
    // 2. BFS + final top-K
    BfsArgs2 a{};
    a.nbrs = d_neighbors;
    a.degree = degree;
    a.E = s->d_E;
    a.ts = s->d_ts;
    a.imp = s->d_imp;
    a.mod = s->d_mod;
    a.pitch4 = s->pitch / 4;
    a.nc = (s->dim + 3) / 4;
    a.N = s->n;
    a.Q = d_queries;
    a.qpitch = query_pitch;
    a.nq = nq;
    a.t_q = t_q;
    a.lambda = cfg->time_decay_lambda;
    a.hop_decay = bfs_score_decay;
    a.use_imp = use_importance;
    a.hops = bfs_hops;
    a.K = cfg->K;
    a.seed_ids = c->d_seed_ids;
    a.seed_scores = c->d_seed_scores;
    a.seed_cnt = c->d_seed_cnt;
    a.seed_stride = cfg->K;
    a.tags = c->d_tags;
    a.states = c->d_states;
    a.lists = c->d_lists;
    a.epochs = c->d_epochs;
    a.table = c->table;
    a.vcap = c->vcap;
    a.out_ids = d_ids;
    a.out_scores = d_scores;
    a.out_mods = d_mods;
    a.out_hops = d_hops;
    a.out_cnt = d_counts;
    a.out_visited = d_visited;
    a.err = c->d_err;
    const int grid = std::min(c->grid, nq);
    auto launch = [&](auto kfn, size_t smem) { kfn<<<grid, kThreads, smem, st>>>(a); };
    if (c->smem_nodes > 0) {
        // shared-memory visited tables first; the queries that outgrow them
        // go to the global-table kernel, which answers only those
        a.redo = c->d_redo;
        a.redo_cnt = c->d_redo + c->max_queries;
        a.smem_nodes = c->smem_nodes;
        a.ticket = tickets + 1;
        MARS_CUDA_TRY(cudaMemsetAsync(a.redo_cnt, 0, sizeof(int32_t), st));
        MARS_CUDA_TRY(cudaMemsetAsync(a.ticket, 0, sizeof(int), st));
        if (cfg->K <= 32) launch(bfs_smem_kernel<1>, kBfsSmemBytes);
        else if (cfg->K <= 64) launch(bfs_smem_kernel<2>, kBfsSmemBytes);
        else if (cfg->K <= 128) launch(bfs_smem_kernel<4>, kBfsSmemBytes);
        else launch(bfs_smem_kernel<8>, kBfsSmemBytes);
        MARS_CUDA_TRY(cudaGetLastError());
    }
    if (cfg->K <= 32) launch(bfs_kernel<1>, 0);
    else if (cfg->K <= 64) launch(bfs_kernel<2>, 0);
    else if (cfg->K <= 128) launch(bfs_kernel<4>, 0);
    else launch(bfs_kernel<8>, 0);
    MARS_CUDA_TRY(cudaGetLastError());
    return MARS_OK;
}

}  // extern "C"
