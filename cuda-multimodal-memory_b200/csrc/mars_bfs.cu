// mars_bfs.cu -- B1/B2: deterministic multi-hop BFS from the top-K seeds and
// the final top-K over every visited node.
//
// Reference: bfs_init_seeds_kernel / bfs_expand_device_driven_kernel /
// compact_results_kernel + host sort (src/memory_cuda.cu:450-549, :1024-1064,
// :1127-1146).  The reference claims a neighbour with atomicCAS (the first
// parent to arrive sets its score), launches min(N, 20K) warps per hop (large
// frontiers are cut) and then scans all N hop counts to compact the visited
// set.  Here:
//
//  * one 64-bit word per node holds (stamp << 32 | score key) where
//    stamp = (epoch << 4) | (15 - level).  A single atomicMax per edge both
//    claims the node for level h+1 (exactly one thread sees an older epoch and
//    appends the node to the visited list) and keeps the best parent
//    candidate score; nodes of earlier levels carry larger stamps and are
//    left untouched.  The epoch changes every query, so nothing is cleared
//    between queries (the reference memsets N hop counts per query).
//  * the visited list is the concatenation of the levels, so the final
//    selection reads O(visited) entries instead of scanning N.
//  * a node's own score is recomputed with the same canonical dot product as
//    the scan kernel (bit-identical), when the node is first expanded or in
//    the finalize kernel for the last level.
//  * frontiers are never truncated; persistent grids walk the device-side
//    level bounds, and the last CTA of each launch (ticket counter) publishes
//    the bounds of the next level.
#include "mars_common.cuh"
#include "mars_kernels.cuh"
#include "mars_b200.h"

namespace mars {

__device__ __forceinline__ float node_score(const BfsArgs& a, const MarsQueryDesc& d, int32_t u,
                                            int lane) {
    if (d.filter >= 0 && __ldg(a.s.mod + u) != d.filter) return -FLT_MAX;
    const float4* row = reinterpret_cast<const float4*>(a.s.E) + (int64_t)u * a.s.pitch4;
    const float dot = warp_dot_canonical(row, a.q, a.s.nc, lane);
    float f = fused_weight_apply(dot, __ldg(a.s.ts + u), desc_tq(d, a.dyn), d.lambda);
    if (d.use_imp != 0 && a.s.imp != nullptr) f = f * __ldg(a.s.imp + u);
    return f;
}

// Finalize the score of a node of level >= 1:
// max over parents of (parent * decay) is in the low word of its stamp.
__device__ __forceinline__ float level_score(const BfsArgs& a, const MarsQueryDesc& d, int32_t u,
                                             int lane) {
    const float own = node_score(a, d, u, lane);
    const float best_parent = key2f((uint32_t)(__ldcg(a.stamp + u) & 0xffffffffull));
    return fmaxf(best_parent, own * 0.8f);
}

__device__ __forceinline__ void claim(const BfsArgs& a, int32_t v, unsigned long long word,
                                      uint32_t epoch_base) {
    const unsigned long long old = atomicMax(a.stamp + v, word);
    if ((uint32_t)(old >> 32) < epoch_base) {
        const int32_t pos = atomicAdd(a.lvl + 16, 1);
        a.vis_ids[pos] = v;
    }
}

__device__ __forceinline__ bool last_block(unsigned int* ticket) {
    __shared__ bool s_last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(ticket, 1u) == gridDim.x - 1;
    __syncthreads();
    if (s_last) __threadfence();
    return s_last;
}

// Expand level `hop` into level hop + 1.
__global__ void __launch_bounds__(kBfsThreads) bfs_hop_kernel(const BfsArgs a, int hop) {
    const MarsQueryDesc& d = a.d;
    const int lane = threadIdx.x & 31;
    const int gw = blockIdx.x * kBfsWarps + (threadIdx.x >> 5);
    const int nw = gridDim.x * kBfsWarps;
    const int32_t beg = a.lvl[hop], end = a.lvl[hop + 1];
    const int32_t n = *a.s.d_n;
    const uint32_t epoch_base = desc_epoch(d, a.dyn) << 4;
    const unsigned long long next_stamp =
        (unsigned long long)(epoch_base | (uint32_t)(15 - (hop + 1))) << 32;

    for (int32_t idx = beg + gw; idx < end; idx += nw) {
        const int32_t u = a.vis_ids[idx];
        float su;
        if (hop == 0) {
            su = a.vis_score[idx];
        } else {
            su = level_score(a, d, u, lane);
            if (lane == 0) a.vis_score[idx] = su;
        }
        const unsigned long long word = next_stamp | f2key(su * d.hop_decay);
        if (a.s.row_offsets != nullptr && u < a.s.csr_n) {
            const int32_t e0 = __ldg(a.s.row_offsets + u), e1 = __ldg(a.s.row_offsets + u + 1);
            for (int32_t e = e0 + lane; e < e1; e += 32) {
                const int32_t v = __ldg(a.s.col_indices + e);
                if (v >= 0 && v < n) claim(a, v, word, epoch_base);
            }
        }
        if (a.s.extra != nullptr && a.s.slack > 0) {
            const int32_t cnt = min(__ldg(a.s.extra_cnt + u), a.s.slack);
            const int32_t* ex = a.s.extra + (int64_t)u * a.s.slack;
            for (int32_t e = lane; e < cnt; e += 32) {
                const int32_t v = __ldg(ex + e);
                if (v >= 0 && v < n) claim(a, v, word, epoch_base);
            }
        }
    }
    if (last_block(a.ticket)) {
        if (threadIdx.x == 0) {
            a.lvl[hop + 2] = atomicAdd(a.lvl + 16, 0);
            *a.ticket = 0u;
        }
    }
}

// Finalize the scores of level `last` and select the top-K of all visited
// nodes by (score desc, id asc).
constexpr int kFinStage = 3072;

template <int KPL>
__global__ void __launch_bounds__(kBfsThreads) bfs_finalize_kernel(const BfsArgs a, int last) {
    __shared__ float   s_val[kBfsWarps][kMaxTopK];
    __shared__ int32_t s_idx[kBfsWarps][kMaxTopK];
    __shared__ float   s_stage_v[kFinStage];
    __shared__ int32_t s_stage_i[kFinStage];
    const MarsQueryDesc& d = a.d;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gw = blockIdx.x * kBfsWarps + warp;
    const int nw = gridDim.x * kBfsWarps;
    if (last > 0) {
        const int32_t beg = a.lvl[last], end = a.lvl[last + 1];
        for (int32_t idx = beg + gw; idx < end; idx += nw) {
            const int32_t u = a.vis_ids[idx];
            const float su = level_score(a, d, u, lane);
            if (lane == 0) a.vis_score[idx] = su;
        }
    }
    if (!last_block(a.ticket)) return;

    const int K = d.K;
    const int32_t total = a.lvl[last + 1];
    WarpTopK<KPL> top;
    top.init(K);
    // rank every visited node by (score desc, node id asc); a node's level
    // is recovered from its stamp when the result is written.  The visited
    // list is staged in shared memory batch by batch so that every thread's
    // loads are in flight together.
    for (int32_t b0 = 0; b0 < total; b0 += kFinStage) {
        const int ne = min(kFinStage, total - b0);
#pragma unroll 4
        for (int j = threadIdx.x; j < ne; j += kBfsThreads) {
            s_stage_v[j] = __ldcg(a.vis_score + b0 + j);
            s_stage_i[j] = __ldcg(a.vis_ids + b0 + j);
        }
        __syncthreads();
        for (int base = warp * 32; base < ne; base += kBfsWarps * 32) {
            const int j = base + lane;
            float s = -INFINITY;
            int32_t id = INT32_MAX;
            if (j < ne) { s = s_stage_v[j]; id = s_stage_i[j]; }
            top.offer_lanes(s, id, j < ne, lane);
        }
        __syncthreads();
    }
    top.store(s_val[warp], s_idx[warp], lane);
    __syncthreads();
    if (warp != 0) return;
    for (int ww = 1; ww < kBfsWarps; ++ww) top.offer_sorted(s_val[ww], s_idx[ww], K, lane);

    mars_query_result* out = reinterpret_cast<mars_query_result*>(a.results);
    int cnt = 0;
#pragma unroll
    for (int sl = 0; sl < KPL; ++sl) {
        const int p = sl * 32 + lane;
        const bool valid = p < K && top.i[sl] != INT32_MAX;
        cnt += __popc(__ballot_sync(MARS_FULL_MASK, valid));
        if (valid) {
            const int32_t u = top.i[sl];
            // level of u from its stamp: stamp low nibble = 15 - level
            const uint32_t st = (uint32_t)(__ldcg(a.stamp + u) >> 32);
            mars_query_result r;
            r.node_id = u + d.row_offset;
            r.score = top.v[sl];
            r.modality = __ldg(a.s.mod + u);
            r.hops_from_seed = 15 - (int)(st & 15u);
            out[p] = r;
        }
    }
    if (lane == 0) {
        a.result_cnt[0] = cnt;
        a.result_cnt[1] = total;
        *a.ticket = 0u;
    }
}

cudaError_t launch_bfs_hop(const BfsArgs& a, int hop, int grid, cudaStream_t st) {
    bfs_hop_kernel<<<grid, kBfsThreads, 0, st>>>(a, hop);
    return cudaGetLastError();
}

cudaError_t launch_bfs_finalize(const BfsArgs& a, int last_level, int k_max, int grid,
                                cudaStream_t st) {
    if (k_max <= 32)
        bfs_finalize_kernel<1><<<grid, kBfsThreads, 0, st>>>(a, last_level);
    else if (k_max <= 64)
        bfs_finalize_kernel<2><<<grid, kBfsThreads, 0, st>>>(a, last_level);
    else if (k_max <= 128)
        bfs_finalize_kernel<4><<<grid, kBfsThreads, 0, st>>>(a, last_level);
    else
        bfs_finalize_kernel<8><<<grid, kBfsThreads, 0, st>>>(a, last_level);
    return cudaGetLastError();
}

}  // namespace mars
