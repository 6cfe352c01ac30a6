// mars_scan.cu -- S1: fused score x decay x importance -> top-K in one pass.
//
// Replaces stages 1-3 of the reference pipeline (src/memory_cuda.cu:936-1021:
// cublasSgemv or cosine_similarity_kernel -> temporal_rerank_kernel -> CUB
// radix sort of N pairs) with a single streaming kernel that never writes a
// score array:
//
//  * the streaming part (mars_scan_body.cuh) keeps a warp-resident ranked
//    list per warp, merges them per CTA and writes one partial list per CTA;
//  * the last CTA to finish (ticket counter, no spinning) merges the partial
//    lists, writes the top-K and, for the multi-kernel query pipeline, seeds
//    the BFS state.
//
// HBM traffic per row: pitch*4 bytes of embedding + 4 B timestamp
// (+4 B importance, +4 B modality when used); nothing else scales with N.
#include "mars_scan_body.cuh"

namespace mars {

template <int KPL, int CPL, bool ALL>
__global__ void __launch_bounds__(kScanThreads, 2) scan_topk_kernel(const ScanArgs a) {
    __shared__ ScanShared sm;
    const MarsQueryDesc& d = a.d;
    const SlotOne sl{a};
    if (!scan_rows<KPL, CPL, ALL>(a, sl, a.q, desc_tq(d, a.dyn), sm)) return;

    // ---- last CTA: merge every CTA's list ----------------------------------
    const int cnt = final_merge<KPL>(a, sl, sm);
    const int K = d.K;
    const int32_t id_off = d.row_offset;
    for (int p = threadIdx.x; p < K; p += kScanThreads) {
        const bool valid = p < cnt;
        a.out_val[p] = valid ? key_score(sm.keys()[p]) : -INFINITY;
        a.out_idx[p] = valid ? key_id(sm.keys()[p]) : -1;
    }
    if (threadIdx.x == 0) {
        *a.out_cnt = cnt;
        rearm(sl);
    }
    if (a.vis_ids != nullptr) {
        // seed the BFS: level 0 = the top-K, stamp (epoch, level 0)
        const unsigned long long st0 =
            (unsigned long long)((desc_epoch(d, a.dyn) << 4) | 15u) << 32;
        for (int p = threadIdx.x; p < cnt; p += kScanThreads) {
            const unsigned long long k = sm.keys()[p];
            const float v = key_score(k);
            const int32_t u = key_id(k) - id_off;
            a.stamp[u] = st0 | f2key(v);
            a.vis_ids[p] = u;
            a.vis_score[p] = v;
        }
        if (threadIdx.x == 0) {
            a.lvl[0] = 0;
            a.lvl[1] = cnt;
            a.lvl[16] = cnt;
        }
    }
}

// ---------------------------------------------------------------------------
// Several queries' scans in one launch: a 2-D grid, blockIdx.y = query.  The
// block scheduler starts query i + 1's CTAs as query i's finish, so the last
// CTA of query i merges while the others already stream the next query, and
// there is one launch instead of nq.  Each query has its own slot (partial
// lists, ticket, row counter); query i's results are those of a
// scan_topk_kernel launch for it alone.
template <int KPL, int CPL>
__global__ void __launch_bounds__(kScanThreads, 2) scan_multi_kernel(const __grid_constant__ ScanArgs a,
                                                                      const float* __restrict__ Q,
                                                                      int64_t qpitch) {
    __shared__ ScanShared sm;
    const int qi = blockIdx.y;
    if (a.only != nullptr && a.only[qi] == 0) return;   // every CTA of the query leaves
    const SlotMulti sl{a, qi};
    const float4* q = reinterpret_cast<const float4*>(Q + qi * qpitch);
    if (!scan_rows<KPL, CPL, false>(a, sl, q, a.d.t_q, sm)) return;
    const int K = a.d.K;
    const int cnt = final_merge<KPL>(a, sl, sm);
    for (int p = threadIdx.x; p < K; p += kScanThreads) {
        const bool valid = p < cnt;
        a.out_val[(int64_t)qi * K + p] = valid ? key_score(sm.keys()[p]) : -INFINITY;
        a.out_idx[(int64_t)qi * K + p] = valid ? key_id(sm.keys()[p]) : -1;
    }
    if (threadIdx.x == 0) {
        if (a.out_cnt != nullptr) a.out_cnt[qi] = cnt;
        rearm(sl);
    }
}

// ---------------------------------------------------------------------------
// Merge of ranked lists (sharded top-K after an all-gather).  Block q merges
// the n_lists lists of query q; list l of query q starts at (l * Q + q) * K,
// i.e. the rank-major layout of an all-gather of per-rank [Q][K] buffers.
template <int KPL>
__global__ void __launch_bounds__(kScanThreads) topk_merge_kernel(const int32_t* __restrict__ ids_in,
                                                                  const float* __restrict__ vals_in,
                                                                  int n_lists, int K, int Q,
                                                                  int32_t* ids_out, float* vals_out,
                                                                  int32_t* cnt_out) {
    __shared__ float   s_val[kScanWarps][kMaxTopK];
    __shared__ int32_t s_idx[kScanWarps][kMaxTopK];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int qi = blockIdx.x;
    ids_out += (int64_t)qi * K;
    vals_out += (int64_t)qi * K;
    if (cnt_out) cnt_out += qi;
    WarpTopK<KPL> top;
    top.init(K);
    for (int b = warp; b < n_lists; b += kScanWarps) {
        const float* pv = vals_in + ((int64_t)b * Q + qi) * K;
        const int32_t* pi = ids_in + ((int64_t)b * Q + qi) * K;
        for (int base = 0; base < K; base += 32) {
            const int j = base + lane;
            float s = -INFINITY;
            int32_t id = INT32_MAX;
            if (j < K && pi[j] >= 0) { s = pv[j]; id = pi[j]; }
            const unsigned m = __ballot_sync(MARS_FULL_MASK, top.admits(s, id));
            if (m == 0) break;
            top.offer_lanes(s, id, j < K, lane);
        }
    }
    top.store(s_val[warp], s_idx[warp], lane);
    __syncthreads();
    if (warp != 0) return;
    for (int ww = 1; ww < kScanWarps; ++ww) top.offer_sorted(s_val[ww], s_idx[ww], K, lane);
    int cnt = 0;
#pragma unroll
    for (int sl = 0; sl < KPL; ++sl) {
        const int p = sl * 32 + lane;
        const bool valid = p < K && top.i[sl] != INT32_MAX;
        cnt += __popc(__ballot_sync(MARS_FULL_MASK, valid));
        if (p < K) {
            vals_out[p] = valid ? top.v[sl] : -INFINITY;
            ids_out[p] = valid ? top.i[sl] : -1;
        }
    }
    if (lane == 0 && cnt_out) *cnt_out = cnt;
}

// The same merge when all of a query's entries fit the key buffer
// (n_lists * K <= kMergeKeys): every valid entry becomes a 64-bit rank key in
// shared memory and the block's radix selection picks the top-K; no serial
// inserts.
__global__ void __launch_bounds__(kScanThreads) topk_merge_select_kernel(const int32_t* __restrict__ ids_in,
                                                                         const float* __restrict__ vals_in,
                                                                         int n_lists, int K, int Q,
                                                                         int32_t* ids_out, float* vals_out,
                                                                         int32_t* cnt_out) {
    __shared__ unsigned long long s_keys[kMergeKeys];
    __shared__ __align__(16) int s_hist[2048];   // also read as 64-bit keys
    __shared__ int s_misc[16];
    constexpr int kPer = kMergeKeys / kScanThreads;
    const int qi = blockIdx.x;
    const int total = n_lists * K;
    if (threadIdx.x == 0) s_misc[15] = 0;
    int32_t id[kPer];
    float v[kPer];
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
        const int j = u * kScanThreads + threadIdx.x;
        id[u] = -1;
        if (j < total) {
            const int l = j / K, e = j - l * K;
            const int64_t p = ((int64_t)l * Q + qi) * K + e;
            id[u] = __ldg(ids_in + p);
            v[u] = __ldg(vals_in + p);
        }
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < kPer; ++u)
        warp_append(id[u] >= 0, id[u] >= 0 ? rank_key(v[u], id[u]) : 0ull, s_keys, &s_misc[15], kMergeKeys);
    __syncthreads();
    const int M = s_misc[15];
    __syncthreads();
    const int cnt = block_select_topk<kScanThreads>(s_keys, M, K, s_hist, s_misc);
    ids_out += (int64_t)qi * K;
    vals_out += (int64_t)qi * K;
    for (int p = threadIdx.x; p < K; p += kScanThreads) {
        const bool valid = p < cnt;
        vals_out[p] = valid ? key_score(s_keys[p]) : -INFINITY;
        ids_out[p] = valid ? key_id(s_keys[p]) : -1;
    }
    if (threadIdx.x == 0 && cnt_out) cnt_out[qi] = cnt;
}

// ---------------------------------------------------------------------------
// Dispatch.  CPL: float4 chunks per lane (D = 128 * CPL covers 768 with 6).
template <int KPL, bool ALL>
static cudaError_t launch_scan_kpl(const ScanArgs& a, int grid, cudaStream_t st) {
    const int cpl = (a.s.nc + 31) / 32;
    switch (cpl) {
    case 1: scan_topk_kernel<KPL, 1, ALL><<<grid, kScanThreads, 0, st>>>(a); break;
    case 2: scan_topk_kernel<KPL, 2, ALL><<<grid, kScanThreads, 0, st>>>(a); break;
    case 3: scan_topk_kernel<KPL, 3, ALL><<<grid, kScanThreads, 0, st>>>(a); break;
    case 4: scan_topk_kernel<KPL, 4, ALL><<<grid, kScanThreads, 0, st>>>(a); break;
    case 5: scan_topk_kernel<KPL, 5, ALL><<<grid, kScanThreads, 0, st>>>(a); break;
    case 6: scan_topk_kernel<KPL, 6, ALL><<<grid, kScanThreads, 0, st>>>(a); break;
    case 7: scan_topk_kernel<KPL, 7, ALL><<<grid, kScanThreads, 0, st>>>(a); break;
    case 8: scan_topk_kernel<KPL, 8, ALL><<<grid, kScanThreads, 0, st>>>(a); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_scan_topk(const ScanArgs& a, int k_max, int grid, cudaStream_t st) {
    const bool all = a.all_scores != nullptr;
    if (k_max <= 32) return all ? launch_scan_kpl<1, true>(a, grid, st) : launch_scan_kpl<1, false>(a, grid, st);
    if (k_max <= 64) return all ? launch_scan_kpl<2, true>(a, grid, st) : launch_scan_kpl<2, false>(a, grid, st);
    if (k_max <= 128) return all ? launch_scan_kpl<4, true>(a, grid, st) : launch_scan_kpl<4, false>(a, grid, st);
    return all ? launch_scan_kpl<8, true>(a, grid, st) : launch_scan_kpl<8, false>(a, grid, st);
}

template <int KPL>
static cudaError_t launch_multi_kpl(const ScanArgs& a, const float* Q, int64_t qpitch, int nq, int grid,
                                    cudaStream_t st) {
    switch ((a.s.nc + 31) / 32) {
    case 1: scan_multi_kernel<KPL, 1><<<dim3(grid, nq), kScanThreads, 0, st>>>(a, Q, qpitch); break;
    case 2: scan_multi_kernel<KPL, 2><<<dim3(grid, nq), kScanThreads, 0, st>>>(a, Q, qpitch); break;
    case 3: scan_multi_kernel<KPL, 3><<<dim3(grid, nq), kScanThreads, 0, st>>>(a, Q, qpitch); break;
    case 4: scan_multi_kernel<KPL, 4><<<dim3(grid, nq), kScanThreads, 0, st>>>(a, Q, qpitch); break;
    case 5: scan_multi_kernel<KPL, 5><<<dim3(grid, nq), kScanThreads, 0, st>>>(a, Q, qpitch); break;
    case 6: scan_multi_kernel<KPL, 6><<<dim3(grid, nq), kScanThreads, 0, st>>>(a, Q, qpitch); break;
    case 7: scan_multi_kernel<KPL, 7><<<dim3(grid, nq), kScanThreads, 0, st>>>(a, Q, qpitch); break;
    case 8: scan_multi_kernel<KPL, 8><<<dim3(grid, nq), kScanThreads, 0, st>>>(a, Q, qpitch); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_scan_multi(const ScanArgs& a, const float* Q, int64_t qpitch, int nq, int grid,
                              cudaStream_t st) {
    const int K = a.d.K;
    if (K <= 32) return launch_multi_kpl<1>(a, Q, qpitch, nq, grid, st);
    if (K <= 64) return launch_multi_kpl<2>(a, Q, qpitch, nq, grid, st);
    if (K <= 128) return launch_multi_kpl<4>(a, Q, qpitch, nq, grid, st);
    return launch_multi_kpl<8>(a, Q, qpitch, nq, grid, st);
}

cudaError_t launch_topk_merge(const int32_t* ids_in, const float* vals_in, int n_lists, int K, int Q,
                              int32_t* ids_out, float* vals_out, int32_t* cnt, cudaStream_t st) {
    if ((int64_t)n_lists * K <= kMergeKeys) {
        topk_merge_select_kernel<<<Q, kScanThreads, 0, st>>>(ids_in, vals_in, n_lists, K, Q, ids_out, vals_out, cnt);
        return cudaGetLastError();
    }
    if (K <= 32)
        topk_merge_kernel<1><<<Q, kScanThreads, 0, st>>>(ids_in, vals_in, n_lists, K, Q, ids_out, vals_out, cnt);
    else if (K <= 64)
        topk_merge_kernel<2><<<Q, kScanThreads, 0, st>>>(ids_in, vals_in, n_lists, K, Q, ids_out, vals_out, cnt);
    else if (K <= 128)
        topk_merge_kernel<4><<<Q, kScanThreads, 0, st>>>(ids_in, vals_in, n_lists, K, Q, ids_out, vals_out, cnt);
    else
        topk_merge_kernel<8><<<Q, kScanThreads, 0, st>>>(ids_in, vals_in, n_lists, K, Q, ids_out, vals_out, cnt);
    return cudaGetLastError();
}

// Load every scan_topk_kernel variant for K <= 128 and D <= 1024 into the
// current device now (with lazy module loading a kernel's code is otherwise
// placed in device memory at its first launch).
int preload_scan_topk_kernels() {
    cudaFuncAttributes fa;
    cudaError_t e = cudaSuccess;
#define MARS_LOAD(KPL_)                                                                               \
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, scan_topk_kernel<KPL_, 1, false>);           \
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, scan_topk_kernel<KPL_, 2, false>);           \
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, scan_topk_kernel<KPL_, 3, false>);           \
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, scan_topk_kernel<KPL_, 4, false>);           \
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, scan_topk_kernel<KPL_, 5, false>);           \
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, scan_topk_kernel<KPL_, 6, false>);           \
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, scan_topk_kernel<KPL_, 7, false>);           \
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, scan_topk_kernel<KPL_, 8, false>)
    MARS_LOAD(1);
    MARS_LOAD(2);
    MARS_LOAD(4);
#undef MARS_LOAD
    return e == cudaSuccess ? 0 : (int)e;
}

int scan_blocks_per_sm(int nc, int k_max) {
    int nb = 0;
    const int cpl = (nc + 31) / 32;
    cudaError_t e = cudaErrorInvalidValue;
#define MARS_OCC(KPL_, CPL_) \
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, scan_topk_kernel<KPL_, CPL_, false>, kScanThreads, 0)
    const int kpl = k_max <= 32 ? 1 : (k_max <= 64 ? 2 : (k_max <= 128 ? 4 : 8));
    if (kpl == 1) {
        switch (cpl) { case 1: MARS_OCC(1, 1); break; case 2: MARS_OCC(1, 2); break; case 3: MARS_OCC(1, 3); break;
                       case 4: MARS_OCC(1, 4); break; case 5: MARS_OCC(1, 5); break; case 6: MARS_OCC(1, 6); break;
                       case 7: MARS_OCC(1, 7); break; default: MARS_OCC(1, 8); break; }
    } else if (kpl == 2) {
        switch (cpl) { case 1: MARS_OCC(2, 1); break; case 2: MARS_OCC(2, 2); break; case 3: MARS_OCC(2, 3); break;
                       case 4: MARS_OCC(2, 4); break; case 5: MARS_OCC(2, 5); break; case 6: MARS_OCC(2, 6); break;
                       case 7: MARS_OCC(2, 7); break; default: MARS_OCC(2, 8); break; }
    } else if (kpl == 4) {
        switch (cpl) { case 1: MARS_OCC(4, 1); break; case 2: MARS_OCC(4, 2); break; case 3: MARS_OCC(4, 3); break;
                       case 4: MARS_OCC(4, 4); break; case 5: MARS_OCC(4, 5); break; case 6: MARS_OCC(4, 6); break;
                       case 7: MARS_OCC(4, 7); break; default: MARS_OCC(4, 8); break; }
    } else {
        switch (cpl) { case 1: MARS_OCC(8, 1); break; case 2: MARS_OCC(8, 2); break; case 3: MARS_OCC(8, 3); break;
                       case 4: MARS_OCC(8, 4); break; case 5: MARS_OCC(8, 5); break; case 6: MARS_OCC(8, 6); break;
                       case 7: MARS_OCC(8, 7); break; default: MARS_OCC(8, 8); break; }
    }
#undef MARS_OCC
    return (e == cudaSuccess && nb > 0) ? nb : 1;
}

}  // namespace mars
