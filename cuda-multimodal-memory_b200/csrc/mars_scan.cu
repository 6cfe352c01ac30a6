// mars_scan.cu -- S1: fused score x decay x importance -> top-K in one pass.
//
// Replaces stages 1-3 of the reference pipeline (src/memory_cuda.cu:936-1021:
// cublasSgemv or cosine_similarity_kernel -> temporal_rerank_kernel -> CUB
// radix sort of N pairs) with a single streaming kernel that never writes a
// score array:
//
//  * each warp owns a contiguous range of rows (balanced to +-1 row) and
//    streams them with 128-bit read-only loads, two rows in flight per warp;
//  * the query lives in registers (lane l holds float4 chunks l, l+32, ...);
//  * the row's fused score is formed in registers and offered to a
//    warp-resident ranked list (WarpTopK) -- almost every row is rejected by a
//    single compare against the list's threshold;
//  * warps merge into a CTA list in shared memory, CTAs write their list to a
//    small partial buffer, and the last CTA to finish (ticket counter, no
//    spinning) merges all partial lists and, for the query pipeline, seeds the
//    BFS state.
//
// HBM traffic per row: pitch*4 bytes of embedding + 4 B timestamp
// (+4 B importance, +4 B modality when used); nothing else scales with N.
#include "mars_common.cuh"
#include "mars_kernels.cuh"

namespace mars {

constexpr int kStageEntries = 3072;   // 24 KB of staged (score, id) pairs

template <int KPL, int CPL, bool ALL>
__global__ void __launch_bounds__(kScanThreads, 2) scan_topk_kernel(const ScanArgs a) {
    __shared__ float   s_val[kScanWarps][kMaxTopK];
    __shared__ int32_t s_idx[kScanWarps][kMaxTopK];
    __shared__ float   s_stage_v[kStageEntries];
    __shared__ int32_t s_stage_i[kStageEntries];
    __shared__ bool    s_last;

    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const MarsQueryDesc& d = a.d;
    const float t_q = desc_tq(d, a.dyn), lambda = d.lambda;
    const int32_t filter = d.filter;
    const bool use_imp = d.use_imp != 0 && a.s.imp != nullptr;
    const int K = d.K;
    const int32_t id_off = d.row_offset;
    const int32_t n = *a.s.d_n;
    const int nc = a.s.nc;

    // query chunks in registers
    float4 qv[CPL];
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
        const int c = lane + 32 * j;
        qv[j] = c < nc ? a.q[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    }

    WarpTopK<KPL> top;
    top.init(K);

    // balanced contiguous row range of this warp
    const int64_t W = (int64_t)gridDim.x * kScanWarps;
    const int64_t w = (int64_t)blockIdx.x * kScanWarps + warp;
    const int32_t r0 = (int32_t)((int64_t)n * w / W);
    const int32_t r1 = (int32_t)((int64_t)n * (w + 1) / W);

    // metadata window: lane l holds row wbase + l
    int32_t wbase = r0;
    float ts_w = 0.f, imp_w = 1.f;
    int32_t mod_w = 0;
    auto load_meta = [&](int32_t base) {
        const int32_t r = base + lane;
        if (r < r1) {
            ts_w = __ldg(a.s.ts + r);
            if (use_imp) imp_w = __ldg(a.s.imp + r);
            if (filter >= 0) mod_w = __ldg(a.s.mod + r);
        }
    };
    load_meta(wbase);

    auto process = [&](int32_t row, float dot) {
        if (row - wbase >= 32) { wbase += 32; load_meta(wbase); }
        const int src = row - wbase;
        const float t = __shfl_sync(MARS_FULL_MASK, ts_w, src);
        const float im = __shfl_sync(MARS_FULL_MASK, imp_w, src);
        const int32_t m = __shfl_sync(MARS_FULL_MASK, mod_w, src);
        if ((filter >= 0 && m != filter) || row + 1 == d.exclude_plus1) {
            if (ALL && lane == 0) a.all_scores[row] = -FLT_MAX;
            return;
        }
        float f = fused_weight_apply(dot, t, t_q, lambda);
        if (use_imp) f = f * im;
        if (ALL && lane == 0) a.all_scores[row] = f;
        top.push(f, row + id_off, lane);
    };

    const float4* __restrict__ E4 = reinterpret_cast<const float4*>(a.s.E);
    int32_t r = r0;
    for (; r + 1 < r1; r += 2) {
        const float4* p0 = E4 + (int64_t)r * a.s.pitch4;
        const float4* p1 = p0 + a.s.pitch4;
        float4 e0[CPL], e1[CPL];
#pragma unroll
        for (int j = 0; j < CPL; ++j) {
            const int c = lane + 32 * j;
            if (c < nc) { e0[j] = ldg_stream(p0 + c); e1[j] = ldg_stream(p1 + c); }
        }
        float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
        for (int j = 0; j < CPL; ++j) {
            const int c = lane + 32 * j;
            if (c < nc) { acc0 = fma4(e0[j], qv[j], acc0); acc1 = fma4(e1[j], qv[j], acc1); }
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
            const float x0 = __shfl_xor_sync(MARS_FULL_MASK, acc0, off);
            const float x1 = __shfl_xor_sync(MARS_FULL_MASK, acc1, off);
            acc0 = __fadd_rn(acc0, x0);
            acc1 = __fadd_rn(acc1, x1);
        }
        process(r, acc0);
        process(r + 1, acc1);
    }
    if (r < r1) {
        const float4* p0 = E4 + (int64_t)r * a.s.pitch4;
        float acc0 = 0.f;
#pragma unroll
        for (int j = 0; j < CPL; ++j) {
            const int c = lane + 32 * j;
            if (c < nc) acc0 = fma4(ldg_stream(p0 + c), qv[j], acc0);
        }
        process(r, warp_butterfly_sum(acc0));
    }

    // ---- CTA merge ---------------------------------------------------------
    top.store(s_val[warp], s_idx[warp], lane);
    __syncthreads();
    if (warp == 0) {
        for (int ww = 1; ww < kScanWarps; ++ww) top.offer_sorted(s_val[ww], s_idx[ww], K, lane);
        top.store(a.part_val + (int64_t)blockIdx.x * K, a.part_idx + (int64_t)blockIdx.x * K, lane);
        __threadfence();
        __syncwarp();
        if (lane == 0) s_last = atomicAdd(a.ticket, 1u) == gridDim.x - 1;
        __syncwarp();
    }
    __syncthreads();
    if (!s_last) return;

    // ---- last CTA: merge every CTA's list ----------------------------------
    // Stage the lists in shared memory with all threads' loads in flight at
    // once (one memory round trip per batch instead of one per list), then
    // let each warp merge a subset of the staged lists.
    __threadfence();
    top.init(K);
    const int lists_per_batch = kStageEntries / K;
    for (int b0 = 0; b0 < (int)gridDim.x; b0 += lists_per_batch) {
        const int nl = min(lists_per_batch, (int)gridDim.x - b0);
        const int ne = nl * K;
        const float* pv = a.part_val + (int64_t)b0 * K;
        const int32_t* pi = a.part_idx + (int64_t)b0 * K;
#pragma unroll 4
        for (int j = threadIdx.x; j < ne; j += kScanThreads) {
            s_stage_v[j] = __ldcg(pv + j);   // written by other SMs: bypass L1
            s_stage_i[j] = __ldcg(pi + j);
        }
        __syncthreads();
        for (int l = warp; l < nl; l += kScanWarps)
            top.offer_sorted(s_stage_v + l * K, s_stage_i + l * K, K, lane);
        __syncthreads();
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
            a.out_val[p] = valid ? top.v[sl] : -INFINITY;
            a.out_idx[p] = valid ? top.i[sl] : -1;
        }
    }
    if (lane == 0) {
        *a.out_cnt = cnt;
        *a.ticket = 0u;   // re-arm for the next launch
    }
    if (a.vis_ids != nullptr) {
        // seed the BFS: level 0 = the top-K, stamp (epoch, level 0)
        const unsigned long long st0 =
            (unsigned long long)((desc_epoch(d, a.dyn) << 4) | 15u) << 32;
#pragma unroll
        for (int sl = 0; sl < KPL; ++sl) {
            const int p = sl * 32 + lane;
            if (p < cnt) {
                const int32_t u = top.i[sl] - id_off;
                a.stamp[u] = st0 | f2key(top.v[sl]);
                a.vis_ids[p] = u;
                a.vis_score[p] = top.v[sl];
            }
        }
        if (lane == 0) {
            a.lvl[0] = 0;
            a.lvl[1] = cnt;
            a.lvl[16] = cnt;
        }
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

cudaError_t launch_topk_merge(const int32_t* ids_in, const float* vals_in, int n_lists, int K, int Q,
                              int32_t* ids_out, float* vals_out, int32_t* cnt, cudaStream_t st) {
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
