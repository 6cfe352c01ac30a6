// mars_fastq.cu -- the whole single-query pipeline in one kernel launch.
//
// query_memory_fast (src/memory_cuda.cu:924-1158) runs 6-9 dependent launches
// plus host copies per query (SGEMV, rerank, radix sort, seed, one expand per
// hop, compaction, host sort).  For a single query most of that is launch and
// memory latency, so here one launch does everything:
//
//  * the query vector travels inside the kernel's parameter block
//    (__grid_constant__, up to 1024 floats): no host-to-device copy;
//  * every CTA streams its rows as in the scan kernel (mars_scan_body.cuh);
//    with BFS hops each row's fused score is also stored, so the BFS never
//    recomputes a dot product;
//  * the last CTA merges the partial lists, then runs the BFS itself
//    (visited list and level bookkeeping in shared memory, claims by 64-bit
//    atomicMax on the per-node stamp words exactly as bfs_hop_kernel does),
//    ranks the visited set and writes the results straight into the
//    caller's (host-mapped) result buffer.
//
// The last CTA's BFS holds at most kTailCap visited nodes and kLevelCap
// nodes per level.  If a query needs more, the kernel reports count -1 and
// the host runs the multi-kernel pipeline instead (same results).
#include "mars_scan_body.cuh"
#include "mars_b200.h"

namespace mars {

// Store with release semantics at system scope: every write this thread
// made or observed (through the preceding barrier) becomes visible to the
// host no later than the stored value.
__device__ __forceinline__ void store_release_sys(int32_t* p, int32_t v) {
    asm volatile("st.release.sys.global.s32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}

constexpr int kTailCap = kStageEntries;   // visited nodes held by the last CTA
constexpr int kLevelCap = 1024;           // nodes of one BFS level

// Inclusive prefix sum of v[0, L) in place (L <= 4 * NT); returns the total.
template <int NT>
__device__ __forceinline__ int block_inclusive_scan(int* v, int L, int* s_warp) {
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    int x[4], sum = 0;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const int i = t * 4 + u;
        x[u] = i < L ? v[i] : 0;
        sum += x[u];
    }
    int inc = sum;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(MARS_FULL_MASK, inc, off);
        if (lane >= off) inc += y;
    }
    __syncthreads();
    if (lane == 31) s_warp[warp] = inc;
    __syncthreads();
    int run = inc - sum, total = 0;
#pragma unroll
    for (int w = 0; w < NT / 32; ++w) {
        if (w < warp) run += s_warp[w];
        total += s_warp[w];
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const int i = t * 4 + u;
        run += x[u];
        if (i < L) v[i] = run;
    }
    __syncthreads();
    return total;
}

template <int KPL, int CPL, bool ALL>
__global__ void __launch_bounds__(kScanThreads, 2) query_fused_kernel(const __grid_constant__ FusedQueryArgs p) {
    __shared__ ScanShared sm;
    __shared__ int s_warp[kScanWarps];
    const ScanArgs& a = p.a;
    const MarsQueryDesc& d = a.d;
    const float4* q = a.q != nullptr ? a.q : p.qbuf;
    const SlotOne sl{a};
    if (!scan_rows<KPL, CPL, ALL>(a, sl, q, d.t_q, sm)) return;

    int cnt = final_merge<KPL>(a, sl, sm);
    const int K = d.K;
    const int32_t id_off = d.row_offset;
    int total = cnt;

    if (ALL) {
        // ---- BFS from the seeds, all in this CTA ------------------------
        int32_t* vis = sm.stage_i();
        float* vsc = sm.stage_v();
        const int32_t n = *a.s.d_n;
        const uint32_t epoch_base = d.epoch << 4;
        int* s_e0 = reinterpret_cast<int*>(sm.buf);    // per-level node info
        int* s_dc = s_e0 + kLevelCap;                  // CSR degree
        int* s_off = s_dc + kLevelCap;                 // inclusive edge prefix
        uint32_t* s_word = reinterpret_cast<uint32_t*>(s_off + kLevelCap);
        const unsigned long long st0 = (unsigned long long)(epoch_base | 15u) << 32;
        for (int i = threadIdx.x; i < cnt; i += kScanThreads) {
            const unsigned long long k = sm.keys()[i];
            vis[i] = key_id(k) - id_off;
            vsc[i] = key_score(k);
        }
        __syncthreads();   // the key buffer is reused for the level arrays
        for (int i = threadIdx.x; i < cnt; i += kScanThreads) atomicMax(a.stamp + vis[i], st0 | f2key(vsc[i]));
        if (threadIdx.x == 0) { sm.misc[0] = cnt; sm.misc[1] = 0; }
        int lv_beg = 0, lv_end = cnt;
        for (int h = 0; h < d.hops && lv_end > lv_beg; ++h) {
            const int L = lv_end - lv_beg;
            if (L > kLevelCap) { if (threadIdx.x == 0) sm.misc[1] = 1; break; }
            const unsigned long long next_stamp =
                (unsigned long long)(epoch_base | (uint32_t)(15 - (h + 1))) << 32;
            for (int t = threadIdx.x; t < L; t += kScanThreads) {
                const int32_t u = vis[lv_beg + t];
                int e0 = 0, dc = 0, de = 0;
                if (a.s.row_offsets != nullptr && u < a.s.csr_n) {
                    e0 = __ldg(a.s.row_offsets + u);
                    dc = __ldg(a.s.row_offsets + u + 1) - e0;
                }
                if (a.s.extra != nullptr && a.s.slack > 0) de = min(__ldcg(a.s.extra_cnt + u), a.s.slack);
                s_e0[t] = e0;
                s_dc[t] = dc;
                s_off[t] = dc + de;
                s_word[t] = f2key(vsc[lv_beg + t] * d.hop_decay);
            }
            __syncthreads();
            const int n_edges = block_inclusive_scan<kScanThreads>(s_off, L, s_warp);
            // every edge of the level: claim its head for level h + 1
            constexpr int kEB = 4;
            for (int e_base = 0; e_base < n_edges; e_base += kScanThreads * kEB) {
                int32_t vv[kEB];
                int tt[kEB];
#pragma unroll
                for (int b = 0; b < kEB; ++b) {
                    const int e = e_base + b * kScanThreads + threadIdx.x;
                    vv[b] = -1;
                    tt[b] = 0;
                    if (e < n_edges) {
                        int lo = 0, hi = L - 1;   // first t with s_off[t] > e
                        while (lo < hi) {
                            const int mid = (lo + hi) >> 1;
                            if (s_off[mid] > e) hi = mid; else lo = mid + 1;
                        }
                        const int k = e - (lo > 0 ? s_off[lo - 1] : 0);
                        tt[b] = lo;
                        if (k < s_dc[lo]) {
                            vv[b] = __ldg(a.s.col_indices + s_e0[lo] + k);
                        } else {
                            const int32_t u = vis[lv_beg + lo];
                            vv[b] = __ldcg(a.s.extra + (int64_t)u * a.s.slack + (k - s_dc[lo]));
                        }
                    }
                }
#pragma unroll
                for (int b = 0; b < kEB; ++b) {
                    const int32_t v = vv[b];
                    if (v >= 0 && v < n) {
                        const unsigned long long old = atomicMax(a.stamp + v, next_stamp | s_word[tt[b]]);
                        if ((uint32_t)(old >> 32) < epoch_base) {
                            const int pos = atomicAdd(&sm.misc[0], 1);
                            if (pos < kTailCap) vis[pos] = v; else sm.misc[1] = 1;
                        }
                    }
                }
            }
            __syncthreads();
            if (sm.misc[1] != 0) break;
            const int new_end = sm.misc[0];
            // scores of the new level: best parent (low word of the stamp)
            // against 0.8 x the node's own fused score
            for (int i = lv_end + threadIdx.x; i < new_end; i += kScanThreads) {
                const int32_t v = vis[i];
                const float bp = key2f((uint32_t)(__ldcg(a.stamp + v) & 0xffffffffull));
                vsc[i] = fmaxf(bp, __ldcg(a.all_scores + v) * 0.8f);
            }
            __syncthreads();
            lv_beg = lv_end;
            lv_end = new_end;
        }
        __syncthreads();
        if (sm.misc[1] != 0) {
            if (threadIdx.x == 0) {
                rearm(sl);
                p.out_cnt[1] = 0;
                store_release_sys(p.out_cnt, -1);
            }
            return;
        }
        total = lv_end;

        // ---- rank the visited set by (score desc, node id asc) -----------
        // (the candidate keys overwrite the visited arrays: read them first)
        constexpr int kPer = kTailCap / kScanThreads;
        unsigned long long k_own[kPer];
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
            const int i = u * kScanThreads + threadIdx.x;
            k_own[u] = i < total ? rank_key(vsc[i], vis[i]) : 0ull;
        }
        __syncthreads();
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
            const int i = u * kScanThreads + threadIdx.x;
            if (i < total) sm.keys()[i] = k_own[u];
        }
        __syncthreads();
        cnt = block_select_topk<kScanThreads>(sm.keys(), total, K, sm.hist(), sm.misc);
    }

    // ---- results ------------------------------------------------------------
    mars_query_result* out = reinterpret_cast<mars_query_result*>(p.out);
    for (int i = threadIdx.x; i < cnt; i += kScanThreads) {
        const unsigned long long k = sm.keys()[i];
        const int32_t id = key_id(k);
        const int32_t u = ALL ? id : id - id_off;   // local row
        mars_query_result r;
        r.node_id = u + id_off;
        r.score = key_score(k);
        r.modality = __ldg(a.s.mod + u);
        r.hops_from_seed = ALL ? 15 - (int)((uint32_t)(__ldcg(a.stamp + u) >> 32) & 15u) : 0;
        out[i] = r;
    }
    // the count is written last, by a system-scope release store: a host
    // that polls it sees every result (and the visited count) once it changes
    __syncthreads();
    if (threadIdx.x == 0) {
        rearm(sl);
        p.out_cnt[1] = total;
        store_release_sys(p.out_cnt, cnt);
    }
}

template <int KPL, bool ALL>
static cudaError_t launch_fused_kpl(const FusedQueryArgs& p, int grid, cudaStream_t st) {
    switch ((p.a.s.nc + 31) / 32) {
    case 1: query_fused_kernel<KPL, 1, ALL><<<grid, kScanThreads, 0, st>>>(p); break;
    case 2: query_fused_kernel<KPL, 2, ALL><<<grid, kScanThreads, 0, st>>>(p); break;
    case 3: query_fused_kernel<KPL, 3, ALL><<<grid, kScanThreads, 0, st>>>(p); break;
    case 4: query_fused_kernel<KPL, 4, ALL><<<grid, kScanThreads, 0, st>>>(p); break;
    case 5: query_fused_kernel<KPL, 5, ALL><<<grid, kScanThreads, 0, st>>>(p); break;
    case 6: query_fused_kernel<KPL, 6, ALL><<<grid, kScanThreads, 0, st>>>(p); break;
    case 7: query_fused_kernel<KPL, 7, ALL><<<grid, kScanThreads, 0, st>>>(p); break;
    case 8: query_fused_kernel<KPL, 8, ALL><<<grid, kScanThreads, 0, st>>>(p); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_query_fused(const FusedQueryArgs& p, int grid, cudaStream_t st) {
    const bool bfs = p.a.d.hops > 0;
    if (p.a.d.K <= 32) return bfs ? launch_fused_kpl<1, true>(p, grid, st) : launch_fused_kpl<1, false>(p, grid, st);
    if (p.a.d.K <= 64) return bfs ? launch_fused_kpl<2, true>(p, grid, st) : launch_fused_kpl<2, false>(p, grid, st);
    return cudaErrorInvalidValue;
}

}  // namespace mars
