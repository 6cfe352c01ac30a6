// mars_scan_body.cuh -- the streaming part of the fused scan, shared by the
// scan kernel (mars_scan.cu) and the single-launch query kernel
// (mars_fastq.cu).
//
//  * each warp owns a contiguous range of the rows (balanced to +-1 row); for
//    large row counts the last sixteenth is handed out from a counter; rows
//    stream with 128-bit read-only loads, two rows in flight per warp;
//  * the query lives in registers (lane l holds float4 chunks l, l+32, ...);
//  * the row's fused score (src/memory_cuda.cu:292-310 applied to the
//    similarity of :50-93) is formed in registers and offered to a
//    warp-resident ranked list (WarpTopK); almost every row is rejected by a
//    single compare against the list's threshold;
//  * warps merge into a CTA list, CTAs write their list to a partial buffer,
//    and the last CTA to finish (ticket counter, no spinning) merges the
//    partial lists (final_merge).
#pragma once

#include "mars_common.cuh"
#include "mars_kernels.cuh"
#include "mars_select.cuh"

namespace mars {

constexpr int kStageEntries = 3072;   // staged (score, id) pairs of the fallback merge
constexpr int kMergeKeys = 4096;      // 64-bit candidate keys of the last CTA's selection

// Shared memory of the scan kernels, 40 KB, reused phase by phase
// (offsets in 64-bit words):
//   CTA merge      per-warp ranked lists            [0, 2048)
//   last CTA       candidate keys                   [0, 4096)
//                  radix histogram (2048 ints)      [4096, 5120)
//   fallback merge staged lists                     [2048, 5120)
//   query BFS      per-level arrays                 [0, 2048)
//                  visited ids / scores             [2048, 5120)
struct ScanShared {
    unsigned long long buf[5120];
    unsigned long long red[kScanWarps];
    int     misc[16];
    bool    last;

    __device__ unsigned long long* keys() { return buf; }
    __device__ int* hist() { return reinterpret_cast<int*>(buf + kMergeKeys); }
    __device__ float* stage_v() { return reinterpret_cast<float*>(buf + 2048); }
    __device__ int32_t* stage_i() { return reinterpret_cast<int32_t*>(buf + 2048) + kStageEntries; }
    __device__ float*   warp_val(int w) { return reinterpret_cast<float*>(buf) + w * kMaxTopK; }
    __device__ int32_t* warp_idx(int w) {
        return reinterpret_cast<int32_t*>(buf) + kScanWarps * kMaxTopK + w * kMaxTopK;
    }
};
static_assert(2 * kScanWarps * kMaxTopK * 4 <= 2048 * 8, "warp lists must fit their region");
static_assert(2048 * 8 + 2 * kStageEntries * 4 <= 5120 * 8, "staging must fit its region");

// Where one query's per-CTA lists, completion ticket and row counter live.
// The addresses are formed on use from the launch's parameters (and, for the
// multi-query kernel, the query's index), so no pointer stays in a register
// across the row loop.
struct SlotOne {     // one query per launch
    const ScanArgs& a;
    __device__ float* part_val() const { return a.part_val; }
    __device__ int32_t* part_idx() const { return a.part_idx; }
    __device__ unsigned int* ticket() const { return a.ticket; }
    __device__ unsigned int* cursor() const { return a.cursor; }
    __device__ bool excluded(int32_t) const { return false; }
};
struct SlotMulti {   // query qi of a multi-query launch (gridDim.x CTAs per query)
    const ScanArgs& a;
    int qi;
    __device__ int64_t off() const { return (int64_t)qi * gridDim.x * a.d.K; }
    __device__ float* part_val() const { return a.part_val + off(); }
    __device__ int32_t* part_idx() const { return a.part_idx + off(); }
    __device__ unsigned int* ticket() const { return a.ticket + qi; }
    __device__ unsigned int* cursor() const { return a.cursor != nullptr ? a.cursor + qi : nullptr; }
    __device__ bool excluded(int32_t row) const { return a.exclude_base1 != 0 && row == a.exclude_base1 - 1 + qi; }
};

// Stream this CTA's rows and leave the CTA's ranked list in the partial
// buffer.  Returns true in the last CTA to finish (all partial lists and,
// with ALL, all per-row scores are then visible to it).
template <int KPL, int CPL, bool ALL, class Slot>
__device__ __forceinline__ bool scan_rows(const ScanArgs& a, const Slot& sl, const float4* __restrict__ q,
                                          float t_q, ScanShared& sm) {
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const MarsQueryDesc& d = a.d;
    const float lambda = d.lambda;
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
        qv[j] = c < nc ? q[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    }

    WarpTopK<KPL> top;
    top.init(K);

    // Rows [0, n_st) are split statically: a balanced contiguous range per
    // warp.  With at least 32 rows per warp, the last sixteenth, [n_st, n),
    // is handed out from a counter in grabs of `grab` rows (even, 2..16,
    // about a quarter of a warp's share of that part), so that warps on
    // faster-served SMs take more of it and the CTAs finish together.  The
    // order in which rows are offered does not change the result: the
    // ranking is total.
    const int64_t W = (int64_t)gridDim.x * kScanWarps;
    int32_t grab = 0, n_dyn = 0;
    if (sl.cursor() != nullptr && (int64_t)n >= 32 * W) {
        const int64_t gq = ((int64_t)(n >> 4) / (W * 4)) & ~1ll;
        grab = (int32_t)(gq < 2 ? 2 : (gq > 16 ? 16 : gq));
        n_dyn = ((n >> 4) / grab) * grab;
    }
    const int32_t n_st = n - n_dyn;
    const int64_t w = (int64_t)blockIdx.x * kScanWarps + warp;
    const int32_t r0 = (int32_t)((int64_t)n_st * w / W);
    const int32_t r1 = (int32_t)((int64_t)n_st * (w + 1) / W);

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

    auto offer = [&](int32_t row, float dot, float t, float im, int32_t m) {
        if ((filter >= 0 && m != filter) || row + 1 == d.exclude_plus1 || sl.excluded(row)) {
            if (ALL && lane == 0) a.all_scores[row] = -FLT_MAX;
            return;
        }
        float f = fused_weight_apply(dot, t, t_q, lambda);
        if (use_imp) f = f * im;
        if (ALL && lane == 0) a.all_scores[row] = f;
        top.push(f, row + id_off, lane);
    };
    auto process = [&](int32_t row, float dot) {
        if (row - wbase >= 32) { wbase += 32; load_meta(wbase); }
        const int src = row - wbase;
        const float t = __shfl_sync(MARS_FULL_MASK, ts_w, src);
        const float im = __shfl_sync(MARS_FULL_MASK, imp_w, src);
        const int32_t m = __shfl_sync(MARS_FULL_MASK, mod_w, src);
        offer(row, dot, t, im, m);
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
    if (n_dyn > 0) {
        // grabs of `grab` rows from the counter, scored two rows at a time;
        // the next grab is requested while the current one is scored
        int32_t g = 0;
        if (lane == 0) g = (int32_t)atomicAdd(sl.cursor(), (unsigned)grab);
        g = __shfl_sync(MARS_FULL_MASK, g, 0);
        while (g < n_dyn) {
            int32_t nxt = 0;
            if (lane == 0) nxt = (int32_t)atomicAdd(sl.cursor(), (unsigned)grab);
            for (int32_t pp = 0; pp < grab; pp += 2) {
                // rr + 1 < n: n_dyn is a multiple of the even grab
                const int32_t rr = n_st + g + pp;
                float tm = 0.f, im = 1.f;
                int32_t mm = 0;
                if (lane < 2) {
                    tm = __ldg(a.s.ts + rr + lane);
                    if (use_imp) im = __ldg(a.s.imp + rr + lane);
                    if (filter >= 0) mm = __ldg(a.s.mod + rr + lane);
                }
                const float4* p0 = E4 + (int64_t)rr * a.s.pitch4;
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
                offer(rr, acc0, __shfl_sync(MARS_FULL_MASK, tm, 0), __shfl_sync(MARS_FULL_MASK, im, 0),
                      __shfl_sync(MARS_FULL_MASK, mm, 0));
                offer(rr + 1, acc1, __shfl_sync(MARS_FULL_MASK, tm, 1), __shfl_sync(MARS_FULL_MASK, im, 1),
                      __shfl_sync(MARS_FULL_MASK, mm, 1));
            }
            g = __shfl_sync(MARS_FULL_MASK, nxt, 0);
        }
    }
    // per-row scores written by every warp are published before the ticket
    if (ALL) __threadfence();

    // ---- CTA merge ---------------------------------------------------------
    top.store(sm.warp_val(warp), sm.warp_idx(warp), lane);
    __syncthreads();
    if (warp == 0) {
        if constexpr (KPL == 1) {
            for (int ww = 1; ww < kScanWarps; ++ww) top.merge_sorted32(sm.warp_val(ww), sm.warp_idx(ww), K, lane);
        } else {
            for (int ww = 1; ww < kScanWarps; ++ww) top.offer_sorted(sm.warp_val(ww), sm.warp_idx(ww), K, lane);
        }
        top.store(sl.part_val() + (int64_t)blockIdx.x * K, sl.part_idx() + (int64_t)blockIdx.x * K, lane);
        __threadfence();
        __syncwarp();
        if (lane == 0) sm.last = atomicAdd(sl.ticket(), 1u) == gridDim.x - 1;
        __syncwarp();
    }
    __syncthreads();
    if (!sm.last) return false;
    __threadfence();
    return true;
}

// In the last CTA, once its reads of the shared counters are done: make the
// ticket and the row counter ready for the next launch.
template <class Slot>
__device__ __forceinline__ void rearm(const Slot& sl) {
    *sl.ticket() = 0u;
    if (sl.cursor() != nullptr) *sl.cursor() = 0u;
}

// In the last CTA: merge the gridDim.x partial lists into the top-K.  On
// return (all threads) sm.keys()[0, cnt) holds it in rank order as
// rank_key() keys; returns cnt.
template <int KPL, class Slot>
__device__ __forceinline__ int final_merge(const ScanArgs& a, const Slot& sl, ScanShared& sm) {
    const int K = a.d.K;
    const int nl = (int)gridDim.x;
    int cnt = merge_ranked_lists<kScanThreads>(sl.part_val(), sl.part_idx(), nl, K, sm.keys(), kMergeKeys, sm.hist(),
                                               sm.misc, sm.red);
    if (cnt >= 0) return cnt;

    // More than kMergeKeys entries tie with or beat the bound (heavily tied
    // scores): merge list by list.  The lists are staged in shared memory
    // with every thread's loads in flight at once, then each warp merges a
    // subset of the staged lists.
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int kPer = kStageEntries / kScanThreads;
    WarpTopK<KPL> top;
    top.init(K);
    const int lists_per_batch = kStageEntries / K;
    for (int b0 = 0; b0 < nl; b0 += lists_per_batch) {
        const int nb = min(lists_per_batch, nl - b0);
        const int ne = nb * K;
        const float* pv = sl.part_val() + (int64_t)b0 * K;
        const int32_t* pi = sl.part_idx() + (int64_t)b0 * K;
        float rv[kPer];
        int32_t ri[kPer];
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
            const int j = threadIdx.x + u * kScanThreads;
            if (j < ne) { rv[u] = __ldcg(pv + j); ri[u] = __ldcg(pi + j); }
        }
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
            const int j = threadIdx.x + u * kScanThreads;
            if (j < ne) { sm.stage_v()[j] = rv[u]; sm.stage_i()[j] = ri[u]; }
        }
        __syncthreads();
        for (int l = warp; l < nb; l += kScanWarps)
            top.offer_sorted(sm.stage_v() + l * K, sm.stage_i() + l * K, K, lane);
        __syncthreads();
    }
    top.store(sm.warp_val(warp), sm.warp_idx(warp), lane);
    __syncthreads();
    if (warp == 0) {
        for (int ww = 1; ww < kScanWarps; ++ww) top.offer_sorted(sm.warp_val(ww), sm.warp_idx(ww), K, lane);
        __syncwarp();
        int c = 0;
#pragma unroll
        for (int sl = 0; sl < KPL; ++sl) {
            const int p = sl * 32 + lane;
            const bool valid = p < K && top.i[sl] != INT32_MAX;
            c += __popc(__ballot_sync(MARS_FULL_MASK, valid));
            if (p < K) sm.keys()[p] = valid ? rank_key(top.v[sl], top.i[sl]) : 0ull;
        }
        if (lane == 0) sm.misc[0] = c;
    }
    __syncthreads();
    cnt = sm.misc[0];
    __syncthreads();
    return cnt;
}

}  // namespace mars
