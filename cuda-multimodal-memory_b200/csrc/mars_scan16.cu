// mars_scan16.cu -- the fused scan top-K with an fp16 filter pass: exact
// results from half the bytes.
//
// The store keeps an fp16 copy of its rows (mars_store.cu, store_f16_rows).
// A query streams that copy instead of the fp32 rows.  fp16 keeps 10
// mantissa bits, so the approximate dot product a of a row is within a
// proven margin m of the canonical fp32 dot product d:
//   |a - d| <= 6e-4 |q| max|e| + 2^-24 sqrt(D) |q|
// The row's rounding to fp16 moves the dot product by at most
// 2^-11 sum|q_i e_i| + 2^-25 sum|q_i| (2^-11 relative error in the normal
// range, 2^-25 absolute below it), i.e. 4.9e-4 |q||e| + 2^-25 sqrt(D) |q| by
// Cauchy-Schwarz; each fp32 sum (at most 32 fused multiply-adds per lane and
// 5 butterfly steps for D <= 1024) adds at most 37 * 2^-24 |q||e| = 2.2e-6
// |q||e|.  |q| and max|e| are rounded up by 1e-4 relative.  The fused score is monotone in the dot product (a positive
// decay weight, then the importance), so applying it to a + m and a - m
// brackets the exact score f: L <= f <= U.
//
//  * every warp keeps the K best lower bounds L of its rows and sets aside
//    each row whose U reaches its running K-th lower bound (that bound never
//    exceeds the final one, so no row of the answer is dropped);
//  * per CTA, the set-aside rows are filtered again against the CTA's K-th
//    lower bound and written to a per-query candidate list;
//  * the last CTA takes the global K-th lower bound theta (the K rows with the
//    best lower bounds all score at least theta, so the K-th exact score is
//    >= theta), keeps the candidates with U >= theta, scores them exactly with
//    the canonical fp32 dot product of the scan kernel and selects the top-K.
//
// The results are therefore those of scan_topk_kernel bit for bit.  A query
// whose candidate list overflows is reported and re-run by the host with the
// fp32 scan.
#include <cuda_fp16.h>

#include "mars_scan_body.cuh"

namespace mars {

// Set-aside rows buffered per warp before the CTA filter.  The buffers sit in
// the part of the scan's shared buffer that only the last CTA's merge uses.
constexpr int kWarpCand = 256;
static_assert(2048 + kScanWarps * kWarpCand <= kMergeKeys, "warp buffers must fit below the histogram");

struct Scan16Args {
    ScanArgs a;                       // store view, descriptor, partial lists, ticket, outputs
    const float* Q;                   // nq x qpitch fp32 queries
    int64_t qpitch;
    const __half* E16;                // fp16 rows, pitch16 halves each
    int64_t pitch16;
    int32_t nc16;                     // 16-byte chunks holding the D values
    const unsigned int* norm_bits;    // largest row norm (float bits)
    unsigned long long* cand;         // [nq][cand_cap]: (f2key(U) << 32) | row
    int32_t* cand_cnt;                // [nq]
    int32_t cand_cap;
    int32_t* overflow;                // [nq]: 1 = the candidate list overflowed
    int32_t* stats;                   // [nq][2]: candidates, survivors of the last CTA's filter
    int32_t* out_mod;                 // [nq][K] modality of each result (may be null)
};

__device__ __forceinline__ uint4 ldg_stream_u4(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

// Sum of the 8 halves of c times the 8 floats of (qa, qb), in order.
__device__ __forceinline__ float fma8(const uint4 c, const float4 qa, const float4 qb, float acc) {
    const float2 e0 = __half22float2(*reinterpret_cast<const __half2*>(&c.x));
    const float2 e1 = __half22float2(*reinterpret_cast<const __half2*>(&c.y));
    const float2 e2 = __half22float2(*reinterpret_cast<const __half2*>(&c.z));
    const float2 e3 = __half22float2(*reinterpret_cast<const __half2*>(&c.w));
    acc = fmaf(e0.x, qa.x, acc);
    acc = fmaf(e0.y, qa.y, acc);
    acc = fmaf(e1.x, qa.z, acc);
    acc = fmaf(e1.y, qa.w, acc);
    acc = fmaf(e2.x, qb.x, acc);
    acc = fmaf(e2.y, qb.y, acc);
    acc = fmaf(e3.x, qb.z, acc);
    acc = fmaf(e3.y, qb.w, acc);
    return acc;
}

__device__ __forceinline__ unsigned long long cand_key(float u, int32_t row) {
    return ((unsigned long long)f2key(u) << 32) | (uint32_t)row;
}

template <int KPL, int CPL16>
__global__ void __launch_bounds__(kScanThreads, 2) scan16_kernel(const __grid_constant__ Scan16Args p) {
    __shared__ ScanShared sm;
    __shared__ float s_theta;
    const ScanArgs& a = p.a;
    const MarsQueryDesc& d = a.d;
    const int qi = blockIdx.y;
    const SlotMulti sl{a, qi};
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const float t_q = d.t_q, lambda = d.lambda;
    const int32_t filter = d.filter;
    const bool use_imp = d.use_imp != 0 && a.s.imp != nullptr;
    const int K = d.K;
    const int32_t id_off = d.row_offset;
    const int32_t n = *a.s.d_n;
    const int nc = a.s.nc, nc16 = p.nc16;
    const float4* q4 = reinterpret_cast<const float4*>(p.Q + qi * p.qpitch);
    unsigned long long* cand = p.cand + (int64_t)qi * p.cand_cap;
    int32_t* cand_cnt = p.cand_cnt + qi;

    // query in registers: chunk c16 = lane + 32 j covers values 8 c16 .. 8 c16 + 7
    float4 qa[CPL16], qb[CPL16];
    float qss = 0.f;
#pragma unroll
    for (int j = 0; j < CPL16; ++j) {
        const int c16 = lane + 32 * j;
        qa[j] = (c16 < nc16 && 2 * c16 < nc) ? q4[2 * c16] : make_float4(0.f, 0.f, 0.f, 0.f);
        qb[j] = (c16 < nc16 && 2 * c16 + 1 < nc) ? q4[2 * c16 + 1] : make_float4(0.f, 0.f, 0.f, 0.f);
        qss += qa[j].x * qa[j].x + qa[j].y * qa[j].y + qa[j].z * qa[j].z + qa[j].w * qa[j].w;
        qss += qb[j].x * qb[j].x + qb[j].y * qb[j].y + qb[j].z * qb[j].z + qb[j].w * qb[j].w;
    }
    const float qn = sqrtf(warp_butterfly_sum(qss)) * 1.0001f;
    const float emax = __uint_as_float(__ldg(p.norm_bits));
    const float mg = 6.0e-4f * qn * emax + 5.9604645e-8f * sqrtf(8.0f * nc16) * qn * 1.0001f;
    // a query too large for the bound to be computed: every row is a candidate
    // (the list overflows and the host answers with the fp32 scan)
    const bool wide = !(qn * emax <= 1e37f);

    WarpTopK<KPL> top;
    top.init(K);
    unsigned long long* wc = sm.buf + 2048 + warp * kWarpCand;   // this warp's set-aside rows
    int wn = 0;                                                  // warp-uniform count

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

    auto append_global = [&](bool take, unsigned long long key) {
        const unsigned m = __ballot_sync(MARS_FULL_MASK, take);
        if (m == 0) return;
        int base = 0;
        if (lane == __ffs(m) - 1) base = atomicAdd(cand_cnt, __popc(m));
        base = __shfl_sync(MARS_FULL_MASK, base, __ffs(m) - 1);
        const int pos = base + __popc(m & ((1u << lane) - 1u));
        if (take && pos < p.cand_cap) cand[pos] = key;
    };

    // drop the set-aside rows whose upper bound fell below the warp's threshold
    auto compact = [&]() {
        __syncwarp();
        const float th = top.thr_v;
        int out = 0;
        for (int i0 = 0; i0 < wn; i0 += 32) {
            const int i = i0 + lane;
            const unsigned long long k = i < wn ? wc[i] : 0ull;
            const bool keep = i < wn && key2f((uint32_t)(k >> 32)) >= th;
            const unsigned m = __ballot_sync(MARS_FULL_MASK, keep);
            if (keep) wc[out + __popc(m & ((1u << lane) - 1u))] = k;   // never past what this chunk read
            out += __popc(m);
        }
        wn = out;
        __syncwarp();
    };

    // R rows per step.  Their approximate dot products are reduced with a
    // transposed butterfly (the order of the fp32 sum does not matter here:
    // the margin bounds any order of depth <= 37), after which lanes
    // (32 / R) i .. (32 / R) (i + 1) - 1 hold row i's sum and bound it.
    constexpr int R = CPL16 <= 3 ? 4 : 2;
    constexpr int kGroup = 32 / R;
    constexpr unsigned kLeaders = R == 4 ? 0x01010101u : 0x00010001u;
    const int grp = lane / kGroup;
    const char* E16b = reinterpret_cast<const char*>(p.E16);
    const int64_t rowb = p.pitch16 * 2;
    for (int32_t r = r0; r < r1; r += R) {
        if (r + R - wbase > 32) { wbase = r; load_meta(wbase); }
        uint4 e[R][CPL16];
#pragma unroll
        for (int i = 0; i < R; ++i) {
            const char* pi = E16b + (int64_t)(r + i) * rowb;
#pragma unroll
            for (int j = 0; j < CPL16; ++j) {
                const int c16 = lane + 32 * j;
                e[i][j] = (c16 < nc16 && r + i < r1) ? ldg_stream_u4(pi + 16 * c16) : make_uint4(0u, 0u, 0u, 0u);
            }
        }
        float acc[R];
#pragma unroll
        for (int i = 0; i < R; ++i) {
            acc[i] = 0.f;
#pragma unroll
            for (int j = 0; j < CPL16; ++j)
                if (lane + 32 * j < nc16) acc[i] = fma8(e[i][j], qa[j], qb[j], acc[i]);
        }
        float t;
        if constexpr (R == 4) {
            const bool h16 = (lane & 16) != 0, h8 = (lane & 8) != 0;
            const float s0 = (h16 ? acc[2] : acc[0]) + __shfl_xor_sync(MARS_FULL_MASK, h16 ? acc[0] : acc[2], 16);
            const float s1 = (h16 ? acc[3] : acc[1]) + __shfl_xor_sync(MARS_FULL_MASK, h16 ? acc[1] : acc[3], 16);
            t = (h8 ? s1 : s0) + __shfl_xor_sync(MARS_FULL_MASK, h8 ? s0 : s1, 8);
        } else {
            const bool h16 = (lane & 16) != 0;
            t = (h16 ? acc[1] : acc[0]) + __shfl_xor_sync(MARS_FULL_MASK, h16 ? acc[0] : acc[1], 16);
            t += __shfl_xor_sync(MARS_FULL_MASK, t, 8);
        }
        t += __shfl_xor_sync(MARS_FULL_MASK, t, 4);
        t += __shfl_xor_sync(MARS_FULL_MASK, t, 2);
        t += __shfl_xor_sync(MARS_FULL_MASK, t, 1);

        // every lane bounds its group's row
        const int32_t row = r + grp;
        const int src = row - wbase;   // < 32
        const float ts = __shfl_sync(MARS_FULL_MASK, ts_w, src);
        const float im = __shfl_sync(MARS_FULL_MASK, imp_w, src);
        const int32_t m = __shfl_sync(MARS_FULL_MASK, mod_w, src);
        const bool valid = row < r1 && !(filter >= 0 && m != filter) && row + 1 != d.exclude_plus1;
        // fl(x * w) and fl(x * im) are monotone in x, so with a - mg <= dot <= a + mg
        // the scan's score of the row lies in [lo, hi]
        const float wgt = fused_weight(ts, t_q, lambda);
        float hi = (t + mg) * wgt;
        float lo = (t - mg) * wgt;
        if (use_imp) {
            hi = hi * im;
            lo = lo * im;
            if (im < 0.f) { const float x = hi; hi = lo; lo = x; }
        }
        if (wide) { hi = INFINITY; lo = -INFINITY; }
        // rows whose upper bound is below the running K-th lower bound can
        // neither enter the list nor place (the bound only rises)
        unsigned live = __ballot_sync(MARS_FULL_MASK, valid && hi >= top.thr_v) & kLeaders;
        while (live != 0u) {   // warp-uniform, in row order
            const int b = __ffs(live) - 1;
            live &= live - 1u;
            const float lo_b = __shfl_sync(MARS_FULL_MASK, lo, b);
            const float hi_b = __shfl_sync(MARS_FULL_MASK, hi, b);
            const int32_t row_b = r + b / kGroup;
            top.push(lo_b, row_b + id_off, lane);
            if (hi_b >= top.thr_v) {   // can still place: set aside
                if (wn == kWarpCand) compact();
                if (wn < kWarpCand) {
                    if (lane == 0) wc[wn] = cand_key(hi_b, row_b);
                    ++wn;
                } else {
                    append_global(lane == 0, cand_key(hi_b, row_b));
                }
            }
        }
    }

    // ---- CTA: merge the warps' lower bounds, filter the set-aside rows -------
    top.store(sm.warp_val(warp), sm.warp_idx(warp), lane);
    __syncthreads();
    if (warp == 0) {
        if constexpr (KPL == 1) {
            for (int ww = 1; ww < kScanWarps; ++ww) top.merge_sorted32(sm.warp_val(ww), sm.warp_idx(ww), K, lane);
        } else {
            for (int ww = 1; ww < kScanWarps; ++ww) top.offer_sorted(sm.warp_val(ww), sm.warp_idx(ww), K, lane);
        }
        top.store(sl.part_val() + (int64_t)blockIdx.x * K, sl.part_idx() + (int64_t)blockIdx.x * K, lane);
        if (lane == 0) s_theta = top.thr_v;   // the CTA's K-th lower bound (-inf with fewer than K rows)
    }
    __syncthreads();
    {
        const float th = s_theta;
        for (int i0 = 0; i0 < wn; i0 += 32) {
            const int i = i0 + lane;
            const unsigned long long k = i < wn ? wc[i] : 0ull;
            append_global(i < wn && key2f((uint32_t)(k >> 32)) >= th, k);
        }
    }
    __threadfence();
    __syncthreads();
    if (warp == 0) {
        __syncwarp();
        if (lane == 0) sm.last = atomicAdd(sl.ticket(), 1u) == gridDim.x - 1;
        __syncwarp();
    }
    __syncthreads();
    if (!sm.last) return;
    __threadfence();

    // ---- last CTA: global K-th lower bound, exact scores of what can place ----
    const int cnt_lb = final_merge<KPL>(a, sl, sm);
    const float theta = cnt_lb >= K ? key_score(sm.keys()[K - 1]) : -INFINITY;
    const int nc_all = __ldcg(cand_cnt);
    if (threadIdx.x == 0) p.stats[2 * qi] = nc_all;
    int* s_n = sm.misc + 14;
    if (threadIdx.x == 0) *s_n = 0;
    __syncthreads();
    if (nc_all > p.cand_cap) {
        if (threadIdx.x == 0) {
            p.stats[2 * qi + 1] = -1;
            p.overflow[qi] = 1;
            *cand_cnt = 0;
            rearm(sl);
        }
        return;
    }
    // survivors (row ids) into the key buffer's second half
    int32_t* surv = reinterpret_cast<int32_t*>(sm.keys() + 2048);
    constexpr int kSurvCap = 2048;
    for (int i0 = 0; i0 < nc_all; i0 += kScanThreads) {
        const int i = i0 + threadIdx.x;
        const unsigned long long k = i < nc_all ? __ldcg(cand + i) : 0ull;
        const bool take = i < nc_all && key2f((uint32_t)(k >> 32)) >= theta;
        const unsigned m = __ballot_sync(MARS_FULL_MASK, take);
        int base = 0;
        if (m != 0 && lane == __ffs(m) - 1) base = atomicAdd(s_n, __popc(m));
        base = __shfl_sync(MARS_FULL_MASK, base, m != 0 ? __ffs(m) - 1 : 0);
        const int pos = base + __popc(m & ((1u << lane) - 1u));
        if (take && pos < kSurvCap) surv[pos] = (int32_t)(uint32_t)(k & 0xffffffffull);
    }
    __syncthreads();
    const int ns = *s_n;
    if (threadIdx.x == 0) p.stats[2 * qi + 1] = ns;
    if (ns > kSurvCap) {
        if (threadIdx.x == 0) {
            p.overflow[qi] = 1;
            *cand_cnt = 0;
            rearm(sl);
        }
        return;
    }
    // exact canonical scores (the scan kernel's arithmetic), one row per warp
    unsigned long long* keys = sm.keys();   // [0, 2048): exact keys
    const float4* E4 = reinterpret_cast<const float4*>(a.s.E);
    for (int i = warp; i < ns; i += kScanWarps) {
        const int32_t row = surv[i];
        const float dot = warp_dot_canonical(E4 + (int64_t)row * a.s.pitch4, q4, nc, lane);
        float f = fused_weight_apply(dot, __ldg(a.s.ts + row), t_q, lambda);
        if (use_imp) f = f * __ldg(a.s.imp + row);
        if (lane == 0) keys[i] = rank_key(f, row + id_off);
    }
    __syncthreads();
    const int cnt = block_select_topk<kScanThreads>(keys, ns, K, sm.hist(), sm.misc);
    for (int pp = threadIdx.x; pp < K; pp += kScanThreads) {
        const bool valid = pp < cnt;
        a.out_val[(int64_t)qi * K + pp] = valid ? key_score(keys[pp]) : -INFINITY;
        a.out_idx[(int64_t)qi * K + pp] = valid ? key_id(keys[pp]) : -1;
        if (p.out_mod != nullptr)
            p.out_mod[(int64_t)qi * K + pp] = valid ? __ldg(a.s.mod + (key_id(keys[pp]) - id_off)) : -1;
    }
    if (threadIdx.x == 0) {
        if (a.out_cnt != nullptr) a.out_cnt[qi] = cnt;
        p.overflow[qi] = 0;
        *cand_cnt = 0;
        rearm(sl);
    }
}

template <int KPL>
static cudaError_t launch16_kpl(const Scan16Args& p, int grid, int nq, cudaStream_t st) {
    switch ((p.nc16 + 31) / 32) {
    case 1: scan16_kernel<KPL, 1><<<dim3(grid, nq), kScanThreads, 0, st>>>(p); break;
    case 2: scan16_kernel<KPL, 2><<<dim3(grid, nq), kScanThreads, 0, st>>>(p); break;
    case 3: scan16_kernel<KPL, 3><<<dim3(grid, nq), kScanThreads, 0, st>>>(p); break;
    case 4: scan16_kernel<KPL, 4><<<dim3(grid, nq), kScanThreads, 0, st>>>(p); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_scan16(const Scan16Args& p, int grid, int nq, cudaStream_t st) {
    const int K = p.a.d.K;
    if (K <= 32) return launch16_kpl<1>(p, grid, nq, st);
    if (K <= 64) return launch16_kpl<2>(p, grid, nq, st);
    return cudaErrorInvalidValue;
}

}  // namespace mars

// ---------------------------------------------------------------------------
// Host entry point.
#include <algorithm>
#include <cstring>
#include <string>

#include "mars_b200.h"
#include "mars_internal.h"

using namespace mars;

extern "C" int mars_scan_topk_f16(const mars_store* s, mars_query_ctx* c, const float* d_queries,
                                  int32_t query_pitch, int32_t nq, float t_q, float lambda,
                                  int32_t modality_filter, int32_t use_importance, int32_t K,
                                  int32_t row_offset, int32_t* d_ids, float* d_vals, int32_t* d_counts,
                                  void* stream) {
    if (s == nullptr || c == nullptr || d_queries == nullptr || d_ids == nullptr || d_vals == nullptr || nq < 0)
        return fail(MARS_ERR_INVALID, "mars_scan_topk_f16: NULL argument or nq < 0");
    if (K <= 0 || K > 64 || s->dim > 1024 || (s->dim & 3) != 0 ||
        (reinterpret_cast<uintptr_t>(d_queries) & 15u) != 0 || query_pitch < s->pitch || (query_pitch & 3) != 0)
        return mars_scan_topk_multi(s, c, d_queries, query_pitch, nq, t_q, lambda, modality_filter,
                                    use_importance, K, row_offset, d_ids, d_vals, d_counts, stream);
    if (nq == 0) return MARS_OK;
    if (s->device != c->device || s->dim != c->dim || s->n > c->max_nodes || K > c->max_k)
        return fail(MARS_ERR_INVALID, "mars_scan_topk_f16: store, context or K do not match");
    MarsDeviceGuard g(c->device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    MARS_CUDA_TRY(cudaStreamWaitEvent(st, s->written, 0));
    bool ok = false;
    MARS_TRY(store_f16_rows(s, st, &ok));
    if (!ok)   // values beyond the fp16 range: the fp32 scan
        return mars_scan_topk_multi(s, c, d_queries, query_pitch, nq, t_q, lambda, modality_filter,
                                    use_importance, K, row_offset, d_ids, d_vals, d_counts, stream);
    MARS_TRY(query_ctx_f16_buffers(c));
    c->f16_max_cand = 0;
    c->f16_max_surv = 0;
    Scan16Args p{};
    ScanArgs& a = p.a;
    a.s.E = s->d_E;
    a.s.ts = s->d_ts;
    a.s.imp = s->d_imp;
    a.s.mod = s->d_mod;
    a.s.d_n = s->d_n;
    a.s.pitch4 = s->pitch / 4;
    a.s.nc = (s->dim + 3) / 4;
    a.d.t_q = t_q;
    a.d.lambda = lambda;
    a.d.filter = modality_filter;
    a.d.use_imp = use_importance;
    a.d.K = K;
    a.d.row_offset = row_offset;
    a.part_val = c->d_part_val;
    a.part_idx = c->d_part_idx;
    a.ticket = c->d_f16_ticket;
    a.cursor = nullptr;
    p.qpitch = query_pitch;
    p.E16 = static_cast<const __half*>(s->d_E16);
    p.pitch16 = s->e16_pitch;
    p.nc16 = (s->dim + 7) / 8;
    p.norm_bits = s->d_norm_bits;
    p.cand = c->d_f16_cand;
    p.cand_cnt = c->d_f16_cnt;
    p.cand_cap = kF16CandCap;
    p.overflow = c->d_f16_overflow;
    p.stats = c->d_f16_overflow + kF16Slots;
    const int32_t per = std::max(1, std::min(kF16Slots, (int)MARS_MAX_TOP_K / K));   // partial lists fit
    for (int32_t q0 = 0; q0 < nq; q0 += per) {
        const int32_t n = std::min(per, nq - q0);
        p.Q = d_queries + (size_t)q0 * query_pitch;
        a.out_val = d_vals + (size_t)q0 * K;
        a.out_idx = d_ids + (size_t)q0 * K;
        a.out_cnt = d_counts ? d_counts + q0 : nullptr;
        // one wave (two CTAs per SM) for the whole launch: the queries walk
        // the same rows in step and share them through L2, and each warp's
        // longer row range lets its threshold settle (fewer candidates)
        const int gx = std::max(1, std::min(c->scan_blocks, 2 * c->num_sms / n));
        MARS_CUDA_TRY(launch_scan16(p, gx, n, st));
        MARS_CUDA_TRY(cudaMemcpyAsync(c->h_f16_overflow, c->d_f16_overflow, 3 * kF16Slots * sizeof(int32_t),
                                      cudaMemcpyDeviceToHost, st));
        MARS_CUDA_TRY(cudaStreamSynchronize(st));
        for (int32_t i = 0; i < n; ++i) {
            const int32_t* stats = c->h_f16_overflow + kF16Slots;
            c->f16_max_cand = std::max(c->f16_max_cand, stats[2 * i]);
            c->f16_max_surv = std::max(c->f16_max_surv, stats[2 * i + 1]);
            if (c->h_f16_overflow[i] == 0) continue;
            // more candidates than the list holds: this query on the fp32 scan
            MARS_TRY(mars_scan_topk(s, c, d_queries + (size_t)(q0 + i) * query_pitch, t_q, lambda,
                                    modality_filter, use_importance, K, row_offset,
                                    d_ids + (size_t)(q0 + i) * K, d_vals + (size_t)(q0 + i) * K,
                                    d_counts ? d_counts + q0 + i : nullptr, st));
            ++c->f16_reruns;
        }
    }
    return MARS_OK;
}

extern "C" int mars_query_ctx_f16_stats(const mars_query_ctx* c, uint64_t* reruns, int32_t* max_candidates,
                                        int32_t* max_survivors) {
    if (c == nullptr) return fail(MARS_ERR_INVALID, "mars_query_ctx_f16_stats: NULL context");
    if (reruns != nullptr) *reruns = c->f16_reruns;
    if (max_candidates != nullptr) *max_candidates = c->f16_max_cand;
    if (max_survivors != nullptr) *max_survivors = c->f16_max_surv;
    return MARS_OK;
}

int mars::query_f16(const mars_store* s, mars_query_ctx* c, const float* query, float t_q,
                    const mars_retrieval_config* cfg, mars_query_result* out, int32_t* n_out,
                    mars_retrieval_stats* stats, int* done) {
    *done = 0;
    cudaStream_t st = c->stream;
    bool ok = false;
    MARS_TRY(store_f16_rows(s, st, &ok));
    if (!ok) return MARS_OK;   // values beyond the fp16 range
    MARS_TRY(query_ctx_f16_buffers(c));
    const int K = cfg->top_k;
    // the query on the device: in place when aligned, else through the
    // context's descriptor buffer
    const float* dq = nullptr;
    cudaPointerAttributes pa{};
    const bool on_device = cudaPointerGetAttributes(&pa, query) == cudaSuccess && pa.type == cudaMemoryTypeDevice;
    (void)cudaGetLastError();
    float* d_slot = reinterpret_cast<float*>(static_cast<char*>(c->d_desc) + kDescQueryOffset);
    if (on_device && (reinterpret_cast<uintptr_t>(query) & 15u) == 0) {
        dq = query;
    } else if (on_device) {
        MARS_CUDA_TRY(cudaMemcpyAsync(d_slot, query, (size_t)s->dim * sizeof(float), cudaMemcpyDeviceToDevice, st));
        dq = d_slot;
    } else {
        float* h_slot = reinterpret_cast<float*>(static_cast<char*>(c->h_desc) + kDescQueryOffset);
        std::memcpy(h_slot, query, (size_t)s->dim * sizeof(float));
        MARS_CUDA_TRY(cudaMemcpyAsync(d_slot, h_slot, (size_t)s->dim * sizeof(float), cudaMemcpyHostToDevice, st));
        dq = d_slot;
    }
    Scan16Args p{};
    ScanArgs& a = p.a;
    a.s.E = s->d_E;
    a.s.ts = s->d_ts;
    a.s.imp = s->d_imp;
    a.s.mod = s->d_mod;
    a.s.d_n = s->d_n;
    a.s.pitch4 = s->pitch / 4;
    a.s.nc = (s->dim + 3) / 4;
    a.d.t_q = t_q;
    a.d.lambda = cfg->time_decay_lambda;
    a.d.filter = cfg->modality_filter;
    a.d.use_imp = cfg->use_importance;
    a.d.K = K;
    a.part_val = c->d_part_val;
    a.part_idx = c->d_part_idx;
    a.ticket = c->d_f16_ticket;
    int32_t* qo = c->d_f16_qout;
    a.out_cnt = qo + 1;
    a.out_idx = qo + 4;
    a.out_val = reinterpret_cast<float*>(qo + 4 + K);
    p.out_mod = qo + 4 + 2 * K;
    p.Q = dq;
    p.qpitch = s->dim;
    p.E16 = static_cast<const __half*>(s->d_E16);
    p.pitch16 = s->e16_pitch;
    p.nc16 = (s->dim + 7) / 8;
    p.norm_bits = s->d_norm_bits;
    p.cand = c->d_f16_cand;
    p.cand_cnt = c->d_f16_cnt;
    p.cand_cap = kF16CandCap;
    p.overflow = qo;
    p.stats = c->d_f16_overflow + kF16Slots;
    if (stats) MARS_CUDA_TRY(cudaEventRecord(c->ev[0], st));
    MARS_CUDA_TRY(launch_scan16(p, std::min(c->scan_blocks, 2 * c->num_sms), 1, st));
    if (stats) MARS_CUDA_TRY(cudaEventRecord(c->ev[2], st));
    MARS_CUDA_TRY(cudaMemcpyAsync(c->h_f16_qout, qo, (4 + 3 * (size_t)K) * sizeof(int32_t), cudaMemcpyDeviceToHost,
                                  st));
    MARS_CUDA_TRY(cudaStreamSynchronize(st));
    const int32_t* h = c->h_f16_qout;
    if (h[0] != 0) {   // the candidate list overflowed
        ++c->f16_reruns;
        return MARS_OK;
    }
    const int32_t cnt = std::min(h[1], K);
    for (int32_t i = 0; i < cnt; ++i) {
        out[i].node_id = h[4 + i];
        std::memcpy(&out[i].score, h + 4 + K + i, sizeof(float));
        out[i].modality = h[4 + 2 * K + i];
        out[i].hops_from_seed = 0;
    }
    *n_out = cnt;
    if (stats) {
        float ms = 0.f;
        cudaEventElapsedTime(&ms, c->ev[0], c->ev[2]);
        *stats = mars_retrieval_stats{};
        stats->gpu_ms_similarity = ms;
        stats->gpu_ms_total = ms;
        stats->nodes_scanned = s->n;
        stats->nodes_visited = cnt;
    }
    ++c->fused_queries;
    *done = 1;
    return MARS_OK;
}
