// mars_common.cuh -- device building blocks shared by the MARS B200 kernels.
//
//  * the canonical warp dot product (the one summation order used by every
//    kernel of the library, restated on the CPU by the test oracle),
//  * order-preserving float <-> uint32 keys for 64-bit atomicMax,
//  * a warp-resident top-K list ranked by (score desc, id asc).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <float.h>

#define MARS_FULL_MASK 0xffffffffu

namespace mars {

constexpr int kWarp = 32;
constexpr int kMaxTopK = 256;

// ---------------------------------------------------------------------------
// Streaming 128-bit load: read-only path, no L1 allocation (each embedding
// row is touched once per query).
__device__ __forceinline__ float4 ldg_stream(const float4* p) {
    float4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
    return v;
}

// Bulk prefetch of `bytes` (a multiple of 16) at a 16-byte aligned global
// address into L2 (cp.async.bulk.prefetch.L2, sm_90+): one instruction asks
// for a whole row, so a warp can request the rows it will gather next while
// it computes on the current one.  Nothing is written and no wait follows.
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// L2 prefetch of the 128-byte lines covering [p, p + bytes) at any
// alignment (prefetch.global.L2, one per line): for short spans such as a
// graph node's neighbour list.
__device__ __forceinline__ void prefetch_l2_span(const void* p, uint32_t bytes) {
    const uintptr_t lo = reinterpret_cast<uintptr_t>(p);
    for (uintptr_t a = lo & ~(uintptr_t)127; a < lo + bytes; a += 128)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(a) : "memory");
}

// ---------------------------------------------------------------------------
// Canonical dot product.  Lane l owns float4 chunks c = l, l+32, ... of the
// row (chunks past nc are skipped), accumulates each chunk with fmaf in
// component order x, y, z, w into one fp32 accumulator, and the 32 lane sums
// are combined by an xor butterfly (offsets 16, 8, 4, 2, 1).  Every lane
// ends with the same value because fp32 addition is commutative.
__device__ __forceinline__ float fma4(const float4 e, const float4 q, float acc) {
    acc = __fmaf_rn(e.x, q.x, acc);
    acc = __fmaf_rn(e.y, q.y, acc);
    acc = __fmaf_rn(e.z, q.z, acc);
    acc = __fmaf_rn(e.w, q.w, acc);
    return acc;
}

__device__ __forceinline__ float warp_butterfly_sum(float v) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(MARS_FULL_MASK, v, off));
    return v;
}

// The canonical dot with the query in shared memory and at most C float4
// chunks per lane (nc <= 32 C): the row's loads are all issued before the
// first fused multiply-add, and the query is read from shared memory as the
// chain runs, so only the row occupies registers.  The same chain and
// butterfly as warp_dot_canonical, bit for bit.
template <int C>
__device__ __forceinline__ float warp_dot_canonical_smemq(const float4* __restrict__ row,
                                                          const float4* __restrict__ q_smem, int nc, int lane) {
    float4 e[C];
#pragma unroll
    for (int k = 0; k < C; ++k) {
        const int c = lane + k * kWarp;
        if (c < nc) e[k] = ldg_stream(row + c);
    }
    float acc = 0.0f;
#pragma unroll
    for (int k = 0; k < C; ++k) {
        const int c = lane + k * kWarp;
        if (c < nc) acc = fma4(e[k], q_smem[c], acc);
    }
    return warp_butterfly_sum(acc);
}

// Row dot with the query held in shared or global memory (generic D).
__device__ __forceinline__ float warp_dot_canonical(const float4* __restrict__ row,
                                                    const float4* __restrict__ q,
                                                    int nc, int lane) {
    // chunk c = lane + 32 k in increasing k, one fused multiply-add chain per
    // lane; the loads of up to 8 chunks are issued before the first FMA so a
    // lone row (a BFS node, a rescored candidate) costs one memory latency,
    // not one per chunk.  The arithmetic is the same as the streaming scan's.
    float acc = 0.0f;
    for (int c0 = lane; c0 < nc; c0 += 8 * kWarp) {
        float4 e[8], qv[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int c = c0 + k * kWarp;
            if (c < nc) { e[k] = ldg_stream(row + c); qv[k] = q[c]; }
        }
#pragma unroll
        for (int k = 0; k < 8; ++k)
            if (c0 + k * kWarp < nc) acc = fma4(e[k], qv[k], acc);
    }
    return warp_butterfly_sum(acc);
}

__device__ __forceinline__ int warp_reduce_sum_int(int v) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(MARS_FULL_MASK, v, off);
    return v;
}

// The one definition of the temporal decay (src/memory_cuda.cu:292-310:
// final = sim * __expf(-lambda * max(0, t_q - ts))), shared by the scan and
// the BFS kernels so a node's score is bit-identical whichever computes it.
__device__ __forceinline__ float fused_weight(float ts, float t_q, float lambda) {
    const float age = fmaxf(0.0f, t_q - ts);
    return __expf(-lambda * age);
}
__device__ __forceinline__ float fused_weight_apply(float dot, float ts, float t_q, float lambda) {
    return dot * fused_weight(ts, t_q, lambda);
}

// ---------------------------------------------------------------------------
// Order-preserving map float -> uint32 (larger float -> larger key).
__device__ __forceinline__ uint32_t f2key(float f) {
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
    uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
    return __uint_as_float(u);
}

// (score desc, id asc)
__device__ __forceinline__ bool better(float sa, int32_t ia, float sb, int32_t ib) {
    return sa > sb || (sa == sb && ia < ib);
}

// ---------------------------------------------------------------------------
// Warp-resident ranked list.  Position p = slot * 32 + lane holds the p-th
// best entry; positions >= K may hold evicted entries and are ignored.  All
// member functions are warp-collective and must be called with warp-uniform
// arguments.
template <int KPL>
struct WarpTopK {
    float   v[KPL];
    int32_t i[KPL];
    float   thr_v;     // entry at position K-1 (the admission threshold)
    int32_t thr_i;
    int     K;

    __device__ __forceinline__ void init(int k) {
        K = k;
#pragma unroll
        for (int s = 0; s < KPL; ++s) { v[s] = -INFINITY; i[s] = INT32_MAX; }
        thr_v = -INFINITY;
        thr_i = INT32_MAX;
    }

    __device__ __forceinline__ bool admits(float s, int32_t id) const {
        return better(s, id, thr_v, thr_i);
    }

    __device__ __forceinline__ void insert(float s, int32_t id, int lane) {
        int pos = 0;
#pragma unroll
        for (int sl = 0; sl < KPL; ++sl)
            pos += __popc(__ballot_sync(MARS_FULL_MASK, better(v[sl], i[sl], s, id)));
#pragma unroll
        for (int sl = KPL - 1; sl >= 0; --sl) {
            const float   up_v = __shfl_up_sync(MARS_FULL_MASK, v[sl], 1);
            const int32_t up_i = __shfl_up_sync(MARS_FULL_MASK, i[sl], 1);
            float   carry_v = -INFINITY;
            int32_t carry_i = INT32_MAX;
            if (sl > 0) {
                carry_v = __shfl_sync(MARS_FULL_MASK, v[sl > 0 ? sl - 1 : 0], 31);
                carry_i = __shfl_sync(MARS_FULL_MASK, i[sl > 0 ? sl - 1 : 0], 31);
            }
            const int p = sl * kWarp + lane;
            if (p > pos) {
                v[sl] = lane == 0 ? carry_v : up_v;
                i[sl] = lane == 0 ? carry_i : up_i;
            } else if (p == pos) {
                v[sl] = s;
                i[sl] = id;
            }
        }
        refresh_threshold();
    }

    __device__ __forceinline__ void refresh_threshold() {
        const int kk = (K - 1) >> 5;
        float tv = v[0];
        int32_t ti = i[0];
#pragma unroll
        for (int sl = 1; sl < KPL; ++sl)
            if (sl == kk) { tv = v[sl]; ti = i[sl]; }
        thr_v = __shfl_sync(MARS_FULL_MASK, tv, (K - 1) & 31);
        thr_i = __shfl_sync(MARS_FULL_MASK, ti, (K - 1) & 31);
    }

    __device__ __forceinline__ void push(float s, int32_t id, int lane) {
        if (admits(s, id)) insert(s, id, lane);
    }

    // Write positions < K to (vals, ids).
    __device__ __forceinline__ void store(float* vals, int32_t* ids, int lane) const {
#pragma unroll
        for (int sl = 0; sl < KPL; ++sl) {
            const int p = sl * kWarp + lane;
            if (p < K) { vals[p] = v[sl]; ids[p] = i[sl]; }
        }
    }

    // Offer a ranked list of n entries (desc); stops at the first entry the
    // list does not admit, since every later entry is worse.
    __device__ __forceinline__ void offer_sorted(const float* vals, const int32_t* ids, int n,
                                                 int lane) {
        for (int base = 0; base < n; base += kWarp) {
            const int j = base + lane;
            float s = -INFINITY;
            int32_t id = INT32_MAX;
            if (j < n) { s = vals[j]; id = ids[j]; }
            unsigned m = __ballot_sync(MARS_FULL_MASK, j < n && admits(s, id));
            if (m == 0) return;
            // entries are sorted: admitted ones form a prefix of this chunk
            while (m) {
                const int src = __ffs(m) - 1;
                m &= m - 1;
                const float   cs = __shfl_sync(MARS_FULL_MASK, s, src);
                const int32_t ci = __shfl_sync(MARS_FULL_MASK, id, src);
                if (!admits(cs, ci)) return;
                insert(cs, ci, lane);
            }
        }
    }

    // Merge a ranked list of n <= 32 entries into this one without serial
    // inserts (KPL == 1): the element-wise better of this list and the other
    // list reversed is a bitonic sequence holding the 32 best entries of
    // both, and five half-cleaner steps sort it.
    __device__ __forceinline__ void merge_sorted32(const float* vals, const int32_t* ids, int n,
                                                   int lane) {
        static_assert(KPL == 1, "merge_sorted32 needs one slot per lane");
        const int j = 31 - lane;
        float bv = -INFINITY;
        int32_t bi = INT32_MAX;
        if (j < n) { bv = vals[j]; bi = ids[j]; }
        if (better(bv, bi, v[0], i[0])) { v[0] = bv; i[0] = bi; }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
            const float ov = __shfl_xor_sync(MARS_FULL_MASK, v[0], off);
            const int32_t oi = __shfl_xor_sync(MARS_FULL_MASK, i[0], off);
            const bool ob = better(ov, oi, v[0], i[0]);
            if (((lane & off) == 0) == ob) { v[0] = ov; i[0] = oi; }
        }
        refresh_threshold();
    }

    // Offer unsorted candidates held one per lane (warp-collective).
    __device__ __forceinline__ void offer_lanes(float s, int32_t id, bool valid, int lane) {
        unsigned m = __ballot_sync(MARS_FULL_MASK, valid && admits(s, id));
        while (m) {
            const int src = __ffs(m) - 1;
            m &= m - 1;
            const float   cs = __shfl_sync(MARS_FULL_MASK, s, src);
            const int32_t ci = __shfl_sync(MARS_FULL_MASK, id, src);
            if (admits(cs, ci)) insert(cs, ci, lane);
        }
    }
};

}  // namespace mars
