// mars_select.cuh -- block-wide selection helpers for the tails of the scan
// and query kernels (one CTA, after every other CTA has finished).
//
// A candidate (score, id) is packed into one 64-bit key
//     key = f2key(score) << 32 | (0xffffffff - id)
// so that "larger key" is exactly the ranking order of the library
// (score desc, id asc) and a plain integer compare ranks candidates.
#pragma once

#include "mars_common.cuh"

namespace mars {

__device__ __forceinline__ unsigned long long rank_key(float s, int32_t id) {
    return ((unsigned long long)f2key(s) << 32) | (unsigned long long)(0xffffffffu - (uint32_t)id);
}
__device__ __forceinline__ int32_t key_id(unsigned long long k) {
    return (int32_t)(0xffffffffu - (uint32_t)(k & 0xffffffffull));
}
__device__ __forceinline__ float key_score(unsigned long long k) { return key2f((uint32_t)(k >> 32)); }

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        const unsigned long long o = __shfl_xor_sync(MARS_FULL_MASK, v, off);
        v = o > v ? o : v;
    }
    return v;
}

// Sort keys[0, P) in descending order; P is a power of two.  Every thread of
// the block calls it; it starts and ends with a __syncthreads().
template <int NT>
__device__ __forceinline__ void block_bitonic_desc(unsigned long long* keys, int P) {
    __syncthreads();
    for (int k = 2; k <= P; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int t = threadIdx.x; t < (P >> 1); t += NT) {
                const int i = ((t & ~(j - 1)) << 1) | (t & (j - 1));   // bit j of i is clear
                const int l = i | j;
                const unsigned long long a = keys[i], b = keys[l];
                const bool desc = (i & k) == 0;
                if (desc ? (a < b) : (a > b)) { keys[i] = b; keys[l] = a; }
            }
            __syncthreads();
        }
    }
}

// Sort keys[0, M) (M <= 32) in descending order within warp 0, in
// registers (no block barriers); every thread calls it, it ends with a
// __syncthreads().
__device__ __forceinline__ void warp0_sort32_desc(unsigned long long* keys, int M) {
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        unsigned long long v = lane < M ? keys[lane] : 0ull;
#pragma unroll
        for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
            for (int j = k >> 1; j > 0; j >>= 1) {
                const unsigned long long o = __shfl_xor_sync(MARS_FULL_MASK, v, j);
                const bool lower = (lane & j) == 0;
                const bool desc = (lane & k) == 0;
                // the lower lane of a descending pair keeps the larger key
                const bool take = (lower == desc) ? (o > v) : (o < v);
                if (take) v = o;
            }
        }
        if (lane < M) keys[lane] = v;
    }
    __syncthreads();
}

__device__ __forceinline__ float4 ld_cg_f4(const float4* p) {
    float4 v;
    asm volatile("ld.global.cg.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ int4 ld_cg_i4(const int4* p) {
    int4 v;
    asm volatile("ld.global.cg.v4.s32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

// Append `key` to list[] at a shared counter, one shared atomic per warp.
// Warp-collective: every lane of the warp calls it.
__device__ __forceinline__ void warp_append(bool take, unsigned long long key, unsigned long long* list,
                                            int* counter, int cap) {
    const unsigned m = __ballot_sync(MARS_FULL_MASK, take);
    if (m == 0) return;
    const int lane = threadIdx.x & 31;
    int base = 0;
    if (lane == __ffs(m) - 1) base = atomicAdd(counter, __popc(m));
    base = __shfl_sync(MARS_FULL_MASK, base, __ffs(m) - 1);
    const int pos = base + __popc(m & ((1u << lane) - 1u));
    if (take && pos < cap) list[pos] = key;
}

// Exclusive prefix sum of one int per thread over the block; *total gets
// the sum.  s_warp: NT / 32 + 1 ints.  Starts and ends with __syncthreads().
template <int NT>
__device__ __forceinline__ int block_exclusive_scan1(int x, int* total, int* s_warp) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int inc = x;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(MARS_FULL_MASK, inc, off);
        if (lane >= off) inc += y;
    }
    __syncthreads();
    if (lane == 31) s_warp[warp] = inc;
    __syncthreads();
    int before = inc - x, sum = 0;
#pragma unroll
    for (int w = 0; w < NT / 32; ++w) {
        if (w < warp) before += s_warp[w];
        sum += s_warp[w];
    }
    *total = sum;
    __syncthreads();
    return before;
}

__host__ __device__ __forceinline__ int next_pow2(int x) {
    int p = 1;
    while (p < x) p <<= 1;
    return p;
}

// Top-K of cand[0, M) (unique keys, any order), K <= 256, by MSD radix
// selection: 11 bits per pass, each pass histograms the candidates that
// still share the selected prefix and keeps the bucket that holds the K-th
// largest key.  The passes stop once that bucket holds at most 32 keys; the
// keys above the bucket plus the bucket itself (at most K + 31, since keys
// are unique) are then sorted.  On return cand[0, min(M, K)) holds the top-K
// in rank order; cand needs room for next_pow2(min(M, K + 31)) keys.
// hist: 2048 ints of shared scratch (not overlapping cand); s_misc: 12 ints.
template <int NT>
__device__ int block_select_topk(unsigned long long* cand, int M, int K, int* hist, int* s_misc) {
    if (M <= 0) return 0;
    constexpr int kW = NT / 32;
    int* s_scan = s_misc;   // [0, kW) warp partial sums, [kW, kW + 4) results
    if (M > K) {
        unsigned long long prefix = 0ull, pmask = 0ull;
        int need = K, shift = 64;
        while (true) {
            const int bits = shift >= 11 ? 11 : shift;
            shift -= bits;
            const int nb = 1 << bits;
            for (int b = threadIdx.x; b < 2048; b += NT) hist[b] = 0;
            __syncthreads();
            for (int i = threadIdx.x; i < M; i += NT) {
                const unsigned long long k = cand[i];
                if ((k & pmask) == prefix) atomicAdd(&hist[(int)((k >> shift) & (unsigned long long)(nb - 1))], 1);
            }
            __syncthreads();
            // the bucket holding the need-th largest, counted from the top
            constexpr int kPer = 2048 / NT;
            int local[kPer], lsum = 0;
#pragma unroll
            for (int u = 0; u < kPer; ++u) {
                const int b = nb - 1 - (threadIdx.x * kPer + u);   // descending bucket order
                local[u] = b >= 0 ? hist[b] : 0;
                lsum += local[u];
            }
            const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
            int inc = lsum;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int y = __shfl_up_sync(MARS_FULL_MASK, inc, off);
                if (lane >= off) inc += y;
            }
            if (lane == 31) s_scan[warp] = inc;
            __syncthreads();
            int above = inc - lsum;
#pragma unroll
            for (int w = 0; w < kW; ++w)
                if (w < warp) above += s_scan[w];
            if (above < need && need <= above + lsum) {
                int acc = above;
#pragma unroll
                for (int u = 0; u < kPer; ++u) {
                    if (acc < need && need <= acc + local[u]) {
                        s_scan[kW + 0] = nb - 1 - (threadIdx.x * kPer + u);
                        s_scan[kW + 1] = acc;
                        s_scan[kW + 2] = local[u];
                    }
                    acc += local[u];
                }
            }
            __syncthreads();
            const int bsel = s_scan[kW + 0];
            need -= s_scan[kW + 1];
            const int in_bucket = s_scan[kW + 2];
            prefix |= (unsigned long long)bsel << shift;
            pmask |= (unsigned long long)(nb - 1) << shift;
            __syncthreads();
            // stop once the keys to keep fit one warp's sort (K <= 32) or
            // the bucket is down to 32 keys
            if ((K <= 32 ? (K - need) + in_bucket <= 32 : in_bucket <= 32) || shift == 0) break;
        }
        // keep the keys at or above the selected prefix (K - need above the
        // bucket plus the bucket): gathered in the histogram's space, then
        // moved to the front of cand
        unsigned long long* kept = reinterpret_cast<unsigned long long*>(hist);
        int* s_cnt = s_scan + kW + 3;
        if (threadIdx.x == 0) *s_cnt = 0;
        __syncthreads();
        for (int i0 = 0; i0 < M; i0 += NT) {
            const int i = i0 + threadIdx.x;
            const unsigned long long k = i < M ? cand[i] : 0ull;
            warp_append(i < M && (k & pmask) >= prefix, k, kept, s_cnt, 1024);
        }
        __syncthreads();
        // (more than 1024 only if keys repeat; the copies beyond are dropped)
        M = min(*s_cnt, 1024);
        for (int i = threadIdx.x; i < M; i += NT) cand[i] = kept[i];
        __syncthreads();
    }
    if (M <= 32) {
        warp0_sort32_desc(cand, M);
        return min(M, K);
    }
    const int P = next_pow2(M);
    for (int j = M + threadIdx.x; j < P; j += NT) cand[j] = 0ull;
    block_bitonic_desc<NT>(cand, P);
    return min(M, K);
}

// The k-th largest of n 32-bit keys (1 <= k <= n), key i = load(i), by MSD
// radix selection: 11, 11 and 10 bits, each pass a shared histogram of the
// keys that share the prefix chosen so far.  Every thread of the block calls
// it; hist: 2048 ints, s_sel: 2 words of shared scratch.  Starts and ends
// with __syncthreads().
template <int NT, class Load>
__device__ uint32_t block_kth_largest_key(Load load, int n, int k, int* hist, uint32_t* s_sel) {
    static_assert(NT % 32 == 0 && 1024 % NT == 0, "whole warps, bucket groups of equal size");
    __shared__ int s_wsum[NT / 32];   // each warp's share of the bucket counts
    const int lane = threadIdx.x & 31;
    uint32_t prefix = 0, pmask = 0;
    int rem = k;
    __syncthreads();
#pragma unroll 1
    for (int pass = 0; pass < 3; ++pass) {
        const int sh = pass == 0 ? 21 : (pass == 1 ? 10 : 0);
        const int nb = pass == 2 ? 1024 : 2048;
        for (int i = threadIdx.x; i < nb; i += NT) hist[i] = 0;
        __syncthreads();
        // keys crowd into few buckets (one exponent range): lanes that hit
        // the same bucket add their count with one atomic
        for (int i0 = threadIdx.x - (threadIdx.x & 31); i0 < n; i0 += NT) {
            const int i = i0 + (threadIdx.x & 31);
            const uint32_t key = i < n ? load(i) : 0u;
            const bool in = i < n && (key & pmask) == prefix;
            const int bucket = in ? (int)((key >> sh) & (uint32_t)(nb - 1)) : -1;
            const unsigned peers = __match_any_sync(0xffffffffu, bucket);
            if (in && (threadIdx.x & 31) == __ffs(peers) - 1) atomicAdd(&hist[bucket], __popc(peers));
        }
        __syncthreads();
        // the bucket holding the rem-th largest key: thread t sums the t-th
        // group of nb / NT buckets counted from the top, a block-wide
        // prefix sum over the groups (warp scans, then the warps' totals)
        // finds the one group that holds it, and its thread walks it
        {
            const int per = nb / NT;
            const int top = nb - (int)threadIdx.x * per;
            int sum = 0;
            for (int b = top - 1; b >= top - per; --b) sum += hist[b];
            int incl = sum;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int t = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += t;
            }
            if (lane == 31) s_wsum[threadIdx.x >> 5] = incl;
            __syncthreads();
            int before = 0;
            for (int w = 0; w < (int)(threadIdx.x >> 5); ++w) before += s_wsum[w];
            incl += before;
            const int excl = incl - sum;
            if (excl < rem && rem <= incl) {
                int acc = excl;
                for (int b = top - 1; b >= top - per; --b) {
                    if (acc + hist[b] >= rem) {
                        s_sel[0] = prefix | ((uint32_t)b << sh);
                        s_sel[1] = (uint32_t)(rem - acc);
                        break;
                    }
                    acc += hist[b];
                }
            }
        }
        __syncthreads();
        prefix = s_sel[0];
        rem = (int)s_sel[1];
        pmask |= (uint32_t)(nb - 1) << sh;
        __syncthreads();
    }
    return prefix;
}

// Merge nl ranked lists of K entries each (list l at vals/ids + l * K, rank
// order, empty slots id == INT32_MAX) into their top-K.
//
// Any list's K-th entry bounds the answer: that list alone holds K entries
// ranked at or above it, so every entry of the merged top-K ranks at or above
// the largest such K-th entry.  Entries at or above that bound are gathered
// into cand[] (at most `cap`) and the top-K of them selected.  On return
// cand[0, cnt) holds the merged top-K in rank order and the function returns
// cnt (<= K), or -1 when more than `cap` entries passed the bound (the caller
// then merges another way).
//
// hist: 2048 ints of shared scratch; s_misc: 16 ints; s_red: NT / 32 keys.
template <int NT>
__device__ int merge_ranked_lists(const float* __restrict__ vals, const int32_t* __restrict__ ids,
                                  int nl, int K, unsigned long long* cand, int cap, int* hist,
                                  int* s_misc, unsigned long long* s_red) {
    constexpr int kWarps = NT / 32;
    constexpr int kG = 4;                   // 16-byte groups per thread and batch
    constexpr int kBatch = NT * kG * 4;     // entries per batch
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int total = nl * K;
    // 16-byte loads need 16-byte aligned arrays (the partial buffers are);
    // otherwise every entry is read on its own
    const bool vec = ((reinterpret_cast<uintptr_t>(vals) | reinterpret_cast<uintptr_t>(ids)) & 15u) == 0;

    // one batch of entries in registers: group g holds entries 4g .. 4g+3
    float4 v4[kG];
    int4 i4[kG];
    auto load_batch = [&](int b0) {
#pragma unroll
        for (int u = 0; u < kG; ++u) {
            const int e = b0 + (u * NT + threadIdx.x) * 4;
            v4[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            i4[u] = make_int4(INT32_MAX, INT32_MAX, INT32_MAX, INT32_MAX);
            if (vec && e + 3 < total) {
                v4[u] = ld_cg_f4(reinterpret_cast<const float4*>(vals + e));
                i4[u] = ld_cg_i4(reinterpret_cast<const int4*>(ids + e));
            } else {
                if (e + 0 < total) { v4[u].x = __ldcg(vals + e + 0); i4[u].x = __ldcg(ids + e + 0); }
                if (e + 1 < total) { v4[u].y = __ldcg(vals + e + 1); i4[u].y = __ldcg(ids + e + 1); }
                if (e + 2 < total) { v4[u].z = __ldcg(vals + e + 2); i4[u].z = __ldcg(ids + e + 2); }
                if (e + 3 < total) { v4[u].w = __ldcg(vals + e + 3); i4[u].w = __ldcg(ids + e + 3); }
            }
        }
    };
    auto key_of = [&](int u, int c) -> unsigned long long {
        const float v = c == 0 ? v4[u].x : c == 1 ? v4[u].y : c == 2 ? v4[u].z : v4[u].w;
        const int32_t id = c == 0 ? i4[u].x : c == 1 ? i4[u].y : c == 2 ? i4[u].z : i4[u].w;
        return id != INT32_MAX ? rank_key(v, id) : 0ull;
    };

    // the bound: the largest K-th entry over the lists (taken from the
    // first batch when it holds everything)
    unsigned long long t = 0;
    load_batch(0);
    if (total <= kBatch) {
#pragma unroll
        for (int u = 0; u < kG; ++u) {
            const int e = (u * NT + threadIdx.x) * 4;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                if ((e + c) % K == K - 1) {
                    const unsigned long long k = key_of(u, c);
                    t = k > t ? k : t;
                }
            }
        }
    } else {
        for (int l = threadIdx.x; l < nl; l += NT) {
            const int32_t id = __ldcg(ids + (int64_t)l * K + K - 1);
            const float v = __ldcg(vals + (int64_t)l * K + K - 1);
            if (id != INT32_MAX) {
                const unsigned long long k = rank_key(v, id);
                t = k > t ? k : t;
            }
        }
    }
    t = warp_max_u64(t);
    if (lane == 0) s_red[warp] = t;
    __syncthreads();
    t = s_red[0];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) t = s_red[w] > t ? s_red[w] : t;

    // gather every valid entry ranked at or above the bound: per-thread
    // counts, one block prefix sum, then every thread writes its own
    int n = 0;
    for (int b0 = 0; b0 < total; b0 += kBatch) {
        if (b0 > 0) load_batch(b0);
        unsigned pass = 0u;
        int mine = 0;
#pragma unroll
        for (int u = 0; u < kG; ++u) {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const unsigned long long k = key_of(u, c);
                if (k != 0ull && k >= t) { pass |= 1u << (u * 4 + c); ++mine; }
            }
        }
        int batch_n = 0;
        int pos = n + block_exclusive_scan1<NT>(mine, &batch_n, s_misc);
#pragma unroll
        for (int u = 0; u < kG; ++u) {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                if (pass & (1u << (u * 4 + c))) {
                    if (pos < cap) cand[pos] = key_of(u, c);
                    ++pos;
                }
            }
        }
        n += batch_n;
    }
    __syncthreads();
    if (n > cap) return -1;
    return block_select_topk<NT>(cand, n, K, hist, s_misc);
}

}  // namespace mars
