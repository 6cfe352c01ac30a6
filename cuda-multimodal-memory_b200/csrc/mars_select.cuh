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
            if (in_bucket <= 32 || shift == 0) break;
        }
        // keep the keys at or above the selected prefix (K - need above the
        // bucket plus the bucket): gathered in the histogram's space, then
        // moved to the front of cand
        unsigned long long* kept = reinterpret_cast<unsigned long long*>(hist);
        int* s_cnt = s_scan + kW + 3;
        if (threadIdx.x == 0) *s_cnt = 0;
        __syncthreads();
        for (int i = threadIdx.x; i < M; i += NT) {
            const unsigned long long k = cand[i];
            if ((k & pmask) >= prefix) kept[atomicAdd(s_cnt, 1)] = k;
        }
        __syncthreads();
        M = *s_cnt;
        for (int i = threadIdx.x; i < M; i += NT) cand[i] = kept[i];
        __syncthreads();
    }
    const int P = next_pow2(max(M, 2));
    for (int j = M + threadIdx.x; j < P; j += NT) cand[j] = 0ull;
    block_bitonic_desc<NT>(cand, P);
    return min(M, K);
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
    constexpr int kBatch = 16;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int total = nl * K;
    int* s_cnt = s_misc + 15;

    // the first batch goes to registers with every load in flight; when the
    // whole input fits in it, the K-th entries (the bound) are among them
    unsigned long long key[kBatch];
    unsigned long long t = 0;
    const bool one_batch = total <= NT * kBatch;
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
        const int j = u * NT + threadIdx.x;
        key[u] = 0ull;
        if (j < total) {
            const int32_t id = __ldcg(ids + j);
            const float v = __ldcg(vals + j);
            if (id != INT32_MAX) {
                key[u] = rank_key(v, id);
                if (one_batch && (j % K) == K - 1) t = key[u] > t ? key[u] : t;
            }
        }
    }
    if (!one_batch) {
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
    if (threadIdx.x == 0) *s_cnt = 0;
    if (lane == 0) s_red[warp] = t;
    __syncthreads();
    t = s_red[0];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) t = s_red[w] > t ? s_red[w] : t;

    // gather every valid entry ranked at or above the bound
    for (int b0 = 0; b0 < total; b0 += NT * kBatch) {
        if (b0 > 0) {
#pragma unroll
            for (int u = 0; u < kBatch; ++u) {
                const int j = b0 + u * NT + threadIdx.x;
                key[u] = 0ull;
                if (j < total) {
                    const int32_t id = __ldcg(ids + j);
                    const float v = __ldcg(vals + j);
                    if (id != INT32_MAX) key[u] = rank_key(v, id);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            if (key[u] != 0ull && key[u] >= t) {
                const int pos = atomicAdd(s_cnt, 1);
                if (pos < cap) cand[pos] = key[u];
            }
        }
    }
    __syncthreads();
    const int n = *s_cnt;
    __syncthreads();
    if (n > cap) return -1;
    return block_select_topk<NT>(cand, n, K, hist, s_misc);
}

}  // namespace mars
