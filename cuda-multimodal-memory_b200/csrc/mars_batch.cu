// mars_batch.cu -- batched fused scan on the tensor cores (tcgen05 + TMEM).
//
// B queries x N rows: scores = Q * E^T (a dense contraction, 2*B*N*D flops)
// followed by decay x importance and a per-query top-K.  The reference has no
// batched path; its single-query pipeline (src/memory_cuda.cu:924-1067) run B
// times reads E B times.  Here E streams through the tensor cores once per
// 128 queries:
//
//  1. prep:      per-row weight w = __expf(-lambda*age) [x importance] (NaN for
//                rows the modality filter rejects), per-query error margin.
//  2. sample:    the GEMM over a strided sample of row tiles; each (query,
//                32-row chunk) keeps its 4 best lower bounds.
//  3. threshold: per query the j-th best sampled lower bound, theta.  j is
//                chosen so that theta lies, with overwhelming probability,
//                below the query's true K-th best score.
//  4. candidates: the GEMM over all rows; a row becomes a candidate of a query
//                when its upper bound reaches theta.
//  5. rescore:   completeness check from the candidates' bounds (K of them
//                with lower bound >= theta prove that no row outside the list
//                can place), pruning by the K-th best lower bound, then the
//                exact fp32 score of the survivors with the canonical dot (the
//                same arithmetic as the single-query scan) and the top-K.
//                Queries that fail the check are rescanned exactly on the
//                device (the fused scan, only those queries).
//
// GEMM: kind::tf32 (fp32 operands read by TMA straight from the store, 128-byte
// swizzled K-major tiles), M = 128 queries x N = 256 rows per tile, K steps of
// 32, 4-stage TMA ring, accumulators double-buffered in TMEM (2 x 256 columns).
// Warp roles: warp 0 TMA producer, warp 1 MMA issuer + TMEM owner, warps 2-9
// epilogue (one query row per thread and half of the tile's columns,
// tcgen05.ld 32x32b).
//
// Error bound of the approximate score: operands keep 10 mantissa bits, so
// |A - dot| <= (2^-9 + 2^-20) |q||e| + accumulation (<= D 2^-23 |q||e|); the
// margin used is 2.6e-3 |q| max|e|, covering D <= 4096.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "mars_b200.h"
#include "mars_common.cuh"
#include "mars_internal.h"
#include "mars_kernels.cuh"
#include "mars_select.cuh"
#include "mars_sm100.cuh"

namespace mars {
namespace batch {

constexpr int kBM = 128;              // queries per tile (UMMA M)
constexpr int kBN = 256;              // rows per tile (UMMA N)
constexpr int kBK = 32;               // fp32 per 128-byte swizzle row
constexpr int kStages = 4;
constexpr int kStageA = kBM * kBK * 4;    // 16 KB
constexpr int kStageB = kBN * kBK * 4;    // 32 KB
constexpr int kStageBytes = kStageA + kStageB;
// 128 x 256 tiles: producer, MMA and 8 epilogue warps -- two per TMEM lane
// quarter, each taking half of the tile's 256 columns (with 4 the epilogue
// was the slower half of the pipeline)
constexpr int kGemmThreads = 320;
constexpr int kGemmEpi = kGemmThreads - 64;  // epilogue threads
constexpr int kTmemCols = 512;
constexpr int kJ = 16;                // sampled lower bounds kept per (query, tile half)
constexpr int kSampleKeep = 4;        // ... as the 4 best of each of the half's 4 32-row chunks
static_assert(kJ == kSampleKeep * (kBN / 64), "a tile half's chunks fill its kJ values");
// Relative error margin of a short-listed score, times ||q|| max||e||.
// TF32 operands: the tensor cores may truncate each fp32 operand to 10
// mantissa bits (2^-10 relative each, 1.95e-3 for the product's two
// factors), plus the fp32 accumulation.  fp16 operands: both copies are
// rounded to nearest here (2^-11 each, 9.8e-4 together; products of fp16
// values are exact in fp32), plus the accumulation over at most 64 16-wide
// steps, far below the remaining 6e-4.
constexpr float kMarginRel = 2.6e-3f;
// fp16 operands: the rounding of both copies is bounded exactly instead
// (|q.e - q16.e16| <= ||q|| ||e - e16|| + ||q - q16|| ||e16||, Cauchy-Schwarz,
// with ||e - e16|| the store's largest measured row error and ||q - q16||
// measured per query); this term, times ||q|| max||e||, covers the rest: the
// fp32 accumulation inside and across the tensor-core steps (D / 16 <= 64
// steps; fp32 accumulation errs by ~2^-23 of the running magnitude per
// step, so the budget holds ~2^-19 per step) and the canonical fp32 dot's
// own rounding (<= (D / 32 + 5) 2^-24).
constexpr float kAccRelF16 = 2.0e-4f;

enum Mode { kSample = 0, kCandidates = 1, kFused = 2 };

// What a row's fused score multiplies its dot product by: the decay
// exp(-lambda * max(0, t_q - ts)), times the importance when asked, NaN for a
// row of another modality than the filter's (never a candidate).  The same
// expression as the exact score's, computed where it is needed.
struct RowMeta {
    const float* ts;
    const float* imp;
    const int32_t* mod;
    float t_q, lambda;
    int32_t filter, use_imp;
};

__device__ __forceinline__ float row_weight(const RowMeta& m, int32_t row) {
    if (m.filter >= 0 && __ldg(m.mod + row) != m.filter) return NAN;
    float w = __expf(-m.lambda * fmaxf(0.0f, m.t_q - __ldg(m.ts + row)));
    if (m.use_imp) w = w * __ldg(m.imp + row);
    return w;
}

// One short-listed candidate as a single 16-byte record: row, approximate
// fused score and its error slack (margin x |weight|) as float bits (the
// exact score lies in score -+ slack).  One store per candidate.
__device__ __forceinline__ int4 cand_entry(int32_t row, float f, float slack) {
    return make_int4(row, __float_as_int(f), __float_as_int(slack), 0);
}

struct GemmArgs {
    int32_t B, n, nkb;               // queries, rows, K blocks
    int32_t qtiles, rtiles;          // tiles along queries / rows
    int32_t n_tiles;                 // total tiles of this launch
    const int32_t* sample_rt;        // sample mode: row tile of sample tile i
    RowMeta meta;                    // row weights
    const float* theta;              // B thresholds (candidate mode)
    const float* margin;             // B margins
    float* sample_buf;               // [sample tiles][B][2 halves][kJ]
    int4* cand;                      // [B][cap] candidates (cand_entry)
    int32_t* cand_cnt;               // [B]
    int32_t cap;
    int32_t self_base;               // query b leaves out row self_base + b (-1: none)
    int* err;
};

__device__ __forceinline__ void tile_coords(const GemmArgs& a, int t, int mode, int& qt, int& row0) {
    if (mode == kSample) {
        qt = t % a.qtiles;
        row0 = a.sample_rt[t / a.qtiles] * kBN;
    } else {
        qt = t % a.qtiles;          // query tiles innermost: CTAs running side by
        row0 = (t / a.qtiles) * kBN;  // side share the row tile through L2
    }
}

// F16: operands are fp16 copies of the queries and rows (kind::f16, 64
// elements per 128-byte row of a stage); otherwise fp32 read as TF32
// (kind::tf32, 32 elements).  Both keep 10 mantissa bits; the stage layout in
// bytes is the same.
template <int MODE, bool F16>
__global__ void __launch_bounds__(kGemmThreads, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_e,
            const GemmArgs a) {
    constexpr int kElemsK = F16 ? 64 : 32;      // elements per 128-byte k-block
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
    uint64_t* empty = full + kStages;
    uint64_t* tfull = empty + kStages;
    uint64_t* tempty = tfull + 2;
    uint64_t* mdrain = tempty + 2;      // the MMA issuer's last commit
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mdrain + 1);
    float* s_w = reinterpret_cast<float*>(smem + kStages * kStageBytes + 256);   // [kBN] row weights

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) { sm100::mbar_init(full + s, 1); sm100::mbar_init(empty + s, 1); }
        for (int b = 0; b < 2; ++b) { sm100::mbar_init(tfull + b, 1); sm100::mbar_init(tempty + b, kGemmEpi); }
        sm100::mbar_init(mdrain, 1);
        sm100::fence_mbar_init();
        sm100::prefetch_tmap(&tmap_q);
        sm100::prefetch_tmap(&tmap_e);
    }
    if (warp == 1) {
        sm100::tmem_alloc(tmem_slot, kTmemCols);
        sm100::tmem_relinquish();
    }
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued_phase[kStages];
            bool issued[kStages];
            for (int s = 0; s < kStages; ++s) { issued[s] = false; issued_phase[s] = 0; }
            bool ok = true;
            for (int t = blockIdx.x; t < a.n_tiles && ok; t += gridDim.x) {
                int qt, row0;
                tile_coords(a, t, MODE, qt, row0);
                for (int kb = 0; kb < a.nkb; ++kb) {
                    if (!sm100::mbar_wait(empty + stage, phase ^ 1u, a.err, 1)) { ok = false; break; }
                    uint8_t* sa = smem + stage * kStageBytes;
                    sm100::mbar_arrive_expect_tx(full + stage, kStageBytes);
                    sm100::tma_load_2d(sa, &tmap_q, full + stage, kb * kElemsK, qt * kBM);
                    sm100::tma_load_2d(sa + kStageA, &tmap_e, full + stage, kb * kElemsK, row0);
                    issued[stage] = true;
                    issued_phase[stage] = phase;
                    if (++stage == kStages) { stage = 0; phase ^= 1u; }
                }
            }
            // every copy this thread started has landed before the CTA may exit
            // (also after a wait gave up: the drain does not stop at the error word)
            for (int s = 0; s < kStages; ++s)
                if (issued[s]) sm100::mbar_wait_drain(full + s, issued_phase[s], a.err, 2);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = F16 ? sm100::idesc_f16(kBM, kBN) : sm100::idesc_tf32(kBM, kBN);
            int stage = 0;
            uint32_t phase = 0;
            int buf = 0;
            uint32_t bphase = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < a.n_tiles && ok; t += gridDim.x) {
                if (!sm100::mbar_wait(tempty + buf, bphase ^ 1u, a.err, 3)) break;
                sm100::tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(buf * kBN);
                for (int kb = 0; kb < a.nkb; ++kb) {
                    if (!sm100::mbar_wait(full + stage, phase, a.err, 4)) { ok = false; break; }
                    sm100::tc_fence_after();
                    const uint32_t sa = sm100::smem_u32(smem + stage * kStageBytes);
                    const uint64_t da = sm100::smem_desc_sw128(sa);
                    const uint64_t db = sm100::smem_desc_sw128(sa + kStageA);
#pragma unroll
                    for (int k = 0; k < 4; ++k) {      // 32 bytes of K per MMA: 8 tf32 or 16 fp16
                        if constexpr (F16)
                            sm100::mma_f16(d, da + (uint64_t)(2 * k), db + (uint64_t)(2 * k), idesc,
                                           (kb > 0 || k > 0) ? 1u : 0u);
                        else
                            sm100::mma_tf32(d, da + (uint64_t)(2 * k), db + (uint64_t)(2 * k), idesc,
                                            (kb > 0 || k > 0) ? 1u : 0u);
                    }
                    sm100::mma_commit(empty + stage);   // stage reusable when these MMAs finish
                    if (++stage == kStages) { stage = 0; phase ^= 1u; }
                }
                if (!ok) break;
                sm100::mma_commit(tfull + buf);         // accumulator ready
                if (++buf == 2) { buf = 0; bphase ^= 1u; }
            }
            // every MMA this thread issued has finished before TMEM is freed
            // (also when a wait gave up and the loop ended early)
            sm100::mma_commit(mdrain);
            sm100::mbar_wait_drain(mdrain, 0, a.err, 6);
        }
    } else {
        // ---------------- epilogue (warps 2..9) ----------------
        const int sub = warp & 3;                   // TMEM lane quarter of this warp
        const int half = (warp - 2) >> 2;           // columns [128 half, 128 half + 128)
        const int row_in_tile = sub * 32 + lane;    // query row of this thread
        int buf = 0;
        uint32_t bphase = 0;
        const int et = threadIdx.x - 64;           // 0..255 among the epilogue threads
        float* stg = s_w + kBN + (warp - 2) * (32 * 32);   // this warp's 32 x 32 score stage
        for (int t = blockIdx.x; t < a.n_tiles; t += gridDim.x) {
            int qt, row0;
            tile_coords(a, t, MODE, qt, row0);
            const int q = qt * kBM + row_in_tile;
            const bool qv = q < a.B;
            const int32_t self_row = a.self_base >= 0 ? a.self_base + q : -1;
            // per-tile operands fetched while the tensor cores still work on
            // this tile: the row weights go to shared memory in one round trip
            const float th = (MODE == kCandidates && qv) ? __ldg(a.theta + q) : 0.f;
            const float mg = qv ? __ldg(a.margin + q) : 0.f;
            asm volatile("bar.sync 1, 256;" ::: "memory");   // previous tile's reads of s_w done
            for (int i = et; i < kBN; i += kGemmEpi) s_w[i] = (row0 + i < a.n) ? row_weight(a.meta, row0 + i) : NAN;
            asm volatile("bar.sync 1, 256;" ::: "memory");
            if (!sm100::mbar_wait(tfull + buf, bphase, a.err, 5)) break;
            sm100::tc_fence_after();
            // one 32-row chunk of the accumulator at a time (the chunk loop is
            // left rolled: the epilogue's code shares the instruction cache
            // with the producer and MMA warps)
#pragma unroll 1
            for (int c = half * (kBN / 64); c < (half + 1) * (kBN / 64); ++c) {
                uint32_t r[32];
                sm100::tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(sub * 32) << 16) +
                                              (uint32_t)(buf * kBN + c * 32), r);
                sm100::tmem_ld_wait();
                const int rbase = row0 + c * 32;
                if constexpr (MODE == kCandidates) {
                    // which of the 32 rows pass (none for an absent query)
                    uint32_t pass = 0u;
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const float w = (rbase + j == self_row) ? NAN : s_w[c * 32 + j];
                        const float f = __uint_as_float(r[j]) * w;
                        if (qv && f + mg * fabsf(w) >= th) pass |= 1u << j;   // NaN weights never pass
                    }
                    if (__any_sync(0xffffffffu, pass != 0u)) {
                        // the warp's 32 x 32 scores go to its shared-memory
                        // stage, column j of lane l at [j][l] (no bank
                        // conflicts writing or reading), so each lane then
                        // walks only its own hits: one atomic for all of them
                        // (clustered data can make a query's candidates dense
                        // in a few tiles) and one 16-byte record per hit
#pragma unroll
                        for (int j = 0; j < 32; ++j) stg[j * 32 + lane] = __uint_as_float(r[j]);
                        __syncwarp();
                        if (pass != 0u) {
                            int pos = atomicAdd(a.cand_cnt + q, __popc(pass));
                            int4* dst = a.cand + (int64_t)q * a.cap;
                            while (pass != 0u) {
                                const int j = __ffs(pass) - 1;
                                pass &= pass - 1u;
                                if (pos < a.cap) {
                                    const float w = s_w[c * 32 + j];
                                    dst[pos] = cand_entry(rbase + j, stg[j * 32 + lane] * w, mg * fabsf(w));
                                }
                                ++pos;
                            }
                        }
                        __syncwarp();   // the next chunk rewrites the stage
                    }
                } else {
                    if (!qv) continue;
                    // sample mode: this chunk's kSampleKeep best lower bounds
                    // of query q, out to sample_buf[tile][query][half][chunk]
                    // (-inf where fewer).  A subset of the sampled values: the
                    // j-th largest of them is at most the j-th largest of all
                    // (a threshold never above the full sample's), and with j
                    // small against the sample the two almost always agree.
                    float best[kSampleKeep];
#pragma unroll
                    for (int s = 0; s < kSampleKeep; ++s) best[s] = -INFINITY;
#pragma unroll
                    for (int j4 = 0; j4 < 8; ++j4) {
                        const float4 w4 = reinterpret_cast<const float4*>(s_w + c * 32)[j4];
                        const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const int j = 4 * j4 + u;
                            const float w = (rbase + j == self_row) ? NAN : wv[u];
                            const float f = __uint_as_float(r[j]) * w;
                            const float slack = mg * fabsf(w);
                            float lo = f - slack;
                            if (lo > best[kSampleKeep - 1]) {    // NaN never passes
#pragma unroll
                                for (int s = 0; s < kSampleKeep; ++s) {
                                    if (lo > best[s]) { const float tmp = best[s]; best[s] = lo; lo = tmp; }
                                }
                            }
                        }
                    }
                    float* dst = a.sample_buf + (((int64_t)(t / a.qtiles) * a.B + q) * 2 + half) * kJ +
                                 (c - half * (kBN / 64)) * kSampleKeep;
#pragma unroll
                    for (int s = 0; s < kSampleKeep; ++s) dst[s] = best[s];
                }
            }
            sm100::tc_fence_before();
            sm100::mbar_arrive(tempty + buf);
            if (++buf == 2) { buf = 0; bphase ^= 1u; }
        }
    }
    sm100::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        sm100::tc_fence_after();
        sm100::tmem_dealloc(tmem_base, kTmemCols);
    }
}

// ---------------------------------------------------------------------------
// Per query (one warp): the error margin, the fp16 range flag, the fp16 copy
// of the query when q16 is given (rows of pitch16 halves, zero padded), and
// the per-call counters zeroed (candidate count, rescored count; the error
// word by query 0).
__global__ void prep_queries_kernel(const float* __restrict__ Q, int64_t qpitch, int32_t B, int32_t nc,
                                    const unsigned int* __restrict__ norm_bits, int32_t f16,
                                    float* __restrict__ margin, int32_t* __restrict__ cand_cnt,
                                    int32_t* __restrict__ rescored, int32_t* __restrict__ bad,
                                    int32_t* __restrict__ err, __half* __restrict__ q16, int32_t pitch16) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= B) return;
    const float4* q = reinterpret_cast<const float4*>(Q + (int64_t)warp * qpitch);
    __half2* h = q16 != nullptr ? reinterpret_cast<__half2*>(q16 + (int64_t)warp * pitch16) : nullptr;
    float s = 0.f, dq2 = 0.f;    // ||q||^2 and ||q - fp16(q)||^2
    bool out = false;
    for (int c = lane; c < nc; c += 32) {
        const float4 v = q[c];
        s += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        out = out || !(fabsf(v.x) <= kF16Max) || !(fabsf(v.y) <= kF16Max) || !(fabsf(v.z) <= kF16Max) ||
              !(fabsf(v.w) <= kF16Max);
        if (h != nullptr) {
            const __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
            h[2 * c] = a;
            h[2 * c + 1] = b;
            const float ex = v.x - __low2float(a), ey = v.y - __high2float(a);   // exact differences
            const float ez = v.z - __low2float(b), ew = v.w - __high2float(b);
            dq2 = fmaf(ex, ex, fmaf(ey, ey, fmaf(ez, ez, fmaf(ew, ew, dq2))));
        }
    }
    if (h != nullptr)
        for (int p = 2 * nc + lane; p < pitch16 / 2; p += 32) h[p] = __floats2half2_rn(0.0f, 0.0f);
    s = warp_butterfly_sum(s);
    dq2 = warp_butterfly_sum(dq2);
    out = __any_sync(0xffffffffu, out);
    if (lane == 0) {
        bad[warp] = out ? 1 : 0;
        rescored[warp] = 0;
        if (warp == 0) { err[0] = 0; err[1] = 0; }   // the pipeline's and the arrival wait's words
        // 1.0001: covers the fp32 rounding of this norm itself
        const float qn = sqrtf(s) * 1.0001f, en = __uint_as_float(norm_bits[0]);
        float mg;
        if (f16) {
            // measured rounding: the rows' largest ||e - e16|| (norm_bits[1])
            // and this query's ||q - q16||; ||e16|| <= ||e|| + ||e - e16||.
            // Components below the fp16 normal range are included: the
            // differences are taken from the converted values themselves.
            const float err = __uint_as_float(norm_bits[1]);
            const float dq = sqrtf(dq2) * 1.001f;
            mg = (qn * err + dq * (en + err) + kAccRelF16 * qn * en) * 1.001f;
        } else {
            mg = kMarginRel * qn * en;
        }
        margin[warp] = mg;
        cand_cnt[warp] = 0;
    }
}

// theta[q] = the j-th largest of query q's sampled values (-inf when fewer
// than j exist; j <= kThrKeep), over n_sample_tiles * per_tile values laid out
// [tile][query][per_tile], empty slots -inf.  One warp per query: each lane
// keeps its kThrKeep largest values sorted in registers while the warp
// streams the values, then the warp takes the largest lane head j times (a
// max butterfly; the lowest lane holding it drops it).  No block barrier, no
// shared memory: the problem is a few thousand values per query.
constexpr int kThrThreads = 256;
constexpr int kThrKeep = 32;

// Streams `total` values (load(i); -inf marks an empty slot) through one
// warp: each lane keeps its KEEP largest sorted in registers (enough for
// the warp's j <= KEEP largest: no lane holds more than j of them).
// Returns the warp's count of non-empty values.
template <int KEEP, class Load>
__device__ __forceinline__ int warp_keep_largest(Load load, int total, float (&keep)[KEEP], int lane) {
#pragma unroll
    for (int s = 0; s < KEEP; ++s) keep[s] = -INFINITY;
    int valid = 0;
    for (int i0 = lane; i0 < total; i0 += 8 * 32) {
        float v[8];   // eight loads in flight per lane
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int i = i0 + 32 * k;
            v[k] = i < total ? load(i) : -INFINITY;
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            float x = v[k];
            if (!(x > -INFINITY)) continue;   // empty slot
            ++valid;
            if (x > keep[KEEP - 1]) {
#pragma unroll
                for (int s = 0; s < KEEP; ++s)
                    if (x > keep[s]) { const float t = keep[s]; keep[s] = x; x = t; }
            }
        }
    }
    return warp_reduce_sum_int(valid);
}

// Takes the warp's largest kept value n times (a max butterfly; the lowest
// lane holding it drops it); emit(r, m) receives the (r+1)-th largest, -inf
// once the kept values are used up.
template <int KEEP, class Emit>
__device__ __forceinline__ void warp_take_largest(float (&keep)[KEEP], int n, int lane, Emit emit) {
    for (int r = 0; r < n; ++r) {
        float m = keep[0];
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
        const unsigned who = __ballot_sync(0xffffffffu, keep[0] == m);
        if (lane == __ffs(who) - 1) {
#pragma unroll
            for (int s = 0; s < KEEP - 1; ++s) keep[s] = keep[s + 1];
            keep[KEEP - 1] = -INFINITY;
        }
        emit(r, m);
    }
}

// The j-th largest of query q's values for one warp (see threshold_kernel);
// j <= KEEP.
template <int KEEP>
__device__ float warp_threshold(const float* __restrict__ sample_buf, int32_t n_sample_tiles, int32_t B, int q,
                                int32_t j, int32_t per_tile, int lane) {
    float keep[KEEP];
    // L2 loads: other CTAs may have written the values
    const int valid = warp_keep_largest(
        [&](int i) { return __ldcg(sample_buf + ((int64_t)(i / per_tile) * B + q) * per_tile + (i % per_tile)); },
        n_sample_tiles * per_tile, keep, lane);
    float th = -INFINITY;
    if (valid >= j) warp_take_largest(keep, j, lane, [&](int, float m) { th = m; });
    return th;
}

template <int KEEP>   // j <= KEEP
__global__ void __launch_bounds__(kThrThreads)
threshold_kernel(const float* __restrict__ sample_buf, int32_t n_sample_tiles, int32_t B, int32_t j,
                 int32_t per_tile, float* __restrict__ theta) {
    const int q = (int)((blockIdx.x * (unsigned)blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (q >= B) return;
    const float th = warp_threshold<KEEP>(sample_buf, n_sample_tiles, B, q, j, per_tile, lane);
    if (lane == 0) theta[q] = th;
}

// Row shards, before the candidates pass: query q's kJ largest sampled
// values (descending, -inf past the valid ones) go to rec[q kJ, (q+1) kJ)
// and the shard's sampled rows, rows and mode (1: it takes the shared
// threshold) to rec[B kJ + 0, 1, 2] as int bits -- the record that one
// all-gather sends to every shard.  kJ >= every shard's own j, so the j-th
// largest of the shards' union is among their records.
static_assert(kShardJ == kJ, "the shard threshold record holds kJ values per query");
__global__ void __launch_bounds__(kThrThreads)
sample_record_kernel(const float* __restrict__ sample_buf, int32_t n_sample_tiles, int32_t B, int32_t per_tile,
                     int32_t sample_rows, int32_t rows, float* __restrict__ rec) {
    const int q = (int)((blockIdx.x * (unsigned)blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (q == 0 && lane == 0) {
        int32_t* h = reinterpret_cast<int32_t*>(rec + (int64_t)B * kJ);
        h[0] = sample_rows;
        h[1] = rows;
        h[2] = 1;
    }
    if (q >= B) return;
    float keep[kJ];
    warp_keep_largest(
        [&](int i) { return __ldcg(sample_buf + ((int64_t)(i / per_tile) * B + q) * per_tile + (i % per_tile)); },
        n_sample_tiles * per_tile, keep, lane);
    warp_take_largest(keep, kJ, lane, [&](int r, float m) { if (lane == 0) rec[(int64_t)q * kJ + r] = m; });
}

// Row shards: query q's threshold from every shard's record (rank-major,
// `stride` floats each).  Over the shards of mode 1, mu = K x (sampled rows)
// / (rows) and j = ceil(mu + 5 sqrt(mu) + 3) -- one store's rule applied to
// the union of the samples -- and theta = the j-th largest of their values
// (-inf when fewer exist).  Every shard computes the same value from the
// same records.
__global__ void __launch_bounds__(kThrThreads)
union_threshold_kernel(const float* __restrict__ recs, int32_t world, int32_t stride, int32_t B, int32_t K,
                       float* __restrict__ theta) {
    const int q = (int)((blockIdx.x * (unsigned)blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (q >= B) return;
    long long srows = 0, rows = 0;
    for (int r = 0; r < world; ++r) {
        const int32_t* h = reinterpret_cast<const int32_t*>(recs + (int64_t)r * stride + (int64_t)B * kJ);
        if (__ldcg(h + 2) == 1) { srows += __ldcg(h + 0); rows += __ldcg(h + 1); }
    }
    const double mu = rows > 0 ? (double)K * (double)srows / (double)rows : 0.0;
    const int j = max(1, min(kJ, (int)ceil(mu + 5.0 * sqrt(mu) + 3.0)));
    float keep[kJ];
    const int valid = warp_keep_largest(
        [&](int i) {
            const int r = i / kJ;
            const float* rec = recs + (int64_t)r * stride;
            const int32_t mode = __ldcg(reinterpret_cast<const int32_t*>(rec + (int64_t)B * kJ) + 2);
            return mode == 1 ? __ldcg(rec + (int64_t)q * kJ + (i - r * kJ)) : -INFINITY;
        },
        world * kJ, keep, lane);
    float th = -INFINITY;
    if (valid >= j) warp_take_largest(keep, j, lane, [&](int, float m) { th = m; });
    if (lane == 0) theta[q] = th;
}

// Neutral shard records, for a shard whose call does not reach an exchange
// with data of its own: no sampled values, mode 0 (threshold record);
// counts 0, bounds -inf and the failure flag (bound record).
__global__ void neutral_thr_kernel(float* __restrict__ rec, int32_t B) {
    const int64_t n = (int64_t)B * kJ;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n + 3; i += (int64_t)gridDim.x * blockDim.x)
        rec[i] = i < n ? -INFINITY : 0.0f;   // 0.0f: the int 0 as bits
}

__global__ void neutral_rec_kernel(float* __restrict__ rec, int32_t B, float failed) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i <= 3 * (int64_t)B;
         i += (int64_t)gridDim.x * blockDim.x)
        rec[i] = i < B ? 0.0f : (i < 3 * (int64_t)B ? -INFINITY : failed);
}

// Exact rescoring of candidates: one block per query.
//
// Every candidate c carries its approximate score f_c; with the row weight w_c
// and the query margin m its exact score lies in [lo_c, hi_c] =
// [f_c - m|w_c|, f_c + m|w_c|].
//  * Completeness: if at least K candidates have lo_c >= theta, K rows score
//    >= theta exactly, so every row of the true top-K scores >= theta and --
//    its upper bound being at least its exact score -- was short-listed.
//    Otherwise (or on overflow) the query is flagged for the exact scan.
//  * Pruning: with theta2 the K-th largest lo_c, a candidate with
//    hi_c < theta2 cannot enter the top-K, so only candidates with
//    hi_c >= theta2 are rescored exactly (typically K plus a few).
//  * Row shards (the record layout is kShardRec*): pass 1 (bound_out) writes
//    this shard's record and stops: the count of candidates with
//    lo_c >= theta, the K-th largest lo_c (theta2) and the m-th largest lo_c
//    (m = ceil(K / world); -inf where fewer exist).  With a threshold shared
//    by every shard (shard_global) the counts add up: K candidates over all
//    shards with lo_c >= theta certify every shard's short list; with this
//    shard's own threshold its own count must reach K.  Pass 2 (bound_in,
//    every shard's record) prunes with the largest of theta (once certified),
//    every shard's theta2 (K rows of that shard score at least that much) and
//    the smallest m-th bound (each of `world` shards has m rows above its
//    own, world x m >= K rows in all): each is a lower bound of the global
//    K-th score, so only rows that can still enter the global top-K are
//    rescored (about K / world + a few per shard).
// Both selections are block-wide bitonic sorts in shared memory ranked by
// rank key (score desc, id asc; -0 below +0, as the fp32 scan ranks).
constexpr int kSortCap = 4096;
constexpr int kRescoreThreads = 256;

__device__ __forceinline__ void block_bitonic_desc(float* key, int32_t* id, int n) {
    for (int k = 2; k <= n; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < n; i += kRescoreThreads) {
                const int p = i ^ j;
                if (p > i) {
                    const float a = key[i], b = key[p];
                    const int32_t ia = id[i], ib = id[p];
                    // rank-key order (the fp32 scan's): with -0 below +0, so
                    // the lists are sorted as their packed keys
                    const bool a_first = rank_key(a, ia) > rank_key(b, ib);
                    const bool desc = (i & k) == 0;
                    if (desc != a_first) {
                        key[i] = b; key[p] = a;
                        id[i] = ib; id[p] = ia;
                    }
                }
            }
            __syncthreads();
        }
    }
}

__device__ __forceinline__ int pow2_at_least(int n) {
    int p = 32;
    while (p < n) p <<= 1;
    return p;
}

// Rank by counting over at most this many lower bounds (shard pass 1):
// every order statistic from one sweep, cheaper than radix passes.
constexpr int kCountCap = 256;
// ... and over at most this many rescored rows (their final order; the rank
// keys fit the histogram's 8 KB).
constexpr int kCountSortCap = 512;
// Rows each rescoring warp keeps requested ahead of the one it scores.
constexpr int kRescoreAhead = 4;
// Batches of at least this many queries take their final rescore pass in
// three kernels (rows listed / scored / ranked), smaller ones in one.
constexpr int kSplitRescoreMinB = 256;

__global__ void __launch_bounds__(kRescoreThreads, 3)
rescore_kernel(StoreView s, const float* __restrict__ Q, int64_t qpitch, int32_t B, float t_q,
               float lambda, int32_t use_imp, int32_t K, int32_t row_offset,
               const float* __restrict__ theta, const float* __restrict__ margin,
               int4* __restrict__ cand, const int32_t* __restrict__ cand_cnt, int32_t cap,
               int32_t* __restrict__ out_ids, float* __restrict__ out_vals,
               int32_t* __restrict__ out_cnt, int32_t* __restrict__ fallback,
               int32_t* __restrict__ rescored, const int32_t* __restrict__ bad,
               const int32_t* __restrict__ status, float* __restrict__ bound_out,
               const float* __restrict__ bound_in, int32_t shard_world, int32_t shard_global,
               int32_t* __restrict__ status_mirror, int32_t max_batch, int32_t split) {
    // The call's status words, [err, sync_err, fallback[], cand_cnt[],
    // rescored[], bad[]] (max_batch each), also go straight to the caller's
    // host-mapped mirror by the final pass (status_mirror != NULL), so no
    // device-to-host copy follows the call: block qi publishes its query's
    // words on its way out, block 0 the two error words.
    auto publish = [&](int32_t fb, int32_t resc) {
        if (status_mirror == nullptr || threadIdx.x != 0) return;
        if (blockIdx.x == 0) { status_mirror[0] = status[0]; status_mirror[1] = status[1]; }
        status_mirror[2 + blockIdx.x] = fb;
        status_mirror[2 + max_batch + blockIdx.x] = cand_cnt[blockIdx.x];
        status_mirror[2 + 2 * max_batch + blockIdx.x] = resc;
        status_mirror[2 + 3 * max_batch + blockIdx.x] = bad != nullptr ? bad[blockIdx.x] : 0;
    };
    __shared__ float   s_key[kSortCap];
    __shared__ int32_t s_id[kSortCap];
    __shared__ int     s_ge, s_n2, s_nk;
    __shared__ float   s_wv[kRescoreThreads];      // K <= 32: each warp's K best lower bounds
    __shared__ int32_t s_wi[kRescoreThreads];
    __shared__ float   s_th2, s_mth;
    __shared__ __align__(16) int s_hist[2048];   // also read as 64-bit keys
    __shared__ uint32_t s_sel[2];
    const int qi = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int kWarps = kRescoreThreads / 32;
    const bool call_failed = status[0] != 0 || status[1] != 0;
    const bool shard_pass1 = bound_out != nullptr;
    if (shard_pass1 && threadIdx.x == 0) {
        // this shard's record, neutral until pass 1 fills it in
        reinterpret_cast<int32_t*>(bound_out)[qi] = 0;
        bound_out[B + qi] = -INFINITY;
        bound_out[2 * B + qi] = -INFINITY;
        // the flag: 1 when this shard's call failed (no result is served)
        if (qi == 0) bound_out[3 * B] = call_failed ? 1.0f : 0.0f;
    }
    if (call_failed) {
        // a bounded wait of this call's GEMM gave up: the short lists and the
        // thresholds may be incomplete, so no result of the call is served
        for (int p = threadIdx.x; p < K; p += kRescoreThreads) {
            out_vals[(int64_t)qi * K + p] = -INFINITY;
            out_ids[(int64_t)qi * K + p] = -1;
        }
        if (threadIdx.x == 0) { if (out_cnt) out_cnt[qi] = -1; fallback[qi] = 0; rescored[qi] = 0; }
        if (!shard_pass1) publish(0, 0);
        return;
    }
    const int ncand = cand_cnt[qi];
    const int nc_ = min(ncand, cap);
    if (threadIdx.x == 0) { s_ge = 0; s_n2 = 0; }
    __syncthreads();
    // Too many candidates to sort here, or a query outside the fp16 range
    // (its short list is meaningless): the exact scan answers it.  Fewer
    // than K candidates only rule out a threshold of this shard's own; with
    // a shared one the count over all shards decides.
    const bool unsortable = ncand > kSortCap || (bad != nullptr && bad[qi] != 0);
    if (unsortable || (nc_ < K && shard_global == 0)) {
        if (shard_pass1) return;   // the record stays neutral
        if (threadIdx.x == 0) { fallback[qi] = 1; rescored[qi] = 0; if (out_cnt) out_cnt[qi] = 0; }
        publish(1, 0);
        return;
    }
    const float th = theta[qi];
    // candidate i: row .x, approximate score .y and slack .z (float bits);
    // the exact score lies in score -+ slack
    int4* cq = cand + (int64_t)qi * cap;

    // ---- pass 1: lower bounds, completeness, K-th largest lower bound -------
    // Unsharded, K <= 32: every warp keeps its K best lower bounds (ranked by
    // value, then candidate index) and warp 0 merges the eight lists; larger
    // K: a radix selection over all of them.  Either way th2 is the K-th
    // largest.  Shard pass 1 writes the record; shard pass 2 takes its
    // bound from every shard's record, so only the count runs here.
    const bool need_th2 = bound_in == nullptr && !shard_pass1;
    const bool warp_lists = need_th2 && K <= 32;
    WarpTopK<1> top;
    top.init(warp_lists ? K : 1);
    int ge = 0;
    for (int i0 = warp * 32; i0 < nc_; i0 += kRescoreThreads) {
        const int i = i0 + lane;
        const bool in = i < nc_;
        float lo = -INFINITY;
        if (in) {
            const int4 e = __ldcg(cq + i);
            lo = __int_as_float(e.y) - __int_as_float(e.z);
        }
        ge += (in && lo >= th) ? 1 : 0;
        if (warp_lists) top.offer_lanes(lo, i, in, lane);
        else if ((need_th2 || shard_pass1) && in) s_key[i] = lo;
    }
    ge = warp_reduce_sum_int(ge);
    if (lane == 0) atomicAdd(&s_ge, ge);
    if (warp_lists) top.store(s_wv + warp * 32, s_wi + warp * 32, lane);
    __syncthreads();
    if (shard_pass1) {
        // the K-th and the m-th largest lower bounds of this shard
        const int m = (K + shard_world - 1) / shard_world;
        float kth = -INFINITY, mth = -INFINITY;
        if (nc_ <= kCountCap) {
            // candidate i's rank = the lower bounds above it (ties by index)
            if (threadIdx.x == 0) { s_th2 = -INFINITY; s_mth = -INFINITY; }
            __syncthreads();
            for (int i = threadIdx.x; i < nc_; i += kRescoreThreads) {
                const float v = s_key[i];
                int r = 0;
                for (int t = 0; t < nc_; ++t) {
                    const float u = s_key[t];
                    r += (u > v || (u == v && t < i)) ? 1 : 0;
                }
                if (r == K - 1) s_th2 = v;
                if (r == m - 1) s_mth = v;
            }
            __syncthreads();
            kth = s_th2;
            mth = s_mth;
        } else {
            auto key = [&](int i) { return f2key(s_key[i]); };
            if (nc_ >= K) kth = key2f(block_kth_largest_key<kRescoreThreads>(key, nc_, K, s_hist, s_sel));
            mth = m == K ? kth : key2f(block_kth_largest_key<kRescoreThreads>(key, nc_, m, s_hist, s_sel));
        }
        if (threadIdx.x == 0) {
            reinterpret_cast<int32_t*>(bound_out)[qi] = shard_global ? s_ge : 0;
            bound_out[B + qi] = kth;
            bound_out[2 * B + qi] = mth;
        }
        return;
    }
    float th2;
    bool certified;
    if (bound_in != nullptr) {
        // every shard's record (rank-major): the completeness count and the
        // pruning bound, the same on every shard
        long long total = 0;
        float best = -INFINITY, mmin = INFINITY;
        const int64_t stride = 3 * (int64_t)B + 1;
        for (int r = 0; r < shard_world; ++r) {
            const float* rec = bound_in + r * stride;
            total += __ldcg(reinterpret_cast<const int32_t*>(rec) + qi);
            best = fmaxf(best, __ldcg(rec + B + qi));
            mmin = fminf(mmin, __ldcg(rec + 2 * B + qi));
        }
        certified = shard_global ? total >= K : s_ge >= K;
        th2 = fmaxf(fmaxf(best, mmin), th);
    } else {
        certified = s_ge >= K;
    }
    if (!certified) {
        if (threadIdx.x == 0) { fallback[qi] = 1; rescored[qi] = 0; if (out_cnt) out_cnt[qi] = 0; }
        publish(1, 0);
        return;
    }
    if (bound_in == nullptr) {
        if (warp_lists) {
            if (warp == 0) {
                for (int ww = 1; ww < kWarps; ++ww) top.merge_sorted32(s_wv + ww * 32, s_wi + ww * 32, K, lane);
                if (lane == 0) s_th2 = top.thr_v;
            }
            __syncthreads();
            th2 = s_th2;
        } else {
            th2 = key2f(block_kth_largest_key<kRescoreThreads>(
                [&](int i) { return f2key(s_key[i]); }, nc_, K, s_hist, s_sel));
        }
    }

    // ---- pass 2: exact scores of the candidates that can still place -------
    // Their rows are listed first (in the histogram's space, free now) and
    // dealt to the warps in turn, one row per warp at a time.
    const float4* q4 = reinterpret_cast<const float4*>(Q + (int64_t)qi * qpitch);
    const bool use_w = use_imp != 0 && s.imp != nullptr;
    int32_t* s_rows = s_hist;
    constexpr int kRowsCap = 2048;
    if (threadIdx.x == 0) s_nk = 0;
    __syncthreads();
    for (int i0 = warp * 32; i0 < nc_; i0 += kWarps * 32) {
        const int i = i0 + lane;
        int32_t r = 0;
        bool keep = false;
        if (i < nc_) {
            const int4 e = __ldcg(cq + i);
            r = e.x;
            keep = __int_as_float(e.y) + __int_as_float(e.z) >= th2;
        }
        const unsigned mk = __ballot_sync(0xffffffffu, keep);
        int base = 0;
        if (lane == 0 && mk != 0u) base = atomicAdd(&s_nk, __popc(mk));
        base = __shfl_sync(0xffffffffu, base, 0);
        const int pos = base + __popc(mk & ((1u << lane) - 1u));
        if (keep && pos < kRowsCap) s_rows[pos] = r;
    }
    __syncthreads();
    const int nk = min(s_nk, kRowsCap);
    if (split != 0) {
        // split rescore (large batches): the rows go back to the front of
        // this query's candidate list (every read of it is done) for
        // rescore_rows_kernel; a longer row list than this block's is
        // answered by the exact scan instead
        if (s_nk > kRowsCap) {
            if (threadIdx.x == 0) { fallback[qi] = 1; rescored[qi] = 0; if (out_cnt) out_cnt[qi] = 0; }
            return;
        }
        for (int t = threadIdx.x; t < nk; t += kRescoreThreads) cq[t].x = s_rows[t];
        if (threadIdx.x == 0) { fallback[qi] = 0; rescored[qi] = nk; }
        return;
    }
    // each warp requests its next four rows into L2 (one bulk prefetch each)
    // while it scores the current one: five of its rows travel at a time
    // instead of one, and L2 holds only rows about to be read
    const uint32_t row_bytes = (uint32_t)s.nc * 16u;
    auto prefetch_row = [&](int t) {
        if (lane == 0 && t < nk)
            prefetch_l2_bulk(reinterpret_cast<const float4*>(s.E) + (int64_t)s_rows[t] * s.pitch4, row_bytes);
    };
    auto score_row = [&](int32_t rr) {
        const float4* row = reinterpret_cast<const float4*>(s.E) + (int64_t)rr * s.pitch4;
        const float dot = warp_dot_canonical(row, q4, s.nc, lane);
        float f = fused_weight_apply(dot, __ldg(s.ts + rr), t_q, lambda);
        if (use_w) f = f * __ldg(s.imp + rr);
        if (lane == 0) {
            const int pos = atomicAdd(&s_n2, 1);
            s_key[pos] = f;
            s_id[pos] = rr + row_offset;
        }
    };
    for (int d = 1; d < kRescoreAhead; ++d) prefetch_row(warp + d * kWarps);
    for (int t = warp; t < nk; t += kWarps) {
        prefetch_row(t + kRescoreAhead * kWarps);
        score_row(s_rows[t]);
    }
    if (s_nk > kRowsCap) {
        // more rows than the list holds: the rest in candidate order
        __syncthreads();
        for (int i0 = warp * 32; i0 < nc_; i0 += kWarps * 32) {
            const int i = i0 + lane;
            int32_t r = 0;
            bool keep = false;
            if (i < nc_) {
                const int4 e = __ldcg(cq + i);
                r = e.x;
                keep = __int_as_float(e.y) + __int_as_float(e.z) >= th2;
            }
            // the first kRowsCap kept rows (in list order) are done; ranks are
            // not known here, so every kept row not in the list is scored by
            // membership test against the list
            unsigned mk = __ballot_sync(0xffffffffu, keep);
            while (mk) {
                const int src = __ffs(mk) - 1;
                mk &= mk - 1;
                const int32_t rr = __shfl_sync(0xffffffffu, r, src);
                bool listed = false;
                for (int t = lane; t < kRowsCap && !listed; t += 32) listed = s_rows[t] == rr;
                if (__any_sync(0xffffffffu, listed)) continue;
                score_row(rr);
            }
        }
    }
    __syncthreads();
    const int n2 = s_n2;
    if (n2 <= 32) {
        // few rows: ranked in warp 0's registers (score desc, id asc)
        unsigned long long* keys = reinterpret_cast<unsigned long long*>(s_hist);   // the row list is done
        if (threadIdx.x < 32) keys[threadIdx.x] = threadIdx.x < n2 ? rank_key(s_key[threadIdx.x], s_id[threadIdx.x]) : 0ull;
        __syncthreads();
        warp0_sort32_desc(keys, n2);
        for (int p = threadIdx.x; p < n2; p += kRescoreThreads) {
            s_key[p] = key_score(keys[p]);
            s_id[p] = key_id(keys[p]);
        }
        __syncthreads();
    } else if (n2 <= kCountSortCap) {
        // a few hundred rows: each row's place is the number of rank keys
        // above its own (keys are unique), so the first K go straight to the
        // output -- one pass and one barrier instead of a bitonic network
        unsigned long long* keys = reinterpret_cast<unsigned long long*>(s_hist);   // the row list is done
        for (int p = threadIdx.x; p < n2; p += kRescoreThreads) keys[p] = rank_key(s_key[p], s_id[p]);
        __syncthreads();
        for (int i = threadIdx.x; i < n2; i += kRescoreThreads) {
            const unsigned long long k = keys[i];
            int r = 0;
            for (int t = 0; t < n2; ++t) r += keys[t] > k ? 1 : 0;
            if (r < K) {
                out_vals[(int64_t)qi * K + r] = key_score(k);
                out_ids[(int64_t)qi * K + r] = key_id(k);
            }
        }
    } else {
        const int p2 = pow2_at_least(n2);
        for (int i = n2 + threadIdx.x; i < p2; i += kRescoreThreads) { s_key[i] = -INFINITY; s_id[i] = INT32_MAX; }
        __syncthreads();
        block_bitonic_desc(s_key, s_id, p2);
    }
    const bool ranked_out = n2 > 32 && n2 <= kCountSortCap;   // written above
    for (int p = ranked_out ? n2 + threadIdx.x : threadIdx.x; p < K; p += kRescoreThreads) {
        const bool valid = p < n2;
        out_vals[(int64_t)qi * K + p] = valid ? s_key[p] : -INFINITY;
        out_ids[(int64_t)qi * K + p] = valid ? s_id[p] : -1;
    }
    if (threadIdx.x == 0) {
        if (out_cnt) out_cnt[qi] = min(n2, K);
        fallback[qi] = 0;
        rescored[qi] = n2;
    }
    publish(0, n2);
}

// Split rescore of large batches, after rescore_kernel listed each query's
// rows (split = 1): the rows' exact scores with nothing else in the kernel --
// the query in 3 KB of shared memory, the row alone in registers -- so six
// 256-thread blocks fit an SM and about twice as many rows travel at once as
// in the one-kernel form, whose selection arrays allow three blocks per SM.  Warp w of block q takes
// rows w, w + 8, ... of query q, each warp keeping its next rows requested
// into L2; the score (the canonical dot, the same arithmetic as the fp32
// scan) replaces the approximate one in the row's record.
template <int C>   // float4 chunks per lane and row: D <= 128 C
__global__ void __launch_bounds__(kRescoreThreads, 6)
rescore_rows_kernel(StoreView s, const float* __restrict__ Q, int64_t qpitch, float t_q, float lambda,
                    int32_t use_imp, int4* __restrict__ cand, int32_t cap, const int32_t* __restrict__ rescored,
                    const int32_t* __restrict__ fallback, const int32_t* __restrict__ status) {
    __shared__ float4 s_q[32 * C];
    const int qi = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int kWarps = kRescoreThreads / 32;
    if (status[0] != 0 || status[1] != 0 || fallback[qi] != 0) return;
    const int nk = rescored[qi];
    const float4* q4 = reinterpret_cast<const float4*>(Q + (int64_t)qi * qpitch);
    for (int i = threadIdx.x; i < s.nc; i += kRescoreThreads) s_q[i] = q4[i];
    __syncthreads();
    int4* cq = cand + (int64_t)qi * cap;
    const bool use_w = use_imp != 0 && s.imp != nullptr;
    const float4* E4 = reinterpret_cast<const float4*>(s.E);
    const uint32_t row_bytes = (uint32_t)s.nc * 16u;
    auto prefetch_row = [&](int t) {
        if (lane == 0 && t < nk) prefetch_l2_bulk(E4 + (int64_t)__ldcg(&cq[t].x) * s.pitch4, row_bytes);
    };
    for (int d = 1; d < kRescoreAhead; ++d) prefetch_row(warp + d * kWarps);
    for (int t = warp; t < nk; t += kWarps) {
        prefetch_row(t + kRescoreAhead * kWarps);
        const int32_t rr = __ldcg(&cq[t].x);
        const float dot = warp_dot_canonical_smemq<C>(E4 + (int64_t)rr * s.pitch4, s_q, s.nc, lane);
        float f = fused_weight_apply(dot, __ldg(s.ts + rr), t_q, lambda);
        if (use_w) f = f * __ldg(s.imp + rr);
        if (lane == 0) cq[t].y = __float_as_int(f);
    }
}

// Split rescore, last step: each query's rescored rows ranked by rank key
// (score desc, id asc) into the outputs, and the call's status words
// published (as rescore_kernel's final pass does).
__global__ void __launch_bounds__(kRescoreThreads)
rescore_rank_kernel(int32_t K, int32_t row_offset, const int4* __restrict__ cand, int32_t cap,
                    int32_t* __restrict__ out_ids, float* __restrict__ out_vals, int32_t* __restrict__ out_cnt,
                    const int32_t* __restrict__ fallback, const int32_t* __restrict__ rescored,
                    const int32_t* __restrict__ cand_cnt, const int32_t* __restrict__ bad,
                    const int32_t* __restrict__ status, int32_t* __restrict__ status_mirror, int32_t max_batch) {
    __shared__ __align__(16) unsigned long long s_keys[kSortCap / 2];
    __shared__ float s_key[kSortCap / 2];
    __shared__ int32_t s_id[kSortCap / 2];
    const int qi = blockIdx.x;
    auto publish = [&](int32_t fb, int32_t resc) {
        if (status_mirror == nullptr || threadIdx.x != 0) return;
        if (blockIdx.x == 0) { status_mirror[0] = status[0]; status_mirror[1] = status[1]; }
        status_mirror[2 + blockIdx.x] = fb;
        status_mirror[2 + max_batch + blockIdx.x] = cand_cnt[blockIdx.x];
        status_mirror[2 + 2 * max_batch + blockIdx.x] = resc;
        status_mirror[2 + 3 * max_batch + blockIdx.x] = bad != nullptr ? bad[blockIdx.x] : 0;
    };
    if (status[0] != 0 || status[1] != 0) { publish(0, 0); return; }   // outputs already marked invalid
    if (fallback[qi] != 0) { publish(1, 0); return; }                   // answered by the exact scan
    const int n2 = rescored[qi];
    const int4* cq = cand + (int64_t)qi * cap;
    if (n2 <= kCountSortCap) {
        for (int p = threadIdx.x; p < n2; p += kRescoreThreads) {
            const int4 e = __ldcg(cq + p);
            s_keys[p] = rank_key(__int_as_float(e.y), e.x + row_offset);
        }
        __syncthreads();
        for (int i = threadIdx.x; i < n2; i += kRescoreThreads) {
            const unsigned long long k = s_keys[i];
            int r = 0;
            for (int t = 0; t < n2; ++t) r += s_keys[t] > k ? 1 : 0;
            if (r < K) {
                out_vals[(int64_t)qi * K + r] = key_score(k);
                out_ids[(int64_t)qi * K + r] = key_id(k);
            }
        }
    } else {
        const int p2 = pow2_at_least(n2);
        for (int p = threadIdx.x; p < p2; p += kRescoreThreads) {
            if (p < n2) {
                const int4 e = __ldcg(cq + p);
                s_key[p] = __int_as_float(e.y);
                s_id[p] = e.x + row_offset;
            } else {
                s_key[p] = -INFINITY;
                s_id[p] = INT32_MAX;
            }
        }
        __syncthreads();
        block_bitonic_desc(s_key, s_id, p2);
        for (int p = threadIdx.x; p < min(n2, K); p += kRescoreThreads) {
            out_vals[(int64_t)qi * K + p] = s_key[p];
            out_ids[(int64_t)qi * K + p] = s_id[p];
        }
    }
    for (int p = n2 + threadIdx.x; p < K; p += kRescoreThreads) {
        out_vals[(int64_t)qi * K + p] = -INFINITY;
        out_ids[(int64_t)qi * K + p] = -1;
    }
    if (threadIdx.x == 0 && out_cnt) out_cnt[qi] = min(n2, K);
    publish(0, n2);
}

// ---------------------------------------------------------------------------
// Small batches (B <= kSmallMaxB queries, fp16 operands): the roles of the
// operands swap.  A tile is 128 rows (UMMA M) x NQ queries (UMMA N = B
// rounded up to 16), so the tensor cores do no work for absent queries, the
// queries' fp16 k-blocks stay in shared memory for the whole kernel (loaded
// once), and the rest of shared memory is a ring of row stages (16 KB each,
// up to kSmallMaxStages) -- more row bytes in flight per SM than the
// 128 x 256 tile's ring, whose stages also carry a 128-row query tile.
// TMEM holds D[row][query] (lanes = rows, columns = queries), double
// buffered; epilogue thread t owns row t of the tile.
//
// Candidates mode appends (query, row) when the row's upper bound reaches the
// query's threshold, as gemm_kernel does.  Sample mode writes, per sampled
// tile and query, the tile's largest lower bound (of its 128 rows), or each
// epilogue warp's (of its 32 rows) when the sample has few tiles:
// sample_buf[tile][query][1 or kSmallWarps].  The j-th largest of these is at
// most the j-th largest sampled bound (j of them are the maxima of j
// distinct row sets), so the threshold stays as safe.
constexpr int kSmallMaxB = 64;
constexpr int kSmallRows = 128;
constexpr int kSmallStage = kSmallRows * 128;      // 16 KB: 128 rows x 64 halves
constexpr int kSmallMaxStages = 12;
constexpr int kSmallWarps = 4;                       // TMEM lane quarters: 32 rows each
// producer, MMA and 8 epilogue warps: two per lane quarter, taking
// alternate 16-query column chunks (with one per quarter the epilogue paced
// the launch at 48-64 queries)
constexpr int kSmallThreads = 320;
constexpr int kSmallEpi = kSmallThreads - 64;
constexpr int kSmallStaticSmem = 6144;               // bound on the kernel's static shared memory
constexpr int kStageCand = 256;                      // candidates staged in shared memory per CTA
// Accumulator buffers in TMEM (as many as 512 columns hold, up to this many):
// the MMAs run this many tiles ahead of the epilogue, which covers the
// fused launch's wait for every CTA's sample tile and its thresholds.
constexpr int kSmallAccBufs = 8;

struct SmallArgs {
    int32_t B, NQ;                   // queries, MMA N (B rounded up to 16)
    int32_t n, nkb;                  // rows, 64-half k-blocks
    int32_t n_tiles;                 // 128-row tiles of this launch
    int32_t stages;                  // row stages in the ring
    uint32_t tmem_cols;              // columns allocated (power of two >= nbuf NQ, >= 32)
    int32_t nbuf;                    // accumulator buffers in TMEM (2 .. kSmallAccBufs)
    const int32_t* sample_rt;        // sample mode: 128-row tile of sample tile i
    RowMeta meta;
    const float* theta;
    const float* margin;
    float* sample_buf;               // sample mode: [n_tiles][B][sample_per_tile] maxima
    int4* cand;                      // [B][cap] candidates (cand_entry)
    int32_t* cand_cnt;
    int32_t cap;
    int32_t self_base;
    int* err;
    // kFused: CTA b < n_sample first runs sample tile sample_rt[b]; after
    // every CTA's sample maxima are written (grid counter), each CTA takes
    // the thresholds itself; CTA 0 also stores them in theta_out
    int32_t n_sample, j;
    int32_t sample_per_tile;         // values per sampled tile and query: 1 (the tile's
                                     // maximum) or kSmallWarps (each epilogue warp's)
    unsigned long long* grid_sync;   // monotone arrival counter
    unsigned long long sync_target;  // its value once every CTA of this launch arrived
    uint32_t sync_spin_limit;        // polls of the arrival wait before it gives up
    int* sync_err;                   // set (17) when the arrival wait gave up
    float* theta_out;
};

// The it-th tile of this CTA: first row, sample or candidates, and (sample)
// its index in sample_buf; false past the CTA's last tile.  kFused: the
// CTA's sample tile (if it has one), then its candidate tiles.
struct SmallTile {
    int row0;
    bool sample;
    int sidx;
};
template <int MODE>
__device__ __forceinline__ bool small_tile(const SmallArgs& a, int it, SmallTile& tl) {
    if (MODE == kFused) {
        const int hs = (int)blockIdx.x < a.n_sample ? 1 : 0;
        if (it < hs) {
            tl.row0 = a.sample_rt[blockIdx.x] * kSmallRows;
            tl.sample = true;
            tl.sidx = blockIdx.x;
            return true;
        }
        const int t = blockIdx.x + (it - hs) * gridDim.x;
        if (t >= a.n_tiles) return false;
        tl.row0 = t * kSmallRows;
        tl.sample = false;
        tl.sidx = 0;
        return true;
    }
    const int t = blockIdx.x + it * gridDim.x;
    if (t >= a.n_tiles) return false;
    tl.row0 = (MODE == kSample ? a.sample_rt[t] : t) * kSmallRows;
    tl.sample = MODE == kSample;
    tl.sidx = t;
    return true;
}

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__host__ __device__ constexpr size_t small_smem_bytes(int nkb, int NQ, int stages) {
    return 1024 /*align*/ + (size_t)nkb * NQ * 128 + (size_t)stages * kSmallStage + 512 /*barriers*/;
}

template <int MODE>
__global__ void __launch_bounds__(kSmallThreads, 1)
gemm_small_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_e,
                  const SmallArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int qkb_bytes = a.NQ * 128;                          // one query k-block
    uint8_t* qs = smem;                                        // nkb query k-blocks
    uint8_t* rs = smem + (size_t)a.nkb * qkb_bytes;            // row stages
    uint64_t* full = reinterpret_cast<uint64_t*>(rs + (size_t)a.stages * kSmallStage);
    uint64_t* empty = full + kSmallMaxStages;
    uint64_t* qfull = empty + kSmallMaxStages;
    uint64_t* tfull = qfull + 1;
    uint64_t* tempty = tfull + kSmallAccBufs;
    uint64_t* mdrain = tempty + kSmallAccBufs;      // the MMA issuer's last commit
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mdrain + 1);

    // this launch's thresholds (kFused: after the grid wait) and the queries'
    // error margins; past B: +inf and 0, so those columns never pass
    __shared__ __align__(16) float s_theta[kSmallMaxB];
    __shared__ __align__(16) float s_mg[kSmallMaxB];
    __shared__ float s_wmax[kSmallWarps][kSmallMaxB];   // sample tile: each epilogue warp's maxima
    // candidates of the candidate tiles, staged in shared memory (a shared
    // atomic each) and written out in groups with ONE global atomic per
    // query: a global atomic per candidate is a dependent round trip
    __shared__ int s_ccnt;
    __shared__ int16_t s_cq[kStageCand];
    __shared__ int32_t s_crow[kStageCand];
    __shared__ float s_cf[kStageCand], s_cs[kStageCand];
    __shared__ int s_qn[kSmallMaxB], s_qbase[kSmallMaxB];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < a.stages; ++s) { sm100::mbar_init(full + s, 1); sm100::mbar_init(empty + s, 1); }
        sm100::mbar_init(qfull, 1);
        for (int b = 0; b < a.nbuf; ++b) { sm100::mbar_init(tfull + b, 1); sm100::mbar_init(tempty + b, kSmallEpi); }
        sm100::mbar_init(mdrain, 1);
        sm100::fence_mbar_init();
        sm100::prefetch_tmap(&tmap_q);
        sm100::prefetch_tmap(&tmap_e);
    }
    if (warp == 1) {
        sm100::tmem_alloc(tmem_slot, a.tmem_cols);
        sm100::tmem_relinquish();
    }
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            // the queries, once
            sm100::mbar_arrive_expect_tx(qfull, (uint32_t)(a.nkb * qkb_bytes));
            for (int kb = 0; kb < a.nkb; ++kb)
                sm100::tma_load_2d(qs + (size_t)kb * qkb_bytes, &tmap_q, qfull, kb * 64, 0);
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued_phase[kSmallMaxStages];
            bool issued[kSmallMaxStages];
            for (int s = 0; s < kSmallMaxStages; ++s) { issued[s] = false; issued_phase[s] = 0; }
            bool ok = true;
            SmallTile tl;
            for (int it = 0; ok && small_tile<MODE>(a, it, tl); ++it) {
                const int row0 = tl.row0;
                for (int kb = 0; kb < a.nkb; ++kb) {
                    if (!sm100::mbar_wait(empty + stage, phase ^ 1u, a.err, 11)) { ok = false; break; }
                    sm100::mbar_arrive_expect_tx(full + stage, kSmallStage);
                    sm100::tma_load_2d(rs + (size_t)stage * kSmallStage, &tmap_e, full + stage, kb * 64, row0);
                    issued[stage] = true;
                    issued_phase[stage] = phase;
                    if (++stage == a.stages) { stage = 0; phase ^= 1u; }
                }
            }
            // every copy this thread started has landed before the CTA may exit
            // (also after a wait gave up: the drain does not stop at the error word)
            sm100::mbar_wait_drain(qfull, 0, a.err, 12);
            for (int s = 0; s < a.stages; ++s)
                if (issued[s]) sm100::mbar_wait_drain(full + s, issued_phase[s], a.err, 12);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = sm100::idesc_f16(kSmallRows, a.NQ);
            bool ok = sm100::mbar_wait(qfull, 0, a.err, 13);
            sm100::tc_fence_after();
            const uint32_t qs_addr = sm100::smem_u32(qs);
            int stage = 0;
            uint32_t phase = 0;
            int buf = 0;
            uint32_t bphase = 0;
            SmallTile tl;
            for (int it = 0; ok && small_tile<MODE>(a, it, tl); ++it) {
                if (!sm100::mbar_wait(tempty + buf, bphase ^ 1u, a.err, 14)) break;
                sm100::tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(buf * a.NQ);
                for (int kb = 0; kb < a.nkb; ++kb) {
                    if (!sm100::mbar_wait(full + stage, phase, a.err, 15)) { ok = false; break; }
                    sm100::tc_fence_after();
                    const uint64_t da = sm100::smem_desc_sw128(sm100::smem_u32(rs + (size_t)stage * kSmallStage));
                    const uint64_t db = sm100::smem_desc_sw128(qs_addr + (uint32_t)(kb * qkb_bytes));
#pragma unroll
                    for (int k = 0; k < 4; ++k)      // 32 bytes of K (16 halves) per MMA
                        sm100::mma_f16(d, da + (uint64_t)(2 * k), db + (uint64_t)(2 * k), idesc,
                                       (kb > 0 || k > 0) ? 1u : 0u);
                    sm100::mma_commit(empty + stage);   // stage reusable when these MMAs finish
                    if (++stage == a.stages) { stage = 0; phase ^= 1u; }
                }
                if (!ok) break;
                sm100::mma_commit(tfull + buf);         // accumulator ready
                if (++buf == a.nbuf) { buf = 0; bphase ^= 1u; }
            }
            // every MMA this thread issued has finished before TMEM is freed
            // (also when a wait gave up and the loop ended early)
            sm100::mma_commit(mdrain);
            sm100::mbar_wait_drain(mdrain, 0, a.err, 18);
        }
    } else {
        // ---------------- epilogue (warps 2..5): thread = row ----------------
        const int sub = warp & 3;                   // TMEM lane quarter of this warp
        const int rt = sub * 32 + lane;             // row within the tile
        const int ew = warp - 2;                    // epilogue warp 0..7
        const int qh = ew >> 2;                     // 16-query column chunks qh, qh + 2, ...
        const int et = threadIdx.x - 64;            // 0..255 among the epilogue threads
        int buf = 0;
        uint32_t bphase = 0;
        bool have_theta = MODE != kFused;
        bool pipe_ok = true;
        // per-query values every row compares against, once per CTA
        for (int q = et; q < kSmallMaxB; q += kSmallEpi) {
            s_mg[q] = q < a.B ? __ldg(a.margin + q) : 0.0f;
            s_theta[q] = (MODE == kCandidates && q < a.B) ? __ldg(a.theta + q) : INFINITY;
            s_qn[q] = 0;
        }
        if (et == 0) s_ccnt = 0;
        asm volatile("bar.sync 1, 256;" ::: "memory");
        // the staged candidates to the per-query lists: per query one global
        // atomic reserves its slots; called by all 128 epilogue threads
        auto flush = [&]() {
            const int m = min(s_ccnt, kStageCand);
            for (int i = et; i < m; i += kSmallEpi) atomicAdd(&s_qn[s_cq[i]], 1);
            asm volatile("bar.sync 1, 256;" ::: "memory");
            for (int q = et; q < a.B; q += kSmallEpi) {
                const int c = s_qn[q];
                s_qbase[q] = c > 0 ? atomicAdd(a.cand_cnt + q, c) : 0;
                s_qn[q] = 0;
            }
            asm volatile("bar.sync 1, 256;" ::: "memory");
            for (int i = et; i < m; i += kSmallEpi) {
                const int q = s_cq[i];
                const int pos = s_qbase[q] + atomicAdd(&s_qn[q], 1);
                if (pos < a.cap) a.cand[(int64_t)q * a.cap + pos] = cand_entry(s_crow[i], s_cf[i], s_cs[i]);
            }
            asm volatile("bar.sync 1, 256;" ::: "memory");
            for (int q = et; q < a.B; q += kSmallEpi) s_qn[q] = 0;
            if (et == 0) s_ccnt = 0;
            asm volatile("bar.sync 1, 256;" ::: "memory");
        };
        SmallTile tl;
        for (int it = 0; small_tile<MODE>(a, it, tl); ++it) {
            if (MODE == kFused && !tl.sample && !have_theta) {
                // every CTA's sample maxima written: a grid-wide arrival count
                // (the launch is cooperative, so every CTA is resident and the
                // wait ends; it is bounded all the same)
                asm volatile("bar.sync 1, 256;" ::: "memory");
                if (et == 0) {
                    __threadfence();
                    atomicAdd(a.grid_sync, 1ull);
                    uint32_t spins = 0;
                    while (ld_acquire_u64(a.grid_sync) < a.sync_target) {
                        // a CTA whose pipeline wait gave up may never arrive
                        if (*((volatile int*)a.err) != 0) break;
                        // given up: recorded in its own word, so the pipeline
                        // runs on and drains normally; the rescore then marks
                        // every result of the call invalid
                        if (++spins > a.sync_spin_limit) { atomicCAS(a.sync_err, 0, 17); break; }
                        __nanosleep(128);
                    }
                    __threadfence();
                }
                asm volatile("bar.sync 1, 256;" ::: "memory");
                for (int q = ew; q < a.B; q += 2 * kSmallWarps) {
                    const float th = a.j <= kJ
                        ? warp_threshold<kJ>(a.sample_buf, a.n_sample, a.B, q, a.j, a.sample_per_tile, lane)
                        : warp_threshold<kThrKeep>(a.sample_buf, a.n_sample, a.B, q, a.j, a.sample_per_tile, lane);
                    if (lane == 0) {
                        s_theta[q] = th;
                        if (blockIdx.x == 0) a.theta_out[q] = th;
                    }
                }
                asm volatile("bar.sync 1, 256;" ::: "memory");
                have_theta = true;
            }
            const int row = tl.row0 + rt;
            const float w = row < a.n ? row_weight(a.meta, row) : NAN;   // NaN: never a candidate
            // every epilogue thread runs the same tiles and named barriers:
            // after a wait gave up, the remaining tiles are skipped, not left
            // (the TMEM loads are warp-collective, so the warp decides as one)
            pipe_ok = pipe_ok && sm100::mbar_wait(tfull + buf, bphase, a.err, 16);
            pipe_ok = __all_sync(0xffffffffu, pipe_ok);
            if (pipe_ok) {
            sm100::tc_fence_after();
            const int selfq = a.self_base >= 0 ? row - a.self_base : -1;   // the query that leaves this row out
            for (int q0 = 16 * qh; q0 < a.NQ; q0 += 32) {
                uint32_t r[16];
                sm100::tmem_ld_32x32b_x16(tmem_base + ((uint32_t)(sub * 32) << 16) + (uint32_t)(buf * a.NQ + q0), r);
                sm100::tmem_ld_wait();
                if (!tl.sample) {
                    // the 16 queries' tests without a branch each (columns
                    // past B carry theta = +inf), then the rare hits
                    uint32_t pass = 0u;
#pragma unroll
                    for (int u4 = 0; u4 < 4; ++u4) {
                        const float4 th4 = reinterpret_cast<const float4*>(s_theta + q0)[u4];
                        const float4 mg4 = reinterpret_cast<const float4*>(s_mg + q0)[u4];
                        const float thv[4] = {th4.x, th4.y, th4.z, th4.w};
                        const float mgv[4] = {mg4.x, mg4.y, mg4.z, mg4.w};
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            const int u = 4 * u4 + k;
                            const float wq = (q0 + u == selfq) ? NAN : w;
                            const float f = __uint_as_float(r[u]) * wq;
                            if (f + mgv[k] * fabsf(wq) >= thv[k]) pass |= 1u << u;   // NaN weights never pass
                        }
                    }
                    if (pass != 0u) {
#pragma unroll
                    for (int u = 0; u < 16; ++u) {   // compile-time indices: r[] stays in registers
                        if (!(pass & (1u << u))) continue;
                        const int q = q0 + u;
                        const float wq = (q == selfq) ? NAN : w;
                        const float f = __uint_as_float(r[u]) * wq;
                        const float slack = s_mg[q] * fabsf(wq);
                        const int p = atomicAdd(&s_ccnt, 1);
                        if (p < kStageCand) {
                            s_cq[p] = (int16_t)q;
                            s_crow[p] = row;
                            s_cf[p] = f;
                            s_cs[p] = slack;
                        } else {   // the stage is full: straight to the query's list
                            const int pos = atomicAdd(a.cand_cnt + q, 1);
                            if (pos < a.cap) a.cand[(int64_t)q * a.cap + pos] = cand_entry(row, f, slack);
                        }
                    }
                    }
                    continue;
                }
#pragma unroll
                for (int u = 0; u < 16; ++u) {
                    const int q = q0 + u;
                    if (q >= a.B) break;
                    const float wq = (q == selfq) ? NAN : w;
                    const float f = __uint_as_float(r[u]) * wq;
                    const float slack = s_mg[q] * fabsf(wq);
                    {
                        // the warp's largest lower bound (its 32 rows) for query q
                        float lo = f - slack;
                        if (!(lo == lo)) lo = -INFINITY;
#pragma unroll
                        for (int off = 16; off >= 1; off >>= 1)
                            lo = fmaxf(lo, __shfl_xor_sync(0xffffffffu, lo, off));
                        if (lane == 0) {
                            if (a.sample_per_tile == 1) s_wmax[sub][q] = lo;
                            else a.sample_buf[((int64_t)tl.sidx * a.B + q) * kSmallWarps + sub] = lo;
                        }
                    }
                }
            }
            sm100::tc_fence_before();
            sm100::mbar_arrive(tempty + buf);
            }   // pipe_ok
            if (++buf == a.nbuf) { buf = 0; bphase ^= 1u; }
            if (tl.sample && a.sample_per_tile == 1) {
                // the tile's largest lower bound per query: sample_buf[tile][query]
                asm volatile("bar.sync 1, 256;" ::: "memory");
                if (et < a.B)
                    a.sample_buf[(int64_t)tl.sidx * a.B + et] =
                        fmaxf(fmaxf(s_wmax[0][et], s_wmax[1][et]), fmaxf(s_wmax[2][et], s_wmax[3][et]));
                asm volatile("bar.sync 1, 256;" ::: "memory");
            }
            if (!tl.sample) {   // the stage half full: out to the lists
                asm volatile("bar.sync 1, 256;" ::: "memory");
                if (s_ccnt >= kStageCand / 2) flush();
            }
        }
        asm volatile("bar.sync 1, 256;" ::: "memory");
        if (s_ccnt > 0) flush();
    }
    sm100::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        sm100::tc_fence_after();
        sm100::tmem_dealloc(tmem_base, a.tmem_cols);
    }
}

}  // namespace batch
}  // namespace mars

using namespace mars;
using namespace mars::batch;

// ---------------------------------------------------------------------------
// Host side

// A tensor map and the arguments it was encoded for.
struct MapCache {
    const void* base = nullptr;
    int64_t rows = -1, cols = -1, pitch = -1;
    int box = 0;
    bool f16 = false;
    CUtensorMap map{};
};

struct mars_batch_ctx {
    int32_t device = 0;
    int32_t max_batch = 0;
    int32_t dim = 0;
    int32_t max_k = 0;
    int32_t max_nodes = 0;
    int32_t cap = 0;
    int32_t num_sms = 0;
    cudaStream_t stream = nullptr;
    float* d_margin = nullptr;       // max_batch
    float* d_theta = nullptr;
    int4* d_cand = nullptr;          // max_batch * cap candidate records
    // the call's status words, one block read back with one copy:
    // [err, sync_err, fallback[max_batch], cand_cnt[max_batch], rescored[max_batch], bad[max_batch]]
    // (err: a pipeline wait gave up; sync_err: the grid-wide arrival wait gave up)
    int32_t* d_status = nullptr;
    int32_t* h_status = nullptr;     // pinned, device-mapped mirror (written by the rescore kernel)
    int32_t* dm_status = nullptr;    // its device address
    int32_t* d_err = nullptr;        // views into d_status / h_status
    int32_t* d_fallback = nullptr;
    int32_t* d_cand_cnt = nullptr;
    int32_t* d_rescored = nullptr;
    int32_t* d_bad = nullptr;        // a query component outside the fp16 range
    int32_t* h_err = nullptr;
    int32_t* h_fallback = nullptr;
    int32_t* h_cand_cnt = nullptr;
    int32_t* h_rescored = nullptr;
    int32_t* h_bad = nullptr;
    float* d_sample = nullptr;       // sample_tiles_cap * max_batch * kJ
    int32_t* d_sample_rt = nullptr;
    int32_t sample_tiles_cap = 0;
    size_t sample_floats_cap = 0;
    int32_t sample_rt_n = -1, sample_rt_rtiles = -1, sample_rt_rows = -1;   // the row-tile list on the device
    int32_t max_smem = 0;            // opt-in shared memory per block
    unsigned long long* d_grid_sync = nullptr;   // the small-batch launch's arrival counter (monotone)
    unsigned long long grid_sync_count = 0;      // its value after the launches issued so far
    bool coop = false;               // the device runs cooperative launches
    bool single_launch = false;      // small batches: sample + thresholds + candidates in one launch
    __half* d_q16 = nullptr;         // max_batch x q16_pitch: fp16 queries
    int32_t q16_pitch = 0;
    int32_t precision = 0;           // 0: fp16 when in range, 1: TF32 always
    MapCache map_q, map_e;           // tensor maps of the last call's operands
    mars_query_ctx* scan_ctx = nullptr;   // exact single-query scans for fallbacks
    mars_batch_stats last{};
    cudaEvent_t ev_gemm[2] = {nullptr, nullptr};   // around the candidates pass
    // exact rescans of the queries the rescore could not certify, on the
    // device (a multi-query scan that skips unflagged queries)
    int32_t fb_grid = 1;                // CTAs per query at max_batch queries
    float* d_fb_val = nullptr;          // max_batch * fb_grid * max_k
    int32_t* d_fb_idx = nullptr;
    unsigned int* d_fb_slots = nullptr; // tickets [max_batch], row counters [max_batch]
    // the last call's status block, read when asked for
    cudaStream_t last_stream = nullptr;
    cudaEvent_t ev_status = nullptr;    // after the status copy
    bool status_pending = false;
    int32_t last_B = 0;
    // test hook (mars_batch_ctx_debug_wait): polls of the arrival wait (0:
    // the default) and arrivals the next call waits for beyond its CTAs'
    uint32_t dbg_spin_limit = 0;
    int32_t dbg_extra_arrivals = 0;
};

int batch_collect_stats(mars_batch_ctx* c);

namespace {

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 2D tensor [rows][cols] (fp32, or fp16 when f16) with a row stride of
// `pitch` elements; box (128 bytes of cols x box_rows), 128-byte swizzle,
// out-of-range elements read as 0.
int make_map(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t pitch, int box_rows,
             bool f16 = false) {
    auto enc = get_encode();
    if (enc == nullptr) return fail(MARS_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    const int64_t esz = f16 ? 2 : 4;
    cuuint64_t gdim[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t gstride[1] = {(cuuint64_t)(pitch * esz)};
    cuuint32_t box[2] = {(cuuint32_t)(128 / esz), (cuuint32_t)box_rows};
    cuuint32_t estride[2] = {1, 1};
    CUresult r = enc(m, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                     const_cast<void*>(base), gdim, gstride, box,
                     estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(MARS_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
    return MARS_OK;
}

// make_map through a cache: the same operands as the last call reuse its map.
int cached_map(MapCache& mc, const void* base, int64_t rows, int64_t cols, int64_t pitch, int box_rows, bool f16) {
    if (mc.base == base && mc.rows == rows && mc.cols == cols && mc.pitch == pitch && mc.box == box_rows &&
        mc.f16 == f16)
        return MARS_OK;
    mc.base = nullptr;
    MARS_TRY(make_map(&mc.map, base, rows, cols, pitch, box_rows, f16));
    mc.base = base;
    mc.rows = rows;
    mc.cols = cols;
    mc.pitch = pitch;
    mc.box = box_rows;
    mc.f16 = f16;
    return MARS_OK;
}

constexpr size_t kGemmSmem = (size_t)kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/ +
                             kBN * sizeof(float) /*row weights*/ +
                             (kGemmEpi / 32) * 32 * 32 * sizeof(float) /*epilogue warps' score stages*/;
static_assert(kGemmSmem <= 232448, "the 128 x 256 tile's shared memory exceeds the opt-in limit");

}  // namespace

extern "C" {

int mars_batch_ctx_create(int32_t device, int32_t max_nodes, int32_t dim, int32_t max_batch, int32_t max_k,
                          mars_batch_ctx** out) {
    if (out == nullptr) return fail(MARS_ERR_INVALID, "mars_batch_ctx_create: out is NULL");
    *out = nullptr;
    if (max_nodes <= 0 || dim <= 0 || dim > 1024 || max_batch <= 0 || max_k <= 0 || max_k > MARS_MAX_TOP_K)
        return fail(MARS_ERR_INVALID, "mars_batch_ctx_create: bad sizes");
    MarsDeviceGuard g(device);
    if (!g.ok) return fail(MARS_ERR_NO_DEVICE, "mars_batch_ctx_create: cudaSetDevice failed");
    cudaDeviceProp prop;
    MARS_CUDA_TRY(cudaGetDeviceProperties(&prop, device));
    if (prop.major < 10) return fail(MARS_ERR_NO_DEVICE, "mars_batch_ctx_create: needs sm_100a");
    auto* c = new mars_batch_ctx();
    c->device = device;
    c->max_batch = max_batch;
    c->dim = dim;
    c->max_k = max_k;
    c->max_nodes = max_nodes;
    c->cap = kSortCap;   // a query with more candidates is rescanned exactly anyway
    c->num_sms = prop.multiProcessorCount;
    c->max_smem = (int32_t)prop.sharedMemPerBlockOptin;
    c->coop = prop.cooperativeLaunch != 0;
    c->single_launch = c->coop;
    c->sample_tiles_cap = 0;
    int rc = MARS_OK;
    auto T = [&](cudaError_t e, const char* w) {
        if (e == cudaSuccess) return;
        if (rc == MARS_OK) rc = cuda_fail(e, w, __FILE__, __LINE__);   // records the first failure
        else (void)cudaGetLastError();                                 // later ones only clear the state
    };
    T(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking), "stream");
    T(cudaEventCreate(&c->ev_gemm[0]), "event");
    T(cudaEventCreate(&c->ev_gemm[1]), "event");
    T(cudaMalloc(&c->d_margin, (size_t)max_batch * 4), "margins");
    T(cudaMalloc(&c->d_theta, (size_t)max_batch * 4), "thresholds");
    T(cudaMalloc(&c->d_cand, (size_t)max_batch * c->cap * sizeof(int4)), "candidates");
    const size_t status_words = 2 + 4 * (size_t)max_batch;
    T(cudaMalloc(&c->d_status, status_words * 4), "status words");
    T(cudaHostAlloc(&c->h_status, status_words * 4, cudaHostAllocMapped), "pinned status words");
    if (rc == MARS_OK) T(cudaHostGetDevicePointer(&c->dm_status, c->h_status, 0), "mapped status words");
    if (rc == MARS_OK) {
        c->d_err = c->d_status;
        c->d_fallback = c->d_status + 2;
        c->d_cand_cnt = c->d_fallback + max_batch;
        c->d_rescored = c->d_cand_cnt + max_batch;
        c->d_bad = c->d_rescored + max_batch;
        c->h_err = c->h_status;
        c->h_fallback = c->h_status + 2;
        c->h_cand_cnt = c->h_fallback + max_batch;
        c->h_rescored = c->h_cand_cnt + max_batch;
        c->h_bad = c->h_rescored + max_batch;
        T(cudaMemset(c->d_status, 0, status_words * 4), "memset");
    }
    c->q16_pitch = (dim + 7) & ~7;
    T(cudaMalloc(&c->d_q16, (size_t)max_batch * c->q16_pitch * sizeof(__half)), "fp16 queries");
    c->fb_grid = std::max(1, std::min(2 * c->num_sms, 2 * c->num_sms / max_batch));
    T(cudaMalloc(&c->d_fb_val, (size_t)max_batch * c->fb_grid * max_k * 4), "rescan partials");
    T(cudaMalloc(&c->d_fb_idx, (size_t)max_batch * c->fb_grid * max_k * 4), "rescan partials");
    T(cudaMalloc(&c->d_fb_slots, (size_t)max_batch * 2 * sizeof(unsigned int)), "rescan slots");
    if (rc == MARS_OK) T(cudaMemset(c->d_fb_slots, 0, (size_t)max_batch * 2 * sizeof(unsigned int)), "memset");
    T(cudaEventCreateWithFlags(&c->ev_status, cudaEventDisableTiming), "event");
    T(cudaMalloc(&c->d_grid_sync, sizeof(unsigned long long)), "grid counter");
    if (rc == MARS_OK) T(cudaMemset(c->d_grid_sync, 0, sizeof(unsigned long long)), "memset");
    if (rc == MARS_OK) {
        static bool attr_done[64] = {};
        if (device < 64 && !attr_done[device]) {
            T(cudaFuncSetAttribute(gemm_kernel<kSample, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemmSmem), "smem attr");
            T(cudaFuncSetAttribute(gemm_kernel<kCandidates, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemmSmem), "smem attr");
            T(cudaFuncSetAttribute(gemm_kernel<kSample, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemmSmem), "smem attr");
            T(cudaFuncSetAttribute(gemm_kernel<kCandidates, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemmSmem), "smem attr");
            T(cudaFuncSetAttribute(gemm_small_kernel<kSample>, cudaFuncAttributeMaxDynamicSharedMemorySize, c->max_smem - kSmallStaticSmem), "smem attr");
            T(cudaFuncSetAttribute(gemm_small_kernel<kCandidates>, cudaFuncAttributeMaxDynamicSharedMemorySize, c->max_smem - kSmallStaticSmem), "smem attr");
            T(cudaFuncSetAttribute(gemm_small_kernel<kFused>, cudaFuncAttributeMaxDynamicSharedMemorySize, c->max_smem - kSmallStaticSmem), "smem attr");
            attr_done[device] = rc == MARS_OK;
        }
    }
    if (rc == MARS_OK) rc = mars_query_ctx_create(device, max_nodes, dim, max_k, &c->scan_ctx);
    if (rc != MARS_OK) { mars_batch_ctx_destroy(c); return rc; }
    *out = c;
    return MARS_OK;
}

int mars_batch_ctx_set_precision(mars_batch_ctx* c, int32_t tf32_only) {
    if (c == nullptr) return fail(MARS_ERR_INVALID, "mars_batch_ctx_set_precision: NULL context");
    c->precision = tf32_only != 0 ? 1 : 0;
    return MARS_OK;
}

int mars_batch_ctx_set_single_launch(mars_batch_ctx* c, int32_t enable) {
    if (c == nullptr) return fail(MARS_ERR_INVALID, "mars_batch_ctx_set_single_launch: NULL context");
    c->single_launch = enable != 0 && c->coop;
    return MARS_OK;
}

int mars_batch_ctx_debug_wait(mars_batch_ctx* c, uint32_t spin_limit, int32_t extra_arrivals) {
    if (c == nullptr || extra_arrivals < 0)
        return fail(MARS_ERR_INVALID, "mars_batch_ctx_debug_wait: NULL context or negative arrivals");
    c->dbg_spin_limit = spin_limit;
    c->dbg_extra_arrivals = extra_arrivals;
    return MARS_OK;
}

int mars_batch_ctx_destroy(mars_batch_ctx* c) {
    if (c == nullptr) return MARS_OK;
    MarsDeviceGuard g(c->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    cudaFree(c->d_margin); cudaFree(c->d_theta); cudaFree(c->d_cand);
    cudaFree(c->d_sample); cudaFree(c->d_sample_rt);
    cudaFree(c->d_status); cudaFreeHost(c->h_status);
    cudaFree(c->d_q16);
    cudaFree(c->d_fb_val); cudaFree(c->d_fb_idx); cudaFree(c->d_fb_slots);
    cudaFree(c->d_grid_sync);
    if (c->ev_status) cudaEventDestroy(c->ev_status);
    mars_query_ctx_destroy(c->scan_ctx);
    for (cudaEvent_t e : c->ev_gemm)
        if (e) cudaEventDestroy(e);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
    return MARS_OK;
}

int mars_batch_last_stats(const mars_batch_ctx* c, mars_batch_stats* out) {
    if (c == nullptr || out == nullptr) return fail(MARS_ERR_INVALID, "mars_batch_last_stats: NULL argument");
    const int rc = batch_collect_stats(const_cast<mars_batch_ctx*>(c));   // the statistics are a cache
    *out = c->last;
    return rc;
}

int mars_query_batch_topk(const mars_store* s, mars_batch_ctx* c, const float* d_queries, int32_t query_pitch,
                          int32_t B, float t_q, float lambda, int32_t modality_filter, int32_t use_importance,
                          int32_t K, int32_t row_offset, int32_t* d_ids, float* d_vals, int32_t* d_counts,
                          void* stream) {
    return mars::batch_topk(s, c, d_queries, query_pitch, B, t_q, lambda, modality_filter, use_importance, K,
                            row_offset, -1, d_ids, d_vals, d_counts, stream);
}

}  // extern "C"

int batch_topk_pass(const mars_store* s, mars_batch_ctx* c, const float* d_queries, int32_t query_pitch,
                    int32_t B, float t_q, float lambda, int32_t modality_filter, int32_t use_importance,
                    int32_t K, int32_t row_offset, int32_t self_base, int32_t* d_ids, float* d_vals,
                    int32_t* d_counts, void* stream, bool allow_f16, mars::BoundExchange* xchg);

// After a wait that gave up, some CTAs of the small-batch launch may not
// have counted their arrival: once the stream is idle, the grid counter and
// its expected value start again from zero.
void batch_reset_grid_sync(mars_batch_ctx* c) {
    if (c->last_stream != nullptr) cudaStreamSynchronize(c->last_stream);
    if (cudaMemset(c->d_grid_sync, 0, sizeof(unsigned long long)) == cudaSuccess) c->grid_sync_count = 0;
}

// The previous call's pipeline error word, if its status copy has landed
// (never waits).
int batch_prev_status(mars_batch_ctx* c) {
    if (!c->status_pending || cudaEventQuery(c->ev_status) != cudaSuccess) return MARS_OK;
    if (c->h_err[0] != 0 || c->h_err[1] != 0) {
        const int code = c->h_err[0] != 0 ? c->h_err[0] : c->h_err[1];
        c->h_err[0] = c->h_err[1] = 0;
        c->status_pending = false;
        batch_reset_grid_sync(c);
        return fail(MARS_ERR_TIMEOUT, "mars_query_batch_topk: a tensor-core pipeline wait gave up (code " +
                                          std::to_string(code) + ")");
    }
    return MARS_OK;
}

// Fill c->last from the last call's status words (waits for the call).
int batch_collect_stats(mars_batch_ctx* c) {
    if (!c->status_pending) return MARS_OK;
    MarsDeviceGuard g(c->device);
    MARS_CUDA_TRY(cudaEventSynchronize(c->ev_status));
    c->status_pending = false;
    int64_t total = 0, rescored = 0;
    int32_t fb = 0, maxc = 0;
    for (int32_t b = 0; b < c->last_B; ++b) {
        total += c->h_cand_cnt[b];
        rescored += c->h_rescored[b];
        maxc = std::max(maxc, c->h_cand_cnt[b]);
        fb += c->h_fallback[b] != 0 ? 1 : 0;
    }
    float gms = 0.f;
    MARS_CUDA_TRY(cudaEventElapsedTime(&gms, c->ev_gemm[0], c->ev_gemm[1]));
    c->last.gemm_ms = gms;
    c->last.fallbacks = fb;
    c->last.candidates = total;
    c->last.max_candidates = maxc;
    c->last.rescored = rescored;
    if (c->h_err[0] != 0 || c->h_err[1] != 0) {
        const int code = c->h_err[0] != 0 ? c->h_err[0] : c->h_err[1];
        c->h_err[0] = c->h_err[1] = 0;
        batch_reset_grid_sync(c);
        return fail(MARS_ERR_TIMEOUT, "mars_query_batch_topk: a tensor-core pipeline wait gave up (code " +
                                          std::to_string(code) + ")");
    }
    return MARS_OK;
}

// Asynchronous on the stream: queries that the rescore cannot certify (and
// queries outside the fp16 range) are rescanned exactly on the device, so no
// step waits for the host.  The statistics of the call are read when
// mars_batch_last_stats asks for them.
int mars::batch_topk(const mars_store* s, mars_batch_ctx* c, const float* d_queries, int32_t query_pitch,
                     int32_t B, float t_q, float lambda, int32_t modality_filter, int32_t use_importance,
                     int32_t K, int32_t row_offset, int32_t self_base, int32_t* d_ids, float* d_vals,
                     int32_t* d_counts, void* stream) {
    return batch_topk_pass(s, c, d_queries, query_pitch, B, t_q, lambda, modality_filter, use_importance, K,
                           row_offset, self_base, d_ids, d_vals, d_counts, stream,
                           c != nullptr && c->precision == 0, nullptr);
}

cudaStream_t mars::batch_ctx_stream(const mars_batch_ctx* c) { return c->stream; }

int mars::batch_topk_sharded(const mars_store* s, mars_batch_ctx* c, const float* d_queries, int32_t query_pitch,
                             int32_t B, float t_q, float lambda, int32_t modality_filter, int32_t use_importance,
                             int32_t K, int32_t row_offset, int32_t* d_ids, float* d_vals, int32_t* d_counts,
                             void* stream, BoundExchange* xchg) {
    return batch_topk_pass(s, c, d_queries, query_pitch, B, t_q, lambda, modality_filter, use_importance, K,
                           row_offset, -1, d_ids, d_vals, d_counts, stream, c != nullptr && c->precision == 0,
                           xchg);
}

int mars::shard_neutral_thr(float* d_rec, int32_t B, cudaStream_t st) {
    neutral_thr_kernel<<<(shard_thr_floats(B) + 255) / 256, 256, 0, st>>>(d_rec, B);
    MARS_CUDA_TRY(cudaGetLastError());
    return MARS_OK;
}

int mars::shard_neutral_rec(float* d_rec, int32_t B, bool failed, cudaStream_t st) {
    neutral_rec_kernel<<<(shard_rec_floats(B) + 255) / 256, 256, 0, st>>>(d_rec, B, failed ? 1.0f : 0.0f);
    MARS_CUDA_TRY(cudaGetLastError());
    return MARS_OK;
}

int batch_topk_pass(const mars_store* s, mars_batch_ctx* c, const float* d_queries, int32_t query_pitch,
                    int32_t B, float t_q, float lambda, int32_t modality_filter, int32_t use_importance,
                    int32_t K, int32_t row_offset, int32_t self_base, int32_t* d_ids, float* d_vals,
                    int32_t* d_counts, void* stream, bool allow_f16, mars::BoundExchange* xchg) {
    if (s == nullptr || c == nullptr || d_queries == nullptr || d_ids == nullptr || d_vals == nullptr)
        return fail(MARS_ERR_INVALID, "mars_query_batch_topk: NULL argument");
    if (s->device != c->device || s->dim != c->dim)
        return fail(MARS_ERR_INVALID, "mars_query_batch_topk: store and context do not match");
    if (B < 0 || B > c->max_batch || K <= 0 || K > c->max_k)
        return fail(MARS_ERR_INVALID, "mars_query_batch_topk: B or K out of range");
    if (query_pitch < s->pitch || (query_pitch & 3) != 0 || (reinterpret_cast<uintptr_t>(d_queries) & 15u) != 0)
        return fail(MARS_ERR_INVALID, "mars_query_batch_topk: queries must be 16-byte aligned rows with pitch >= the store's");
    if (s->n > c->max_nodes)
        return fail(MARS_ERR_CAPACITY, "mars_query_batch_topk: store larger than the context");
    if (s->d_norm_bits == nullptr)
        return fail(MARS_ERR_UNSUPPORTED, "mars_query_batch_topk: store has no row-norm bound (a view of caller memory)");
    MARS_TRY(batch_prev_status(c));
    const int32_t dbg_extra = c->dbg_extra_arrivals;   // the test hook holds for one call
    c->dbg_extra_arrivals = 0;
    c->last = mars_batch_stats{};
    c->status_pending = false;
    if (B == 0) return MARS_OK;
    MarsDeviceGuard g(c->device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    MARS_CUDA_TRY(cudaStreamWaitEvent(st, s->written, 0));
    const int32_t n = s->n;
    const int32_t rtiles = (n + kBN - 1) / kBN;
    const int32_t qtiles = (B + kBM - 1) / kBM;
    int32_t nkb = (s->pitch + kBK - 1) / kBK;

    // sample size: one row tile in 48.  The threshold is the j-th best
    // sampled lower bound, about the level of the 48 j best rows of the
    // whole store, so a few hundred candidates per query whatever K is (the
    // rescore sorts up to kSortCap); mu, the expected number of true top-K
    // members in the sample, sets j so the threshold stays below the K-th
    // score with high probability (else the query is rescanned exactly).
    int32_t n_sample = (int32_t)std::ceil((double)n / (48.0 * kBN));
    n_sample = std::max(1, std::min(n_sample, rtiles));
    const double mu = (double)K * std::min<int64_t>((int64_t)n_sample * kBN, n) / std::max(n, 1);
    int32_t j = (int32_t)std::ceil(mu + 5.0 * std::sqrt(mu) + 3.0);
    const bool use_gemm = n >= 4 * kBN && K >= 3 && n_sample < rtiles && j <= kJ;
    if (!use_gemm) {
        // small corpora: exact single-query scans, one per query
        for (int32_t b = 0; b < B; ++b)
            MARS_TRY(mars::scan_topk_excluding(s, c->scan_ctx, d_queries + (int64_t)b * query_pitch, t_q,
                                               lambda, modality_filter, use_importance, K, row_offset,
                                               self_base >= 0 ? self_base + b : -1, d_ids + (int64_t)b * K,
                                               d_vals + (int64_t)b * K, d_counts ? d_counts + b : nullptr, st));
        c->last.fallbacks = B;
        c->last.path = 0;
        return MARS_OK;
    }

    // operands: fp16 copies (twice the tensor-core rate, half the bytes,
    // the same 10 mantissa bits as TF32) when every value is in range
    bool f16 = false;
    if (allow_f16) MARS_TRY(mars::store_f16_rows(s, st, &f16));
    // small batches on fp16 operands: rows as the MMA's M (gemm_small_kernel)
    const int32_t NQ = (B + 15) & ~15;
    int32_t stages = 0;
    if (f16 && B <= kSmallMaxB) {
        const size_t fixed = small_smem_bytes((s->e16_pitch + 63) / 64, NQ, 0);
        const size_t room = (size_t)c->max_smem - kSmallStaticSmem;   // the kernel's static array aside
        if (fixed < room) stages = (int32_t)std::min<size_t>(kSmallMaxStages, (room - fixed) / kSmallStage);
    }
    bool small = stages >= 2;
    if (small) {   // the same one-in-48 rule over 128-row tiles, at most one wave of them
        const int32_t tiles128 = (n + kSmallRows - 1) / kSmallRows;
        const int32_t ns = std::max(1, std::min({(int32_t)std::ceil((double)n / (48.0 * kSmallRows)), tiles128 - 1,
                                                 c->num_sms}));
        const double mu_s = (double)K * std::min<int64_t>((int64_t)ns * kSmallRows, n) / std::max(n, 1);
        const int32_t js = (int32_t)std::ceil(mu_s + 5.0 * std::sqrt(mu_s) + 3.0);
        small = js <= kThrKeep;
        if (small) {
            n_sample = ns;
            j = js;
        }
    }
    const int32_t tile_rows = small ? kSmallRows : kBN;
    const int32_t all_tiles = small ? (n + kSmallRows - 1) / kSmallRows : rtiles;
    // small tiles: one maximum per sampled tile and query when the sample has
    // plenty of tiles for the j-th largest, else one per epilogue warp
    const int32_t per_tile = small ? (n_sample >= 4 * j ? 1 : kSmallWarps) : 2 * kJ;
    const size_t sample_floats = (size_t)n_sample * (small ? B : c->max_batch) * per_tile;
    if (c->d_sample == nullptr || n_sample > c->sample_tiles_cap || sample_floats > c->sample_floats_cap) {
        MARS_CUDA_TRY(cudaStreamSynchronize(st));
        cudaFree(c->d_sample);
        cudaFree(c->d_sample_rt);
        c->d_sample = nullptr;
        c->d_sample_rt = nullptr;
        c->sample_tiles_cap = std::max(n_sample, 16);
        c->sample_floats_cap = std::max(sample_floats, (size_t)c->sample_tiles_cap * c->max_batch * 2 * kJ);
        MARS_CUDA_TRY(cudaMalloc(&c->d_sample, c->sample_floats_cap * 4));
        MARS_CUDA_TRY(cudaMalloc(&c->d_sample_rt, (size_t)c->sample_tiles_cap * 4));
        c->sample_rt_n = -1;
    }
    // strided sample of row tiles (uploaded again only when it changes)
    if (c->sample_rt_n != n_sample || c->sample_rt_rtiles != all_tiles || c->sample_rt_rows != tile_rows) {
        std::vector<int32_t> srt(n_sample);
        for (int32_t i = 0; i < n_sample; ++i) srt[i] = (int32_t)(((int64_t)i * all_tiles) / n_sample);
        MARS_CUDA_TRY(cudaMemcpyAsync(c->d_sample_rt, srt.data(), (size_t)n_sample * 4, cudaMemcpyHostToDevice,
                                      st));
        MARS_CUDA_TRY(cudaStreamSynchronize(st));   // srt lives on this stack frame
        c->sample_rt_n = n_sample;
        c->sample_rt_rtiles = all_tiles;
        c->sample_rt_rows = tile_rows;
    }

    if (f16) {
        MARS_TRY(cached_map(c->map_q, c->d_q16, B, c->q16_pitch, c->q16_pitch, small ? NQ : kBM, true));
        MARS_TRY(cached_map(c->map_e, s->d_E16, n, s->e16_pitch, s->e16_pitch, tile_rows, true));
        nkb = (s->e16_pitch + 63) / 64;
    } else {
        MARS_TRY(cached_map(c->map_q, d_queries, B, s->pitch, query_pitch, kBM, false));
        MARS_TRY(cached_map(c->map_e, s->d_E, n, s->pitch, s->pitch, kBN, false));
    }
    const CUtensorMap& mq = c->map_q.map;
    const CUtensorMap& me = c->map_e.map;
    bool shard_global = false;   // row shards: the threshold came from every shard's sample

    RowMeta meta{};
    meta.ts = s->d_ts;
    meta.imp = s->d_imp;
    meta.mod = s->d_mod;
    meta.t_q = t_q;
    meta.lambda = lambda;
    meta.filter = modality_filter;
    meta.use_imp = use_importance;
    prep_queries_kernel<<<(B * 32 + 255) / 256, 256, 0, st>>>(d_queries, query_pitch, B, (s->dim + 3) / 4,
                                                              s->d_norm_bits, f16 ? 1 : 0, c->d_margin,
                                                              c->d_cand_cnt, c->d_rescored, c->d_bad,
                                                              c->d_err, f16 ? c->d_q16 : nullptr, c->q16_pitch);
    MARS_CUDA_TRY(cudaGetLastError());

    if (small) {
        SmallArgs sa{};
        sa.B = B;
        sa.NQ = NQ;
        sa.n = n;
        sa.nkb = nkb;
        sa.stages = stages;
        sa.nbuf = std::max(2, std::min(kSmallAccBufs, 512 / NQ));
        uint32_t cols = 32;
        while (cols < (uint32_t)(sa.nbuf * NQ)) cols <<= 1;
        sa.tmem_cols = cols;
        sa.sample_rt = c->d_sample_rt;
        sa.meta = meta;
        sa.theta = c->d_theta;
        sa.margin = c->d_margin;
        sa.sample_buf = c->d_sample;
        sa.cand = c->d_cand;
        sa.cand_cnt = c->d_cand_cnt;
        sa.cap = c->cap;
        sa.self_base = self_base;
        sa.err = c->d_err;
        const size_t smem = small_smem_bytes(nkb, NQ, stages);
        const int grid = std::min(all_tiles, c->num_sms);
        sa.n_tiles = all_tiles;
        sa.n_sample = n_sample;
        sa.j = j;
        sa.sample_per_tile = per_tile;
        if (c->single_launch) {
            // 2.-4. sample, thresholds and candidates in one cooperative launch
            // (one CTA per SM, every CTA resident): CTA b < n_sample first runs
            // sample tile b; the epilogue warps meet on a grid-wide counter,
            // take the thresholds, and go on with the candidate tiles that the
            // producer and MMA warps have kept streaming meanwhile
            sa.grid_sync = c->d_grid_sync;
            sa.sync_target = c->grid_sync_count + (unsigned long long)grid + (unsigned long long)dbg_extra;
            sa.sync_spin_limit = c->dbg_spin_limit != 0 ? c->dbg_spin_limit : sm100::kSpinLimit;
            sa.sync_err = c->d_status + 1;
            sa.theta_out = c->d_theta;
            void* args[] = {const_cast<CUtensorMap*>(&mq), const_cast<CUtensorMap*>(&me), &sa};
            MARS_CUDA_TRY(cudaEventRecord(c->ev_gemm[0], st));
            MARS_CUDA_TRY(cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(&gemm_small_kernel<kFused>),
                                                      dim3(grid), dim3(kSmallThreads), args, smem, st));
            c->grid_sync_count += (unsigned long long)grid;
            MARS_CUDA_TRY(cudaEventRecord(c->ev_gemm[1], st));
        } else {
            // the same three steps as separate launches (no cooperative launch)
            sa.n_tiles = n_sample;
            gemm_small_kernel<kSample><<<n_sample, kSmallThreads, smem, st>>>(mq, me, sa);
            MARS_CUDA_TRY(cudaGetLastError());
            if (j <= kJ)
                threshold_kernel<kJ><<<(B * 32 + kThrThreads - 1) / kThrThreads, kThrThreads, 0, st>>>(
                    c->d_sample, n_sample, B, j, sa.sample_per_tile, c->d_theta);
            else
                threshold_kernel<kThrKeep><<<(B * 32 + kThrThreads - 1) / kThrThreads, kThrThreads, 0, st>>>(
                    c->d_sample, n_sample, B, j, sa.sample_per_tile, c->d_theta);
            MARS_CUDA_TRY(cudaGetLastError());
            sa.n_tiles = all_tiles;
            MARS_CUDA_TRY(cudaEventRecord(c->ev_gemm[0], st));
            gemm_small_kernel<kCandidates><<<grid, kSmallThreads, smem, st>>>(mq, me, sa);
            MARS_CUDA_TRY(cudaGetLastError());
            MARS_CUDA_TRY(cudaEventRecord(c->ev_gemm[1], st));
        }
    } else {
        GemmArgs ga{};
        ga.B = B;
        ga.n = n;
        ga.nkb = nkb;
        ga.qtiles = qtiles;
        ga.rtiles = rtiles;
        ga.sample_rt = c->d_sample_rt;
        ga.meta = meta;
        ga.theta = c->d_theta;
        ga.margin = c->d_margin;
        ga.sample_buf = c->d_sample;
        ga.cand = c->d_cand;
        ga.cand_cnt = c->d_cand_cnt;
        ga.cap = c->cap;
        ga.self_base = self_base;
        ga.err = c->d_err;

        // 2. sample
        ga.n_tiles = n_sample * qtiles;
        if (f16)
            gemm_kernel<kSample, true><<<std::min(ga.n_tiles, c->num_sms), kGemmThreads, kGemmSmem, st>>>(mq, me, ga);
        else
            gemm_kernel<kSample, false><<<std::min(ga.n_tiles, c->num_sms), kGemmThreads, kGemmSmem, st>>>(mq, me, ga);
        MARS_CUDA_TRY(cudaGetLastError());
        // 3. thresholds (2 kJ values per tile and query)
        const int thr_grid = (B * 32 + kThrThreads - 1) / kThrThreads;
        if (xchg != nullptr) {
            // row shards: every shard's kJ best sampled bounds per query, one
            // all-gather, and the same threshold on every shard from their
            // union (a sample of the whole corpus, so each shard short-lists
            // about 1 / world of the rows it would list on its own)
            sample_record_kernel<<<thr_grid, kThrThreads, 0, st>>>(
                c->d_sample, n_sample, B, per_tile, (int32_t)std::min<int64_t>((int64_t)n_sample * kBN, n), n,
                xchg->send[0]);
            MARS_CUDA_TRY(cudaGetLastError());
            xchg->theta_done = true;
            MARS_TRY(xchg->gather(xchg->arg, 0, shard_thr_floats(B), st));
            union_threshold_kernel<<<thr_grid, kThrThreads, 0, st>>>(xchg->recv[0], xchg->world,
                                                                     shard_thr_floats(B), B, K, c->d_theta);
            shard_global = true;
        } else {
            threshold_kernel<kJ><<<thr_grid, kThrThreads, 0, st>>>(c->d_sample, n_sample, B, j, per_tile, c->d_theta);
        }
        MARS_CUDA_TRY(cudaGetLastError());
        // 4. candidates
        ga.n_tiles = rtiles * qtiles;
        MARS_CUDA_TRY(cudaEventRecord(c->ev_gemm[0], st));
        if (f16)
            gemm_kernel<kCandidates, true><<<std::min(ga.n_tiles, c->num_sms), kGemmThreads, kGemmSmem, st>>>(mq, me,
                                                                                                            ga);
        else
            gemm_kernel<kCandidates, false><<<std::min(ga.n_tiles, c->num_sms), kGemmThreads, kGemmSmem, st>>>(mq, me,
                                                                                                             ga);
        MARS_CUDA_TRY(cudaGetLastError());
        MARS_CUDA_TRY(cudaEventRecord(c->ev_gemm[1], st));
    }
    // 5. rescore
    StoreView v{};
    v.E = s->d_E; v.ts = s->d_ts; v.imp = s->d_imp; v.mod = s->d_mod; v.d_n = s->d_n;
    v.pitch4 = s->pitch / 4; v.nc = (s->dim + 3) / 4;
    auto rescore = [&](float* bound_out, const float* bound_in, bool split) {
        rescore_kernel<<<B, kRescoreThreads, 0, st>>>(v, d_queries, query_pitch, B, t_q, lambda, use_importance, K,
                                                      row_offset, c->d_theta, c->d_margin, c->d_cand,
                                                      c->d_cand_cnt, c->cap, d_ids, d_vals, d_counts,
                                                      c->d_fallback, c->d_rescored, f16 ? c->d_bad : nullptr,
                                                      c->d_status, bound_out, bound_in,
                                                      xchg != nullptr ? xchg->world : 1, shard_global ? 1 : 0,
                                                      (bound_out == nullptr && !split) ? c->dm_status : nullptr,
                                                      c->max_batch, split ? 1 : 0);
        return cudaGetLastError();
    };
    // large batches: the final pass lists each query's rows, a light kernel
    // scores them (more rows in flight per SM), a third ranks them and
    // publishes the status words
    const bool split = B >= kSplitRescoreMinB;
    auto final_pass = [&](const float* bound_in) -> int {
        MARS_CUDA_TRY(rescore(nullptr, bound_in, split));
        if (!split) return MARS_OK;
        const int cpl = (v.nc + 31) / 32;   // float4 chunks per lane and row
        auto rows = [&](auto kfn) {
            kfn<<<B, kRescoreThreads, 0, st>>>(v, d_queries, query_pitch, t_q, lambda, use_importance, c->d_cand,
                                               c->cap, c->d_rescored, c->d_fallback, c->d_status);
        };
        if (cpl <= 2) rows(rescore_rows_kernel<2>);
        else if (cpl <= 4) rows(rescore_rows_kernel<4>);
        else if (cpl <= 6) rows(rescore_rows_kernel<6>);
        else rows(rescore_rows_kernel<8>);
        MARS_CUDA_TRY(cudaGetLastError());
        rescore_rank_kernel<<<B, kRescoreThreads, 0, st>>>(K, row_offset, c->d_cand, c->cap, d_ids, d_vals, d_counts,
                                                           c->d_fallback, c->d_rescored, c->d_cand_cnt,
                                                           f16 ? c->d_bad : nullptr, c->d_status, c->dm_status,
                                                           c->max_batch);
        MARS_CUDA_TRY(cudaGetLastError());
        return MARS_OK;
    };
    if (xchg != nullptr) {
        // row shards: a small batch took its thresholds inside the fused
        // launch (its own shard's), so it joins the threshold exchange with a
        // neutral record; then every shard's bound record, one all-gather,
        // and the rescore against all of them
        if (!xchg->theta_done) {
            MARS_TRY(shard_neutral_thr(xchg->send[0], B, st));
            xchg->theta_done = true;
            MARS_TRY(xchg->gather(xchg->arg, 0, shard_thr_floats(B), st));
        }
        MARS_CUDA_TRY(rescore(xchg->send[1], nullptr, false));
        xchg->done = true;
        MARS_TRY(xchg->gather(xchg->arg, 1, shard_rec_floats(B), st));
        MARS_TRY(final_pass(xchg->recv[1]));
    } else {
        MARS_TRY(final_pass(nullptr));
    }
    // 6. exact rescans of the flagged queries (every CTA of an unflagged
    // query leaves at once)
    ScanArgs fa{};
    fa.s = StoreView{};
    fa.s.E = s->d_E; fa.s.ts = s->d_ts; fa.s.imp = s->d_imp; fa.s.mod = s->d_mod; fa.s.d_n = s->d_n;
    fa.s.pitch4 = s->pitch / 4; fa.s.nc = (s->dim + 3) / 4;
    fa.d.t_q = t_q;
    fa.d.lambda = lambda;
    fa.d.filter = modality_filter;
    fa.d.use_imp = use_importance;
    fa.d.K = K;
    fa.d.row_offset = row_offset;
    fa.part_val = c->d_fb_val;
    fa.part_idx = c->d_fb_idx;
    fa.ticket = c->d_fb_slots;
    fa.cursor = c->d_fb_slots + c->max_batch;
    fa.out_val = d_vals;
    fa.out_idx = d_ids;
    fa.out_cnt = d_counts;
    fa.only = c->d_fallback;
    fa.exclude_base1 = self_base >= 0 ? self_base + 1 : 0;
    const int fgx = std::max(1, std::min(c->fb_grid, 2 * c->num_sms / B));
    MARS_CUDA_TRY(launch_scan_multi(fa, d_queries, query_pitch, B, fgx, st));
    // the status words (read by mars_batch_last_stats and checked for a
    // pipeline error by the next call) were written to the mapped mirror by
    // the rescore kernel; they are readable once this event has completed
    MARS_CUDA_TRY(cudaEventRecord(c->ev_status, st));
    c->status_pending = true;
    c->last_stream = st;
    c->last_B = B;
    c->last.path = small ? 3 : (f16 ? 2 : 1);
    c->last.sample_tiles = n_sample;
    c->last.sample_rank = j;
    return MARS_OK;
}


