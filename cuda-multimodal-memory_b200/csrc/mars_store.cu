// mars_store.cu -- the device store (DeviceMemoryGraph) and streaming insert.
//
// Layout in HBM (one allocation per array, capacity rows, 256-byte aligned):
//   E        capacity x pitch fp32, pitch = D rounded up to 4 (16-byte rows),
//            pad columns zero;
//   ts, imp  capacity fp32 (imp initialised to 1), mod capacity int32;
//   d_n      the current row count, read by every kernel so that appends need
//            no relaunch or graph re-capture;
//   CSR      row_offsets / col_indices over the rows present at upload;
//   slack    capacity x edge_slack int32 append-only neighbour lists + counts.
//
// Reference: upload_to_device / free_device (src/memory_cuda.cu:593-627) and
// engine_server's add_node + ensure_device (src/engine_server.cu:154-213),
// which grows host vectors and re-uploads the whole corpus on the next query.
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "mars_b200.h"
#include "mars_internal.h"

namespace mars {

static thread_local std::string g_last_error = "no error";

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int status, const std::string& msg) {
    g_last_error = msg;
    return status;
}

int cuda_fail(cudaError_t e, const char* what, const char* file, int line) {
    char buf[512];
    std::snprintf(buf, sizeof(buf), "CUDA error %s (%s) in %s at %s:%d", cudaGetErrorName(e),
                  cudaGetErrorString(e), what, file, line);
    g_last_error = buf;
    // a failed call (an allocation that ran out of memory, say) also left
    // the runtime's last-error state set; clear it, or the next launch check
    // anywhere in the process would report this failure as its own (errors
    // that corrupted the context stay: they are sticky)
    (void)cudaGetLastError();
    return e == cudaErrorMemoryAllocation ? MARS_ERR_OOM : MARS_ERR_CUDA;
}

// ---------------------------------------------------------------------------
// Normalisation of appended rows, bit-identical to the reference's host rule
// (src/engine_server.cu:165-171): norm = sqrtf(sequential fp32 sum of x*x)
// + 1e-8f, then x / norm.  One thread forms the sequential sum of its row
// (the order is what makes it bit-exact); the warp then divides the row.
__global__ void normalize_rows_kernel(float* __restrict__ E, int64_t pitch, int32_t first,
                                      int32_t count, int32_t dim) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= count) return;
    float* row = E + (int64_t)(first + warp) * pitch;
    float norm = 0.0f;
    if (lane == 0) {
        for (int32_t d = 0; d < dim; ++d) norm = __fadd_rn(norm, __fmul_rn(row[d], row[d]));
        norm = __fadd_rn(__fsqrt_rn(norm), 1e-8f);
    }
    norm = __shfl_sync(0xffffffffu, norm, 0);
    for (int32_t d = lane; d < dim; d += 32) row[d] = __fdiv_rn(row[d], norm);
}

// Largest L2 norm of rows [first, first + count): one warp per row, the
// maximum kept as the bit pattern of a non-negative float (order-preserving).
__global__ void row_norm_max_kernel(const float* __restrict__ E, int64_t pitch, int32_t first,
                                    int32_t count, int32_t dim, unsigned int* __restrict__ out_bits) {
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= count) return;
    const float* row = E + (first + warp) * pitch;
    float s = 0.f;
    for (int32_t d = lane; d < dim; d += 32) s = fmaf(row[d], row[d], s);
    for (int off = 16; off >= 1; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) atomicMax(out_bits, __float_as_uint(sqrtf(s) * 1.0001f));
}

// Small appends in one launch: one warp per row copies the row from the
// (host-mapped) staging area into E, normalises it with exactly the rule of
// normalize_rows_kernel when asked, folds its norm into the store's bound,
// copies the row's metadata and publishes the new row count.  Kernels that
// read the store run after this one (the store's `written` event).
constexpr int kAppendWarps = 8;
struct AppendArgs {
    float* E;
    int64_t pitch;
    int32_t first, count, dim, normalize;
    const float* rows;        // count x dim, packed
    const int32_t* mod;
    const float* ts;
    const float* imp;         // may be null: importance 1
    int32_t* d_mod;
    float* d_ts;
    float* d_imp;
    unsigned int* norm_bits;
    int32_t* d_n;
    int32_t new_n;
};

__global__ void __launch_bounds__(kAppendWarps * 32) append_rows_kernel(const AppendArgs a) {
    __shared__ float s_row[kAppendWarps][1024];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = blockIdx.x * kAppendWarps + w;
    if (blockIdx.x == 0 && threadIdx.x == 0) *a.d_n = a.new_n;
    if (r >= a.count) return;
    const float* src = a.rows + (int64_t)r * a.dim;
    float* dst = a.E + (int64_t)(a.first + r) * a.pitch;
    for (int d = lane; d < a.dim; d += 32) s_row[w][d] = src[d];
    __syncwarp();
    float norm = 1.0f;
    if (a.normalize) {
        if (lane == 0) {
            float acc = 0.0f;
            for (int d = 0; d < a.dim; ++d) acc = __fadd_rn(acc, __fmul_rn(s_row[w][d], s_row[w][d]));
            norm = __fadd_rn(__fsqrt_rn(acc), 1e-8f);
        }
        norm = __shfl_sync(0xffffffffu, norm, 0);
    }
    float ss = 0.f;
    for (int d = lane; d < a.dim; d += 32) {
        const float x = a.normalize ? __fdiv_rn(s_row[w][d], norm) : s_row[w][d];
        dst[d] = x;
        ss = fmaf(x, x, ss);
    }
    for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (lane == 0) {
        atomicMax(a.norm_bits, __float_as_uint(sqrtf(ss) * 1.0001f));
        a.d_mod[a.first + r] = a.mod[r];
        a.d_ts[a.first + r] = a.ts[r];
        a.d_imp[a.first + r] = a.imp != nullptr ? a.imp[r] : 1.0f;
    }
}

// Tombstones (src/engine_server.cu:178-185): the row's embedding becomes
// zero and its timestamp -1.  One warp per id; ids outside [0, n) are ignored.
__global__ void delete_rows_kernel(float* __restrict__ E, int64_t pitch, float* __restrict__ ts,
                                   const int32_t* __restrict__ ids, int32_t count, const int32_t* __restrict__ d_n,
                                   int32_t dim) {
    const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (w >= count) return;
    const int32_t u = ids[w];
    if (u < 0 || u >= *d_n) return;
    float* row = E + (int64_t)u * pitch;
    for (int d = lane; d < dim; d += 32) row[d] = 0.0f;
    if (lane == 0) ts[u] = -1.0f;
}

// fp16 copy of rows [r0, r1) (row pitch `pitch16` halves, pad zero), one
// warp per row.  Each row's rounding error ||e - fp16(e)|| (exact
// differences, fp32 sum of squares rounded up by 0.1 %) raises *err_bits,
// the largest over the rows: the batched short list bounds its error with it.
__global__ void to_f16_rows_kernel(const float* __restrict__ E, int64_t pitch, int32_t r0, int32_t r1, int32_t dim,
                                   __half* __restrict__ E16, int64_t pitch16, unsigned int* __restrict__ err_bits) {
    const int lane = threadIdx.x & 31;
    const int64_t w0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t r = r0 + w0; r < r1; r += nw) {
        float ss = 0.0f;
        for (int64_t d = lane; d < pitch16; d += 32) {
            const float x = d < dim ? E[r * pitch + d] : 0.0f;
            const __half h = __float2half_rn(x);
            E16[r * pitch16 + d] = h;
            const float e = x - __half2float(h);    // exact
            ss = fmaf(e, e, ss);
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
        if (lane == 0 && ss > 0.0f) atomicMax(err_bits, __float_as_uint(sqrtf(ss) * 1.001f));
    }
}

__global__ void fill_f32_kernel(float* p, int64_t n, float v) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) p[i] = v;
}

__global__ void scatter_edges_kernel(int32_t* __restrict__ extra, int32_t* __restrict__ cnt,
                                     const int32_t* __restrict__ slot_pos,
                                     const int32_t* __restrict__ dst,
                                     const int32_t* __restrict__ src,
                                     const int32_t* __restrict__ new_cnt, int32_t n) {
    const int32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    extra[slot_pos[i]] = dst[i];
    // every edge of a node writes the same final count; the value is the
    // node's count after this whole batch
    cnt[src[i]] = new_cnt[i];
}

__global__ void importance_decay_kernel(float* __restrict__ imp, const int32_t* __restrict__ d_n,
                                        float retain) {
    const int32_t n = *d_n;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        imp[i] *= retain;
}

__global__ void importance_boost_kernel(float* __restrict__ imp, const int32_t* __restrict__ d_n,
                                        const int32_t* __restrict__ ids, int32_t count, float boost,
                                        float max_imp) {
    const int32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= count) return;
    const int32_t u = ids[i];
    if (u < 0 || u >= *d_n) return;
    unsigned int* p = reinterpret_cast<unsigned int*>(imp + u);
    unsigned int old = *p, assumed;
    do {
        assumed = old;
        const float nv = fminf(__uint_as_float(assumed) + boost, max_imp);
        old = atomicCAS(p, assumed, __float_as_uint(nv));
    } while (old != assumed);
}

}  // namespace mars

using namespace mars;

static int alloc_store(mars_store* s) {
    const size_t rows = (size_t)s->capacity;
    MARS_CUDA_TRY(cudaMalloc(&s->d_E, rows * (size_t)s->pitch * sizeof(float)));
    MARS_CUDA_TRY(cudaMemsetAsync(s->d_E, 0, rows * (size_t)s->pitch * sizeof(float), s->stream));
    MARS_CUDA_TRY(cudaMalloc(&s->d_ts, rows * sizeof(float)));
    MARS_CUDA_TRY(cudaMemsetAsync(s->d_ts, 0, rows * sizeof(float), s->stream));
    MARS_CUDA_TRY(cudaMalloc(&s->d_imp, rows * sizeof(float)));
    if (rows > 0) {
        fill_f32_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, s->stream>>>(s->d_imp, (int64_t)rows, 1.0f);
        MARS_CUDA_TRY(cudaGetLastError());
    }
    MARS_CUDA_TRY(cudaMalloc(&s->d_mod, rows * sizeof(int32_t)));
    MARS_CUDA_TRY(cudaMemsetAsync(s->d_mod, 0, rows * sizeof(int32_t), s->stream));
    MARS_CUDA_TRY(cudaMalloc(&s->d_n, sizeof(int32_t)));
    MARS_CUDA_TRY(cudaMemsetAsync(s->d_n, 0, sizeof(int32_t), s->stream));
    // [0]: the largest row norm; [1]: the largest fp16 rounding error of a
    // row of the fp16 copy (both as the bits of non-negative floats)
    MARS_CUDA_TRY(cudaMalloc(&s->d_norm_bits, 2 * sizeof(unsigned int)));
    MARS_CUDA_TRY(cudaMemsetAsync(s->d_norm_bits, 0, 2 * sizeof(unsigned int), s->stream));
    if (s->edge_slack > 0) {
        MARS_CUDA_TRY(cudaMalloc(&s->d_extra, rows * (size_t)s->edge_slack * sizeof(int32_t)));
        MARS_CUDA_TRY(cudaMalloc(&s->d_extra_cnt, rows * sizeof(int32_t)));
        MARS_CUDA_TRY(cudaMemsetAsync(s->d_extra_cnt, 0, rows * sizeof(int32_t), s->stream));
        s->h_extra_cnt.assign(rows, 0);
    }
    MARS_CUDA_TRY(cudaEventRecord(s->written, s->stream));
    return MARS_OK;
}

static void release_store(mars_store* s) {
    if (s->owns) {
        cudaFree(s->d_E);
        cudaFree(s->d_ts);
        cudaFree(s->d_imp);
        cudaFree(s->d_mod);
        cudaFree(s->d_row_offsets);
        cudaFree(s->d_col_indices);
    }
    cudaFree(s->d_n);
    cudaFree(s->d_norm_bits);
    cudaFree(s->d_extra);
    cudaFree(s->d_extra_cnt);
    cudaFree(s->d_E16);
    if (s->e16_ready) cudaEventDestroy(s->e16_ready);
    if (s->build.bc) mars_batch_ctx_destroy(s->build.bc);
    cudaFree(s->build.d_knn);
    cudaFree(s->build.d_vals);
    cudaFree(s->build.d_cnt);
    for (auto& sg : s->stage) {
        if (sg.done) {
            cudaEventSynchronize(sg.done);
            cudaEventDestroy(sg.done);
        }
        if (sg.h) cudaFreeHost(sg.h);
    }
    if (s->written) cudaEventDestroy(s->written);
    if (s->stream) cudaStreamDestroy(s->stream);
}

namespace {

constexpr size_t kStageBytes = 4u << 20;

bool on_host(const void* p) {
    if (p == nullptr) return true;
    cudaPointerAttributes pa{};
    if (cudaPointerGetAttributes(&pa, p) != cudaSuccess) {
        (void)cudaGetLastError();
        return true;
    }
    return pa.type != cudaMemoryTypeDevice;
}

// The next staging buffer with room for `bytes`, after its previous user
// finished; nullptr when the request is larger than a buffer.
mars_store::HostStage* stage_acquire(mars_store* s, size_t bytes, int* rc) {
    *rc = MARS_OK;
    if (bytes > kStageBytes) return nullptr;
    mars_store::HostStage& sg = s->stage[s->stage_next];
    if (sg.h == nullptr) {
        cudaError_t e = cudaHostAlloc(reinterpret_cast<void**>(&sg.h), kStageBytes, cudaHostAllocMapped);
        if (e == cudaSuccess) e = cudaHostGetDevicePointer(reinterpret_cast<void**>(&sg.d), sg.h, 0);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&sg.done, cudaEventDisableTiming);
        if (e != cudaSuccess) {
            *rc = cuda_fail(e, "append staging", __FILE__, __LINE__);
            return nullptr;
        }
        sg.cap = kStageBytes;
    } else {
        const cudaError_t e = cudaEventSynchronize(sg.done);
        if (e != cudaSuccess) {
            *rc = cuda_fail(e, "append staging wait", __FILE__, __LINE__);
            return nullptr;
        }
    }
    s->stage_next ^= 1;
    return &sg;
}

}  // namespace


// Bring the store's fp16 copy of the rows up to date on stream st (after the
// store's writes).  *ok: the copy may be used, i.e. every component is
// within kF16Max (the row-norm bound says so).
int mars::store_f16_rows(const mars_store* cs, cudaStream_t st, bool* ok) {
    auto* s = const_cast<mars_store*>(cs);   // the copy is a cache of the rows
    *ok = false;
    if (!s->owns || s->d_norm_bits == nullptr) return MARS_OK;
    const int32_t n = s->n;
    if (s->e16_rows < n) {
        unsigned int bits = 0;
        MARS_CUDA_TRY(cudaMemcpyAsync(&bits, s->d_norm_bits, sizeof(bits), cudaMemcpyDeviceToHost, st));
        MARS_CUDA_TRY(cudaStreamSynchronize(st));
        float bound;
        std::memcpy(&bound, &bits, sizeof(bound));
        s->e16_in_range = bound <= kF16Max;   // |component| <= row norm
        if (!s->e16_in_range) return MARS_OK;
        if (s->d_E16 == nullptr) {
            s->e16_pitch = (s->dim + 7) & ~7;
            MARS_CUDA_TRY(cudaMalloc(&s->d_E16, (size_t)s->capacity * s->e16_pitch * sizeof(__half)));
        }
        if (s->e16_ready == nullptr) MARS_CUDA_TRY(cudaEventCreateWithFlags(&s->e16_ready, cudaEventDisableTiming));
        const int32_t r0 = s->e16_rows;
        // a rebuilt copy starts its rounding-error bound again
        if (r0 == 0) MARS_CUDA_TRY(cudaMemsetAsync(s->d_norm_bits + 1, 0, sizeof(unsigned int), st));
        const int64_t rows = n - r0;
        const int grid = (int)std::min<int64_t>((rows * 32 + 255) / 256, 148 * 16);
        to_f16_rows_kernel<<<grid, 256, 0, st>>>(s->d_E, s->pitch, r0, n, s->dim,
                                                 static_cast<__half*>(s->d_E16), s->e16_pitch, s->d_norm_bits + 1);
        MARS_CUDA_TRY(cudaGetLastError());
        MARS_CUDA_TRY(cudaEventRecord(s->e16_ready, st));
        s->e16_rows = n;
    } else if (s->e16_ready != nullptr) {
        // another stream may still be converting the last rows
        MARS_CUDA_TRY(cudaStreamWaitEvent(st, s->e16_ready, 0));
    }
    *ok = s->e16_in_range;
    return MARS_OK;
}

extern "C" {

const char* mars_last_error(void) { return g_last_error.c_str(); }

const char* mars_status_string(int status) {
    switch (status) {
    case MARS_OK: return "ok";
    case MARS_ERR_INVALID: return "invalid argument";
    case MARS_ERR_CUDA: return "CUDA error";
    case MARS_ERR_OOM: return "out of memory";
    case MARS_ERR_CAPACITY: return "capacity exceeded";
    case MARS_ERR_UNSUPPORTED: return "unsupported";
    case MARS_ERR_TIMEOUT: return "device wait timed out";
    case MARS_ERR_NO_DEVICE: return "no sm_100 device";
    case MARS_ERR_DEVICE: return "device-side check failed";
    default: return "unknown status";
    }
}

int mars_abi_version(void) { return MARS_B200_ABI_VERSION; }

int mars_store_create(int32_t device, int32_t capacity, int32_t dim, int32_t edge_slack,
                      mars_store** out) {
    if (out == nullptr) return fail(MARS_ERR_INVALID, "mars_store_create: out is NULL");
    *out = nullptr;
    if (capacity < 0 || dim <= 0 || dim > 1024 || edge_slack < 0)
        return fail(MARS_ERR_INVALID, "mars_store_create: need capacity >= 0, 0 < dim <= 1024, edge_slack >= 0");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev)
        return fail(MARS_ERR_NO_DEVICE, "mars_store_create: no such CUDA device");
    MarsDeviceGuard g(device);
    if (!g.ok) return fail(MARS_ERR_CUDA, "mars_store_create: cudaSetDevice failed");
    mars_store* s = new mars_store();
    s->device = device;
    s->capacity = capacity;
    s->dim = dim;
    s->pitch = (dim + 3) & ~3;
    s->edge_slack = edge_slack;
    int st = MARS_OK;
    if (cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&s->written, cudaEventDisableTiming) != cudaSuccess) {
        st = fail(MARS_ERR_CUDA, "mars_store_create: stream/event creation failed");
    } else {
        st = alloc_store(s);
    }
    if (st == MARS_OK) st = (cudaStreamSynchronize(s->stream) == cudaSuccess)
                                ? MARS_OK : fail(MARS_ERR_CUDA, "mars_store_create: initialisation failed");
    if (st != MARS_OK) {
        release_store(s);
        delete s;
        return st;
    }
    *out = s;
    return MARS_OK;
}

int mars_store_upload(mars_store* s, int32_t n, const float* embeddings, const int32_t* modalities,
                      const float* timestamps, const float* importance, const int32_t* row_offsets,
                      const int32_t* col_indices, int32_t num_edges) {
    if (s == nullptr) return fail(MARS_ERR_INVALID, "mars_store_upload: store is NULL");
    if (n < 0 || n > s->capacity)
        return fail(MARS_ERR_CAPACITY, "mars_store_upload: n exceeds the store capacity");
    if (n > 0 && (embeddings == nullptr || modalities == nullptr || timestamps == nullptr))
        return fail(MARS_ERR_INVALID, "mars_store_upload: embeddings, modalities and timestamps are required");
    if (row_offsets != nullptr && (num_edges < 0 || (num_edges > 0 && col_indices == nullptr)))
        return fail(MARS_ERR_INVALID, "mars_store_upload: bad CSR arguments");
    if (!s->owns) return fail(MARS_ERR_INVALID, "mars_store_upload: store wraps caller memory");
    MarsDeviceGuard g(s->device);
    cudaStream_t st = s->stream;
    const size_t D = (size_t)s->dim, P = (size_t)s->pitch;
    if (n > 0) {
        MARS_CUDA_TRY(cudaMemcpy2DAsync(s->d_E, P * sizeof(float), embeddings, D * sizeof(float),
                                        D * sizeof(float), (size_t)n, cudaMemcpyDefault, st));
        MARS_CUDA_TRY(cudaMemcpyAsync(s->d_mod, modalities, (size_t)n * 4, cudaMemcpyDefault, st));
        MARS_CUDA_TRY(cudaMemcpyAsync(s->d_ts, timestamps, (size_t)n * 4, cudaMemcpyDefault, st));
        if (importance != nullptr) {
            MARS_CUDA_TRY(cudaMemcpyAsync(s->d_imp, importance, (size_t)n * 4, cudaMemcpyDefault, st));
        } else {
            fill_f32_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(s->d_imp, n, 1.0f);
            MARS_CUDA_TRY(cudaGetLastError());
        }
    }
    // graph
    if (row_offsets != nullptr) {
        if (s->d_row_offsets == nullptr || s->csr_n < n) {
            cudaFree(s->d_row_offsets);
            s->d_row_offsets = nullptr;
            MARS_CUDA_TRY(cudaMalloc(&s->d_row_offsets, ((size_t)n + 1) * sizeof(int32_t)));
        }
        if (s->d_col_indices == nullptr || s->csr_edge_cap < num_edges) {
            cudaFree(s->d_col_indices);
            s->d_col_indices = nullptr;
            MARS_CUDA_TRY(cudaMalloc(&s->d_col_indices, (size_t)std::max(num_edges, 1) * sizeof(int32_t)));
            s->csr_edge_cap = std::max(num_edges, 1);
        }
        MARS_CUDA_TRY(cudaMemcpyAsync(s->d_row_offsets, row_offsets, ((size_t)n + 1) * 4, cudaMemcpyDefault, st));
        if (num_edges > 0)
            MARS_CUDA_TRY(cudaMemcpyAsync(s->d_col_indices, col_indices, (size_t)num_edges * 4, cudaMemcpyDefault, st));
        s->csr_n = n;
        s->num_edges = num_edges;
    } else {
        s->csr_n = 0;
        s->num_edges = 0;
    }
    if (s->edge_slack > 0) {
        MARS_CUDA_TRY(cudaMemsetAsync(s->d_extra_cnt, 0, (size_t)s->capacity * 4, st));
        std::fill(s->h_extra_cnt.begin(), s->h_extra_cnt.end(), 0);
    }
    MARS_CUDA_TRY(cudaMemcpyAsync(s->d_n, &n, sizeof(int32_t), cudaMemcpyHostToDevice, st));
    MARS_CUDA_TRY(cudaMemsetAsync(s->d_norm_bits, 0, sizeof(unsigned int), st));
    if (n > 0) {
        row_norm_max_kernel<<<(unsigned)(((int64_t)n * 32 + 255) / 256), 256, 0, st>>>(
            s->d_E, (int64_t)P, 0, n, s->dim, s->d_norm_bits);
        MARS_CUDA_TRY(cudaGetLastError());
    }
    MARS_CUDA_TRY(cudaStreamSynchronize(st));   // n lives on this stack frame
    s->n = n;
    s->e16_rows = 0;
    MARS_CUDA_TRY(cudaEventRecord(s->written, st));
    return MARS_OK;
}

int mars_store_append(mars_store* s, int32_t n, const float* embeddings, const int32_t* modalities,
                      const float* timestamps, const float* importance, int32_t normalize,
                      int32_t* first_id) {
    if (s == nullptr) return fail(MARS_ERR_INVALID, "mars_store_append: store is NULL");
    if (n < 0) return fail(MARS_ERR_INVALID, "mars_store_append: n < 0");
    if (n > 0 && (embeddings == nullptr || modalities == nullptr || timestamps == nullptr))
        return fail(MARS_ERR_INVALID, "mars_store_append: embeddings, modalities and timestamps are required");
    if (!s->owns) return fail(MARS_ERR_INVALID, "mars_store_append: store wraps caller memory");
    if ((int64_t)s->n + n > s->capacity)
        return fail(MARS_ERR_CAPACITY, "mars_store_append: store is full (capacity " +
                                           std::to_string(s->capacity) + ")");
    if (first_id) *first_id = s->n;
    if (n == 0) return MARS_OK;
    MarsDeviceGuard g(s->device);
    cudaStream_t st = s->stream;
    const size_t D = (size_t)s->dim, P = (size_t)s->pitch;
    const int32_t first = s->n;

    // small host-side appends: pack into mapped staging, one launch, no wait
    const size_t row_bytes = (size_t)n * D * sizeof(float);
    const size_t bytes = row_bytes + (size_t)n * 12;
    if (bytes <= kStageBytes && on_host(embeddings) && on_host(modalities) && on_host(timestamps) &&
        on_host(importance)) {
        int rc = MARS_OK;
        mars_store::HostStage* sg = stage_acquire(s, bytes, &rc);
        MARS_TRY(rc);
        if (sg != nullptr) {
            std::memcpy(sg->h, embeddings, row_bytes);
            std::memcpy(sg->h + row_bytes, modalities, (size_t)n * 4);
            std::memcpy(sg->h + row_bytes + (size_t)n * 4, timestamps, (size_t)n * 4);
            if (importance) std::memcpy(sg->h + row_bytes + (size_t)n * 8, importance, (size_t)n * 4);
            AppendArgs aa{};
            aa.E = s->d_E;
            aa.pitch = (int64_t)P;
            aa.first = first;
            aa.count = n;
            aa.dim = s->dim;
            aa.normalize = normalize != 0;
            aa.rows = reinterpret_cast<const float*>(sg->d);
            aa.mod = reinterpret_cast<const int32_t*>(sg->d + row_bytes);
            aa.ts = reinterpret_cast<const float*>(sg->d + row_bytes + (size_t)n * 4);
            aa.imp = importance ? reinterpret_cast<const float*>(sg->d + row_bytes + (size_t)n * 8) : nullptr;
            aa.d_mod = s->d_mod;
            aa.d_ts = s->d_ts;
            aa.d_imp = s->d_imp;
            aa.norm_bits = s->d_norm_bits;
            aa.d_n = s->d_n;
            aa.new_n = first + n;
            append_rows_kernel<<<(n + kAppendWarps - 1) / kAppendWarps, kAppendWarps * 32, 0, st>>>(aa);
            MARS_CUDA_TRY(cudaGetLastError());
            MARS_CUDA_TRY(cudaEventRecord(sg->done, st));
            MARS_CUDA_TRY(cudaEventRecord(s->written, st));
            s->n = first + n;
            return MARS_OK;
        }
    }

    MARS_CUDA_TRY(cudaMemcpy2DAsync(s->d_E + (size_t)first * P, P * sizeof(float), embeddings,
                                    D * sizeof(float), D * sizeof(float), (size_t)n,
                                    cudaMemcpyDefault, st));
    if (normalize) {
        const int threads = 256;
        const int blocks = (int)(((int64_t)n * 32 + threads - 1) / threads);
        normalize_rows_kernel<<<blocks, threads, 0, st>>>(s->d_E, (int64_t)P, first, n, s->dim);
        MARS_CUDA_TRY(cudaGetLastError());
    }
    MARS_CUDA_TRY(cudaMemcpyAsync(s->d_mod + first, modalities, (size_t)n * 4, cudaMemcpyDefault, st));
    MARS_CUDA_TRY(cudaMemcpyAsync(s->d_ts + first, timestamps, (size_t)n * 4, cudaMemcpyDefault, st));
    if (importance != nullptr)
        MARS_CUDA_TRY(cudaMemcpyAsync(s->d_imp + first, importance, (size_t)n * 4, cudaMemcpyDefault, st));
    row_norm_max_kernel<<<(unsigned)(((int64_t)n * 32 + 255) / 256), 256, 0, st>>>(
        s->d_E, (int64_t)P, first, n, s->dim, s->d_norm_bits);
    MARS_CUDA_TRY(cudaGetLastError());
    // publish the new count after the rows (same stream)
    const int32_t new_n = first + n;
    MARS_CUDA_TRY(cudaMemcpyAsync(s->d_n, &new_n, sizeof(int32_t), cudaMemcpyHostToDevice, st));
    MARS_CUDA_TRY(cudaStreamSynchronize(st));   // new_n and caller buffers live on the host
    s->n = new_n;
    MARS_CUDA_TRY(cudaEventRecord(s->written, st));
    return MARS_OK;
}

int mars_store_append_edges(mars_store* s, int32_t n, const int32_t* src, const int32_t* dst) {
    if (s == nullptr) return fail(MARS_ERR_INVALID, "mars_store_append_edges: store is NULL");
    if (n < 0 || (n > 0 && (src == nullptr || dst == nullptr)))
        return fail(MARS_ERR_INVALID, "mars_store_append_edges: bad arguments");
    if (n == 0) return MARS_OK;
    if (s->edge_slack <= 0)
        return fail(MARS_ERR_CAPACITY, "mars_store_append_edges: store was created with edge_slack 0");
    // plan on the host (deterministic slot order = call order), then scatter;
    // the host counts are advanced in place and rolled back on failure
    std::vector<int32_t> slot(n), fin(n);
    int32_t* cnt = s->h_extra_cnt.data();
    auto rollback = [&](int32_t upto) {
        for (int32_t j = 0; j < upto; ++j) cnt[src[j]] -= 1;
    };
    for (int32_t i = 0; i < n; ++i) {
        const int32_t u = src[i], v = dst[i];
        if (u < 0 || u >= s->n || v < 0 || v >= s->n) {
            rollback(i);
            return fail(MARS_ERR_INVALID, "mars_store_append_edges: endpoint out of range");
        }
        if (cnt[u] >= s->edge_slack) {
            rollback(i);
            return fail(MARS_ERR_CAPACITY, "mars_store_append_edges: node " + std::to_string(u) +
                                               " has no free neighbour slot");
        }
        slot[i] = u * s->edge_slack + cnt[u];
        cnt[u] += 1;
    }
    for (int32_t i = 0; i < n; ++i) fin[i] = cnt[src[i]];
    MarsDeviceGuard g(s->device);
    cudaStream_t st = s->stream;
    int rc = MARS_OK;
    {   // small batches: mapped staging, one launch, no wait
        mars_store::HostStage* sg = stage_acquire(s, (size_t)n * 16, &rc);
        if (rc != MARS_OK) { rollback(n); return rc; }
        if (sg != nullptr) {
            int32_t* h = reinterpret_cast<int32_t*>(sg->h);
            const int32_t* d = reinterpret_cast<const int32_t*>(sg->d);
            std::memcpy(h, slot.data(), (size_t)n * 4);
            std::memcpy(h + n, dst, (size_t)n * 4);
            std::memcpy(h + 2 * (size_t)n, src, (size_t)n * 4);
            std::memcpy(h + 3 * (size_t)n, fin.data(), (size_t)n * 4);
            scatter_edges_kernel<<<(n + 255) / 256, 256, 0, st>>>(s->d_extra, s->d_extra_cnt, d, d + n,
                                                                   d + 2 * (size_t)n, d + 3 * (size_t)n, n);
            const cudaError_t e = cudaGetLastError();
            if (e != cudaSuccess) { rollback(n); return cuda_fail(e, "scatter_edges_kernel", __FILE__, __LINE__); }
            MARS_CUDA_TRY(cudaEventRecord(sg->done, st));
            MARS_CUDA_TRY(cudaEventRecord(s->written, st));
            return MARS_OK;
        }
    }
    int32_t* d_tmp = nullptr;
    if (cudaMallocAsync(&d_tmp, (size_t)n * 4 * 4, st) != cudaSuccess) {
        (void)cudaGetLastError();   // reported here, not by the next launch check
        rollback(n);
        return fail(MARS_ERR_OOM, "mars_store_append_edges: scratch allocation failed");
    }
    do {
        if (cudaMemcpyAsync(d_tmp, slot.data(), (size_t)n * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
            cudaMemcpyAsync(d_tmp + n, dst, (size_t)n * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
            cudaMemcpyAsync(d_tmp + 2 * (size_t)n, src, (size_t)n * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
            cudaMemcpyAsync(d_tmp + 3 * (size_t)n, fin.data(), (size_t)n * 4, cudaMemcpyHostToDevice, st) != cudaSuccess) {
            rc = fail(MARS_ERR_CUDA, "mars_store_append_edges: copy failed");
            break;
        }
        scatter_edges_kernel<<<(n + 255) / 256, 256, 0, st>>>(s->d_extra, s->d_extra_cnt, d_tmp, d_tmp + n,
                                                               d_tmp + 2 * (size_t)n, d_tmp + 3 * (size_t)n, n);
        if (cudaGetLastError() != cudaSuccess) { rc = fail(MARS_ERR_CUDA, "mars_store_append_edges: launch failed"); break; }
    } while (0);
    cudaFreeAsync(d_tmp, st);
    MARS_CUDA_TRY(cudaStreamSynchronize(st));
    if (rc != MARS_OK) { rollback(n); return rc; }
    MARS_CUDA_TRY(cudaEventRecord(s->written, st));
    return MARS_OK;
}

int mars_store_delete(mars_store* s, int32_t n, const int32_t* ids) {
    if (s == nullptr || n < 0 || (n > 0 && ids == nullptr))
        return fail(MARS_ERR_INVALID, "mars_store_delete: bad arguments");
    if (!s->owns) return fail(MARS_ERR_INVALID, "mars_store_delete: store wraps caller memory");
    if (n == 0) return MARS_OK;
    MarsDeviceGuard g(s->device);
    cudaStream_t st = s->stream;
    int rc = MARS_OK;
    mars_store::HostStage* sg = stage_acquire(s, (size_t)n * 4, &rc);
    MARS_TRY(rc);
    const int32_t* d_ids = nullptr;
    int32_t* d_tmp = nullptr;
    if (sg != nullptr) {
        std::memcpy(sg->h, ids, (size_t)n * 4);
        d_ids = reinterpret_cast<const int32_t*>(sg->d);
    } else {
        MARS_CUDA_TRY(cudaMallocAsync(&d_tmp, (size_t)n * 4, st));
        MARS_CUDA_TRY(cudaMemcpyAsync(d_tmp, ids, (size_t)n * 4, cudaMemcpyHostToDevice, st));
        d_ids = d_tmp;
    }
    s->e16_rows = 0;   // rows change in place: the fp16 copy is rebuilt on next use
    delete_rows_kernel<<<(unsigned)(((int64_t)n * 32 + 255) / 256), 256, 0, st>>>(
        s->d_E, (int64_t)s->pitch, s->d_ts, d_ids, n, s->d_n, s->dim);
    MARS_CUDA_TRY(cudaGetLastError());
    if (sg != nullptr) {
        MARS_CUDA_TRY(cudaEventRecord(sg->done, st));
    } else {
        MARS_CUDA_TRY(cudaFreeAsync(d_tmp, st));
        MARS_CUDA_TRY(cudaStreamSynchronize(st));   // the caller's ids were copied synchronously above
    }
    MARS_CUDA_TRY(cudaEventRecord(s->written, st));
    return MARS_OK;
}

int mars_store_set_importance(mars_store* s, int32_t first, int32_t n, const float* importance) {
    if (s == nullptr || importance == nullptr || first < 0 || n < 0 || (int64_t)first + n > s->capacity)
        return fail(MARS_ERR_INVALID, "mars_store_set_importance: bad arguments");
    if (n == 0) return MARS_OK;
    MarsDeviceGuard g(s->device);
    MARS_CUDA_TRY(cudaMemcpyAsync(s->d_imp + first, importance, (size_t)n * 4, cudaMemcpyDefault, s->stream));
    MARS_CUDA_TRY(cudaStreamSynchronize(s->stream));
    MARS_CUDA_TRY(cudaEventRecord(s->written, s->stream));
    return MARS_OK;
}

int mars_importance_fill(mars_store* s, float value) {
    if (s == nullptr) return fail(MARS_ERR_INVALID, "mars_importance_fill: store is NULL");
    if (s->capacity == 0) return MARS_OK;
    MarsDeviceGuard g(s->device);
    fill_f32_kernel<<<(unsigned)((s->capacity + 255) / 256), 256, 0, s->stream>>>(s->d_imp, s->capacity, value);
    MARS_CUDA_TRY(cudaGetLastError());
    MARS_CUDA_TRY(cudaStreamSynchronize(s->stream));
    MARS_CUDA_TRY(cudaEventRecord(s->written, s->stream));
    return MARS_OK;
}

int mars_importance_update(mars_store* s, const int32_t* d_ids, int32_t n, float boost,
                           float decay_rate, float max_importance, void* stream) {
    if (s == nullptr || n < 0 || (n > 0 && d_ids == nullptr))
        return fail(MARS_ERR_INVALID, "mars_importance_update: bad arguments");
    MarsDeviceGuard g(s->device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : s->stream;
    MARS_CUDA_TRY(cudaStreamWaitEvent(st, s->written, 0));
    const float retain = 1.0f - decay_rate;
    if (s->capacity > 0) {
        int blocks = std::min((s->n + 255) / 256 + 1, 4096);
        importance_decay_kernel<<<blocks, 256, 0, st>>>(s->d_imp, s->d_n, retain);
        MARS_CUDA_TRY(cudaGetLastError());
    }
    if (n > 0) {
        importance_boost_kernel<<<(n + 255) / 256, 256, 0, st>>>(s->d_imp, s->d_n, d_ids, n, boost,
                                                                 max_importance);
        MARS_CUDA_TRY(cudaGetLastError());
    }
    MARS_CUDA_TRY(cudaEventRecord(s->written, st));
    return MARS_OK;
}

int mars_store_info_get(const mars_store* s, mars_store_info* out) {
    if (s == nullptr || out == nullptr) return fail(MARS_ERR_INVALID, "mars_store_info_get: NULL argument");
    out->device = s->device;
    out->num_nodes = s->n;
    out->capacity = s->capacity;
    out->embedding_dim = s->dim;
    out->row_pitch = s->pitch;
    out->num_edges = s->num_edges;
    out->csr_nodes = s->csr_n;
    out->edge_slack = s->edge_slack;
    out->d_embeddings = s->d_E;
    out->d_modalities = s->d_mod;
    out->d_timestamps = s->d_ts;
    out->d_importance = s->d_imp;
    out->d_row_offsets = s->d_row_offsets;
    out->d_col_indices = s->d_col_indices;
    out->d_num_nodes = s->d_n;
    return MARS_OK;
}

int mars_store_read(const mars_store* s, int32_t first, int32_t n, float* embeddings,
                    int32_t* modalities, float* timestamps, float* importance) {
    if (s == nullptr || first < 0 || n < 0 || (int64_t)first + n > s->n)
        return fail(MARS_ERR_INVALID, "mars_store_read: rows out of range");
    if (n == 0) return MARS_OK;
    MarsDeviceGuard g(s->device);
    cudaStream_t st = s->stream;
    const size_t D = (size_t)s->dim, P = (size_t)s->pitch;
    if (embeddings)
        MARS_CUDA_TRY(cudaMemcpy2DAsync(embeddings, D * 4, s->d_E + (size_t)first * P, P * 4, D * 4,
                                        (size_t)n, cudaMemcpyDefault, st));
    if (modalities) MARS_CUDA_TRY(cudaMemcpyAsync(modalities, s->d_mod + first, (size_t)n * 4, cudaMemcpyDefault, st));
    if (timestamps) MARS_CUDA_TRY(cudaMemcpyAsync(timestamps, s->d_ts + first, (size_t)n * 4, cudaMemcpyDefault, st));
    if (importance) MARS_CUDA_TRY(cudaMemcpyAsync(importance, s->d_imp + first, (size_t)n * 4, cudaMemcpyDefault, st));
    MARS_CUDA_TRY(cudaStreamSynchronize(st));
    return MARS_OK;
}

int mars_store_destroy(mars_store* s) {
    if (s == nullptr) return MARS_OK;
    MarsDeviceGuard g(s->device);
    if (s->stream) cudaStreamSynchronize(s->stream);
    release_store(s);
    delete s;
    return MARS_OK;
}

}  // extern "C"
