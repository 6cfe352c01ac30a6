// mars_noalloc.cu -- the fused scan top-K for callers that cannot allocate
// GPU memory.
//
// Some callers must not call cudaMalloc: code that runs inside a memory
// budget fixed at start-up (an embedded or real-time loop that reserves all
// device memory before its deadline-bound phase), or a host that hands this
// library pointers it owns and forbids it from growing the footprint.  The
// regular entry points need a store and a query context, and both allocate.
// mars_scan_topk_noalloc takes the caller's own device arrays and keeps its
// working memory (per-block partial lists and two counters) in the
// file-scope device array below, which exists once per GPU that loads the
// library and lives until the process exits.
//
// Rules of use:
//  * the first call on a device sets that device up: it looks up the array's
//    device address with cudaGetSymbolAddress (which loads this file's code
//    and commits the array), reads the SM count, and loads every scan kernel
//    variant this entry point can launch (K <= 128, D <= 1024).  With lazy
//    module loading (the CUDA default) that is the only point where the
//    entry point grows the process's device memory.  Make that first call
//    -- any K, any D -- before reserving the rest of the device memory and
//    before any stream capture on that device, or run the process with
//    CUDA_MODULE_LOADING=EAGER;
//  * every call shares the one array and finds it as the previous call left
//    it; the counters that must start at zero are cleared by each call;
//  * calls whose work overlaps on the GPU (two streams, or two host threads)
//    race on the array: serialise them;
//  * K <= 128 (MARS_NOALLOC_MAX_K); larger K is rejected.
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <string>

#include "mars_b200.h"
#include "mars_internal.h"
#include "mars_kernels.cuh"

namespace {

constexpr int kNoallocMaxBlocks = 512;
constexpr int kNoallocMaxK = MARS_NOALLOC_MAX_K;

struct NoallocScratch {
    unsigned int ticket;          // completion counter of the scan's blocks
    int32_t      n;               // row count read by the scan kernel
    unsigned int cursor;          // rows handed out dynamically by the scan
    int32_t      pad[61];
    float        part_val[kNoallocMaxBlocks * kNoallocMaxK];
    int32_t      part_idx[kNoallocMaxBlocks * kNoallocMaxK];
    int32_t      count;           // used when the caller passes no d_count
};
static_assert(sizeof(NoallocScratch) == MARS_NOALLOC_SCRATCH_BYTES, "scratch size");

// 512 blocks x 128 entries x 8 bytes + 260 bytes: 524,548 bytes per device.
static __device__ __align__(256) NoallocScratch g_noalloc_scratch;

__global__ void noalloc_prepare_kernel(int32_t n) {
    g_noalloc_scratch.ticket = 0u;
    g_noalloc_scratch.cursor = 0u;
    g_noalloc_scratch.n = n;
}

struct DeviceSetup {
    bool ready = false;
    NoallocScratch* scratch = nullptr;   // device address of g_noalloc_scratch
    int num_sms = 0;
};

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
DeviceSetup g_setup[kMaxDevices];

int setup_device(int dev, DeviceSetup** out) {
    std::lock_guard<std::mutex> lk(g_setup_mu);
    DeviceSetup& s = g_setup[dev];
    if (!s.ready) {
        void* p = nullptr;
        MARS_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
        int sms = 0;
        MARS_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        // the kernels' code too, so no later call loads a module
        cudaFuncAttributes fa;
        MARS_CUDA_TRY(cudaFuncGetAttributes(&fa, noalloc_prepare_kernel));
        const int le = mars::preload_scan_topk_kernels();
        if (le != 0) return mars::cuda_fail(static_cast<cudaError_t>(le), "preload_scan_topk_kernels", __FILE__, __LINE__);
        s.scratch = static_cast<NoallocScratch*>(p);
        s.num_sms = sms;
        s.ready = true;
    }
    *out = &s;
    return MARS_OK;
}

}  // namespace

using namespace mars;

extern "C" int mars_scan_topk_noalloc(const float* d_embeddings, int32_t row_pitch,
                                      const float* d_timestamps, const float* d_importance,
                                      const int32_t* d_modalities, int32_t n, int32_t dim,
                                      const float* d_query, float query_timestamp, float lambda,
                                      int32_t modality_filter, int32_t use_importance, int32_t K,
                                      int32_t row_offset, int32_t* d_ids, float* d_vals,
                                      int32_t* d_count, void* stream) {
    if (K <= 0 || K > kNoallocMaxK)
        return fail(MARS_ERR_CAPACITY, "mars_scan_topk_noalloc: K must be in [1, " +
                                           std::to_string(kNoallocMaxK) + "]");
    if (n < 0 || dim <= 0 || dim > 1024 || (dim & 3) != 0 || row_pitch < dim || (row_pitch & 3) != 0)
        return fail(MARS_ERR_INVALID, "mars_scan_topk_noalloc: need n >= 0, dim a multiple of 4 "
                                      "in (0, 1024], row_pitch >= dim and a multiple of 4");
    if (d_query == nullptr || d_ids == nullptr || d_vals == nullptr ||
        (n > 0 && (d_embeddings == nullptr || d_timestamps == nullptr)) ||
        (modality_filter >= 0 && n > 0 && d_modalities == nullptr))
        return fail(MARS_ERR_INVALID, "mars_scan_topk_noalloc: NULL argument");
    if (((reinterpret_cast<uintptr_t>(d_query) | reinterpret_cast<uintptr_t>(d_embeddings)) & 15u) != 0)
        return fail(MARS_ERR_INVALID, "mars_scan_topk_noalloc: embeddings and query must be 16-byte aligned");
    int dev = 0;
    MARS_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return fail(MARS_ERR_NO_DEVICE, "mars_scan_topk_noalloc: device index");
    DeviceSetup* ds = nullptr;
    MARS_TRY(setup_device(dev, &ds));
    cudaStream_t st = static_cast<cudaStream_t>(stream);

    const int nc = dim / 4;
    const int grid = std::min(ds->num_sms * scan_blocks_per_sm(nc, K), kNoallocMaxBlocks);
    noalloc_prepare_kernel<<<1, 1, 0, st>>>(n);
    MARS_CUDA_TRY(cudaGetLastError());

    ScanArgs sa{};
    sa.s.E = d_embeddings;
    sa.s.ts = d_timestamps;
    sa.s.imp = d_importance;
    sa.s.mod = d_modalities;
    sa.s.d_n = &ds->scratch->n;
    sa.s.pitch4 = row_pitch / 4;
    sa.s.nc = nc;
    sa.d.t_q = query_timestamp;
    sa.d.lambda = lambda;
    sa.d.filter = modality_filter;
    sa.d.use_imp = (use_importance != 0 && d_importance != nullptr) ? 1 : 0;
    sa.d.K = K;
    sa.d.row_offset = row_offset;
    sa.q = reinterpret_cast<const float4*>(d_query);
    sa.part_val = ds->scratch->part_val;
    sa.part_idx = ds->scratch->part_idx;
    sa.ticket = &ds->scratch->ticket;
    sa.cursor = &ds->scratch->cursor;
    sa.out_val = d_vals;
    sa.out_idx = d_ids;
    sa.out_cnt = d_count ? d_count : &ds->scratch->count;
    MARS_CUDA_TRY(launch_scan_topk(sa, K, grid, st));
    return MARS_OK;
}
