// mars_nccl.h -- NCCL resolved at run time.
//
// The library does not link against NCCL.  The first shard communicator
// opens "libnccl.so.2" with dlopen: in a process that already loaded NCCL
// (PyTorch links it by that soname) this returns the copy in use, so the
// library and its host share one NCCL; elsewhere the dynamic linker's search
// path finds the system's.  Only the types come from nccl.h.
#pragma once

#include <nccl.h>

namespace mars {

struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*);
    ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*);
    ncclResult_t (*CommFinalize)(ncclComm_t);
    ncclResult_t (*CommDestroy)(ncclComm_t);
    ncclResult_t (*CommAbort)(ncclComm_t);
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*);
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t);
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    const char* (*GetErrorString)(ncclResult_t);
    ncclResult_t (*GetVersion)(int*);
};

// The resolved API, or nullptr (with the reason in *why) when NCCL cannot be
// loaded.  Thread-safe; resolved once.
const NcclApi* nccl_api(const char** why);

}  // namespace mars
