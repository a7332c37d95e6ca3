// Lazy NCCL binding: the engine only needs NCCL for tensor parallelism, so libnccl is
// opened with dlopen on first use instead of being a link-time dependency. Whichever
// libnccl.so.2 the process already has loaded (e.g. PyTorch's) is reused.
#pragma once

#include <nccl.h>

namespace jinf {

struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
    bool ok = false;
};

// Returns nullptr (and logs) if libnccl cannot be loaded.
const NcclApi* nccl_api();

}  // namespace jinf
