// nccl_dl.h -- NCCL entry points resolved at run time.
//
// Expert parallelism is the only user of NCCL, so the library is opened with
// dlopen when lm_moe_ep_init first runs instead of being a link-time dependency:
// single-GPU users never load it, and a process that already holds a libnccl.so.2
// (PyTorch's, say) keeps using that one copy.
#pragma once

#include <nccl.h>

#include <string>

namespace lm {

struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    // Optional (NCCL >= 2.14): null when the loaded library lacks it.
    ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

// Loads libnccl.so.2 once; returns nullptr and sets `error` when it is missing.
const NcclApi* nccl_api(std::string& error);

}  // namespace lm
