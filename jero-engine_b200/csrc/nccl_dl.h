// nccl_dl.h -- NCCL entry points resolved at run time (dlopen of libnccl.so.2).
//
// The library links no NCCL: a host process that already loaded one (PyTorch
// bundles its own) shares it, and a process without one loads the system
// libnccl.so.2 on first use. Only the calls of the expert-parallel exchange
// are resolved.
#pragma once

#include <cuda_runtime.h>
#include <nccl.h>

namespace jmoe {

struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId *);
    ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int);
    ncclResult_t (*CommDestroy)(ncclComm_t);
    ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*Send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*Recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*GroupStart)();
    ncclResult_t (*GroupEnd)();
    const char *(*GetErrorString)(ncclResult_t);
};

// nullptr when no libnccl.so.2 can be loaded or a symbol is missing; *why
// (optional) then names the failure.
const NcclApi *nccl_api(const char **why = nullptr);

}  // namespace jmoe
