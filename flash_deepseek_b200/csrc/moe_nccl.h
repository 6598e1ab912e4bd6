// moe_nccl.h -- NCCL entry points resolved at run time with dlopen, so that
// libmoe_cuda.so has no link-time dependency on a particular libnccl: a
// single-GPU context never loads NCCL, and an expert-parallel one reuses the
// libnccl.so.2 already in the process (e.g. the one bundled with PyTorch)
// before falling back to the system library (or MOE_NCCL_LIB).
#pragma once
#include <nccl.h>

struct MoeNccl {
    ncclResult_t (*GetUniqueId)(ncclUniqueId *);
    ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int);
    ncclResult_t (*CommDestroy)(ncclComm_t);
    ncclResult_t (*CommAbort)(ncclComm_t);
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *);
    ncclResult_t (*GroupStart)();
    ncclResult_t (*GroupEnd)();
    ncclResult_t (*Send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*Recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    const char *(*GetErrorString)(ncclResult_t);
};

// The loaded API, or nullptr (message on stderr) when no usable libnccl.
const MoeNccl *moe_nccl();
