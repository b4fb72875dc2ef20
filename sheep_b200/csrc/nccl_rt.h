// NCCL at run time: loaded (dlopen of libnccl.so.2) the first time an
// expert-parallel layer or a tensor-parallel engine with MoE layers needs it,
// so single-GPU users need no NCCL, and in a process that already loaded one
// (PyTorch's) the same library is reused.
#pragma once

#include <cuda_runtime.h>
#include <nccl.h>

namespace sb {

struct NcclApi {
    ncclResult_t (*get_id)(ncclUniqueId *);
    ncclResult_t (*init_rank)(ncclComm_t *, int, ncclUniqueId, int);
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*destroy)(ncclComm_t);
    const char * (*error)(ncclResult_t);
    // the all-to-all exchange
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*group_start)();
    ncclResult_t (*group_end)();
};

// The loaded entry points, or NULL when NCCL is unavailable.
const NcclApi * nccl_api();

}  // namespace sb
