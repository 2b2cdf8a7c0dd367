// NCCL entry points, resolved at run time from libnccl.so.2 (the copy the process already
// loaded, e.g. torch's, or the system one), so the library links without NCCL.
#pragma once

#include <nccl.h>

namespace socb {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*);
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int);
    ncclResult_t (*comm_destroy)(ncclComm_t);
    ncclResult_t (*comm_abort)(ncclComm_t);
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    const char* (*error_string)(ncclResult_t);
};

// Throws Error(SOC_B200_ERR_CUDA) when libnccl.so.2 or one of its symbols is missing.
const NcclApi& nccl();
void nccl_check(ncclResult_t r, const char* what);

}  // namespace socb
