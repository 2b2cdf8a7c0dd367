// Peer-memory all-reduce of the residual stream for tensor parallelism (tp_allreduce.cu).
#pragma once

#include <nccl.h>

#include <vector>

#include "common.cuh"

namespace socb {

// SOC_B200_TP_ALLREDUCE=p2p: use the peer-memory all-reduce instead of NCCL's (every rank must
// set the same).
bool tp_p2p_requested();

struct TpExchange {
    int rank = 0, tp = 1;
    size_t max_elems = 0;  // floats of h one all-reduce can carry (multiple of 4)
    size_t bytes = 0;
    float* own = nullptr;             // this rank's exchange buffer
    std::vector<float*> peers;        // every rank's buffer as mapped here (own at [rank])
    float** d_peers = nullptr;        // the same on the device
    unsigned epoch = 0;               // all-reduces so far (the same count on every rank)
    // Collective over `comm`: every rank calls it once, in the same order as its other collectives.
    void setup(ncclComm_t comm, int rank, int tp, size_t max_elems, cudaStream_t st);
    void release();
    // In-place sum of h[0, elems) over the ranks; elems <= max_elems and a multiple of 4.
    void all_reduce(float* h, size_t elems, int* err, cudaStream_t st);
};

}  // namespace socb
