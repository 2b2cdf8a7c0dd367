// Peer-memory all-reduce of the residual stream for tensor parallelism (tp_allreduce.cu).
#pragma once

#include <nccl.h>

#include <vector>

#include "common.cuh"

namespace socb {

// SOC_B200_TP_ALLREDUCE=p2p: use the peer-memory all-reduce instead of NCCL's (every rank must
// set the same).
bool tp_p2p_requested();

// Every rank's verdict on a local step, combined over `comm` (minimum of `ok`), with the
// host's wait for the collective bounded by `seconds`.  When the ranks do not all arrive in
// time (one of them died or never called), the communicator is aborted -- which ends the
// waiting NCCL kernel instead of leaving it on the GPU -- and Error is thrown.
bool tp_agree(ncclComm_t comm, bool ok, cudaStream_t st, double seconds = 60.0);

struct TpExchange {
    int rank = 0, tp = 1;
    size_t max_elems = 0;  // floats of h one all-reduce can carry (multiple of 4)
    size_t bytes = 0;
    float* own = nullptr;             // this rank's exchange buffer
    std::vector<float*> peers;        // every rank's buffer as mapped here (own at [rank])
    float** d_peers = nullptr;        // the same on the device
    unsigned epoch = 0;               // all-reduces so far (the same count on every rank)
    // Set after a bounded wait of an all-reduce gave up (DERR_WAIT_TIMEOUT): the epochs of the
    // ranks may then disagree, and two buffers no longer keep a read from seeing a slot of
    // another all-reduce, so a poisoned exchange is never used again (the model must be
    // reloaded).  A rank that stops waits out its peers' next all-reduce, which poisons
    // theirs in turn.
    bool poisoned = false;
    // Collective over `comm`: every rank calls it once, in the same order as its other
    // collectives, whether or not the rest of its own load succeeded (`load_ok`).  The
    // ranks agree (tp_agree) before each collective step, so a rank that failed earlier
    // makes every rank throw instead of leaving the others waiting.
    void setup(ncclComm_t comm, int rank, int tp, size_t max_elems, bool load_ok, cudaStream_t st);
    void release();
    // In-place sum of h[0, elems) over the ranks; elems <= max_elems and a multiple of 4.
    void all_reduce(float* h, size_t elems, int* err, cudaStream_t st);
};

}  // namespace socb
