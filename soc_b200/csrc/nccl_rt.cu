// Run-time binding of the few NCCL calls tensor parallelism needs (all-reduce of the
// residual stream, all-gather of vocab-shard argmax keys and logits, communicator set-up).
#include <dlfcn.h>

#include <mutex>
#include <string>

#include "common.cuh"
#include "nccl_rt.h"

namespace socb {

const NcclApi& nccl() {
    static NcclApi api{};
    static std::string error;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            error = std::string("cannot load libnccl.so.2: ") + dlerror();
            return;
        }
        auto sym = [&](const char* n) -> void* {
            void* p = dlsym(h, n);
            if (!p && error.empty()) error = std::string("libnccl.so.2 lacks ") + n;
            return p;
        };
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(sym("ncclCommInitRank"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
        api.comm_abort = reinterpret_cast<decltype(api.comm_abort)>(sym("ncclCommAbort"));
        api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(sym("ncclAllReduce"));
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(sym("ncclAllGather"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
    });
    if (!error.empty()) throw Error(-2, error);
    return api;
}

void nccl_check(ncclResult_t r, const char* what) {
    if (r != ncclSuccess)
        throw Error(-2, std::string("NCCL error in ") + what + ": " + nccl().error_string(r));
}

}  // namespace socb
