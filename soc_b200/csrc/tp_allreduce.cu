// One-shot all-reduce of the residual stream over NVLink peer memory, for tensor-parallel
// decode (the sum after the row-parallel o_proj / down_proj).
//
// Every rank owns one exchange buffer (cudaMalloc, shared with the other ranks through CUDA IPC
// handles that NCCL all-gathers once at load time):
//   data  [2 buffers][tp writers][max_elems] fp32
//   flags [2 buffers][tp writers] u32, one 128-byte line each, + [2] CTA arrival counters
// All-reduce number e (epochs 1, 2, ... counted by the host, the same on every rank) uses
// buffer b = e & 1:
//   1. each CTA stores its slice of this rank's h into slot [b][rank] of every rank's buffer
//      (plain stores over NVLink; its own buffer too);
//   2. the last CTA to finish (a local arrival counter) fences at system scope and writes
//      flag [b][rank] = e into every rank's buffer with release semantics;
//   3. every CTA waits until all tp flags [b][*] of its own buffer reach e (acquire, bounded),
//      then sums the tp slots of its slice in rank order into h.
// A rank can write epoch e + 1 into buffer (e + 1) & 1 only after it saw every rank's flag
// for e, i.e. after every rank finished all-reduce e - 1, the last reader of that buffer; so
// two buffers suffice.  The CTAs of one launch wait on one another (step 2 -> 3), so the
// kernel is launched cooperatively (all CTAs resident).  Waits give up after 2 s with
// DERR_WAIT_TIMEOUT.  Plain peer loads and stores only, and no TMA on peer memory.
//
// Opt-in (SOC_B200_TP_ALLREDUCE=p2p at load time, on every rank); rows beyond the buffer's
// capacity still go through NCCL.  Validated on 2 GPUs (the tensor-parallel parity test).
#include <chrono>
#include <cstdlib>
#include <string>
#include <thread>
#include <vector>

#include "../../include/soc_b200.h"
#include "kernels.h"
#include "nccl_rt.h"
#include "tp_allreduce.h"

namespace socb {
namespace {

constexpr int AR_CTAS = 32, AR_THREADS = 256;
constexpr int FLAG_WORDS = 32;  // one 128-byte line per flag
constexpr unsigned long long AR_WAIT_NS = 2000000000ull;

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__global__ void __launch_bounds__(AR_THREADS) k_tp_allreduce(float* __restrict__ h, int n, float* const* bufs,
                                                              int rank, int tp, size_t max_elems, unsigned epoch,
                                                              int* err) {
    const int b = static_cast<int>(epoch & 1u);
    const size_t data_elems = 2 * static_cast<size_t>(tp) * max_elems;
    auto flag = [&](float* base, int buf, int writer) {
        return reinterpret_cast<unsigned*>(base + data_elems) + (buf * tp + writer) * FLAG_WORDS;
    };
    float* mine = bufs[rank];
    unsigned* arrivals = flag(mine, 2, 0) + b * FLAG_WORDS;  // [2] counters after the flags
    // this CTA's slice of h, in float4 (n is a multiple of 4)
    const int n4 = n / 4;
    const int per = (n4 + gridDim.x - 1) / gridDim.x;
    const int a = blockIdx.x * per, e = min(n4, a + per);
    const float4* src = reinterpret_cast<const float4*>(h);
    // 1. push the slice to every rank
    for (int p = 0; p < tp; ++p) {
        float4* dst = reinterpret_cast<float4*>(bufs[p] + (static_cast<size_t>(b) * tp + rank) * max_elems);
        for (int i = a + threadIdx.x; i < e; i += blockDim.x) dst[i] = src[i];
    }
    __syncthreads();
    // 2. the last CTA publishes this rank's flag everywhere
    if (threadIdx.x == 0) {
        __threadfence_system();
        const unsigned old = atomicAdd(arrivals, 1u);
        if (old == gridDim.x - 1) {
            *arrivals = 0;  // next use of this counter is epoch + 2, after this launch
            __threadfence_system();
            for (int p = 0; p < tp; ++p) st_release_sys(flag(bufs[p], b, rank), epoch);
        }
    }
    // 3. wait for every rank's flag in this rank's buffer, then sum the slots in rank order
    if (threadIdx.x == 0) {
        unsigned long long t0 = 0;
        for (int r = 0; r < tp; ++r) {
            const unsigned* f = flag(mine, b, r);
            for (unsigned i = 0; ld_acquire_sys(f) < epoch; ++i) {
                if ((i & 255u) == 255u) {
                    if (*reinterpret_cast<volatile int*>(err) & DERR_WAIT_TIMEOUT) break;
                    unsigned long long now;
                    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
                    if (t0 == 0) {
                        t0 = now;
                    } else if (now - t0 > AR_WAIT_NS) {
                        atomicOr(err, DERR_WAIT_TIMEOUT);
                        break;
                    }
                }
                __nanosleep(64);
            }
        }
    }
    __syncthreads();
    float4* out = reinterpret_cast<float4*>(h);
    for (int i = a + threadIdx.x; i < e; i += blockDim.x) {
        float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int r = 0; r < tp; ++r) {
            const float4 v = __ldcv(reinterpret_cast<const float4*>(mine + (static_cast<size_t>(b) * tp + r) * max_elems) + i);
            s.x += v.x;
            s.y += v.y;
            s.z += v.z;
            s.w += v.w;
        }
        out[i] = s;
    }
}

}  // namespace

bool tp_p2p_requested() {
    const char* e = std::getenv("SOC_B200_TP_ALLREDUCE");
    return e && std::string(e) == "p2p";
}

namespace {
// Device buffer freed on every exit path.
struct DevBuf {
    void* p = nullptr;
    explicit DevBuf(size_t bytes) { SOCB_CUDA(cudaMalloc(&p, bytes)); }
    ~DevBuf() {
        if (p) cudaFree(p);
    }
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
};

// Waits for `st` at most `seconds`; on expiry aborts `comm` (ending its pending kernels) and throws.
void wait_bounded(cudaStream_t st, ncclComm_t comm, double seconds, const char* what) {
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        const cudaError_t e = cudaStreamQuery(st);
        if (e == cudaSuccess) return;
        if (e != cudaErrorNotReady) SOCB_CUDA(e);
        const double waited = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (waited > seconds) {
            nccl().comm_abort(comm);
            cudaStreamSynchronize(st);
            throw Error(SOC_B200_ERR_DEVICE, std::string(what) + ": the other ranks did not join within " +
                                                 std::to_string(static_cast<int>(seconds)) +
                                                 " s; the NCCL communicator was aborted");
        }
        std::this_thread::sleep_for(std::chrono::milliseconds(1));
    }
}
}  // namespace

bool tp_agree(ncclComm_t comm, bool ok, cudaStream_t st, double seconds) {
    DevBuf d(sizeof(int));
    const int v = ok ? 1 : 0;
    SOCB_CUDA(cudaMemcpyAsync(d.p, &v, sizeof(int), cudaMemcpyHostToDevice, st));
    nccl_check(nccl().all_reduce(d.p, d.p, 1, ncclInt32, ncclMin, comm, st), "rank agreement all-reduce");
    wait_bounded(st, comm, seconds, "rank agreement");
    int all = 0;
    SOCB_CUDA(cudaMemcpy(&all, d.p, sizeof(int), cudaMemcpyDeviceToHost));
    return all == 1;
}

void TpExchange::setup(ncclComm_t comm, int rank_, int tp_, size_t max_elems_, bool load_ok, cudaStream_t st) {
    rank = rank_;
    tp = tp_;
    max_elems = max_elems_;
    const size_t data = 2 * static_cast<size_t>(tp) * max_elems;
    const size_t flags = (2 * static_cast<size_t>(tp) + 2) * FLAG_WORDS;
    bytes = (data + flags) * sizeof(float);
    // 1. local: the exchange buffer and its IPC handle (only when the rest of the load succeeded)
    cudaIpcMemHandle_t mine{};
    bool ok = load_ok;
    if (ok) {
        try {
            SOCB_CUDA(cudaMalloc(&own, bytes));
            SOCB_CUDA(cudaMemset(own, 0, bytes));
            SOCB_CUDA(cudaIpcGetMemHandle(&mine, own));
        } catch (const Error&) {
            ok = false;
        }
    }
    // 2. every rank agrees before the handle all-gather
    if (!tp_agree(comm, ok, st)) throw Error(SOC_B200_ERR_DEVICE, "peer all-reduce set-up failed on a rank");
    // 3. all-gather the 64-byte handles through NCCL (device buffers), bounded
    std::vector<cudaIpcMemHandle_t> all(tp);
    {
        DevBuf d_h(sizeof(cudaIpcMemHandle_t) * (tp + 1));
        char* hb = static_cast<char*>(d_h.p);
        SOCB_CUDA(cudaMemcpy(hb + sizeof(cudaIpcMemHandle_t) * tp, &mine, sizeof(mine), cudaMemcpyHostToDevice));
        nccl_check(nccl().all_gather(hb + sizeof(cudaIpcMemHandle_t) * tp, hb, sizeof(cudaIpcMemHandle_t), ncclInt8,
                                     comm, st),
                   "exchange-buffer handle all-gather");
        wait_bounded(st, comm, 60.0, "exchange-buffer handle all-gather");
        SOCB_CUDA(cudaMemcpy(all.data(), hb, sizeof(cudaIpcMemHandle_t) * tp, cudaMemcpyDeviceToHost));
    }
    // 4. local: map the peers' buffers
    peers.assign(tp, nullptr);
    ok = true;
    try {
        for (int p = 0; p < tp; ++p) {
            if (p == rank) {
                peers[p] = own;
                continue;
            }
            void* ptr = nullptr;
            SOCB_CUDA(cudaIpcOpenMemHandle(&ptr, all[p], cudaIpcMemLazyEnablePeerAccess));
            peers[p] = static_cast<float*>(ptr);
        }
        SOCB_CUDA(cudaMalloc(&d_peers, sizeof(float*) * tp));
        SOCB_CUDA(cudaMemcpy(d_peers, peers.data(), sizeof(float*) * tp, cudaMemcpyHostToDevice));
    } catch (const Error&) {
        ok = false;
    }
    // 5. every rank mapped every buffer, or none uses the exchange
    if (!tp_agree(comm, ok, st)) throw Error(SOC_B200_ERR_DEVICE, "peer all-reduce set-up failed on a rank");
    epoch = 0;
    poisoned = false;
}

void TpExchange::release() {
    for (int p = 0; p < static_cast<int>(peers.size()); ++p)
        if (p != rank && peers[p]) cudaIpcCloseMemHandle(peers[p]);
    peers.clear();
    if (d_peers) cudaFree(d_peers);
    if (own) cudaFree(own);
    d_peers = nullptr;
    own = nullptr;
}

void TpExchange::all_reduce(float* h, size_t elems, int* err, cudaStream_t st) {
    if (poisoned)
        throw Error(SOC_B200_ERR_DEVICE, "peer all-reduce: an earlier exchange timed out; reload the model");
    if (elems > max_elems || elems % 4 != 0) throw Error(SOC_B200_ERR_INVALID, "peer all-reduce: size outside the buffer");
    unsigned e = ++epoch;
    int n = static_cast<int>(elems);
    float* const* bufs = d_peers;
    int r = rank, t = tp;
    size_t me = max_elems;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.gridDim = dim3(AR_CTAS);
    cfg.blockDim = dim3(AR_THREADS);
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    SOCB_CUDA(cudaLaunchKernelEx(&cfg, k_tp_allreduce, h, n, bufs, r, t, me, e, err));
    count_launches(1);
}

}  // namespace socb
