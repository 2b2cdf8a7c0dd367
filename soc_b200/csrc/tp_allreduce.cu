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
// capacity still go through NCCL.  Not yet run on a GPU.
#include <cstdlib>
#include <string>
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

void TpExchange::setup(ncclComm_t comm, int rank_, int tp_, size_t max_elems_, cudaStream_t st) {
    rank = rank_;
    tp = tp_;
    max_elems = max_elems_;
    const size_t data = 2 * static_cast<size_t>(tp) * max_elems;
    const size_t flags = (2 * static_cast<size_t>(tp) + 2) * FLAG_WORDS;
    bytes = (data + flags) * sizeof(float);
    SOCB_CUDA(cudaMalloc(&own, bytes));
    SOCB_CUDA(cudaMemset(own, 0, bytes));
    cudaIpcMemHandle_t mine{};
    SOCB_CUDA(cudaIpcGetMemHandle(&mine, own));
    // all-gather the 64-byte handles through NCCL (device buffers)
    char* d_h = nullptr;
    SOCB_CUDA(cudaMalloc(&d_h, sizeof(cudaIpcMemHandle_t) * (tp + 1)));
    SOCB_CUDA(cudaMemcpy(d_h + sizeof(cudaIpcMemHandle_t) * tp, &mine, sizeof(mine), cudaMemcpyHostToDevice));
    nccl_check(nccl().all_gather(d_h + sizeof(cudaIpcMemHandle_t) * tp, d_h, sizeof(cudaIpcMemHandle_t), ncclInt8,
                                 comm, st),
               "exchange-buffer handle all-gather");
    std::vector<cudaIpcMemHandle_t> all(tp);
    SOCB_CUDA(cudaStreamSynchronize(st));
    SOCB_CUDA(cudaMemcpy(all.data(), d_h, sizeof(cudaIpcMemHandle_t) * tp, cudaMemcpyDeviceToHost));
    cudaFree(d_h);
    peers.assign(tp, nullptr);
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
    epoch = 0;
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
