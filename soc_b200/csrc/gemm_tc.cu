// Persistent tcgen05 GEMM for sm_100a: y = epilogue(A W^T), A [M, K] activations and
// W [N, K] weights (fp16 or bf16, K-major), fp32 accumulation in tensor memory.
//
// Restates Linear::Forward (Mac/cpu/src/linear.cpp:51-84) for many rows at once; the
// SwiGLU epilogue is ApplySiLU * up (qwen_mlp.cpp:20-54), the residual epilogue the
// AddTensors of the block (qwen_block.cpp:19-34).
//
// One CTA per SM walks the 128 x 256 output tiles (m fastest, so concurrently running CTAs
// share the weight tile in L2).  Warp 0 lane 0 streams 64-column slices of A and W with
// 2-D TMA (128-byte swizzle) into a 4-stage shared-memory ring; warp 1 owns 512 TMEM
// columns (two 256-column accumulators) and lane 0 issues tcgen05.mma (M128 N256 K16, four
// per slice), releasing each ring slot with tcgen05.commit; warps 2-5 drain the other
// accumulator with tcgen05.ld while the next tile accumulates.  Every mbarrier wait is
// bounded: on expiry the kernel records DERR_WAIT_TIMEOUT, stops issuing, frees TMEM and
// returns.  Every TMA load fills only this CTA's own shared memory.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <string>

#include "gemm_tc.h"
#include "kernels.h"

namespace socb {
namespace {

constexpr int BM = 128, BN = 256, BK = 64, MAX_STAGES = 4;
constexpr int A_BYTES = BM * BK * 2, W_BYTES = BN * BK * 2;
// Split mode carries the activations as hi + lo halves (x = hi + lo, both fp16/bf16) and
// issues two MMAs per K step, which keeps about twice the input significand bits.
template <bool SPLIT>
struct TcCfg {
    static constexpr int A_TILES = SPLIT ? 2 : 1;
    static constexpr int STAGE_BYTES = A_TILES * A_BYTES + W_BYTES;
    static constexpr int STAGES = SPLIT ? 3 : 4;
};
static_assert(TcCfg<true>::STAGES * TcCfg<true>::STAGE_BYTES <= MAX_STAGES * (A_BYTES + W_BYTES), "ring size");
constexpr int TC_THREADS = 192;
constexpr unsigned long long WAIT_NS = 2000000000ull;  // 2 s
constexpr int RING_BYTES = MAX_STAGES * (A_BYTES + W_BYTES);
// fp32 outputs leave through shared memory: per epilogue warp two 32 x 32 fp32 staging
// tiles (128-byte swizzle) that TMA stores (or reduce-adds, for the residual) to global.
constexpr int STG_BYTES = 32 * 32 * 4;
constexpr int STG_TOTAL = 4 * 2 * STG_BYTES;
constexpr size_t TC_SMEM = RING_BYTES + STG_TOTAL + 1024 /* barriers */ + 1024 /* alignment */;
static_assert(TC_SMEM <= 232448, "shared memory per CTA");

struct TcBars {
    unsigned long long full[MAX_STAGES], empty[MAX_STAGES], acc_full[2], acc_empty[2];
    uint32_t tmem;
};

__device__ __forceinline__ uint32_t su32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void mbar_init(unsigned long long* b, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ bool mbar_try(unsigned long long* b, unsigned parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(su32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait for the phase with `parity` (WAIT_NS of wall time); false once this or
// another thread of the grid gave up.
__device__ __forceinline__ bool mbar_wait(unsigned long long* b, unsigned parity, int* err) {
    unsigned long long t0 = 0;
    for (unsigned i = 0;; ++i) {
        if (mbar_try(b, parity)) return true;
        if ((i & 255u) == 255u) {
            if (*reinterpret_cast<volatile int*>(err) & DERR_WAIT_TIMEOUT) return false;
            const unsigned long long now = gtimer();
            if (t0 == 0) {
                t0 = now;
            } else if (now - t0 > WAIT_NS) {
                atomicOr(err, DERR_WAIT_TIMEOUT);
                return false;
            }
        }
    }
}
__device__ __forceinline__ void mbar_expect_tx(unsigned long long* b, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(unsigned long long* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, unsigned long long* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            su32(dst)),
        "l"(map), "r"(su32(bar)), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor of a K-major tile written by TMA with 128-byte swizzle:
// rows of 128 bytes, 8-row groups 1024 bytes apart (stride byte offset), version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(1) << 16) |
           (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
           (static_cast<uint64_t>(2) << 61);
}
// Instruction descriptor: fp32 accumulator, A/B type (0 fp16, 1 bf16), both K-major, N, M.
__host__ __device__ constexpr uint32_t f16_idesc(uint32_t ab, int m, int n) {
    return (1u << 4) | (ab << 7) | (ab << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(m >> 4) << 24);
}
__device__ __forceinline__ void umma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void umma_commit(unsigned long long* b) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(b))
                 : "memory");
}
// 32 lanes x 32 consecutive fp32 columns of tensor memory (one row per thread).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

template <typename T>
__device__ __forceinline__ T to_w(float f);
template <>
__device__ __forceinline__ __half to_w<__half>(float f) { return __float2half_rn(f); }
template <>
__device__ __forceinline__ __nv_bfloat16 to_w<__nv_bfloat16>(float f) { return __float2bfloat16_rn(f); }

template <typename T>
__device__ __forceinline__ void store_half(T* hi, T* lo, size_t i, float f) {
    const T h = to_w<T>(f);
    hi[i] = h;
    if (lo != nullptr) lo[i] = to_w<T>(f - static_cast<float>(h));
}

// 8 consecutive values -> 8 T in one 16-byte store (and their remainders when lo != null).
template <typename T>
__device__ __forceinline__ void store8_half(T* hi, T* lo, const float* f) {
    uint4 ph, pl;
    uint32_t* h = reinterpret_cast<uint32_t*>(&ph);
    uint32_t* l = reinterpret_cast<uint32_t*>(&pl);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const T a = to_w<T>(f[2 * j]), b = to_w<T>(f[2 * j + 1]);
        h[j] = static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&a)) |
               (static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&b)) << 16);
        if (lo != nullptr) {
            const T c = to_w<T>(f[2 * j] - static_cast<float>(a)), d = to_w<T>(f[2 * j + 1] - static_cast<float>(b));
            l[j] = static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&c)) |
                   (static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&d)) << 16);
        }
    }
    *reinterpret_cast<uint4*>(hi) = ph;
    if (lo != nullptr) *reinterpret_cast<uint4*>(lo) = pl;
}

template <typename T>
__device__ __forceinline__ bool aligned16(const void* p) {
    return (reinterpret_cast<uintptr_t>(p) & 15) == 0;
}

template <typename T>
__device__ __forceinline__ void epilogue(const float (&v)[32], int row, int col, int M, int N, void* y, void* y_lo,
                                         int ldy, int mode, int out_half) {
    if (row >= M) return;
    if (mode == LIN_SWIGLU) {
        const int o = col >> 1, no = N >> 1;
        if (out_half) {
            T* yr = static_cast<T*>(y) + static_cast<size_t>(row) * ldy;
            T* yl = y_lo ? static_cast<T*>(y_lo) + static_cast<size_t>(row) * ldy : nullptr;
            if (o + 16 <= no && aligned16<T>(yr + o) && (yl == nullptr || aligned16<T>(yl + o))) {
                float g[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) g[j] = silu_f(v[2 * j]) * v[2 * j + 1];
                store8_half<T>(yr + o, yl ? yl + o : nullptr, g);
                store8_half<T>(yr + o + 8, yl ? yl + o + 8 : nullptr, g + 8);
                return;
            }
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (o + j < no) store_half<T>(yr, yl, o + j, silu_f(v[2 * j]) * v[2 * j + 1]);
        } else {
            float* yr = static_cast<float*>(y) + static_cast<size_t>(row) * ldy;
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (o + j < no) yr[o + j] = silu_f(v[2 * j]) * v[2 * j + 1];
        }
        return;
    }
    if (out_half) {
        T* yr = static_cast<T*>(y) + static_cast<size_t>(row) * ldy;
        T* yl = y_lo ? static_cast<T*>(y_lo) + static_cast<size_t>(row) * ldy : nullptr;
        if (col + 32 <= N && aligned16<T>(yr + col) && (yl == nullptr || aligned16<T>(yl + col))) {
#pragma unroll
            for (int j = 0; j < 32; j += 8) store8_half<T>(yr + col + j, yl ? yl + col + j : nullptr, v + j);
            return;
        }
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (col + j < N) store_half<T>(yr, yl, col + j, v[j]);
        return;
    }
    float* yr = static_cast<float*>(y) + static_cast<size_t>(row) * ldy + col;
    const bool vec = col + 32 <= N && ((reinterpret_cast<uintptr_t>(yr) & 15) == 0);
    if (vec) {
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
            float4* p = reinterpret_cast<float4*>(yr + j);
            float4 o = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
            if (mode == LIN_RESIDUAL) {
                const float4 q = *p;
                o.x += q.x; o.y += q.y; o.z += q.z; o.w += q.w;
            }
            *p = o;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (col + j < N) yr[j] = mode == LIN_RESIDUAL ? yr[j] + v[j] : v[j];
    }
}

template <typename T, bool SPLIT>
__global__ void __launch_bounds__(TC_THREADS, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap ta_lo,
              const __grid_constant__ CUtensorMap tw, int M, int N, int K, void* __restrict__ y,
              void* __restrict__ y_lo, int ldy, int mode, int out_half, int ksplit,
              const __grid_constant__ CUtensorMap ty, int out_tma, int* err) {
    pdl_enter();
    using Cfg = TcCfg<SPLIT>;
    constexpr int STAGES = Cfg::STAGES, STAGE_BYTES = Cfg::STAGE_BYTES, W_OFF = Cfg::A_TILES * A_BYTES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    static_assert(STAGES * STAGE_BYTES <= RING_BYTES, "ring");
    TcBars* bars = reinterpret_cast<TcBars*>(smem + RING_BYTES + STG_TOTAL);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int mt = (M + BM - 1) / BM, nt = (N + BN - 1) / BN, tiles = mt * nt, kbn = (K + BK - 1) / BK;
    // Work unit u = (tile u % tiles, K slice u / tiles); with ksplit > 1 every slice writes
    // its fp32 partial tile to y + slice * M * N (ld N) for a separate reduction.
    const int kper = (kbn + ksplit - 1) / ksplit, units = tiles * ksplit;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&bars->full[s], 1);
            mbar_init(&bars->empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bars->acc_full[b], 1);
            mbar_init(&bars->acc_empty[b], 4);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(su32(&bars->tmem))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem;

    if (warp == 0) {
        if (lane == 0) {  // TMA producer
            unsigned it = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
                const int t = u % tiles, kb0 = (u / tiles) * kper, kb1 = min(kbn, kb0 + kper);
                const int m0 = (t % mt) * BM, n0 = (t / mt) * BN;
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const int s = static_cast<int>(it % STAGES);
                    if (!mbar_wait(&bars->empty[s], ((it / STAGES) & 1u) ^ 1u, err)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(&bars->full[s], STAGE_BYTES);
                    tma_load_2d(smem + s * STAGE_BYTES, &ta, &bars->full[s], kb * BK, m0);
                    if (SPLIT) tma_load_2d(smem + s * STAGE_BYTES + A_BYTES, &ta_lo, &bars->full[s], kb * BK, m0);
                    tma_load_2d(smem + s * STAGE_BYTES + W_OFF, &tw, &bars->full[s], kb * BK, n0);
                }
            }
            // Let the copies already issued land before the CTA can exit (bounded).
            const unsigned issued = it;
            for (unsigned j = issued > STAGES ? issued - STAGES : 0; j < issued; ++j)
                mbar_wait(&bars->full[j % STAGES], (j / STAGES) & 1u, err);
        }
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issuer
            constexpr uint32_t idesc = f16_idesc(sizeof(T) == 2 && __is_same(T, __nv_bfloat16) ? 1u : 0u, BM, BN);
            unsigned it = 0, local = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++local) {
                const int kb0 = (u / tiles) * kper, kb1 = min(kbn, kb0 + kper);
                const unsigned b = local & 1u;
                if (!mbar_wait(&bars->acc_empty[b], ((local >> 1) & 1u) ^ 1u, err)) break;
                tc_fence_after();
                const uint32_t d = tmem + b * BN;
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const int s = static_cast<int>(it % STAGES);
                    if (!mbar_wait(&bars->full[s], (it / STAGES) & 1u, err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = su32(smem + s * STAGE_BYTES), w0 = a0 + W_OFF;
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k) {
                        umma(d, sw128_desc(a0 + k * 32), sw128_desc(w0 + k * 32), idesc,
                             (kb != kb0 || k != 0) ? 1u : 0u);
                        if (SPLIT) umma(d, sw128_desc(a0 + A_BYTES + k * 32), sw128_desc(w0 + k * 32), idesc, 1u);
                    }
                    umma_commit(&bars->empty[s]);
                }
                umma_commit(&bars->acc_full[b]);
            }
        }
    } else {  // epilogue warps 2..5: TMEM lane quarter = warp % 4
        const int q = warp & 3;
        unsigned local = 0;
        const bool partial = ksplit > 1;
        uint8_t* stg = smem + RING_BYTES + q * 2 * STG_BYTES;
        unsigned sbuf = 0;
        for (int u = blockIdx.x; u < units; u += gridDim.x, ++local) {
            const int t = u % tiles;
            const unsigned b = local & 1u;
            if (!mbar_wait(&bars->acc_full[b], (local >> 1) & 1u, err)) break;
            tc_fence_after();
            const int m0 = (t % mt) * BM, n0 = (t / mt) * BN;
            void* yy = partial ? static_cast<void*>(static_cast<float*>(y) + static_cast<size_t>(u / tiles) * M * N) : y;
            const int row = m0 + q * 32 + lane;
            const uint32_t base = tmem + (static_cast<uint32_t>(q * 32) << 16) + b * BN;
#pragma unroll 1
            for (int c = 0; c < BN; c += 32) {
                if (n0 + c >= N) break;
                float v[32];
                tmem_ld32(base + c, v);
                if (out_tma) {
                    // row `lane` of the warp's 32 x 32 fp32 block -> swizzled staging tile -> TMA
                    uint8_t* buf = stg + (sbuf & 1) * STG_BYTES;
                    if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
                    __syncwarp();
                    float4* rowp = reinterpret_cast<float4*>(buf + lane * 128);
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        rowp[j ^ (lane & 7)] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    __syncwarp();
                    if (lane == 0) {
                        const int x = n0 + c, yr = m0 + q * 32;
                        if (partial)
                            asm volatile(
                                "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                                    &ty),
                                "r"(su32(buf)), "r"(x), "r"(yr), "r"(u / tiles)
                                : "memory");
                        else if (mode == LIN_RESIDUAL)
                            asm volatile(
                                "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                                    &ty),
                                "r"(su32(buf)), "r"(x), "r"(yr)
                                : "memory");
                        else
                            asm volatile(
                                "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(&ty),
                                "r"(su32(buf)), "r"(x), "r"(yr)
                                : "memory");
                        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                    }
                    ++sbuf;
                } else if (partial) {
                    epilogue<T>(v, row, n0 + c, M, N, yy, nullptr, N, LIN_STORE, 0);
                } else {
                    epilogue<T>(v, row, n0 + c, M, N, y, y_lo, ldy, mode, out_half);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->acc_empty[b]);
        }
        // every TMA store of this warp has written global memory before the CTA exits
        if (out_tma && lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
    }
}

// One CTA per row: optional RMSNorm (x * (1/sqrt(mean(x^2) + eps)) * w), cast to T; with
// out_lo also the remainder x' - float(T(x')) cast to T.  Each thread keeps up to RV float4
// of the row in registers between the sum of squares and the scaled store.
constexpr int R2H_RV = 4;
template <typename T>
__global__ void __launch_bounds__(1024) k_rows_to_half(const float* __restrict__ x, int ldx, int cols,
                                                       const float* __restrict__ w, float eps, T* __restrict__ out,
                                                       T* __restrict__ out_lo, int ldo) {
    pdl_enter();
    __shared__ float red[32];
    __shared__ float scale;
    const float* xr = x + static_cast<size_t>(blockIdx.x) * ldx;
    T* orow = out + static_cast<size_t>(blockIdx.x) * ldo;
    T* lrow = out_lo ? out_lo + static_cast<size_t>(blockIdx.x) * ldo : nullptr;
    const int n4 = cols >> 2;
    float4 v[R2H_RV];
    float ss = 0.0f;
#pragma unroll
    for (int u = 0; u < R2H_RV; ++u) {
        const int i = threadIdx.x + u * blockDim.x;
        v[u] = i < n4 ? reinterpret_cast<const float4*>(xr)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        ss += v[u].x * v[u].x + v[u].y * v[u].y + v[u].z * v[u].z + v[u].w * v[u].w;
    }
    float s = 1.0f;
    if (w != nullptr) {
        ss = warp_sum(ss);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
        __syncthreads();
        if (threadIdx.x < 32) {
            float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
            t = warp_sum(t);
            if (threadIdx.x == 0) scale = 1.0f / sqrtf(t / static_cast<float>(cols) + eps);
        }
        __syncthreads();
        s = scale;
    }
#pragma unroll
    for (int u = 0; u < R2H_RV; ++u) {
        const int i = threadIdx.x + u * blockDim.x;
        if (i >= n4) break;
        float f[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
        if (w != nullptr) {
            const float4 g = reinterpret_cast<const float4*>(w)[i];
            f[0] = f[0] * s * g.x;
            f[1] = f[1] * s * g.y;
            f[2] = f[2] * s * g.z;
            f[3] = f[3] * s * g.w;
        }
        uint2 ph, pl;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const T a = to_w<T>(f[2 * j]), b = to_w<T>(f[2 * j + 1]);
            (&ph.x)[j] = static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&a)) |
                         (static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&b)) << 16);
            const T c = to_w<T>(f[2 * j] - static_cast<float>(a)), d = to_w<T>(f[2 * j + 1] - static_cast<float>(b));
            (&pl.x)[j] = static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&c)) |
                         (static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&d)) << 16);
        }
        reinterpret_cast<uint2*>(orow)[i] = ph;
        if (lrow != nullptr) reinterpret_cast<uint2*>(lrow)[i] = pl;
    }
}

// Group-quantised [rows, cols] matrix -> T (q * scale rounded once), one 16-byte vector
// per thread per step.
template <int F, typename T>
__global__ void k_dequant(const uint8_t* __restrict__ W, const __half* __restrict__ S, size_t rows, int cols,
                          T* __restrict__ out) {
    pdl_enter();
    using C = Codec<F>;
    const size_t vpr = static_cast<size_t>(cols) / C::EPV, total = rows * vpr;
    const int ng = cols / C::GROUP;
    for (size_t v = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; v < total;
         v += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t r = v / vpr, vi = v - r * vpr;
        const uint4 u = *reinterpret_cast<const uint4*>(W + v * 16);
        const float sc = __half2float(S[r * ng + vi * C::EPV / C::GROUP]);
        T* o = out + r * cols + vi * C::EPV;
#pragma unroll
        for (int p = 0; p < C::EPV / 8; ++p) {
            float w8[8];
            C::part(u, p, w8);
            uint4 pk;
            uint32_t* pw = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const T lo = to_w<T>(w8[2 * j] * sc), hi = to_w<T>(w8[2 * j + 1] * sc);
                pw[j] = static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&lo)) |
                        (static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&hi)) << 16);
            }
            *reinterpret_cast<uint4*>(o + p * 8) = pk;
        }
    }
}

// Sum of the ksplit fp32 partial tiles [ksplit][M][N] followed by the GEMM epilogue; one
// thread per pair of columns.
template <typename T>
__global__ void k_splitk_reduce(const float* __restrict__ ws, int ksplit, int M, int N, void* __restrict__ y,
                                void* __restrict__ y_lo, int ldy, int mode, int out_half) {
    pdl_enter();
    const size_t pairs = static_cast<size_t>(M) * (N / 2);
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < pairs;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const int row = static_cast<int>(i / (N / 2)), p = static_cast<int>(i % (N / 2));
        float2 acc = make_float2(0.f, 0.f);
        for (int k = 0; k < ksplit; ++k) {
            const float2 v = *reinterpret_cast<const float2*>(ws + (static_cast<size_t>(k) * M + row) * N + 2 * p);
            acc.x += v.x;
            acc.y += v.y;
        }
        if (mode == LIN_SWIGLU) {
            const float g = silu_f(acc.x) * acc.y;
            if (out_half)
                store_half<T>(static_cast<T*>(y) + static_cast<size_t>(row) * ldy,
                              y_lo ? static_cast<T*>(y_lo) + static_cast<size_t>(row) * ldy : nullptr, p, g);
            else
                static_cast<float*>(y)[static_cast<size_t>(row) * ldy + p] = g;
        } else if (out_half) {
            T* yr = static_cast<T*>(y) + static_cast<size_t>(row) * ldy;
            T* yl = y_lo ? static_cast<T*>(y_lo) + static_cast<size_t>(row) * ldy : nullptr;
            store_half<T>(yr, yl, 2 * p, acc.x);
            store_half<T>(yr, yl, 2 * p + 1, acc.y);
        } else {
            float* yr = static_cast<float*>(y) + static_cast<size_t>(row) * ldy + 2 * p;
            if (mode == LIN_RESIDUAL) {
                yr[0] += acc.x;
                yr[1] += acc.y;
            } else {
                yr[0] = acc.x;
                yr[1] = acc.y;
            }
        }
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

}  // namespace

bool tc_available() { return encode_fn() != nullptr; }

int tc_min_rows() {
    const char* e = std::getenv("SOC_B200_TC_MIN_ROWS");
    return e && *e ? std::atoi(e) : 16;
}

bool tc_rows_ok(int rows, long long out_f, long long in_f, int wfmt) {
    const bool quant = wfmt == WF_I8G64 || wfmt == WF_I4G32;
    const char* e = std::getenv("SOC_B200_TC_MIN_ROWS");
    if (e && *e) {
        const int t = std::atoi(e);
        return t > 0 && rows >= (quant ? 2 * t : t);
    }
    // measured crossovers against the small-batch kernels (linear_mma.cu: fp16, int8, int4): below
    // 32 rows (fp16) those stream every Qwen3-0.6B shape faster, the lm_head included (fp16 at 16
    // rows: 7.0 against 12.6 us for 2048 x 1024, 71.8 against 77.1 us for the lm_head); int8 / int4,
    // whose GEMM route first expands the matrix to fp16, stay on them up to 63 rows (at 32 rows the
    // int8 lm_head takes 92.5 against 178.8 us, the 1-6 M-weight matrices 6-14 against 13-17 us).
    // bf16 has only the CUDA-core GEMV below the GEMM, which the GEMM beats from 16 rows.
    (void)out_f;
    (void)in_f;
    return rows >= (wfmt == WF_BF16 ? 16 : quant ? 64 : 32);
}

// SOC_B200_TC_OUT=registers keeps the fp32 GEMM outputs on the register-store epilogue.
int tc_out_tma() {
    const char* e = std::getenv("SOC_B200_TC_OUT");
    return (e && std::string(e) == "registers") ? 0 : 1;
}

int tc_split_max_rows() {
    const char* e = std::getenv("SOC_B200_TC_SPLIT_MAX_ROWS");
    return e && *e ? std::atoi(e) : 512;
}

void tc_make_map(CUtensorMap* map, const void* base, int wfmt, uint64_t rows, uint64_t cols, uint64_t ld,
                 uint32_t box_rows) {
    auto fn = encode_fn();
    if (!fn) throw Error(-2, "cuTensorMapEncodeTiled is not available from the driver");
    if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (ld * 2) % 16 != 0 || cols % 8 != 0)
        throw Error(-1, "tensor-core GEMM operands need 16-byte aligned rows");
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {ld * 2};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(BK), box_rows};
    const cuuint32_t es[2] = {1, 1};
    const CUresult r = fn(map, wfmt == WF_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                          const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw Error(-2, "cuTensorMapEncodeTiled failed with code " + std::to_string(static_cast<int>(r)));
}

// fp32 output descriptor for the TMA epilogue: [M, N] (ld `ld`), or [slices][M][N] for the
// split-K partials; 32 x 32 boxes with 128-byte swizzle.  False when the operand breaks the
// TMA alignment rules (the epilogue then stores from registers).
bool make_out_map(CUtensorMap* map, void* base, int M, int N, int ld, int slices) {
    auto fn = encode_fn();
    if (!fn || (reinterpret_cast<uintptr_t>(base) & 15) != 0 || ld % 4 != 0 || N % 4 != 0) return false;
    const cuuint32_t es[3] = {1, 1, 1};
    CUresult r;
    if (slices <= 1) {
        const cuuint64_t dims[2] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(M)};
        const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 4};
        const cuuint32_t box[2] = {32, 32};
        r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    } else {
        const cuuint64_t dims[3] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(M),
                                    static_cast<cuuint64_t>(slices)};
        const cuuint64_t strides[2] = {static_cast<cuuint64_t>(N) * 4, static_cast<cuuint64_t>(M) * N * 4};
        const cuuint32_t box[3] = {32, 32, 1};
        r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    }
    return r == CUDA_SUCCESS;
}

template <typename T, bool SPLIT>
static void gemm_t(const CUtensorMap& a, const CUtensorMap& a_lo, const CUtensorMap& w, int M, int N, int K, void* y,
                   void* y_lo, int ldy, int mode, bool out_half, int ksplit, float* ws, int* err, int grid,
                   cudaStream_t st) {
    static bool set = false;
    if (!set) {
        SOCB_CUDA(cudaFuncSetAttribute(k_gemm_tc<T, SPLIT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(TC_SMEM)));
        set = true;
    }
    CUtensorMap ty{};
    if (ksplit <= 1) {
        const bool tma = !out_half && mode != LIN_SWIGLU && tc_out_tma() && make_out_map(&ty, y, M, N, ldy, 1);
        launch_pdl(k_gemm_tc<T, SPLIT>, dim3(grid), dim3(TC_THREADS), TC_SMEM, st, a, a_lo, w, M, N, K, y, y_lo, ldy,
                   mode, out_half ? 1 : 0, 1, ty, tma ? 1 : 0, err);
        return;
    }
    const bool tma = tc_out_tma() && make_out_map(&ty, ws, M, N, N, ksplit);
    launch_pdl(k_gemm_tc<T, SPLIT>, dim3(grid), dim3(TC_THREADS), TC_SMEM, st, a, a_lo, w, M, N, K, ws, nullptr, N,
               LIN_STORE, 0, ksplit, ty, tma ? 1 : 0, err);
    const size_t pairs = static_cast<size_t>(M) * (N / 2);
    const int rgrid = static_cast<int>(std::min<size_t>((pairs + 255) / 256, 148 * 16));
    launch_pdl(k_splitk_reduce<T>, dim3(rgrid), dim3(256), 0, st, ws, ksplit, M, N, y, y_lo, ldy, mode,
               out_half ? 1 : 0);
}

void launch_gemm_tc(int wfmt, const CUtensorMap& a, const CUtensorMap* a_lo, const CUtensorMap& w, int M, int N,
                    int K, void* y, int ldy, int mode, bool out_half, void* y_lo, float* ws, size_t ws_floats,
                    int* err, cudaStream_t st) {
    if (M <= 0 || N <= 0) return;
    if (K <= 0 || K % BK != 0) throw Error(-1, "tensor-core GEMM needs K to be a multiple of 64");
    if (mode == LIN_SWIGLU && N % 2 != 0) throw Error(-1, "SwiGLU GEMM needs an even number of rows");
    if (mode == LIN_RESIDUAL && out_half) throw Error(-1, "residual GEMM output is fp32");
    if (y_lo != nullptr && !out_half) throw Error(-1, "a low-half output needs a half output");
    int dev = 0, sms = 0;
    SOCB_CUDA(cudaGetDevice(&dev));
    SOCB_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN), kbn = K / BK;
    // Split K when the output tiles cannot occupy the SMs (small M): partial tiles go to
    // the fp32 workspace and a reduction applies the epilogue.
    int ks = 1;
    if (ws != nullptr && tiles * 2 <= sms && N % 2 == 0) {
        ks = std::min(kbn, sms / tiles);
        while (ks > 1 && static_cast<size_t>(ks) * M * N > ws_floats) --ks;
        if (ks > 1) {
            const int kper = (kbn + ks - 1) / ks;
            ks = (kbn + kper - 1) / kper;  // no empty slices
        }
    }
    const int units = tiles * ks;
    const int grid = units < sms ? units : sms;
    const bool split = a_lo != nullptr;
    if (wfmt == WF_BF16) {
        if (split)
            gemm_t<__nv_bfloat16, true>(a, *a_lo, w, M, N, K, y, y_lo, ldy, mode, out_half, ks, ws, err, grid, st);
        else
            gemm_t<__nv_bfloat16, false>(a, a, w, M, N, K, y, y_lo, ldy, mode, out_half, ks, ws, err, grid, st);
    } else if (wfmt == WF_F16) {
        if (split)
            gemm_t<__half, true>(a, *a_lo, w, M, N, K, y, y_lo, ldy, mode, out_half, ks, ws, err, grid, st);
        else
            gemm_t<__half, false>(a, a, w, M, N, K, y, y_lo, ldy, mode, out_half, ks, ws, err, grid, st);
    } else {
        throw Error(-1, "tensor-core GEMM supports fp16 and bf16 weights");
    }
    SOCB_CUDA(cudaGetLastError());
    count_launches(ks > 1 ? 2 : 1);
}

void launch_rows_to_half(int wfmt, const float* x, int ldx, int rows, int cols, const float* norm_w, float eps,
                         void* out, void* out_lo, int ldo, cudaStream_t st) {
    if (rows <= 0) return;
    if (cols % 4 != 0 || ldx % 4 != 0 || ldo % 4 != 0) throw Error(-1, "row conversion needs multiples of 4 columns");
    const int n4 = cols / 4;
    int threads = (n4 + R2H_RV - 1) / R2H_RV;
    threads = (threads + 31) / 32 * 32;
    if (threads > 1024) throw Error(-1, "row conversion supports at most 16384 columns");
    if (threads < 32) threads = 32;
    if (wfmt == WF_BF16)
        launch_pdl(k_rows_to_half<__nv_bfloat16>, dim3(rows), dim3(threads), 0, st, x, ldx, cols, norm_w, eps,
                                                                static_cast<__nv_bfloat16*>(out),
                                                                static_cast<__nv_bfloat16*>(out_lo), ldo);
    else
        launch_pdl(k_rows_to_half<__half>, dim3(rows), dim3(threads), 0, st, x, ldx, cols, norm_w, eps,
                   static_cast<__half*>(out), static_cast<__half*>(out_lo), ldo);
    SOCB_CUDA(cudaGetLastError());
    count_launches(1);
}

void launch_dequant(int wfmt, const void* W, const void* scales, int rows, int cols, int out_fmt, void* out,
                    cudaStream_t st) {
    const int grid = 148 * 8;
    if (out_fmt != WF_F16) throw Error(-1, "dequantisation writes fp16");
    if (wfmt == WF_I8G64)
        launch_pdl(k_dequant<WF_I8G64, __half>, dim3(grid), dim3(256), 0, st, static_cast<const uint8_t*>(W),
                                                          static_cast<const __half*>(scales), rows, cols,
                                                          static_cast<__half*>(out));
    else if (wfmt == WF_I4G32)
        launch_pdl(k_dequant<WF_I4G32, __half>, dim3(grid), dim3(256), 0, st, static_cast<const uint8_t*>(W),
                                                          static_cast<const __half*>(scales), rows, cols,
                                                          static_cast<__half*>(out));
    else
        throw Error(-1, "dequantisation needs a group-quantised format");
    SOCB_CUDA(cudaGetLastError());
    count_launches(1);
}

}  // namespace socb
