// Causal GQA prefill attention on the 5th-generation tensor cores (tcgen05, accumulators in
// tensor memory), over the paged fp16 KV cache.
//
// Same mathematics as k_flash_prefill (attn_prefill.cu) and the reference's
// GroupedQueryAttention::ForwardWithPrefix (Mac/cpu/src/grouped_query_attention.cpp:59-142):
// row r of the chunk is position start + r, it sees keys [0, start + r], query head h reads kv
// head h / (hq / hkv), scores q.k / sqrt(D) in base 2 (log2(e) folded into the query scale),
// online softmax over 128-key blocks, one division by the row sum at the end.  Q and P are fp16
// operands, accumulation is fp32 (as in the mma.sync kernel).
//
// CTA = 128 query rows of one head; 192 threads:
//   warps 0-3  one thread per row: stage Q (fp32 -> scaled fp16, 128-byte swizzle), then per
//              key block read S from tensor memory, mask, update the running max and sum,
//              rescale O in tensor memory when the max moved, write P (fp16, swizzled) and zero
//              the V rows past the last visible key; finally O / l to global memory.
//   warp 4     lane 0: TMA producer, two K/V slots; each block is 8 pages x (D / 64) boxes of
//              64 dims x 16 keys for K and for V (the cache's 2-D maps), pages past the last
//              visible key are fetched from a negative row and arrive as zeros.
//   warp 5     owns 256 tensor-memory columns (S: 128, O: D); lane 0 issues
//              S = Q K^T (M128 N128, K-major operands) and O += P V (M128 N=D, V MN-major).
// Every mbarrier wait is bounded (DERR_WAIT_TIMEOUT); the producer lets its copies land before
// the CTA exits and warp 5 frees tensor memory on every path.
//
// Status: compiled for sm_100a; not yet called by the library (it replaces launch_flash_prefill
// only once it matches it on a B200).
#include <cudaTypedefs.h>

#include "kernels.h"

namespace socb {
namespace {

constexpr int TBM = 128;         // query rows per CTA
constexpr int TBN = 128;         // keys per block
constexpr int T_THREADS = 192;
constexpr int REGION = 128 * 128;  // bytes of one [128 rows x 64 fp16] 128-byte-swizzled region
constexpr unsigned long long T_WAIT_NS = 2000000000ull;

struct TBars {
    unsigned long long kv_full[2], kv_empty[2], s_full, p_full, o_done;
    uint32_t tmem;
};

__device__ __forceinline__ uint32_t s32a(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ bool t_try(unsigned long long* b, unsigned parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(s32a(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool t_wait(unsigned long long* b, unsigned parity, int* err) {
    unsigned long long t0 = 0;
    for (unsigned i = 0;; ++i) {
        if (t_try(b, parity)) return true;
        if ((i & 255u) == 255u) {
            if (*reinterpret_cast<volatile int*>(err) & DERR_WAIT_TIMEOUT) return false;
            unsigned long long now;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
            if (t0 == 0) {
                t0 = now;
            } else if (now - t0 > T_WAIT_NS) {
                atomicOr(err, DERR_WAIT_TIMEOUT);
                return false;
            }
        }
    }
}
__device__ __forceinline__ void t_init(unsigned long long* b, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(s32a(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void t_arrive(unsigned long long* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(s32a(b)) : "memory");
}
__device__ __forceinline__ void t_commit(unsigned long long* b) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(s32a(b))
                 : "memory");
}
__device__ __forceinline__ void t_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void t_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// K-major operand, 128-byte swizzle: 128-byte rows, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t desc_k(uint32_t saddr) {
    return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(1) << 16) |
           (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
           (static_cast<uint64_t>(2) << 61);
}
// MN-major operand, 128-byte swizzle (V as the B operand of P V): 64 contiguous N elements
// per 128-byte row, rows along K; 8-row K groups 1024 bytes apart (stride byte offset), the
// next 64 N elements one region further (leading byte offset).
__device__ __forceinline__ uint64_t desc_mn(uint32_t saddr) {
    return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(REGION >> 4) << 16) |
           (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
           (static_cast<uint64_t>(2) << 61);
}
// kind::f16 instruction descriptor: fp32 accumulator, fp16 A and B, B MN-major when asked.
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n, bool b_mn) {
    return (1u << 4) | (b_mn ? (1u << 16) : 0u) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(m >> 4) << 24);
}
__device__ __forceinline__ void t_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void t_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void t_st32(uint32_t taddr, const float (&v)[32]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
                 "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])), "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
                 : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t pack2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
// 16-byte chunk `c` (8 fp16 values) of row `r` in a 128-byte-swizzled K-major tile whose rows
// are `width` values wide (one 16 KB region per 64 values).
__device__ __forceinline__ uint32_t sw_chunk(int r, int c) {
    return static_cast<uint32_t>((c >> 3) * REGION + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

template <int D>
__global__ void __launch_bounds__(T_THREADS, 1)
    k_flash_prefill_tc(const float* __restrict__ q, int n, int hq, int hkv, int seq, int start, KVLayerView kv,
                       float qscale, float* __restrict__ out, const __grid_constant__ CUtensorMap tk,
                       const __grid_constant__ CUtensorMap tv, int* err) {
    pdl_enter();
    constexpr int QR = D / 64;                // regions of a Q / K / V row
    constexpr int KV_BYTES = QR * REGION;     // one K (or V) block of 128 keys
    constexpr int O_COL = TBN;                // O accumulator columns [128, 128 + D)
    extern __shared__ uint8_t tc_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tc_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* qs = sm;                               // [QR][128 rows x 128 B]
    uint8_t* ks = qs + KV_BYTES;                    // [2 slots][QR regions]
    uint8_t* vs = ks + 2 * KV_BYTES;                // [2 slots][QR regions]
    uint8_t* ps = vs + 2 * KV_BYTES;                // [2 regions] P, 128 rows x 128 keys
    TBars* bars = reinterpret_cast<TBars*>(ps + 2 * REGION);

    // CTAs start in blockIdx order, x fastest: every head's longest causal extent comes first, then
    // every head's next longest, so the heaviest CTAs never wait for a second wave
    const int qb = gridDim.y - 1 - blockIdx.y;
    const int head = blockIdx.x, kvh = head / (hq / hkv);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = qb * TBM;
    const int last_row = min(n, r0 + TBM) - 1;
    const int kv_end = start + last_row + 1;  // keys [0, kv_end) are visible to some row here
    const int nkb = (kv_end + TBN - 1) / TBN;
    const int qw = hq * D;

    if (threadIdx.x == 0) {
        for (int s = 0; s < 2; ++s) {
            t_init(&bars->kv_full[s], 1);
            t_init(&bars->kv_empty[s], 1);
        }
        t_init(&bars->s_full, 1);
        t_init(&bars->p_full, TBM);
        t_init(&bars->o_done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 5) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 256;" ::"r"(s32a(&bars->tmem))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (warp < 4) {  // stage Q: row t, scaled, fp16, swizzled (zeros past the chunk)
        const int t = threadIdx.x, row = r0 + t;
#pragma unroll 1
        for (int c = 0; c < D / 8; ++c) {
            float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
            if (row < n) {
                const float* p = q + static_cast<size_t>(row) * qw + head * D + c * 8;
                a = *reinterpret_cast<const float4*>(p);
                b = *reinterpret_cast<const float4*>(p + 4);
            }
            const uint4 h = make_uint4(pack2(a.x * qscale, a.y * qscale), pack2(a.z * qscale, a.w * qscale),
                                       pack2(b.x * qscale, b.y * qscale), pack2(b.z * qscale, b.w * qscale));
            *reinterpret_cast<uint4*>(qs + sw_chunk(t, c)) = h;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    t_fence_before();
    __syncthreads();
    t_fence_after();
    const uint32_t tmem = bars->tmem;

    if (warp == 4) {
        if (lane == 0) {  // TMA producer
            const int* pt = kv.page_table + static_cast<size_t>(seq) * kv.max_pages;
            const int pages_used = (kv_end + 15) / 16;
            int j = 0;
            for (; j < nkb; ++j) {
                const int s = j & 1;
                if (!t_wait(&bars->kv_empty[s], ((j >> 1) & 1u) ^ 1u, err)) break;
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(s32a(&bars->kv_full[s])),
                             "r"(2 * KV_BYTES)
                             : "memory");
#pragma unroll 1
                for (int i = 0; i < TBN / 16; ++i) {
                    const int pg = j * (TBN / 16) + i;
                    // a page with no visible key comes from row -16: all out of bounds, zeros
                    const int y = pg < pages_used ? kv.row0 + (pt[pg] * hkv + kvh) * 16 : -16;
#pragma unroll
                    for (int r = 0; r < QR; ++r) {
                        const uint32_t off = static_cast<uint32_t>(s * KV_BYTES + r * REGION + i * 2048);
                        asm volatile(
                            "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
                                s32a(ks + off)),
                            "l"(&tk), "r"(s32a(&bars->kv_full[s])), "r"(r * 64), "r"(y)
                            : "memory");
                        asm volatile(
                            "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
                                s32a(vs + off)),
                            "l"(&tv), "r"(s32a(&bars->kv_full[s])), "r"(r * 64), "r"(y)
                            : "memory");
                    }
                }
            }
            // never leave with copies in flight (bounded)
            for (int i = j > 2 ? j - 2 : 0; i < j; ++i) t_wait(&bars->kv_full[i & 1], (i >> 1) & 1u, err);
        }
    } else if (warp == 5) {
        if (lane == 0) {  // MMA issuer
            constexpr uint32_t id_s = idesc_f16(TBM, TBN, false), id_o = idesc_f16(TBM, D, true);
            const uint32_t tS = tmem, tO = tmem + O_COL;
            for (int j = 0; j < nkb; ++j) {
                const int s = j & 1;
                if (!t_wait(&bars->kv_full[s], (j >> 1) & 1u, err)) break;
                t_fence_after();
                const uint32_t q0 = s32a(qs), k0 = s32a(ks + s * KV_BYTES);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t off = static_cast<uint32_t>((kk >> 2) * REGION + (kk & 3) * 32);
                    t_mma(tS, desc_k(q0 + off), desc_k(k0 + off), id_s, kk > 0 ? 1u : 0u);
                }
                t_commit(&bars->s_full);
                if (!t_wait(&bars->p_full, j & 1u, err)) break;
                t_fence_after();
                const uint32_t p0 = s32a(ps), v0 = s32a(vs + s * KV_BYTES);
#pragma unroll
                for (int kk = 0; kk < TBN / 16; ++kk) {
                    const uint32_t poff = static_cast<uint32_t>((kk >> 2) * REGION + (kk & 3) * 32);
                    t_mma(tO, desc_k(p0 + poff), desc_mn(v0 + kk * 2048), id_o, (j > 0 || kk > 0) ? 1u : 0u);
                }
                t_commit(&bars->kv_empty[s]);
                t_commit(&bars->o_done);
            }
        }
    } else {  // softmax warps: thread t = row r0 + t = tensor-memory lane t
        const int t = threadIdx.x, row = r0 + t, pos = start + row;
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
        float m = -INFINITY, l = 0.0f;
        // tcgen05.ld / st are warp-collective: every wait result is made warp-uniform first
        constexpr unsigned ALL = 0xffffffffu;
        bool ok = true;
        for (int j = 0; j < nkb && ok; ++j) {
            const int s = j & 1, kb = j * TBN;
            if (!__all_sync(ALL, t_wait(&bars->s_full, j & 1u, err))) {
                ok = false;
                break;
            }
            t_fence_after();
            float sv[TBN];
#pragma unroll
            for (int c = 0; c < TBN; c += 32) {
                float v[32];
                t_ld32(lane_base + c, v);
#pragma unroll
                for (int i = 0; i < 32; ++i) sv[c + i] = kb + c + i > pos ? -INFINITY : v[i];
            }
            float mx = m;
#pragma unroll
            for (int i = 0; i < TBN; ++i) mx = fmaxf(mx, sv[i]);
            // rows past the chunk see no key at all; keep their state finite
            const float mnew = mx == -INFINITY ? 0.0f : mx;
            const float corr = m == -INFINITY ? 0.0f : exp2f(m - mnew);
            if (j > 0) {
                // PV of the previous block has finished: O may be rescaled and P rewritten
                if (!__all_sync(ALL, t_wait(&bars->o_done, (j - 1) & 1u, err))) {
                    ok = false;
                    break;
                }
                t_fence_after();
                if (__any_sync(ALL, corr != 1.0f)) {
#pragma unroll 1
                    for (int c = 0; c < D; c += 32) {
                        float v[32];
                        t_ld32(lane_base + O_COL + c, v);
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] *= corr;
                        t_st32(lane_base + O_COL + c, v);
                    }
                }
            }
            m = mnew;
            float psum = 0.0f;
#pragma unroll
            for (int c = 0; c < TBN / 8; ++c) {
                float p[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float x = sv[c * 8 + i];
                    p[i] = x == -INFINITY ? 0.0f : exp2f(x - m);
                    psum += p[i];
                }
                *reinterpret_cast<uint4*>(ps + sw_chunk(t, c)) =
                    make_uint4(pack2(p[0], p[1]), pack2(p[2], p[3]), pack2(p[4], p[5]), pack2(p[6], p[7]));
            }
            l = l * corr + psum;
            // V rows past the last visible key hold whatever the cache had there: zero them
            if (kb + t >= kv_end) {
#pragma unroll
                for (int r = 0; r < QR; ++r) {
                    uint4* vr = reinterpret_cast<uint4*>(vs + s * KV_BYTES + r * REGION + t * 128);
#pragma unroll
                    for (int c = 0; c < 8; ++c) vr[c] = make_uint4(0u, 0u, 0u, 0u);
                }
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            t_fence_before();
            t_arrive(&bars->p_full);
        }
        if (ok && nkb > 0 && __all_sync(ALL, t_wait(&bars->o_done, (nkb - 1) & 1u, err))) {
            t_fence_after();
            const float inv = l > 0.0f ? 1.0f / l : 0.0f;
#pragma unroll 1
            for (int c = 0; c < D; c += 32) {
                float v[32];
                t_ld32(lane_base + O_COL + c, v);
                if (row < n) {
                    float* o = out + static_cast<size_t>(row) * qw + head * D + c;
#pragma unroll
                    for (int i = 0; i < 32; i += 4)
                        *reinterpret_cast<float4*>(o + i) =
                            make_float4(v[i] * inv, v[i + 1] * inv, v[i + 2] * inv, v[i + 3] * inv);
                }
            }
        }
    }
    t_fence_before();
    __syncthreads();
    if (warp == 5) {
        t_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;" ::"r"(tmem) : "memory");
    }
}

template <int D>
void flash_tc_d(const float* q, int n, int hq, int hkv, int seq, int start, const KVLayerView& kv, float* out,
                int* err, cudaStream_t st) {
    constexpr int QR = D / 64;
    constexpr int smem = 1024 + QR * REGION + 4 * QR * REGION + 2 * REGION + static_cast<int>(sizeof(TBars)) + 64;
    static_assert(smem <= 232448, "shared memory per CTA");
    static bool set = false;
    if (!set) {
        SOCB_CUDA(cudaFuncSetAttribute(k_flash_prefill_tc<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        set = true;
    }
    const float qscale = 1.4426950408889634f / sqrtf(static_cast<float>(D));
    dim3 grid(hq, (n + TBM - 1) / TBM);
    launch_pdl(k_flash_prefill_tc<D>, dim3(grid), dim3(T_THREADS), smem, st, q, n, hq, hkv, seq, start, kv, qscale,
               out, *kv.tmk, *kv.tmv, err);
}

}  // namespace

void launch_flash_prefill_tc(const float* q, int n, int hq, int hkv, int head_dim, int seq, int start,
                             const KVLayerView& kv, float* out, int* err, cudaStream_t st) {
    if (n <= 0) return;
    if (hq % hkv != 0) throw Error(-1, "attention: unsupported head grouping");
    if (kv.page_tokens != 16) throw Error(-1, "flash prefill expects 16-token pages");
    if (kv.tmk == nullptr || kv.tmv == nullptr) throw Error(-1, "tensor-core prefill attention needs the cache's TMA maps");
    if (head_dim == 128)
        flash_tc_d<128>(q, n, hq, hkv, seq, start, kv, out, err, st);
    else if (head_dim == 64)
        flash_tc_d<64>(q, n, hq, hkv, seq, start, kv, out, err, st);
    else
        throw Error(-1, "head_dim must be 64 or 128");
    SOCB_CUDA(cudaGetLastError());
    count_launches(1);
}

}  // namespace socb
