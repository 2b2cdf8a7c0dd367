// Decode attention over the paged fp16 KV cache with bulk-copy (TMA) page streaming.
//
// Restates GroupedQueryAttention::ForwardWithPrefix (Mac/cpu/src/grouped_query_attention.cpp:59-142)
// for rows that each carry one query position (decode steps, short prefill tails): visible
// keys [0, pos] (:98), kv head = q head / (hq / hkv) (:101), scale 1/sqrt(D) (:81),
// max-subtracted softmax (:104-123).
//
// CTA = (row, kv head, key split of whole 16-token pages).  Warp 4 lane 0 streams each page
// of the split (K: 16 x D fp16 = 4 KB at D = 128, V the same) with cp.async.bulk into a ring
// of NSLOT shared-memory slots; warps 0-3 consume a page at a time: a group of LPK lanes
// owns one key (LPK = 8, or 16 for 4 or more query heads per kv head at D = 128), each lane
// DPL = D / LPK dims, and keeps an online softmax (base 2, log2(e) folded into the query
// scale) for the G query heads of the kv head.  The ring keeps NSLOT pages (48 KB) in flight
// per CTA without registers.  Groups and warps are merged in shared memory at the end; a
// split writes unnormalised partials (natural-log max, sum) for k_attn_combine.  Every
// mbarrier wait is bounded (2 s of %globaltimer): on expiry DERR_WAIT_TIMEOUT is recorded.
#include <cstdlib>
#include <string>

#include "kernels.h"

namespace socb {
namespace {

constexpr int NSLOT = 6;                 // ring slots of the lane-group kernel (every warp reads every page)
constexpr int CW = 4;                    // consumer warps
constexpr int NSLOT_MMA = 8;             // ring slots of the tensor-core kernel (a page per warp)
constexpr int AP_THREADS = (CW + 1) * 32;
constexpr unsigned long long AP_WAIT_NS = 2000000000ull;

__device__ __forceinline__ uint32_t su32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ unsigned long long gtime() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ bool mb_try(unsigned long long* b, unsigned parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(su32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mb_wait(unsigned long long* b, unsigned parity, int* err) {
    unsigned long long t0 = 0;
    for (unsigned i = 0;; ++i) {
        if (mb_try(b, parity)) return true;
        if ((i & 255u) == 255u) {
            if (*reinterpret_cast<volatile int*>(err) & DERR_WAIT_TIMEOUT) return false;
            const unsigned long long now = gtime();
            if (t0 == 0) {
                t0 = now;
            } else if (now - t0 > AP_WAIT_NS) {
                atomicOr(err, DERR_WAIT_TIMEOUT);
                return false;
            }
        }
    }
}

template <int D, int G>
__global__ void __launch_bounds__(AP_THREADS) k_attn_pages(const float* __restrict__ q, const int* __restrict__ row_seq,
                                                          const int* __restrict__ row_pos, int hq, int hkv,
                                                          KVLayerView kv, int n_splits, float* __restrict__ out,
                                                          float* __restrict__ part, int* err) {
    pdl_enter();
    constexpr int PT = 16;                    // tokens per page
    constexpr int PAGE_B = PT * D * 2;        // bytes of one kv head's K (or V) page
    constexpr int LPK = (G >= 4 && D >= 128) ? 16 : 8, DPL = D / LPK, NV = DPL / 8;
    constexpr int GPW = 32 / LPK, NG = CW * GPW, KPG = PT / NG;  // groups, keys per group per page
    extern __shared__ __align__(128) uint8_t sm[];
    uint8_t* ring = sm;                                                   // [NSLOT][K | V][PAGE_B]
    unsigned long long* full = reinterpret_cast<unsigned long long*>(sm + NSLOT * 2 * PAGE_B);
    unsigned long long* empty = full + NSLOT;
    float* mstate = reinterpret_cast<float*>(sm);  // reuses the ring after the loop: [NG][G][D + 2]

    const int row = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int seq = row_seq[row];
    const int nvis = row_pos[row] + 1;
    const int chunk = ((nvis + n_splits - 1) / n_splits + PT - 1) / PT * PT;
    const int kb = split * chunk, ke = min(nvis, kb + chunk);
    const int pg0 = kb / PT, npages = ke > kb ? (ke - kb + PT - 1) / PT : 0;
    const int* pt = kv.page_table + static_cast<size_t>(seq) * kv.max_pages;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NSLOT; ++s) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(full + s)) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(empty + s)), "r"(CW) : "memory");
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    __syncthreads();

    float m[G], l[G], o[G][DPL];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.0f;
#pragma unroll
        for (int j = 0; j < DPL; ++j) o[g][j] = 0.0f;
    }
    const int grp = lane / LPK, sub = lane % LPK, gid = warp * GPW + grp;

    if (warp == CW) {
        if (lane == 0) {  // page producer
            int i = 0;
            for (; i < npages; ++i) {
                const int s = i % NSLOT;
                if (!mb_wait(empty + s, ((i / NSLOT) & 1u) ^ 1u, err)) break;
                const int page = pt[pg0 + i];
                const size_t off = (static_cast<size_t>(page) * hkv + kvh) * PT * D;
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(full + s)),
                             "r"(2 * PAGE_B)
                             : "memory");
                asm volatile(
                    "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                        su32(ring + s * 2 * PAGE_B)),
                    "l"(kv.k + off), "r"(PAGE_B), "r"(su32(full + s))
                    : "memory");
                asm volatile(
                    "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                        su32(ring + s * 2 * PAGE_B + PAGE_B)),
                    "l"(kv.v + off), "r"(PAGE_B), "r"(su32(full + s))
                    : "memory");
            }
            // copies already issued land before the ring is reused for the merge (bounded)
            for (int j = i > NSLOT ? i - NSLOT : 0; j < i; ++j) mb_wait(full + j % NSLOT, (j / NSLOT) & 1u, err);
        }
    } else {
        const float qs = 1.4426950408889634f / sqrtf(static_cast<float>(D));
        float qr[G][DPL];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float* qp = q + (static_cast<size_t>(row) * hq + kvh * G + g) * D + sub * DPL;
#pragma unroll
            for (int j = 0; j < DPL; j += 4) {
                const float4 v = *reinterpret_cast<const float4*>(qp + j);
                qr[g][j] = v.x * qs;
                qr[g][j + 1] = v.y * qs;
                qr[g][j + 2] = v.z * qs;
                qr[g][j + 3] = v.w * qs;
            }
        }
        for (int i = 0; i < npages; ++i) {
            const int s = i % NSLOT;
            if (!mb_wait(full + s, (i / NSLOT) & 1u, err)) break;
            const uint8_t* kpage = ring + s * 2 * PAGE_B;
            const uint8_t* vpage = kpage + PAGE_B;
#pragma unroll
            for (int r = 0; r < KPG; ++r) {
                const int kin = gid + r * NG;
                const int key = (pg0 + i) * PT + kin;
                float kf[DPL], vf[DPL];
#pragma unroll
                for (int c = 0; c < NV; ++c) {
                    float w8[8];
                    const uint4 ku = *reinterpret_cast<const uint4*>(kpage + (kin * D + sub * DPL + c * 8) * 2);
                    const uint4 vu = *reinterpret_cast<const uint4*>(vpage + (kin * D + sub * DPL + c * 8) * 2);
                    Codec<WF_F16>::part(ku, 0, w8);
#pragma unroll
                    for (int j = 0; j < 8; ++j) kf[c * 8 + j] = w8[j];
                    Codec<WF_F16>::part(vu, 0, w8);
#pragma unroll
                    for (int j = 0; j < 8; ++j) vf[c * 8 + j] = w8[j];
                }
                const bool valid = key < ke;  // the split starts on a page boundary
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    float sc = 0.0f;
#pragma unroll
                    for (int j = 0; j < DPL; ++j) sc += qr[g][j] * kf[j];
#pragma unroll
                    for (int off = 1; off < LPK; off <<= 1) sc += __shfl_xor_sync(0xffffffffu, sc, off);
                    if (valid) {
                        const float mn = fmaxf(m[g], sc);
                        const float corr = exp2f(m[g] - mn);
                        const float pe = exp2f(sc - mn);
                        l[g] = l[g] * corr + pe;
#pragma unroll
                        for (int j = 0; j < DPL; ++j) o[g][j] = o[g][j] * corr + pe * vf[j];
                        m[g] = mn;
                    }
                }
            }
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(empty + s)) : "memory");
        }
    }
    __syncthreads();
    // merge the NG group states (the ring is free now)
    if (warp < CW) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float* st = mstate + (static_cast<size_t>(gid) * G + g) * (D + 2);
            if (sub == 0) {
                st[D] = m[g];
                st[D + 1] = l[g];
            }
#pragma unroll
            for (int j = 0; j < DPL; ++j) st[sub * DPL + j] = o[g][j];
        }
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < G * D; idx += AP_THREADS) {
        const int g = idx / D, d = idx % D;
        float M = -INFINITY;
        for (int w = 0; w < NG; ++w) M = fmaxf(M, mstate[(static_cast<size_t>(w) * G + g) * (D + 2) + D]);
        float Lt = 0.0f, acc = 0.0f;
        if (M != -INFINITY) {
            for (int w = 0; w < NG; ++w) {
                const float* st = mstate + (static_cast<size_t>(w) * G + g) * (D + 2);
                const float f = st[D] == -INFINITY ? 0.0f : exp2f(st[D] - M);
                Lt += st[D + 1] * f;
                acc += st[d] * f;
            }
        }
        const int h = kvh * G + g;
        if (n_splits == 1) {
            out[(static_cast<size_t>(row) * hq + h) * D + d] = Lt > 0.0f ? acc / Lt : 0.0f;
        } else {
            float* pp = part + ((static_cast<size_t>(row) * hq + h) * n_splits + split) * (D + 2);
            pp[d] = acc;
            if (d == 0) {
                pp[D] = M == -INFINITY ? -INFINITY : M * 0.6931471805599453f;
                pp[D + 1] = Lt;
            }
        }
    }
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

// Tensor-core variant: pages arrive by 2-D TMA (64-dim x 16-key boxes, 128-byte swizzle, so
// the ldmatrix reads below are free of bank conflicts); one consumer warp owns a whole page
// (16 keys) at a time and runs
// the page as two m16n8k16 products with the G query heads padded to n = 8:
//   S^T [16 keys x 8 heads] = K [16 x D] . Q^T        (A = K rows, ldmatrix)
//   O^T [D x 8 heads]      += V^T [D x 16 keys] . P^T (A = V rows, ldmatrix.trans)
// Q and P enter the MMAs as hi + lo fp16 halves (two MMAs each), which keeps the scores and
// weights at about 22 significand bits; K and V are fp16 in the cache, so the products are
// exact.  P goes through per-warp shared tiles to become the second product's B operand.  Each
// warp keeps its own online softmax (one max and one rescale per page and head); the four
// warps' states are merged at the end.
// Byte offset of (key k, dim d) in a page landed by the 64 x 16 TMA boxes with 128-byte
// swizzle: box d / 64 (2 KB each), row k (128 B), 16-byte chunk ((d % 64) / 8) ^ (k % 8).
__device__ __forceinline__ uint32_t sw_off(int k, int d) {
    return static_cast<uint32_t>((d >> 6) * 2048 + k * 128 + ((((d & 63) >> 3) ^ (k & 7)) << 4) + (d & 7) * 2);
}

template <int D, int G>
__global__ void __launch_bounds__(AP_THREADS) k_attn_pages_mma(const float* __restrict__ q,
                                                              const int* __restrict__ row_seq,
                                                              const int* __restrict__ row_pos, int hq, int hkv,
                                                              KVLayerView kv, int n_splits, float* __restrict__ out,
                                                              float* __restrict__ part,
                                                              const __grid_constant__ CUtensorMap tk,
                                                              const __grid_constant__ CUtensorMap tv, int* err) {
    pdl_enter();
    constexpr int PT = 16, PAGE_B = PT * D * 2, KS = D / 16;
    // Page i goes to slot i % NSLOT and warp i % CW; NSLOT a multiple of CW keeps every slot
    // with one warp, so no warp can wait on a slot's phase parity two phases ahead.
    constexpr int NSLOT = NSLOT_MMA;
    static_assert(NSLOT % CW == 0, "each ring slot must belong to one consumer warp");
    static_assert(G <= 8, "at most 8 query heads per kv head");
    static_assert(D % 64 == 0, "pages arrive as 64-dim boxes");
    extern __shared__ __align__(1024) uint8_t sm_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* ring = sm;                                                   // [NSLOT][K | V][PAGE_B], swizzled
    unsigned long long* full = reinterpret_cast<unsigned long long*>(sm + NSLOT * 2 * PAGE_B);
    unsigned long long* empty = full + NSLOT;
    __half* ptile = reinterpret_cast<__half*>(sm + NSLOT * 2 * PAGE_B + 2 * NSLOT * 8);  // [CW][hi|lo][8][16]
    float* mstate = reinterpret_cast<float*>(sm);  // after the loop: [CW][8][D + 2]

    const int row = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int seq = row_seq[row];
    const int nvis = row_pos[row] + 1;
    const int chunk = ((nvis + n_splits - 1) / n_splits + PT - 1) / PT * PT;
    const int kb = split * chunk, ke = min(nvis, kb + chunk);
    const int pg0 = kb / PT, npages = ke > kb ? (ke - kb + PT - 1) / PT : 0;
    const int* pt = kv.page_table + static_cast<size_t>(seq) * kv.max_pages;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NSLOT; ++s) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(full + s)) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(empty + s)) : "memory");
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    __syncthreads();

    // per thread: heads h0 = (lane % 4) * 2, h0 + 1 of the S / O fragments
    const int h0 = (lane & 3) * 2;
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.0f, 0.0f};
    float o[KS][4];
#pragma unroll
    for (int t = 0; t < KS; ++t) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.0f;

    if (warp == CW) {
        if (lane == 0) {  // page producer
            int i = 0;
            for (; i < npages; ++i) {
                const int s = i % NSLOT;
                if (!mb_wait(empty + s, ((i / NSLOT) & 1u) ^ 1u, err)) break;
                const int page = pt[pg0 + i];
                const int y = kv.row0 + (page * hkv + kvh) * PT;
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(full + s)),
                             "r"(2 * PAGE_B)
                             : "memory");
#pragma unroll
                for (int bx = 0; bx < D / 64; ++bx) {
                    asm volatile(
                        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
                            su32(ring + s * 2 * PAGE_B + bx * 2048)),
                        "l"(&tk), "r"(su32(full + s)), "r"(bx * 64), "r"(y)
                        : "memory");
                    asm volatile(
                        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
                            su32(ring + s * 2 * PAGE_B + PAGE_B + bx * 2048)),
                        "l"(&tv), "r"(su32(full + s)), "r"(bx * 64), "r"(y)
                        : "memory");
                }
            }
            for (int j = i > NSLOT ? i - NSLOT : 0; j < i; ++j) mb_wait(full + j % NSLOT, (j / NSLOT) & 1u, err);
        }
    } else {
        // Q^T as the B operand: b0 = (dims kk*16 + (lane%4)*2, +1; head lane/4), b1 = dims + 8.
        const float qs = 1.4426950408889634f / sqrtf(static_cast<float>(D));
        const int hb = lane >> 2;
        // hi + lo fp16 halves of the scaled query (x = hi + lo): the score keeps ~22 bits
        uint32_t qb[KS][2], ql[KS][2];
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
            float2 a = make_float2(0.f, 0.f), b = a;
            if (hb < G) {
                const float* qp = q + (static_cast<size_t>(row) * hq + kvh * G + hb) * D + kk * 16 + (lane & 3) * 2;
                a = *reinterpret_cast<const float2*>(qp);
                b = *reinterpret_cast<const float2*>(qp + 8);
            }
            const float f[4] = {a.x * qs, a.y * qs, b.x * qs, b.y * qs};
            __half hi[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) hi[e] = __float2half_rn(f[e]);
            qb[kk][0] = pack_h2(__half2float(hi[0]), __half2float(hi[1]));
            qb[kk][1] = pack_h2(__half2float(hi[2]), __half2float(hi[3]));
            ql[kk][0] = pack_h2(f[0] - __half2float(hi[0]), f[1] - __half2float(hi[1]));
            ql[kk][1] = pack_h2(f[2] - __half2float(hi[2]), f[3] - __half2float(hi[3]));
        }
        __half* pw = ptile + warp * 2 * 8 * PT;  // hi tile, then lo tile
        for (int i = warp; i < npages; i += CW) {
            const int s = i % NSLOT;
            if (!mb_wait(full + s, (i / NSLOT) & 1u, err)) break;
            const uint32_t kpage = su32(ring + s * 2 * PAGE_B), vpage = kpage + PAGE_B;
            // Positions past the split's last key hold whatever the pool held (possibly NaN
            // patterns): their V rows are zeroed, since P = 0 times NaN is NaN in the MMA.
            const int kvalid = ke - (pg0 + i) * PT;
            if (kvalid < PT) {
                // rows kvalid..15 of every 64-dim box (each row 128 B, 8 chunks)
                uint8_t* vbase = ring + s * 2 * PAGE_B + PAGE_B;
                for (int z = lane; z < (PT - kvalid) * 8 * (D / 64); z += 32) {
                    const int bx = z / ((PT - kvalid) * 8), rem = z % ((PT - kvalid) * 8);
                    *reinterpret_cast<uint4*>(vbase + bx * 2048 + (kvalid + rem / 8) * 128 + (rem % 8) * 16) =
                        make_uint4(0u, 0u, 0u, 0u);
                }
                __syncwarp();
            }
            // S^T = K . Q^T
            float sc[4] = {0.f, 0.f, 0.f, 0.f};
            const int arow = (lane & 7) + ((lane >> 3) & 1) * 8, acol = (lane >> 4) * 8;
#pragma unroll
            for (int kk = 0; kk < KS; ++kk) {
                uint32_t a[4];
                ldsm_x4(kpage + sw_off(arow, kk * 16 + acol), a);
                mma16816(sc, a, qb[kk][0], qb[kk][1]);
                mma16816(sc, a, ql[kk][0], ql[kk][1]);
            }
            // sc[0], sc[1]: key lane/4, heads h0, h0+1; sc[2], sc[3]: key lane/4 + 8
            const int key0 = (pg0 + i) * PT + (lane >> 2);
            if (key0 >= ke) sc[0] = sc[1] = -INFINITY;
            if (key0 + 8 >= ke) sc[2] = sc[3] = -INFINITY;
            float pmax0 = fmaxf(sc[0], sc[2]), pmax1 = fmaxf(sc[1], sc[3]);
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) {
                pmax0 = fmaxf(pmax0, __shfl_xor_sync(0xffffffffu, pmax0, off));
                pmax1 = fmaxf(pmax1, __shfl_xor_sync(0xffffffffu, pmax1, off));
            }
            // the page's first key is always visible, so pmax is finite
            const float mn0 = fmaxf(m[0], pmax0), mn1 = fmaxf(m[1], pmax1);
            const float c0 = exp2f(m[0] - mn0), c1 = exp2f(m[1] - mn1);
            m[0] = mn0;
            m[1] = mn1;
            const float p00 = exp2f(sc[0] - mn0), p01 = exp2f(sc[1] - mn1);
            const float p10 = exp2f(sc[2] - mn0), p11 = exp2f(sc[3] - mn1);
            l[0] = l[0] * c0 + p00 + p10;
            l[1] = l[1] * c1 + p01 + p11;
#pragma unroll
            for (int t = 0; t < KS; ++t) {
                o[t][0] *= c0;
                o[t][1] *= c1;
                o[t][2] *= c0;
                o[t][3] *= c1;
            }
            // P [8 heads][16 keys] through the warp's tiles as hi + lo fp16 halves
            const int kr = lane >> 2;
            auto put = [&](int idx, float v) {
                const __half h = __float2half_rn(v);
                pw[idx] = h;
                pw[8 * PT + idx] = __float2half_rn(v - __half2float(h));
            };
            put(h0 * PT + kr, p00);
            put((h0 + 1) * PT + kr, p01);
            put(h0 * PT + kr + 8, p10);
            put((h0 + 1) * PT + kr + 8, p11);
            __syncwarp();
            const uint32_t pb0 = *reinterpret_cast<const uint32_t*>(pw + hb * PT + (lane & 3) * 2);
            const uint32_t pb1 = *reinterpret_cast<const uint32_t*>(pw + hb * PT + 8 + (lane & 3) * 2);
            const uint32_t pl0 = *reinterpret_cast<const uint32_t*>(pw + 8 * PT + hb * PT + (lane & 3) * 2);
            const uint32_t pl1 = *reinterpret_cast<const uint32_t*>(pw + 8 * PT + hb * PT + 8 + (lane & 3) * 2);
            // O^T += V^T . P^T ; A tile t = dims t*16.. from the V page, transposed
            const int vkey = (lane & 7) + (lane >> 4) * 8, vdim = ((lane >> 3) & 1) * 8;
#pragma unroll
            for (int t = 0; t < KS; ++t) {
                uint32_t a[4];
                ldsm_x4_t(vpage + sw_off(vkey, t * 16 + vdim), a);
                mma16816(o[t], a, pb0, pb1);
                mma16816(o[t], a, pl0, pl1);
            }
            // order this warp's generic writes to the slot before the next bulk copy into it
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(empty + s)) : "memory");
        }
        // sum of p over the 16 keys of each head: lanes sharing lane % 4
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
            l[0] += __shfl_xor_sync(0xffffffffu, l[0], off);
            l[1] += __shfl_xor_sync(0xffffffffu, l[1], off);
        }
    }
    __syncthreads();
    // merge the CW warp states (the ring is free now): o[t][0..1] = dims t*16 + lane/4, heads
    // h0, h0 + 1; o[t][2..3] = dims + 8
    if (warp < CW) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int h = h0 + hh;
            float* st = mstate + (static_cast<size_t>(warp) * 8 + h) * (D + 2);
            if ((lane >> 2) == 0) {
                st[D] = m[hh];
                st[D + 1] = l[hh];
            }
#pragma unroll
            for (int t = 0; t < KS; ++t) {
                st[t * 16 + (lane >> 2)] = o[t][hh];
                st[t * 16 + (lane >> 2) + 8] = o[t][2 + hh];
            }
        }
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < G * D; idx += AP_THREADS) {
        const int g = idx / D, d = idx % D;
        float M = -INFINITY;
        for (int w = 0; w < CW; ++w) M = fmaxf(M, mstate[(static_cast<size_t>(w) * 8 + g) * (D + 2) + D]);
        float Lt = 0.0f, acc = 0.0f;
        if (M != -INFINITY) {
            for (int w = 0; w < CW; ++w) {
                const float* st = mstate + (static_cast<size_t>(w) * 8 + g) * (D + 2);
                const float f = st[D] == -INFINITY ? 0.0f : exp2f(st[D] - M);
                Lt += st[D + 1] * f;
                acc += st[d] * f;
            }
        }
        const int h = kvh * G + g;
        if (n_splits == 1) {
            out[(static_cast<size_t>(row) * hq + h) * D + d] = Lt > 0.0f ? acc / Lt : 0.0f;
        } else {
            float* pp = part + ((static_cast<size_t>(row) * hq + h) * n_splits + split) * (D + 2);
            pp[d] = acc;
            if (d == 0) {
                pp[D] = M == -INFINITY ? -INFINITY : M * 0.6931471805599453f;
                pp[D + 1] = Lt;
            }
        }
    }
}

// The tensor-core page kernel runs whenever the cache has its TMA views;
// SOC_B200_ATTENTION=lanes selects the CUDA-core lane-group kernel instead.
bool use_lane_groups(int) {
    const char* e = std::getenv("SOC_B200_ATTENTION");
    return e && std::string(e) == "lanes";
}

template <int D, int G>
void pages_dg(dim3 grid, const float* q, const Rows& rows, int hq, int hkv, const KVLayerView& kv, int splits,
              float* out, float* scratch, int* err, cudaStream_t st) {
    constexpr int PAGE_B = 16 * D * 2;
    constexpr int ring = NSLOT * 2 * PAGE_B + 2 * NSLOT * 8;
    if (!use_lane_groups(G) && kv.tmk != nullptr && kv.tmv != nullptr) {
        constexpr int ring_m = NSLOT_MMA * 2 * PAGE_B + 2 * NSLOT_MMA * 8;
        constexpr int smem_m = ring_m + CW * 2 * 8 * 16 * 2 + 1024;  // + alignment of the swizzled ring
        constexpr int merge_m = CW * 8 * (D + 2) * 4;
        static_assert(merge_m <= NSLOT_MMA * 2 * PAGE_B, "merge area fits in the ring");
        static bool set_m = false;
        if (!set_m) {
            SOCB_CUDA(cudaFuncSetAttribute(k_attn_pages_mma<D, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_m));
            set_m = true;
        }
        launch_pdl(k_attn_pages_mma<D, G>, dim3(grid), dim3(AP_THREADS), smem_m, st, q, rows.seq, rows.pos, hq, hkv,
                   kv, splits, out, scratch, *kv.tmk, *kv.tmv, err);
        return;
    }
    constexpr int LPK = (G >= 4 && D >= 128) ? 16 : 8;
    constexpr int merge = CW * (32 / LPK) * G * (D + 2) * 4;
    constexpr int smem = ring > merge ? ring : merge;
    static bool set = false;
    if (!set) {
        SOCB_CUDA(cudaFuncSetAttribute(k_attn_pages<D, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        set = true;
    }
    launch_pdl(k_attn_pages<D, G>, dim3(grid), dim3(AP_THREADS), smem, st, q, rows.seq, rows.pos, hq, hkv, kv, splits,
               out, scratch, err);
}

template <int D>
bool pages_d(int G, dim3 grid, const float* q, const Rows& rows, int hq, int hkv, const KVLayerView& kv, int splits,
             float* out, float* scratch, int* err, cudaStream_t st) {
    switch (G) {
        case 1: pages_dg<D, 1>(grid, q, rows, hq, hkv, kv, splits, out, scratch, err, st); return true;
        case 2: pages_dg<D, 2>(grid, q, rows, hq, hkv, kv, splits, out, scratch, err, st); return true;
        case 4: pages_dg<D, 4>(grid, q, rows, hq, hkv, kv, splits, out, scratch, err, st); return true;
        case 8: pages_dg<D, 8>(grid, q, rows, hq, hkv, kv, splits, out, scratch, err, st); return true;
        default: return false;
    }
}

}  // namespace

bool launch_attention_pages(const float* q, const Rows& rows, int splits, int hq, int hkv, int head_dim,
                            const KVLayerView& kv, float* out, float* scratch, int* err, cudaStream_t st) {
    if (kv.page_tokens != 16 || err == nullptr) return false;
    dim3 grid(rows.n, hkv, splits);
    const int G = hq / hkv;
    if (head_dim == 128) return pages_d<128>(G, grid, q, rows, hq, hkv, kv, splits, out, scratch, err, st);
    if (head_dim == 64) return pages_d<64>(G, grid, q, rows, hq, hkv, kv, splits, out, scratch, err, st);
    return false;
}

}  // namespace socb
