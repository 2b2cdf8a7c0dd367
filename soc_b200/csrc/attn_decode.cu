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
#include "kernels.h"

namespace socb {
namespace {

constexpr int NSLOT = 6;
constexpr int CW = 4;                    // consumer warps
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

template <int D, int G>
void pages_dg(dim3 grid, const float* q, const Rows& rows, int hq, int hkv, const KVLayerView& kv, int splits,
              float* out, float* scratch, int* err, cudaStream_t st) {
    constexpr int PAGE_B = 16 * D * 2;
    constexpr int ring = NSLOT * 2 * PAGE_B + 2 * NSLOT * 8;
    constexpr int LPK = (G >= 4 && D >= 128) ? 16 : 8;
    constexpr int merge = CW * (32 / LPK) * G * (D + 2) * 4;
    constexpr int smem = ring > merge ? ring : merge;
    static bool set = false;
    if (!set) {
        SOCB_CUDA(cudaFuncSetAttribute(k_attn_pages<D, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        set = true;
    }
    k_attn_pages<D, G><<<grid, AP_THREADS, smem, st>>>(q, rows.seq, rows.pos, hq, hkv, kv, splits, out, scratch, err);
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
