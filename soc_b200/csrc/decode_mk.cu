// Persistent batch-1 decode kernel for sm_100a.
//
// One cooperative launch, one CTA per SM, runs `steps` greedy decode steps of
// one sequence: embedding -> L x [RMSNorm -> qkv -> q/k norm + RoPE + KV append
// -> GQA attention -> o_proj + residual -> RMSNorm -> gate/up + SwiGLU -> down +
// residual] -> final RMSNorm -> tied lm_head -> argmax, feeding each id to the
// next step on the device.  Same arithmetic as the modular kernels (and the
// reference: Mac/cpu/src/qwen_block.cpp:63-72, qwen_attention.cpp:142-205,
// qwen_mlp.cpp:65-74, qwen_causal_lm.cpp:82-116, sampler.cpp:26-62).
//
// Batch-1 decode streams every weight byte once per token (1.19 GB for
// Qwen3-0.6B), so the kernel is HBM-bound.  Layout of the work:
//   * warp 0, lane 0 is a producer: it walks this CTA's share of every weight
//     matrix in execution order and streams it into a 5 x 32 KB shared-memory
//     ring with cp.async.bulk (TMA bulk copies, mbarrier completion, L2
//     evict-first).  It never waits on activations, so HBM keeps streaming the
//     next matrices while the consumers wait at a dependency.
//   * warps 1..8 are consumers: per matrix they stage the input vector once per
//     CTA (with the RMSNorm fused), hold their slice of it in registers, and
//     reduce 16-byte weight vectors from the ring with fp32 FMAs and warp
//     shuffles.  Each matrix's rows are split into contiguous per-CTA ranges.
//   * dependencies between matrices are monotonic global counters: a CTA
//     releases (fence + atomic add) after its rows are written; consumers of
//     the next phase acquire (ld.acquire.gpu spin, bounded).  Attention runs on
//     kv_heads x splits CTAs with a split-K combine by the last arriving CTA.
// Every wait is bounded: on expiry the kernel sets DERR_WAIT_TIMEOUT in *err,
// which makes every other wait return at once, and the kernel winds down.
#include "decode_mk.h"

namespace socb {
namespace {

constexpr int NC = 8;                   // consumer warps
constexpr int THREADS = (NC + 1) * 32;  // + producer warp
constexpr int SLOTS = 5;
constexpr int SLOT_BYTES = 32 * 1024;
constexpr int XBUF = 4352;              // floats: max K (4096) and the attention merge area
constexpr int MAXG = 4;                 // query heads per kv head
constexpr unsigned SPIN_LIMIT = 1u << 21;

enum Kind { K_QKV = 0, K_O = 1, K_GU = 2, K_D = 3, K_LM = 4 };

struct __align__(128) Smem {
    uint8_t ring[SLOTS][SLOT_BYTES];
    float x[XBUF];
    float red[NC];
    unsigned long long best[NC];
    unsigned long long full[SLOTS];
    unsigned long long empty[SLOTS];
    int flag;
};

// ---------------------------------------------------------------- PTX helpers
__device__ __forceinline__ uint32_t s32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void mbar_init(unsigned long long* b, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(s32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(unsigned long long* b, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(s32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(unsigned long long* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(s32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_test(unsigned long long* b, unsigned parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(s32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
// 1-D bulk copy global -> this CTA's shared memory, completing on `bar` (16-byte aligned, size % 16 == 0).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, unsigned long long* bar,
                                         uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            s32(dst)),
        "l"(src), "r"(bytes), "r"(s32(bar)), "l"(pol)
        : "memory");
}
__device__ __forceinline__ void nbar() { asm volatile("bar.sync 1, %0;" ::"n"(NC * 32) : "memory"); }

__device__ __forceinline__ bool aborted(const int* err) {
    return (*reinterpret_cast<const volatile int*>(err) & DERR_WAIT_TIMEOUT) != 0;
}

// Bounded wait on an mbarrier phase (non-blocking test + short sleep per try).
__device__ bool mbar_wait(unsigned long long* b, unsigned parity, int* err) {
    for (unsigned i = 0;; ++i) {
        if (mbar_test(b, parity)) return true;
        if ((i & 255u) == 255u && aborted(err)) return false;
        if (i > 4 * SPIN_LIMIT) {
            atomicOr(err, DERR_WAIT_TIMEOUT);
            return false;
        }
        if (i > 64) __nanosleep(20);
    }
}

// Bounded acquire-wait until *c >= target.
__device__ bool wait_count(const unsigned* c, unsigned target, int* err) {
    for (unsigned i = 0;; ++i) {
        unsigned v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(c) : "memory");
        if (v >= target) return true;
        if (aborted(err)) return false;
        if (i > SPIN_LIMIT) {
            atomicOr(err, DERR_WAIT_TIMEOUT);
            return false;
        }
        __nanosleep(64);
    }
}

__device__ __forceinline__ void release_add(unsigned* c) {
    __threadfence();
    atomicAdd(c, 1u);
}

// Consumer-side dependency wait: one thread spins, the others meet it at the named barrier.
__device__ __forceinline__ void cwait(const unsigned* c, unsigned target, int* err, int ctid) {
    if (ctid == 0) {
        wait_count(c, target, err);
        __threadfence();
    }
    nbar();
}

// ------------------------------------------------------------------- schedule
struct Phase {
    const uint8_t* w;
    int units, unit_bytes, K, rows;  // rows per unit: 1, or 2 for (gate, up)
};

__device__ __forceinline__ Phase phase_of(const MKParams& p, int l, int kind) {
    Phase ph;
    if (kind == K_LM) {
        ph.w = static_cast<const uint8_t*>(p.lm_head);
        ph.units = p.V;
        ph.K = p.H;
        ph.rows = 1;
    } else {
        const MKLayer& ly = p.layers[l];
        switch (kind) {
            case K_QKV:
                ph.w = static_cast<const uint8_t*>(ly.wqkv);
                ph.units = (p.hq + 2 * p.hkv) * p.D;
                ph.K = p.H;
                ph.rows = 1;
                break;
            case K_O:
                ph.w = static_cast<const uint8_t*>(ly.wo);
                ph.units = p.H;
                ph.K = p.hq * p.D;
                ph.rows = 1;
                break;
            case K_GU:
                ph.w = static_cast<const uint8_t*>(ly.wgu);
                ph.units = p.I;
                ph.K = p.H;
                ph.rows = 2;
                break;
            default:
                ph.w = static_cast<const uint8_t*>(ly.wd);
                ph.units = p.H;
                ph.K = p.I;
                ph.rows = 1;
                break;
        }
    }
    ph.unit_bytes = ph.rows * ph.K * 2;
    return ph;
}

// Contiguous unit range of CTA `cta`; the rotation moves the larger shares around
// so every CTA streams about the same number of bytes per token.
__device__ __forceinline__ void cta_range(int units, int cta, int G, int l, int kind, int& a, int& b) {
    const int v = (cta + (l * 5 + kind) * 37) % G;
    a = static_cast<int>(static_cast<long long>(units) * v / G);
    b = static_cast<int>(static_cast<long long>(units) * (v + 1) / G);
}

// Barrier counter indices.
__device__ __forceinline__ int bar_phase(int l, int k) { return l * 5 + k; }  // k: 0 qkv, 1 attn, 2 o, 3 gu, 4 d
__device__ __forceinline__ int bar_lm(const MKParams& p) { return p.L * 5; }
__device__ __forceinline__ int bar_split(const MKParams& p, int l, int j) { return p.L * 5 + 1 + l * p.hkv + j; }

// ------------------------------------------------------------------- producer
__device__ void produce_phase(const MKParams& p, Smem& sm, const Phase& ph, int l, int kind, long long& k, uint64_t pol,
                              bool& ok) {
    int a, b;
    cta_range(ph.units, blockIdx.x, gridDim.x, l, kind, a, b);
    const int cu = max(1, SLOT_BYTES / ph.unit_bytes);
    for (int u = a; u < b && ok; u += cu, ++k) {
        const int n = min(cu, b - u);
        const int slot = static_cast<int>(k % SLOTS);
        const long long round = k / SLOTS;
        if (round > 0 && !mbar_wait(&sm.empty[slot], static_cast<unsigned>((round - 1) & 1), p.err)) {
            ok = false;
            break;
        }
        const unsigned bytes = static_cast<unsigned>(n) * ph.unit_bytes;
        mbar_expect_tx(&sm.full[slot], bytes);
        bulk_g2s(sm.ring[slot], ph.w + static_cast<size_t>(u) * ph.unit_bytes, bytes, &sm.full[slot], pol);
    }
}

__device__ void producer(const MKParams& p, Smem& sm) {
    const uint64_t pol = evict_first_policy();
    long long k = 0;
    bool ok = true;
    for (int t = 0; t < p.steps && ok; ++t) {
        for (int l = 0; l < p.L && ok; ++l)
            for (int kind = K_QKV; kind <= K_D && ok; ++kind) produce_phase(p, sm, phase_of(p, l, kind), l, kind, k, pol, ok);
        if (ok) produce_phase(p, sm, phase_of(p, 0, K_LM), 0, K_LM, k, pol, ok);
    }
    // Never leave with copies in flight: wait (bounded) for the last fills to land.
    const long long first = k > SLOTS ? k - SLOTS : 0;
    for (long long q = first; q < k; ++q) {
        const int slot = static_cast<int>(q % SLOTS);
        for (unsigned i = 0; i < SPIN_LIMIT; ++i) {
            if (mbar_test(&sm.full[slot], static_cast<unsigned>((q / SLOTS) & 1))) break;
            __nanosleep(32);
        }
    }
}

// ------------------------------------------------------------------ consumers
template <typename T>
__device__ __forceinline__ void unpack8(const uint4& u, float (&w)[8]) {
    const float2 a = WTraits<T>::pair(u.x), b = WTraits<T>::pair(u.y), c = WTraits<T>::pair(u.z),
                 d = WTraits<T>::pair(u.w);
    w[0] = a.x; w[1] = a.y; w[2] = b.x; w[3] = b.y;
    w[4] = c.x; w[5] = c.y; w[6] = d.x; w[7] = d.y;
}

template <typename T>
__device__ __forceinline__ float emb_at(const void* table, size_t idx) {
    const T v = static_cast<const T*>(table)[idx];
    return static_cast<float>(v);
}

// Stage the phase input into sm.x: RMSNorm of h (or of the token's embedding row) with weight w,
// or a plain copy.  All consumer threads take part; ends with a named barrier.
template <typename T>
__device__ void stage(Smem& sm, const float* src, const void* emb_row_table, size_t emb_base, int K, const float* w,
                      float eps, int ctid) {
    const int lane = ctid & 31, cw = ctid >> 5;
    float ss = 0.0f;
    for (int i = ctid * 4; i < K; i += NC * 32 * 4) {
        float4 v;
        if (src != nullptr) {
            v = __ldcg(reinterpret_cast<const float4*>(src + i));
        } else {
            v.x = emb_at<T>(emb_row_table, emb_base + i);
            v.y = emb_at<T>(emb_row_table, emb_base + i + 1);
            v.z = emb_at<T>(emb_row_table, emb_base + i + 2);
            v.w = emb_at<T>(emb_row_table, emb_base + i + 3);
        }
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        *reinterpret_cast<float4*>(&sm.x[i]) = v;
    }
    if (w == nullptr) {
        nbar();
        return;
    }
    ss = warp_sum(ss);
    if (lane == 0) sm.red[cw] = ss;
    nbar();
    float tot = 0.0f;
#pragma unroll
    for (int q = 0; q < NC; ++q) tot += sm.red[q];
    const float s = 1.0f / sqrtf(tot / static_cast<float>(K) + eps);
    for (int i = ctid; i < K; i += NC * 32) sm.x[i] = sm.x[i] * s * w[i];
    nbar();
}

template <int KI, typename T>
__device__ __forceinline__ void dot2(const uint8_t* r0, const uint8_t* r1, const float (&xr)[KI][8], int lane,
                                     float& a0, float& a1, bool two) {
    float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
    for (int it = 0; it < KI; ++it) {
        const int off = (it * 256 + lane * 8) * 2;
        float w[8];
        unpack8<T>(*reinterpret_cast<const uint4*>(r0 + off), w);
#pragma unroll
        for (int j = 0; j < 8; ++j) s0 += w[j] * xr[it][j];
        if (two) {
            unpack8<T>(*reinterpret_cast<const uint4*>(r1 + off), w);
#pragma unroll
            for (int j = 0; j < 8; ++j) s1 += w[j] * xr[it][j];
        }
    }
    a0 = warp_sum(s0);
    a1 = two ? warp_sum(s1) : 0.0f;
}

struct StepCtx {
    int t, tok, pos;
};

// Consume one phase's chunks from the ring and apply its epilogue.
template <int KI, typename T>
__device__ void consume(const MKParams& p, Smem& sm, const Phase& ph, int l, int kind, long long& k, const StepCtx& sc,
                        int cw, int lane, unsigned long long& wbest) {
    float xr[KI][8];
#pragma unroll
    for (int it = 0; it < KI; ++it) {
        const float4 u = *reinterpret_cast<const float4*>(&sm.x[it * 256 + lane * 8]);
        const float4 v = *reinterpret_cast<const float4*>(&sm.x[it * 256 + lane * 8 + 4]);
        xr[it][0] = u.x; xr[it][1] = u.y; xr[it][2] = u.z; xr[it][3] = u.w;
        xr[it][4] = v.x; xr[it][5] = v.y; xr[it][6] = v.z; xr[it][7] = v.w;
    }
    int a, b;
    cta_range(ph.units, blockIdx.x, gridDim.x, l, kind, a, b);
    const int cu = max(1, SLOT_BYTES / ph.unit_bytes);
    const int rowb = ph.K * 2;
    for (int u = a; u < b; u += cu, ++k) {
        const int n = min(cu, b - u);
        const int slot = static_cast<int>(k % SLOTS);
        const bool ok = mbar_wait(&sm.full[slot], static_cast<unsigned>((k / SLOTS) & 1), p.err);
        if (ok) {
            for (int i = cw; i < n; i += NC) {
                const uint8_t* base = sm.ring[slot] + static_cast<size_t>(i) * ph.unit_bytes;
                const int unit = u + i;
                if (kind == K_GU) {
                    float g, up;
                    dot2<KI, T>(base, base + rowb, xr, lane, g, up, true);
                    if (lane == 0) p.act[unit] = silu_f(g) * up;
                } else if (kind == K_LM) {
                    float y, unused;
                    dot2<KI, T>(base, base, xr, lane, y, unused, false);
                    if (lane == 0) {
                        if (p.logits) p.logits[static_cast<size_t>(sc.t) * p.V + unit] = y;
                        if (y == y) {
                            const unsigned long long key = argmax_key(y, unit);
                            wbest = key > wbest ? key : wbest;
                        }
                    }
                } else {
                    float y, unused;
                    dot2<KI, T>(base, base, xr, lane, y, unused, false);
                    if (lane == 0) {
                        if (kind == K_QKV) {
                            p.qkv[unit] = y;
                        } else if (kind == K_O && l == 0) {
                            p.h[unit] = emb_at<T>(p.embed, static_cast<size_t>(sc.tok) * p.H + unit) + y;
                        } else {
                            p.h[unit] = __ldcg(p.h + unit) + y;
                        }
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.empty[slot]);
    }
}

template <typename T>
__device__ void consume_k(const MKParams& p, Smem& sm, const Phase& ph, int l, int kind, long long& k,
                          const StepCtx& sc, int cw, int lane, unsigned long long& wbest) {
    switch (ph.K / 256) {
        case 1: consume<1, T>(p, sm, ph, l, kind, k, sc, cw, lane, wbest); break;
        case 2: consume<2, T>(p, sm, ph, l, kind, k, sc, cw, lane, wbest); break;
        case 4: consume<4, T>(p, sm, ph, l, kind, k, sc, cw, lane, wbest); break;
        case 8: consume<8, T>(p, sm, ph, l, kind, k, sc, cw, lane, wbest); break;
        case 12: consume<12, T>(p, sm, ph, l, kind, k, sc, cw, lane, wbest); break;
        default: consume<16, T>(p, sm, ph, l, kind, k, sc, cw, lane, wbest); break;
    }
}

// q/k RMSNorm + rotate-half RoPE of one head held as DL dims per lane (dims lane*DL + j).
template <int D>
__device__ __forceinline__ void norm_rope(float (&v)[D / 32], const float* nw, const float2* cs_row, float eps, int lane) {
    constexpr int DL = D / 32, HALF = D / 2;
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < DL; ++j) ss += v[j] * v[j];
    ss = warp_sum(ss);
    const float s = 1.0f / sqrtf(ss / static_cast<float>(D) + eps);
#pragma unroll
    for (int j = 0; j < DL; ++j) v[j] = v[j] * s * nw[lane * DL + j];
    const bool first = lane < 16;
    float o[DL];
#pragma unroll
    for (int j = 0; j < DL; ++j) {
        const float partner = __shfl_xor_sync(0xffffffffu, v[j], 16);
        const float2 c = cs_row[(lane * DL + j) % HALF];
        o[j] = first ? (v[j] * c.x - partner * c.y) : (partner * c.y + v[j] * c.x);
    }
#pragma unroll
    for (int j = 0; j < DL; ++j) v[j] = o[j];
}

// Attention units of layer l for this CTA: unit u = (kv head j, split s), u < hkv * S.
template <int D>
__device__ void attention_phase(const MKParams& p, Smem& sm, int l, const StepCtx& sc, int cw, int lane, int ctid) {
    constexpr int DL = D / 32;
    const int S = p.att_splits, G = p.hq / p.hkv, units = p.hkv * S;
    const int GRID = gridDim.x;
    bool waited = false;
    __half* kp = p.kpool + l * p.kv_layer_stride;
    __half* vp = p.vpool + l * p.kv_layer_stride;
    const float scale = 1.0f / sqrtf(static_cast<float>(D));
    const int pos = sc.pos, nvis = pos + 1;
    const int chunk = ((nvis + S - 1) / S + 15) / 16 * 16;
    float* qs = sm.x;                       // [MAXG][D] normalised + rotated queries
    float* ks = sm.x + MAXG * D;            // [D] new key (fp16-rounded)
    float* vs = sm.x + (MAXG + 1) * D;      // [D] new value (fp16-rounded)
    float* merge = sm.x + (MAXG + 2) * D;   // [NC][G][D + 2]
    for (int u = 0; u < units; ++u) {
        if (static_cast<int>(static_cast<long long>(u) * GRID / units) != static_cast<int>(blockIdx.x)) continue;
        if (!waited) {
            cwait(&p.bars[bar_phase(l, 0)], static_cast<unsigned>(GRID * (sc.t + 1)), p.err, ctid);
            waited = true;
        }
        const int j = u / S, s = u % S;
        const int kb = s * chunk, ke = min(nvis, kb + chunk);
        const bool owns_new = pos >= kb && pos < ke;
        const float2* cs_row = p.rope_cs + static_cast<size_t>(pos) * (D / 2);
        const int page = p.page_table[pos / p.page_tokens];
        const size_t new_off = ((static_cast<size_t>(page) * p.hkv + j) * p.page_tokens + pos % p.page_tokens) * D;
        // warps 0..G-1: queries of the group; warp G: the new key / value
        if (cw < G) {
            float v[DL];
            const float* src = p.qkv + (static_cast<size_t>(j) * G + cw) * D + lane * DL;
#pragma unroll
            for (int q = 0; q < DL; ++q) v[q] = __ldcg(src + q);
            norm_rope<D>(v, p.layers[l].q_norm, cs_row, p.eps, lane);
#pragma unroll
            for (int q = 0; q < DL; ++q) qs[cw * D + lane * DL + q] = v[q];
        } else if (cw == G && owns_new) {
            float v[DL], w[DL];
            const float* ksrc = p.qkv + static_cast<size_t>(p.hq) * D + static_cast<size_t>(j) * D + lane * DL;
            const float* vsrc = p.qkv + static_cast<size_t>(p.hq + p.hkv) * D + static_cast<size_t>(j) * D + lane * DL;
#pragma unroll
            for (int q = 0; q < DL; ++q) {
                v[q] = __ldcg(ksrc + q);
                w[q] = __ldcg(vsrc + q);
            }
            norm_rope<D>(v, p.layers[l].k_norm, cs_row, p.eps, lane);
#pragma unroll
            for (int q = 0; q < DL; ++q) {
                const __half kh = __float2half_rn(v[q]), vh = __float2half_rn(w[q]);
                kp[new_off + lane * DL + q] = kh;
                vp[new_off + lane * DL + q] = vh;
                ks[lane * DL + q] = __half2float(kh);
                vs[lane * DL + q] = __half2float(vh);
            }
        }
        nbar();
        float qr[MAXG][DL], m[MAXG], lsum[MAXG], o[MAXG][DL];
#pragma unroll
        for (int g = 0; g < MAXG; ++g) {
            m[g] = -INFINITY;
            lsum[g] = 0.0f;
#pragma unroll
            for (int q = 0; q < DL; ++q) {
                o[g][q] = 0.0f;
                qr[g][q] = g < G ? qs[g * D + lane * DL + q] : 0.0f;
            }
        }
        for (int key = kb + cw; key < ke; key += NC) {
            float kf[DL], vf[DL];
            if (key == pos) {
#pragma unroll
                for (int q = 0; q < DL; ++q) {
                    kf[q] = ks[lane * DL + q];
                    vf[q] = vs[lane * DL + q];
                }
            } else {
                const int pg = p.page_table[key / p.page_tokens];
                const size_t off = ((static_cast<size_t>(pg) * p.hkv + j) * p.page_tokens + key % p.page_tokens) * D +
                                   lane * DL;
#pragma unroll
                for (int q = 0; q < DL; ++q) {
                    kf[q] = __half2float(kp[off + q]);
                    vf[q] = __half2float(vp[off + q]);
                }
            }
#pragma unroll
            for (int g = 0; g < MAXG; ++g) {
                if (g >= G) break;
                float sc_ = 0.0f;
#pragma unroll
                for (int q = 0; q < DL; ++q) sc_ += qr[g][q] * kf[q];
                sc_ = warp_sum(sc_) * scale;
                const float mn = fmaxf(m[g], sc_);
                const float corr = expf(m[g] - mn);
                const float pe = expf(sc_ - mn);
                lsum[g] = lsum[g] * corr + pe;
#pragma unroll
                for (int q = 0; q < DL; ++q) o[g][q] = o[g][q] * corr + pe * vf[q];
                m[g] = mn;
            }
        }
        // merge the warps
        for (int g = 0; g < G; ++g) {
            float* mr = merge + (cw * G + g) * (D + 2);
#pragma unroll
            for (int q = 0; q < DL; ++q) mr[lane * DL + q] = o[g][q];
            if (lane == 0) {
                mr[D] = m[g];
                mr[D + 1] = lsum[g];
            }
        }
        nbar();
        float* part = p.att_part + (static_cast<size_t>(j) * S + s) * G * (D + 2);
        for (int idx = ctid; idx < G * D; idx += NC * 32) {
            const int g = idx / D, d = idx % D;
            float M = -INFINITY;
            for (int w = 0; w < NC; ++w) M = fmaxf(M, merge[(w * G + g) * (D + 2) + D]);
            float L = 0.0f, acc = 0.0f;
            if (M != -INFINITY) {
                for (int w = 0; w < NC; ++w) {
                    const float* mr = merge + (w * G + g) * (D + 2);
                    const float f = mr[D] == -INFINITY ? 0.0f : expf(mr[D] - M);
                    L += mr[D + 1] * f;
                    acc += mr[d] * f;
                }
            }
            if (S == 1) {
                p.attn[(static_cast<size_t>(j) * G + g) * D + d] = L > 0.0f ? acc / L : 0.0f;
            } else {
                part[g * (D + 2) + d] = acc;
                if (d == 0) {
                    part[g * (D + 2) + D] = M;
                    part[g * (D + 2) + D + 1] = L;
                }
            }
        }
        nbar();
        if (S == 1) {
            if (ctid == 0) release_add(&p.bars[bar_phase(l, 1)]);
            continue;
        }
        // split-K: the last CTA to finish a kv head combines its splits.
        if (ctid == 0) {
            __threadfence();
            const unsigned old = atomicAdd(&p.bars[bar_split(p, l, j)], 1u);
            sm.flag = (old + 1 == static_cast<unsigned>(S * (sc.t + 1))) ? 1 : 0;
            __threadfence();
        }
        nbar();
        if (sm.flag) {
            const float* hp = p.att_part + static_cast<size_t>(j) * S * G * (D + 2);
            for (int idx = ctid; idx < G * D; idx += NC * 32) {
                const int g = idx / D, d = idx % D;
                float M = -INFINITY;
                for (int q = 0; q < S; ++q) M = fmaxf(M, __ldcg(hp + (q * G + g) * (D + 2) + D));
                float L = 0.0f, acc = 0.0f;
                if (M != -INFINITY) {
                    for (int q = 0; q < S; ++q) {
                        const float* pp = hp + (q * G + g) * (D + 2);
                        const float mq = __ldcg(pp + D);
                        const float f = mq == -INFINITY ? 0.0f : expf(mq - M);
                        L += __ldcg(pp + D + 1) * f;
                        acc += __ldcg(pp + d) * f;
                    }
                }
                p.attn[(static_cast<size_t>(j) * G + g) * D + d] = L > 0.0f ? acc / L : 0.0f;
            }
            nbar();
            if (ctid == 0) release_add(&p.bars[bar_phase(l, 1)]);
        }
    }
}

template <typename T>
__device__ void consumers(const MKParams& p, Smem& sm, int cw, int lane) {
    const int ctid = cw * 32 + lane;
    const unsigned GRID = gridDim.x;
    long long k = 0;
    for (int t = 0; t < p.steps; ++t) {
        StepCtx sc;
        sc.t = t;
        sc.pos = p.start + t;
        if (t == 0) {
            sc.tok = __ldcg(p.ids);
        } else {
            cwait(&p.bars[bar_lm(p)], GRID * t, p.err, ctid);
            const unsigned long long b = *reinterpret_cast<volatile unsigned long long*>(&p.best[t - 1]);
            sc.tok = b == 0ull ? 0 : argmax_key_index(b);
            if (blockIdx.x == 0 && ctid == 0) p.ids[t] = sc.tok;
        }
        unsigned long long wbest = 0ull;
        for (int l = 0; l < p.L; ++l) {
            const MKLayer& ly = p.layers[l];
            // qkv
            if (l > 0) cwait(&p.bars[bar_phase(l - 1, 4)], GRID * (t + 1), p.err, ctid);
            if (l == 0)
                stage<T>(sm, nullptr, p.embed, static_cast<size_t>(sc.tok) * p.H, p.H, ly.in_norm, p.eps, ctid);
            else
                stage<T>(sm, p.h, nullptr, 0, p.H, ly.in_norm, p.eps, ctid);
            consume_k<T>(p, sm, phase_of(p, l, K_QKV), l, K_QKV, k, sc, cw, lane, wbest);
            nbar();
            if (ctid == 0) release_add(&p.bars[bar_phase(l, 0)]);
            // attention (its own wait on the qkv phase)
            if (p.D == 128)
                attention_phase<128>(p, sm, l, sc, cw, lane, ctid);
            else
                attention_phase<64>(p, sm, l, sc, cw, lane, ctid);
            // o_proj + residual
            cwait(&p.bars[bar_phase(l, 1)], static_cast<unsigned>(p.hkv * (t + 1)), p.err, ctid);
            stage<T>(sm, p.attn, nullptr, 0, p.hq * p.D, nullptr, p.eps, ctid);
            consume_k<T>(p, sm, phase_of(p, l, K_O), l, K_O, k, sc, cw, lane, wbest);
            nbar();
            if (ctid == 0) release_add(&p.bars[bar_phase(l, 2)]);
            // gate/up + SwiGLU
            cwait(&p.bars[bar_phase(l, 2)], GRID * (t + 1), p.err, ctid);
            stage<T>(sm, p.h, nullptr, 0, p.H, ly.post_norm, p.eps, ctid);
            consume_k<T>(p, sm, phase_of(p, l, K_GU), l, K_GU, k, sc, cw, lane, wbest);
            nbar();
            if (ctid == 0) release_add(&p.bars[bar_phase(l, 3)]);
            // down + residual
            cwait(&p.bars[bar_phase(l, 3)], GRID * (t + 1), p.err, ctid);
            stage<T>(sm, p.act, nullptr, 0, p.I, nullptr, p.eps, ctid);
            consume_k<T>(p, sm, phase_of(p, l, K_D), l, K_D, k, sc, cw, lane, wbest);
            nbar();
            if (ctid == 0) release_add(&p.bars[bar_phase(l, 4)]);
        }
        // final norm + lm_head + argmax
        cwait(&p.bars[bar_phase(p.L - 1, 4)], GRID * (t + 1), p.err, ctid);
        stage<T>(sm, p.h, nullptr, 0, p.H, p.final_norm, p.eps, ctid);
        consume_k<T>(p, sm, phase_of(p, 0, K_LM), 0, K_LM, k, sc, cw, lane, wbest);
        if (lane == 0) sm.best[cw] = wbest;
        nbar();
        if (ctid == 0) {
            unsigned long long b = 0ull;
            for (int q = 0; q < NC; ++q) b = sm.best[q] > b ? sm.best[q] : b;
            if (b != 0ull) atomicMax(&p.best[t], b);
            release_add(&p.bars[bar_lm(p)]);
        }
    }
    if (blockIdx.x == 0) {
        cwait(&p.bars[bar_lm(p)], GRID * p.steps, p.err, ctid);
        if (ctid == 0) {
            const unsigned long long b = *reinterpret_cast<volatile unsigned long long*>(&p.best[p.steps - 1]);
            p.ids[p.steps] = b == 0ull ? 0 : argmax_key_index(b);
        }
    }
}

template <typename T>
__global__ void __launch_bounds__(THREADS, 1) k_decode_mk(MKParams p) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < SLOTS; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], NC);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    __syncthreads();
    if (warp == 0) {
        if (lane == 0) producer(p, sm);
    } else {
        consumers<T>(p, sm, warp - 1, lane);
    }
}

}  // namespace

int mk_bar_count(int L, int hkv) { return L * 5 + 1 + L * hkv; }

bool mk_supported(int H, int I, int hq, int hkv, int D, int wfmt) {
    auto ki_ok = [](int K) {
        const int ki = K / 256;
        return K % 256 == 0 && (ki == 1 || ki == 2 || ki == 4 || ki == 8 || ki == 12 || ki == 16);
    };
    if (wfmt != WF_F16 && wfmt != WF_BF16) return false;
    if (!ki_ok(H) || !ki_ok(I) || !ki_ok(hq * D)) return false;
    if (D != 64 && D != 128) return false;
    if (hq % hkv != 0 || hq / hkv > MAXG) return false;
    if (hq * D > XBUF || I > XBUF || H > XBUF) return false;
    if ((MAXG + 2) * D + NC * (hq / hkv) * (D + 2) > XBUF) return false;
    // one unit must fit a ring slot: (gate, up) pair rows and the widest single row
    if (2 * H * 2 > SLOT_BYTES || I * 2 > SLOT_BYTES || hq * D * 2 > SLOT_BYTES) return false;
    return true;
}

int mk_grid(int device) {
    int sms = 0;
    SOCB_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
    return sms;
}

void mk_launch(const MKParams& p, int grid, cudaStream_t st) {
    const size_t smem = sizeof(Smem);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (p.wfmt == WF_BF16) {
        SOCB_CUDA(cudaFuncSetAttribute(k_decode_mk<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem)));
        SOCB_CUDA(cudaLaunchKernelEx(&cfg, k_decode_mk<__nv_bfloat16>, p));
    } else {
        SOCB_CUDA(cudaFuncSetAttribute(k_decode_mk<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem)));
        SOCB_CUDA(cudaLaunchKernelEx(&cfg, k_decode_mk<__half>, p));
    }
}

}  // namespace socb
