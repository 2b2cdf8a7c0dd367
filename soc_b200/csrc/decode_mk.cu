// Persistent batch-1 decode kernel for sm_100a.
//
// One cooperative launch, one CTA per SM, runs `steps` greedy decode steps of
// one sequence: embedding -> L x [RMSNorm -> qkv -> q/k norm + RoPE + KV append
// -> GQA attention -> o_proj + residual -> RMSNorm -> gate/up + SwiGLU -> down +
// residual] -> final RMSNorm -> tied lm_head -> argmax, feeding each id to the
// next step on the device.  Same arithmetic as the modular kernels (and the
// reference: Mac/cpu/src/qwen_block.cpp:63-72, qwen_attention.cpp:142-205,
// qwen_mlp.cpp:65-74, qwen_causal_lm.cpp:82-116, sampler.cpp:26-62), except
// that the RMSNorm scale is applied after the dot product:
// sum_i W[r,i] (x_i s w_i) = s * sum_i W[r,i] (x_i w_i).
//
// Batch-1 decode streams every weight byte once per token (1.19 GB for
// Qwen3-0.6B) and is a chain of ~140 dependent matrix-vector phases, so the
// design works on two things: keeping HBM busy across the dependencies, and
// making each dependency hand-off short.
//   * warp 0, lane 0 is a producer: it walks this CTA's share of every weight
//     matrix in execution order and streams it into a 6 x 32 KB shared-memory
//     ring with cp.async.bulk (TMA bulk copies, mbarrier completion, L2
//     evict-first).  It never waits on activations; with an EOS id set it waits
//     at each step boundary for the step's argmax, so that no weight of a step
//     that will not run is loaded.
//   * warps 1..7 are consumers: per matrix they stage the input vector once per
//     CTA (double-buffered, one CTA barrier per phase), hold their slice of it in
//     registers and reduce 16-byte weight vectors from the ring with fp32 FMAs
//     and warp shuffles.  Each matrix's rows are split into contiguous per-CTA
//     ranges.
//   * hand-offs between matrices are monotonic counters, one per layer and
//     phase: a CTA adds 1 with release semantics after its rows are stored, and
//     a CTA that needs the vector waits (one thread, acquire) for the count.
//   * attention runs on kv_heads x splits CTAs; the cached keys, the RoPE row
//     and the norm weights are loaded before the q/k/v rows arrive.  With more
//     than one split the last CTA of a kv head combines the partials.
// Every wait is bounded: on expiry the kernel sets DERR_WAIT_TIMEOUT in *err,
// which makes every other wait return at once, and the kernel winds down
// (the producer first waits, bounded, for its copies in flight).
#include "decode_mk.h"

namespace socb {
namespace {

constexpr int NC = 7;                   // consumer warps (256 threads per CTA: up to 255 registers)
constexpr int CT = NC * 32;             // consumer threads
constexpr int THREADS = CT + 32;        // + producer warp
constexpr int SLOTS = 6;
constexpr int SLOT_BYTES = 32 * 1024;
constexpr int INFLIGHT = SLOTS;         // TMA loads into shared memory in flight per CTA
constexpr int PF_CHUNKS = 0;            // chunks prefetched into L2 ahead of the load cursor
constexpr int XMAX = 3072;              // widest staged input (floats)
constexpr int HMAX = 1024;              // widest hidden size
constexpr int MAXG = 2;                 // query heads per kv head
constexpr int KPF = 8;                  // keys per warp per attention batch
constexpr int MAXFL = 5;                // phase flags polled per lane (grid <= 160)
constexpr unsigned SPIN_LIMIT = 1u << 21;

enum Kind { K_QKV = 0, K_O = 1, K_GU = 2, K_D = 3, K_LM = 4 };
enum Ep { E_QKV = 0, E_ATT = 1, E_HO = 2, E_ACT = 3, E_HD = 4, E_LM = 5 };

struct __align__(128) Smem {
    uint8_t ring[SLOTS][SLOT_BYTES];
    float x[2][XMAX];
    float hraw[2][HMAX];
    float red[2][NC];
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
// Fire-and-forget prefetch of a global range into L2 (no data returns to the SM).
__device__ __forceinline__ void prefetch_l2(const void* src, unsigned bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void nbar() { asm volatile("bar.sync 1, %0;" ::"n"(CT) : "memory"); }

__device__ __forceinline__ unsigned long long gtime() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ bool aborted(const int* err) {
    return (*reinterpret_cast<const volatile int*>(err) & DERR_WAIT_TIMEOUT) != 0;
}

// Bounded wait on an mbarrier phase (non-blocking test + short sleep per try).
__device__ __forceinline__ bool mbar_wait(unsigned long long* b, unsigned parity, int* err) {
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

// Hand-offs between phases are monotonic counters, one per (layer, phase): when a CTA's
// part of a phase is stored it adds 1 with release semantics; a CTA that needs the phase's
// output waits (one thread, acquire) until the counter reaches (step + 1) * contributors.
// A device-wide hand-off of this kind measured about 1 us on B200 with 148 CTAs; polling
// one flag per CTA instead was about 4 us (148 writers and pollers on the same lines).
// Every counter sits on its own 128-byte line (FLAG_STRIDE words): counters that shared a
// line made the pollers of one phase queue behind the adds of another.
//   slot l * 6 + e     e in {E_QKV, E_ATT, E_HO, E_ACT, E_HD}; E_ATT counts kv heads
//   slot L * 6         lm_head done (per CTA)
//   slot L * 6 + 1 + l * hkv + j  split-K arrivals of kv head j
constexpr int FLAG_STRIDE = 32;
__device__ __forceinline__ unsigned* ctr(const MKParams& p, int l, int e) { return p.flags + (l * 6 + e) * FLAG_STRIDE; }
__device__ __forceinline__ unsigned* ctr_lm(const MKParams& p) { return p.flags + p.L * 6 * FLAG_STRIDE; }
__device__ __forceinline__ unsigned* split_ctr(const MKParams& p, int l, int j) {
    return p.flags + (p.L * 6 + 1 + l * p.hkv + j) * FLAG_STRIDE;
}

__device__ __forceinline__ void red_release_add(unsigned* c) {
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(c) : "memory");
}

// One consumer thread waits (bounded) until *c >= target with acquire semantics; then the CTA barrier.
__device__ __forceinline__ void wait_ctr(const unsigned* c, unsigned target, int* err, int ctid) {
    if (ctid == 0) {
        for (unsigned i = 0;; ++i) {
            unsigned v;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(c) : "memory");
            if (v >= target) break;
            if (i > SPIN_LIMIT) {
                atomicOr(err, DERR_WAIT_TIMEOUT);
                break;
            }
            if ((i & 63u) == 63u && aborted(err)) break;
            if (i > 4) __nanosleep(32);
        }
    }
    nbar();
}

// One thread's bounded wait for c >= target (the producer's); false when it gave up.
__device__ __forceinline__ bool wait_ctr_thread(const unsigned* c, unsigned target, int* err) {
    for (unsigned i = 0;; ++i) {
        unsigned v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(c) : "memory");
        if (v >= target) return true;
        if (i > SPIN_LIMIT) {
            atomicOr(err, DERR_WAIT_TIMEOUT);
            return false;
        }
        if ((i & 63u) == 63u && aborted(err)) return false;
        if (i > 4) __nanosleep(32);
    }
}

// After this CTA's part of a phase is stored: the CTA barrier, then one release add.
__device__ __forceinline__ void signal(unsigned* c, int ctid) {
    nbar();
    if (ctid == 0) red_release_add(c);
}

// Trace slot `e` of layer `l` (first step only, consumer thread 0).  Slots per layer:
// 0 start, 1 qkv input ready, 2 qkv staged, 3 qkv first chunk, 4 qkv done, 5 attention input
// ready, 6 attention done, 7 o input ready, 8 o first chunk, 9 o done, 10 gu input ready,
// 11 gu first chunk, 12 gu done, 13 down input ready, 14 down first chunk, 15 down done.
// Layer L holds the lm_head: 1 input ready, 2 staged, 3 first chunk, 4 done.
#define MK_TR(l, e)                                                                                                  \
    do {                                                                                                             \
        if (p.trace != nullptr && sc.t == 0 && ctid == 0)                                                            \
            p.trace[static_cast<size_t>(blockIdx.x) * mk_trace_stride(p.L) + (l) * MK_TRACE_PER_LAYER + (e)] =      \
                gtime();                                                                                             \
    } while (0)

// ------------------------------------------------------------------- schedule
struct Phase {
    const uint8_t* w;
    int units, unit_bytes, K, rows;  // rows per unit: 1, or 2 for (gate, up)
};

__device__ __forceinline__ Phase phase_of(const MKParams& p, const MKLayer& ly, int kind) {
    Phase ph;
    ph.rows = 1;
    switch (kind) {
        case K_QKV:
            ph.w = static_cast<const uint8_t*>(ly.wqkv);
            ph.units = (p.hq + 2 * p.hkv) * p.D;
            ph.K = p.H;
            break;
        case K_O:
            ph.w = static_cast<const uint8_t*>(ly.wo);
            ph.units = p.H;
            ph.K = p.hq * p.D;
            break;
        case K_GU:
            ph.w = static_cast<const uint8_t*>(ly.wgu);
            ph.units = p.I;
            ph.K = p.H;
            ph.rows = 2;
            break;
        case K_D:
            ph.w = static_cast<const uint8_t*>(ly.wd);
            ph.units = p.H;
            ph.K = p.I;
            break;
        default:
            ph.w = static_cast<const uint8_t*>(p.lm_head);
            ph.units = p.V;
            ph.K = p.H;
            break;
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

// ------------------------------------------------------------------- producer
// Walks this CTA's chunks in consumption order: per step, per layer the qkv, o, gate/up and
// down matrices, then the lm_head.  A chunk is up to SLOT_BYTES of whole units.
struct Cursor {
    int t, l, kind, u;  // kind == K_LM means the lm_head of step t
    int a, b, cu;       // unit range of this CTA in the current phase, units per chunk
    const uint8_t* w;
    int unit_bytes;
    bool done;
};

__device__ __forceinline__ void cursor_phase(const MKParams& p, Cursor& c) {
    const Phase ph = phase_of(p, p.layers[c.kind == K_LM ? 0 : c.l], c.kind);
    cta_range(ph.units, blockIdx.x, gridDim.x, c.l, c.kind, c.a, c.b);
    c.cu = max(1, SLOT_BYTES / ph.unit_bytes);
    c.w = ph.w;
    c.unit_bytes = ph.unit_bytes;
    c.u = c.a;
}

__device__ __forceinline__ void cursor_init(const MKParams& p, Cursor& c) {
    c.t = 0;
    c.l = 0;
    c.kind = K_QKV;
    c.done = p.steps <= 0;
    if (!c.done) cursor_phase(p, c);
}

// Move to the next phase that has units (every phase has some for this CTA, see mk_supported;
// an empty one would be skipped here exactly as the consumers' loops skip it).
__device__ __forceinline__ void cursor_next_phase(const MKParams& p, Cursor& c);
__device__ __forceinline__ void cursor_next_phase1(const MKParams& p, Cursor& c) {
    if (c.kind == K_LM) {
        c.kind = K_QKV;
        c.l = 0;
        if (++c.t >= p.steps) {
            c.done = true;
            return;
        }
    } else if (c.kind == K_D) {
        if (++c.l >= p.L) {
            c.kind = K_LM;
            c.l = 0;
        } else {
            c.kind = K_QKV;
        }
    } else {
        ++c.kind;
    }
    cursor_phase(p, c);
}

__device__ __forceinline__ void cursor_next_phase(const MKParams& p, Cursor& c) {
    do {
        cursor_next_phase1(p, c);
    } while (!c.done && c.a >= c.b);
}

// Current chunk of the cursor (pointer and bytes), then advance.
__device__ __forceinline__ void cursor_take(const MKParams& p, Cursor& c, const uint8_t*& ptr, unsigned& bytes) {
    const int n = min(c.cu, c.b - c.u);
    ptr = c.w + static_cast<size_t>(c.u) * c.unit_bytes;
    bytes = static_cast<unsigned>(n) * c.unit_bytes;
    c.u += n;
    if (c.u >= c.b) cursor_next_phase(p, c);
}

__device__ __forceinline__ void producer(const MKParams& p, Smem& sm) {
    const uint64_t pol = evict_first_policy();
    Cursor ld, pf;
    cursor_init(p, ld);
    cursor_init(p, pf);
    // L2 prefetch runs PF_CHUNKS ahead of the loads into shared memory.
    for (int i = 0; i < PF_CHUNKS && !pf.done; ++i) {
        const uint8_t* ptr;
        unsigned bytes;
        cursor_take(p, pf, ptr, bytes);
        prefetch_l2(ptr, bytes);
    }
    long long k = 0;
    bool ok = true;
    int checked = -1;  // last step whose input id was compared with p.eos
    while (!ld.done && ok) {
        if (p.eos >= 0 && ld.t != checked) {
            // The first chunk of step ld.t: load it only if that step runs, i.e. its input id
            // (step 0: ids[0]; later: the merged argmax of the step before) is not eos.  The
            // consumers take the same decision from the same keys at the top of the step.
            checked = ld.t;
            int tok;
            if (ld.t == 0) {
                tok = __ldcg(p.ids);
            } else {
                if (!wait_ctr_thread(ctr_lm(p), static_cast<unsigned>(gridDim.x * ld.t), p.err)) break;
                unsigned long long b = 0ull;
                for (int c = 0; c < static_cast<int>(gridDim.x); ++c) {
                    const unsigned long long kk = __ldcg(p.best + static_cast<size_t>(ld.t - 1) * gridDim.x + c);
                    b = kk > b ? kk : b;
                }
                tok = b == 0ull ? 0 : argmax_key_index(b);
            }
            if (tok == p.eos) break;
        }
        const int slot = static_cast<int>(k % SLOTS);
        const long long round = k / SLOTS;
        if (round > 0 && !mbar_wait(&sm.empty[slot], static_cast<unsigned>((round - 1) & 1), p.err)) {
            ok = false;
            break;
        }
        // keep at most INFLIGHT loads into shared memory outstanding
        if (INFLIGHT < SLOTS && k >= INFLIGHT) {
            const long long q = k - INFLIGHT;
            if (!mbar_wait(&sm.full[q % SLOTS], static_cast<unsigned>((q / SLOTS) & 1), p.err)) {
                ok = false;
                break;
            }
        }
        const uint8_t* ptr;
        unsigned bytes;
        cursor_take(p, ld, ptr, bytes);
        if (p.trace != nullptr && k < MK_TRACE_CHUNKS)
            p.trace[static_cast<size_t>(blockIdx.x) * mk_trace_stride(p.L) + (p.L + 1) * MK_TRACE_PER_LAYER + k] = gtime();
        mbar_expect_tx(&sm.full[slot], bytes);
        bulk_g2s(sm.ring[slot], ptr, bytes, &sm.full[slot], pol);
        if (!pf.done) {
            const uint8_t* pp;
            unsigned pb;
            cursor_take(p, pf, pp, pb);
            prefetch_l2(pp, pb);
        }
        ++k;
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

// Stage K floats (already known ready) into x (and hraw), all consumer threads, 4 per load.
//   norm_w == nullptr: x = v.
//   norm_w != nullptr: hraw = v, x = v * w, per-warp sum of squares of v into red.
//   emb != nullptr: v is the embedding row (layer 0) instead of `src`.
// Ends with the CTA barrier.
template <typename T>
__device__ __forceinline__ void stage(const float* src, const void* emb, size_t emb_base, int K, const float* norm_w,
                                   float* x, float* hraw, float* red, int ctid) {
    const int lane = ctid & 31, cw = ctid >> 5;
    float ss = 0.0f;
    for (int i = 4 * ctid; i < K; i += 4 * CT) {
        float4 v;
        if (emb != nullptr) {
            const uint2 r = *reinterpret_cast<const uint2*>(static_cast<const T*>(emb) + emb_base + i);
            const float2 a = WTraits<T>::pair(r.x), b = WTraits<T>::pair(r.y);
            v = make_float4(a.x, a.y, b.x, b.y);
        } else {
            v = __ldcg(reinterpret_cast<const float4*>(src + i));
        }
        if (norm_w) {
            const float4 w = *reinterpret_cast<const float4*>(norm_w + i);
            *reinterpret_cast<float4*>(hraw + i) = v;
            ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
            *reinterpret_cast<float4*>(x + i) = make_float4(v.x * w.x, v.y * w.y, v.z * w.z, v.w * w.w);
        } else {
            *reinterpret_cast<float4*>(x + i) = v;
        }
    }
    if (norm_w) {
        ss = warp_sum(ss);
        if (lane == 0) red[cw] = ss;
    }
    nbar();
}

__device__ __forceinline__ float norm_scale(const float* red, int K, float eps) {
    float tot = 0.0f;
#pragma unroll
    for (int q = 0; q < NC; ++q) tot += red[q];
    return 1.0f / sqrtf(tot / static_cast<float>(K) + eps);
}

template <int KI, typename T, bool two>
__device__ __forceinline__ void dot2(const uint8_t* r0, const uint8_t* r1, const float (&xr)[KI][8], int lane,
                                     float& a0, float& a1) {
    float s0 = 0.0f, s0b = 0.0f, s1 = 0.0f, s1b = 0.0f;
#pragma unroll
    for (int it = 0; it < KI; ++it) {
        const int off = (it * 256 + lane * 8) * 2;
        float w[8];
        unpack8<T>(*reinterpret_cast<const uint4*>(r0 + off), w);
        s0 += w[0] * xr[it][0] + w[1] * xr[it][1] + w[2] * xr[it][2] + w[3] * xr[it][3];
        s0b += w[4] * xr[it][4] + w[5] * xr[it][5] + w[6] * xr[it][6] + w[7] * xr[it][7];
        if (two) {
            unpack8<T>(*reinterpret_cast<const uint4*>(r1 + off), w);
            s1 += w[0] * xr[it][0] + w[1] * xr[it][1] + w[2] * xr[it][2] + w[3] * xr[it][3];
            s1b += w[4] * xr[it][4] + w[5] * xr[it][5] + w[6] * xr[it][6] + w[7] * xr[it][7];
        }
    }
    a0 = warp_sum(s0 + s0b);
    a1 = two ? warp_sum(s1 + s1b) : 0.0f;
}

struct StepCtx {
    int t, tok, pos;
};

// Consume one phase's chunks from the ring and apply its epilogue.  `s` is the folded
// RMSNorm scale (1 for phases without a norm), `hraw` the residual stream staged earlier.
template <int KI, typename T, bool TWO>
__device__ __forceinline__ void consume(const MKParams& p, Smem& sm, const Phase& ph, int l, int kind, long long& k,
                                    const StepCtx& sc, const float* x, const float* hraw, float s, int tr_first,
                                    int ctid, unsigned long long& wbest) {
    const int cw = ctid >> 5, lane = ctid & 31;
    float xr[KI][8];
#pragma unroll
    for (int it = 0; it < KI; ++it) {
        const float4 u = *reinterpret_cast<const float4*>(&x[it * 256 + lane * 8]);
        const float4 v = *reinterpret_cast<const float4*>(&x[it * 256 + lane * 8 + 4]);
        xr[it][0] = u.x; xr[it][1] = u.y; xr[it][2] = u.z; xr[it][3] = u.w;
        xr[it][4] = v.x; xr[it][5] = v.y; xr[it][6] = v.z; xr[it][7] = v.w;
    }
    int a, b;
    cta_range(ph.units, blockIdx.x, gridDim.x, l, kind, a, b);
    const int cu = max(1, SLOT_BYTES / ph.unit_bytes);
    const int rowb = ph.K * 2;
    bool first = true;
    for (int u = a; u < b; u += cu, ++k) {
        const int n = min(cu, b - u);
        const int slot = static_cast<int>(k % SLOTS);
        if (p.trace != nullptr && k < MK_TRACE_CHUNKS && ctid == 0)
            p.trace[static_cast<size_t>(blockIdx.x) * mk_trace_stride(p.L) + (p.L + 1) * MK_TRACE_PER_LAYER +
                    2 * MK_TRACE_CHUNKS + k] = gtime();
        const bool ok = mbar_wait(&sm.full[slot], static_cast<unsigned>((k / SLOTS) & 1), p.err);
        if (p.trace != nullptr && k < MK_TRACE_CHUNKS && ctid == 0)
            p.trace[static_cast<size_t>(blockIdx.x) * mk_trace_stride(p.L) + (p.L + 1) * MK_TRACE_PER_LAYER +
                    MK_TRACE_CHUNKS + k] = gtime();
        if (first) {
            MK_TR(kind == K_LM ? p.L : l, tr_first);
            first = false;
        }
        if (ok) {
            // unit g of the phase belongs to warp (g - a) % NC, so the warps stay balanced over
            // the whole phase even when a chunk's unit count is not a multiple of NC
            const int i0 = ((cw - (u - a)) % NC + NC) % NC;
            if (TWO) {
                // (gate, up) row pairs: one unit per warp at a time
                for (int i = i0; i < n; i += NC) {
                    const uint8_t* base = sm.ring[slot] + static_cast<size_t>(i) * ph.unit_bytes;
                    float g, up;
                    dot2<KI, T, true>(base, base + rowb, xr, lane, g, up);
                    if (lane == 0) p.act[u + i] = silu_f(g * s) * (up * s);
                }
            } else {
                // two independent rows per warp at a time (their loads and FMAs interleave)
                for (int i = i0; i < n; i += 2 * NC) {
                    const int i2 = i + NC;
                    const bool has2 = i2 < n;
                    const uint8_t* r0 = sm.ring[slot] + static_cast<size_t>(i) * ph.unit_bytes;
                    const uint8_t* r1 = has2 ? sm.ring[slot] + static_cast<size_t>(i2) * ph.unit_bytes : r0;
                    float y[2];
                    dot2<KI, T, true>(r0, r1, xr, lane, y[0], y[1]);
                    if (lane != 0) continue;
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        if (q == 1 && !has2) break;
                        const int unit = u + (q == 0 ? i : i2);
                        switch (kind) {
                            case K_QKV: p.qkv[unit] = y[q] * s; break;
                            case K_O:
                            case K_D: p.h[unit] = hraw[unit] + y[q]; break;
                            default: {
                                const float yy = y[q] * s;
                                if (p.logits) p.logits[static_cast<size_t>(sc.t) * p.V + unit] = yy;
                                const float sv = p.temperature == 1.0f ? yy : __fdiv_rn(yy, p.temperature);
                                if (sv == sv) {
                                    const unsigned long long key = argmax_key(sv, unit);
                                    wbest = key > wbest ? key : wbest;
                                }
                            }
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
                          const StepCtx& sc, const float* x, const float* hraw, float s, int trf, int ctid,
                          unsigned long long& wbest) {
    if (kind == K_GU) {  // (gate, up) row pairs; K = hidden
        switch (ph.K / 256) {
            case 1: consume<1, T, true>(p, sm, ph, l, kind, k, sc, x, hraw, s, trf, ctid, wbest); break;
            case 2: consume<2, T, true>(p, sm, ph, l, kind, k, sc, x, hraw, s, trf, ctid, wbest); break;
            default: consume<4, T, true>(p, sm, ph, l, kind, k, sc, x, hraw, s, trf, ctid, wbest); break;
        }
        return;
    }
    switch (ph.K / 256) {
        case 1: consume<1, T, false>(p, sm, ph, l, kind, k, sc, x, hraw, s, trf, ctid, wbest); break;
        case 2: consume<2, T, false>(p, sm, ph, l, kind, k, sc, x, hraw, s, trf, ctid, wbest); break;
        case 4: consume<4, T, false>(p, sm, ph, l, kind, k, sc, x, hraw, s, trf, ctid, wbest); break;
        case 8: consume<8, T, false>(p, sm, ph, l, kind, k, sc, x, hraw, s, trf, ctid, wbest); break;
        default: consume<12, T, false>(p, sm, ph, l, kind, k, sc, x, hraw, s, trf, ctid, wbest); break;
    }
}

// ------------------------------------------------------------------ attention
template <int DL>
struct KVRaw;
template <>
struct KVRaw<4> {
    using type = uint2;
};
template <>
struct KVRaw<2> {
    using type = uint32_t;
};

__device__ __forceinline__ void unpack_kv(const uint2& r, float (&f)[4]) {
    const float2 a = h2_to_f2(r.x), b = h2_to_f2(r.y);
    f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
}
__device__ __forceinline__ void unpack_kv(const uint32_t& r, float (&f)[2]) {
    const float2 a = h2_to_f2(r);
    f[0] = a.x; f[1] = a.y;
}

// Attention units of layer l on this CTA: unit u = (kv head j, split s), u < hkv * S.
// Scratch: the x buffer `scr` (free between the qkv and o phases).
template <int D>
__device__ __forceinline__ void attention_phase(const MKParams& p, Smem& sm, const MKLayer& ly, int l, const StepCtx& sc,
                                             float* scr, int ctid) {
    constexpr int DL = D / 32, HALF = D / 2;
    using Raw = typename KVRaw<DL>::type;
    const int cw = ctid >> 5, lane = ctid & 31;
    const int S = p.att_splits, G = p.hq / p.hkv, units = p.hkv * S;
    const int GRID = gridDim.x;
    __half* kp = p.kpool + l * p.kv_layer_stride;
    __half* vp = p.vpool + l * p.kv_layer_stride;
    const float scale = 1.0f / sqrtf(static_cast<float>(D));
    const int pos = sc.pos, nvis = pos + 1;
    const int chunk = ((nvis + S - 1) / S + 15) / 16 * 16;
    float* qs = scr;                      // [MAXG][D] normalised + rotated queries
    float* ks = scr + MAXG * D;           // [D] new key (fp16-rounded)
    float* vs = scr + (MAXG + 1) * D;     // [D] new value (fp16-rounded)
    float* merge = scr + (MAXG + 2) * D;  // [NC][G][D + 2]
    for (int u = 0; u < units; ++u) {
        if (static_cast<int>(static_cast<long long>(u) * GRID / units) != static_cast<int>(blockIdx.x)) continue;
        const int j = u / S, s = u % S;
        const int kb = s * chunk, ke = min(nvis, kb + chunk);
        const bool owns_new = pos >= kb && pos < ke;
        // -- loads that do not depend on this step's q/k/v: RoPE row, norm weights, cached keys
        float2 cs[DL];
        float nw[DL];
#pragma unroll
        for (int q = 0; q < DL; ++q) {
            cs[q] = p.rope_cs[static_cast<size_t>(pos) * HALF + (lane * DL + q) % HALF];
            nw[q] = (cw < G ? ly.q_norm : ly.k_norm)[lane * DL + q];
        }
        Raw kraw[KPF], vraw[KPF];
        const int key0 = kb + cw;
#pragma unroll
        for (int i = 0; i < KPF; ++i) {
            const int key = key0 + NC * i;
            if (key < ke && key != pos) {
                const int pg = __ldg(p.page_table + key / p.page_tokens);
                const size_t off =
                    ((static_cast<size_t>(pg) * p.hkv + j) * p.page_tokens + key % p.page_tokens) * D + lane * DL;
                kraw[i] = __ldcg(reinterpret_cast<const Raw*>(kp + off));
                vraw[i] = __ldcg(reinterpret_cast<const Raw*>(vp + off));
            }
        }
        // -- wait for this layer's q/k/v rows (every CTA's qkv part)
        wait_ctr(ctr(p, l, E_QKV), static_cast<unsigned>(GRID * (sc.t + 1)), p.err, ctid);
        MK_TR(l, 5);
        if (cw < G || (cw == G && owns_new)) {
            const int hrow = cw < G ? (j * G + cw) * D : (p.hq + j) * D;
            float v[DL], vv[DL];
#pragma unroll
            for (int q = 0; q < DL; ++q) v[q] = __ldcg(p.qkv + hrow + lane * DL + q);
            if (cw == G) {
                const int vrow = (p.hq + p.hkv + j) * D;
#pragma unroll
                for (int q = 0; q < DL; ++q) vv[q] = __ldcg(p.qkv + vrow + lane * DL + q);
            }
            // per-head RMSNorm + rotate-half RoPE (dims lane*DL + q; partner in lane ^ 16)
            float ssq = 0.0f;
#pragma unroll
            for (int q = 0; q < DL; ++q) ssq += v[q] * v[q];
            ssq = warp_sum(ssq);
            const float rs = 1.0f / sqrtf(ssq / static_cast<float>(D) + p.eps);
#pragma unroll
            for (int q = 0; q < DL; ++q) v[q] = v[q] * rs * nw[q];
            const bool first = lane < 16;
            float o[DL];
#pragma unroll
            for (int q = 0; q < DL; ++q) {
                const float partner = __shfl_xor_sync(0xffffffffu, v[q], 16);
                o[q] = first ? (v[q] * cs[q].x - partner * cs[q].y) : (partner * cs[q].y + v[q] * cs[q].x);
            }
            if (cw < G) {
#pragma unroll
                for (int q = 0; q < DL; ++q) qs[cw * D + lane * DL + q] = o[q];
            } else {
                const int page = __ldg(p.page_table + pos / p.page_tokens);
                const size_t off =
                    ((static_cast<size_t>(page) * p.hkv + j) * p.page_tokens + pos % p.page_tokens) * D + lane * DL;
#pragma unroll
                for (int q = 0; q < DL; ++q) {
                    const __half kh = __float2half_rn(o[q]), vh = __float2half_rn(vv[q]);
                    kp[off + q] = kh;
                    vp[off + q] = vh;
                    ks[lane * DL + q] = __half2float(kh);
                    vs[lane * DL + q] = __half2float(vh);
                }
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
        for (int base = key0; base < ke; base += NC * KPF) {
            if (base != key0) {
#pragma unroll
                for (int i = 0; i < KPF; ++i) {
                    const int key = base + NC * i;
                    if (key < ke && key != pos) {
                        const int pg = __ldg(p.page_table + key / p.page_tokens);
                        const size_t off =
                            ((static_cast<size_t>(pg) * p.hkv + j) * p.page_tokens + key % p.page_tokens) * D +
                            lane * DL;
                        kraw[i] = __ldcg(reinterpret_cast<const Raw*>(kp + off));
                        vraw[i] = __ldcg(reinterpret_cast<const Raw*>(vp + off));
                    }
                }
            }
            // KB keys at a time: their dot products reduce in one interleaved shuffle tree and
            // the running softmax is rescaled once per batch (KB + 1 exponentials, not 2 KB).
            constexpr int KB = 4;
#pragma unroll
            for (int i0 = 0; i0 < KPF; i0 += KB) {
                if (base + NC * i0 >= ke) break;
                float kf[KB][DL], vf[KB][DL];
                bool ok[KB];
#pragma unroll
                for (int b = 0; b < KB; ++b) {
                    const int key = base + NC * (i0 + b);
                    ok[b] = key < ke;
                    if (!ok[b]) {  // past the split: the prefetch registers hold nothing (0 * NaN)
#pragma unroll
                        for (int q = 0; q < DL; ++q) kf[b][q] = vf[b][q] = 0.0f;
                    } else if (key == pos) {
#pragma unroll
                        for (int q = 0; q < DL; ++q) {
                            kf[b][q] = ks[lane * DL + q];
                            vf[b][q] = vs[lane * DL + q];
                        }
                    } else {
                        unpack_kv(kraw[i0 + b], kf[b]);
                        unpack_kv(vraw[i0 + b], vf[b]);
                    }
                }
#pragma unroll
                for (int g = 0; g < MAXG; ++g) {
                    if (g >= G) break;
                    float d[KB];
#pragma unroll
                    for (int b = 0; b < KB; ++b) {
                        d[b] = 0.0f;
#pragma unroll
                        for (int q = 0; q < DL; ++q) d[b] += qr[g][q] * kf[b][q];
                    }
#pragma unroll
                    for (int off = 16; off > 0; off >>= 1)
#pragma unroll
                        for (int b = 0; b < KB; ++b) d[b] += __shfl_xor_sync(0xffffffffu, d[b], off);
                    float mn = m[g];
#pragma unroll
                    for (int b = 0; b < KB; ++b) {
                        d[b] = ok[b] ? d[b] * scale : -INFINITY;
                        mn = fmaxf(mn, d[b]);
                    }
                    const float corr = expf(m[g] - mn);
                    float ps = 0.0f, pe[KB];
#pragma unroll
                    for (int b = 0; b < KB; ++b) {
                        pe[b] = ok[b] ? expf(d[b] - mn) : 0.0f;
                        ps += pe[b];
                    }
                    lsum[g] = lsum[g] * corr + ps;
#pragma unroll
                    for (int q = 0; q < DL; ++q) {
                        float acc = o[g][q] * corr;
#pragma unroll
                        for (int b = 0; b < KB; ++b) acc += pe[b] * vf[b][q];
                        o[g][q] = acc;
                    }
                    m[g] = mn;
                }
            }
        }
        // unrolled over MAXG with a guard: a loop bounded by the run-time G would index o / m /
        // lsum dynamically and move them (and every update of them above) to local memory
#pragma unroll
        for (int g = 0; g < MAXG; ++g) {
            if (g >= G) break;
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
        for (int idx = ctid; idx < G * D; idx += CT) {
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
        if (S == 1) {
            signal(ctr(p, l, E_ATT), ctid);
            MK_TR(l, 6);
            continue;
        }
        // split-K: the last CTA to finish kv head j combines its splits.
        nbar();
        if (ctid == 0) {
            __threadfence();
            const unsigned old = atomicAdd(split_ctr(p, l, j), 1u);
            sm.flag = (old + 1 == static_cast<unsigned>(S * (sc.t + 1))) ? 1 : 0;
            __threadfence();
        }
        nbar();
        if (sm.flag) {
            const float* hp = p.att_part + static_cast<size_t>(j) * S * G * (D + 2);
            for (int idx = ctid; idx < G * D; idx += CT) {
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
            signal(ctr(p, l, E_ATT), ctid);
            MK_TR(l, 6);
        }
        nbar();
    }
}

template <typename T>
__device__ void consumers(const MKParams& p, Smem& sm, int cw, int lane) {
    const int ctid = cw * 32 + lane;
    const int GRID = gridDim.x;
    const int me = blockIdx.x;
    long long k = 0;
    bool stopped = false;
    for (int t = 0; t < p.steps; ++t) {
        StepCtx sc;
        sc.t = t;
        sc.pos = p.start + t;
        const unsigned full = static_cast<unsigned>(GRID * (t + 1));
        if (t == 0) {
            sc.tok = __ldcg(p.ids);
        } else {
            wait_ctr(ctr_lm(p), static_cast<unsigned>(GRID * t), p.err, ctid);
            // every CTA reduces the per-CTA argmax keys of the previous step
            unsigned long long b = 0ull;
            for (int c = lane; c < GRID; c += 32) {
                const unsigned long long kk = __ldcg(p.best + static_cast<size_t>(t - 1) * GRID + c);
                b = kk > b ? kk : b;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long other = __shfl_xor_sync(0xffffffffu, b, o);
                b = other > b ? other : b;
            }
            sc.tok = b == 0ull ? 0 : argmax_key_index(b);
            if (me == 0 && ctid == 0) p.ids[t] = sc.tok;
        }
        if (sc.tok == p.eos) {
            // every CTA reads the same id, so all of them (and their producers) stop here
            stopped = true;
            break;
        }
        unsigned long long wbest = 0ull;
        for (int l = 0; l < p.L; ++l) {
            const MKLayer ly = p.layers[l];
            MK_TR(l, 0);
            // ---- qkv: stage h (or the embedding row) into x[0] / hraw[0]
            if (l == 0) {
                stage<T>(nullptr, p.embed, static_cast<size_t>(sc.tok) * p.H, p.H, ly.in_norm, sm.x[0], sm.hraw[0],
                         sm.red[0], ctid);
            } else {
                wait_ctr(ctr(p, l - 1, E_HD), full, p.err, ctid);
                MK_TR(l, 1);
                stage<T>(p.h, nullptr, 0, p.H, ly.in_norm, sm.x[0], sm.hraw[0], sm.red[0], ctid);
            }
            MK_TR(l, 2);
            const float s_in = norm_scale(sm.red[0], p.H, p.eps);
            consume_k<T>(p, sm, phase_of(p, ly, K_QKV), l, K_QKV, k, sc, sm.x[0], sm.hraw[0], s_in, 3, ctid, wbest);
            signal(ctr(p, l, E_QKV), ctid);
            MK_TR(l, 4);
            // ---- attention (scratch: x[1])
            if (p.D == 128)
                attention_phase<128>(p, sm, ly, l, sc, sm.x[1], ctid);
            else
                attention_phase<64>(p, sm, ly, l, sc, sm.x[1], ctid);
            // ---- o_proj + residual: stage attn into x[1]; h = hraw[0] + W_o attn
            wait_ctr(ctr(p, l, E_ATT), static_cast<unsigned>(p.hkv * (t + 1)), p.err, ctid);
            MK_TR(l, 7);
            stage<T>(p.attn, nullptr, 0, p.hq * p.D, nullptr, sm.x[1], nullptr, nullptr, ctid);
            consume_k<T>(p, sm, phase_of(p, ly, K_O), l, K_O, k, sc, sm.x[1], sm.hraw[0], 1.0f, 8, ctid, wbest);
            signal(ctr(p, l, E_HO), ctid);
            MK_TR(l, 9);
            // ---- gate/up + SwiGLU: stage h into x[0] / hraw[1]
            wait_ctr(ctr(p, l, E_HO), full, p.err, ctid);
            MK_TR(l, 10);
            stage<T>(p.h, nullptr, 0, p.H, ly.post_norm, sm.x[0], sm.hraw[1], sm.red[1], ctid);
            const float s_post = norm_scale(sm.red[1], p.H, p.eps);
            consume_k<T>(p, sm, phase_of(p, ly, K_GU), l, K_GU, k, sc, sm.x[0], nullptr, s_post, 11, ctid, wbest);
            signal(ctr(p, l, E_ACT), ctid);
            MK_TR(l, 12);
            // ---- down + residual: stage act into x[1]; h = hraw[1] + W_d act
            wait_ctr(ctr(p, l, E_ACT), full, p.err, ctid);
            MK_TR(l, 13);
            stage<T>(p.act, nullptr, 0, p.I, nullptr, sm.x[1], nullptr, nullptr, ctid);
            consume_k<T>(p, sm, phase_of(p, ly, K_D), l, K_D, k, sc, sm.x[1], sm.hraw[1], 1.0f, 14, ctid, wbest);
            signal(ctr(p, l, E_HD), ctid);
            MK_TR(l, 15);
        }
        // ---- final norm + lm_head + argmax
        wait_ctr(ctr(p, p.L - 1, E_HD), full, p.err, ctid);
        MK_TR(p.L, 1);
        stage<T>(p.h, nullptr, 0, p.H, p.final_norm, sm.x[0], sm.hraw[0], sm.red[0], ctid);
        MK_TR(p.L, 2);
        const float s_fin = norm_scale(sm.red[0], p.H, p.eps);
        consume_k<T>(p, sm, phase_of(p, p.layers[0], K_LM), 0, K_LM, k, sc, sm.x[0], nullptr, s_fin, 3, ctid, wbest);
        if (lane == 0) sm.best[cw] = wbest;
        nbar();
        if (ctid == 0) {
            unsigned long long b = 0ull;
            for (int q = 0; q < NC; ++q) b = sm.best[q] > b ? sm.best[q] : b;
            p.best[static_cast<size_t>(t) * GRID + me] = b;
            red_release_add(ctr_lm(p));
        }
        MK_TR(p.L, 4);
    }
    if (me == 0 && !stopped) {
        const int t = p.steps - 1;
        wait_ctr(ctr_lm(p), static_cast<unsigned>(GRID * p.steps), p.err, ctid);
        if (cw == 0) {
            unsigned long long b = 0ull;
            for (int c = lane; c < GRID; c += 32) {
                const unsigned long long kk = __ldcg(p.best + static_cast<size_t>(t) * GRID + c);
                b = kk > b ? kk : b;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long other = __shfl_xor_sync(0xffffffffu, b, o);
                b = other > b ? other : b;
            }
            if (lane == 0) p.ids[p.steps] = b == 0ull ? 0 : argmax_key_index(b);
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

int mk_flag_count(int L, int hkv, int grid) { return (L * 6 + 1 + L * hkv) * FLAG_STRIDE + 0 * grid; }

size_t mk_vec_floats(int H, int I, int hq, int hkv, int D) {
    return static_cast<size_t>(H) + static_cast<size_t>(hq + 2 * hkv) * D + static_cast<size_t>(hq) * D + I;
}

bool mk_supported(int H, int I, int hq, int hkv, int D, int wfmt, int grid) {
    auto ki_ok = [](int K, bool pair) {
        const int ki = K / 256;
        if (K % 256 != 0) return false;
        return pair ? (ki == 1 || ki == 2 || ki == 4) : (ki == 1 || ki == 2 || ki == 4 || ki == 8 || ki == 12);
    };
    if (wfmt != WF_F16 && wfmt != WF_BF16) return false;
    if (!ki_ok(H, true) || !ki_ok(I, false) || !ki_ok(hq * D, false)) return false;
    if (D != 64 && D != 128) return false;
    if (hq % hkv != 0 || hq / hkv > MAXG || hq / hkv >= NC) return false;
    if (H > HMAX || I > XMAX || hq * D > XMAX) return false;
    if ((MAXG + 2) * D + NC * (hq / hkv) * (D + 2) > XMAX) return false;
    // one unit must fit a ring slot: (gate, up) pair rows and the widest single row
    if (2 * H * 2 > SLOT_BYTES || I * 2 > SLOT_BYTES || hq * D * 2 > SLOT_BYTES) return false;
    // every CTA owns rows of every phase (the hand-offs rely on it); flags polled per lane
    if (H < grid || I < grid || (hq + 2 * hkv) * D < grid || grid > 32 * MAXFL) return false;
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
