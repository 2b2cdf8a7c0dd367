// Persistent batch-1 decode kernel for sm_100a.
//
// One cooperative launch, one CTA per SM, runs `steps` greedy decode steps of one sequence:
// embedding -> L x [RMSNorm -> qkv -> q/k norm + RoPE + KV append -> GQA attention ->
// o_proj + residual -> RMSNorm -> gate/up + SwiGLU -> down + residual] -> final RMSNorm ->
// lm_head -> argmax, feeding each id to the next step on the device.  Same arithmetic as the
// reference (Mac/cpu/src/qwen_block.cpp:63-72, qwen_attention.cpp:142-205, qwen_mlp.cpp:65-74,
// qwen_causal_lm.cpp:82-116, sampler.cpp:26-62) except that an RMSNorm's scale is applied after
// the dot product: sum_i W[r,i] (x_i s w_i) = s * sum_i W[r,i] (x_i w_i).
//
// Batch-1 decode streams every weight byte once per token (1.19 GB for Qwen3-0.6B) through a
// chain of ~140 dependent matrix-vector products, so the design works on two things: keeping HBM
// busy across the dependencies, and making each dependency short.
//   * Weights are stored for this kernel in 8-row tiles (mk_tile_matrix): a tile's bytes are
//     contiguous and already in the register order of the B operand of mma.sync.m16n8k16, so a
//     lane reads its fragment of a 16-column step with one 8-byte shared-memory load (int8 / int4
//     tiles carry their group scales inline).
//   * warp 0, lane 0 is a producer: it walks this CTA's tiles of every matrix in execution order
//     and streams them into a 4 x 48 KB shared-memory ring with cp.async.bulk (mbarrier
//     completion, L2 evict-first).  It never waits on activations.
//   * warps 1..8 are consumers.  In a matrix phase each warp owns a K-slice (K / 8 columns) of
//     every tile the CTA holds: it waits for just its slice of the input vector, splits it into
//     fp16 (bf16: three) parts times a power of two (x = hi + lo, about 22 significant bits), and
//     runs the tensor-core MMAs with the parts as rows of the A operand and the weights as B;
//     fp32 accumulation.  The slices' partial sums are added in a fixed order (deterministic).
//   * Hand-offs carry their own readiness: every activation value is a 64-bit word {fp32 value,
//     32-bit tag}, stored with one relaxed 8-byte store; a reader polls the words it needs until
//     they carry the tag of the phase that writes them.  No counters and no fences between
//     phases; a reader starts on its slice as soon as that slice is complete.
//   * attention runs on kv_heads x splits units (one CTA each); the cached keys, the RoPE row and
//     the norm weights are loaded before the q/k/v rows arrive.  With more than one split the
//     unit of split 0 combines the partials.
//   * Between steps every CTA publishes its argmax key after a fence and reads all keys with a
//     fence after them: that orders everything of step t (the KV appends included) before step
//     t + 1.
// Every wait is bounded: on expiry the kernel sets DERR_WAIT_TIMEOUT in *err, which makes every
// other wait return at once, and the kernel winds down (the producer first waits, bounded, for
// its copies in flight).
#include <algorithm>
#include <type_traits>

#include "decode_mk.h"

namespace socb {
namespace {

constexpr int NW = 8;                    // consumer warps
constexpr int CT = NW * 32;              // consumer threads
constexpr int THREADS = CT + 32;         // + producer warp
constexpr int SLOTS = 4;
constexpr int SLOT_BYTES = 48 * 1024;
constexpr int KS_MAX = 384;              // widest per-warp slice of an input vector
constexpr int NSPLIT = 3;                // parts of a split input (fp16 uses 2, bf16 3)
constexpr int MAXG = 2;                  // query heads per kv head
constexpr int MAX_ROWS = 64;             // rows of one matrix phase on one CTA
constexpr int KPF = 4;                   // keys per warp per attention batch
constexpr int UNIT_KEYS = 64;            // keys per attention unit (two batches per warp)
constexpr unsigned SPIN_LIMIT = 1u << 22;
constexpr int LMAX = 48;                 // layers whose weight pointers are kept in shared memory
constexpr int XS_PAD = 16;               // halves of padding per part row of xs

enum Ph { P_QKV = 0, P_ATT = 1, P_O = 2, P_GU = 3, P_D = 4 };
// producer / tile-range phases (the lm_head is phase 4 of "layer" L)
enum MPh { M_QKV = 0, M_O = 1, M_GU = 2, M_D = 3, M_LM = 4 };

struct __align__(128) Smem {
    uint8_t ring[SLOTS][SLOT_BYTES];
    // split input slices in A-fragment order (xs_pos); attention scratch.  The rows are padded
    // so that part rows start 8 banks apart (the A loads of one step hit distinct banks).
    uint16_t xs[NSPLIT][NW * KS_MAX + XS_PAD];
    float red[2][NW][MAX_ROWS];        // per-warp partial sums, double-buffered across phases
    float wss[2][NW];                  // per-warp sums of squares (same double buffering)
    float lss[NW], lmax[NW];           // the lm_head's staging
    unsigned long long best[NW];
    unsigned long long full[SLOTS];
    unsigned long long empty[SLOTS];
    MKLayer layers[LMAX];
    int tok;
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
        if (i > SPIN_LIMIT) {
            atomicOr(err, DERR_WAIT_TIMEOUT);
            return false;
        }
        if (i > 64) __nanosleep(20);
    }
}

// ------------------------------------------------------------ tagged words
__device__ __forceinline__ void st_word(unsigned long long* p, float v, uint32_t tag) {
    const unsigned long long w = (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ld_word(const unsigned long long* p) {
    unsigned long long w;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
__device__ __forceinline__ uint32_t word_tag(unsigned long long w) { return static_cast<uint32_t>(w >> 32); }
// Loads issued ahead of a poll (norm weights, RoPE rows, cached keys).  They are relaxed (strong)
// loads so that they stay in program order with the poll's loads: a weak load may be scheduled
// after the poll, which would put a second memory round trip on the critical path.
__device__ __forceinline__ uint32_t ld_ahead_u32(const void* p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint2 ld_ahead_u64(const void* p) {
    uint2 v;
    asm volatile("ld.relaxed.gpu.global.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ float ld_ahead_f32(const float* p) { return __uint_as_float(ld_ahead_u32(p)); }
__device__ __forceinline__ float2 ld_ahead_f2(const float2* p) {
    const uint2 v = ld_ahead_u64(p);
    return make_float2(__uint_as_float(v.x), __uint_as_float(v.y));
}
// Largest of the lanes' values, for values >= 0 (their bit patterns order like the values).
__device__ __forceinline__ float warp_max_nonneg(float v) {
    return __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(v)));
}
__device__ __forceinline__ float word_val(unsigned long long w) { return __uint_as_float(static_cast<uint32_t>(w)); }

__device__ __forceinline__ uint32_t mk_tag(const MKParams& p, int t, int l, int ph) {
    return p.tag0 + static_cast<uint32_t>((t * p.L + l) * MK_PHASES + ph) + 1u;
}

// Reads words src[STRIDE * i] (i < M), waiting (bounded) until each carries `tag`.  Every round
// issues all of its loads before it checks any, so a round costs one memory round trip; rounds follow
// each other without a sleep (measured: a 32 ns sleep between rounds costs 6 % of the decode step,
// an 8 ns one 3 %), and the round count bounds the wait.
template <int M, int STRIDE>
__device__ __forceinline__ bool poll_words(const unsigned long long* src, uint32_t tag, float (&v)[M], int* err) {
    uint32_t pending = (M >= 32) ? 0xffffffffu : ((1u << M) - 1u);
    for (unsigned it = 0;; ++it) {
        unsigned long long w[M];
#pragma unroll
        for (int i = 0; i < M; ++i) w[i] = ((pending >> i) & 1u) ? ld_word(src + STRIDE * i) : 0ull;
        uint32_t still = 0u;
#pragma unroll
        for (int i = 0; i < M; ++i) {
            if ((pending >> i) & 1u) {
                if (word_tag(w[i]) == tag)
                    v[i] = word_val(w[i]);
                else
                    still |= 1u << i;
            }
        }
        pending = still;
        if (pending == 0u) return true;
        if ((it & 15u) == 15u && aborted(err)) return false;
        if (it > SPIN_LIMIT) {
            atomicOr(err, DERR_WAIT_TIMEOUT);
            return false;
        }
    }
}

// As poll_words with a run-time stride; words i >= n are not read (v[i] = 0).
template <int M>
__device__ __forceinline__ bool poll_strided(const unsigned long long* src, int stride, int n, uint32_t tag,
                                             float (&v)[M], int* err) {
    uint32_t pending = 0u;
#pragma unroll
    for (int i = 0; i < M; ++i) {
        v[i] = 0.0f;
        if (i < n) pending |= 1u << i;
    }
    for (unsigned it = 0; pending != 0u; ++it) {
        unsigned long long w[M];
#pragma unroll
        for (int i = 0; i < M; ++i) w[i] = ((pending >> i) & 1u) ? ld_word(src + static_cast<size_t>(stride) * i) : 0ull;
        uint32_t still = 0u;
#pragma unroll
        for (int i = 0; i < M; ++i) {
            if ((pending >> i) & 1u) {
                if (word_tag(w[i]) == tag)
                    v[i] = word_val(w[i]);
                else
                    still |= 1u << i;
            }
        }
        pending = still;
        if (pending == 0u) break;
        if ((it & 15u) == 15u && aborted(err)) return false;
        if (it > SPIN_LIMIT) {
            atomicOr(err, DERR_WAIT_TIMEOUT);
            return false;
        }
    }
    return true;
}


// One word, waiting (bounded) for its tag.
__device__ __forceinline__ float poll_one(const unsigned long long* src, uint32_t tag, int* err) {
    float v[1] = {0.0f};
    poll_words<1, 1>(src, tag, v, err);
    return v[0];
}

// The argmax keys of `n` CTAs (nonzero once written), this lane's share (c = lane + 32 i), maxed;
// bounded like every other wait.
__device__ __forceinline__ unsigned long long poll_keys(const unsigned long long* src, int n, int lane, int* err) {
    constexpr int KMAX = 8;  // grids up to 256 CTAs
    uint32_t pending = 0u;
#pragma unroll
    for (int i = 0; i < KMAX; ++i)
        if (lane + 32 * i < n) pending |= 1u << i;
    unsigned long long best = 0ull;
    for (unsigned it = 0;; ++it) {
        unsigned long long w[KMAX];
#pragma unroll
        for (int i = 0; i < KMAX; ++i) w[i] = ((pending >> i) & 1u) ? ld_word(src + lane + 32 * i) : 0ull;
#pragma unroll
        for (int i = 0; i < KMAX; ++i) {
            if (((pending >> i) & 1u) && w[i] != 0ull) {
                best = w[i] > best ? w[i] : best;
                pending &= ~(1u << i);
            }
        }
        if (pending == 0u) break;
        if ((it & 15u) == 15u && aborted(err)) break;
        if (it > SPIN_LIMIT) {
            atomicOr(err, DERR_WAIT_TIMEOUT);
            break;
        }
    }
    return best;
}

// Trace slot `e` of layer `l` (first step only, consumer thread 0).  Slots per layer: 0 start;
// per matrix phase (base 1 qkv, 6 o, 11 gu, 16 down): +0 entry, +1 slice ready, +2 products
// done, +3 after the CTA barrier, +4 outputs stored; 26 + phase: first chunk resident; 36 +
// phase: first chunk's products done; 30 / 31: the residual of the o / down epilogue in hand;
// attention: 21 input ready, 32 normed and rotated, 23 q/k/v staged, 33 first keys unpacked,
// 24 keys done, 25 partials merged, 34 merge weights ready, 35 outputs stored, 22 done.
// Layer L holds the lm_head: 1 input ready, 2 staged, 4 done.
#define MK_TR(l, e)                                                                                                  \
    do {                                                                                                             \
        if (p.trace != nullptr && sc.t == 0 && cw == 0 && lane == 0)                                                 \
            p.trace[static_cast<size_t>(blockIdx.x) * mk_trace_stride(p.L) + (l) * MK_TRACE_PER_LAYER + (e)] =      \
                gtime();                                                                                             \
    } while (0)

// ------------------------------------------------------------------- tile formats
// fp16 / bf16: 16 columns of a tile = 256 bytes, lane l's 8 bytes at 8 l:
//   W[8 t + g][16 kt + 2 q + {0, 1, 8, 9}] with g = l / 4, q = l % 4.
// int8 g64: per group of 64 columns 528 bytes: four 128-byte column steps (lane l's 4 bytes at
//   4 l, the same elements, biased by +128) then the 8 rows' fp16 scales.
// int4 g32: per group of 32 columns 144 bytes: lane l's 4 bytes at 4 l hold both 16-column
//   steps (byte 2s: elements 0 and 2 of step s as nibbles, byte 2s + 1: elements 1 and 3;
//   biased by +8), then the 8 rows' fp16 scales.
__host__ __device__ __forceinline__ size_t tile_bytes(int wfmt, int K) {
    switch (wfmt) {
        case WF_I8G64: return static_cast<size_t>(K / 64) * 528;
        case WF_I4G32: return static_cast<size_t>(K / 32) * 144;
        default: return static_cast<size_t>(K) * 16;
    }
}

// int8 bytes (biased) -> two half2 of the integers, exactly
__device__ __forceinline__ void i8_to_h2(uint32_t w, uint32_t& lo, uint32_t& hi) {
    const uint32_t a = __byte_perm(w, 0x64646464u, 0x4140u), b = __byte_perm(w, 0x64646464u, 0x4342u);
    const __half2 bias = __halves2half2(__ushort_as_half(0x6480u), __ushort_as_half(0x6480u));  // 1152
    const __half2 x = __hsub2(*reinterpret_cast<const __half2*>(&a), bias);
    const __half2 y = __hsub2(*reinterpret_cast<const __half2*>(&b), bias);
    lo = *reinterpret_cast<const uint32_t*>(&x);
    hi = *reinterpret_cast<const uint32_t*>(&y);
}
// two int4 bytes (biased nibbles, see above) -> two half2, exactly; `sel` picks bytes (0,1) or (2,3)
__device__ __forceinline__ void i4_to_h2(uint32_t w, uint32_t sel, uint32_t& lo, uint32_t& hi) {
    const uint32_t v = __byte_perm(w, 0u, sel);
    const uint32_t a = (v & 0x000F000Fu) | 0x64006400u, b = ((v >> 4) & 0x000F000Fu) | 0x64006400u;
    const __half2 bias = __halves2half2(__ushort_as_half(0x6408u), __ushort_as_half(0x6408u));  // 1032
    const __half2 x = __hsub2(*reinterpret_cast<const __half2*>(&a), bias);
    const __half2 y = __hsub2(*reinterpret_cast<const __half2*>(&b), bias);
    lo = *reinterpret_cast<const uint32_t*>(&x);
    hi = *reinterpret_cast<const uint32_t*>(&y);
}

// D += A(16x16: rows g = the input's parts) * B(16x8: 8 weight rows), fp32 accumulation.
template <typename TX>
__device__ __forceinline__ void mma(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma<__half>(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma<__nv_bfloat16>(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0,
                                                    uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}

template <typename TX>
struct Split;
template <>
struct Split<__half> {
    static constexpr int N = 2;
    static __device__ __forceinline__ void run(float x, uint16_t (&o)[NSPLIT]) {
        const __half h = __float2half_rn(x);
        const __half l = __float2half_rn(x - __half2float(h));
        o[0] = __half_as_ushort(h);
        o[1] = __half_as_ushort(l);
        o[2] = 0;
    }
};
template <>
struct Split<__nv_bfloat16> {
    static constexpr int N = 3;
    static __device__ __forceinline__ void run(float x, uint16_t (&o)[NSPLIT]) {
        const __nv_bfloat16 h = __float2bfloat16_rn(x);
        const float r = x - __bfloat162float(h);
        const __nv_bfloat16 m = __float2bfloat16_rn(r);
        const __nv_bfloat16 l = __float2bfloat16_rn(r - __bfloat162float(m));
        o[0] = __bfloat16_as_ushort(h);
        o[1] = __bfloat16_as_ushort(m);
        o[2] = __bfloat16_as_ushort(l);
    }
};

// 2^e for |e| <= 126 (exact)
__device__ __forceinline__ float pow2i(int e) { return __int_as_float((e + 127) << 23); }

// Exponent that scales `mx` into [2^14, 2^15) (fp16 parts keep ~22 bits, far from overflow).
__device__ __forceinline__ int split_exponent(float mx) {
    if (!(mx > 0.0f) || !(mx < 3.0e38f)) return 0;
    const int ex = static_cast<int>((__float_as_uint(mx) >> 23) & 0xffu) - 127;
    return max(-100, min(100, 14 - ex));
}

// Position of input element x in a part row of xs: within each 16-column step the elements a
// lane with q = lane % 4 feeds to the MMA (2q, 2q + 1, 2q + 8, 2q + 9) sit together at 4q, so
// the lane reads its A registers of a step with one 8-byte load.
__device__ __forceinline__ int xs_pos(int x) {
    const int j = x & 15;
    return (x & ~15) | (((j & 7) >> 1) << 2) | ((j >> 3) << 1) | (j & 1);
}

// Writes this lane's M values (already scaled) as parts into xs[part][xs_pos(base + 32 i + lane)].
template <typename TX, int M>
__device__ __forceinline__ void write_parts(Smem& sm, int base, int lane, const float (&v)[M]) {
#pragma unroll
    for (int i = 0; i < M; ++i) {
        uint16_t o[NSPLIT];
        Split<TX>::run(v[i], o);
#pragma unroll
        for (int s = 0; s < Split<TX>::N; ++s) sm.xs[s][xs_pos(base + 32 * i + lane)] = o[s];
    }
}

// Reads words src[32 i + lane], i < M (a warp's slice, coalesced), waiting (bounded) for `tag`.
template <int M>
__device__ __forceinline__ bool poll_slice(const unsigned long long* src, int lane, uint32_t tag, float (&v)[M],
                                           int* err) {
    return poll_words<M, 32>(src + lane, tag, v, err);
}

// ------------------------------------------------------------------- schedule
// Contiguous tile range of CTA `cta` in phase `ph` of layer l; the rotation moves the larger
// shares around so every CTA streams about the same number of bytes per token.
__device__ __forceinline__ void cta_tiles(int tiles, int cta, int G, int l, int ph, int& a, int& b) {
    // 32-bit unsigned arithmetic (tiles * G < 2^32 for every supported shape)
    const unsigned v = static_cast<unsigned>(cta + (l * 5 + ph) * 37) % static_cast<unsigned>(G);
    a = static_cast<int>(static_cast<unsigned>(tiles) * v / static_cast<unsigned>(G));
    b = static_cast<int>(static_cast<unsigned>(tiles) * (v + 1u) / static_cast<unsigned>(G));
}

struct Mat {
    const uint8_t* w;
    int tiles, K, fmt;
    size_t tb;  // bytes per tile
    int tpc;    // tiles per chunk
};

__device__ __forceinline__ Mat mat_of(const MKParams& p, const MKLayer& ly, int ph) {
    Mat m;
    m.fmt = p.wfmt;
    switch (ph) {
        case M_QKV:
            m.w = static_cast<const uint8_t*>(ly.wqkv);
            m.tiles = (p.hq + 2 * p.hkv) * p.D / 8;
            m.K = p.H;
            break;
        case M_O:
            m.w = static_cast<const uint8_t*>(ly.wo);
            m.tiles = p.H / 8;
            m.K = p.hq * p.D;
            break;
        case M_GU:
            m.w = static_cast<const uint8_t*>(ly.wgu);
            m.tiles = 2 * p.I / 8;
            m.K = p.H;
            break;
        case M_D:
            m.w = static_cast<const uint8_t*>(ly.wd);
            m.tiles = p.H / 8;
            m.K = p.I;
            break;
        default:
            m.w = static_cast<const uint8_t*>(p.lm_tiles);
            m.tiles = p.V / 8;
            m.K = p.H;
            m.fmt = p.efmt;
            break;
    }
    m.tb = tile_bytes(m.fmt, m.K);
    m.tpc = max(1, static_cast<int>(static_cast<unsigned>(SLOT_BYTES) / static_cast<unsigned>(m.tb)));
    return m;
}

// ------------------------------------------------------------------- producer
// Walks this CTA's chunks in consumption order: per step, per layer the qkv, o, gate/up and
// down tiles, then the lm_head's.  A chunk is up to `tpc` whole tiles of one phase.
struct Cursor {
    int t, l, ph;
    int u, b;  // next tile and end of this CTA's range in the current phase
    Mat m;
    bool done;
};

__device__ __forceinline__ void cursor_phase(const MKParams& p, const Smem& sm, Cursor& c) {
    c.m = mat_of(p, sm.layers[c.ph == M_LM ? 0 : c.l], c.ph);
    int a, b;
    cta_tiles(c.m.tiles, blockIdx.x, gridDim.x, c.ph == M_LM ? 0 : c.l, c.ph, a, b);
    c.u = a;
    c.b = b;
}

__device__ __forceinline__ void cursor_next_phase(const MKParams& p, const Smem& sm, Cursor& c) {
    do {
        if (c.ph == M_LM) {
            c.ph = M_QKV;
            c.l = 0;
            if (++c.t >= p.steps) {
                c.done = true;
                return;
            }
        } else if (c.ph == M_D) {
            if (++c.l >= p.L) {
                c.ph = M_LM;
                c.l = 0;
            } else {
                c.ph = M_QKV;
            }
        } else {
            ++c.ph;
        }
        cursor_phase(p, sm, c);
    } while (c.u >= c.b);
}

__device__ __forceinline__ void cursor_init(const MKParams& p, const Smem& sm, Cursor& c) {
    c.t = 0;
    c.l = 0;
    c.ph = M_QKV;
    c.done = p.steps <= 0;
    if (c.done) return;
    cursor_phase(p, sm, c);
    if (c.u >= c.b) cursor_next_phase(p, sm, c);
}

// lm_head prefetch: issued at the start of the last layer(s), this many KB per CTA.  Measured at
// config 0: 1 layer x 250 KB gives 0.5194 -> 0.5166 ms/token; 3-5 layers or 400-500 KB give
// nothing or lose (the prefetch then competes with the layers' own weight stream).
constexpr int MK_LM_PF_LAYERS = 1;
constexpr int MK_LM_PF_KB = 250;
// The first bytes of this CTA's lm_head range, prefetched into L2 (kept, evict-last) while the last
// layers run: HBM is mostly idle during the layers' dependent phases, and the lm_head phase then
// reads part of its 311 MB from L2.
__device__ __forceinline__ void prefetch_lm(const MKParams& p, const Smem& sm) {
    const Mat m = mat_of(p, sm.layers[0], M_LM);
    int a, b;
    cta_tiles(m.tiles, blockIdx.x, gridDim.x, 0, M_LM, a, b);
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    const size_t total = static_cast<size_t>(b - a) * m.tb;
    const size_t want = min(total, static_cast<size_t>(MK_LM_PF_KB) * 1024);
    const uint8_t* src = m.w + static_cast<size_t>(a) * m.tb;
    for (size_t off = 0; off < want; off += 32768) {
        const unsigned bytes = static_cast<unsigned>(min(static_cast<size_t>(32768), want - off));
        asm volatile("cp.async.bulk.prefetch.L2.global.L2::cache_hint [%0], %1, %2;" ::"l"(src + off), "r"(bytes & ~15u),
                     "l"(pol)
                     : "memory");
    }
}

// The whole warp 0 runs the loop in step (so that the end-of-step argmax keys are read 32 at a
// time); lane 0 issues the copies.
__device__ __forceinline__ void producer(const MKParams& p, Smem& sm, int lane) {
    const uint64_t pol = evict_first_policy();
    Cursor c;
    cursor_init(p, sm, c);
    long long k = 0;
    int checked = -1;  // last step whose input id was compared with p.eos
    int prefetched = -1;  // last step whose lm_head head was prefetched
    while (!c.done) {
        if (c.t != prefetched && c.ph == M_QKV && c.l >= p.L - MK_LM_PF_LAYERS) {
            prefetched = c.t;
            if (lane == 0) prefetch_lm(p, sm);
        }
        if (p.eos >= 0 && c.t != checked) {
            // The first chunk of step c.t: load it only if that step runs, i.e. its input id
            // (step 0: ids[0]; later: the merged argmax of the step before) is not eos.  The
            // consumers take the same decision from the same keys at the top of the step.
            checked = c.t;
            int tok = 0;
            if (c.t == 0) {
                tok = __ldcg(p.ids);
            } else {
                unsigned long long bk = poll_keys(p.best + static_cast<size_t>(c.t - 1) * gridDim.x,
                                                  static_cast<int>(gridDim.x), lane, p.err);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const unsigned long long other = __shfl_xor_sync(0xffffffffu, bk, o);
                    bk = other > bk ? other : bk;
                }
                if (aborted(p.err)) break;
                tok = bk <= 1ull ? 0 : argmax_key_index(bk);
            }
            if (tok == p.eos) break;
        }
        const int slot = static_cast<int>(k % SLOTS);
        const long long round = k / SLOTS;
        bool ok = true;
        if (lane == 0) {
            if (round > 0 && !mbar_wait(&sm.empty[slot], static_cast<unsigned>((round - 1) & 1), p.err)) ok = false;
            // at most `inflight` copies outstanding: more bytes in flight than the memory system
            // needs to stay busy only lengthen every other load's queueing
            if (ok && p.inflight < SLOTS && k >= p.inflight) {
                const long long q = k - p.inflight;
                if (!mbar_wait(&sm.full[q % SLOTS], static_cast<unsigned>((q / SLOTS) & 1), p.err)) ok = false;
            }
            if (ok) {
                const int n = min(c.m.tpc, c.b - c.u);
                const uint8_t* src = c.m.w + static_cast<size_t>(c.u) * c.m.tb;
                const unsigned bytes = static_cast<unsigned>(n) * static_cast<unsigned>(c.m.tb);
                mbar_expect_tx(&sm.full[slot], bytes);
                bulk_g2s(sm.ring[slot], src, bytes, &sm.full[slot], pol);
            }
        }
        if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
        c.u += min(c.m.tpc, c.b - c.u);
        if (c.u >= c.b) cursor_next_phase(p, sm, c);
        ++k;
    }
    // Never leave with copies in flight: wait (bounded) for the last fills to land.
    if (lane == 0) {
        const long long first = k > SLOTS ? k - SLOTS : 0;
        for (long long q = first; q < k; ++q) {
            const int slot = static_cast<int>(q % SLOTS);
            for (unsigned i = 0; i < SPIN_LIMIT; ++i) {
                if (mbar_test(&sm.full[slot], static_cast<unsigned>((q / SLOTS) & 1))) break;
                __nanosleep(32);
            }
        }
    }
}

// ------------------------------------------------------------------ consumers
struct StepCtx {
    int t, tok, pos;
};

// Source of a matrix phase's input vector.
struct Input {
    const unsigned long long* words;  // tagged words (nullptr: the embedding row of the token)
    uint32_t tag;
    const float* norm;  // RMSNorm weight, or nullptr
};

// Output epilogues of a matrix phase.
enum Epi { E_STORE_SCALED = 0, E_RESIDUAL = 1, E_SWIGLU = 2 };

struct Output {
    unsigned long long* words;  // destination (row index = global row of the phase's matrix)
    uint32_t tag;
    int epi;
    // E_RESIDUAL: the residual stream before this phase (words with `res_tag`, or the embedding)
    const unsigned long long* res;
    uint32_t res_tag;
};

// Loads this warp's slice [base, base + KS) of the input (times the norm weight; lane l holds
// elements base + 32 i + l), returning the raw sum of squares (for the norm) and writing the
// scaled parts into xs.  Returns the power-of-two exponent of the scaling.
template <typename TX, typename TE, int KS>
__device__ __forceinline__ int load_slice(const MKParams& p, Smem& sm, const Input& in, const StepCtx& sc, int base,
                                          int lane, float& ss) {
    constexpr int M = KS / 32;
    float v[M], nv[M];
    // the norm weights do not depend on the input: load them before waiting for it
#pragma unroll
    for (int i = 0; i < M; ++i) nv[i] = in.norm ? ld_ahead_f32(in.norm + base + 32 * i + lane) : 1.0f;
    if (in.words == nullptr) {
        const TE* e = static_cast<const TE*>(p.embed) + static_cast<size_t>(sc.tok) * p.H + base + lane;
#pragma unroll
        for (int i = 0; i < M; ++i) {
            if constexpr (std::is_same<TE, __half>::value)
                v[i] = __half2float(e[32 * i]);
            else
                v[i] = __bfloat162float(e[32 * i]);
        }
    } else {
        poll_slice<M>(in.words + base, lane, in.tag, v, p.err);
    }
    ss = 0.0f;
    float mx = 0.0f;
#pragma unroll
    for (int i = 0; i < M; ++i) {
        ss += v[i] * v[i];
        v[i] *= nv[i];
        mx = fmaxf(mx, fabsf(v[i]));
    }
    mx = warp_max_nonneg(mx);
    const int e = split_exponent(mx);
    const float sc2 = pow2i(e);
#pragma unroll
    for (int i = 0; i < M; ++i) v[i] *= sc2;
    write_parts<TX, M>(sm, base, lane, v);
    __syncwarp();
    return e;
}

// The A fragment of 16-column step kt of this warp's slice.  Rows g < parts hold the input's
// parts (read from xs); the other rows repeat them (row g reads part g mod parts).  Row g of the
// product depends only on row g of A, and only rows g < parts are used, so the repeats cost
// nothing and every lane loads without a branch.
struct AFrag {
    const uint16_t* row;  // this lane's part row at the slice start, plus 4 q (xs_pos order)
    __device__ __forceinline__ void at(int kt, uint32_t& a0, uint32_t& a2) const {
        const uint2 v = *reinterpret_cast<const uint2*>(row + kt * 16);
        a0 = v.x;
        a2 = v.y;
    }
};

template <typename TX>
__device__ __forceinline__ AFrag afrag_of(const Smem& sm, int base, int lane) {
    const int g = lane >> 2, q = lane & 3;
    AFrag f;
    f.row = sm.xs[g % Split<TX>::N] + base + 4 * q;
    return f;
}

// Sum of the parts' rows (lanes 0..3 end up with rows 2q, 2q + 1 of the tile).
template <typename TX>
__device__ __forceinline__ void combine_parts(float& d0, float& d1) {
    const float a0 = __shfl_down_sync(0xffffffffu, d0, 4), a1 = __shfl_down_sync(0xffffffffu, d1, 4);
    float b0 = 0.0f, b1 = 0.0f;
    if (Split<TX>::N == 3) {
        b0 = __shfl_down_sync(0xffffffffu, d0, 8);
        b1 = __shfl_down_sync(0xffffffffu, d1, 8);
    }
    d0 = d0 + a0 + b0;
    d1 = d1 + a1 + b1;
}

// This warp's slice of up to NT tiles at once (t0 + i * tb, i < nt): the partial dot products of
// each tile's 8 rows (d0[i], d1[i] on lanes 0..3).  The tiles share each A fragment and their
// MMAs are independent, so they overlap.
template <typename TX, int F, int KT, int NT, typename AOp>
__device__ __forceinline__ void tiles_slice(const uint8_t* t0, size_t tb, int nt, int kt0, int lane, const AOp& af,
                                            float (&d0)[NT], float (&d1)[NT]) {
    if constexpr (F == WF_F16 || F == WF_BF16) {
        constexpr int NA = NT > 1 ? 1 : (KT >= 16 ? 4 : 2);  // independent accumulators per tile
        float acc[NT][NA][4];
#pragma unroll
        for (int i = 0; i < NT; ++i)
#pragma unroll
            for (int a = 0; a < NA; ++a) acc[i][a][0] = acc[i][a][1] = acc[i][a][2] = acc[i][a][3] = 0.0f;
        const uint8_t* bp = t0 + static_cast<size_t>(kt0) * 256 + lane * 8;
        // several tiles at once: blocks of (at most) 8 steps, each unrolled, bound the registers;
        // one tile (the o_proj and down_proj slices, 16 and 24 steps): the whole slice unrolled
        // (measured 2.5 % faster per decode step than blocks of 8)
        constexpr int KB = NT > 1 ? (KT < 8 ? KT : 8) : KT;
#pragma unroll 1
        for (int k8 = 0; k8 < KT; k8 += KB) {
#pragma unroll
            for (int c = 0; c < KB; ++c) {
                uint32_t a0, a2;
                af.at(k8 + c, a0, a2);
#pragma unroll
                for (int i = 0; i < NT; ++i) {
                    if (i < nt) {
                        const uint2 b = *reinterpret_cast<const uint2*>(bp + i * tb + (k8 + c) * 256);
                        mma<TX>(acc[i][c % NA], a0, a2, b.x, b.y);
                    }
                }
            }
        }
#pragma unroll
        for (int i = 0; i < NT; ++i) {
            d0[i] = 0.0f;
            d1[i] = 0.0f;
#pragma unroll
            for (int a = 0; a < NA; ++a) {
                d0[i] += acc[i][a][0];
                d1[i] += acc[i][a][1];
            }
        }
    } else if constexpr (F == WF_I8G64) {
        // groups of 64 columns = 4 steps
        constexpr int NG = KT / 4;
        const int q0 = kt0 / 4;
        const int q = lane & 3;
#pragma unroll
        for (int i = 0; i < NT; ++i) d0[i] = d1[i] = 0.0f;
#pragma unroll
        for (int gq = 0; gq < NG; ++gq) {
            float acc[NT][4];
#pragma unroll
            for (int i = 0; i < NT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;
#pragma unroll
            for (int st = 0; st < 4; ++st) {
                uint32_t a0, a2;
                af.at(gq * 4 + st, a0, a2);
#pragma unroll
                for (int i = 0; i < NT; ++i) {
                    if (i < nt) {
                        const uint8_t* gp = t0 + i * tb + static_cast<size_t>(q0 + gq) * 528;
                        uint32_t b0, b1;
                        i8_to_h2(*reinterpret_cast<const uint32_t*>(gp + st * 128 + lane * 4), b0, b1);
                        mma<__half>(acc[i], a0, a2, b0, b1);
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < NT; ++i) {
                if (i < nt) {
                    const uint8_t* gp = t0 + i * tb + static_cast<size_t>(q0 + gq) * 528;
                    const float2 s2 = __half22float2(*reinterpret_cast<const __half2*>(gp + 512 + q * 4));
                    d0[i] = fmaf(acc[i][0], s2.x, d0[i]);
                    d1[i] = fmaf(acc[i][1], s2.y, d1[i]);
                }
            }
        }
    } else {  // WF_I4G32: groups of 32 columns = 2 steps
        constexpr int NG = KT / 2;
        const int q0 = kt0 / 2;
        const int q = lane & 3;
#pragma unroll
        for (int i = 0; i < NT; ++i) d0[i] = d1[i] = 0.0f;
#pragma unroll
        for (int gq = 0; gq < NG; ++gq) {
            uint32_t a0, a2, a4, a6;
            af.at(gq * 2, a0, a2);
            af.at(gq * 2 + 1, a4, a6);
#pragma unroll
            for (int i = 0; i < NT; ++i) {
                if (i < nt) {
                    const uint8_t* gp = t0 + i * tb + static_cast<size_t>(q0 + gq) * 144;
                    const uint32_t w = *reinterpret_cast<const uint32_t*>(gp + lane * 4);
                    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                    uint32_t b0, b1;
                    i4_to_h2(w, 0x4140u, b0, b1);
                    mma<__half>(acc, a0, a2, b0, b1);
                    i4_to_h2(w, 0x4342u, b0, b1);
                    mma<__half>(acc, a4, a6, b0, b1);
                    const float2 s2 = __half22float2(*reinterpret_cast<const __half2*>(gp + 128 + q * 4));
                    d0[i] = fmaf(acc[0], s2.x, d0[i]);
                    d1[i] = fmaf(acc[1], s2.y, d1[i]);
                }
            }
        }
    }
}

// One matrix phase on this CTA: its tiles [a, b) of `mt`, input `in`, epilogue `out`.
// `k` counts the ring chunks consumed so far; `rb` selects the reduction buffer.
template <typename TX, typename TE, int F, int KS>
__device__ __forceinline__ bool matrix_phase(const MKParams& p, Smem& sm, const Mat& mt, int a, int b, const Input& in,
                                          const Output& out, const StepCtx& sc, long long& k, int rb, int l, int tr,
                                          int cw, int lane) {
    constexpr int KT = KS / 16;
    if (a >= b) return false;
    MK_TR(l, tr);
    const int base = cw * KS;
    const int ctid = cw * 32 + lane;
    const int rows = (b - a) * 8;
    // the residual words of this thread's output row were written phases ago: load them now,
    // check their tag in the epilogue
    unsigned long long res_w = 0ull;
    if (out.epi == E_RESIDUAL && out.res != nullptr && ctid < rows) res_w = ld_word(out.res + a * 8 + ctid);
    float ss;
    const int e = load_slice<TX, TE, KS>(p, sm, in, sc, base, lane, ss);
    MK_TR(l, tr + 1);
    const AFrag afs = afrag_of<TX>(sm, base, lane);
    const float unscale = pow2i(-e);
    const int kt0 = cw * KT;
    for (int u = a; u < b; ++k) {
        const int n = min(mt.tpc, b - u);
        const int slot = static_cast<int>(k % SLOTS);
        const bool ok = mbar_wait(&sm.full[slot], static_cast<unsigned>((k / SLOTS) & 1), p.err);
        if (u == a) MK_TR(l, 26 + tr / 5);
        if (ok) {
            constexpr int NT = KS <= 128 ? 4 : 1;  // tiles in flight per warp
            for (int i0 = 0; i0 < n; i0 += NT) {
                const int nt = min(NT, n - i0);
                float d0[NT], d1[NT];
                tiles_slice<TX, F, KT, NT>(sm.ring[slot] + static_cast<size_t>(i0) * mt.tb, mt.tb, nt, kt0, lane, afs,
                                           d0, d1);
#pragma unroll
                for (int i = 0; i < NT; ++i) {
                    if (i < nt) {
                        combine_parts<TX>(d0[i], d1[i]);
                        if (lane < 4) {
                            float* r = sm.red[rb][cw] + (u - a + i0 + i) * 8 + 2 * lane;
                            r[0] = d0[i] * unscale;
                            r[1] = d1[i] * unscale;
                        }
                    }
                }
            }
        }
        if (u == a) MK_TR(l, 36 + tr / 5);
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.empty[slot]);
        u += n;
    }
    if (in.norm) {
        ss = warp_sum(ss);
        if (lane == 0) sm.wss[rb][cw] = ss;
    }
    MK_TR(l, tr + 2);
    nbar();
    MK_TR(l, tr + 3);
    // epilogue: one thread per output row (SwiGLU: per (gate, up) pair)
    float s = 1.0f;
    if (in.norm) {
        float tot = 0.0f;
#pragma unroll
        for (int w = 0; w < NW; ++w) tot += sm.wss[rb][w];
        s = 1.0f / sqrtf(tot / static_cast<float>(mt.K) + p.eps);
    }
    if (out.epi == E_SWIGLU) {
        if (ctid < rows / 2) {
            float g = 0.0f, up = 0.0f;
#pragma unroll
            for (int w = 0; w < NW; ++w) {
                g += sm.red[rb][w][2 * ctid];
                up += sm.red[rb][w][2 * ctid + 1];
            }
            const int j = (a * 8) / 2 + ctid;
            st_word(out.words + j, silu_f(g * s) * (up * s), out.tag);
        }
    } else if (ctid < rows) {
        float y = 0.0f;
#pragma unroll
        for (int w = 0; w < NW; ++w) y += sm.red[rb][w][ctid];
        const int r = a * 8 + ctid;
        if (out.epi == E_STORE_SCALED) {
            st_word(out.words + r, y * s, out.tag);
        } else {
            float hr;
            if (out.res == nullptr) {
                const TE* e = static_cast<const TE*>(p.embed) + static_cast<size_t>(sc.tok) * p.H + r;
                if constexpr (std::is_same<TE, __half>::value)
                    hr = __half2float(*e);
                else
                    hr = __bfloat162float(*e);
            } else {
                hr = word_tag(res_w) == out.res_tag ? word_val(res_w) : poll_one(out.res + r, out.res_tag, p.err);
            }
            if (tr == 6) MK_TR(l, 30);
            if (tr == 16) MK_TR(l, 31);
            st_word(out.words + r, hr + y, out.tag);
        }
    }
    MK_TR(l, tr + 4);
    return true;
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


// A lane's DL consecutive floats of a head row in shared memory, as one vector access (16 bytes for
// D = 128, 8 for D = 64): a warp's row is then a few conflict-free wavefronts.
template <int DL>
__device__ __forceinline__ void st_row(float* p, const float (&v)[DL]) {
    if constexpr (DL == 4)
        *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    else
        *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]);
}
template <int DL>
__device__ __forceinline__ void ld_row(const float* p, float (&v)[DL]) {
    if constexpr (DL == 4) {
        const float4 x = *reinterpret_cast<const float4*>(p);
        v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
    } else {
        const float2 x = *reinterpret_cast<const float2*>(p);
        v[0] = x.x; v[1] = x.y;
    }
}

// Attention units of layer l on this CTA: unit u = (GU query heads from h, split s), u < hq / GU * S.
// With GU = 1 (short contexts) the query heads of one kv head j run as separate units on separate
// CTAs, each reading j's keys, and the first of them appends the new k and v; with GU = hq / hkv
// (long contexts, more key splits) a unit takes every query head of j.  Scratch: the xs area (free
// between the qkv and o phases).
template <int D>
__device__ __forceinline__ void attention_phase(const MKParams& p, Smem& sm, const MKLayer& ly, int l,
                                             const StepCtx& sc, int cw, int lane) {
    constexpr int DL = D / 32, HALF = D / 2;
    using Raw = typename KVRaw<DL>::type;
    const int S = p.att_splits, G = p.hq / p.hkv, GU = p.att_group, units = p.hq / GU * S;
    const int GRID = gridDim.x;
    const int ctid = cw * 32 + lane;
    __half* kp = p.kpool + l * p.kv_layer_stride;
    __half* vp = p.vpool + l * p.kv_layer_stride;
    const float scale = 1.0f / sqrtf(static_cast<float>(D));
    const int pos = sc.pos, nvis = pos + 1;
    const int chunk = ((nvis + S - 1) / S + 15) / 16 * 16;
    const uint32_t tq = mk_tag(p, sc.t, l, P_QKV), ta = mk_tag(p, sc.t, l, P_ATT);
    const unsigned long long* qkvw = p.vec + p.H;
    unsigned long long* attw = p.vec + p.H + (p.hq + 2 * p.hkv) * p.D;
    float* scr = reinterpret_cast<float*>(&sm.xs[0][0]);
    float* qs = scr;                      // [MAXG][D] normalised + rotated queries
    float* ks = scr + MAXG * D;           // [D] new key (fp16-rounded)
    float* vs = scr + (MAXG + 1) * D;     // [D] new value (fp16-rounded)
    constexpr int MS = D + 4;             // a warp's merge row: o[D], max, sum (16-byte aligned rows)
    float* merge = scr + (MAXG + 2) * D;  // [NW][GU][MS]
    bool traced = false;
    // the units u with unit_cta(u) == this CTA: [ceil(me units / GRID), ceil((me + 1) units / GRID))
    const unsigned me = blockIdx.x;
    const int u_begin = static_cast<int>((me * units + GRID - 1) / static_cast<unsigned>(GRID));
    const int u_end = static_cast<int>(((me + 1) * units + GRID - 1) / static_cast<unsigned>(GRID));
    for (int u = u_begin; u < u_end; ++u) {
        // heads h .. h + GU - 1 (all of kv head j's, or one), split s
        const int h = u / S * GU, s = u % S, j = h / G, gs = h % G;
        const int kb = s * chunk, ke = min(nvis, kb + chunk);
        const bool owns_new = pos >= kb && pos < ke;
        // -- loads that do not depend on this step's q/k/v: RoPE row, norm weights, cached keys
        float2 cs[DL];
        float nw[DL];
#pragma unroll
        for (int q = 0; q < DL; ++q) {
            cs[q] = ld_ahead_f2(p.rope_cs + static_cast<size_t>(pos) * HALF + (lane * DL + q) % HALF);
            nw[q] = ld_ahead_f32((cw < GU ? ly.q_norm : ly.k_norm) + lane * DL + q);
        }
        // the page of the new position (the warp that appends k and v)
        const int page_new =
            (cw == GU && owns_new && gs == 0) ? static_cast<int>(ld_ahead_u32(p.page_table + pos / p.page_tokens)) : 0;
        Raw kraw[KPF], vraw[KPF];
        const int key0 = kb + cw;
#pragma unroll
        for (int i = 0; i < KPF; ++i) {
            const int key = key0 + NW * i;
            if (key < ke && key != pos) {
                const int pg = __ldg(p.page_table + key / p.page_tokens);
                const size_t off =
                    ((static_cast<size_t>(pg) * p.hkv + j) * p.page_tokens + key % p.page_tokens) * D + lane * DL;
                if constexpr (DL == 4) {
                    kraw[i] = ld_ahead_u64(kp + off);
                    vraw[i] = ld_ahead_u64(vp + off);
                } else {
                    kraw[i] = ld_ahead_u32(kp + off);
                    vraw[i] = ld_ahead_u32(vp + off);
                }
            }
        }
        // -- this layer's q (and, for the split holding the new position, k and v) rows
        if (cw < GU || (cw == GU && owns_new)) {
            const int hrow = cw < GU ? (h + cw) * D : (p.hq + j) * D;
            float v[DL], vv[DL];
            poll_words<DL, 1>(qkvw + hrow + lane * DL, tq, v, p.err);
            if (cw == GU) poll_words<DL, 1>(qkvw + (p.hq + p.hkv + j) * D + lane * DL, tq, vv, p.err);
            if (!traced) {
                MK_TR(l, 21);
                traced = true;
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
            MK_TR(l, 32);
            if (cw < GU) {
                st_row<DL>(qs + cw * D + lane * DL, o);
            } else {
                // every unit of kv head j rounds the new k and v the same way; the first appends them
                const size_t off =
                    ((static_cast<size_t>(page_new) * p.hkv + j) * p.page_tokens + pos % p.page_tokens) * D +
                    lane * DL;
                float kr[DL], vr[DL];
#pragma unroll
                for (int q = 0; q < DL; ++q) {
                    const __half kh = __float2half_rn(o[q]), vh = __float2half_rn(vv[q]);
                    if (gs == 0) {
                        kp[off + q] = kh;
                        vp[off + q] = vh;
                    }
                    kr[q] = __half2float(kh);
                    vr[q] = __half2float(vh);
                }
                st_row<DL>(ks + lane * DL, kr);
                st_row<DL>(vs + lane * DL, vr);
            }
        }
        nbar();
        MK_TR(l, 23);
        float qr[MAXG][DL], m[MAXG], lsum[MAXG], o[MAXG][DL];
#pragma unroll
        for (int g = 0; g < MAXG; ++g) {
            m[g] = -INFINITY;
            lsum[g] = 0.0f;
#pragma unroll
            for (int q = 0; q < DL; ++q) {
                o[g][q] = 0.0f;
                qr[g][q] = 0.0f;
            }
            if (g < GU) ld_row<DL>(qs + g * D + lane * DL, qr[g]);
        }
        for (int base = key0; base < ke; base += NW * KPF) {
            if (base != key0) {
#pragma unroll
                for (int i = 0; i < KPF; ++i) {
                    const int key = base + NW * i;
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
            // the running softmax is rescaled once per batch.
            constexpr int KB = 4;
#pragma unroll
            for (int i0 = 0; i0 < KPF; i0 += KB) {
                if (base + NW * i0 >= ke) break;
                float kf[KB][DL], vf[KB][DL];
                bool okk[KB];
#pragma unroll
                for (int bb = 0; bb < KB; ++bb) {
                    const int key = base + NW * (i0 + bb);
                    okk[bb] = key < ke;
                    if (!okk[bb]) {
#pragma unroll
                        for (int q = 0; q < DL; ++q) kf[bb][q] = vf[bb][q] = 0.0f;
                    } else if (key == pos) {
                        ld_row<DL>(ks + lane * DL, kf[bb]);
                        ld_row<DL>(vs + lane * DL, vf[bb]);
                    } else {
                        unpack_kv(kraw[i0 + bb], kf[bb]);
                        unpack_kv(vraw[i0 + bb], vf[bb]);
                    }
                }
                if (base == key0 && i0 == 0) MK_TR(l, 33);
#pragma unroll
                for (int g = 0; g < MAXG; ++g) {
                    if (g >= GU) break;
                    float d[KB];
#pragma unroll
                    for (int bb = 0; bb < KB; ++bb) {
                        d[bb] = 0.0f;
#pragma unroll
                        for (int q = 0; q < DL; ++q) d[bb] += qr[g][q] * kf[bb][q];
                    }
#pragma unroll
                    for (int off = 16; off > 0; off >>= 1)
#pragma unroll
                        for (int bb = 0; bb < KB; ++bb) d[bb] += __shfl_xor_sync(0xffffffffu, d[bb], off);
                    float mn = m[g];
#pragma unroll
                    for (int bb = 0; bb < KB; ++bb) {
                        d[bb] = okk[bb] ? d[bb] * scale : -INFINITY;
                        mn = fmaxf(mn, d[bb]);
                    }
                    const float corr = expf(m[g] - mn);
                    float ps = 0.0f, pe[KB];
#pragma unroll
                    for (int bb = 0; bb < KB; ++bb) {
                        pe[bb] = okk[bb] ? expf(d[bb] - mn) : 0.0f;
                        ps += pe[bb];
                    }
                    lsum[g] = lsum[g] * corr + ps;
#pragma unroll
                    for (int q = 0; q < DL; ++q) {
                        float acc = o[g][q] * corr;
#pragma unroll
                        for (int bb = 0; bb < KB; ++bb) acc += pe[bb] * vf[bb][q];
                        o[g][q] = acc;
                    }
                    m[g] = mn;
                }
            }
        }
        // unrolled over MAXG with a guard: a loop bounded by the run-time G would index o / m /
        // lsum dynamically and move them to local memory
#pragma unroll
        for (int g = 0; g < MAXG; ++g) {
            if (g >= GU) break;
            float* mr = merge + (cw * GU + g) * MS;
            st_row<DL>(mr + lane * DL, o[g]);
            if (lane == 0) {
                mr[D] = m[g];
                mr[D + 1] = lsum[g];
            }
        }
        MK_TR(l, 24);
        nbar();
        MK_TR(l, 25);
        // partials [hkv][S][G][D + 2]: this head's at (j, s, gs)
        unsigned long long* part = p.part + ((static_cast<size_t>(j) * S + s) * G + gs) * (D + 2);
        // each warp's weight in the merge, once per (warp, head): f = exp(m_w - M), and the sum L
        float* fw = ks;  // [G][NW] (the new key is no longer needed)
        if (cw < GU) {
            const int g = cw;
            const float mw = lane < NW ? merge[(lane * GU + g) * MS + D] : -INFINITY;
            float M = mw;
#pragma unroll
            for (int o2 = 4; o2 > 0; o2 >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o2));
            const float f = (lane < NW && mw != -INFINITY) ? expf(mw - M) : 0.0f;
            float L = lane < NW ? merge[(lane * GU + g) * MS + D + 1] * f : 0.0f;
#pragma unroll
            for (int o2 = 4; o2 > 0; o2 >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o2);
            if (lane < NW) fw[g * NW + lane] = f;
            if (lane == 0) {
                vs[2 * g] = M;
                vs[2 * g + 1] = L;
            }
        }
        nbar();
        MK_TR(l, 34);
        for (int idx = ctid; idx < GU * D; idx += CT) {
            const int g = idx / D, d = idx % D;
            const float M = vs[2 * g], L = vs[2 * g + 1];
            float acc = 0.0f;
#pragma unroll
            for (int w = 0; w < NW; ++w) acc += merge[(w * GU + g) * MS + d] * fw[g * NW + w];
            if (S == 1) {
                st_word(attw + static_cast<size_t>(h + g) * D + d, L > 0.0f ? acc / L : 0.0f, ta);
            } else {
                st_word(part + g * (D + 2) + d, acc, ta);
                if (d == 0) {
                    st_word(part + g * (D + 2) + D, M, ta);
                    st_word(part + g * (D + 2) + D + 1, L, ta);
                }
            }
        }
        MK_TR(l, 35);
        nbar();
    }
    // split-K: the unit of split 0 of each kv head combines the partials of its splits (after
    // every unit of this CTA has written its own partials, so no unit waits on a later one)
    if (S > 1) {
        const int sstride = G * (D + 2);  // words between the same entry of consecutive splits
        float* mq = scr;                  // [GU][32] split maxima, then [GU][32] split sums
        float* lq = scr + MAXG * 32;
        for (int u = u_begin; u < u_end; ++u) {
            if (u % S != 0) continue;
            const int h = u / S * GU, j = h / G, gs = h % G;
            const unsigned long long* hp = p.part + static_cast<size_t>(j) * S * sstride + gs * (D + 2);
            // (max, sum) of every split and head: one thread per pair, both words in one round
            if (ctid < S * GU) {
                const int q = ctid / GU, g = ctid % GU;
                float ml[2];
                poll_words<2, 1>(hp + q * sstride + g * (D + 2) + D, ta, ml, p.err);
                mq[g * 32 + q] = ml[0];
                lq[g * 32 + q] = ml[1];
            }
            nbar();
            for (int idx = ctid; idx < GU * D; idx += CT) {
                const int g = idx / D, d = idx % D;
                float M = -INFINITY;
                for (int q = 0; q < S; ++q) M = fmaxf(M, mq[g * 32 + q]);
                float L = 0.0f, acc = 0.0f;
                for (int q0 = 0; q0 < S; q0 += 8) {
                    float a8[8];
                    poll_strided<8>(hp + q0 * sstride + g * (D + 2) + d, sstride, min(8, S - q0), ta, a8, p.err);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        if (q0 + i < S) {
                            const float mqv = mq[g * 32 + q0 + i];
                            const float f = (M == -INFINITY || mqv == -INFINITY) ? 0.0f : expf(mqv - M);
                            L += lq[g * 32 + q0 + i] * f;
                            acc += a8[i] * f;
                        }
                    }
                }
                st_word(attw + static_cast<size_t>(h + g) * D + d, L > 0.0f ? acc / L : 0.0f, ta);
            }
            nbar();
        }
    }
}

// ------------------------------------------------------------------ lm_head
// Every warp takes whole tiles (all H columns), so the whole final-normed h is staged once as
// parts, part s in xs[s] (xs_pos order).
template <typename TE, int KSH>
__device__ __forceinline__ void lm_phase(const MKParams& p, Smem& sm, const StepCtx& sc, long long& k, int cw, int lane,
                                      unsigned long long& wbest) {
    constexpr int M = KSH / 32;
    const Mat mt = mat_of(p, sm.layers[0], M_LM);
    int a, b;
    cta_tiles(mt.tiles, blockIdx.x, gridDim.x, 0, M_LM, a, b);
    const int base = cw * KSH;
    float v[M], nv[M];
#pragma unroll
    for (int i = 0; i < M; ++i) nv[i] = ld_ahead_f32(p.final_norm + base + 32 * i + lane);
    poll_slice<M>(p.vec + base, lane, mk_tag(p, sc.t, p.L - 1, P_D), v, p.err);
    float ss = 0.0f, mx = 0.0f;
#pragma unroll
    for (int i = 0; i < M; ++i) {
        ss += v[i] * v[i];
        v[i] *= nv[i];
        mx = fmaxf(mx, fabsf(v[i]));
    }
    ss = warp_sum(ss);
    mx = warp_max_nonneg(mx);
    if (lane == 0) {
        sm.lss[cw] = ss;
        sm.lmax[cw] = mx;
    }
    MK_TR(p.L, 1);
    nbar();
    float tot = 0.0f, gmx = 0.0f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
        tot += sm.lss[w];
        gmx = fmaxf(gmx, sm.lmax[w]);
    }
    const float s_fin = 1.0f / sqrtf(tot / static_cast<float>(p.H) + p.eps);
    const int e = split_exponent(gmx);
    const float sc2 = pow2i(e), unscale = pow2i(-e) * s_fin;
#pragma unroll
    for (int i = 0; i < M; ++i) {
        uint16_t o[NSPLIT];
        Split<TE>::run(v[i] * sc2, o);
        const int r = base + 32 * i + lane;
#pragma unroll
        for (int s2 = 0; s2 < Split<TE>::N; ++s2) sm.xs[s2][xs_pos(r)] = o[s2];
    }
    nbar();
    MK_TR(p.L, 2);
    const AFrag af = afrag_of<TE>(sm, 0, lane);
    const int KT4 = p.H / 64;
    for (int u = a; u < b; ++k) {
        const int n = min(mt.tpc, b - u);
        const int slot = static_cast<int>(k % SLOTS);
        const bool ok = mbar_wait(&sm.full[slot], static_cast<unsigned>((k / SLOTS) & 1), p.err);
        if (ok) {
            for (int i = 0; i < n; ++i) {
                if ((u - a + i) % NW != cw) continue;
                const uint8_t* tile = sm.ring[slot] + static_cast<size_t>(i) * mt.tb + lane * 8;
                float acc[4][4];
#pragma unroll
                for (int c = 0; c < 4; ++c) acc[c][0] = acc[c][1] = acc[c][2] = acc[c][3] = 0.0f;
                for (int k4 = 0; k4 < KT4; ++k4) {
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const int kt = k4 * 4 + c;
                        uint32_t a0, a2;
                        af.at(kt, a0, a2);
                        const uint2 bw = *reinterpret_cast<const uint2*>(tile + kt * 256);
                        mma<TE>(acc[c], a0, a2, bw.x, bw.y);
                    }
                }
                float d0 = acc[0][0] + acc[1][0] + acc[2][0] + acc[3][0];
                float d1 = acc[0][1] + acc[1][1] + acc[2][1] + acc[3][1];
                combine_parts<TE>(d0, d1);
                if (lane < 4) {
                    const int r0 = (u + i) * 8 + 2 * lane;
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int r = r0 + h;
                        const float yy = (h == 0 ? d0 : d1) * unscale;
                        if (r < p.V) {
                            if (p.logits) p.logits[static_cast<size_t>(sc.t) * p.V + r] = yy;
                            const float sv = p.temperature == 1.0f ? yy : __fdiv_rn(yy, p.temperature);
                            if (sv == sv) {
                                const unsigned long long key = argmax_key(sv, r);
                                wbest = key > wbest ? key : wbest;
                            }
                        }
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.empty[slot]);
        u += n;
    }
}

// ------------------------------------------------------------------ the step loop
template <typename TX, typename TE, int F, int KSH, int KSA, int KSI, int D>
__device__ void consumers(const MKParams& p, Smem& sm, int cw, int lane) {
    const int ctid = cw * 32 + lane;
    const int GRID = gridDim.x;
    const int me = blockIdx.x;
    long long k = 0;
    bool stopped = false;
    unsigned long long* hw = p.vec;
    unsigned long long* qkvw = p.vec + p.H;
    unsigned long long* attw = qkvw + (p.hq + 2 * p.hkv) * p.D;
    unsigned long long* actw = attw + p.hq * p.D;
    int rb = 0;
    for (int t = 0; t < p.steps; ++t) {
        StepCtx sc;
        sc.t = t;
        sc.pos = p.start + t;
        if (t == 0) {
            sc.tok = __ldcg(p.ids);
        } else {
            // every CTA reduces the per-CTA argmax keys of the previous step
            if (cw == 0) {
                unsigned long long bk = poll_keys(p.best + static_cast<size_t>(t - 1) * GRID, GRID, lane, p.err);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const unsigned long long other = __shfl_xor_sync(0xffffffffu, bk, o);
                    bk = other > bk ? other : bk;
                }
                // everything written in step t - 1 (by every CTA, KV appends included) is
                // visible from here on: the writers fenced before publishing their keys
                __threadfence();
                if (lane == 0) sm.tok = bk <= 1ull ? 0 : argmax_key_index(bk);
            }
            nbar();
            sc.tok = sm.tok;
            if (me == 0 && ctid == 0) p.ids[t] = sc.tok;
        }
        if (sc.tok == p.eos) {
            // every CTA reads the same id, so all of them (and their producers) stop here
            stopped = true;
            break;
        }
        unsigned long long wbest = 0ull;
        for (int l = 0; l < p.L; ++l) {
            const MKLayer& ly = sm.layers[l];
            MK_TR(l, 0);
            int a, b;
            // ---- qkv: h (or the embedding row) -> q, k, v rows (input RMSNorm folded)
            {
                const Mat mt = mat_of(p, ly, M_QKV);
                cta_tiles(mt.tiles, me, GRID, l, M_QKV, a, b);
                const Input in{l == 0 ? nullptr : hw, l == 0 ? 0u : mk_tag(p, t, l - 1, P_D), ly.in_norm};
                const Output out{qkvw, mk_tag(p, t, l, P_QKV), E_STORE_SCALED, nullptr, 0u};
                if (matrix_phase<TX, TE, F, KSH>(p, sm, mt, a, b, in, out, sc, k, rb, l, 1, cw, lane)) rb ^= 1;
            }
            // ---- attention
            attention_phase<D>(p, sm, ly, l, sc, cw, lane);
            MK_TR(l, 22);
            // ---- o_proj + residual: h = h + W_o attn
            {
                const Mat mt = mat_of(p, ly, M_O);
                cta_tiles(mt.tiles, me, GRID, l, M_O, a, b);
                const Input in{attw, mk_tag(p, t, l, P_ATT), nullptr};
                const Output out{hw, mk_tag(p, t, l, P_O), E_RESIDUAL, l == 0 ? nullptr : hw,
                                 l == 0 ? 0u : mk_tag(p, t, l - 1, P_D)};
                if (matrix_phase<TX, TE, F, KSA>(p, sm, mt, a, b, in, out, sc, k, rb, l, 6, cw, lane)) rb ^= 1;
            }
            // ---- gate/up + SwiGLU (post-attention RMSNorm folded)
            {
                const Mat mt = mat_of(p, ly, M_GU);
                cta_tiles(mt.tiles, me, GRID, l, M_GU, a, b);
                const Input in{hw, mk_tag(p, t, l, P_O), ly.post_norm};
                const Output out{actw, mk_tag(p, t, l, P_GU), E_SWIGLU, nullptr, 0u};
                if (matrix_phase<TX, TE, F, KSH>(p, sm, mt, a, b, in, out, sc, k, rb, l, 11, cw, lane)) rb ^= 1;
            }
            // ---- down + residual: h = h + W_d act
            {
                const Mat mt = mat_of(p, ly, M_D);
                cta_tiles(mt.tiles, me, GRID, l, M_D, a, b);
                const Input in{actw, mk_tag(p, t, l, P_GU), nullptr};
                const Output out{hw, mk_tag(p, t, l, P_D), E_RESIDUAL, hw, mk_tag(p, t, l, P_O)};
                if (matrix_phase<TX, TE, F, KSI>(p, sm, mt, a, b, in, out, sc, k, rb, l, 16, cw, lane)) rb ^= 1;
            }
        }
        // ---- final norm + lm_head + argmax
        lm_phase<TE, KSH>(p, sm, sc, k, cw, lane, wbest);
        // rows were spread over lanes 0..3: the warp's best of them
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, wbest, o);
            wbest = other > wbest ? other : wbest;
        }
        if (lane == 0) sm.best[cw] = wbest;
        nbar();
        if (ctid == 0) {
            unsigned long long bk = 1ull;  // nonzero: "written" even with no rows
            for (int q = 0; q < NW; ++q) bk = sm.best[q] > bk ? sm.best[q] : bk;
            // publish after a fence: this CTA's writes of step t (KV appends included, ordered
            // by the barrier above) happen before any reader's fence after it sees this key
            __threadfence();
            asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p.best + static_cast<size_t>(t) * GRID + me),
                         "l"(bk)
                         : "memory");
        }
        MK_TR(p.L, 4);
        nbar();  // the xs / red scratch of the lm_head is reused by the next step
    }
    if (me == 0 && !stopped && cw == 0) {
        const int t = p.steps - 1;
        unsigned long long bk = poll_keys(p.best + static_cast<size_t>(t) * GRID, GRID, lane, p.err);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, bk, o);
            bk = other > bk ? other : bk;
        }
        if (lane == 0) p.ids[p.steps] = bk <= 1ull ? 0 : argmax_key_index(bk);
    }
}

static_assert(sizeof(Smem) <= 227 * 1024, "shared memory of the persistent kernel");

template <typename TX, typename TE, int F, int KSH, int KSA, int KSI, int D>
__global__ void __launch_bounds__(THREADS, 1) k_decode_mk(MKParams p) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int l = threadIdx.x; l < p.L; l += blockDim.x) sm.layers[l] = p.layers[l];
    if (threadIdx.x == 0) {
        for (int s = 0; s < SLOTS; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], NW);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    __syncthreads();
    if (warp == 0) {
        producer(p, sm, lane);
    } else {
        consumers<TX, TE, F, KSH, KSA, KSI, D>(p, sm, warp - 1, lane);
    }
}

// ---------------------------------------------------------------- weight tiling
template <int F>
__global__ void k_tile(const uint8_t* __restrict__ w, const __half* __restrict__ scales, int rows, int K,
                       uint8_t* __restrict__ dst) {
    const size_t tb = tile_bytes(F, K);
    const int tiles = rows / 8;
    if constexpr (F == WF_F16 || F == WF_BF16) {
        const int KT = K / 16;
        const size_t n = static_cast<size_t>(tiles) * KT * 32;
        for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
             i += static_cast<size_t>(gridDim.x) * blockDim.x) {
            const int lane = static_cast<int>(i % 32), kt = static_cast<int>((i / 32) % KT);
            const int tile = static_cast<int>(i / (32 * static_cast<size_t>(KT)));
            const int r = tile * 8 + (lane >> 2), c = kt * 16 + 2 * (lane & 3);
            const uint16_t* src = reinterpret_cast<const uint16_t*>(w) + static_cast<size_t>(r) * K + c;
            uint16_t* o = reinterpret_cast<uint16_t*>(dst + static_cast<size_t>(tile) * tb + kt * 256 + lane * 8);
            o[0] = src[0];
            o[1] = src[1];
            o[2] = src[8];
            o[3] = src[9];
        }
    } else if constexpr (F == WF_I8G64) {
        const int NG = K / 64;
        const size_t n = static_cast<size_t>(tiles) * NG * 4 * 32;
        for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
             i += static_cast<size_t>(gridDim.x) * blockDim.x) {
            const int lane = static_cast<int>(i % 32), s = static_cast<int>((i / 32) % 4);
            const int gq = static_cast<int>((i / 128) % NG), tile = static_cast<int>(i / (128 * static_cast<size_t>(NG)));
            const int r = tile * 8 + (lane >> 2), c = (gq * 4 + s) * 16 + 2 * (lane & 3);
            const uint8_t* src = w + static_cast<size_t>(r) * K + c;
            uint8_t* o = dst + static_cast<size_t>(tile) * tb + gq * 528 + s * 128 + lane * 4;
            o[0] = src[0] ^ 0x80u;
            o[1] = src[1] ^ 0x80u;
            o[2] = src[8] ^ 0x80u;
            o[3] = src[9] ^ 0x80u;
            if (s == 0 && (lane & 3) == 0) {
                __half* so = reinterpret_cast<__half*>(dst + static_cast<size_t>(tile) * tb + gq * 528 + 512);
                so[lane >> 2] = scales[static_cast<size_t>(r) * NG + gq];
            }
        }
    } else {  // WF_I4G32: source [rows, K / 2], low nibble = even column
        const int NG = K / 32;
        const size_t n = static_cast<size_t>(tiles) * NG * 32;
        for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
             i += static_cast<size_t>(gridDim.x) * blockDim.x) {
            const int lane = static_cast<int>(i % 32), gq = static_cast<int>((i / 32) % NG);
            const int tile = static_cast<int>(i / (32 * static_cast<size_t>(NG)));
            const int r = tile * 8 + (lane >> 2);
            const uint8_t* row = w + static_cast<size_t>(r) * (K / 2);
            auto nib = [&](int c) -> uint32_t {
                const uint8_t by = row[c >> 1];
                return ((c & 1) ? (by >> 4) : (by & 0xFu)) ^ 0x8u;  // biased
            };
            uint8_t* o = dst + static_cast<size_t>(tile) * tb + gq * 144 + lane * 4;
#pragma unroll
            for (int s = 0; s < 2; ++s) {
                const int c = (gq * 2 + s) * 16 + 2 * (lane & 3);
                o[2 * s] = static_cast<uint8_t>(nib(c) | (nib(c + 8) << 4));
                o[2 * s + 1] = static_cast<uint8_t>(nib(c + 1) | (nib(c + 9) << 4));
            }
            if ((lane & 3) == 0) {
                __half* so = reinterpret_cast<__half*>(dst + static_cast<size_t>(tile) * tb + gq * 144 + 128);
                so[lane >> 2] = scales[static_cast<size_t>(r) * NG + gq];
            }
        }
    }
}

// Kernel instance for a shape: slices of H, hq * D and I per warp, and the head size.
template <typename TX, typename TE, int F>
bool pick_kernel(int H, int QW, int I, int D, void (**fn)(MKParams)) {
#define MK_CASE(KH, KA, KI, DD)                                                              \
    if (H == (KH) * NW && QW == (KA) * NW && I == (KI) * NW && D == (DD)) {                  \
        *fn = k_decode_mk<TX, TE, F, KH, KA, KI, DD>;                                        \
        return true;                                                                         \
    }
    MK_CASE(128, 256, 384, 128)  // Qwen3-0.6B: H 1024, 16 x 128 heads, I 3072
    MK_CASE(32, 32, 64, 64)      // the tiny parity shapes: H 256, 4 x 64 heads, I 512
    MK_CASE(32, 64, 64, 128)     // H 256, 4 x 128 heads, I 512
    MK_CASE(32, 32, 128, 64)     // H 256, 4 x 64 heads, I 1024
#undef MK_CASE
    return false;
}

bool kernel_for(int wfmt, int efmt, int H, int QW, int I, int D, void (**fn)(MKParams)) {
    if (wfmt == WF_F16 && efmt == WF_F16) return pick_kernel<__half, __half, WF_F16>(H, QW, I, D, fn);
    if (wfmt == WF_BF16 && efmt == WF_BF16) return pick_kernel<__nv_bfloat16, __nv_bfloat16, WF_BF16>(H, QW, I, D, fn);
    if (wfmt == WF_I8G64 && efmt == WF_F16) return pick_kernel<__half, __half, WF_I8G64>(H, QW, I, D, fn);
    if (wfmt == WF_I4G32 && efmt == WF_F16) return pick_kernel<__half, __half, WF_I4G32>(H, QW, I, D, fn);
    return false;
}

}  // namespace

size_t mk_vec_words(int H, int I, int hq, int hkv, int D) {
    return static_cast<size_t>(H) + static_cast<size_t>(hq + 2 * hkv) * D + static_cast<size_t>(hq) * D + I;
}

size_t mk_part_words(int hq, int hkv, int D, int splits) {
    return static_cast<size_t>(hkv) * splits * (hq / hkv) * (D + 2);
}

int mk_att_plan(int max_ctx, int hq, int hkv, int grid, int* group) {
    // up to UNIT_KEYS keys per unit, at most one unit per CTA, at most 32 splits (the combine's
    // shared arrays).  One query head per unit while that still leaves every unit at most UNIT_KEYS
    // keys (measured 4 % faster per batch-1 step at short contexts: half the work per unit, twice
    // the units); beyond that every query head of a kv head per unit, which allows twice the splits.
    const int need = (max_ctx + UNIT_KEYS - 1) / UNIT_KEYS;
    const bool per_head = need <= grid / hq;
    *group = per_head ? 1 : hq / hkv;
    const int units_per_split = per_head ? hq : hkv;
    return std::max(1, std::min(std::min(need, grid / units_per_split), 32));
}

bool mk_supported(int L, int H, int I, int hq, int hkv, int D, int V, int wfmt, int efmt, int grid) {
    if (L < 1 || L > LMAX) return false;
    void (*fn)(MKParams) = nullptr;
    if (!kernel_for(wfmt, efmt, H, hq * D, I, D, &fn)) return false;
    if (hq % hkv != 0 || hq / hkv > MAXG || hq > grid || grid > 256) return false;
    if (V % 8 != 0 || V < 8) return false;
    // quantised slices must hold whole groups
    const int g = wfmt == WF_I8G64 ? 64 : wfmt == WF_I4G32 ? 32 : 16;
    if ((H / NW) % g || (I / NW) % g || (hq * D / NW) % g) return false;
    // a tile fits a ring slot; a CTA's tiles of one phase fit the reduction buffer
    if (tile_bytes(wfmt, std::max(std::max(H, I), hq * D)) > static_cast<size_t>(SLOT_BYTES)) return false;
    if (tile_bytes(efmt, H) > static_cast<size_t>(SLOT_BYTES)) return false;
    auto per_cta = [&](int rows) { return (rows / 8 + grid - 1) / grid * 8; };
    if (per_cta((hq + 2 * hkv) * D) > MAX_ROWS || per_cta(2 * I) > MAX_ROWS || per_cta(H) > MAX_ROWS) return false;
    if ((H / 16) % 4 != 0) return false;  // the lm_head's column steps run in fours
    // attention scratch fits the xs area
    if (static_cast<size_t>((MAXG + 2) * D + NW * (hq / hkv) * (D + 4)) * 4 > sizeof(uint16_t) * NSPLIT * NW * KS_MAX)
        return false;
    return true;
}

int mk_grid(int device) {
    int sms = 0;
    SOCB_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
    return sms;
}

size_t mk_tiled_bytes(int wfmt, int rows, int K) { return static_cast<size_t>(rows / 8) * tile_bytes(wfmt, K); }

void mk_tile_matrix(int wfmt, const void* w, const void* scales, int rows, int K, void* dst, cudaStream_t st) {
    if (rows % 8 != 0) throw Error(-2, "mk_tile_matrix: rows must be a multiple of 8");
    const int threads = 256, blocks = 1024;
    const uint8_t* src = static_cast<const uint8_t*>(w);
    const __half* sc = static_cast<const __half*>(scales);
    uint8_t* d = static_cast<uint8_t*>(dst);
    switch (wfmt) {
        case WF_F16:
        case WF_BF16: k_tile<WF_F16><<<blocks, threads, 0, st>>>(src, sc, rows, K, d); break;
        case WF_I8G64: k_tile<WF_I8G64><<<blocks, threads, 0, st>>>(src, sc, rows, K, d); break;
        case WF_I4G32: k_tile<WF_I4G32><<<blocks, threads, 0, st>>>(src, sc, rows, K, d); break;
        default: throw Error(-2, "mk_tile_matrix: unknown weight format");
    }
    SOCB_CUDA(cudaGetLastError());
}

void mk_launch(const MKParams& p, int grid, cudaStream_t st) {
    void (*fn)(MKParams) = nullptr;
    if (!kernel_for(p.wfmt, p.efmt, p.H, p.hq * p.D, p.I, p.D, &fn))
        throw Error(-2, "persistent decode kernel: shape not supported");
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
    SOCB_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    SOCB_CUDA(cudaLaunchKernelEx(&cfg, fn, p));
}

}  // namespace socb
