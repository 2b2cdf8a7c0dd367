// Small-batch linear layers on the tensor cores: y[r, o] (mode)= sum_i x'[r, i] * W[o, i] for a
// handful of input rows r, with W in fp16, int8 group-64 or int4 group-32 (fp16 group scales).
// It replaces the per-element fp32 FMAs of the CUDA-core GEMV (k_linear), whose integer formats
// are bound by instruction issue rather than by HBM: here the decode of a weight byte into fp16
// is 1-2 logic/half2 instructions and the multiply-adds run as mma.sync.m16n8k16 (fp32
// accumulation).  The reference computes the same products in fp32 on the CPU
// (Mac/cpu/src/linear.cpp:51-84, Linear::Forward; its int8 matmul Mac/cpu/header/matrix_ops.h:308-350
// over the per-column rule of QuantizeMatMulRhs8, matrix_ops.h:42-73); the group-wise int8 g64 / int4 g32
// layout with fp16 scales is this build's bundle format, which keeps that rule inside each group.
//
// Exactness.  Integer weights are exact in fp16 (|q| <= 127).  An input row is scaled by a power
// of two 2^e chosen from its largest magnitude and split into two fp16 parts hi + lo, which keep
// about 22 significant bits; the parts are two B columns of the same MMA, so the fp32 accumulator
// sees w*hi + w*lo.  Group scales multiply the fp32 result of each group, never a weight.
//
// Tiling.  A warp owns 16 output rows (a tile).  Lane (g = lane/4, t = lane%4) streams 16 bytes of
// rows g and g+8 per chunk: byte offset 64*c + 16*t of the row, so the four lanes of a row read
// 64 contiguous bytes and a chunk of 16 rows is 1 KB in every format (32 fp16, 64 int8 or 128
// int4 elements per row).  The k order inside an MMA is a free permutation: the decoded pairs
// sit in the A registers in whatever order the decode produces them, and the input row is stored
// in shared memory in the same permuted order, so every B fragment is one 16-byte shared load.
//
// Columns.  fp16/int8: column n = 2b + part (b = input row of the CTA's row block, part = hi/lo),
// four input rows per n8 tile; for int8 the four lanes of a row cover one 64-element group, so one
// chunk is one group.  int4: the four lanes of a row hold four different 32-element groups, so
// column n = 2*t' + part takes input values only from lane t' = n/2 (the other B entries are
// zero): D[row][2t' + part] is then lane t''s group alone and gets that group's scale.  One input
// row per tile.
//
// K split.  When the matrix has too few tiles to give every SM several warps, the 8 warps of a
// CTA share fewer tiles and each takes every ks-th chunk; the partial sums meet in shared memory.
#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "kernels.h"

namespace socb {
namespace {

constexpr int LM_WARPS = 8;
constexpr int LM_THREADS = LM_WARPS * 32;
constexpr int LM_ZERO_HALVES = 64;  // zero area read by lanes whose B column is empty

template <int F>
struct MmaFmt;
template <>
struct MmaFmt<WF_F16> {
    static constexpr int KC = 32, GROUP = 0;
    // fp16 weights are their own A pairs: natural k order.
    static __host__ __device__ __forceinline__ int slot(int k) { return k; }
};
template <>
struct MmaFmt<WF_I8G64> {
    static constexpr int KC = 64, GROUP = 64;
    // a word (4 int8) decodes to the pairs (k0, k2), (k1, k3)
    static __host__ __device__ __forceinline__ int slot(int k) {
        return (k & ~3) | ((k & 1) << 1) | ((k >> 1) & 1);
    }
};
template <>
struct MmaFmt<WF_I4G32> {
    static constexpr int KC = 128, GROUP = 32;
    // a word (8 int4) decodes to the pairs (k0, k4), (k1, k5), (k2, k6), (k3, k7)
    static __host__ __device__ __forceinline__ int slot(int k) { return (k & ~7) | ((k & 3) << 1) | ((k >> 2) & 1); }
};

// Column scheme for NB input rows.  PER_T (int4, one input row): column 2t' + part holds lane t''s
// group only.  XPOSE (int4, two or more input rows): the four lanes of a row first swap words so
// that lane t holds word t of each of the chunk's four groups; a group is then two MMA steps over
// all four lanes and the columns are 2b + part as for int8.  RPT = input rows per n8 tile.
template <int F, int NB>
struct Sch {
    static constexpr bool PER_T = F == WF_I4G32 && NB == 1;
    static constexpr bool XPOSE = F == WF_I4G32 && NB > 1;
    static constexpr int RPT = PER_T ? 1 : 4;
    static constexpr int NT = (NB + RPT - 1) / RPT;
};

__device__ __forceinline__ uint4 ld_w16(const uint8_t* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
__device__ __forceinline__ float ld_scale(const __half* p) {
    unsigned short u;
    asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(u) : "l"(p));
    return __half2float(__ushort_as_half(u));
}
__device__ __forceinline__ uint2 ld_scale4(const __half* p) {  // four consecutive fp16 scales (8-byte aligned)
    uint2 r;
    asm volatile("ld.global.nc.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}
__device__ __forceinline__ uint4 lds16(uint32_t addr) {
    uint4 r;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(addr));
    return r;
}
__device__ __forceinline__ uint32_t lop_and_xor(uint32_t v, uint32_t mask, uint32_t flip) {
    return (v & mask) ^ flip;  // one LOP3
}
__device__ __forceinline__ uint32_t h2_add(uint32_t a, uint32_t b) {
    __half2 r = __hadd2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t h2_fma(uint32_t a, uint32_t b, uint32_t c) {
    __half2 r = __hfma2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b),
                        *reinterpret_cast<__half2*>(&c));
    return *reinterpret_cast<uint32_t*>(&r);
}

// D += A * B, m16n8k16, fp16 inputs, fp32 accumulation.  a = {row g k-lo, row g+8 k-lo,
// row g k-hi, row g+8 k-hi}, b = {k-lo, k-hi}.
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// D = A * B (zero accumulator input).
__device__ __forceinline__ void mma16816_z(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                           uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.0f));
}

// fp16 constants as packed pairs
constexpr uint32_t H2_M1152 = 0xE480E480u;  // -1152 = -(1024 + 128)
constexpr uint32_t H2_M1032 = 0xE408E408u;  // -1032 = -(1024 + 8)
constexpr uint32_t H2_1_16 = 0x2C002C00u;   // 1/16
constexpr uint32_t H2_M72 = 0xD480D480u;    // -72 = -(1024/16 + 8)

// Decode one 16-byte weight vector of a row into the A pairs of the chunk's MMA steps:
// p[s][0] = logical k 2t..2t+1 of step s, p[s][1] = logical k 2t+8..2t+9.
template <int F>
struct Decode;
template <>
struct Decode<WF_F16> {
    static constexpr int STEPS = 2;
    // steps 2v and 2v+1 of the chunk (v = 0 only)
    static __device__ __forceinline__ void pair(const uint4& u, int, uint32_t (&p)[2][2]) {
        p[0][0] = u.x; p[0][1] = u.y; p[1][0] = u.z; p[1][1] = u.w;
    }
};
template <>
struct Decode<WF_I8G64> {
    static constexpr int STEPS = 4;
    // (v & 0x00ff00ff) ^ 0x64806480 puts the biased bytes 0 and 2 in the mantissas of 1024:
    // 1024 + (q + 128); adding -1152 leaves q exactly.
    // steps 2v and 2v+1 of the chunk: words 2v and 2v+1
    static __device__ __forceinline__ void pair(const uint4& u, int v, uint32_t (&p)[2][2]) {
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const uint32_t w = u4_word(u, 2 * v + k);
            p[k][0] = h2_add(lop_and_xor(w, 0x00FF00FFu, 0x64806480u), H2_M1152);
            p[k][1] = h2_add(lop_and_xor(w >> 8, 0x00FF00FFu, 0x64806480u), H2_M1152);
        }
    }
};
template <>
struct Decode<WF_I4G32> {
    static constexpr int STEPS = 8;
    // Nibbles 0/4 land in the low mantissa bits of 1024 (+ (q + 8)); nibbles 1/5 in bits 4-7,
    // i.e. 1024 + 16 (q + 8), which one fma by 1/16 and -72 brings back to q.  Shifting the word by
    // 8 does the same for nibbles 2/6 and 3/7.  Every intermediate is exact in fp16.
    static __device__ __forceinline__ void word(uint32_t v, uint32_t (&p)[2][2]) {
        const uint32_t v8 = v >> 8;
        p[0][0] = h2_add(lop_and_xor(v, 0x000F000Fu, 0x64086408u), H2_M1032);
        p[0][1] = h2_fma(lop_and_xor(v, 0x00F000F0u, 0x64806480u), H2_1_16, H2_M72);
        p[1][0] = h2_add(lop_and_xor(v8, 0x000F000Fu, 0x64086408u), H2_M1032);
        p[1][1] = h2_fma(lop_and_xor(v8, 0x00F000F0u, 0x64806480u), H2_1_16, H2_M72);
    }
    // steps 2v and 2v+1 of the chunk: word v
    static __device__ __forceinline__ void pair(const uint4& u, int v, uint32_t (&p)[2][2]) { word(u4_word(u, v), p); }
};

// 4 x 4 word transpose across the four lanes of a row (lanes t = 0..3 of one g): on entry lane t
// holds words 0..3 of its own 16 bytes, on exit word t of lane 0..3's 16 bytes.  Two butterfly
// stages; each sends the two words that the lane gives up and takes the partner's two.
__device__ __forceinline__ void quad_transpose(uint4& u, int t) {
    const bool odd = t & 1, hi = t & 2;
    uint32_t s0 = odd ? u.x : u.y, s1 = odd ? u.z : u.w;
    uint32_t r0 = __shfl_xor_sync(0xffffffffu, s0, 1), r1 = __shfl_xor_sync(0xffffffffu, s1, 1);
    if (odd) {
        u.x = r0;
        u.z = r1;
    } else {
        u.y = r0;
        u.w = r1;
    }
    s0 = hi ? u.x : u.z;
    s1 = hi ? u.y : u.w;
    r0 = __shfl_xor_sync(0xffffffffu, s0, 2);
    r1 = __shfl_xor_sync(0xffffffffu, s1, 2);
    if (hi) {
        u.x = r0;
        u.y = r1;
    } else {
        u.z = r0;
        u.w = r1;
    }
}

// Sum of squares and largest |x * norm_w| of one input row, by one warp (every lane gets both); the loads of
// four iterations are in flight together.
__device__ __forceinline__ void row_stats(const float* __restrict__ xr, const float* __restrict__ norm_w, int in_f,
                                          int lane, float& ss, float& mx) {
    ss = 0.0f;
    mx = 0.0f;
#pragma unroll 4
    for (int i = lane * 4; i < in_f; i += 128) {
        const float4 v = *reinterpret_cast<const float4*>(xr + i);
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        float4 nw = make_float4(1.f, 1.f, 1.f, 1.f);
        if (norm_w != nullptr) nw = *reinterpret_cast<const float4*>(norm_w + i);
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x * nw.x), fabsf(v.y * nw.y)), fmaxf(fabsf(v.z * nw.z), fabsf(v.w * nw.w))));
    }
    ss = warp_sum(ss);
    mx = warp_max(mx);
}

// 2^e for |e| <= 126 (exact)
__device__ __forceinline__ float pow2i_f(int e) { return __int_as_float((e + 127) << 23); }

// Exponent that scales a row whose largest magnitude is mx into [2^14, 2^15).
__device__ __forceinline__ int row_exponent(float mx) {
    if (!(mx > 0.0f) || !(mx < 3.0e38f)) return 0;
    const int ex = static_cast<int>((__float_as_uint(mx) >> 23) & 0xffu) - 127;
    return max(-100, min(100, 14 - ex));
}

}  // namespace

// Weight chunks in flight per warp (8 registers per lane each).  A shared-memory ring filled by
// cp.async (8 slots of 1 KB per warp) measured slower on every shape: lm_head fp16 b=1 73.5 against
// 53.2 us.
#ifndef LM_RING1
#define LM_RING1 4
#endif
template <int F, int NB>
__host__ __device__ constexpr int ring_depth() {
    return Sch<F, NB>::XPOSE ? (Sch<F, NB>::NT >= 4 ? 2 : 3)
           : NB == 1         ? LM_RING1
                             : (Sch<F, NB>::NT == 1 ? 4 : Sch<F, NB>::NT == 2 ? 3 : 2);
}

// Per-warp work stream.  Big matrices (ks == 1): warp gw of the grid takes tiles gw, gw + NW, ...
// (NW = warps of one row block) and streams all chunks of each.  Small ones (ks > 1): warp
// (wt, kp) of a CTA takes chunks kp, kp + ks, ... of its one tile.  The weight chunks run through a
// ring of UNR register slots, each refilled as soon as it is consumed, so a warp always has UNR
// chunk loads in flight; the first UNR loads are issued before the wait on the previous kernel
// (weights are never written by the kernel before this one in the stream).
template <int F, int NB, int DEPTH = ring_depth<F, NB>()>
struct Stream {
    using M = MmaFmt<F>;
    using Z = Sch<F, NB>;
    static constexpr int NT = Z::NT;
    static constexpr int UNR = DEPTH;
    // scale index step per chunk: one int8 group, four int4 groups
    static constexpr int SSTEP = F == WF_I4G32 ? 4 : 1;
    int tile, c;  // next chunk to load
    int tstride, kp, ks, nch, tiles, out_f, ng;
    size_t row_bytes;
    const uint8_t* W;
    const __half* S;
    int g, t;
    // addresses of the next load (rows g and g+8), set per tile and advanced per chunk
    const uint8_t* wp0;
    const uint8_t* wp8;
    const __half* sp0;
    const __half* sp8;
    uint4 a[UNR][2];
    float s0[UNR], s8[UNR];
    uint2 v0[UNR], v8[UNR];  // XPOSE: the chunk's four group scales of rows g and g+8

    // The 16-byte vectors of rows g and g+8 of the chunk in slot u.
    __device__ __forceinline__ void fetch(int u, uint4& a0, uint4& a8) {
        a0 = a[u][0];
        a8 = a[u][1];
    }

    // Addresses of chunk c of the current tile.
    __device__ __forceinline__ void set_tile() {
        const int rg = min(tile * 16 + g, out_f - 1), rg8 = min(tile * 16 + g + 8, out_f - 1);
        const size_t off = static_cast<size_t>(c) * 64 + 16 * t;
        wp0 = W + static_cast<size_t>(rg) * row_bytes + off;
        wp8 = W + static_cast<size_t>(rg8) * row_bytes + off;
        if (M::GROUP) {
            const int gi = SSTEP * c + (Z::PER_T ? t : 0);
            sp0 = S + static_cast<size_t>(rg) * ng + gi;
            sp8 = S + static_cast<size_t>(rg8) * ng + gi;
        }
    }

    // Refill slot u with the next chunk of the stream.
    __device__ __forceinline__ void load(int u) {
        if (tile >= tiles) return;
        a[u][0] = ld_w16(wp0);
        a[u][1] = ld_w16(wp8);
        if (Z::XPOSE) {
            v0[u] = ld_scale4(sp0);
            v8[u] = ld_scale4(sp8);
        } else if (M::GROUP) {
            s0[u] = ld_scale(sp0);
            s8[u] = ld_scale(sp8);
        }
        c += ks;
        if (c < nch) {
            wp0 += 64 * ks;
            wp8 += 64 * ks;
            if (M::GROUP) {
                sp0 += SSTEP * ks;
                sp8 += SSTEP * ks;
            }
        } else {
            c = kp;
            tile += tstride;
            if (tile < tiles) set_tile();
        }
    }
};

// Per-lane results of a tile: rows g and g+8 for input row b(j) of tile j.
template <int F, int NB, int NT>
__device__ __forceinline__ void tile_results(const float (&acc)[NT][4], float (&res)[NT][2]) {
#pragma unroll
    for (int j = 0; j < NT; ++j) {
        res[j][0] = acc[j][0] + acc[j][1];
        res[j][1] = acc[j][2] + acc[j][3];
        if (Sch<F, NB>::PER_T) {  // the four groups of a chunk sit in the four lanes of the row
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                res[j][h] += __shfl_xor_sync(0xffffffffu, res[j][h], 1);
                res[j][h] += __shfl_xor_sync(0xffffffffu, res[j][h], 2);
            }
        }
    }
}

template <int F, int NB, int NT>
__device__ __forceinline__ void tile_store(const float (&res)[NT][2], int o0, int g, int t, int nr, const int* ex_s,
                                           float* __restrict__ y, int ldy, int r0, int out_f, int mode) {
    using Z = Sch<F, NB>;
#pragma unroll
    for (int j = 0; j < NT; ++j) {
        const int b = Z::PER_T ? j : 4 * j + t;
        const bool writer = Z::PER_T ? t == 0 : true;
        const float unscale = b < nr ? pow2i_f(-ex_s[b]) : 0.0f;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int o = o0 + g + 8 * h;
            const float v = res[j][h] * unscale;
            if (mode == LIN_SWIGLU) {
                const float up = __shfl_down_sync(0xffffffffu, v, 4);  // row o + 1 sits in lane + 4
                if (writer && b < nr && (g & 1) == 0 && o + 1 < out_f)
                    y[static_cast<size_t>(r0 + b) * ldy + o / 2] = silu_f(v) * up;
            } else if (writer && b < nr && o < out_f) {
                float* dst = y + static_cast<size_t>(r0 + b) * ldy + o;
                if (mode == LIN_RESIDUAL)
                    *dst += v;
                else
                    *dst = v;
            }
        }
    }
}

// One CTA: 8 warps, NB input rows (row block yb).  Dynamic shared memory: 2*NB part rows of padk
// halves (row 2b + part), LM_ZERO_HALVES zeros, then the k-split partials (8 warps x tiles x 2 x 32
// floats).
template <int F, int NB>
__global__ void __launch_bounds__(LM_THREADS, 2)
    k_linear_mma(const uint8_t* __restrict__ W, const __half* __restrict__ S, int out_f, int in_f,
                 const float* __restrict__ x, int ldx, int rows, const float* __restrict__ norm_w, float eps,
                 float* __restrict__ y, int ldy, int mode, int ks, int ny) {
    using M = MmaFmt<F>;
    using St = Stream<F, NB>;
    constexpr int KC = M::KC, G = M::GROUP, NT = St::NT, UNR = St::UNR;
    constexpr int STEPS = Decode<F>::STEPS;
    extern __shared__ uint4 lm_smem[];
    __shared__ int ex_s[NB];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    // Row blocks that share weight tiles are neighbours in launch order (the second read of the
    // weights hits L2).
    const int yb = blockIdx.x % ny, xb = blockIdx.x / ny;
    const int nxb = gridDim.x / ny;
    const int r0 = yb * NB;
    const int nr = min(NB, rows - r0);
    const int tiles = (out_f + 15) / 16;

    St sr;
    sr.W = W;
    sr.S = S;
    sr.g = g;
    sr.t = t;
    sr.ks = ks;
    sr.nch = in_f / KC;
    sr.tiles = tiles;
    sr.out_f = out_f;
    sr.ng = G ? in_f / G : 0;
    sr.row_bytes = static_cast<size_t>(in_f) * 64 / KC;
    if (ks == 1) {
        sr.tile = xb * LM_WARPS + warp;
        sr.tstride = nxb * LM_WARPS;
        sr.kp = 0;
    } else {
        sr.tile = xb * (LM_WARPS / ks) + warp / ks;
        sr.tstride = tiles;  // one tile
        sr.kp = warp % ks;
    }
    sr.c = sr.kp;
    if (sr.tile < tiles) sr.set_tile();
    int pt = sr.tile, pc = sr.kp;  // next chunk to consume
    const int tstride = sr.tstride;
    const int padk = in_f + 8;  // halves; the 16-byte pad spreads the part rows over the banks
    __half* xs = reinterpret_cast<__half*>(lm_smem);
    __half* zero = xs + static_cast<size_t>(2 * NB) * padk;
    float* part = reinterpret_cast<float*>(zero + LM_ZERO_HALVES);
#pragma unroll
    for (int u = 0; u < UNR; ++u) sr.load(u);

    pdl_enter();
    // ---- stage the input rows: rmsnorm (optional), power-of-two scale, fp16 hi/lo, permuted k.
    // One or two rows: all warps share each row (block-wide sums); from four rows on one warp owns a
    // row (warp sums only, one barrier), measured 5.5 -> 4.2 us (b=4) and 12.6 -> 7.0 us (b=16) on
    // a 2048 x 1024 matrix, while at one row the shared version is faster (3.2 against 4.0 us).
    for (int i = tid; i < LM_ZERO_HALVES / 2; i += LM_THREADS) reinterpret_cast<uint32_t*>(zero)[i] = 0u;
    if constexpr (NB <= 2) {
        __shared__ float red_s[NB][LM_WARPS][2];
        __shared__ float rs_s[NB];
        for (int r = 0; r < nr; ++r) {
            const float* xr = x + static_cast<size_t>(r0 + r) * ldx;
            float ss = 0.0f, mx = 0.0f;
            for (int i = tid * 4; i < in_f; i += LM_THREADS * 4) {
                const float4 v = *reinterpret_cast<const float4*>(xr + i);
                ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
                float4 nw = make_float4(1.f, 1.f, 1.f, 1.f);
                if (norm_w != nullptr) nw = *reinterpret_cast<const float4*>(norm_w + i);
                mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x * nw.x), fabsf(v.y * nw.y)), fmaxf(fabsf(v.z * nw.z), fabsf(v.w * nw.w))));
            }
            ss = warp_sum(ss);
            mx = warp_max(mx);
            if (lane == 0) {
                red_s[r][warp][0] = ss;
                red_s[r][warp][1] = mx;
            }
        }
        __syncthreads();
        if (tid < nr) {
            float ss = 0.0f, mx = 0.0f;
            for (int w = 0; w < LM_WARPS; ++w) {
                ss += red_s[tid][w][0];
                mx = fmaxf(mx, red_s[tid][w][1]);
            }
            const float rs = norm_w != nullptr ? 1.0f / sqrtf(ss / static_cast<float>(in_f) + eps) : 1.0f;
            const int e = row_exponent(mx * rs);
            rs_s[tid] = rs;
            ex_s[tid] = e;
        }
        __syncthreads();
        for (int r = 0; r < nr; ++r) {
            const float* xr = x + static_cast<size_t>(r0 + r) * ldx;
            const float sc = rs_s[r] * pow2i_f(ex_s[r]);
            for (int i = tid * 8; i < in_f; i += LM_THREADS * 8) {
                float v[8];
                *reinterpret_cast<float4*>(v) = *reinterpret_cast<const float4*>(xr + i);
                *reinterpret_cast<float4*>(v + 4) = *reinterpret_cast<const float4*>(xr + i + 4);
                if (norm_w != nullptr) {
                    const float4 a = *reinterpret_cast<const float4*>(norm_w + i);
                    const float4 b = *reinterpret_cast<const float4*>(norm_w + i + 4);
                    v[0] *= a.x; v[1] *= a.y; v[2] *= a.z; v[3] *= a.w;
                    v[4] *= b.x; v[5] *= b.y; v[6] *= b.z; v[7] *= b.w;
                }
                __align__(16) __half hi[8], lo[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float s = v[j] * sc;
                    const __half h = __float2half_rn(s);
                    hi[M::slot(j)] = h;  // slot() permutes within aligned groups of 8 (i is a multiple of 8)
                    lo[M::slot(j)] = __float2half_rn(s - __half2float(h));
                }
                *reinterpret_cast<uint4*>(xs + static_cast<size_t>(2 * r) * padk + i) = *reinterpret_cast<uint4*>(hi);
                *reinterpret_cast<uint4*>(xs + static_cast<size_t>(2 * r + 1) * padk + i) = *reinterpret_cast<uint4*>(lo);
            }
        }
        __syncthreads();
    } else {
        for (int r = warp; r < nr; r += LM_WARPS) {
            const float* xr = x + static_cast<size_t>(r0 + r) * ldx;
            float ss, mx;
            row_stats(xr, norm_w, in_f, lane, ss, mx);
            const float rs = norm_w != nullptr ? 1.0f / sqrtf(ss / static_cast<float>(in_f) + eps) : 1.0f;
            const int ex = row_exponent(mx * rs);
            if (lane == 0) ex_s[r] = ex;
            const float sc = rs * pow2i_f(ex);
#pragma unroll 2
            for (int i = lane * 8; i < in_f; i += 256) {
                float v[8];
                *reinterpret_cast<float4*>(v) = *reinterpret_cast<const float4*>(xr + i);
                *reinterpret_cast<float4*>(v + 4) = *reinterpret_cast<const float4*>(xr + i + 4);
                if (norm_w != nullptr) {
                    const float4 a = *reinterpret_cast<const float4*>(norm_w + i);
                    const float4 b = *reinterpret_cast<const float4*>(norm_w + i + 4);
                    v[0] *= a.x; v[1] *= a.y; v[2] *= a.z; v[3] *= a.w;
                    v[4] *= b.x; v[5] *= b.y; v[6] *= b.z; v[7] *= b.w;
                }
                __align__(16) __half hi[8], lo[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float q = v[j] * sc;
                    const __half h = __float2half_rn(q);
                    hi[M::slot(j)] = h;  // slot() permutes within aligned groups of 8 (i is a multiple of 8)
                    lo[M::slot(j)] = __float2half_rn(q - __half2float(h));
                }
                *reinterpret_cast<uint4*>(xs + static_cast<size_t>(2 * r) * padk + i) = *reinterpret_cast<uint4*>(hi);
                *reinterpret_cast<uint4*>(xs + static_cast<size_t>(2 * r + 1) * padk + i) = *reinterpret_cast<uint4*>(lo);
            }
        }
        __syncthreads();
    }

    // B source of this lane per tile: shared address of chunk 0 and whether the column has data.
    uint32_t bbase[NT];
    bool bval[NT];
    const uint32_t zaddr = static_cast<uint32_t>(__cvta_generic_to_shared(zero));
#pragma unroll
    for (int j = 0; j < NT; ++j) {
        int b, koff;
        if (Sch<F, NB>::PER_T) {
            b = j;
            bval[j] = (g >> 1) == t && b < nr;
            koff = 32 * t;  // lane t's 32-element group inside a chunk
        } else {
            b = 4 * j + (g >> 1);
            bval[j] = b < nr;
            koff = Sch<F, NB>::XPOSE ? 8 * t : (KC / 4) * t;  // XPOSE: word t of each group
        }
        const int row = 2 * min(b, NB - 1) + (g & 1);
        bbase[j] = static_cast<uint32_t>(__cvta_generic_to_shared(xs + static_cast<size_t>(row) * padk + koff));
    }

    float acc[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[j][q] = 0.0f;

    constexpr int BV = STEPS / 2;  // 16-byte B loads per chunk and tile (two steps each)
    const int nch = sr.nch;
    while (pt < tiles) {
#pragma unroll
        for (int u = 0; u < UNR; ++u) {
            if (pt >= tiles) break;
            const int c = pc;
            if constexpr (Sch<F, NB>::XPOSE) {
                uint4 w0, w8;
                sr.fetch(u, w0, w8);
                const uint2 sv0 = sr.v0[u], sv8 = sr.v8[u];
                quad_transpose(w0, t);
                quad_transpose(w8, t);
                sr.load(u);  // refill the slot with the chunk UNR ahead
                const float2 sa = h2_to_f2(sv0.x), sb = h2_to_f2(sv0.y);
                const float2 ta = h2_to_f2(sv8.x), tb = h2_to_f2(sv8.y);
                const float sg[4] = {sa.x, sa.y, sb.x, sb.y}, sg8[4] = {ta.x, ta.y, tb.x, tb.y};
#pragma unroll
                for (int q = 0; q < 4; ++q) {  // group 4c + q: word t of it in every lane
                    uint32_t e0[2][2], e8[2][2];
                    Decode<WF_I4G32>::word(u4_word(w0, q), e0);
                    Decode<WF_I4G32>::word(u4_word(w8, q), e8);
#pragma unroll
                    for (int j = 0; j < NT; ++j) {
                        float d[4];
                        const uint32_t addr =
                            bval[j] ? bbase[j] + static_cast<uint32_t>(c * KC * 2 + 64 * q) : zaddr;
                        const uint4 bb = lds16(addr);
                        mma16816_z(d, e0[0][0], e8[0][0], e0[0][1], e8[0][1], bb.x, bb.y);
                        mma16816(d, e0[1][0], e8[1][0], e0[1][1], e8[1][1], bb.z, bb.w);
                        acc[j][0] = fmaf(sg[q], d[0], acc[j][0]);
                        acc[j][1] = fmaf(sg[q], d[1], acc[j][1]);
                        acc[j][2] = fmaf(sg8[q], d[2], acc[j][2]);
                        acc[j][3] = fmaf(sg8[q], d[3], acc[j][3]);
                    }
                }
            } else {
            uint4 a0, a8;
            sr.fetch(u, a0, a8);
            const float sc0 = G ? sr.s0[u] : 1.0f, sc8 = G ? sr.s8[u] : 1.0f;
            sr.load(u);  // refill the slot with the chunk UNR ahead
            float d[NT][4];
            if (!G) {
#pragma unroll
                for (int j = 0; j < NT; ++j)
#pragma unroll
                    for (int q = 0; q < 4; ++q) d[j][q] = acc[j][q];
            }
            uint32_t addr[NT];
#pragma unroll
            for (int j = 0; j < NT; ++j) addr[j] = bval[j] ? bbase[j] + static_cast<uint32_t>(c * KC * 2) : zaddr;
            // decode two steps at a time right before their MMAs (fewer live registers)
#pragma unroll
            for (int v = 0; v < BV; ++v) {
                uint32_t q0[2][2], q8[2][2];
                Decode<F>::pair(a0, v, q0);
                Decode<F>::pair(a8, v, q8);
#pragma unroll
                for (int j = 0; j < NT; ++j) {
                    const uint4 bb = lds16(addr[j] + 16 * v);
                    if (G && v == 0)  // a group starts here: zero accumulator input
                        mma16816_z(d[j], q0[0][0], q8[0][0], q0[0][1], q8[0][1], bb.x, bb.y);
                    else
                        mma16816(d[j], q0[0][0], q8[0][0], q0[0][1], q8[0][1], bb.x, bb.y);
                    mma16816(d[j], q0[1][0], q8[1][0], q0[1][1], q8[1][1], bb.z, bb.w);
                }
            }
#pragma unroll
            for (int j = 0; j < NT; ++j) {
                if (G) {
                    acc[j][0] = fmaf(sc0, d[j][0], acc[j][0]);
                    acc[j][1] = fmaf(sc0, d[j][1], acc[j][1]);
                    acc[j][2] = fmaf(sc8, d[j][2], acc[j][2]);
                    acc[j][3] = fmaf(sc8, d[j][3], acc[j][3]);
                } else {
#pragma unroll
                    for (int q = 0; q < 4; ++q) acc[j][q] = d[j][q];
                }
            }
            }
            pc += ks;
            if (pc >= nch) {
                if (ks == 1) {  // whole tile done: store it and start the next
                    float res[NT][2];
                    tile_results<F, NB, NT>(acc, res);
                    tile_store<F, NB, NT>(res, pt * 16, g, t, nr, ex_s, y, ldy, r0, out_f, mode);
#pragma unroll
                    for (int j = 0; j < NT; ++j)
#pragma unroll
                        for (int q = 0; q < 4; ++q) acc[j][q] = 0.0f;
                }
                pc = sr.kp;
                pt += tstride;
            }
        }
    }
    if (ks == 1) return;

    // ---- k split: the ks warps of a tile add their partial sums
    float res[NT][2];
    tile_results<F, NB, NT>(acc, res);
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int h = 0; h < 2; ++h) part[((warp * NT + j) * 2 + h) * 32 + lane] = res[j][h];
    __syncthreads();
    const int my_tile = xb * (LM_WARPS / ks) + warp / ks;
    if (warp % ks != 0 || my_tile >= tiles) return;
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            float s = 0.0f;
            for (int k = 0; k < ks; ++k) s += part[(((warp + k) * NT + j) * 2 + h) * 32 + lane];
            res[j][h] = s;
        }
    tile_store<F, NB, NT>(res, my_tile * 16, g, t, nr, ex_s, y, ldy, r0, out_f, mode);
}

// ------------------------------------------------------------ int8 weights on the integer MMA
// int8 g64 weights enter mma.sync.m16n8k32.s8.s8 as they are (no decode).  An input row is scaled
// by 2^e so that its largest magnitude lies in [2^21, 2^22), rounded to an integer and split into
// three balanced base-256 limbs (each in [-128, 127]); limb l of input row 2j + bl is B column
// 3 bl + l of tile j (two input rows per n8 tile, columns 6 and 7 empty).  The int32 products are
// exact; a chunk is one 64-element group, whose int32 result times the group scale is accumulated
// in fp32 per column, and the limbs are recombined (x 2^(8 l)) when the tile is stored.  Lane
// (g, t) holds k 16t..16t+15 of the chunk for rows g and g+8: words 0/1 are the two k quarters of
// MMA step 0 and words 2/3 those of step 1, the natural k order, so the limbs are staged as they are.
__device__ __forceinline__ void imma16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void imma16832_z(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                            uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// Exponent that scales a row whose largest magnitude is mx into [2^21, 2^22).
__device__ __forceinline__ int row_exponent_i(float mx) {
    if (!(mx > 0.0f) || !(mx < 3.0e38f)) return 0;
    const int ex = static_cast<int>((__float_as_uint(mx) >> 23) & 0xffu) - 127;
    return max(-100, min(100, 21 - ex));
}

// Lane (g, t): columns 2t and 2t+1 of rows g and g+8.  Weighted by 2^(8 l) and summed per input row
// (columns 0-2 row 0, 3-5 row 1) over the four lanes of the row, then stored like tile_store.
template <int NB, int NT>
__device__ __forceinline__ void imma_tile_store(const float (&acc)[NT][4], int o0, int g, int t, int nr,
                                                const int* ex_s, float* __restrict__ y, int ldy, int r0, int out_f,
                                                int mode) {
#pragma unroll
    for (int j = 0; j < NT; ++j) {
        float p[2][2] = {{0.0f, 0.0f}, {0.0f, 0.0f}};  // [input row of the tile][h]
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int col = 2 * t + k;
            const float w = col % 3 == 0 ? 1.0f : col % 3 == 1 ? 256.0f : 65536.0f;
            if (col < 3) {
                p[0][0] = fmaf(w, acc[j][k], p[0][0]);
                p[0][1] = fmaf(w, acc[j][2 + k], p[0][1]);
            } else if (col < 6) {
                p[1][0] = fmaf(w, acc[j][k], p[1][0]);
                p[1][1] = fmaf(w, acc[j][2 + k], p[1][1]);
            }
        }
#pragma unroll
        for (int bl = 0; bl < 2; ++bl)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                p[bl][h] += __shfl_xor_sync(0xffffffffu, p[bl][h], 1);
                p[bl][h] += __shfl_xor_sync(0xffffffffu, p[bl][h], 2);
            }
#pragma unroll
        for (int bl = 0; bl < 2; ++bl) {
            const int b = 2 * j + bl;
            const bool writer = t == bl;
            const float unscale = b < nr ? pow2i_f(-ex_s[b]) : 0.0f;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int o = o0 + g + 8 * h;
                const float v = p[bl][h] * unscale;
                if (mode == LIN_SWIGLU) {
                    const float up = __shfl_down_sync(0xffffffffu, v, 4);  // row o + 1 sits in lane + 4
                    if (writer && b < nr && (g & 1) == 0 && o + 1 < out_f)
                        y[static_cast<size_t>(r0 + b) * ldy + o / 2] = silu_f(v) * up;
                } else if (writer && b < nr && o < out_f) {
                    float* dst = y + static_cast<size_t>(r0 + b) * ldy + o;
                    if (mode == LIN_RESIDUAL)
                        *dst += v;
                    else
                        *dst = v;
                }
            }
        }
    }
}

// int8 g64, NB input rows (1, 2, 4 or 8).  Dynamic shared memory: 3*NB limb rows of padk bytes (row
// 3b + l), 64 zero bytes, then the k-split partials (8 warps x tiles x 4 x 32 floats).
template <int NB>
__global__ void __launch_bounds__(LM_THREADS, 2)
    k_linear_imma(const uint8_t* __restrict__ W, const __half* __restrict__ S, int out_f, int in_f,
                  const float* __restrict__ x, int ldx, int rows, const float* __restrict__ norm_w, float eps,
                  float* __restrict__ y, int ldy, int mode, int ks, int ny) {
    using St = Stream<WF_I8G64, NB, NB <= 2 ? 4 : NB == 4 ? 3 : 2>;
    constexpr int KC = 64, G = 64, NT = (NB + 1) / 2, UNR = St::UNR;
    extern __shared__ uint4 lm_smem[];
    __shared__ float red_s[NB][LM_WARPS][2];
    __shared__ float rs_s[NB];
    __shared__ int ex_s[NB];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int yb = blockIdx.x % ny, xb = blockIdx.x / ny;
    const int nxb = gridDim.x / ny;
    const int r0 = yb * NB;
    const int nr = min(NB, rows - r0);
    const int tiles = (out_f + 15) / 16;

    St sr;
    sr.W = W;
    sr.S = S;
    sr.g = g;
    sr.t = t;
    sr.ks = ks;
    sr.nch = in_f / KC;
    sr.tiles = tiles;
    sr.out_f = out_f;
    sr.ng = in_f / G;
    sr.row_bytes = static_cast<size_t>(in_f);
    if (ks == 1) {
        sr.tile = xb * LM_WARPS + warp;
        sr.tstride = nxb * LM_WARPS;
        sr.kp = 0;
    } else {
        sr.tile = xb * (LM_WARPS / ks) + warp / ks;
        sr.tstride = tiles;  // one tile
        sr.kp = warp % ks;
    }
    sr.c = sr.kp;
    if (sr.tile < tiles) sr.set_tile();
    int pt = sr.tile, pc = sr.kp;  // next chunk to consume
    const int tstride = sr.tstride;
#pragma unroll
    for (int u = 0; u < UNR; ++u) sr.load(u);

    pdl_enter();
    const int padk = in_f % 128 == 0 ? in_f + 64 : in_f;  // bytes; limb rows alternate 64-byte bank halves
    int8_t* xs = reinterpret_cast<int8_t*>(lm_smem);
    int8_t* zero = xs + static_cast<size_t>(3 * NB) * padk;
    float* part = reinterpret_cast<float*>(zero + 64);
    if (tid < 16) reinterpret_cast<uint32_t*>(zero)[tid] = 0u;
    for (int r = 0; r < nr; ++r) {
        const float* xr = x + static_cast<size_t>(r0 + r) * ldx;
        float ss = 0.0f, mx = 0.0f;
        for (int i = tid * 4; i < in_f; i += LM_THREADS * 4) {
            const float4 v = *reinterpret_cast<const float4*>(xr + i);
            ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
            float4 nw = make_float4(1.f, 1.f, 1.f, 1.f);
            if (norm_w != nullptr) nw = *reinterpret_cast<const float4*>(norm_w + i);
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x * nw.x), fabsf(v.y * nw.y)), fmaxf(fabsf(v.z * nw.z), fabsf(v.w * nw.w))));
        }
        ss = warp_sum(ss);
        mx = warp_max(mx);
        if (lane == 0) {
            red_s[r][warp][0] = ss;
            red_s[r][warp][1] = mx;
        }
    }
    __syncthreads();
    if (tid < nr) {
        float ss = 0.0f, mx = 0.0f;
        for (int w = 0; w < LM_WARPS; ++w) {
            ss += red_s[tid][w][0];
            mx = fmaxf(mx, red_s[tid][w][1]);
        }
        const float rs = norm_w != nullptr ? 1.0f / sqrtf(ss / static_cast<float>(in_f) + eps) : 1.0f;
        rs_s[tid] = rs;
        ex_s[tid] = row_exponent_i(mx * rs);
    }
    __syncthreads();
    for (int r = 0; r < nr; ++r) {
        const float* xr = x + static_cast<size_t>(r0 + r) * ldx;
        const float sc = rs_s[r] * pow2i_f(ex_s[r]);
        for (int i = tid * 4; i < in_f; i += LM_THREADS * 4) {
            float4 v = *reinterpret_cast<const float4*>(xr + i);
            if (norm_w != nullptr) {
                const float4 nw = *reinterpret_cast<const float4*>(norm_w + i);
                v.x *= nw.x; v.y *= nw.y; v.z *= nw.z; v.w *= nw.w;
            }
            const float e4[4] = {v.x, v.y, v.z, v.w};
            uint32_t lw[3] = {0u, 0u, 0u};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int xi = __float2int_rn(e4[k] * sc);
                const int l0 = ((xi + 128) & 255) - 128;
                const int rr = (xi - l0) >> 8;
                const int l1 = ((rr + 128) & 255) - 128;
                const int l2 = (rr - l1) >> 8;
                lw[0] |= (static_cast<uint32_t>(l0) & 255u) << (8 * k);
                lw[1] |= (static_cast<uint32_t>(l1) & 255u) << (8 * k);
                lw[2] |= (static_cast<uint32_t>(l2) & 255u) << (8 * k);
            }
#pragma unroll
            for (int l = 0; l < 3; ++l) *reinterpret_cast<uint32_t*>(xs + static_cast<size_t>(3 * r + l) * padk + i) = lw[l];
        }
    }
    __syncthreads();

    // B source of this lane per tile: column g = limb g % 3 of input row 2j + g / 3 (g < 6)
    uint32_t bbase[NT];
    bool bval[NT];
    const uint32_t zaddr = static_cast<uint32_t>(__cvta_generic_to_shared(zero));
#pragma unroll
    for (int j = 0; j < NT; ++j) {
        const int b = 2 * j + g / 3, l = g % 3;
        bval[j] = g < 6 && b < nr;
        const int row = 3 * min(b, NB - 1) + l;
        bbase[j] = static_cast<uint32_t>(__cvta_generic_to_shared(xs + static_cast<size_t>(row) * padk + 16 * t));
    }

    float acc[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[j][q] = 0.0f;

    const int nch = sr.nch;
    while (pt < tiles) {
#pragma unroll
        for (int u = 0; u < UNR; ++u) {
            if (pt >= tiles) break;
            const int c = pc;
            uint4 a0, a8;
            sr.fetch(u, a0, a8);
            const float sc0 = sr.s0[u], sc8 = sr.s8[u];
            sr.load(u);  // refill the slot with the chunk UNR ahead
#pragma unroll
            for (int j = 0; j < NT; ++j) {
                const uint32_t addr = bval[j] ? bbase[j] + static_cast<uint32_t>(c * KC) : zaddr;
                const uint4 bb = lds16(addr);
                int d[4];
                imma16832_z(d, a0.x, a8.x, a0.y, a8.y, bb.x, bb.y);
                imma16832(d, a0.z, a8.z, a0.w, a8.w, bb.z, bb.w);
                acc[j][0] = fmaf(sc0, static_cast<float>(d[0]), acc[j][0]);
                acc[j][1] = fmaf(sc0, static_cast<float>(d[1]), acc[j][1]);
                acc[j][2] = fmaf(sc8, static_cast<float>(d[2]), acc[j][2]);
                acc[j][3] = fmaf(sc8, static_cast<float>(d[3]), acc[j][3]);
            }
            pc += ks;
            if (pc >= nch) {
                if (ks == 1) {  // whole tile done: store it and start the next
                    imma_tile_store<NB, NT>(acc, pt * 16, g, t, nr, ex_s, y, ldy, r0, out_f, mode);
#pragma unroll
                    for (int j = 0; j < NT; ++j)
#pragma unroll
                        for (int q = 0; q < 4; ++q) acc[j][q] = 0.0f;
                }
                pc = sr.kp;
                pt += tstride;
            }
        }
    }
    if (ks == 1) return;

    // ---- k split: the ks warps of a tile add their partial sums
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int q = 0; q < 4; ++q) part[((warp * NT + j) * 4 + q) * 32 + lane] = acc[j][q];
    __syncthreads();
    const int my_tile = xb * (LM_WARPS / ks) + warp / ks;
    if (warp % ks != 0 || my_tile >= tiles) return;
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            float s = 0.0f;
            for (int k = 0; k < ks; ++k) s += part[(((warp + k) * NT + j) * 4 + q) * 32 + lane];
            acc[j][q] = s;
        }
    imma_tile_store<NB, NT>(acc, my_tile * 16, g, t, nr, ex_s, y, ldy, r0, out_f, mode);
}

namespace {

constexpr size_t LM_SMEM_CAP = 110 * 1024;  // two CTAs per SM
constexpr int LM_TARGET_WARPS = 148 * 16;   // two 8-warp CTAs on every SM

template <int F>
constexpr int max_nb() {
    return 16;
}

size_t lm_smem_bytes(int nb, int nt, int in_f) {
    return static_cast<size_t>(2 * nb) * (in_f + 8) * 2 + LM_ZERO_HALVES * 2 +
           static_cast<size_t>(LM_WARPS) * nt * 2 * 32 * 4;
}

bool linear_mma_enabled() {
    static const bool on = [] {
        const char* e = std::getenv("SOC_B200_LINEAR_MMA");
        return !(e && e[0] == '0');
    }();
    return on;
}

template <int F, int NB>
void linear_mma_nb(const void* W, const void* S, int out_f, int in_f, const float* x, int ldx, int rows,
                   const float* norm_w, float eps, float* y, int ldy, int mode, cudaStream_t st) {
    constexpr int NT = Sch<F, NB>::NT;
    const size_t smem = lm_smem_bytes(NB, NT, in_f);
    static bool attr_set = false;  // one attribute set per template instance
    if (!attr_set) {
        SOCB_CUDA(cudaFuncSetAttribute(k_linear_mma<F, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       200 * 1024));
        attr_set = true;
    }
    const int tiles = (out_f + 15) / 16;
    const int ny = (rows + NB - 1) / NB;
    const int nch = in_f / MmaFmt<F>::KC;
    int ks = 1;
    while (ks < LM_WARPS && 2 * ks <= nch && static_cast<long long>(tiles) * ny * ks < LM_TARGET_WARPS) ks *= 2;
    const int tpc = LM_WARPS / ks;
    int nx = (tiles + tpc - 1) / tpc;
    // ks == 1: persistent warps, at most two CTAs per SM over all row blocks
    if (ks == 1) nx = std::max(1, std::min(nx, LM_TARGET_WARPS / LM_WARPS / ny));
    launch_pdl(k_linear_mma<F, NB>, dim3(nx * ny), dim3(LM_THREADS), smem, st, static_cast<const uint8_t*>(W),
               static_cast<const __half*>(S), out_f, in_f, x, ldx, rows, norm_w, eps, y, ldy, mode, ks, ny);
    SOCB_CUDA(cudaGetLastError());
    count_launches(1);
}

template <int F>
bool linear_mma_f(const void* W, const void* S, int out_f, int in_f, const float* x, int ldx, int rows,
                  const float* norm_w, float eps, float* y, int ldy, int mode, cudaStream_t st) {
    if (in_f % MmaFmt<F>::KC != 0) return false;
    if (MmaFmt<F>::GROUP && S == nullptr) return false;
    if (mode == LIN_SWIGLU && out_f % 2 != 0) return false;
    // Smallest row block that holds all rows, else the largest whose staging fits the budget.
    // Matrices under 32 M weights take at most 4 rows per row block (four blocks at 16 rows: a quarter
    // of the staging per CTA, four times the CTAs): the config-0 16-token prefill measured 1.85 ms with
    // 16-row blocks, 1.79 with 8-row and 1.77 with 4-row ones (2048 x 1024 at 16 rows: 7.0 -> 5.2 us at
    // 8-row blocks).
    const bool big = static_cast<long long>(out_f) * in_f >= (32ll << 20);
    int nb = 1;
    while (nb < rows && nb < max_nb<F>() && (nb < 4 || big)) nb *= 2;
    auto fits = [&](int b) {
        const int nt = (F == WF_I4G32 && b == 1) ? 1 : (b + 3) / 4;
        return lm_smem_bytes(b, nt, in_f) <= LM_SMEM_CAP;
    };
    while (nb > 1 && !fits(nb)) nb /= 2;
    if (!fits(nb)) return false;
    switch (nb) {
        case 1: linear_mma_nb<F, 1>(W, S, out_f, in_f, x, ldx, rows, norm_w, eps, y, ldy, mode, st); break;
        case 2: linear_mma_nb<F, 2>(W, S, out_f, in_f, x, ldx, rows, norm_w, eps, y, ldy, mode, st); break;
        case 4: linear_mma_nb<F, 4>(W, S, out_f, in_f, x, ldx, rows, norm_w, eps, y, ldy, mode, st); break;
        case 8:
            if constexpr (max_nb<F>() >= 8)
                linear_mma_nb<F, 8>(W, S, out_f, in_f, x, ldx, rows, norm_w, eps, y, ldy, mode, st);
            break;
        default:
            if constexpr (max_nb<F>() >= 16)
                linear_mma_nb<F, 16>(W, S, out_f, in_f, x, ldx, rows, norm_w, eps, y, ldy, mode, st);
            break;
    }
    return true;
}

size_t imma_smem_bytes(int nb, int in_f) {
    const size_t padk = in_f % 128 == 0 ? in_f + 64 : in_f;
    return static_cast<size_t>(3 * nb) * padk + 64 + static_cast<size_t>(LM_WARPS) * ((nb + 1) / 2) * 4 * 32 * 4;
}

bool linear_imma_enabled() {
    static const bool on = [] {
        const char* e = std::getenv("SOC_B200_LINEAR_IMMA");
        return !(e && e[0] == '0');
    }();
    return on;
}

template <int NB>
void linear_imma_nb(const void* W, const void* S, int out_f, int in_f, const float* x, int ldx, int rows,
                    const float* norm_w, float eps, float* y, int ldy, int mode, cudaStream_t st) {
    const size_t smem = imma_smem_bytes(NB, in_f);
    static bool attr_set = false;  // one attribute set per template instance
    if (!attr_set) {
        SOCB_CUDA(cudaFuncSetAttribute(k_linear_imma<NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        attr_set = true;
    }
    const int tiles = (out_f + 15) / 16;
    const int ny = (rows + NB - 1) / NB;
    const int nch = in_f / 64;
    int ks = 1;
    while (ks < LM_WARPS && 2 * ks <= nch && static_cast<long long>(tiles) * ny * ks < LM_TARGET_WARPS) ks *= 2;
    const int tpc = LM_WARPS / ks;
    int nx = (tiles + tpc - 1) / tpc;
    if (ks == 1) nx = std::max(1, std::min(nx, LM_TARGET_WARPS / LM_WARPS / ny));
    launch_pdl(k_linear_imma<NB>, dim3(nx * ny), dim3(LM_THREADS), smem, st, static_cast<const uint8_t*>(W),
               static_cast<const __half*>(S), out_f, in_f, x, ldx, rows, norm_w, eps, y, ldy, mode, ks, ny);
    SOCB_CUDA(cudaGetLastError());
    count_launches(1);
}

// int8 g64 on the integer MMA for one or two input rows (measured: lm_head b=1 29.2 against 31.8 us on
// the fp16 MMA; at 4 rows it loses, 36.7 against 33.9 us); false when the shape is outside it.
constexpr int IMMA_MAX_ROWS = 2;
bool linear_imma(const void* W, const void* S, int out_f, int in_f, const float* x, int ldx, int rows,
                 const float* norm_w, float eps, float* y, int ldy, int mode, cudaStream_t st) {
    if (!linear_imma_enabled() || rows > IMMA_MAX_ROWS || in_f % 64 != 0 || S == nullptr) return false;
    if (mode == LIN_SWIGLU && out_f % 2 != 0) return false;
    int nb = 1;
    while (nb < rows) nb *= 2;
    while (nb > 1 && imma_smem_bytes(nb, in_f) > LM_SMEM_CAP) nb /= 2;
    if (imma_smem_bytes(nb, in_f) > LM_SMEM_CAP) return false;
    switch (nb) {
        case 1: linear_imma_nb<1>(W, S, out_f, in_f, x, ldx, rows, norm_w, eps, y, ldy, mode, st); break;
        case 2: linear_imma_nb<2>(W, S, out_f, in_f, x, ldx, rows, norm_w, eps, y, ldy, mode, st); break;
        case 4: linear_imma_nb<4>(W, S, out_f, in_f, x, ldx, rows, norm_w, eps, y, ldy, mode, st); break;
        default: linear_imma_nb<8>(W, S, out_f, in_f, x, ldx, rows, norm_w, eps, y, ldy, mode, st); break;
    }
    return true;
}

}  // namespace

bool launch_linear_mma(int wfmt, const void* W, const void* scales, int out_f, int in_f, const float* x, int ldx,
                       int rows, const float* norm_w, float eps, float* y, int ldy, int mode, cudaStream_t st) {
    if (!linear_mma_enabled() || rows <= 0 || out_f <= 0 || ldx % 4 != 0) return false;
    switch (wfmt) {
        case WF_F16: return linear_mma_f<WF_F16>(W, scales, out_f, in_f, x, ldx, rows, norm_w, eps, y, ldy, mode, st);
        case WF_I8G64:
            if (linear_imma(W, scales, out_f, in_f, x, ldx, rows, norm_w, eps, y, ldy, mode, st)) return true;
            return linear_mma_f<WF_I8G64>(W, scales, out_f, in_f, x, ldx, rows, norm_w, eps, y, ldy, mode, st);
        case WF_I4G32:
            return linear_mma_f<WF_I4G32>(W, scales, out_f, in_f, x, ldx, rows, norm_w, eps, y, ldy, mode, st);
        default: return false;
    }
}

}  // namespace socb
