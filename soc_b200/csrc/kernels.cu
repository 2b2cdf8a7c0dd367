// Modular sm_100a kernels of the Qwen3 forward (prefill and batched decode).
//
// Reference arithmetic they restate (SongWooYoung/SoC, Mac/cpu/src):
//   embedding gather      embedding.cpp:51-77
//   RMSNorm               rms_norm_module.cpp:52-66   (x * (1/sqrt(mean(x^2)+eps)) * w)
//   Linear                linear.cpp:69-81            (fp32 accumulate of fp32 x times decoded weight)
//   q/k norm + RoPE       qwen_attention.cpp:168-171, rope.cpp:54-89 (rotate-half, double angle)
//   KV write              qwen_attention.cpp:180-193  (post-RoPE K, raw V)
//   GQA attention         grouped_query_attention.cpp:59-142 (scale 1/sqrt(D), causal, kv = h / group)
//   SwiGLU                qwen_mlp.cpp:20-74          (g / (1 + exp(-g)) * up)
//   greedy sampler        sampler.cpp:26-62           (first strict maximum)
// The B200 layout differs from the reference: the KV cache is paged fp16, q/k/v are one
// fused matrix, gate/up rows are interleaved so one warp owns a (gate, up) pair.
#include <atomic>
#include <cstdlib>
#include <string>

#include "kernels.h"

namespace socb {

static std::atomic<long long> g_launches{0};
void count_launches(long long n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
long long launches_so_far() { return g_launches.load(std::memory_order_relaxed); }

bool pdl_enabled() {
    static const bool on = [] {
        const char* e = std::getenv("SOC_B200_PDL");
        return !(e && std::string(e) == "0");
    }();
    return on;
}

// ------------------------------------------------------------------------ helpers
__device__ __forceinline__ uint4 ld_nc16(const void* p) {
    uint4 r;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
        : "l"(p));
    return r;
}

template <typename T>
__device__ __forceinline__ void unpack8(const uint4& u, float (&w)[8]) {
    float2 a = WTraits<T>::pair(u.x), b = WTraits<T>::pair(u.y), c = WTraits<T>::pair(u.z),
           d = WTraits<T>::pair(u.w);
    w[0] = a.x; w[1] = a.y; w[2] = b.x; w[3] = b.y;
    w[4] = c.x; w[5] = c.y; w[6] = d.x; w[7] = d.y;
}

// --------------------------------------------------------------------- embedding
template <typename T>
__global__ void k_embed(const T* __restrict__ table, int H, int V, const int* __restrict__ tokens,
                        float* __restrict__ h, int* err) {
    pdl_enter();
    const int row = blockIdx.x;
    const int tok = tokens[row];
    float* out = h + static_cast<size_t>(row) * H;
    if (tok < 0 || tok >= V) {
        if (threadIdx.x == 0) atomicOr(err, DERR_TOKEN_RANGE);
        for (int i = threadIdx.x; i < H; i += blockDim.x) out[i] = 0.0f;
        return;
    }
    const T* src = table + static_cast<size_t>(tok) * H;
    for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8) {
        float w[8];
        unpack8<T>(*reinterpret_cast<const uint4*>(src + i), w);
#pragma unroll
        for (int j = 0; j < 8; ++j) out[i + j] = w[j];
    }
}

void launch_embed(int wfmt, const void* table, int hidden, int vocab, const int* tokens, int rows, float* h,
                  int* err, cudaStream_t st) {
    if (rows <= 0) return;
    if (wfmt == WF_BF16)
        launch_pdl(k_embed<__nv_bfloat16>, dim3(rows), dim3(128), 0, st, static_cast<const __nv_bfloat16*>(table),
                   hidden, vocab, tokens, h, err);
    else
        launch_pdl(k_embed<__half>, dim3(rows), dim3(128), 0, st, static_cast<const __half*>(table), hidden, vocab,
                   tokens, h, err);
    SOCB_CUDA(cudaGetLastError());
    count_launches(1);
}

// ----------------------------------------------------------------------- RMSNorm
__global__ void k_rmsnorm(const float* __restrict__ x, int n, const float* __restrict__ w, float eps,
                          float* __restrict__ y) {
    pdl_enter();
    __shared__ float red[32];
    const float* xr = x + static_cast<size_t>(blockIdx.x) * n;
    float* yr = y + static_cast<size_t>(blockIdx.x) * n;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss += xr[i] * xr[i];
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
        v = warp_sum(v);
        if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    const float s = 1.0f / sqrtf(red[0] / static_cast<float>(n) + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) yr[i] = xr[i] * s * w[i];
}

void launch_rmsnorm(const float* x, int rows, int n, const float* w, float eps, float* y, cudaStream_t st) {
    if (rows <= 0) return;
    launch_pdl(k_rmsnorm, dim3(rows), dim3(256), 0, st, x, n, w, eps, y);
    SOCB_CUDA(cudaGetLastError());
    count_launches(1);
}

// ------------------------------------------------------------------------ linear
// One CTA = 8 warps x NWR output rows (a warp owns NWR consecutive rows, whole SwiGLU pairs)
// x RB input rows staged in shared memory.  Every lane streams 16-byte weight vectors (Codec<F>::EPV elements) with
// the loads of UNR iterations issued before their FMAs, fp32 accumulation, warp-shuffle
// reduction.  Group-quantised formats multiply the lane's partial sum over one group
// slice by that group's fp16 scale.  The RMSNorm of the input rows (when norm_w !=
// nullptr) is computed in the prologue, so the normalised activations never touch HBM.
//
// Shared-memory order of an input row: inside each block of 32*EPV elements (one warp
// iteration) the 8 elements of part p of lane l sit at (p*32 + l)*8, so the float4 reads
// of one part by the 32 lanes are consecutive (at most 2-way bank conflicts).
constexpr int LIN_WARPS = 8;
constexpr int LIN_THREADS = LIN_WARPS * 32;

template <int EPV>
__host__ __device__ __forceinline__ int lin_padded(int in_f) {
    return (in_f + 32 * EPV - 1) / (32 * EPV) * (32 * EPV);
}
template <int EPV>
__device__ __forceinline__ int lin_slot(int k) {
    const int blk = k / (32 * EPV), r = k - blk * (32 * EPV);
    const int ln = r / EPV, e = r - ln * EPV;
    return blk * (32 * EPV) + ((e >> 3) * 32 + ln) * 8 + (e & 7);
}

template <int F, int RB, int NWR>
__global__ void __launch_bounds__(LIN_THREADS) k_linear(const uint8_t* __restrict__ W, const __half* __restrict__ S,
                                                        int out_f, int in_f, const float* __restrict__ x, int ldx,
                                                        int rows, const float* __restrict__ norm_w, float eps,
                                                        float* __restrict__ y, int ldy, int mode) {
    pdl_enter();
    using C = Codec<F>;
    constexpr int EPV = C::EPV, NP = EPV / 8, G = C::GROUP;
    extern __shared__ float4 xs4[];
    float* xs = reinterpret_cast<float*>(xs4);
    __shared__ float red[RB][LIN_WARPS];
    __shared__ float scale_s[RB];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int r0 = blockIdx.y * RB;
    const int nr = min(RB, rows - r0);
    const int pin = lin_padded<EPV>(in_f);

    // Stage the input rows (fp32) in shared memory, zero past in_f.
    for (int r = 0; r < RB; ++r) {
        float ss = 0.0f;
        for (int i = tid * 4; i < pin; i += LIN_THREADS * 4) {
            float4 v = (r < nr && i < in_f) ? *reinterpret_cast<const float4*>(x + static_cast<size_t>(r0 + r) * ldx + i)
                                            : make_float4(0.f, 0.f, 0.f, 0.f);
            ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
            xs4[(r * pin + lin_slot<EPV>(i)) >> 2] = v;
        }
        if (norm_w != nullptr) {
            ss = warp_sum(ss);
            if (lane == 0) red[r][warp] = ss;
        }
    }
    if (norm_w != nullptr) {
        __syncthreads();
        if (tid < RB) {
            float t = 0.0f;
            for (int wi = 0; wi < LIN_WARPS; ++wi) t += red[tid][wi];
            scale_s[tid] = 1.0f / sqrtf(t / static_cast<float>(in_f) + eps);
        }
        __syncthreads();
        for (int r = 0; r < RB; ++r) {
            const float s = scale_s[r];
            for (int i = tid; i < in_f; i += LIN_THREADS) {
                const int q = r * pin + lin_slot<EPV>(i);
                xs[q] = xs[q] * s * norm_w[i];
            }
        }
    }
    __syncthreads();

    // This warp's NWR consecutive output rows (NWR even: SwiGLU pairs stay together).
    const int o0 = NWR * (blockIdx.x * LIN_WARPS + warp);
    if (o0 >= out_f) return;
    const size_t row_bytes = static_cast<size_t>(in_f) / EPV * 16;
    const int ng = G ? in_f / G : 0;
    const uint8_t* wr[NWR];
    const __half* sr[NWR];
#pragma unroll
    for (int i = 0; i < NWR; ++i) {
        const int o = o0 + i < out_f ? o0 + i : o0;
        wr[i] = W + static_cast<size_t>(o) * row_bytes;
        sr[i] = G ? S + static_cast<size_t>(o) * ng : nullptr;
    }

    float acc[NWR][RB];
#pragma unroll
    for (int i = 0; i < NWR; ++i)
#pragma unroll
        for (int r = 0; r < RB; ++r) acc[i][r] = 0.0f;

    // One 16-byte vector of each row: vector index vv (lane = vv % 32).  Every x float4 read
    // from shared memory feeds NWR rows.
    auto consume = [&](const uint4 (&u)[NWR], const float (&sc)[NWR], int vv) {
        const int base = (vv >> 5) * (32 * EPV) + lane * 8;
        float t[NWR][RB];
#pragma unroll
        for (int i = 0; i < NWR; ++i)
#pragma unroll
            for (int r = 0; r < RB; ++r) t[i][r] = 0.0f;
#pragma unroll
        for (int p = 0; p < NP; ++p) {
            float w[NWR][8];
#pragma unroll
            for (int i = 0; i < NWR; ++i) C::part(u[i], p, w[i]);
            const int off = base + p * 256;
#pragma unroll
            for (int r = 0; r < RB; ++r) {
                const float4 xa = xs4[(r * pin + off) >> 2];
                const float4 xb = xs4[(r * pin + off + 4) >> 2];
#pragma unroll
                for (int i = 0; i < NWR; ++i)
                    t[i][r] += w[i][0] * xa.x + w[i][1] * xa.y + w[i][2] * xa.z + w[i][3] * xa.w + w[i][4] * xb.x +
                               w[i][5] * xb.y + w[i][6] * xb.z + w[i][7] * xb.w;
            }
        }
#pragma unroll
        for (int i = 0; i < NWR; ++i)
#pragma unroll
            for (int r = 0; r < RB; ++r) acc[i][r] = G ? fmaf(sc[i], t[i][r], acc[i][r]) : acc[i][r] + t[i][r];
    };

    constexpr int UNR = (EPV == 8 ? 8 : 4) / NWR;
    const int nv = in_f / EPV;
    int v = lane;
    for (; v + 32 * (UNR - 1) < nv; v += 32 * UNR) {
        uint4 u[UNR][NWR];
        float sc[UNR][NWR];
#pragma unroll
        for (int k = 0; k < UNR; ++k)
#pragma unroll
            for (int i = 0; i < NWR; ++i) {
                u[k][i] = ld_nc16(wr[i] + static_cast<size_t>(v + 32 * k) * 16);
                sc[k][i] = G ? __half2float(sr[i][(v + 32 * k) * EPV / (G ? G : 1)]) : 1.0f;
            }
#pragma unroll
        for (int k = 0; k < UNR; ++k) consume(u[k], sc[k], v + 32 * k);
    }
    for (; v < nv; v += 32) {
        uint4 u[NWR];
        float sc[NWR];
#pragma unroll
        for (int i = 0; i < NWR; ++i) {
            u[i] = ld_nc16(wr[i] + static_cast<size_t>(v) * 16);
            sc[i] = G ? __half2float(sr[i][v * EPV / (G ? G : 1)]) : 1.0f;
        }
        consume(u, sc, v);
    }
#pragma unroll
    for (int i = 0; i < NWR; ++i)
#pragma unroll
        for (int r = 0; r < RB; ++r) acc[i][r] = warp_sum(acc[i][r]);
    if (lane < nr) {
        // lane r writes input row r (register arrays indexed by a compile-time loop).
#pragma unroll
        for (int r = 0; r < RB; ++r) {
            if (r != lane) continue;
            float* yr = y + static_cast<size_t>(r0 + r) * ldy;
#pragma unroll
            for (int i = 0; i < NWR; i += 2) {
                if (mode == LIN_SWIGLU) {
                    if (o0 + i + 1 < out_f) yr[(o0 + i) / 2] = silu_f(acc[i][r]) * acc[i + 1][r];
                } else {
#pragma unroll
                    for (int k = 0; k < 2; ++k) {
                        if (o0 + i + k >= out_f) continue;
                        if (mode == LIN_RESIDUAL)
                            yr[o0 + i + k] += acc[i + k][r];
                        else
                            yr[o0 + i + k] = acc[i + k][r];
                    }
                }
            }
        }
    }
}

constexpr size_t LIN_SMEM_CAP = 96 * 1024;  // fp32 staging budget that picks the row block

template <int F, int RB>
static void linear_rb(const void* W, const void* S, int out_f, int in_f, const float* x, int ldx, int rows,
                      const float* norm_w, float eps, float* y, int ldy, int mode, cudaStream_t st) {
    // One weight row pair per warp for a single input row; from two input rows on, four
    // weight rows per warp halve the shared-memory reads of x per weight.
    constexpr int NWR = RB >= 2 ? 4 : 2;
    const size_t smem = static_cast<size_t>(RB) * lin_padded<Codec<F>::EPV>(in_f) * sizeof(float);
    static bool attr_set = false;  // one attribute set per template instance
    if (!attr_set) {
        SOCB_CUDA(cudaFuncSetAttribute(k_linear<F, RB, NWR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       200 * 1024));
        attr_set = true;
    }
    const int groups = (out_f + NWR - 1) / NWR;
    dim3 grid((groups + LIN_WARPS - 1) / LIN_WARPS, (rows + RB - 1) / RB);
    launch_pdl(k_linear<F, RB, NWR>, dim3(grid), dim3(LIN_THREADS), smem, st, static_cast<const uint8_t*>(W),
                                                          static_cast<const __half*>(S), out_f, in_f, x, ldx, rows,
                                                          norm_w, eps, y, ldy, mode);
    SOCB_CUDA(cudaGetLastError());
    count_launches(1);
}

template <int F>
static void linear_f(const void* W, const void* S, int out_f, int in_f, const float* x, int ldx, int rows,
                     const float* norm_w, float eps, float* y, int ldy, int mode, cudaStream_t st) {
    constexpr int EPV = Codec<F>::EPV, G = Codec<F>::GROUP;
    if (in_f % EPV != 0 || (G > 0 && in_f % (G > 0 ? G : 1) != 0))
        throw Error(-1, "linear: in_features is not a multiple of the weight format's vector/group size");
    if (G && S == nullptr) throw Error(-1, "linear: group-quantised weights need their scales");
    const size_t row_smem = static_cast<size_t>(lin_padded<EPV>(in_f)) * sizeof(float);
    if (row_smem > 200 * 1024) throw Error(-1, "linear: in_features too large");
    // Largest row block whose fp32 staging fits the budget.
    const size_t cap = LIN_SMEM_CAP / row_smem;
    if (rows >= 8 && cap >= 8)
        linear_rb<F, 8>(W, S, out_f, in_f, x, ldx, rows, norm_w, eps, y, ldy, mode, st);
    else if (rows >= 4 && cap >= 4)
        linear_rb<F, 4>(W, S, out_f, in_f, x, ldx, rows, norm_w, eps, y, ldy, mode, st);
    else if (rows >= 2 && cap >= 2)
        linear_rb<F, 2>(W, S, out_f, in_f, x, ldx, rows, norm_w, eps, y, ldy, mode, st);
    else
        linear_rb<F, 1>(W, S, out_f, in_f, x, ldx, rows, norm_w, eps, y, ldy, mode, st);
}

void launch_linear(int wfmt, const void* W, const void* scales, int out_f, int in_f, const float* x, int ldx,
                   int rows, const float* norm_w, float eps, float* y, int ldy, int mode, cudaStream_t st) {
    if (rows <= 0 || out_f <= 0) return;
    if (ldx % 4 != 0) throw Error(-1, "linear: ldx must be a multiple of 4");
    if (launch_linear_mma(wfmt, W, scales, out_f, in_f, x, ldx, rows, norm_w, eps, y, ldy, mode, st)) return;
    switch (wfmt) {
        case WF_F16: linear_f<WF_F16>(W, scales, out_f, in_f, x, ldx, rows, norm_w, eps, y, ldy, mode, st); break;
        case WF_BF16: linear_f<WF_BF16>(W, scales, out_f, in_f, x, ldx, rows, norm_w, eps, y, ldy, mode, st); break;
        case WF_I8G64: linear_f<WF_I8G64>(W, scales, out_f, in_f, x, ldx, rows, norm_w, eps, y, ldy, mode, st); break;
        case WF_I4G32: linear_f<WF_I4G32>(W, scales, out_f, in_f, x, ldx, rows, norm_w, eps, y, ldy, mode, st); break;
        default: throw Error(-1, "linear: unsupported weight format");
    }
}

// ------------------------------------------------- q/k RMSNorm + RoPE + paged KV append
// One CTA per row; warp w handles heads w, w+8, ... over the (q | k | v) head list.
// Lane l holds DL = D/32 consecutive dims; the rotate-half partner of dim i < D/2 lives
// in lane l ^ 16.  cos/sin come from a host table built in double precision exactly as
// the reference computes them (rope.cpp:74-79), so angles match bit for bit.
template <int D>
__global__ void __launch_bounds__(256) k_qk_norm_rope_kv(const float* __restrict__ qkv, int hq, int hkv,
                                                         const float* __restrict__ qn_w,
                                                         const float* __restrict__ kn_w, float eps,
                                                         const float2* __restrict__ rope_cs, int rope_len,
                                                         const int* __restrict__ row_seq,
                                                         const int* __restrict__ row_pos, KVLayerView kv,
                                                         float* __restrict__ q_out, int* err) {
    pdl_enter();
    constexpr int DL = D / 32;
    constexpr int HALF = D / 2;
    const int row = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int pos = row_pos[row];
    const int seq = row_seq[row];
    const int nh = hq + 2 * hkv;
    const float* src_row = qkv + static_cast<size_t>(row) * nh * D;
    const int page_idx = pos / kv.page_tokens;
    const bool pos_ok = pos >= 0 && pos < rope_len && page_idx < kv.max_pages;
    if (!pos_ok) {
        if (threadIdx.x == 0) atomicOr(err, DERR_KV_RANGE);
        return;
    }
    const int page = kv.page_table[static_cast<size_t>(seq) * kv.max_pages + page_idx];
    const int slot = pos % kv.page_tokens;
    for (int h = warp; h < nh; h += 8) {
        const float* src = src_row + h * D + lane * DL;
        float v[DL];
#pragma unroll
        for (int j = 0; j < DL; ++j) v[j] = src[j];
        const bool is_v = h >= hq + hkv;
        if (is_v) {
            const int kvh = h - hq - hkv;
            __half* dst = kv.v + ((static_cast<size_t>(page) * hkv + kvh) * kv.page_tokens + slot) * D + lane * DL;
#pragma unroll
            for (int j = 0; j < DL; ++j) dst[j] = __float2half_rn(v[j]);
            continue;
        }
        const bool is_q = h < hq;
        const float* nw = is_q ? qn_w : kn_w;
        float ss = 0.0f;
#pragma unroll
        for (int j = 0; j < DL; ++j) ss += v[j] * v[j];
        ss = warp_sum(ss);
        const float s = 1.0f / sqrtf(ss / static_cast<float>(D) + eps);
#pragma unroll
        for (int j = 0; j < DL; ++j) v[j] = v[j] * s * nw[lane * DL + j];
        // rotate-half
        float o[DL];
        const bool first = lane < 16;
#pragma unroll
        for (int j = 0; j < DL; ++j) {
            const float partner = __shfl_xor_sync(0xffffffffu, v[j], 16);
            const int i = (lane * DL + j) % HALF;  // pair index
            const float2 cs = rope_cs[static_cast<size_t>(pos) * HALF + i];
            o[j] = first ? (v[j] * cs.x - partner * cs.y) : (partner * cs.y + v[j] * cs.x);
        }
        if (is_q) {
            float* dst = q_out + (static_cast<size_t>(row) * hq + h) * D + lane * DL;
#pragma unroll
            for (int j = 0; j < DL; ++j) dst[j] = o[j];
        } else {
            const int kvh = h - hq;
            __half* dst = kv.k + ((static_cast<size_t>(page) * hkv + kvh) * kv.page_tokens + slot) * D + lane * DL;
#pragma unroll
            for (int j = 0; j < DL; ++j) dst[j] = __float2half_rn(o[j]);
        }
    }
}

void launch_qk_norm_rope_kv(const float* qkv, const Rows& rows, int hq, int hkv, int head_dim, const float* qn_w,
                            const float* kn_w, float eps, const float2* rope_cs, int rope_len, const KVLayerView& kv,
                            float* q_out, int* err, cudaStream_t st) {
    if (rows.n <= 0) return;
    if (head_dim == 128)
        launch_pdl(k_qk_norm_rope_kv<128>, dim3(rows.n), dim3(256), 0, st, qkv, hq, hkv, qn_w, kn_w, eps, rope_cs,
                   rope_len, rows.seq, rows.pos, kv, q_out, err);
    else if (head_dim == 64)
        launch_pdl(k_qk_norm_rope_kv<64>, dim3(rows.n), dim3(256), 0, st, qkv, hq, hkv, qn_w, kn_w, eps, rope_cs,
                   rope_len, rows.seq, rows.pos, kv, q_out, err);
    else
        throw Error(-1, "head_dim must be 64 or 128");
    SOCB_CUDA(cudaGetLastError());
    count_launches(1);
}

// --------------------------------------------------------------------- attention
// Split-K causal GQA over the paged fp16 cache.  CTA = (row, kv head, key split);
// its 4 warps take keys round-robin and keep an online softmax per query head of the
// group, then merge through shared memory.  With one split the CTA writes the
// normalised output; otherwise it writes (m, l, o) partials for k_attn_combine.
constexpr int ATT_WARPS = 4;
constexpr int ATT_MAXG = 8;

template <int D>
__global__ void __launch_bounds__(ATT_WARPS * 32) k_attention(const float* __restrict__ q,
                                                              const int* __restrict__ row_seq,
                                                              const int* __restrict__ row_pos, int hq, int hkv,
                                                              KVLayerView kv, int n_splits,
                                                              float* __restrict__ out, float* __restrict__ part) {
    pdl_enter();
    constexpr int DL = D / 32;
    __shared__ float sm_m[ATT_WARPS][ATT_MAXG], sm_l[ATT_WARPS][ATT_MAXG];
    __shared__ float sm_o[ATT_WARPS][ATT_MAXG][D];
    const int row = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int G = hq / hkv;
    const int seq = row_seq[row];
    const int nvis = row_pos[row] + 1;
    // Key range of this split, derived per row so a captured graph stays valid as rows grow.
    const int chunk = ((nvis + n_splits - 1) / n_splits + 15) / 16 * 16;
    const int kb = split * chunk;
    const int ke = min(nvis, kb + chunk);
    const float scale = 1.0f / sqrtf(static_cast<float>(D));

    float qr[ATT_MAXG][DL];
#pragma unroll
    for (int g = 0; g < ATT_MAXG; ++g) {
        if (g < G) {
            const float* qp = q + (static_cast<size_t>(row) * hq + kvh * G + g) * D + lane * DL;
#pragma unroll
            for (int j = 0; j < DL; ++j) qr[g][j] = qp[j];
        }
    }
    float m[ATT_MAXG], l[ATT_MAXG], o[ATT_MAXG][DL];
#pragma unroll
    for (int g = 0; g < ATT_MAXG; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.0f;
#pragma unroll
        for (int j = 0; j < DL; ++j) o[g][j] = 0.0f;
    }
    const int* pt = kv.page_table + static_cast<size_t>(seq) * kv.max_pages;
    for (int p = kb + warp; p < ke; p += ATT_WARPS) {
        const int page = pt[p / kv.page_tokens];
        const size_t off = ((static_cast<size_t>(page) * hkv + kvh) * kv.page_tokens + (p % kv.page_tokens)) * D +
                           lane * DL;
        float kf[DL], vf[DL];
#pragma unroll
        for (int j = 0; j < DL; ++j) {
            kf[j] = __half2float(kv.k[off + j]);
            vf[j] = __half2float(kv.v[off + j]);
        }
#pragma unroll
        for (int g = 0; g < ATT_MAXG; ++g) {
            if (g >= G) break;
            float s = 0.0f;
#pragma unroll
            for (int j = 0; j < DL; ++j) s += qr[g][j] * kf[j];
            s = warp_sum(s) * scale;
            const float mn = fmaxf(m[g], s);
            const float corr = expf(m[g] - mn);
            const float pe = expf(s - mn);
            l[g] = l[g] * corr + pe;
#pragma unroll
            for (int j = 0; j < DL; ++j) o[g][j] = o[g][j] * corr + pe * vf[j];
            m[g] = mn;
        }
    }
#pragma unroll
    for (int g = 0; g < ATT_MAXG; ++g) {
        if (g >= G) break;
        if (lane == 0) {
            sm_m[warp][g] = m[g];
            sm_l[warp][g] = l[g];
        }
#pragma unroll
        for (int j = 0; j < DL; ++j) sm_o[warp][g][lane * DL + j] = o[g][j];
    }
    __syncthreads();
    // Merge the warps: thread t handles (g, d) pairs.
    for (int idx = threadIdx.x; idx < G * D; idx += ATT_WARPS * 32) {
        const int g = idx / D, d = idx % D;
        float M = -INFINITY;
        for (int w = 0; w < ATT_WARPS; ++w) M = fmaxf(M, sm_m[w][g]);
        float L = 0.0f, acc = 0.0f;
        if (M != -INFINITY) {
            for (int w = 0; w < ATT_WARPS; ++w) {
                const float f = sm_m[w][g] == -INFINITY ? 0.0f : expf(sm_m[w][g] - M);
                L += sm_l[w][g] * f;
                acc += sm_o[w][g][d] * f;
            }
        }
        const int h = kvh * G + g;
        if (n_splits == 1) {
            out[(static_cast<size_t>(row) * hq + h) * D + d] = L > 0.0f ? acc / L : 0.0f;
        } else {
            float* pp = part + ((static_cast<size_t>(row) * hq + h) * n_splits + split) * (D + 2);
            pp[d] = acc;
            if (d == 0) {
                pp[D] = M;
                pp[D + 1] = L;
            }
        }
    }
}

template <int D>
__global__ void k_attn_combine(const float* __restrict__ part, int hq, int n_splits, float* __restrict__ out) {
    pdl_enter();
    const int row = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
    const float* pp = part + (static_cast<size_t>(row) * hq + h) * n_splits * (D + 2);
    float M = -INFINITY;
    for (int s = 0; s < n_splits; ++s) M = fmaxf(M, pp[s * (D + 2) + D]);
    float L = 0.0f, acc = 0.0f;
    if (M != -INFINITY) {
        for (int s = 0; s < n_splits; ++s) {
            const float ms = pp[s * (D + 2) + D];
            const float f = ms == -INFINITY ? 0.0f : expf(ms - M);
            L += pp[s * (D + 2) + D + 1] * f;
            acc += pp[s * (D + 2) + d] * f;
        }
    }
    out[(static_cast<size_t>(row) * hq + h) * D + d] = L > 0.0f ? acc / L : 0.0f;
}

// Decode-shaped attention (few rows per sequence): CTA = (row, kv head, key split), 4
// warps; a group of LPK lanes owns one key at a time (LPK = 8, or 16 for 4 or more query
// heads per kv head at head_dim 128), each lane DPL = D / LPK dims of it, so 32 / LPK keys
// are in flight per warp step and the K/V rows are read as contiguous 16-byte vectors.  Every group keeps its own
// online-softmax state for the G query heads of the kv head (base-2 exponent, log2(e)
// folded into the query scale); the groups and warps are merged in shared memory at the
// end.  The K/V vectors of the next two keys of a group are in flight while it consumes one.
template <int D, int G>
__global__ void __launch_bounds__(128) k_attn_rows(const float* __restrict__ q, const int* __restrict__ row_seq,
                                                   const int* __restrict__ row_pos, int hq, int hkv, KVLayerView kv,
                                                   int n_splits, float* __restrict__ out, float* __restrict__ part) {
    pdl_enter();
    constexpr int LPK = (G >= 4 && D >= 128) ? 16 : 8, DPL = D / LPK, KPW = 32 / LPK, NW = 4, NS = NW * KPW;
    constexpr int NV = DPL / 8;  // 16-byte vectors per lane per key row
    __shared__ float sm_m[NS][G], sm_l[NS][G];
    __shared__ float sm_o[NS][G][D];
    const int row = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int grp = lane / LPK, sub = lane % LPK;
    const int seq = row_seq[row];
    const int nvis = row_pos[row] + 1;
    const int chunk = ((nvis + n_splits - 1) / n_splits + 15) / 16 * 16;
    const int kb = split * chunk;
    const int ke = min(nvis, kb + chunk);
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
    float m[G], l[G], o[G][DPL];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.0f;
#pragma unroll
        for (int j = 0; j < DPL; ++j) o[g][j] = 0.0f;
    }
    const int* pt = kv.page_table + static_cast<size_t>(seq) * kv.max_pages;
    auto load = [&](int p, uint4 (&kx)[NV], uint4 (&vx)[NV]) {
        if (p < ke) {
            const int page = pt[p / kv.page_tokens];
            const size_t off =
                ((static_cast<size_t>(page) * hkv + kvh) * kv.page_tokens + (p % kv.page_tokens)) * D + sub * DPL;
#pragma unroll
            for (int c = 0; c < NV; ++c) {
                kx[c] = ld_nc16(kv.k + off + c * 8);
                vx[c] = ld_nc16(kv.v + off + c * 8);
            }
        }
    };
    // keys p (consumed), p + NS and p + 2 NS (in flight)
    int p = kb + warp * KPW + grp;
    uint4 kc[NV], vc[NV], k1[NV], v1[NV];
    load(p, kc, vc);
    load(p + NS, k1, v1);
    for (; p - grp < ke; p += NS) {
        uint4 kn[NV], vn[NV];
        load(p + 2 * NS, kn, vn);
        if (p < ke) {
            float kf[DPL], vf[DPL];
#pragma unroll
            for (int c = 0; c < NV; ++c) {
                float w8[8];
                Codec<WF_F16>::part(kc[c], 0, w8);
#pragma unroll
                for (int j = 0; j < 8; ++j) kf[c * 8 + j] = w8[j];
                Codec<WF_F16>::part(vc[c], 0, w8);
#pragma unroll
                for (int j = 0; j < 8; ++j) vf[c * 8 + j] = w8[j];
            }
#pragma unroll
            for (int g = 0; g < G; ++g) {
                float sc = 0.0f;
#pragma unroll
                for (int j = 0; j < DPL; ++j) sc += qr[g][j] * kf[j];
#pragma unroll
                for (int off = 1; off < LPK; off <<= 1) sc += __shfl_xor_sync(0xffffffffu, sc, off);
                const float mn = fmaxf(m[g], sc);
                const float corr = exp2f(m[g] - mn);
                const float pe = exp2f(sc - mn);
                l[g] = l[g] * corr + pe;
#pragma unroll
                for (int j = 0; j < DPL; ++j) o[g][j] = o[g][j] * corr + pe * vf[j];
                m[g] = mn;
            }
        } else {
            // keep the shuffles of the other groups of this warp matched
#pragma unroll
            for (int g = 0; g < G; ++g) {
                float sc = 0.0f;
#pragma unroll
                for (int off = 1; off < LPK; off <<= 1) sc += __shfl_xor_sync(0xffffffffu, sc, off);
            }
        }
#pragma unroll
        for (int c = 0; c < NV; ++c) {
            kc[c] = k1[c];
            vc[c] = v1[c];
            k1[c] = kn[c];
            v1[c] = vn[c];
        }
    }
    const int slot = warp * KPW + grp;
#pragma unroll
    for (int g = 0; g < G; ++g) {
        if (sub == 0) {
            sm_m[slot][g] = m[g];
            sm_l[slot][g] = l[g];
        }
#pragma unroll
        for (int j = 0; j < DPL; ++j) sm_o[slot][g][sub * DPL + j] = o[g][j];
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < G * D; idx += NW * 32) {
        const int g = idx / D, d = idx % D;
        float M = -INFINITY;
        for (int w = 0; w < NS; ++w) M = fmaxf(M, sm_m[w][g]);
        float Lt = 0.0f, acc = 0.0f;
        if (M != -INFINITY) {
            for (int w = 0; w < NS; ++w) {
                const float f = sm_m[w][g] == -INFINITY ? 0.0f : exp2f(sm_m[w][g] - M);
                Lt += sm_l[w][g] * f;
                acc += sm_o[w][g][d] * f;
            }
        }
        const int h = kvh * G + g;
        if (n_splits == 1) {
            out[(static_cast<size_t>(row) * hq + h) * D + d] = Lt > 0.0f ? acc / Lt : 0.0f;
        } else {
            // partial in natural-exponent units for the combine kernel: M * ln(2)
            float* pp = part + ((static_cast<size_t>(row) * hq + h) * n_splits + split) * (D + 2);
            pp[d] = acc;
            if (d == 0) {
                pp[D] = M == -INFINITY ? -INFINITY : M * 0.6931471805599453f;
                pp[D + 1] = Lt;
            }
        }
    }
}

template <int D>
static bool attn_rows_d(int G, dim3 grid, const float* q, const Rows& rows, int hq, int hkv, const KVLayerView& kv,
                        int splits, float* out, float* scratch, cudaStream_t st) {
    switch (G) {
        case 1: launch_pdl(k_attn_rows<D, 1>, dim3(grid), dim3(128), 0, st, q, rows.seq, rows.pos, hq, hkv, kv, splits,
                           out, scratch); return true;
        case 2: launch_pdl(k_attn_rows<D, 2>, dim3(grid), dim3(128), 0, st, q, rows.seq, rows.pos, hq, hkv, kv, splits,
                           out, scratch); return true;
        case 4: launch_pdl(k_attn_rows<D, 4>, dim3(grid), dim3(128), 0, st, q, rows.seq, rows.pos, hq, hkv, kv, splits,
                           out, scratch); return true;
        case 8: launch_pdl(k_attn_rows<D, 8>, dim3(grid), dim3(128), 0, st, q, rows.seq, rows.pos, hq, hkv, kv, splits,
                           out, scratch); return true;
        default: return false;
    }
}

// SOC_B200_ATTENTION=rows selects the register-prefetch kernel instead of page streaming.
int attention_path() {
    const char* e = std::getenv("SOC_B200_ATTENTION");
    return (e && std::string(e) == "rows") ? 1 : 0;
}

int attention_splits(int rows, int hkv, int max_visible) {
    // enough CTAs for two waves, and no split longer than 512 keys (long contexts of a
    // ragged batch would otherwise form the tail)
    const int ctas = rows * hkv;
    int splits = (2 * 148 + ctas - 1) / ctas;
    const int by_chunk = (max_visible + 511) / 512;
    if (splits < by_chunk) splits = by_chunk;
    const int max_by_len = (max_visible + 63) / 64;
    if (splits > max_by_len) splits = max_by_len;
    if (splits < 1) splits = 1;
    return splits;
}

void launch_attention(const float* q, const Rows& rows, int splits, int hq, int hkv, int head_dim,
                      const KVLayerView& kv, float* out, float* scratch, size_t scratch_floats, int* err,
                      cudaStream_t st) {
    if (rows.n <= 0) return;
    if (hq % hkv != 0 || hq / hkv > ATT_MAXG) throw Error(-1, "attention: unsupported head grouping");
    if (splits < 1) splits = 1;
    const size_t need = static_cast<size_t>(rows.n) * hq * splits * (head_dim + 2);
    if (splits > 1 && (scratch == nullptr || need > scratch_floats)) throw Error(-5, "attention: split-K scratch too small");
    dim3 grid(rows.n, hkv, splits);
    const int G = hq / hkv;
    bool done = attention_path() == 0 &&
                launch_attention_pages(q, rows, splits, hq, hkv, head_dim, kv, out, scratch, err, st);
    if (!done && head_dim == 128) done = attn_rows_d<128>(G, grid, q, rows, hq, hkv, kv, splits, out, scratch, st);
    else if (!done && head_dim == 64) done = attn_rows_d<64>(G, grid, q, rows, hq, hkv, kv, splits, out, scratch, st);
    if (done) {
        if (splits > 1) {
            if (head_dim == 128) launch_pdl(k_attn_combine<128>, dim3(dim3(rows.n, hq)), dim3(128), 0, st, scratch, hq,
                                            splits, out);
            else launch_pdl(k_attn_combine<64>, dim3(dim3(rows.n, hq)), dim3(64), 0, st, scratch, hq, splits, out);
        }
    } else if (head_dim == 128) {
        launch_pdl(k_attention<128>, dim3(grid), dim3(ATT_WARPS * 32), 0, st, q, rows.seq, rows.pos, hq, hkv, kv,
                   splits, out, scratch);
        if (splits > 1) launch_pdl(k_attn_combine<128>, dim3(dim3(rows.n, hq)), dim3(128), 0, st, scratch, hq, splits,
                                   out);
    } else if (head_dim == 64) {
        launch_pdl(k_attention<64>, dim3(grid), dim3(ATT_WARPS * 32), 0, st, q, rows.seq, rows.pos, hq, hkv, kv,
                   splits, out, scratch);
        if (splits > 1) launch_pdl(k_attn_combine<64>, dim3(dim3(rows.n, hq)), dim3(64), 0, st, scratch, hq, splits,
                                   out);
    } else {
        throw Error(-1, "head_dim must be 64 or 128");
    }
    SOCB_CUDA(cudaGetLastError());
    count_launches(splits > 1 ? 2 : 1);
}

// ------------------------------------------------------- seeded random KV contents
// splitmix64 output function (Steele, Lea and Flood, 2014) applied to x + 0x9E3779B97F4A7C15.
__device__ __forceinline__ unsigned long long mix64(unsigned long long x) {
    unsigned long long z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// Element e = (pos * hkv_total + global head) * D + d of stream (seq * L + layer) * 2 + kind (0 = K,
// 1 = V): the twelve 16-bit fields of mix64(x), mix64(x + 1), mix64(x + 2) with
// x = seed + stream * 0xD1B54A32D192ED03 + 3 e are summed and mapped to sum / 65536 - 6
// (Irwin-Hall approximation of N(0, 1), exact in fp32) and rounded to fp16.
__global__ void k_kv_fill_random(__half* __restrict__ kpool, __half* __restrict__ vpool, size_t layer_stride,
                                 const int* __restrict__ pages, int page_tokens, int hkv, int hkv_total, int head_off,
                                 int D, int L, int n_tokens, int seq, unsigned long long seed) {
    const int d8n = D / 8;
    const size_t total = static_cast<size_t>(L) * 2 * n_tokens * hkv * d8n;
    for (size_t v = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; v < total;
         v += static_cast<size_t>(gridDim.x) * blockDim.x) {
        size_t r = v;
        const int d8 = static_cast<int>(r % d8n);
        r /= d8n;
        const int head = static_cast<int>(r % hkv);
        r /= hkv;
        const int pos = static_cast<int>(r % n_tokens);
        r /= n_tokens;
        const int kind = static_cast<int>(r % 2);
        const int layer = static_cast<int>(r / 2);
        const unsigned long long stream = (static_cast<unsigned long long>(seq) * L + layer) * 2 + kind;
        uint32_t packed[4];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const unsigned long long e =
                (static_cast<unsigned long long>(pos) * hkv_total + head_off + head) * D + d8 * 8 + j;
            const unsigned long long x = seed + stream * 0xD1B54A32D192ED03ull + 3ull * e;
            unsigned sum = 0;
#pragma unroll
            for (int w = 0; w < 3; ++w) {
                const unsigned long long z = mix64(x + w);
                sum += static_cast<unsigned>(z & 0xFFFF) + static_cast<unsigned>((z >> 16) & 0xFFFF) +
                       static_cast<unsigned>((z >> 32) & 0xFFFF) + static_cast<unsigned>(z >> 48);
            }
            const __half h = __float2half_rn(static_cast<float>(sum) * (1.0f / 65536.0f) - 6.0f);
            const uint32_t hb = *reinterpret_cast<const uint16_t*>(&h);
            packed[j >> 1] = (j & 1) ? (packed[j >> 1] | (hb << 16)) : hb;
        }
        const int page = pages[pos / page_tokens];
        __half* pool = (kind == 0 ? kpool : vpool) + layer * layer_stride;
        __half* dst = pool + ((static_cast<size_t>(page) * hkv + head) * page_tokens + pos % page_tokens) * D + d8 * 8;
        *reinterpret_cast<uint4*>(dst) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    }
}

void launch_kv_fill_random(__half* kpool, __half* vpool, size_t layer_stride, const int* pages, int page_tokens,
                           int hkv, int hkv_total, int head_off, int D, int L, int n_tokens, int seq,
                           unsigned long long seed, cudaStream_t st) {
    if (n_tokens <= 0) return;
    k_kv_fill_random<<<148 * 16, 256, 0, st>>>(kpool, vpool, layer_stride, pages, page_tokens, hkv, hkv_total,
                                               head_off, D, L, n_tokens, seq, seed);
    SOCB_CUDA(cudaGetLastError());
    count_launches(1);
}

// ------------------------------------------------------------------------ argmax
// Greedy pick per row: maximum logit / temperature, lowest index on ties (the reference's
// Sampler::SampleFromLogits, Mac/cpu/src/sampler.cpp:22-57, ranks logit / temperature and
// returns the best of its top_k, which is the maximum).  The division is the IEEE
// round-to-nearest one the reference's float division performs, so ties it creates between
// neighbouring logits are ties here too; temperature 1 compares the logits themselves.
// NaNs never win.
//
// One block per ARGMAX_COLS columns of a row (grid: column blocks x rows), so that even a single
// row spreads over dozens of SMs: every thread has four 16-byte loads in flight, the block reduces
// its best (value, index) key and merges it into keys[row] with a 64-bit atomic maximum (keys[row]
// starts at zero, which no value's key equals).  v_off is the global index of column 0 (a vocab
// shard under tensor parallelism).
constexpr int ARGMAX_THREADS = 256;
constexpr int ARGMAX_COLS = ARGMAX_THREADS * 16;

__global__ void __launch_bounds__(ARGMAX_THREADS) k_argmax(const float* __restrict__ logits, int V, int ld, int v_off,
                                                         float temp, unsigned long long* __restrict__ keys) {
    pdl_enter();
    __shared__ unsigned long long red[ARGMAX_THREADS / 32];
    const float* row = logits + static_cast<size_t>(blockIdx.y) * ld;
    const int c0 = blockIdx.x * ARGMAX_COLS;
    unsigned long long best = 0ull;
    auto take = [&](float x, int i) {
        const float v = temp == 1.0f ? x : __fdiv_rn(x, temp);
        if (v == v) {
            const unsigned long long k = argmax_key(v, v_off + i);
            best = k > best ? k : best;
        }
    };
    const bool vec = (ld % 4 == 0) && (reinterpret_cast<uintptr_t>(logits) % 16 == 0) && c0 + ARGMAX_COLS <= V;
    if (vec) {
        float4 f[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
            f[j] = __ldcs(reinterpret_cast<const float4*>(row + c0) + threadIdx.x + ARGMAX_THREADS * j);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int i = c0 + 4 * (threadIdx.x + ARGMAX_THREADS * j);
            take(f[j].x, i);
            take(f[j].y, i + 1);
            take(f[j].z, i + 2);
            take(f[j].w, i + 3);
        }
    } else {
        const int c1 = min(V, c0 + ARGMAX_COLS);
        for (int i = c0 + threadIdx.x; i < c1; i += ARGMAX_THREADS) take(row[i], i);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
    }
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long b = 0ull;
#pragma unroll
        for (int w = 0; w < ARGMAX_THREADS / 32; ++w) b = red[w] > b ? red[w] : b;
        if (b != 0ull) atomicMax(keys + blockIdx.y, b);
    }
}

// keys_all [shards][rows] -> id of the largest key per row (ties: lowest global index).
__global__ void k_argmax_merge(const unsigned long long* __restrict__ keys_all, int shards, int rows,
                               int* __restrict__ next_ids) {
    pdl_enter();
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    unsigned long long b = 0ull;
    for (int s = 0; s < shards; ++s) {
        const unsigned long long k = keys_all[static_cast<size_t>(s) * rows + r];
        b = k > b ? k : b;
    }
    next_ids[r] = b == 0ull ? 0 : argmax_key_index(b);
}

__global__ void k_zero_keys(unsigned long long* keys, int n) {
    pdl_enter();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) keys[i] = 0ull;
}

void launch_argmax_keys(const float* logits, int vocab, int ld, int rows, int v_off, float temperature,
                        unsigned long long* keys, cudaStream_t st) {
    if (rows <= 0) return;
    // a kernel rather than a memset node, so that the step stays a graph of kernels only
    launch_pdl(k_zero_keys, dim3((rows + 255) / 256), dim3(256), 0, st, keys, rows);
    const dim3 grid((vocab + ARGMAX_COLS - 1) / ARGMAX_COLS, rows);
    launch_pdl(k_argmax, dim3(grid), dim3(ARGMAX_THREADS), 0, st, logits, vocab, ld, v_off, temperature, keys);
    SOCB_CUDA(cudaGetLastError());
    count_launches(2);
}

void launch_argmax(const float* logits, int vocab, int ld, int rows, float temperature, unsigned long long* keys,
                   int* next_ids, cudaStream_t st) {
    if (rows <= 0) return;
    launch_argmax_keys(logits, vocab, ld, rows, 0, temperature, keys, st);
    launch_argmax_merge(keys, 1, rows, next_ids, st);
}

void launch_argmax_merge(const unsigned long long* keys_all, int shards, int rows, int* next_ids, cudaStream_t st) {
    if (rows <= 0) return;
    launch_pdl(k_argmax_merge, dim3((rows + 127) / 128), dim3(128), 0, st, keys_all, shards, rows, next_ids);
    SOCB_CUDA(cudaGetLastError());
    count_launches(1);
}

}  // namespace socb

namespace socb {

// ---------------------------------------------------------------- top-k candidates
// The sampler's candidate list (Sampler::SampleFromLogits, Mac/gpu/src/runtime/sampler.cpp:36-68):
// the k largest logit / temperature of a row, larger first; among equal values the lower token
// id first (the order the device argmax already uses).  As orderable keys (argmax_key, unique per
// token) the top k of a set is the top k of the union of its parts' top k, so the row is reduced
// in rounds: every CTA of the first launch sorts TOPK_CHUNK elements and keeps its first k; every
// CTA of a later launch merges up to TOPK_GROUP such lists and keeps its first k, until one list is
// left; the last launch writes the ids with their raw logits.  Element g of the row lives at
//   base + (g / seg_len) * seg_stride + g % seg_len
// (one segment per tensor-parallel vocab shard after the all-gather; one segment otherwise).
namespace {
constexpr int TOPK_CHUNK = 1024;  // elements per CTA of the first round
constexpr int TOPK_GROUP = 16;    // lists merged per CTA of the later rounds (16 x 64 keys at most)
constexpr int TOPK_THREADS = 512;  // two keys per thread: TOPK_CHUNK = 2 * TOPK_THREADS

__device__ __forceinline__ float topk_elem(const float* base, int g, int seg_len, size_t seg_stride) {
    return base[static_cast<size_t>(g / seg_len) * seg_stride + g % seg_len];
}

// Descending bitonic sort of 1,024 keys by the CTA's 512 threads: thread t holds keys t (a0) and
// t + 512 (a1).  Compare-exchange partners less than 32 apart sit in the same warp and swap by
// shuffles; 512 apart, in the same thread; in between, through shared memory `s` (1,024 keys) with a
// barrier per stage (19 barriers in all instead of 55).
__device__ __forceinline__ unsigned long long cx(unsigned long long a, unsigned long long b, bool keep_max) {
    return keep_max ? (a > b ? a : b) : (a < b ? a : b);
}

__device__ void bitonic1024_desc(unsigned long long& a0, unsigned long long& a1, unsigned long long* s) {
    const int t = threadIdx.x;
    for (int size = 2; size <= 2 * TOPK_THREADS; size <<= 1) {
        int stride = size >> 1;
        if (stride == TOPK_THREADS) {
            // keys t and t + 512 of one descending run: the lower index keeps the larger
            const unsigned long long hi = a0 > a1 ? a0 : a1, lo = a0 > a1 ? a1 : a0;
            a0 = hi;
            a1 = lo;
            stride >>= 1;
        }
        if (stride >= 32) {
            s[t] = a0;
            s[t + TOPK_THREADS] = a1;
            __syncthreads();
            for (; stride >= 32; stride >>= 1) {
                // pair q: the lower index i and i + stride
                const int i = (t / stride) * 2 * stride + t % stride, j = i + stride;
                const bool desc = (i & size) == 0;
                const unsigned long long x = s[i], y = s[j];
                if (desc ? (x < y) : (x > y)) {
                    s[i] = y;
                    s[j] = x;
                }
                __syncthreads();
            }
            a0 = s[t];
            a1 = s[t + TOPK_THREADS];
            __syncthreads();
        }
        for (; stride > 0; stride >>= 1) {
            const unsigned long long b0 = __shfl_xor_sync(0xffffffffu, a0, stride);
            const unsigned long long b1 = __shfl_xor_sync(0xffffffffu, a1, stride);
            const bool lower = (t & stride) == 0;
            a0 = cx(a0, b0, lower == ((t & size) == 0));
            a1 = cx(a1, b1, lower == (((t + TOPK_THREADS) & size) == 0));
        }
    }
}

__global__ void __launch_bounds__(TOPK_THREADS) k_topk_chunks(const float* __restrict__ base, int V, int seg_len,
                                                              size_t seg_stride, float temp, int k,
                                                              unsigned long long* __restrict__ cand) {
    pdl_enter();
    __shared__ unsigned long long s[TOPK_CHUNK];
    const int first = blockIdx.x * TOPK_CHUNK;
    unsigned long long a[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int g = first + threadIdx.x + h * TOPK_THREADS;
        unsigned long long key = 0ull;  // below every real key
        if (g < V) {
            const float raw = topk_elem(base, g, seg_len, seg_stride);
            const float v = temp == 1.0f ? raw : __fdiv_rn(raw, temp);
            if (v == v) key = argmax_key(v, g);
        }
        a[h] = key;
    }
    bitonic1024_desc(a[0], a[1], s);
    if (static_cast<int>(threadIdx.x) < k) cand[static_cast<size_t>(blockIdx.x) * k + threadIdx.x] = a[0];
}

// Lists [TOPK_GROUP b, TOPK_GROUP (b + 1)) of `lists` sorted lists of k keys -> list b of `out`;
// with one CTA (the last round) the ids and raw logits instead.
__global__ void __launch_bounds__(TOPK_THREADS) k_topk_merge(const unsigned long long* __restrict__ in, int lists,
                                                             int k, unsigned long long* __restrict__ out,
                                                             const float* __restrict__ base, int seg_len,
                                                             size_t seg_stride, float* __restrict__ top_logits,
                                                             int* __restrict__ top_ids) {
    pdl_enter();
    __shared__ unsigned long long s[TOPK_CHUNK];
    const int l0 = blockIdx.x * TOPK_GROUP, nl = min(TOPK_GROUP, lists - l0);
    const int n = nl * k;  // <= 1,024; the rest of the 1,024 sorted keys are zero
    unsigned long long a[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int i = threadIdx.x + h * TOPK_THREADS;
        a[h] = i < n ? in[static_cast<size_t>(l0) * k + i] : 0ull;
    }
    bitonic1024_desc(a[0], a[1], s);
    const int i = threadIdx.x;
    if (i < k) {
        const unsigned long long key = a[0];
        if (out != nullptr) {
            out[static_cast<size_t>(blockIdx.x) * k + i] = key;
        } else {
            const int id = key == 0ull ? -1 : argmax_key_index(key);
            top_ids[i] = id;
            top_logits[i] = id < 0 ? -INFINITY : topk_elem(base, id, seg_len, seg_stride);
        }
    }
}
}  // namespace

// First-round lists, then each later round's (at most a sixteenth as many), side by side.
int topk_scratch_keys(int V, int k) {
    const int chunks = (V + TOPK_CHUNK - 1) / TOPK_CHUNK;
    return 2 * chunks * k;
}

void launch_topk(const float* base, int V, int seg_len, size_t seg_stride, float temperature, int k,
                 unsigned long long* cand, float* top_logits, int* top_ids, cudaStream_t st) {
    if (k < 1 || k > TOPK_MAX || V < 1) throw Error(-2, "top-k: k out of range");
    int lists = (V + TOPK_CHUNK - 1) / TOPK_CHUNK;
    launch_pdl(k_topk_chunks, dim3(lists), dim3(TOPK_THREADS), 0, st, base, V, seg_len, seg_stride, temperature, k,
               cand);
    int launches = 1;
    unsigned long long* in = cand;
    unsigned long long* out = cand + static_cast<size_t>(lists) * k;
    while (lists > TOPK_GROUP) {
        const int groups = (lists + TOPK_GROUP - 1) / TOPK_GROUP;
        launch_pdl(k_topk_merge, dim3(groups), dim3(TOPK_THREADS), 0, st, in, lists, k, out, base, seg_len, seg_stride,
                   nullptr, nullptr);
        ++launches;
        // the next round reads this one's lists and writes over the ones it just read
        std::swap(in, out);
        lists = groups;
    }
    launch_pdl(k_topk_merge, dim3(1), dim3(TOPK_THREADS), 0, st, in, lists, k, nullptr, base, seg_len, seg_stride,
               top_logits, top_ids);
    SOCB_CUDA(cudaGetLastError());
    count_launches(launches + 1);
}

}  // namespace socb
