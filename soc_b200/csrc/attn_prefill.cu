// Flash-style causal GQA prefill attention on tensor cores (mma.sync m16n8k16, fp16 in,
// fp32 accumulate) over the paged fp16 KV cache.
//
// Restates GroupedQueryAttention::ForwardWithPrefix (Mac/cpu/src/grouped_query_attention.cpp:59-142)
// for the rows of one prefill chunk: row r is position start + r of sequence `seq`, its
// visible keys are [0, start + r] (:98), query head h reads kv head h / (hq / hkv) (:101),
// scores are q.k / sqrt(D) (:81) and the softmax subtracts the running maximum (:104-123).
// The softmax is computed online over 64-key blocks (base-2 exponent with log2(e) folded
// into the query scale) and the output is divided by the row sum once at the end.
//
// CTA = 64 query rows of one head (4 warps x 16 rows); K and V blocks of 64 keys are
// gathered page by page with cp.async into XOR-swizzled shared memory (double buffered)
// and read with ldmatrix (V transposed).  Keys past the chunk's last position are
// zero-filled and masked.
#include "kernels.h"

namespace socb {
namespace {

constexpr int FQ = 64;  // query rows per CTA
constexpr int FK = 64;  // keys per block
constexpr int FW = 4;   // warps per CTA

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
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
// 16-byte async copy; src_bytes = 0 writes zeros without reading.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}

template <int D>
__global__ void __launch_bounds__(FW * 32) k_flash_prefill(const float* __restrict__ q, int n, int hq, int hkv,
                                                           int seq, int start, KVLayerView kv, float qscale,
                                                           float* __restrict__ out) {
    pdl_enter();
    constexpr int CH = D / 8;              // 16-byte chunks per key row
    constexpr int TILE = FK * D * 2;       // bytes of one K (or V) block
    extern __shared__ __align__(128) uint8_t fsm[];
    const uint32_t sbase = static_cast<uint32_t>(__cvta_generic_to_shared(fsm));
    auto ks = [&](int buf) { return sbase + buf * 2 * TILE; };
    auto vs = [&](int buf) { return sbase + buf * 2 * TILE + TILE; };

    const int qb = gridDim.x - 1 - blockIdx.x;  // longest causal extents first
    const int head = blockIdx.y, kvh = head / (hq / hkv);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = qb * FQ + warp * 16;
    const int ra = r0 + (lane >> 2), rb = ra + 8;
    const int qw = hq * D;

    // Query fragments (A operand, row-major 16 x D), scaled by log2(e)/sqrt(D), fp16.
    uint32_t qf[D / 16][4];
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
        const int col = kk * 16 + (lane & 3) * 2;
        float2 a0 = make_float2(0.f, 0.f), a1 = a0, a2 = a0, a3 = a0;
        if (ra < n) {
            const float* p = q + static_cast<size_t>(ra) * qw + head * D + col;
            a0 = *reinterpret_cast<const float2*>(p);
            a2 = *reinterpret_cast<const float2*>(p + 8);
        }
        if (rb < n) {
            const float* p = q + static_cast<size_t>(rb) * qw + head * D + col;
            a1 = *reinterpret_cast<const float2*>(p);
            a3 = *reinterpret_cast<const float2*>(p + 8);
        }
        qf[kk][0] = pack_h2(a0.x * qscale, a0.y * qscale);
        qf[kk][1] = pack_h2(a1.x * qscale, a1.y * qscale);
        qf[kk][2] = pack_h2(a2.x * qscale, a2.y * qscale);
        qf[kk][3] = pack_h2(a3.x * qscale, a3.y * qscale);
    }

    const int last_row = min(n, (qb + 1) * FQ) - 1;
    const int kv_end = start + last_row + 1;  // keys [0, kv_end) are visible to some row here
    const int nkb = (kv_end + FK - 1) / FK;
    const int pos_a = start + ra, pos_b = start + rb;
    const int* ptab = kv.page_table + static_cast<size_t>(seq) * kv.max_pages;

    auto load_block = [&](int kb, int buf) {
        for (int i = threadIdx.x; i < FK * CH; i += FW * 32) {
            const int key = i / CH, ch = i - key * CH;
            const int gk = kb * FK + key;
            const bool valid = gk < kv_end;
            size_t off = 0;
            if (valid) {
                const int page = ptab[gk / kv.page_tokens];
                off = ((static_cast<size_t>(page) * hkv + kvh) * kv.page_tokens + gk % kv.page_tokens) * D + ch * 8;
            }
            const uint32_t so = static_cast<uint32_t>((key * CH + (ch ^ (key & 7))) * 16);
            cp_async16(ks(buf) + so, kv.k + off, valid ? 16 : 0);
            cp_async16(vs(buf) + so, kv.v + off, valid ? 16 : 0);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };

    float o[D / 8][4];
#pragma unroll
    for (int t = 0; t < D / 8; ++t) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.0f;
    float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.0f, l_b = 0.0f;

    load_block(0, 0);
    for (int kb = 0; kb < nkb; ++kb) {
        const int buf = kb & 1;
        if (kb + 1 < nkb) {
            load_block(kb + 1, buf ^ 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();

        // S = Q K^T for this warp's 16 rows x 64 keys.
        float s[8][4];
#pragma unroll
        for (int t = 0; t < 8; ++t) s[t][0] = s[t][1] = s[t][2] = s[t][3] = 0.0f;
        const int qm = lane >> 3, lr = lane & 7;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
            for (int np = 0; np < 4; ++np) {
                const int key = np * 16 + (qm >> 1) * 8 + lr;
                const int ch = kk * 2 + (qm & 1);
                uint32_t b0, b1, b2, b3;
                ldsm_x4(ks(buf) + static_cast<uint32_t>((key * CH + (ch ^ (key & 7))) * 16), b0, b1, b2, b3);
                mma16816(s[2 * np], qf[kk], b0, b1);
                mma16816(s[2 * np + 1], qf[kk], b2, b3);
            }
        }
        // Causal mask (only blocks that reach past this warp's first position need it).
        const int kbase = kb * FK;
        if (kbase + FK - 1 > start + r0) {
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                const int key = kbase + t * 8 + (lane & 3) * 2;
                if (key > pos_a) s[t][0] = -INFINITY;
                if (key + 1 > pos_a) s[t][1] = -INFINITY;
                if (key > pos_b) s[t][2] = -INFINITY;
                if (key + 1 > pos_b) s[t][3] = -INFINITY;
            }
        }
        // Online softmax (rows ra / rb are spread over the 4 lanes of a quad).
        float mx_a = m_a, mx_b = m_b;
#pragma unroll
        for (int t = 0; t < 8; ++t) {
            mx_a = fmaxf(mx_a, fmaxf(s[t][0], s[t][1]));
            mx_b = fmaxf(mx_b, fmaxf(s[t][2], s[t][3]));
        }
        mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
        mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
        // every row sees key 0, so mx is finite after the first block
        const float ca = exp2f(m_a - mx_a), cb = exp2f(m_b - mx_b);
        m_a = mx_a;
        m_b = mx_b;
        l_a *= ca;
        l_b *= cb;
#pragma unroll
        for (int t = 0; t < D / 8; ++t) {
            o[t][0] *= ca;
            o[t][1] *= ca;
            o[t][2] *= cb;
            o[t][3] *= cb;
        }
        uint32_t pa[4][4];
#pragma unroll
        for (int t = 0; t < 8; ++t) {
            s[t][0] = exp2f(s[t][0] - m_a);
            s[t][1] = exp2f(s[t][1] - m_a);
            s[t][2] = exp2f(s[t][2] - m_b);
            s[t][3] = exp2f(s[t][3] - m_b);
            l_a += s[t][0] + s[t][1];
            l_b += s[t][2] + s[t][3];
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            pa[j][0] = pack_h2(s[2 * j][0], s[2 * j][1]);
            pa[j][1] = pack_h2(s[2 * j][2], s[2 * j][3]);
            pa[j][2] = pack_h2(s[2 * j + 1][0], s[2 * j + 1][1]);
            pa[j][3] = pack_h2(s[2 * j + 1][2], s[2 * j + 1][3]);
        }
        // O += P V
#pragma unroll
        for (int j = 0; j < 4; ++j) {
#pragma unroll
            for (int dp = 0; dp < D / 16; ++dp) {
                const int key = j * 16 + (qm & 1) * 8 + lr;
                const int ch = dp * 2 + (qm >> 1);
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(vs(buf) + static_cast<uint32_t>((key * CH + (ch ^ (key & 7))) * 16), b0, b1, b2, b3);
                mma16816(o[2 * dp], pa[j], b0, b1);
                mma16816(o[2 * dp + 1], pa[j], b2, b3);
            }
        }
        __syncthreads();
    }

    l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
    l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
    const float ia = 1.0f / l_a, ib = 1.0f / l_b;
#pragma unroll
    for (int t = 0; t < D / 8; ++t) {
        const int d = t * 8 + (lane & 3) * 2;
        if (ra < n)
            *reinterpret_cast<float2*>(out + static_cast<size_t>(ra) * qw + head * D + d) =
                make_float2(o[t][0] * ia, o[t][1] * ia);
        if (rb < n)
            *reinterpret_cast<float2*>(out + static_cast<size_t>(rb) * qw + head * D + d) =
                make_float2(o[t][2] * ib, o[t][3] * ib);
    }
}

template <int D>
void flash_d(const float* q, int n, int hq, int hkv, int seq, int start, const KVLayerView& kv, float* out,
             cudaStream_t st) {
    constexpr int smem = 2 * 2 * FK * D * 2;
    static bool set = false;
    if (!set) {
        SOCB_CUDA(cudaFuncSetAttribute(k_flash_prefill<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        set = true;
    }
    const float qscale = 1.4426950408889634f / sqrtf(static_cast<float>(D));
    dim3 grid((n + FQ - 1) / FQ, hq);
    launch_pdl(k_flash_prefill<D>, dim3(grid), dim3(FW * 32), smem, st, q, n, hq, hkv, seq, start, kv, qscale, out);
}

}  // namespace

void launch_flash_prefill(const float* q, int n, int hq, int hkv, int head_dim, int seq, int start,
                          const KVLayerView& kv, float* out, cudaStream_t st) {
    if (n <= 0) return;
    if (hq % hkv != 0) throw Error(-1, "attention: unsupported head grouping");
    if (kv.page_tokens != 16) throw Error(-1, "flash prefill expects 16-token pages");
    if (head_dim == 128)
        flash_d<128>(q, n, hq, hkv, seq, start, kv, out, st);
    else if (head_dim == 64)
        flash_d<64>(q, n, hq, hkv, seq, start, kv, out, st);
    else
        throw Error(-1, "head_dim must be 64 or 128");
    SOCB_CUDA(cudaGetLastError());
    count_launches(1);
}

}  // namespace socb
