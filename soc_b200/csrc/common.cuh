// Shared definitions of the soc_b200 CUDA library (host + device).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>

namespace socb {

// Library error with a C-ABI status code.
struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

// Message returned by soc_b200_last_error() on this thread (runtime.cu).
void set_last_error(const std::string& message);

#define SOCB_CUDA(expr)                                                                            \
    do {                                                                                           \
        cudaError_t e_ = (expr);                                                                   \
        if (e_ != cudaSuccess)                                                                     \
            throw ::socb::Error(-2, std::string("CUDA error: ") + cudaGetErrorString(e_) + " at " + \
                                    __FILE__ + ":" + std::to_string(__LINE__) + " (" #expr ")");  \
    } while (0)

// Programmatic dependent launch.  The modular kernels start with pdl_enter(): they wait until the
// kernel before them in the stream has completed and its memory is visible (before touching any
// memory), then let the next kernel launch.  Launched with launch_pdl, a kernel's launch and CTA
// scheduling overlap the tail of the one before it; launched normally, the wait returns at once.
__device__ __forceinline__ void pdl_enter() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Whether launch_pdl asks for programmatic serialization (SOC_B200_PDL=0 turns it off).
bool pdl_enabled();

template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    SOCB_CUDA(cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...));
}

// Weight element formats of the linear layers.
enum WFmt : int { WF_F16 = 1, WF_BF16 = 2, WF_I8G64 = 3, WF_I4G32 = 4 };

// Linear epilogues.
enum LinMode : int {
    LIN_STORE = 0,     // y = W x
    LIN_RESIDUAL = 1,  // y += W x            (o_proj / down_proj into the residual stream)
    LIN_SWIGLU = 2,    // rows (2j, 2j+1) = (gate_j, up_j): y[j] = silu(gate) * up
};

// Device-side error bits (kernels never trap; they record and skip).
enum DevErr : int {
    DERR_TOKEN_RANGE = 1,
    DERR_KV_RANGE = 2,
    DERR_WAIT_TIMEOUT = 4,
};

// ------------------------------------------------------------------ device helpers
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// 16-byte streaming load that bypasses L1 (weights are read exactly once per pass).
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ float2 h2_to_f2(uint32_t u) {
    __half2 h = *reinterpret_cast<__half2*>(&u);
    return __half22float2(h);
}

__device__ __forceinline__ float2 bf2_to_f2(uint32_t u) {
    // bf16 -> f32 is a 16-bit shift (exact).
    return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
}

template <typename T>
struct WTraits;
template <>
struct WTraits<__half> {
    static __device__ __forceinline__ float2 pair(uint32_t u) { return h2_to_f2(u); }
};
template <>
struct WTraits<__nv_bfloat16> {
    static __device__ __forceinline__ float2 pair(uint32_t u) { return bf2_to_f2(u); }
};

// ------------------------------------------------ 16-byte weight vectors per format
// A lane streams one 16-byte vector at a time: 8 fp16/bf16 elements, 16 int8 elements
// (one fp16 scale per 64) or 32 int4 elements (one fp16 scale per 32; two per byte, low
// nibble first, two's complement).  `part(u, p, w)` decodes elements [8p, 8p + 8) to exact
// fp32 values; the group scale is applied to the 8..32-element partial sum afterwards.
// Integer decode: the biased byte is placed in the mantissa of 2^23 with PRMT and the bias
// is subtracted (exact for every value).
__device__ __forceinline__ float biased_byte_f(uint32_t biased, int i, float bias) {
    return __int_as_float(static_cast<int>(__byte_perm(biased, 0x4B000000u, 0x7540u | static_cast<uint32_t>(i)))) - bias;
}
__device__ __forceinline__ uint32_t u4_word(const uint4& u, int i) {
    return i == 0 ? u.x : i == 1 ? u.y : i == 2 ? u.z : u.w;
}

template <int F>
struct Codec;
template <>
struct Codec<WF_F16> {
    static constexpr int EPV = 8, GROUP = 0;
    static __device__ __forceinline__ void part(const uint4& u, int, float (&w)[8]) {
        const float2 a = h2_to_f2(u.x), b = h2_to_f2(u.y), c = h2_to_f2(u.z), d = h2_to_f2(u.w);
        w[0] = a.x; w[1] = a.y; w[2] = b.x; w[3] = b.y; w[4] = c.x; w[5] = c.y; w[6] = d.x; w[7] = d.y;
    }
};
template <>
struct Codec<WF_BF16> {
    static constexpr int EPV = 8, GROUP = 0;
    static __device__ __forceinline__ void part(const uint4& u, int, float (&w)[8]) {
        const float2 a = bf2_to_f2(u.x), b = bf2_to_f2(u.y), c = bf2_to_f2(u.z), d = bf2_to_f2(u.w);
        w[0] = a.x; w[1] = a.y; w[2] = b.x; w[3] = b.y; w[4] = c.x; w[5] = c.y; w[6] = d.x; w[7] = d.y;
    }
};
template <>
struct Codec<WF_I8G64> {
    static constexpr int EPV = 16, GROUP = 64;
    static __device__ __forceinline__ void part(const uint4& u, int p, float (&w)[8]) {
        const uint32_t lo = u4_word(u, 2 * p) ^ 0x80808080u, hi = u4_word(u, 2 * p + 1) ^ 0x80808080u;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            w[i] = biased_byte_f(lo, i, 8388736.0f);  // 2^23 + 128
            w[4 + i] = biased_byte_f(hi, i, 8388736.0f);
        }
    }
};
template <>
struct Codec<WF_I4G32> {
    static constexpr int EPV = 32, GROUP = 32;
    static __device__ __forceinline__ void part(const uint4& u, int p, float (&w)[8]) {
        const uint32_t v = u4_word(u, p);
        const uint32_t ev = (v & 0x0F0F0F0Fu) ^ 0x08080808u, od = ((v >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            w[2 * i] = biased_byte_f(ev, i, 8388616.0f);  // 2^23 + 8
            w[2 * i + 1] = biased_byte_f(od, i, 8388616.0f);
        }
    }
};

__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + expf(-g)); }

// Orderable key for (value, index) argmax with the lowest index winning ties.
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
    uint32_t b = __float_as_uint(v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return (static_cast<unsigned long long>(b) << 32) | static_cast<uint32_t>(0x7fffffff - idx);
}
__device__ __forceinline__ int argmax_key_index(unsigned long long k) {
    return 0x7fffffff - static_cast<int>(static_cast<uint32_t>(k & 0xffffffffull));
}

}  // namespace socb
