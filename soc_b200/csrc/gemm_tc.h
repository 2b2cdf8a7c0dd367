// Tensor-core GEMM for prefill and batched rows (gemm_tc.cu): y = epilogue(A W^T) with
// A = activations [M, K] and W = weights [N, K], both fp16 or both bf16, K-major.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace socb {

// Whether this process can build TMA descriptors (driver entry point present).
bool tc_available();
// Rows from which the fp16/bf16 linears of a forward run on the tensor-core GEMM (default 16;
// SOC_B200_TC_MIN_ROWS overrides it, 0 disables the path); group-quantised linears use it
// from 2 * that many rows (their weights are expanded to fp16 first).
int tc_min_rows();
// Whether a linear of `rows` input rows and an out_f x in_f matrix of weight format wfmt runs on
// the tensor-core GEMM (SOC_B200_TC_MIN_ROWS, when set, is a plain row threshold).
bool tc_rows_ok(int rows, long long out_f, long long in_f, int wfmt);
// Up to this many rows (default 512, SOC_B200_TC_SPLIT_MAX_ROWS) the GEMM input rows are
// carried as hi + lo halves (two MMAs per K step, about 22 significand bits); above it as
// one half (prefill-sized GEMMs, tensor-throughput bound).
int tc_split_max_rows();
// 1 (default): fp32 GEMM outputs leave through shared memory and TMA stores / reduce-adds;
// SOC_B200_TC_OUT=registers: stores from the epilogue threads' registers.
int tc_out_tma();
// 2-D TMA descriptor of a row-major [rows, cols] fp16/bf16 matrix with leading dimension
// `ld` elements, box = 64 columns x box_rows rows, 128-byte swizzle.
void tc_make_map(CUtensorMap* map, const void* base, int wfmt, uint64_t rows, uint64_t cols, uint64_t ld,
                 uint32_t box_rows);
constexpr uint32_t TC_BOX_A = 128;  // rows of an activation tile
constexpr uint32_t TC_BOX_W = 256;  // rows of a weight tile
// y (mode)= A W^T, A = hi (+ lo when a_lo != nullptr).  mode LIN_STORE / LIN_RESIDUAL (fp32
// y += ...) / LIN_SWIGLU (rows (2j, 2j+1) of W are (gate_j, up_j); y[:, j] = silu(gate) *
// up).  out_half: y is fp16/bf16 (the weight type) instead of fp32 (STORE and SWIGLU only),
// with its remainder in y_lo when that is not null.  ws (nullable): fp32 workspace of
// ws_floats for split-K partial tiles, used when the output tiles alone would leave most
// SMs idle (small M); the split never changes which products are summed.
void launch_gemm_tc(int wfmt, const CUtensorMap& a, const CUtensorMap* a_lo, const CUtensorMap& w, int M, int N,
                    int K, void* y, int ldy, int mode, bool out_half, void* y_lo, float* ws, size_t ws_floats,
                    int* err, cudaStream_t st);
constexpr size_t TC_WS_FLOATS = size_t(16) << 20;  // 64 MB split-K workspace per context
// out[r, :] = T(x'[r, :]) with x' = x * (norm_w ? rmsnorm scale * norm_w : 1) (T = fp16/bf16);
// out_lo (nullable) = T(x' - float(out)).
void launch_rows_to_half(int wfmt, const float* x, int ldx, int rows, int cols, const float* norm_w, float eps,
                         void* out, void* out_lo, int ldo, cudaStream_t st);
// Group-quantised matrix [rows, cols] -> fp16 values float(q) * float(scale) rounded once.
void launch_dequant(int wfmt, const void* W, const void* scales, int rows, int cols, int out_fmt, void* out,
                    cudaStream_t st);

}  // namespace socb
