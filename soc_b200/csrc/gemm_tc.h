// Tensor-core GEMM for prefill and batched rows (gemm_tc.cu): y = epilogue(A W^T) with
// A = activations [M, K] and W = weights [N, K], both fp16 or both bf16, K-major.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace socb {

// Whether this process can build TMA descriptors (driver entry point present).
bool tc_available();
// Rows from which the linears of a forward run on the tensor-core GEMM (default 64;
// SOC_B200_TC_MIN_ROWS overrides it, 0 disables the path).
int tc_min_rows();
// 2-D TMA descriptor of a row-major [rows, cols] fp16/bf16 matrix with leading dimension
// `ld` elements, box = 64 columns x box_rows rows, 128-byte swizzle.
void tc_make_map(CUtensorMap* map, const void* base, int wfmt, uint64_t rows, uint64_t cols, uint64_t ld,
                 uint32_t box_rows);
constexpr uint32_t TC_BOX_A = 128;  // rows of an activation tile
constexpr uint32_t TC_BOX_W = 256;  // rows of a weight tile
// y (mode)= A W^T.  mode LIN_STORE / LIN_RESIDUAL (fp32 y += ...) / LIN_SWIGLU (rows
// (2j, 2j+1) of W are (gate_j, up_j); y[:, j] = silu(gate) * up).  out_half: y is fp16/bf16
// (the weight type) instead of fp32 (STORE and SWIGLU only).
void launch_gemm_tc(int wfmt, const CUtensorMap& a, const CUtensorMap& w, int M, int N, int K, void* y, int ldy,
                    int mode, bool out_half, int* err, cudaStream_t st);
// out[r, :] = T(x[r, :] * (norm_w ? rmsnorm scale * norm_w : 1)) for r < rows (T = fp16/bf16).
void launch_rows_to_half(int wfmt, const float* x, int ldx, int rows, int cols, const float* norm_w, float eps,
                         void* out, int ldo, cudaStream_t st);

}  // namespace socb
