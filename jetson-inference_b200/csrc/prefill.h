// Batched prefill (prefill_gemm.cu, prefill.cu): the prompt's tokens through each projection
// as one tensor-core contraction instead of one decode step per token.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace jinf {

// Y[t][m] = tok_scale[t] * sum_k X[t][k] W[m][k] for a Q4M (Q4_0) matrix W [rows][cols] and
// fp16 X [T][cols] (row stride cols, 16-byte aligned base), fp32 Y with row stride ldy.
// *err (device) is set to 1 when a pipeline wait ran out (the output is then incomplete).
cudaError_t prefill_gemm_launch(const uint8_t* w, int rows, int cols, const __half* x, int T, const float* tok_scale,
                                float* y, int ldy, int* err, cudaStream_t s);
size_t prefill_gemm_smem_bytes();

}  // namespace jinf
