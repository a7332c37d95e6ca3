// Batched prefill (prefill_gemm.cu, prefill.cu): the prompt's tokens through each projection
// as one tensor-core contraction instead of one decode step per token.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace jinf {

// Y[t][m] (+)= tok_scale[t] * sum_k X[t][k] W[m][k] for a Q4M (Q4_0) matrix W [rows][cols]
// and fp16 X [T][cols] (row stride cols, 16-byte aligned base), fp32 Y with row stride ldy
// (accum: added to Y). *err (device) is set to 1 when a pipeline wait ran out (the output is
// then incomplete).
cudaError_t prefill_gemm_launch(const uint8_t* w, int rows, int cols, const __half* x, int T, const float* tok_scale,
                                float* y, int ldy, int accum, int* err, cudaStream_t s);

// Element-wise steps and attention (prefill.cu). Rows are tokens.
// x16[t] = fp16(s_t * (gain ? h[t] * rsqrt(mean(h[t]^2) + eps) * gain : h[t])), tok_scale[t] = 1 / s_t
// (s_t a power of two that puts the row's largest magnitude in [2^13, 2^14)).
cudaError_t prefill_rows_to_f16(const float* h, int ldh, int T, int n, const float* gain, float eps, __half* x16,
                                int ldx, float* tok_scale, cudaStream_t s);
// x16[t][i] = fp16(s_t * SiLU(gu[t][2i]) * gu[t][2i + 1]) over ff activations, tok_scale[t] = 1 / s_t.
cudaError_t prefill_silu_to_f16(const float* gu, int ldg, int T, int ff, __half* x16, int ldx, float* tok_scale,
                                cudaStream_t s);
// h[t] = table row tokens[t] (tokens in device memory).
cudaError_t prefill_embed(const float* table, const int* tokens, int T, int d, float* h, cudaStream_t s);
// RoPE of the q and k columns of y ([T][ldy]: q | k | v) at positions p0 + t; q16 [T][nq] = q / sqrt(hd)
// in fp16; k and v into the fp16 caches [Hkv][max_ctx][hd] at positions p0 + t.
cudaError_t prefill_rope_qkv(const float* y, int ldy, int T, int p0, int nq, int nk, int hd, float base, __half* q16,
                             __half* kc, __half* vc, int max_ctx, cudaStream_t s);
// Causal GQA attention of the T queries q16 (positions p0 + t) over cache positions 0 .. p0 + t:
// out [T][n_heads * hd] fp32.
cudaError_t prefill_attention(const __half* q16, int n_heads, int n_kv_heads, int hd, int T, int p0, const __half* kc,
                              const __half* vc, int max_ctx, float* out, cudaStream_t s);
size_t prefill_gemm_smem_bytes();

}  // namespace jinf
