// jinf-b200: the reference's CUDA kernel C-ABI, re-implemented for sm_100a.
//
// The reference declares these inside src/engine.cpp:12-31 and defines them in
// cuda/*.cu. Semantics are kept:
//   - every pointer is a device pointer owned by the caller, nothing is allocated;
//   - calls are asynchronous on `stream` and return void (an unsupported qtype is
//     reported on stderr and through jinf_cuda_last_error(), as the reference only
//     printed it, reference cuda/matmul_kernels.cu:221-223);
//   - `rows`/`cols` are out/in features, blocks run along `cols`;
//   - weights are the reference's AoS blocks (18-byte Q4_0, 144-byte Q4_K, ...).
//
// Numerics: fp32 activations and accumulation. Dequantized weight values are
// bit-exact with the reference's host dequantizer.
#pragma once

#include <stddef.h>
#include <stdint.h>

typedef struct CUstream_st* cudaStream_t;

#ifdef __cplusplus
extern "C" {
#endif

// y[rows] = dequant(W[rows][cols]) . x[cols] for Q4_0 / Q4_K / Q8_0 / Q6_K blocks.
// Replaces reference cuda/matmul_kernels.cu:198-225 (jinf_cuda_dequant_matvec).
void jinf_cuda_dequant_matvec(const void* weight, const float* input, float* output,
                              int rows, int cols, int qtype, cudaStream_t stream);

// a[i] += b[i]. Replaces reference cuda/matmul_kernels.cu:227-231.
void jinf_cuda_residual_add(float* a, const float* b, int n, cudaStream_t stream);

// Block -> fp32. Replace reference cuda/dequant_kernels.cu:116-143.
void jinf_cuda_dequantize_q4_0(const void* data, float* output, int n_blocks, cudaStream_t stream);
void jinf_cuda_dequantize_q4_K(const void* data, float* output, int n_blocks, cudaStream_t stream);
void jinf_cuda_dequantize_q8_0(const void* data, float* output, int n_blocks, cudaStream_t stream);
void jinf_cuda_dequantize_q6_K(const void* data, float* output, int n_blocks, cudaStream_t stream);

// out = in * rsqrt(mean(in^2) + eps) * w; weight_type 0 = f32, 1 = f16 (anything
// else is read as f32, as in the reference). Replaces reference cuda/rmsnorm_kernel.cu:65-85.
void jinf_cuda_rmsnorm(float* output, const float* input, const void* weight,
                       int n, float eps, int weight_type, cudaStream_t stream);

// In-place adjacent-pair RoPE on q [n_heads*head_dim] and k [n_heads_kv*head_dim]
// at position pos, theta_i = freq_base^(-2i/head_dim). Replaces reference cuda/rope_kernel.cu:54-61.
void jinf_cuda_rope(float* q, float* k, int head_dim, int n_heads, int n_heads_kv,
                    int pos, float freq_base, cudaStream_t stream);

// out = gate * sigmoid(gate) * up. Replaces reference cuda/silu_kernel.cu:22-27.
void jinf_cuda_silu_mul(float* output, const float* gate, const float* up, int n, cudaStream_t stream);

// Softmax over n values (no call site in the reference engine; kept for ABI
// completeness). Replaces reference cuda/softmax_kernel.cu:46-51.
void jinf_cuda_softmax(float* output, const float* input, int n, cudaStream_t stream);

// Decode GQA attention over an fp32 cache laid out [max_ctx][n_heads_kv*head_dim]
// (one layer), n_past positions (the current one included). Query head h reads
// kv head h / (n_heads / n_heads_kv). Replaces reference cuda/attention_kernel.cu:103-115.
// The B200 kernel is split-K (flash-decoding) and has no n_past shared-memory limit.
void jinf_cuda_attention(float* output, const float* q, const float* k_cache,
                         const float* v_cache, int head_dim, int n_heads,
                         int n_heads_kv, int n_past, int max_ctx, cudaStream_t stream);

// ---- New: error reporting for the void-returning entry points above ----
// Returns the first launch/argument error recorded since the last call and clears it
// (0 = none, otherwise a jinf_status value).
int jinf_cuda_last_error(void);

#ifdef __cplusplus
}
#endif
