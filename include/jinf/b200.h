// jinf-b200: new entry points with no counterpart in the reference ABI.
//
// These expose the engine's B200 building blocks so callers and tests can use them
// outside the engine: the lossless Q4M weight layout, the tensor-core Q4_0 GEMV over it
// and the fp16-KV split-K decode attention. Same conventions as the reference kernel ABI
// (device pointers owned by the caller, asynchronous on `stream`) except that each
// returns a jinf_status instead of void.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include "jinf/common.h"

typedef struct CUstream_st* cudaStream_t;

#ifdef __cplusplus
extern "C" {
#endif

// Bytes of the Q4M image of a rows x cols Q4_0 matrix; 0 if cols is not a multiple of 32
// (whole blocks; the last 128-column group is zero-padded).
// Q4M is the layout of the tensor-core GEMV: 32-row tile pairs x 128-column groups, 2304
// bytes per (pair, group), every nibble and scale of the AoS blocks moved, none re-quantised.
uint64_t jinf_b200_q4m_bytes(int rows, int cols);

// The same for any weight type the engine streams: qtype JINF_TYPE_Q4_0, JINF_TYPE_Q4_K
// (2432 bytes per (pair, group); cols a multiple of 256), JINF_TYPE_Q6_K (3392 bytes; cols a
// multiple of 256) or JINF_TYPE_Q8_0 (4352 bytes; cols a multiple of 32). 0 for other types
// or shapes. No counterpart in the reference, whose matvecs read the AoS blocks (reference
// cuda/matmul_kernels.cu:47-185).
uint64_t jinf_b200_q4m_bytes_qt(int rows, int cols, int qtype);
jinf_status jinf_b200_q4m_pack_qt(const void* aos, int qtype, void* q4m, int rows, int cols, cudaStream_t stream);
// The same repack on the host (host buffers, no GPU needed), bit-identical to the device's:
// what a conversion tool uses to write pre-packed matrices (jinf_prepare_model_b200).
jinf_status jinf_b200_q4m_pack_host(const void* aos, int qtype, void* q4m, int rows, int cols);
jinf_status jinf_b200_gemv_q4m_qt(const void* q4m, int qtype, const void* x, int x_type, float* y, int rows,
                                  int cols, void* workspace, int kw, cudaStream_t stream);

// Repack reference AoS Q4_0 blocks [rows][cols/32] (device) into Q4M (device, q4m_bytes).
jinf_status jinf_b200_q4m_pack(const void* aos, void* q4m, int rows, int cols, cudaStream_t stream);

// Workspace bytes of jinf_b200_gemv_q4m for this shape (any kw up to 32).
size_t jinf_b200_gemv_q4m_workspace_bytes(int rows, int cols);

// y[rows] = W . x over a Q4M matrix on the tensor cores; x fp32 (JINF_TYPE_F32) or fp16
// (JINF_TYPE_F16), accumulation fp32. kw = K parts per 16-row tile (0 = chosen for the
// device). kw > 1 needs `workspace` (gemv_q4m_workspace_bytes, zeroed once before first
// use, then reusable by calls on the same stream); kw = 1 takes workspace = NULL.
jinf_status jinf_b200_gemv_q4m(const void* q4m, const void* x, int x_type, float* y, int rows, int cols,
                               void* workspace, int kw, cudaStream_t stream);

// Batched: Y[b][rows] = W . X[b] for b < batch (1..8), X [batch][cols] fp32 or fp16, one pass
// over the Q4_0 Q4M matrix (tensor cores: the MMA's columns carry 4 vectors' digits). Needs
// `workspace` (gemv_q4m_batch_workspace_bytes, zeroed once, reusable on the same stream)
// for shapes that split K. No counterpart in the reference (batch-1 GEMVs only).
size_t jinf_b200_gemv_q4m_batch_workspace_bytes(int rows, int cols, int batch);
jinf_status jinf_b200_gemv_q4m_batch(const void* q4m, const void* x, int x_type, float* y, int rows, int cols,
                                     int batch, void* workspace, cudaStream_t stream);
// The same for a Q4M image of reference block type `qtype` (Q4_0 = 2, Q8_0 = 8, Q4_K = 12,
// Q6_K = 14); kw = 0 picks the K split and how it is shared out, kw > 0 forces kw parts with
// each warp taking whole tile pairs, kw < 0 forces -kw parts with a CTA's warps splitting
// each of its tile pairs (1..32 parts, within shared memory).
size_t jinf_b200_gemv_q4m_batch_workspace_bytes_qt(int rows, int cols, int batch, int qtype);
jinf_status jinf_b200_gemv_q4m_batch_qt(const void* q4m, int qtype, const void* x, int x_type, float* y, int rows,
                                        int cols, int batch, void* workspace, int kw, cudaStream_t stream);

// y[rows] = W . (rmsnorm(h) * gain) over a Q4M matrix; workspace and kw as above.
jinf_status jinf_b200_gemv_q4m_rmsnorm(const void* q4m, const float* h, const float* gain, float eps, float* y,
                                       int rows, int cols, void* workspace, int kw, cudaStream_t stream);

// Same as jinf_b200_gemv_q4m with kw = 0, but allocation-free: no counterpart in the
// reference. The split-K workspace is a 4 MB static device array inside the library
// (counters zero at load and left zero by every call), so the caller neither allocates nor
// passes one; the first call on each device looks the array up and must not be inside a
// stream capture. rows <= 262144 (else JINF_ERR_INVALID); where the K split that kw = 0
// would pick needs more partial sums than the array holds, a smaller split is used. Calls
// that overlap in time share the array and race: serialise them.
jinf_status jinf_b200_gemv_q4m_noalloc(const void* q4m, const void* x, int x_type, float* y, int rows, int cols,
                                       cudaStream_t stream);

// ---- batched prefill (new; replaces the reference's one-token-at-a-time prompt loop,
// src/engine.cpp:690-751, with one tensor-core contraction per projection)
//
// y[t * ldy + m] (+)= tok_scale[t] * sum_k x[t][k] W[m][k] for t < T: W a Q4M (Q4_0) matrix
// [rows][cols], x fp16 [T][cols] (16-byte aligned, row stride cols), y fp32 (`accumulate`:
// added to y). tcgen05.mma with the accumulator in tensor memory; x by TMA. `err` is a device
// int the caller zeroed: the kernel sets it to 1 if a pipeline wait ran out (the output is
// then incomplete).
jinf_status jinf_b200_prefill_gemm(const void* q4m, int rows, int cols, const void* x_f16, int T,
                                   const float* tok_scale, float* y, int ldy, int accumulate, int* err,
                                   cudaStream_t stream);

// ---- sparse FFN (engine sparse modes; reference src/engine.cpp:339-415, src/activation_predictor.cpp)
//
// Fixed neuron mask of a layer: runs of 8 consecutive neurons, each kept with probability
// `keep` (seeded). Writes the kept ids ascending when `ids` is not NULL; returns the count.
int jinf_sparse_fixed_mask(uint64_t seed, int layer, int n_ff, float keep, int32_t* ids);
// Predictor matrix `which` (1: W1 [r][d], 2: W2 [n_ff][r]) of a layer as fp16 bits ~ N(0, 0.02)
// (host; the engine generates the same values on the device).
void jinf_sparse_predictor_weights(uint64_t seed, int layer, int which, int64_t n, uint16_t* out);
// Predictor on the device: z = ReLU(W1 x), s = W2 z (W1, W2 fp16, fp32 sums), then the k
// largest scores (ties: lower index first) as ids ascending and bundle byte offsets
// id * bundle_size. d and r multiples of 8 and at most 8192, n_ff <= JINF_TOPK_MAX_N (the scores are selected
// in one CTA's shared memory); scratch: r + n_ff floats (device). No counterpart in the
// reference, whose predictor ran on the host.
#define JINF_TOPK_MAX_N 49152
jinf_status jinf_b200_sparse_predict(const void* w1, const void* w2, const float* x, int d, int r, int n_ff, int k,
                                     int bundle_size, int32_t* ids, int32_t* offsets, float* scratch,
                                     cudaStream_t stream);

// ---- activation profiles (the reference's static-predictor file format, see
// jinf_engine_config.predictor_path): int32 n_layers, n_ff, total_tokens, then n_layers x n_ff
// float32 frequencies. Writer of reference tools/profile_activations.cpp:143-162: frequency =
// counts[l][n] / total_tokens. Reader of reference src/activation_predictor.cpp:226-300: the
// active neurons of layer l are those with frequency > threshold, written ascending to
// ids[l * n_ff ...] with their count in n_active[l]. JINF_ERR_INVALID when the file is of
// another shape, JINF_ERR_PARSE when it is truncated.
jinf_status jinf_activation_profile_write(const char* path, int n_layers, int n_ff, int total_tokens,
                                          const int32_t* counts);
jinf_status jinf_activation_profile_read(const char* path, float threshold, int n_layers, int n_ff, int32_t* ids,
                                         int32_t* n_active);

// Workspace bytes needed by jinf_b200_attention_f16 for this shape.
size_t jinf_b200_attention_workspace_bytes(int n_kv_heads, int head_dim, int max_ctx);

// Decode GQA attention over an fp16 cache laid out [n_kv_heads][max_ctx][head_dim],
// positions 0..n_pos-1, q fp32 [n_heads*head_dim] (no RoPE applied here), out fp32.
// `workspace` (device, attention_workspace_bytes) must be zeroed once before first use;
// it stays valid across calls on the same stream.
jinf_status jinf_b200_attention_f16(float* out, const float* q, const void* k_cache, const void* v_cache,
                                    int head_dim, int n_heads, int n_kv_heads, int n_pos, int max_ctx,
                                    void* workspace, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
