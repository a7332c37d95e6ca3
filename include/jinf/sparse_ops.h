// jinf-b200: sparse FFN over neuron bundles (C-ABI of reference include/jinf/sparse_ops.h:30-40).
//
// Bundle layout per neuron (reference tools/prepare_model.cpp:299-308, :419-448):
//   [gate row: hidden_dim weights, `qtype` blocks][up row: same][down column: hidden_dim fp32]
// padded to `bundle_size` bytes. bundle_offsets[i] is the byte offset of the i-th active
// neuron's bundle inside `bundles`.
//
//   gate_up_tmp[i] = silu(gate_i . x) * (up_i . x)
//   output[d]      = sum_i gate_up_tmp[i] * down_col_i[d]      (output is overwritten)
//
// Differences from the reference, all in the direction of correctness:
//   - Q4_0, Q8_0, Q4_K and Q6_K gate/up rows are decoded with their own format (the
//     reference routes every type other than Q6_K to the Q4_K kernel,
//     reference cuda/sparse_matmul.cu:239-247);
//   - the down reduction is deterministic (fixed order, no atomics);
//   - the two dot products do not share one reduction buffer without a barrier
//     (reference cuda/sparse_matmul.cu:104-105).
#pragma once

#include <stddef.h>
#include <stdint.h>

typedef struct CUstream_st* cudaStream_t;

#ifdef __cplusplus
extern "C" {
#endif

void jinf_cuda_sparse_ffn(const void* bundles, const float* input, float* output,
                          const int* bundle_offsets, int num_activated, int hidden_dim,
                          int bundle_size, int qtype, float* gate_up_tmp, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
