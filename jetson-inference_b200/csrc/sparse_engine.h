// Device building blocks of the engine's sparse-FFN mode (sparse_engine.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace jinf {

// h_out = h_in + y_res; x = rmsnorm(h_out) * gain (d <= 8192).
cudaError_t sparse_ffn_prologue(const float* h_in, const float* y_res, float* h_out, const float* gain, float eps,
                                int d, float* x, cudaStream_t s);
// z = ReLU(W1 x), s = W2 z, the k largest scores -> ids (ascending) and bundle offsets.
// scratch: r + n_ff floats.
cudaError_t sparse_predict(const void* w1, const void* w2, const float* x, int d, int r, int n_ff, int k,
                           int bundle_size, int32_t* ids, int32_t* offsets, float* scratch, cudaStream_t s);
// Neuron bundles (reference tools/prepare_model.cpp:299-308) from the staged AoS matrices.
cudaError_t sparse_bundle_gate_up(const uint8_t* gu_aos, int n_ff, int row_bytes, uint8_t* bundles, int bundle_size,
                                  cudaStream_t s);
cudaError_t sparse_bundle_down(const uint8_t* down_aos, int d, int n_ff, int qtype, uint8_t* bundles, int bundle_size,
                               int col_off, cudaStream_t s);
// Predictor matrix `which` (1: W1, 2: W2) of a layer, n fp16 values (jinf_sparse_predictor_weights).
cudaError_t sparse_fill_predictor(uint64_t seed, int layer, int which, int64_t n, void* dst, cudaStream_t s);
// Bytes of one neuron bundle for a d-wide model of weight type qtype (padded to 256).
int sparse_bundle_bytes(int d, int qtype);

}  // namespace jinf
