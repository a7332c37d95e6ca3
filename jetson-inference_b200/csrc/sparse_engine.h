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
// The same with the FFN prologue fused into the W1 GEMV: h_out = h_in + y_res and
// x = rmsnorm(h_out) * gain are computed by every CTA of that kernel (CTA 0 stores both).
cudaError_t sparse_predict_norm(const void* w1, const void* w2, const float* h_in, const float* y_res, float* h_out,
                                const float* gain, float eps, float* x, int d, int r, int n_ff, int k, int bundle_size,
                                int32_t* ids, int32_t* offsets, float* scratch, cudaStream_t s);
// FFN over the active bundles (jinf_cuda_sparse_ffn, abi_sparse.cu) with the prologue fused into
// its gate/up kernel: h_out = h_in + y_res, x = rmsnorm(h_out) * gain in every CTA (CTA 0 stores
// h_out), out = sum over active n of silu(gate_n . x) (up_n . x) down_n. Q4_0 bundles,
// d % 128 == 0 and d <= 8192 (sparse_ffn_fused_ok).
bool sparse_ffn_fused_ok(int d, int qtype);
cudaError_t sparse_ffn_fused(const uint8_t* bundles, const float* h_in, const float* y_res, float* h_out,
                             const float* gain, float eps, float* out, const int* offs, int n_act, int d,
                             int bundle_size, float* gu_tmp, cudaStream_t s);
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
