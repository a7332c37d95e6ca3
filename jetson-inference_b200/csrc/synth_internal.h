// Library-internal hooks of the synthetic-model generator (not part of the C-ABI).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "jinf/engine.h"

namespace jinf {

// Counter key, standard deviation and role (0 projection, 1 norm = ones, 2 embedding) of a
// synthetic tensor; false if the name is unknown.
bool synth_tensor_params(const jinf_synth_model* m, const char* name, uint64_t* key, float* stdv, int* role);

// Device generation, bit-identical with jinf_synth_read_rows:
// Q4_0 blocks of rows [r0, r0+nr) and columns [c0, c0+nc) (multiples of 32) of a tensor with
// `cols` columns; row i goes to dst + (dst_row0 + i*dst_row_step) * dst_row_bytes.
cudaError_t synth_fill_q4_0(uint64_t key, float stdv, int64_t cols, int64_t r0, int64_t nr, int64_t c0, int64_t nc,
                            uint8_t* dst, int64_t dst_row_bytes, int64_t dst_row0, int64_t dst_row_step,
                            cudaStream_t s);
// The same for Q4_K (columns whole 256-element super-blocks).
cudaError_t synth_fill_q4_k(uint64_t key, float stdv, int64_t cols, int64_t r0, int64_t nr, int64_t c0, int64_t nc,
                            uint8_t* dst, int64_t dst_row_bytes, int64_t dst_row0, int64_t dst_row_step,
                            cudaStream_t s);
// f32 rows [r0, r0+nr) (full rows) into dst.
cudaError_t synth_fill_f32(uint64_t key, float stdv, int64_t cols, int64_t r0, int64_t nr, float* dst,
                           cudaStream_t s);
cudaError_t fill_f32(float* dst, int64_t n, float v, cudaStream_t s);

}  // namespace jinf
