// Host interface of the engine's fp16-KV decode attention (attn_f16.cu).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>

#include "device_state.cuh"

namespace jinf {

struct AttnParams {
    const float* q;        // [n_heads * head_dim] fp32, RoPE applied
    const __half* kcache;  // this layer: [n_kv_heads][max_ctx][head_dim]
    const __half* vcache;
    float* out;            // [n_heads * head_dim]
    float* partial;        // attn_partial_floats(...) floats of scratch
    int n_heads, n_kv_heads, head_dim, max_ctx, n_split;
    DeviceState* st;       // positions 0..st->pos are attended
};

size_t attn_partial_floats(int n_kv_heads, int n_split, int head_dim);
cudaError_t attn_launch(const AttnParams& p, cudaStream_t s, bool pdl);

}  // namespace jinf
