// Host interface of the engine's fp16-KV decode attention (attn_f16.cu).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>

#include "device_state.cuh"

namespace jinf {

struct MultiState;

struct AttnParams {
    const float* q;        // [n_heads * head_dim] fp32, RoPE applied
    const __half* kcache;  // this layer: [n_kv_heads][max_ctx][head_dim]
    const __half* vcache;
    float* out;            // [n_heads * head_dim]
    float* partial;        // attn_partial_floats(...) floats of scratch
    int n_heads, n_kv_heads, head_dim, max_ctx, n_split;
    DeviceState* st;       // positions 0..st->pos are attended
    // Multi-sequence step (multi.h), when ms is set: grid dimension y runs over the n_vec
    // vectors; vector v attends positions 0..ms->pos[v] of sequence ms->seq[v]'s cache (seq_stride
    // elements from sequence 0's), reads q + v q_stride, writes out + v q_stride, uses partial
    // floats [v][...] and the arrival counters ms->attn_count[v * 64 + kv head].
    MultiState* ms = nullptr;
    int n_vec = 1;
    size_t seq_stride = 0;
    int q_stride = 0;
};

size_t attn_partial_floats(int n_kv_heads, int n_split, int head_dim);
cudaError_t attn_launch(const AttnParams& p, cudaStream_t s, bool pdl);

}  // namespace jinf
