// jinf_cuda_sparse_ffn: FFN over the neuron bundles of the active neurons
// (reference cuda/sparse_matmul.cu:223-282, bundle layout tools/prepare_model.cpp:299-308).
//
// Phase 1: one warp per active neuron computes silu(gate . x) * (up . x) for Q4_0, Q8_0,
//          Q4_K or Q6_K rows (each format decoded as itself).
// Phase 2: output[d] = sum_i a_i * down_col_i[d]. A cluster of 8 CTAs splits the active
//          list, each thread owns one output element, and the 8 partial sums are added in
//          rank order through distributed shared memory: deterministic, no atomics, no
//          memset, no scratch beyond the caller's gate_up_tmp.
#include "common.cuh"
#include "jinf/quant.h"
#include "jinf/sparse_ops.h"

#include <cooperative_groups.h>

namespace cg = cooperative_groups;

__device__ __forceinline__ uint32_t ld_u16(const uint8_t* p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8); }

// Dot product of one quantized row (hidden_dim weights) with x; result in every lane.
__device__ float warp_row_dot(const uint8_t* row, int qtype, const float* __restrict__ x, int n) {
    const int lane = threadIdx.x & 31;
    float acc = 0.f;
    if (qtype == JINF_TYPE_Q4_0 || qtype == JINF_TYPE_Q8_0) {
        const int bb = qtype == JINF_TYPE_Q4_0 ? 18 : 34;
        for (int b = lane; b < n / 32; b += 32) {
            const uint8_t* blk = row + (size_t)b * bb;
            const float d = jinf_h2f((uint16_t)ld_u16(blk));
            float s = 0.f;
            if (qtype == JINF_TYPE_Q4_0) {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const uint32_t v = blk[2 + i];
                    s = fmaf((float)((int)(v & 15) - 8), __ldg(x + 32 * b + 2 * i), s);
                    s = fmaf((float)((int)(v >> 4) - 8), __ldg(x + 32 * b + 2 * i + 1), s);
                }
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) s = fmaf((float)(int8_t)blk[2 + i], __ldg(x + 32 * b + i), s);
            }
            acc = fmaf(s, d, acc);
        }
    } else if (qtype == JINF_TYPE_Q4_K) {
        const int j = lane >> 2;
        for (int b = 0; b < n / 256; ++b) {
            const jinf_block_q4_K* blk = reinterpret_cast<const jinf_block_q4_K*>(row + (size_t)b * 144);
            int sc, mn;
            q4k_scale_min_dev(blk->scales, j, sc, mn);
            const float sd = __fmul_rn(jinf_h2f(blk->d), (float)sc), smn = __fmul_rn(jinf_h2f(blk->dmin), (float)mn);
            const uint8_t* q = blk->qs + 16 * j + 4 * (lane & 3);
            const float* xb = x + 256 * b + 8 * lane;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                acc = fmaf(__fsub_rn(__fmul_rn(sd, (float)(q[i] & 15)), smn), __ldg(xb + 2 * i), acc);
                acc = fmaf(__fsub_rn(__fmul_rn(sd, (float)(q[i] >> 4)), smn), __ldg(xb + 2 * i + 1), acc);
            }
        }
    } else {  // Q6_K
        for (int b = 0; b < n / 256; ++b) {
            const uint8_t* blk = row + (size_t)b * 210;
            const float d = jinf_h2f((uint16_t)ld_u16(blk + 208));
            const int e0 = 8 * lane;
            const float s = __fmul_rn(d, (float)(int8_t)blk[192 + (e0 >> 4)]);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int e = e0 + i;
                const int lo = (blk[e >> 1] >> ((e & 1) * 4)) & 15;
                const int hi = (blk[128 + (e >> 2)] >> (2 * (e & 3))) & 3;
                acc = fmaf(__fmul_rn(s, (float)((lo | (hi << 4)) - 32)), __ldg(x + 256 * b + e), acc);
            }
        }
    }
    return warp_sum(acc);
}

__global__ void k_sparse_gate_up(const uint8_t* __restrict__ bundles, const float* __restrict__ x,
                                 float* __restrict__ gu, const int* __restrict__ offs, int n_act, int hidden,
                                 int row_bytes, int qtype) {
    const int i = (int)(((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    if (i >= n_act) return;
    const uint8_t* b = bundles + offs[i];
    const float g = warp_row_dot(b, qtype, x, hidden);
    const float u = warp_row_dot(b + row_bytes, qtype, x, hidden);
    if ((threadIdx.x & 31) == 0) gu[i] = g / (1.0f + expf(-g)) * u;
}

constexpr int SP_CLUSTER = 8;

__global__ void __launch_bounds__(256) k_sparse_down(const uint8_t* __restrict__ bundles, float* __restrict__ out,
                                                     const float* __restrict__ gu, const int* __restrict__ offs,
                                                     int n_act, int hidden, int down_off) {
    cg::cluster_group cluster = cg::this_cluster();
    __shared__ float part[256];
    const int rank = (int)cluster.block_rank();
    const int chunk = blockIdx.x / SP_CLUSTER;
    const int d = chunk * 256 + threadIdx.x;
    const int i0 = (int)((int64_t)n_act * rank / SP_CLUSTER), i1 = (int)((int64_t)n_act * (rank + 1) / SP_CLUSTER);
    float acc = 0.f;
    if (d < hidden) {
        for (int i = i0; i < i1; ++i) {
            const float* col = reinterpret_cast<const float*>(bundles + offs[i] + down_off);
            acc = fmaf(__ldg(gu + i), __ldg(col + d), acc);
        }
    }
    part[threadIdx.x] = acc;
    cluster.sync();
    if (rank == 0 && d < hidden) {
        float s = 0.f;
        for (int r = 0; r < SP_CLUSTER; ++r) s += cluster.map_shared_rank(part, r)[threadIdx.x];
        out[d] = s;
    }
    cluster.sync();
}

extern "C" void jinf_cuda_sparse_ffn(const void* bundles, const float* input, float* output,
                                     const int* bundle_offsets, int num_activated, int hidden_dim,
                                     int bundle_size, int qtype, float* gate_up_tmp, cudaStream_t stream) {
    (void)bundle_size;  // offsets are explicit; the size only bounds them on the caller side
    if (hidden_dim <= 0) return;
    const int bs = jinf_qtype_block_size((jinf_qtype)qtype);
    if (qtype != JINF_TYPE_Q4_0 && qtype != JINF_TYPE_Q8_0 && qtype != JINF_TYPE_Q4_K && qtype != JINF_TYPE_Q6_K) {
        jinf_record_error(JINF_ERR_INVALID, "sparse_ffn: unsupported qtype");
        return;
    }
    if (hidden_dim % bs) {
        jinf_record_error(JINF_ERR_INVALID, "sparse_ffn: hidden_dim not a multiple of the block size");
        return;
    }
    const int row_bytes = (int)((size_t)(hidden_dim / bs) * jinf_qtype_type_size((jinf_qtype)qtype));
    if (num_activated <= 0) {
        // No active neuron: the FFN contributes nothing.
        cudaMemsetAsync(output, 0, sizeof(float) * (size_t)hidden_dim, stream);
        return;
    }
    const int64_t threads = (int64_t)num_activated * 32;
    k_sparse_gate_up<<<(unsigned)((threads + 255) / 256), 256, 0, stream>>>(
        (const uint8_t*)bundles, input, gate_up_tmp, bundle_offsets, num_activated, hidden_dim, row_bytes, qtype);
    jinf_check_launch("sparse_ffn gate_up");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(((hidden_dim + 255) / 256) * SP_CLUSTER);
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = SP_CLUSTER;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, k_sparse_down, (const uint8_t*)bundles, output, (const float*)gate_up_tmp,
                           bundle_offsets, num_activated, hidden_dim, 2 * row_bytes) != cudaSuccess)
        jinf_record_error(JINF_ERR_CUDA, "sparse_ffn down: launch");
}
