// Sparse FFN mode of the engine (reference src/engine.cpp:339-415 forward_layer_sparse_ffn,
// src/activation_predictor.cpp): the FFN of a layer runs over its active neurons only,
// through the neuron bundles of reference tools/prepare_model.cpp:299-308 and the bundle
// kernel jinf_cuda_sparse_ffn (abi_sparse.cu).
//
// Active neurons come from
//   - a fixed mask (jinf_sparse_fixed_mask): runs of 8 consecutive neurons, each run kept
//     with probability `keep` (seeded) — the reference's static predictor with a synthetic
//     profile; or
//   - a predictor on the device: x = RMSNorm(h) * ffn_norm, z = ReLU(W1 x) (W1 fp16
//     [r][d]), s = W2 z (W2 fp16 [n_ff][r]), the k = floor(keep * n_ff) largest scores (ties:
//     lower index first), ids ascending. The reference ran its predictor on the host and
//     copied the hidden state over every layer (src/engine.cpp:350-358); here it never
//     leaves the GPU.
#include "common.cuh"
#include "jinf/b200.h"
#include "jinf/quant.h"
#include "jinf/sparse_ops.h"
#include "sparse_engine.h"
#include "synth_math.h"

#include <math.h>

namespace jinf {

namespace {

constexpr int TOPK_THREADS = 1024;

__device__ __forceinline__ uint32_t order_key(float v) {
    const uint32_t b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// h = h_in + y_res (stored to h_out), x = h * rsqrt(mean(h^2) + eps) * gain. One CTA.
__global__ void __launch_bounds__(1024) k_ffn_prologue(const float* h_in, const float* y_res, float* h_out,
                                                       const float* gain, float eps, int d, float* x) {
    __shared__ float red[32];
    float ss = 0.f;
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        const float h = h_in[i] + y_res[i];
        h_out[i] = h;
        ss = fmaf(h, h, ss);
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        v = warp_sum(v);
        if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    const float r = rsqrtf(red[0] / (float)d + eps);
    for (int i = threadIdx.x; i < d; i += blockDim.x) x[i] = h_out[i] * r * gain[i];
}

// y[row] = W[row] . x (fp16 W [rows][cols], cols a multiple of 256), optionally ReLU. A warp
// per row, eight halves per 16-byte load, fp32 sums in a fixed order.
__global__ void k_gemv_f16(const __half* __restrict__ w, const float* __restrict__ x, float* __restrict__ y, int rows,
                           int cols, int relu) {
    const int lane = threadIdx.x & 31;
    const int warps = (gridDim.x * blockDim.x) >> 5;
    for (int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < rows; row += warps) {
        const uint4* wr = reinterpret_cast<const uint4*>(w + (size_t)row * cols);
        float acc = 0.f;
        for (int c = lane; c < cols / 8; c += 32) {
            const uint4 raw = __ldg(wr + c);
            const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
            const float4 xa = __ldg(reinterpret_cast<const float4*>(x) + 2 * c);
            const float4 xb = __ldg(reinterpret_cast<const float4*>(x) + 2 * c + 1);
            const float2 f0 = __half22float2(h2[0]), f1 = __half22float2(h2[1]);
            const float2 f2 = __half22float2(h2[2]), f3 = __half22float2(h2[3]);
            acc = fmaf(f0.x, xa.x, acc);
            acc = fmaf(f0.y, xa.y, acc);
            acc = fmaf(f1.x, xa.z, acc);
            acc = fmaf(f1.y, xa.w, acc);
            acc = fmaf(f2.x, xb.x, acc);
            acc = fmaf(f2.y, xb.y, acc);
            acc = fmaf(f3.x, xb.z, acc);
            acc = fmaf(f3.y, xb.w, acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) y[row] = relu && acc < 0.f ? 0.f : acc;
    }
}

// Block-wide exclusive prefix sum of one value per thread (TOPK_THREADS threads).
__device__ int block_exclusive_scan(int v, int* tmp, int& total) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(JINF_FULL_MASK, incl, o);
        if (lane >= o) incl += t;
    }
    if (lane == 31) tmp[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        int w = tmp[lane];
        int wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(JINF_FULL_MASK, wi, o);
            if (lane >= o) wi += t;
        }
        tmp[lane] = wi - w;  // exclusive per warp
        if (lane == 31) tmp[32] = wi;
    }
    __syncthreads();
    const int r = tmp[warp] + incl - v;
    total = tmp[32];
    __syncthreads();
    return r;
}

// The k largest of s[0..n) (ties: lower index first), ids ascending, and their bundle byte
// offsets. One CTA: a 4-pass radix select on the ordered keys finds the k-th largest key T,
// then one ordered compaction keeps every key > T and the first (k - #greater) keys == T.
__global__ void __launch_bounds__(TOPK_THREADS) k_topk(const float* __restrict__ s, int n, int k, int bundle_size,
                                                       int32_t* ids, int32_t* offsets) {
    __shared__ int hist[256];
    __shared__ int tmp[33];
    __shared__ uint32_t sel[2];  // prefix, remaining
    const int tid = threadIdx.x;
    if (tid == 0) {
        sel[0] = 0u;
        sel[1] = (uint32_t)k;
    }
    uint32_t mask = 0u;
    for (int pass = 0; pass < 4; ++pass) {
        const int shift = 24 - 8 * pass;
        if (tid < 256) hist[tid] = 0;
        __syncthreads();
        const uint32_t prefix = sel[0];
        for (int i = tid; i < n; i += TOPK_THREADS) {
            const uint32_t key = order_key(s[i]);
            if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255], 1);
        }
        __syncthreads();
        if (tid == 0) {
            uint32_t rem = sel[1];
            int b = 255;
            for (; b > 0; --b) {
                if ((uint32_t)hist[b] >= rem) break;
                rem -= (uint32_t)hist[b];
            }
            sel[0] = prefix | ((uint32_t)b << shift);
            sel[1] = rem;  // how many keys equal to the final prefix still to take (after the last pass)
        }
        mask |= 255u << shift;
        __syncthreads();
    }
    const uint32_t T = sel[0], need_eq = sel[1];
    // contiguous chunk of indices per thread: ordered compaction
    const int per = (n + TOPK_THREADS - 1) / TOPK_THREADS;
    const int i0 = tid * per, i1 = min(n, i0 + per);
    int n_eq = 0;
    for (int i = i0; i < i1; ++i) n_eq += order_key(s[i]) == T;
    int tot;
    int eq_base = block_exclusive_scan(n_eq, tmp, tot);
    int n_sel = 0;
    {
        int e = eq_base;
        for (int i = i0; i < i1; ++i) {
            const uint32_t key = order_key(s[i]);
            if (key > T) ++n_sel;
            else if (key == T && (uint32_t)(e++) < need_eq) ++n_sel;
        }
    }
    int out = block_exclusive_scan(n_sel, tmp, tot);
    int e = eq_base;
    for (int i = i0; i < i1; ++i) {
        const uint32_t key = order_key(s[i]);
        const bool take = key > T || (key == T && (uint32_t)(e++) < need_eq);
        if (take) {
            ids[out] = i;
            offsets[out] = i * bundle_size;
            ++out;
        }
    }
}

// Bundle gate/up rows: AoS rows of the gate|up matrix as staged for the Q4M repack (rows
// interleaved gate_n, up_n; `row_bytes` each) -> bundle n bytes [0, 2 row_bytes).
__global__ void k_bundle_gate_up(const uint8_t* __restrict__ gu, int n_ff, int row_bytes, uint8_t* __restrict__ bundles,
                                 int bundle_size) {
    const int64_t total = (int64_t)n_ff * 2 * row_bytes;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = i / (2 * row_bytes), r = i % (2 * row_bytes);
        bundles[n * bundle_size + r] = gu[i];  // staged row 2n = gate_n, 2n+1 = up_n: contiguous
    }
}

// Bundle down columns: the AoS down matrix [d][n_ff] (Q4_0 or Q4_K) dequantized exactly as
// the reference does (src/quant.cpp:49-93) into fp32 column n of bundle n.
__global__ void k_bundle_down(const uint8_t* __restrict__ down, int d, int n_ff, int qtype, uint8_t* __restrict__ bundles,
                              int bundle_size, int col_off) {
    const int64_t total = (int64_t)d * n_ff;
    const int bs = qtype == JINF_TYPE_Q4_K ? 256 : 32, bb = qtype == JINF_TYPE_Q4_K ? 144 : 18;
    const int64_t row_bytes = (int64_t)(n_ff / bs) * bb;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int row = (int)(i / n_ff), n = (int)(i % n_ff);
        const uint8_t* blk = down + (int64_t)row * row_bytes + (int64_t)(n / bs) * bb;
        const int e = n % bs;
        float v;
        if (qtype == JINF_TYPE_Q4_K) {
            const jinf_block_q4_K* b = reinterpret_cast<const jinf_block_q4_K*>(blk);
            int sc, mn;
            q4k_scale_min_dev(b->scales, e / 32, sc, mn);
            const uint8_t byte = b->qs[(e / 32) * 16 + (e % 32) / 2];
            const int q = (e & 1) ? (byte >> 4) : (byte & 15);
            v = __fsub_rn(__fmul_rn(__fmul_rn(jinf_h2f(b->d), (float)sc), (float)q),
                          __fmul_rn(jinf_h2f(b->dmin), (float)mn));
        } else {
            const float dd = jinf_h2f((uint16_t)(blk[0] | (blk[1] << 8)));
            const uint8_t byte = blk[2 + e / 2];
            const int q = (e & 1) ? (byte >> 4) : (byte & 15);
            v = __fmul_rn((float)(q - 8), dd);
        }
        reinterpret_cast<float*>(bundles + (int64_t)n * bundle_size + col_off)[row] = v;
    }
}

// Seeded N(0, std) fp16 values (synth_math.h: the same bits as the host generator).
__global__ void k_fill_f16_normal(uint64_t key, float stdv, int64_t n, __half* dst) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = __ushort_as_half(jinf_synth::fp32_to_fp16(jinf_synth::normal_at(key, (uint64_t)i, stdv)));
}

unsigned grid_for(int64_t n, int threads) {
    const int64_t g = (n + threads - 1) / threads;
    return (unsigned)(g < 65536 ? (g > 0 ? g : 1) : 65536);
}

}  // namespace

cudaError_t sparse_ffn_prologue(const float* h_in, const float* y_res, float* h_out, const float* gain, float eps,
                                int d, float* x, cudaStream_t s) {
    k_ffn_prologue<<<1, 1024, 0, s>>>(h_in, y_res, h_out, gain, eps, d, x);
    return cudaGetLastError();
}

cudaError_t sparse_predict(const void* w1, const void* w2, const float* x, int d, int r, int n_ff, int k,
                           int bundle_size, int32_t* ids, int32_t* offsets, float* scratch, cudaStream_t s) {
    float* z = scratch;
    float* sc = scratch + r;
    k_gemv_f16<<<grid_for((int64_t)r * 32, 256), 256, 0, s>>>((const __half*)w1, x, z, r, d, 1);
    k_gemv_f16<<<grid_for((int64_t)n_ff * 32, 256), 256, 0, s>>>((const __half*)w2, z, sc, n_ff, r, 0);
    k_topk<<<1, TOPK_THREADS, 0, s>>>(sc, n_ff, k, bundle_size, ids, offsets);
    return cudaGetLastError();
}

cudaError_t sparse_bundle_gate_up(const uint8_t* gu_aos, int n_ff, int row_bytes, uint8_t* bundles, int bundle_size,
                                  cudaStream_t s) {
    k_bundle_gate_up<<<grid_for((int64_t)n_ff * 2 * row_bytes, 256), 256, 0, s>>>(gu_aos, n_ff, row_bytes, bundles,
                                                                                  bundle_size);
    return cudaGetLastError();
}

cudaError_t sparse_bundle_down(const uint8_t* down_aos, int d, int n_ff, int qtype, uint8_t* bundles, int bundle_size,
                               int col_off, cudaStream_t s) {
    k_bundle_down<<<grid_for((int64_t)d * n_ff, 256), 256, 0, s>>>(down_aos, d, n_ff, qtype, bundles, bundle_size,
                                                                   col_off);
    return cudaGetLastError();
}

cudaError_t sparse_fill_predictor(uint64_t seed, int layer, int which, int64_t n, void* dst, cudaStream_t s) {
    k_fill_f16_normal<<<grid_for(n, 256), 256, 0, s>>>(jinf_synth::predictor_key(seed, layer, which), 0.02f, n,
                                                       (__half*)dst);
    return cudaGetLastError();
}

int sparse_bundle_bytes(int d, int qtype) {
    const int bs = qtype == JINF_TYPE_Q4_K ? 256 : 32, bb = qtype == JINF_TYPE_Q4_K ? 144 : 18;
    const int raw = 2 * (d / bs) * bb + 4 * d;
    return (raw + 255) & ~255;
}

}  // namespace jinf

using namespace jinf;

extern "C" jinf_status jinf_b200_sparse_predict(const void* w1, const void* w2, const float* x, int d, int r, int n_ff,
                                                int k, int bundle_size, int32_t* ids, int32_t* offsets,
                                                float* scratch, cudaStream_t stream) {
    if (!w1 || !w2 || !x || !ids || !offsets || !scratch || d <= 0 || d % 8 || r <= 0 || r % 8 ||
        n_ff <= 0 || k <= 0 || k > n_ff)
        return JINF_ERR_INVALID;
    return sparse_predict(w1, w2, x, d, r, n_ff, k, bundle_size, ids, offsets, scratch, stream) == cudaSuccess
               ? JINF_OK
               : JINF_ERR_CUDA;
}
