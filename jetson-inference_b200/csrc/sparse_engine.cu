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

#include <algorithm>

namespace jinf {

namespace {

constexpr int TOPK_THREADS = 1024;

__device__ __forceinline__ uint32_t order_key(float v) {
    const uint32_t b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// h = h_in + y_res (stored to h_out), x = h * rsqrt(mean(h^2) + eps) * gain. One CTA of 1024
// threads, d a multiple of 4 and at most 8192: each thread loads its (at most two) 16-byte
// pieces at once.
__global__ void __launch_bounds__(1024) k_ffn_prologue(const float* h_in, const float* y_res, float* h_out,
                                                       const float* gain, float eps, int d, float* x) {
    __shared__ float red[32];
    float4 h[2];
    float ss = 0.f;
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int i = 4 * (threadIdx.x + 1024 * u);
        if (i < d) {
            const float4 a = *reinterpret_cast<const float4*>(h_in + i), c = *reinterpret_cast<const float4*>(y_res + i);
            h[u] = make_float4(a.x + c.x, a.y + c.y, a.z + c.z, a.w + c.w);
            *reinterpret_cast<float4*>(h_out + i) = h[u];
            ss = fmaf(h[u].x, h[u].x, ss);
            ss = fmaf(h[u].y, h[u].y, ss);
            ss = fmaf(h[u].z, h[u].z, ss);
            ss = fmaf(h[u].w, h[u].w, ss);
        }
    }
    const float r = rsqrtf(block_sum(ss, red) / (float)d + eps);
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int i = 4 * (threadIdx.x + 1024 * u);
        if (i < d) {
            const float4 g = *reinterpret_cast<const float4*>(gain + i);
            *reinterpret_cast<float4*>(x + i) =
                make_float4(h[u].x * r * g.x, h[u].y * r * g.y, h[u].z * r * g.z, h[u].w * r * g.w);
        }
    }
}

// y[row] = W[row] . x (fp16 W [rows][cols], cols a multiple of 8, at most 8192), optionally
// ReLU. x is staged in shared memory once per CTA: read as is, or (NORM) computed in every
// CTA as RMSNorm(h_in + y_res) * gain, CTA 0 also storing h_out and x_out. A warp owns
// 16 / PL rows at a time, PL = 16-byte loads per lane per row (cols <= 256 * PL; PL = 32 walks
// a row in two passes), and issues all 16 loads before it uses any. fp32 sums in a fixed order.
struct NormArgs {
    const float* h_in;
    const float* y_res;
    float* h_out;
    const float* gain;
    float eps;
    float* x_out;
};

template <int PL, bool NORM>
__global__ void __launch_bounds__(256) k_gemv_f16(const __half* __restrict__ w, const float* __restrict__ x,
                                                  float* __restrict__ y, int rows, int cols, int relu, NormArgs na) {
    extern __shared__ float4 xs4[];
    __shared__ float red[32];
    const int tid = threadIdx.x, lane = tid & 31;
    const int n4 = cols >> 2;
    if (NORM) {
        float4 h[8];
        float ss = 0.f;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = tid + 256 * u;
            h[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (i < n4) {
                const float4 a = __ldg(reinterpret_cast<const float4*>(na.h_in) + i);
                const float4 c = __ldg(reinterpret_cast<const float4*>(na.y_res) + i);
                h[u] = make_float4(a.x + c.x, a.y + c.y, a.z + c.z, a.w + c.w);
                ss = fmaf(h[u].x, h[u].x, ss);
                ss = fmaf(h[u].y, h[u].y, ss);
                ss = fmaf(h[u].z, h[u].z, ss);
                ss = fmaf(h[u].w, h[u].w, ss);
            }
        }
        const float r = rsqrtf(block_sum(ss, red) / (float)cols + na.eps);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = tid + 256 * u;
            if (i < n4) {
                const float4 g = __ldg(reinterpret_cast<const float4*>(na.gain) + i);
                const float4 v = make_float4(h[u].x * r * g.x, h[u].y * r * g.y, h[u].z * r * g.z, h[u].w * r * g.w);
                xs4[i] = v;
                if (blockIdx.x == 0) {
                    reinterpret_cast<float4*>(na.h_out)[i] = h[u];
                    reinterpret_cast<float4*>(na.x_out)[i] = v;
                }
            }
        }
    } else {
        float4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = tid + 256 * u;
            v[u] = i < n4 ? __ldg(reinterpret_cast<const float4*>(x) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (tid + 256 * u < n4) xs4[tid + 256 * u] = v[u];
    }
    __syncthreads();
    constexpr int PLC = PL < 16 ? PL : 16;  // loads per row per pass
    constexpr int R = 16 / PLC;             // rows per warp
    const int n8 = cols >> 3;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    for (int r0 = ((blockIdx.x * blockDim.x + tid) >> 5) * R; r0 < rows; r0 += nwarps * R) {
        float acc[R];
#pragma unroll
        for (int j = 0; j < R; ++j) acc[j] = 0.f;
        for (int cb = 0; cb < n8; cb += 32 * PLC) {
            uint4 raw[16];
#pragma unroll
            for (int u = 0; u < 16; ++u) {
                const int row = r0 + u / PLC, c = cb + (u % PLC) * 32 + lane;
                raw[u] = row < rows && c < n8 ? ldg_stream_u4(w + (size_t)row * cols + 8 * (size_t)c)
                                              : make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
            for (int u = 0; u < 16; ++u) {
                const int c = cb + (u % PLC) * 32 + lane;
                if (c < n8) {
                    const __half2* h2 = reinterpret_cast<const __half2*>(&raw[u]);
                    const float4 xa = xs4[2 * c], xb = xs4[2 * c + 1];
                    const float2 f0 = __half22float2(h2[0]), f1 = __half22float2(h2[1]);
                    const float2 f2 = __half22float2(h2[2]), f3 = __half22float2(h2[3]);
                    float a = acc[u / PLC];
                    a = fmaf(f0.x, xa.x, a);
                    a = fmaf(f0.y, xa.y, a);
                    a = fmaf(f1.x, xa.z, a);
                    a = fmaf(f1.y, xa.w, a);
                    a = fmaf(f2.x, xb.x, a);
                    a = fmaf(f2.y, xb.y, a);
                    a = fmaf(f3.x, xb.z, a);
                    a = fmaf(f3.y, xb.w, a);
                    acc[u / PLC] = a;
                }
            }
        }
#pragma unroll
        for (int j = 0; j < R; ++j) {
            const float t = warp_sum(acc[j]);
            if (lane == 0 && r0 + j < rows) y[r0 + j] = relu && t < 0.f ? 0.f : t;
        }
    }
}

template <bool NORM>
cudaError_t launch_gemv_f16(const void* w, const float* x, float* y, int rows, int cols, int relu, const NormArgs& na,
                            cudaStream_t s) {
    const int pl = (cols / 8 + 31) / 32;
    const size_t smem = sizeof(float) * (size_t)cols;
    const int rpw = pl >= 16 ? 1 : 16 / (pl <= 1 ? 1 : pl <= 2 ? 2 : pl <= 4 ? 4 : pl <= 8 ? 8 : 16);
    const int64_t warps = (rows + rpw - 1) / rpw;
    const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>((warps + 7) / 8, 65535));
    const __half* wh = (const __half*)w;
#define JINF_GF16(P) k_gemv_f16<P, NORM><<<grid, 256, smem, s>>>(wh, x, y, rows, cols, relu, na)
    if (pl <= 1) JINF_GF16(1);
    else if (pl <= 2) JINF_GF16(2);
    else if (pl <= 4) JINF_GF16(4);
    else if (pl <= 8) JINF_GF16(8);
    else if (pl <= 16) JINF_GF16(16);
    else JINF_GF16(32);
#undef JINF_GF16
    return cudaGetLastError();
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
// offsets. One CTA with the ordered keys in shared memory: a 4-pass radix select finds the
// k-th largest key T, then one ordered compaction keeps every key > T and the first
// (k - #greater) keys == T. Each pass counts a 256-bin histogram in 32 lane-private copies
// (lane l adds to copy l, so the adds of one warp never meet on an address even when the
// scores crowd a few bins), sums the copies per bin, and one warp locates the bin that holds
// the k-th key with a suffix scan.
constexpr int TOPK_HIST_BYTES = 256 * 32 * 4;

__global__ void __launch_bounds__(TOPK_THREADS) k_topk(const float* __restrict__ s, int n, int k, int bundle_size,
                                                       int32_t* ids, int32_t* offsets) {
    extern __shared__ uint32_t dyn[];
    int* hist32 = reinterpret_cast<int*>(dyn);                 // [256 bins][32 lanes]
    uint32_t* keys = dyn + TOPK_HIST_BYTES / 4;                 // [n]
    __shared__ int hist[256];
    __shared__ int tmp[33];
    __shared__ uint32_t sel[2];  // prefix, remaining
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int i0 = tid; i0 < n; i0 += 8 * TOPK_THREADS) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = i0 + u * TOPK_THREADS;
            v[u] = i < n ? __ldg(s + i) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (i0 + u * TOPK_THREADS < n) keys[i0 + u * TOPK_THREADS] = order_key(v[u]);
    }
    if (tid == 0) {
        sel[0] = 0u;
        sel[1] = (uint32_t)k;
    }
    uint32_t mask = 0u;
    for (int pass = 0; pass < 4; ++pass) {
        const int shift = 24 - 8 * pass;
        for (int j = tid; j < 256 * 32; j += TOPK_THREADS) hist32[j] = 0;
        __syncthreads();
        const uint32_t prefix = sel[0];
        for (int i = tid; i < n; i += TOPK_THREADS) {
            const uint32_t key = keys[i];
            if ((key & mask) == prefix) atomicAdd(&hist32[((key >> shift) & 255) * 32 + lane], 1);
        }
        __syncthreads();
        // warp w sums bins 8w..8w+7 over the 32 copies
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int b = 8 * warp + j;
            int c = hist32[b * 32 + lane];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(JINF_FULL_MASK, c, o);
            if (lane == 0) hist[b] = c;
        }
        __syncthreads();
        if (tid < 32) {
            // lane l owns bins 8l..8l+7; above = number of keys in the bins of higher lanes
            int own = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) own += hist[8 * lane + j];
            int incl = own;  // inclusive suffix sum over lanes l..31
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int t = __shfl_down_sync(JINF_FULL_MASK, incl, o);
                if (lane + o < 32) incl += t;
            }
            const uint32_t rem = sel[1];
            uint32_t above = (uint32_t)(incl - own);
            if (above < rem && (uint32_t)incl >= rem) {
                int b = 8 * lane + 7;
                for (; b > 8 * lane; --b) {
                    if (above + (uint32_t)hist[b] >= rem) break;
                    above += (uint32_t)hist[b];
                }
                sel[0] = prefix | ((uint32_t)b << shift);
                sel[1] = rem - above;  // keys equal to the final prefix still to take (after the last pass)
            }
        }
        mask |= 255u << shift;
        __syncthreads();
    }
    const uint32_t T = sel[0], need_eq = sel[1];
    // contiguous chunk of indices per thread: ordered compaction
    const int per = (n + TOPK_THREADS - 1) / TOPK_THREADS;
    const int i0 = min(n, tid * per), i1 = min(n, i0 + per);
    int n_eq = 0;
    for (int i = i0; i < i1; ++i) n_eq += keys[i] == T;
    int tot;
    int eq_base = block_exclusive_scan(n_eq, tmp, tot);
    int n_sel = 0;
    {
        int e = eq_base;
        for (int i = i0; i < i1; ++i) {
            const uint32_t key = keys[i];
            if (key > T) ++n_sel;
            else if (key == T && (uint32_t)(e++) < need_eq) ++n_sel;
        }
    }
    int out = block_exclusive_scan(n_sel, tmp, tot);
    int e = eq_base;
    for (int i = i0; i < i1; ++i) {
        const uint32_t key = keys[i];
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

static cudaError_t launch_topk(const float* sc, int n_ff, int k, int bundle_size, int32_t* ids, int32_t* offsets,
                               cudaStream_t s) {
    const size_t smem = TOPK_HIST_BYTES + sizeof(uint32_t) * (size_t)n_ff;
    if (smem > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(k_topk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    k_topk<<<1, TOPK_THREADS, smem, s>>>(sc, n_ff, k, bundle_size, ids, offsets);
    return cudaGetLastError();
}

cudaError_t sparse_predict(const void* w1, const void* w2, const float* x, int d, int r, int n_ff, int k,
                           int bundle_size, int32_t* ids, int32_t* offsets, float* scratch, cudaStream_t s) {
    float* z = scratch;
    float* sc = scratch + r;
    const NormArgs none{};
    cudaError_t e = launch_gemv_f16<false>(w1, x, z, r, d, 1, none, s);
    if (e == cudaSuccess) e = launch_gemv_f16<false>(w2, z, sc, n_ff, r, 0, none, s);
    if (e == cudaSuccess) e = launch_topk(sc, n_ff, k, bundle_size, ids, offsets, s);
    return e;
}

cudaError_t sparse_predict_norm(const void* w1, const void* w2, const float* h_in, const float* y_res, float* h_out,
                                const float* gain, float eps, float* x, int d, int r, int n_ff, int k, int bundle_size,
                                int32_t* ids, int32_t* offsets, float* scratch, cudaStream_t s) {
    float* z = scratch;
    float* sc = scratch + r;
    const NormArgs na{h_in, y_res, h_out, gain, eps, x};
    const NormArgs none{};
    cudaError_t e = launch_gemv_f16<true>(w1, nullptr, z, r, d, 1, na, s);
    if (e == cudaSuccess) e = launch_gemv_f16<false>(w2, z, sc, n_ff, r, 0, none, s);
    if (e == cudaSuccess) e = launch_topk(sc, n_ff, k, bundle_size, ids, offsets, s);
    return e;
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
        d > 8192 || r > 8192 || n_ff <= 0 || n_ff > JINF_TOPK_MAX_N || k <= 0 || k > n_ff)
        return JINF_ERR_INVALID;
    return sparse_predict(w1, w2, x, d, r, n_ff, k, bundle_size, ids, offsets, scratch, stream) == cudaSuccess
               ? JINF_OK
               : JINF_ERR_CUDA;
}
