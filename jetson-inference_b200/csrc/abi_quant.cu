// Drop-in kernels on the reference's array-of-structs quant blocks:
//   jinf_cuda_dequantize_{q4_0,q4_K,q8_0,q6_K}   (reference cuda/dequant_kernels.cu)
//   jinf_cuda_dequant_matvec, jinf_cuda_residual_add (reference cuda/matmul_kernels.cu)
//
// Dequantized values are bit-exact with the host dequantizer: Q4_0/Q8_0 are a single
// product; Q4_K rounds d*sc, then sc_d*q and the difference separately
// (__fmul_rn / __fsub_rn keep nvcc from contracting them into an FMA).
//
// The matvec kernels stage the rows a CTA owns in shared memory with the widest
// aligned global loads available (the 18-byte Q4_0 / 34-byte Q8_0 blocks are not
// 16-byte aligned in general), then one warp reduces one row.
#include "common.cuh"
#include "jinf/kernels.h"
#include "jinf/quant.h"

#include <atomic>
#include <stdio.h>

static std::atomic<int> g_last_error{0};

void jinf_record_error(int status, const char* what) {
    int expected = 0;
    g_last_error.compare_exchange_strong(expected, status);
    fprintf(stderr, "[jinf] %s: %s\n", what, jinf_status_str((jinf_status)status));
}

void jinf_check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        int expected = 0;
        g_last_error.compare_exchange_strong(expected, (int)JINF_ERR_CUDA);
        fprintf(stderr, "[jinf] %s: launch failed: %s\n", what, cudaGetErrorString(e));
    }
}

extern "C" int jinf_cuda_last_error(void) { return g_last_error.exchange(0); }

// ---------------------------------------------------------------- dequantize

// Store 8 floats; VEC requires a 16-byte aligned destination.
template <bool VEC>
__device__ __forceinline__ void store8(float* o, const float* v) {
    if (VEC) {
        reinterpret_cast<float4*>(o)[0] = make_float4(v[0], v[1], v[2], v[3]);
        reinterpret_cast<float4*>(o)[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = v[i];
    }
}

// One thread per 8 outputs; a warp covers 8 consecutive Q4_0 blocks and writes 1 KB
// contiguously.
template <bool VEC>
__global__ void k_dequant_q4_0(const uint8_t* __restrict__ blocks, float* __restrict__ out, int n_blocks) {
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t b = g >> 2;
    const int part = (int)(g & 3);
    if (b >= n_blocks) return;
    const uint8_t* blk = blocks + b * 18;
    const float d = jinf_h2f((uint16_t)(blk[0] | (blk[1] << 8)));
    const uint8_t* q = blk + 2 + 4 * part;
    float v[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        v[2 * i] = (float)((int)(q[i] & 15) - 8) * d;
        v[2 * i + 1] = (float)((int)(q[i] >> 4) - 8) * d;
    }
    store8<VEC>(out + b * 32 + 8 * part, v);
}

// One warp per 256-weight Q4_K super-block; lane = 8 consecutive outputs.
template <bool VEC>
__global__ void k_dequant_q4_K(const jinf_block_q4_K* __restrict__ blocks, float* __restrict__ out, int n_blocks) {
    const int64_t b = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (b >= n_blocks) return;
    const jinf_block_q4_K* blk = blocks + b;
    const int j = lane >> 2;
    int sc, mn;
    q4k_scale_min_dev(blk->scales, j, sc, mn);
    const float d = jinf_h2f(blk->d), dmin = jinf_h2f(blk->dmin);
    const float sd = __fmul_rn(d, (float)sc), sm = __fmul_rn(dmin, (float)mn);
    const uint8_t* qb = blk->qs + 16 * j + 4 * (lane & 3);
    const uint32_t q = (uint32_t)qb[0] | ((uint32_t)qb[1] << 8) | ((uint32_t)qb[2] << 16) | ((uint32_t)qb[3] << 24);
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __fsub_rn(__fmul_rn(sd, (float)((q >> (4 * i)) & 15)), sm);
    store8<VEC>(out + b * 256 + 8 * lane, v);
}

template <bool VEC>
__global__ void k_dequant_q8_0(const uint8_t* __restrict__ blocks, float* __restrict__ out, int n_blocks) {
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t b = g >> 2;
    const int part = (int)(g & 3);
    if (b >= n_blocks) return;
    const uint8_t* blk = blocks + b * 34;
    const float d = jinf_h2f((uint16_t)(blk[0] | (blk[1] << 8)));
    const int8_t* q = reinterpret_cast<const int8_t*>(blk + 2 + 8 * part);
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = (float)q[i] * d;
    store8<VEC>(out + b * 32 + 8 * part, v);
}

template <bool VEC>
__global__ void k_dequant_q6_K(const uint8_t* __restrict__ blocks, float* __restrict__ out, int n_blocks) {
    const int64_t b = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (b >= n_blocks) return;
    const jinf_block_q6_K* blk = reinterpret_cast<const jinf_block_q6_K*>(blocks + b * 210);
    const float d = jinf_h2f((uint16_t)(((const uint8_t*)&blk->d)[0] | (((const uint8_t*)&blk->d)[1] << 8)));
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int e = 8 * lane + i;
        const int lo = (blk->ql[e >> 1] >> ((e & 1) * 4)) & 15;
        const int hi = (blk->qh[e >> 2] >> (2 * (e & 3))) & 3;
        v[i] = __fmul_rn(__fmul_rn(d, (float)blk->scales[e >> 4]), (float)((lo | (hi << 4)) - 32));
    }
    store8<VEC>(out + b * 256 + 8 * lane, v);
}

extern "C" void jinf_cuda_dequantize_q4_0(const void* data, float* output, int n_blocks, cudaStream_t stream) {
    if (n_blocks <= 0) return;
    const int64_t threads = (int64_t)n_blocks * 4;
    const unsigned grid = (unsigned)((threads + 255) / 256);
    if (((uintptr_t)output & 15) == 0) k_dequant_q4_0<true><<<grid, 256, 0, stream>>>((const uint8_t*)data, output, n_blocks);
    else k_dequant_q4_0<false><<<grid, 256, 0, stream>>>((const uint8_t*)data, output, n_blocks);
    jinf_check_launch("dequantize_q4_0");
}

extern "C" void jinf_cuda_dequantize_q4_K(const void* data, float* output, int n_blocks, cudaStream_t stream) {
    if (n_blocks <= 0) return;
    const int64_t threads = (int64_t)n_blocks * 32;
    const unsigned grid = (unsigned)((threads + 255) / 256);
    if (((uintptr_t)output & 15) == 0) k_dequant_q4_K<true><<<grid, 256, 0, stream>>>((const jinf_block_q4_K*)data, output, n_blocks);
    else k_dequant_q4_K<false><<<grid, 256, 0, stream>>>((const jinf_block_q4_K*)data, output, n_blocks);
    jinf_check_launch("dequantize_q4_K");
}

extern "C" void jinf_cuda_dequantize_q8_0(const void* data, float* output, int n_blocks, cudaStream_t stream) {
    if (n_blocks <= 0) return;
    const int64_t threads = (int64_t)n_blocks * 4;
    const unsigned grid = (unsigned)((threads + 255) / 256);
    if (((uintptr_t)output & 15) == 0) k_dequant_q8_0<true><<<grid, 256, 0, stream>>>((const uint8_t*)data, output, n_blocks);
    else k_dequant_q8_0<false><<<grid, 256, 0, stream>>>((const uint8_t*)data, output, n_blocks);
    jinf_check_launch("dequantize_q8_0");
}

extern "C" void jinf_cuda_dequantize_q6_K(const void* data, float* output, int n_blocks, cudaStream_t stream) {
    if (n_blocks <= 0) return;
    const int64_t threads = (int64_t)n_blocks * 32;
    const unsigned grid = (unsigned)((threads + 255) / 256);
    if (((uintptr_t)output & 15) == 0) k_dequant_q6_K<true><<<grid, 256, 0, stream>>>((const uint8_t*)data, output, n_blocks);
    else k_dequant_q6_K<false><<<grid, 256, 0, stream>>>((const uint8_t*)data, output, n_blocks);
    jinf_check_launch("dequantize_q6_K");
}

// ---------------------------------------------------------------- matvec (AoS)

// Copy `n` bytes global -> shared with 16-, 4- or 2-byte loads depending on alignment.
__device__ __forceinline__ void stage_bytes(uint8_t* dst, const uint8_t* src, size_t n) {
    const uintptr_t a = (uintptr_t)src;
    if ((a & 15) == 0 && (n & 15) == 0) {
        const uint4* s = reinterpret_cast<const uint4*>(src);
        uint4* d = reinterpret_cast<uint4*>(dst);
        for (size_t i = threadIdx.x; i < n / 16; i += blockDim.x) d[i] = ldg_stream_u4(s + i);
    } else if ((a & 3) == 0 && (n & 3) == 0) {
        const uint32_t* s = reinterpret_cast<const uint32_t*>(src);
        uint32_t* d = reinterpret_cast<uint32_t*>(dst);
        for (size_t i = threadIdx.x; i < n / 4; i += blockDim.x) d[i] = ldg_stream_u1(s + i);
    } else if ((a & 1) == 0 && (n & 1) == 0) {
        const uint16_t* s = reinterpret_cast<const uint16_t*>(src);
        uint16_t* d = reinterpret_cast<uint16_t*>(dst);
        for (size_t i = threadIdx.x; i < n / 2; i += blockDim.x) d[i] = __ldg(s + i);
    } else {
        for (size_t i = threadIdx.x; i < n; i += blockDim.x) dst[i] = __ldg(src + i);
    }
}

// Bytes [off, off+16) of a shared buffer whose start is 16-byte aligned, `off` even: four
// aligned word reads (five and a funnel shift when off % 4 == 2).
__device__ __forceinline__ void smem_16B(const uint8_t* base, int off, uint32_t q[4]) {
    const uint32_t* w = reinterpret_cast<const uint32_t*>(base + (off & ~3));
    if ((off & 3) == 0) {
#pragma unroll
        for (int i = 0; i < 4; ++i) q[i] = w[i];
    } else {
        uint32_t t[5];
#pragma unroll
        for (int i = 0; i < 5; ++i) t[i] = w[i];
#pragma unroll
        for (int i = 0; i < 4; ++i) q[i] = __funnelshift_r(t[i], t[i + 1], 16);
    }
}

__device__ __forceinline__ float dot8_q4(uint32_t q, const float* x, float bias) {
    // sum over 8 nibbles (element k at bits 4k) of (nib + bias) * x[k]
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) s = fmaf((float)((q >> (4 * k)) & 15) + bias, x[k], s);
    return s;
}

constexpr int MV_THREADS = 256;

// 8 consecutive floats; VEC requires a 16-byte aligned address.
template <bool VEC>
__device__ __forceinline__ void load_x8(const float* p, float* o) {
    if (VEC) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(p)), c = __ldg(reinterpret_cast<const float4*>(p) + 1);
        o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w; o[4] = c.x; o[5] = c.y; o[6] = c.z; o[7] = c.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = __ldg(p + i);
    }
}

__device__ __forceinline__ uint32_t load_u32_any(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

// Q4_0 / Q8_0: CTA stages `rows_per_cta` rows (each `row_bytes`) in shared memory; warp w
// reduces rows w, w+8, ...
template <int QT, bool VEC>
__global__ void __launch_bounds__(MV_THREADS) k_matvec_small_blocks(const uint8_t* __restrict__ W,
                                                                    const float* __restrict__ x,
                                                                    float* __restrict__ y, int rows, int cols,
                                                                    int rows_per_cta) {
    extern __shared__ __align__(16) uint8_t sm[];
    constexpr int BB = QT == JINF_TYPE_Q4_0 ? 18 : 34;
    const int nb = cols / 32;
    const size_t row_bytes = (size_t)nb * BB;
    const int r0 = blockIdx.x * rows_per_cta;
    const int nr = min(rows_per_cta, rows - r0);
    stage_bytes(sm, W + (size_t)r0 * row_bytes, row_bytes * nr);
    __syncthreads();
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    for (int r = wid; r < nr; r += MV_THREADS / 32) {
        // Offsets are taken from the (16-byte aligned) start of the staged rows: a row
        // itself starts at r * row_bytes, which is only 2-byte aligned for odd nb.
        const int rbase = (int)((size_t)r * row_bytes);
        float acc = 0.f;
        for (int b = lane; b < nb; b += 32) {
            const int off = rbase + b * BB;
            const float d = jinf_h2f(*reinterpret_cast<const uint16_t*>(sm + off));
            const float* xb = x + 32 * b;
            float s = 0.f;
            if (QT == JINF_TYPE_Q4_0) {
                uint32_t q[4];
                smem_16B(sm, off + 2, q);
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                    float xs[8];
                    load_x8<VEC>(xb + 8 * w, xs);
                    s += dot8_q4(q[w], xs, -8.f);
                }
            } else {
                uint32_t q[8];
                smem_16B(sm, off + 2, q);
                smem_16B(sm, off + 18, q + 4);
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                    float xs[8];
                    load_x8<VEC>(xb + 8 * w, xs);
#pragma unroll
                    for (int k = 0; k < 8; ++k)
                        s = fmaf((float)(int8_t)(q[2 * w + (k >> 2)] >> (8 * (k & 3))), xs[k], s);
                }
            }
            acc = fmaf(s, d, acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) y[r0 + r] = acc;
    }
}

// Q4_K: super-blocks are 144 bytes (16-byte multiples), read straight from global.
// Warp per row; lane = 8 weights of one super-block per step.
template <bool ALIGNED, bool VEC>
__global__ void __launch_bounds__(MV_THREADS) k_matvec_q4_K(const jinf_block_q4_K* __restrict__ W,
                                                            const float* __restrict__ x,
                                                            float* __restrict__ y, int rows, int cols) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * (MV_THREADS / 32) + (threadIdx.x >> 5);
    if (row >= rows) return;
    const int nb = cols / 256;
    const jinf_block_q4_K* rb = W + (size_t)row * nb;
    const int j = lane >> 2;
    float acc = 0.f;
    for (int b = 0; b < nb; ++b) {
        const jinf_block_q4_K* blk = rb + b;
        uint4 head;  // d, dmin, scales[12]
        uint32_t q;
        if (ALIGNED) {
            head = __ldg(reinterpret_cast<const uint4*>(blk));
            q = ldg_stream_u1(blk->qs + 16 * j + 4 * (lane & 3));
        } else {
            const uint8_t* hb = reinterpret_cast<const uint8_t*>(blk);
            head = make_uint4(load_u32_any(hb), load_u32_any(hb + 4), load_u32_any(hb + 8), load_u32_any(hb + 12));
            q = load_u32_any(blk->qs + 16 * j + 4 * (lane & 3));
        }
        const uint8_t* hs = reinterpret_cast<const uint8_t*>(&head);
        int sc, mn;
        q4k_scale_min_dev(hs + 4, j, sc, mn);
        const float d = jinf_h2f((uint16_t)(head.x & 0xffff)), dmin = jinf_h2f((uint16_t)(head.x >> 16));
        const float sd = __fmul_rn(d, (float)sc), sm = __fmul_rn(dmin, (float)mn);
        float xs[8];
        load_x8<VEC>(x + 256 * b + 8 * lane, xs);
#pragma unroll
        for (int k = 0; k < 8; ++k)
            acc = fmaf(__fsub_rn(__fmul_rn(sd, (float)((q >> (4 * k)) & 15)), sm), xs[k], acc);
    }
    acc = warp_sum(acc);
    if (lane == 0) y[row] = acc;
}

// Q6_K in the reference layout: warp per row, lane = 8 weights per super-block.
__global__ void __launch_bounds__(MV_THREADS) k_matvec_q6_K(const uint8_t* __restrict__ W,
                                                            const float* __restrict__ x,
                                                            float* __restrict__ y, int rows, int cols) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * (MV_THREADS / 32) + (threadIdx.x >> 5);
    if (row >= rows) return;
    const int nb = cols / 256;
    float acc = 0.f;
    for (int b = 0; b < nb; ++b) {
        const jinf_block_q6_K* blk = reinterpret_cast<const jinf_block_q6_K*>(W + ((size_t)row * nb + b) * 210);
        const uint8_t* db = reinterpret_cast<const uint8_t*>(&blk->d);
        const float d = jinf_h2f((uint16_t)(db[0] | (db[1] << 8)));
        const int e0 = 8 * lane;
        const float s = __fmul_rn(d, (float)blk->scales[e0 >> 4]);
        const float* xb = x + 256 * b + e0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int e = e0 + i;
            const int lo = (blk->ql[e >> 1] >> ((e & 1) * 4)) & 15;
            const int hi = (blk->qh[e >> 2] >> (2 * (e & 3))) & 3;
            acc = fmaf(__fmul_rn(s, (float)((lo | (hi << 4)) - 32)), __ldg(xb + i), acc);
        }
    }
    acc = warp_sum(acc);
    if (lane == 0) y[row] = acc;
}

extern "C" void jinf_cuda_dequant_matvec(const void* weight, const float* input, float* output, int rows,
                                         int cols, int qtype, cudaStream_t stream) {
    if (rows == 0 || cols == 0) return;
    if (rows < 0 || cols < 0 || !weight || !input || !output) {
        jinf_record_error(JINF_ERR_INVALID, "dequant_matvec: bad arguments");
        return;
    }
    switch (qtype) {
        case JINF_TYPE_Q4_0:
        case JINF_TYPE_Q8_0: {
            if (cols % 32) { jinf_record_error(JINF_ERR_INVALID, "dequant_matvec: cols % 32"); return; }
            const size_t row_bytes = (size_t)(cols / 32) * (qtype == JINF_TYPE_Q4_0 ? 18 : 34);
            // Stage up to ~48 KB of rows per CTA, at least one row (rows up to 200 KB fit
            // with the opt-in shared-memory limit).
            int rpc = (int)((48 * 1024) / row_bytes);
            if (rpc < 1) rpc = 1;
            if (rpc > 32) rpc = 32;
            const size_t smem = (size_t)rpc * row_bytes + 16;
            if (smem > 227 * 1024) { jinf_record_error(JINF_ERR_INVALID, "dequant_matvec: row too long"); return; }
            const unsigned grid = (unsigned)((rows + rpc - 1) / rpc);
            const bool vec = ((uintptr_t)input & 15) == 0;
            auto launch = [&](auto kern) {
                cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
                kern<<<grid, MV_THREADS, smem, stream>>>((const uint8_t*)weight, input, output, rows, cols, rpc);
            };
            if (qtype == JINF_TYPE_Q4_0) {
                if (vec) launch(k_matvec_small_blocks<JINF_TYPE_Q4_0, true>);
                else launch(k_matvec_small_blocks<JINF_TYPE_Q4_0, false>);
            } else {
                if (vec) launch(k_matvec_small_blocks<JINF_TYPE_Q8_0, true>);
                else launch(k_matvec_small_blocks<JINF_TYPE_Q8_0, false>);
            }
            break;
        }
        case JINF_TYPE_Q4_K:
            if (cols % 256) { jinf_record_error(JINF_ERR_INVALID, "dequant_matvec: cols % 256"); return; }
        {
            const bool al = ((uintptr_t)weight & 15) == 0, vec = ((uintptr_t)input & 15) == 0;
            const unsigned grid = (unsigned)((rows + 7) / 8);
            const jinf_block_q4_K* w = (const jinf_block_q4_K*)weight;
            if (al && vec) k_matvec_q4_K<true, true><<<grid, MV_THREADS, 0, stream>>>(w, input, output, rows, cols);
            else if (al) k_matvec_q4_K<true, false><<<grid, MV_THREADS, 0, stream>>>(w, input, output, rows, cols);
            else if (vec) k_matvec_q4_K<false, true><<<grid, MV_THREADS, 0, stream>>>(w, input, output, rows, cols);
            else k_matvec_q4_K<false, false><<<grid, MV_THREADS, 0, stream>>>(w, input, output, rows, cols);
            break;
        }
        case JINF_TYPE_Q6_K:
            if (cols % 256) { jinf_record_error(JINF_ERR_INVALID, "dequant_matvec: cols % 256"); return; }
            k_matvec_q6_K<<<(rows + 7) / 8, MV_THREADS, 0, stream>>>((const uint8_t*)weight, input, output,
                                                                    rows, cols);
            break;
        default:
            fprintf(stderr, "[jinf] Unsupported qtype %d for dequant_matvec\n", qtype);
            jinf_record_error(JINF_ERR_INVALID, "dequant_matvec: unsupported qtype");
            return;
    }
    jinf_check_launch("dequant_matvec");
}

__global__ void k_residual_add(float* __restrict__ a, const float* __restrict__ b, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) a[i] += b[i];
}

extern "C" void jinf_cuda_residual_add(float* a, const float* b, int n, cudaStream_t stream) {
    if (n <= 0) return;
    k_residual_add<<<(n + 255) / 256, 256, 0, stream>>>(a, b, n);
    jinf_check_launch("residual_add");
}
