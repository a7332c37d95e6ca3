// Device building blocks of the Q4M tensor-core GEMV, shared by the stand-alone GEMV kernel
// (gemv_q4m.cu) and the persistent decode-step kernel (step_kernel.cu).
//
// Arithmetic (the reference computes y = sum_b d_b sum_e (q-8) x_e in fp32,
// cuda/matmul_kernels.cu:8-43). Streaming 4-bit weights at HBM speed leaves about three
// issue slots per weight on the CUDA cores, and an exact fp32 decode needs about that many.
// Here the decode is one lop3 per two weights and the multiply-add is retired by
// mma.sync.m16n8k16: the weight tile is the A operand, decoded in registers to the exact
// fp16 values 1024 + s*q (s = 1 or 16, q4m.cuh); the B operand holds x split into fp16
// hi + lo parts (22 significant bits), pre-scaled by 2^k / s. B is block diagonal: its
// column 2j+h carries part h of block j of the group, so one m16n8k16 step advances 16
// rows x 4 blocks at once and the accumulator column pair (2c, 2c+1) of a lane is exactly
// one block's dot product for rows gr and gr+8. Products are exact in fp32; the constant
// 1024 + 8s offset of every weight is removed by starting the accumulator at
// -(1024 + 8s) * sum(B) of the block, and the block scale d multiplies the block sum once.
#pragma once

#include <cuda_fp16.h>
#include <math.h>
#include <stdint.h>

#include "common.cuh"
#include "gemv.h"
#include "q4m.cuh"

namespace jinf {
namespace q4mdev {

typedef unsigned long long u64;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// This lane's 36 bytes of a chunk: nibble words of piece 0 and 1 and its two scales. Each
// lane reads back only what it copied, so a per-warp ring needs no warp synchronisation.
__device__ __forceinline__ void copy_chunk_async(uint32_t slot, const uint8_t* chunk, int lane) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(slot + lane * 16), "l"(chunk + lane * 16)
                 : "memory");
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(slot + 512 + lane * 16),
                 "l"(chunk + 512 + lane * 16)
                 : "memory");
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(slot + 1024 + lane * 4), "l"(chunk + 1024 + lane * 4)
                 : "memory");
}

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// One MMA step: decode the lane's word (eight nibbles -> four fp16x2 A registers) and
// accumulate A x B into d. The lop3 immediate 0xEA is (a & b) | c.
__device__ __forceinline__ void mma_step(uint32_t w, uint32_t b0, uint32_t b1, float (&d)[4]) {
    asm("{\n\t"
        ".reg .b32 a0, a1, a2, a3, u;\n\t"
        "shr.u32 u, %4, 8;\n\t"
        "lop3.b32 a0, %4, 0x000F000F, 0x64006400, 0xEA;\n\t"
        "lop3.b32 a2, %4, 0x00F000F0, 0x64006400, 0xEA;\n\t"
        "lop3.b32 a1, u, 0x000F000F, 0x64006400, 0xEA;\n\t"
        "lop3.b32 a3, u, 0x00F000F0, 0x64006400, 0xEA;\n\t"
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {a0, a1, a2, a3}, {%5, %6}, "
        "{%0, %1, %2, %3};\n\t"
        "}"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(w), "r"(b0), "r"(b1));
}

// B fragment byte selectors of a lane: its staged value goes to half (jn & 1) of b0
// (jn < 2) or b1 (jn >= 2), jn = lane / 8; even steps take bytes 0-1 of the staged word,
// odd steps bytes 2-3.
struct BSel {
    uint32_t s0e, s0o, s1e, s1o;
    __device__ __forceinline__ explicit BSel(int lane) {
        const int jn = lane >> 3;
        s0e = jn == 0 ? 0x4410u : jn == 1 ? 0x1044u : 0x4444u;
        s0o = jn == 0 ? 0x4432u : jn == 1 ? 0x3244u : 0x4444u;
        s1e = jn == 2 ? 0x4410u : jn == 3 ? 0x1044u : 0x4444u;
        s1o = jn == 2 ? 0x4432u : jn == 3 ? 0x3244u : 0x4444u;
    }
};

// One chunk (16 rows x 128 columns) from ring slot `sl` against staged group g:
// acc0 += row gr, acc1 += row gr+8 (block c of the group, c = lane & 3).
__device__ __forceinline__ void chunk_mma(uint32_t sl, const uint16_t* xb, const float* xk, int g, int lane,
                                          const BSel& bs, float& acc0, float& acc1) {
    uint32_t w[8], sc;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]) : "r"(sl + lane * 16));
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(w[4]), "=r"(w[5]), "=r"(w[6]), "=r"(w[7]) : "r"(sl + 512 + lane * 16));
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(sc) : "r"(sl + 1024 + lane * 4));
    const uint4 xv = *reinterpret_cast<const uint4*>(xb + (size_t)g * 256 + lane * 8);
    const float k = xk[g * 4 + (lane & 3)];
    // four independent accumulator chains (steps i, i+4 share one) hide the MMA latency
    float da[4] = {k, 0.f, k, 0.f}, db[4] = {0.f, 0.f, 0.f, 0.f};
    float dc[4] = {0.f, 0.f, 0.f, 0.f}, dd[4] = {0.f, 0.f, 0.f, 0.f};
    const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
    for (int i = 0; i < 8; i += 4) {
        mma_step(w[i], __byte_perm(xw[i >> 1], 0u, bs.s0e), __byte_perm(xw[i >> 1], 0u, bs.s1e), da);
        mma_step(w[i + 1], __byte_perm(xw[i >> 1], 0u, bs.s0o), __byte_perm(xw[i >> 1], 0u, bs.s1o), db);
        mma_step(w[i + 2], __byte_perm(xw[(i >> 1) + 1], 0u, bs.s0e), __byte_perm(xw[(i >> 1) + 1], 0u, bs.s1e), dc);
        mma_step(w[i + 3], __byte_perm(xw[(i >> 1) + 1], 0u, bs.s0o), __byte_perm(xw[(i >> 1) + 1], 0u, bs.s1o), dd);
    }
    const float t0 = ((da[0] + da[1]) + (db[0] + db[1])) + ((dc[0] + dc[1]) + (dd[0] + dd[1]));
    const float t1 = ((da[2] + da[3]) + (db[2] + db[3])) + ((dc[2] + dc[3]) + (dd[2] + dd[3]));
    acc0 = fmaf(jinf_h2f((uint16_t)(sc & 0xffffu)), t0, acc0);
    acc1 = fmaf(jinf_h2f((uint16_t)(sc >> 16)), t1, acc1);
}

// This lane's share of one 2304-byte unit (the chunks of a tile pair and one group).
__device__ __forceinline__ void copy_unit_async(uint32_t slot, const uint8_t* unit, int lane) {
    copy_chunk_async(slot, unit, lane);
    copy_chunk_async(slot + Q4M_CHUNK, unit + Q4M_CHUNK, lane);
}

// One unit (32 rows x 128 columns) from ring slot `sl` against staged group g: both tiles
// of the pair share the B fragments. acc[0], acc[1] += rows gr, gr+8 of the first tile,
// acc[2], acc[3] += rows gr, gr+8 of the second (block c of the group, c = lane & 3).
__device__ __forceinline__ void unit_mma(uint32_t sl, const uint16_t* xb, const float* xk, int g, int lane,
                                         const BSel& bs, float (&acc)[4]) {
    uint32_t w[8], v[8], sca, scb;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]) : "r"(sl + lane * 16));
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(w[4]), "=r"(w[5]), "=r"(w[6]), "=r"(w[7]) : "r"(sl + 512 + lane * 16));
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(sca) : "r"(sl + 1024 + lane * 4));
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]) : "r"(sl + Q4M_CHUNK + lane * 16));
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]) : "r"(sl + Q4M_CHUNK + 512 + lane * 16));
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(scb) : "r"(sl + Q4M_CHUNK + 1024 + lane * 4));
    const uint4 xv = *reinterpret_cast<const uint4*>(xb + (size_t)g * 256 + lane * 8);
    const float k = xk[g * 4 + (lane & 3)];
    float da[4] = {k, 0.f, k, 0.f}, db[4] = {0.f, 0.f, 0.f, 0.f};
    float ea[4] = {k, 0.f, k, 0.f}, eb[4] = {0.f, 0.f, 0.f, 0.f};
    const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
        const uint32_t p0 = __byte_perm(xw[i >> 1], 0u, bs.s0e), p1 = __byte_perm(xw[i >> 1], 0u, bs.s1e);
        const uint32_t q0 = __byte_perm(xw[i >> 1], 0u, bs.s0o), q1 = __byte_perm(xw[i >> 1], 0u, bs.s1o);
        mma_step(w[i], p0, p1, da);
        mma_step(v[i], p0, p1, ea);
        mma_step(w[i + 1], q0, q1, db);
        mma_step(v[i + 1], q0, q1, eb);
    }
    acc[0] = fmaf(jinf_h2f((uint16_t)(sca & 0xffffu)), (da[0] + da[1]) + (db[0] + db[1]), acc[0]);
    acc[1] = fmaf(jinf_h2f((uint16_t)(sca >> 16)), (da[2] + da[3]) + (db[2] + db[3]), acc[1]);
    acc[2] = fmaf(jinf_h2f((uint16_t)(scb & 0xffffu)), (ea[0] + ea[1]) + (eb[0] + eb[1]), acc[2]);
    acc[3] = fmaf(jinf_h2f((uint16_t)(scb >> 16)), (ea[2] + ea[3]) + (eb[2] + eb[3]), acc[3]);
}

// Sum the four accumulators over the lanes of a row group (blocks c = 0..3): afterwards
// lane (gr, c) holds rows gr, gr+8, 16+gr, 24+gr of the unit's 32 rows.
__device__ __forceinline__ void unit_reduce(float (&acc)[4]) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        acc[i] += __shfl_xor_sync(JINF_FULL_MASK, acc[i], 1);
        acc[i] += __shfl_xor_sync(JINF_FULL_MASK, acc[i], 2);
    }
}

// Row r (0..31) of a reduced unit as seen from the calling lane (all lanes participate).
__device__ __forceinline__ float unit_row(const float (&acc)[4], int r) {
    const int rr = r & 15, src = 4 * (rr & 7), which = ((r >> 4) << 1) | (rr >> 3);
    const float v0 = __shfl_sync(JINF_FULL_MASK, acc[0], src);
    const float v1 = __shfl_sync(JINF_FULL_MASK, acc[1], src);
    const float v2 = __shfl_sync(JINF_FULL_MASK, acc[2], src);
    const float v3 = __shfl_sync(JINF_FULL_MASK, acc[3], src);
    return which == 0 ? v0 : which == 1 ? v1 : which == 2 ? v2 : v3;
}

// Index of the reduced row held in acc[i] by lane (gr, c): gr, gr+8, 16+gr, 24+gr.
__device__ __forceinline__ int unit_row_of(int i, int lane) { return (lane >> 2) + 8 * i; }

__device__ __forceinline__ uint32_t ordered_bits(float v) {
    const uint32_t b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Packed argmax key: larger logit wins, the smaller index on ties.
__device__ __forceinline__ u64 argmax_key(float v, int idx) {
    return ((u64)ordered_bits(v) << 32) | (u64)(0xFFFFFFFFu - (uint32_t)idx);
}

// Power-of-two pre-scale 2^k putting amax * 2^k in [2^14, 2^15): the fp16 hi part of
// every scaled x stays finite and the lo part keeps its precision.
__device__ __forceinline__ float pow2_prescale(float amax) {
    int e = (int)((__float_as_uint(amax) >> 23) & 0xff);  // biased exponent of amax
    int k = 127 + 14 - (e - 127);                           // biased exponent of 2^(14 - E)
    k = k < 1 ? 1 : (k > 254 ? 254 : k);
    return __uint_as_float((uint32_t)k << 23);
}

__device__ __forceinline__ float4 ld_f4(const float* p, int i, bool coherent) {
    return coherent ? __ldcg(reinterpret_cast<const float4*>(p) + i) : reinterpret_cast<const float4*>(p)[i];
}

// Stage the GEMV input into the block-diagonal fp16 hi/lo B records (xb: [G][32][8]
// halves) and the accumulator offsets (xk: [4G]), with one round trip to global memory:
// the fp32 input (x, or h * gain in the norm modes) is staged in the B region itself,
// sum(h^2) and max|x| are reduced in one pass, then each warp converts whole groups in
// place. Every thread of the CTA calls this; it ends with the CTA synchronised and returns
// 2^-k (the factor that undoes the pre-scale). `coherent` reads inputs written by other
// CTAs of a running grid through L2. In the norm modes `hsrc` is the residual stream (or
// the embedding row, X_EMBED_NORM) and h is also stored to `hout` when `store_h` is set
// (exactly one CTA of the grid does it).
template <int NT>
__device__ __forceinline__ float stage_x(int xm, const void* x, const float* hsrc, const float* yres, float* hout,
                                         bool store_h_cta, const float* norm_w, float eps, int cols, uint8_t* xbase,
                                         float* xk, float* misc, bool coherent) {
    constexpr int NW = NT / 32;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const bool norm = xm == X_RMSNORM || xm == X_EMBED_NORM;
    float* xf = reinterpret_cast<float*>(xbase);
    uint16_t* xb = reinterpret_cast<uint16_t*>(xbase);
    const bool store_h = norm && store_h_cta && hout;
    float ss = 0.f, amax = 0.f;
#pragma unroll 4
    for (int i = tid; i < cols / 4; i += NT) {
        float4 v;
        if (xm == X_PLAIN_F32) {
            v = ld_f4(reinterpret_cast<const float*>(x), i, coherent);
        } else if (xm == X_PLAIN_F16) {
            const uint2 hv = reinterpret_cast<const uint2*>(x)[i];
            const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&hv.x));
            const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&hv.y));
            v = make_float4(a.x, a.y, b.x, b.y);
        } else {
            float4 h = ld_f4(hsrc, i, coherent && xm != X_EMBED_NORM);
            if (xm == X_RMSNORM && yres) {
                const float4 r = ld_f4(yres, i, coherent);
                h.x += r.x;
                h.y += r.y;
                h.z += r.z;
                h.w += r.w;
            }
            if (store_h) reinterpret_cast<float4*>(hout)[i] = h;
            ss = fmaf(h.x, h.x, ss);
            ss = fmaf(h.y, h.y, ss);
            ss = fmaf(h.z, h.z, ss);
            ss = fmaf(h.w, h.w, ss);
            const float4 g = reinterpret_cast<const float4*>(norm_w)[i];
            v = make_float4(h.x * g.x, h.y * g.y, h.z * g.z, h.w * g.w);
        }
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        reinterpret_cast<float4*>(xf)[i] = v;
    }
    // a padded last group (cols not a multiple of 128) stages zeros: its weights have scale 0
    const int G = (cols + Q4M_KG - 1) / Q4M_KG;
    for (int i = cols / 4 + tid; i < G * 32; i += NT) reinterpret_cast<float4*>(xf)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        ss += __shfl_xor_sync(JINF_FULL_MASK, ss, o);
        amax = fmaxf(amax, __shfl_xor_sync(JINF_FULL_MASK, amax, o));
    }
    if (lane == 0) {
        misc[warp] = ss;
        misc[32 + warp] = amax;
    }
    __syncthreads();
    ss = 0.f;
    amax = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
        ss += misc[w];
        amax = fmaxf(amax, misc[32 + w]);
    }
    const float rnorm = norm ? rsqrtf(ss / (float)cols + eps) : 1.0f;
    const float alpha = pow2_prescale(amax * rnorm * 1.0001f);
    for (int g = warp; g < G; g += NW) {
        // lane l converts elements 4(l%8) .. 4(l%8)+3 of block j = l/8 of the group
        const float4 v = reinterpret_cast<const float4*>(xf + g * 128)[lane];
        __syncwarp();  // the whole group is in registers before it is overwritten
        const int j = lane >> 3, q = lane & 7;
        const float scale = (norm ? rnorm : 1.0f) * alpha * (j < 2 ? 1.0f : 0.0625f);
        const float vv[4] = {v.x * scale, v.y * scale, v.z * scale, v.w * scale};
        float s = 0.f;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const __half hi = __float2half_rn(vv[t]);
            const __half lo = __float2half_rn(vv[t] - __half2float(hi));
            // element e = 4q + t of block j: lane record 4*(2j + h) + t, half q
            uint16_t* rec = xb + (size_t)g * 256 + (8 * j + t) * 8 + q;
            rec[0] = __half_as_ushort(hi);
            rec[32] = __half_as_ushort(lo);  // h = 1: four lane records further
            s += __half2float(hi) + __half2float(lo);
        }
        s += __shfl_xor_sync(JINF_FULL_MASK, s, 1);
        s += __shfl_xor_sync(JINF_FULL_MASK, s, 2);
        s += __shfl_xor_sync(JINF_FULL_MASK, s, 4);
        if (q == 0) xk[g * 4 + j] = -(j < 2 ? 1032.0f : 1152.0f) * s;
    }
    __syncthreads();
    return 1.0f / alpha;  // exact: alpha is a power of two
}

// Sum the partial rows of the lanes of one row group (blocks c = 0..3) and hand rows
// 2q, 2q+1 of the tile to lane q < 8 (full tile owned by this warp).
__device__ __forceinline__ void tile_rows(float acc0, float acc1, int lane, float& v0, float& v1) {
    acc0 += __shfl_xor_sync(JINF_FULL_MASK, acc0, 1);
    acc1 += __shfl_xor_sync(JINF_FULL_MASK, acc1, 1);
    acc0 += __shfl_xor_sync(JINF_FULL_MASK, acc0, 2);
    acc1 += __shfl_xor_sync(JINF_FULL_MASK, acc1, 2);
    const int r0 = 2 * (lane & 7), r1 = r0 + 1;
    const float a0 = __shfl_sync(JINF_FULL_MASK, acc0, 4 * (r0 & 7));
    const float b0 = __shfl_sync(JINF_FULL_MASK, acc1, 4 * (r0 & 7));
    const float a1 = __shfl_sync(JINF_FULL_MASK, acc0, 4 * (r1 & 7));
    const float b1 = __shfl_sync(JINF_FULL_MASK, acc1, 4 * (r1 & 7));
    v0 = r0 < 8 ? a0 : b0;
    v1 = r1 < 8 ? a1 : b1;
}

// Per-row outputs of the fused epilogues for rows `row`, `row + 1` (values v0, v1).
struct EpiArgs {
    int epi;
    int rows;
    float* y;
    __half* kcache;
    __half* vcache;
    int nq, nk, head_dim, max_ctx, pos;
    float rope_base;
    bool coherent;  // EPI_RESID reads h through L2
};

__device__ __forceinline__ void epilogue_pair(const EpiArgs& a, int row, float v0, float v1, float& lmax, int& lidx) {
    if (row >= a.rows) return;
    if (a.epi == EPI_STORE || a.epi == EPI_LMHEAD) {
        a.y[row] = v0;
        if (a.epi == EPI_LMHEAD && v0 > lmax) { lmax = v0; lidx = row; }
        if (row + 1 < a.rows) {
            a.y[row + 1] = v1;
            if (a.epi == EPI_LMHEAD && v1 > lmax) { lmax = v1; lidx = row + 1; }
        }
    } else if (a.epi == EPI_RESID) {
        // h += W x, the reference's residual add (src/engine.cpp:470-472, 505-507)
        const float h0 = a.coherent ? __ldcg(a.y + row) : a.y[row];
        a.y[row] = h0 + v0;
        if (row + 1 < a.rows) {
            const float h1 = a.coherent ? __ldcg(a.y + row + 1) : a.y[row + 1];
            a.y[row + 1] = h1 + v1;
        }
    } else if (a.epi == EPI_GATEUP) {
        a.y[row >> 1] = v0 / (1.0f + expf(-v0)) * v1;
    } else {  // EPI_QKV: rows are [q | k | v], each head_dim-aligned
        const int pos = a.pos;
        if (row < a.nq + a.nk) {
            const int rr = row < a.nq ? row : row - a.nq;
            const int i = (rr % a.head_dim) >> 1;
            const float theta = powf(a.rope_base, -2.0f * (float)i / (float)a.head_dim);
            const float ang = (float)pos * theta;
            const float cs = cosf(ang), sn = sinf(ang);
            const float o0 = v0 * cs - v1 * sn, o1 = v0 * sn + v1 * cs;
            if (row < a.nq) {
                a.y[row] = o0;
                a.y[row + 1] = o1;
            } else {
                const int kvh = rr / a.head_dim, dd = rr % a.head_dim;
                __half* dst = a.kcache + ((size_t)kvh * a.max_ctx + pos) * a.head_dim + dd;
                *reinterpret_cast<__half2*>(dst) = __floats2half2_rn(o0, o1);
            }
        } else {
            const int rr = row - a.nq - a.nk;
            const int kvh = rr / a.head_dim, dd = rr % a.head_dim;
            __half* dst = a.vcache + ((size_t)kvh * a.max_ctx + pos) * a.head_dim + dd;
            *reinterpret_cast<__half2*>(dst) = __floats2half2_rn(v0, v1);
        }
    }
}

}  // namespace q4mdev
}  // namespace jinf
