// Device building blocks of the Q4M tensor-core GEMV, shared by the stand-alone GEMV kernel
// (gemv_q4m.cu) and the persistent decode-step kernel (step_kernel.cu).
//
// Arithmetic (the reference computes y = sum_b d_b sum_e (q-8) x_e in fp32,
// cuda/matmul_kernels.cu:8-43). Streaming 4-bit weights at HBM speed leaves only a few issue
// slots per weight, so the multiply-adds run on the tensor cores (mma.sync m16n8k32, u8 x s8
// -> s32, exact) and the decode is one lop3 per four weights: a unit word's low nibbles are
// tile A's u8 operand, its high nibbles (16 q) tile B's (q4m.cuh).
//
// The input x is staged as int8 digit records: per 32-element block a scale
// alpha = 32639 / max|x| and, per element, v = rint(x alpha) = 256 hi + lo with hi, lo in
// [-128, 127] (relative error <= 2^-16 of the block maximum). B is block diagonal: column
// 2j+h carries digit h of block j, so after the four m16n8k32 steps of a group the
// accumulator columns (2c, 2c+1) of a lane are exactly sum_k q_k hi_k and sum_k q_k lo_k of
// block c for rows gr and gr+8. The zero point is removed by starting the accumulator at
// -8 sum(hi), -8 sum(lo) (x16 for tile B), and the block contributes
// d * (256 D_hi + D_lo) / alpha to the row in fp32.
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

constexpr float XREC_DIGIT_MAX = 32639.0f;  // |x| alpha <= 32639 keeps hi = (v + 128) >> 8 in int8

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// This lane's share of a 2304-byte unit: its nibble words of the four blocks and its two
// scale words. Each lane reads back only what it copied, so a per-warp ring needs no warp
// synchronisation.
__device__ __forceinline__ void copy_unit_async(uint32_t slot, const uint8_t* unit, int lane) {
#pragma unroll
    for (int j = 0; j < 4; ++j)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(slot + 512 * j + lane * 16),
                     "l"(unit + 512 * j + lane * 16)
                     : "memory");
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(slot + Q4M_SCALES + lane * 4),
                 "l"(unit + Q4M_SCALES + lane * 4)
                 : "memory");
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(slot + Q4M_SCALES + 128 + lane * 4),
                 "l"(unit + Q4M_SCALES + 128 + lane * 4)
                 : "memory");
}

// This lane's share of a 2432-byte Q4_K unit: its nibble words (as Q4_0), and lanes 0..23
// one 16-byte piece of the 384-byte scale area each. The scale area is read across lanes,
// so the consumer synchronises the warp after waiting for the copies (unit_mma_k).
__device__ __forceinline__ void copy_unit_k_async(uint32_t slot, const uint8_t* unit, int lane) {
#pragma unroll
    for (int j = 0; j < 4; ++j)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(slot + 512 * j + lane * 16),
                     "l"(unit + 512 * j + lane * 16)
                     : "memory");
    if (lane < 24)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(slot + Q4M_SCALES + lane * 16),
                     "l"(unit + Q4M_SCALES + lane * 16)
                     : "memory");
}

// This lane's share of a 3392-byte Q6_K unit: its nibble words, its two 16-byte crumb
// pieces and its scale words; lanes 0..3 one 16-byte piece of the per-row d each (read by
// other lanes: the consumer synchronises the warp, unit_mma_q6).
__device__ __forceinline__ void copy_unit_6_async(uint32_t slot, const uint8_t* unit, int lane) {
#pragma unroll
    for (int j = 0; j < 4; ++j)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(slot + 512 * j + lane * 16),
                     "l"(unit + 512 * j + lane * 16)
                     : "memory");
#pragma unroll
    for (int jj = 0; jj < 2; ++jj)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(slot + Q4M_CRUMB_6 + 512 * jj + lane * 16),
                     "l"(unit + Q4M_CRUMB_6 + 512 * jj + lane * 16)
                     : "memory");
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(slot + Q4M_SC_6 + lane * 8),
                 "l"(unit + Q4M_SC_6 + lane * 8)
                 : "memory");
    if (lane < 4)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(slot + Q4M_D_6 + lane * 16),
                     "l"(unit + Q4M_D_6 + lane * 16)
                     : "memory");
}

// This lane's share of a 4352-byte Q8_0 unit: its eight weight words of 16 bytes and its
// 8-byte scale record. Each lane reads back only what it copied.
__device__ __forceinline__ void copy_unit_8_async(uint32_t slot, const uint8_t* unit, int lane) {
#pragma unroll
    for (int jt = 0; jt < 8; ++jt)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(slot + 512 * jt + lane * 16),
                     "l"(unit + 512 * jt + lane * 16)
                     : "memory");
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(slot + Q4M_D_8 + lane * 8),
                 "l"(unit + Q4M_D_8 + lane * 8)
                 : "memory");
}

// The copy routine of a unit of format `fmt` (q4m.cuh).
template <int FMT>
__device__ __forceinline__ void copy_unit_fmt(uint32_t slot, const uint8_t* unit, int lane) {
    if (FMT == Q4M_Q4_K) copy_unit_k_async(slot, unit, lane);
    else if (FMT == Q4M_Q6_K) copy_unit_6_async(slot, unit, lane);
    else if (FMT == Q4M_Q8_0) copy_unit_8_async(slot, unit, lane);
    else copy_unit_async(slot, unit, lane);
}

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mma_u8s8(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1, int (&d)[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_s8s8(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1, int (&d)[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// m16n8k16: the first (or second) half of a 32-element block on its own
__device__ __forceinline__ void mma_s8s8_k16(uint32_t a0, uint32_t a1, uint32_t b0, int (&d)[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5}, {%6}, {%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(b0));
}

// The u8 operands of a nibble word: tile A (low nibbles) and tile B (high nibbles, 16 q).
__device__ __forceinline__ uint32_t nib_lo(uint32_t w) { return w & 0x0F0F0F0Fu; }
__device__ __forceinline__ uint32_t nib_hi(uint32_t w) { return w & 0xF0F0F0F0u; }

// Shared-memory addresses of a staged input: digit records and block params (xrec_bytes).
struct XRecS {
    uint32_t dig, prm;
};

// One unit (32 rows x 128 columns) from ring slot `sl` against staged group g: acc[0],
// acc[1] += rows gr, gr+8 of tile A, acc[2], acc[3] += rows 16+gr, 24+gr (tile B), each the
// contribution of block c = lane & 3 of the group.
__device__ __forceinline__ void unit_mma(uint32_t sl, const XRecS& xr, int g, int lane, float (&acc)[4]) {
    uint32_t w[16], sca, scb, b0, b1;
    int kh, kl;
    float ia, ib;
#pragma unroll
    for (int j = 0; j < 4; ++j)
        asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(w[4 * j]), "=r"(w[4 * j + 1]), "=r"(w[4 * j + 2]), "=r"(w[4 * j + 3])
                     : "r"(sl + 512 * j + lane * 16));
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(sca) : "r"(sl + Q4M_SCALES + lane * 4));
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(scb) : "r"(sl + Q4M_SCALES + 128 + lane * 4));
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(b0), "=r"(b1) : "r"(xr.dig + g * 256 + lane * 8));
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(kh), "=r"(kl), "=f"(ia), "=f"(ib)
                 : "r"(xr.prm + (g * 4 + (lane & 3)) * 16));
    const int myblk = lane >> 3;  // the block whose digit column this lane's B fragment holds
    int da[4] = {kh, kl, kh, kl};
    int db[4] = {kh * 16, kl * 16, kh * 16, kl * 16};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t x0 = myblk == j ? b0 : 0u, x1 = myblk == j ? b1 : 0u;
        mma_u8s8(nib_lo(w[4 * j]), nib_lo(w[4 * j + 1]), nib_lo(w[4 * j + 2]), nib_lo(w[4 * j + 3]), x0, x1, da);
        mma_u8s8(nib_hi(w[4 * j]), nib_hi(w[4 * j + 1]), nib_hi(w[4 * j + 2]), nib_hi(w[4 * j + 3]), x0, x1, db);
    }
    acc[0] = fmaf(jinf_h2f((uint16_t)(sca & 0xffffu)) * ia, (float)(da[0] * 256 + da[1]), acc[0]);
    acc[1] = fmaf(jinf_h2f((uint16_t)(sca >> 16)) * ia, (float)(da[2] * 256 + da[3]), acc[1]);
    acc[2] = fmaf(jinf_h2f((uint16_t)(scb & 0xffffu)) * ib, (float)(db[0] * 256 + db[1]), acc[2]);
    acc[3] = fmaf(jinf_h2f((uint16_t)(scb >> 16)) * ib, (float)(db[2] * 256 + db[3]), acc[3]);
}

// unit_mma for a Q4_K unit (q4m.cuh): the accumulators start at zero (the weights are
// d sc q - dmin m, no zero point), and block c of row r contributes
// (d sc (256 D_hi + D_lo) - dmin m (256 S_hi + S_lo)) / alpha, S the block's digit sums
// (recovered exactly from the record's zero-point params, -8 S). The warp synchronises
// before (its lanes read scale words other lanes copied) and after (before a lane copies
// the next unit into the slot).
__device__ __forceinline__ void unit_mma_k(uint32_t sl, const XRecS& xr, int g, int lane, float (&acc)[4]) {
    __syncwarp();
    uint32_t w[16], sca, scb, b0, b1, dA0, dA1, dB0, dB1;
    int kh, kl;
    float ia, ib;
    const int gr = lane >> 2;
#pragma unroll
    for (int j = 0; j < 4; ++j)
        asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(w[4 * j]), "=r"(w[4 * j + 1]), "=r"(w[4 * j + 2]), "=r"(w[4 * j + 3])
                     : "r"(sl + 512 * j + lane * 16));
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(sca) : "r"(sl + Q4M_SCALES + lane * 4));
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(scb) : "r"(sl + Q4M_SCALES + 128 + lane * 4));
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(dA0) : "r"(sl + Q4M_DMIN_K + gr * 4));
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(dA1) : "r"(sl + Q4M_DMIN_K + (gr + 8) * 4));
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(dB0) : "r"(sl + Q4M_DMIN_K + 64 + gr * 4));
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(dB1) : "r"(sl + Q4M_DMIN_K + 64 + (gr + 8) * 4));
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(b0), "=r"(b1) : "r"(xr.dig + g * 256 + lane * 8));
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(kh), "=r"(kl), "=f"(ia), "=f"(ib)
                 : "r"(xr.prm + (g * 4 + (lane & 3)) * 16));
    const int myblk = lane >> 3;
    int da[4] = {0, 0, 0, 0}, db[4] = {0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t x0 = myblk == j ? b0 : 0u, x1 = myblk == j ? b1 : 0u;
        mma_u8s8(nib_lo(w[4 * j]), nib_lo(w[4 * j + 1]), nib_lo(w[4 * j + 2]), nib_lo(w[4 * j + 3]), x0, x1, da);
        mma_u8s8(nib_hi(w[4 * j]), nib_hi(w[4 * j + 1]), nib_hi(w[4 * j + 2]), nib_hi(w[4 * j + 3]), x0, x1, db);
    }
    const float S = (float)(-((kh << 8) + kl) >> 3);  // 256 S_hi + S_lo of block c (exact)
    // tile B's block sums carry the 16 of its high-nibble operand: its min term is taken
    // x16 too and the whole row scaled by 1/(16 alpha) (powers of two: exact)
    auto row = [&](uint32_t scm, uint32_t dd, float dsum, float s) {
        const float sub_d = jinf_h2f((uint16_t)(dd & 0xffffu)) * (float)(scm & 63u);
        const float sub_m = jinf_h2f((uint16_t)(dd >> 16)) * (float)((scm >> 8) & 63u);
        return fmaf(sub_d, dsum, -sub_m * s);
    };
    acc[0] = fmaf(row(sca & 0xffffu, dA0, (float)(da[0] * 256 + da[1]), S), ia, acc[0]);
    acc[1] = fmaf(row(sca >> 16, dA1, (float)(da[2] * 256 + da[3]), S), ia, acc[1]);
    acc[2] = fmaf(row(scb & 0xffffu, dB0, (float)(db[0] * 256 + db[1]), 16.0f * S), ib, acc[2]);
    acc[3] = fmaf(row(scb >> 16, dB1, (float)(db[2] * 256 + db[3]), 16.0f * S), ib, acc[3]);
    __syncwarp();  // every lane's reads of the slot precede the next copy into it
}

// unit_mma for a Q6_K unit (q4m.cuh). Each weight byte is rebuilt as the int8 value
// 4 (q - 32) from its nibble (bits 2..5) and flipped crumb (bits 6..7), so the products need
// no zero point. A Q6_K scale covers 16 elements, so every block is two m16n8k16 steps, one
// per half, each into its own accumulators; block c of row r then contributes
// d sc_0 (256 D0_hi + D0_lo) + d sc_1 (256 D1_hi + D1_lo), times 1 / (4 alpha). The warp
// synchronises before (lanes read the d words lanes 0..3 copied) and after (before a lane
// copies the next unit into the slot).
__device__ __forceinline__ void unit_mma_q6(uint32_t sl, const XRecS& xr, int g, int lane, float (&acc)[4]) {
    __syncwarp();
    uint32_t w[16], cr[8], sca, scb, dlo, dhi, b0, b1;
    float ia;
    const int gr = lane >> 2;
#pragma unroll
    for (int j = 0; j < 4; ++j)
        asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(w[4 * j]), "=r"(w[4 * j + 1]), "=r"(w[4 * j + 2]), "=r"(w[4 * j + 3])
                     : "r"(sl + 512 * j + lane * 16));
#pragma unroll
    for (int jj = 0; jj < 2; ++jj)
        asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(cr[4 * jj]), "=r"(cr[4 * jj + 1]), "=r"(cr[4 * jj + 2]), "=r"(cr[4 * jj + 3])
                     : "r"(sl + Q4M_CRUMB_6 + 512 * jj + lane * 16));
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(sca), "=r"(scb) : "r"(sl + Q4M_SC_6 + lane * 8));
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(dlo), "=r"(dhi) : "r"(sl + Q4M_D_6 + gr * 8));
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(b0), "=r"(b1) : "r"(xr.dig + g * 256 + lane * 8));
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(ia) : "r"(xr.prm + (g * 4 + (lane & 3)) * 16 + 8));
    const int myblk = lane >> 3;
    int a0[4] = {0, 0, 0, 0}, a1[4] = {0, 0, 0, 0}, c0[4] = {0, 0, 0, 0}, c1[4] = {0, 0, 0, 0};
    constexpr uint32_t NM = 0x3C3C3C3Cu, CM = 0xC0C0C0C0u;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t x0 = myblk == j ? b0 : 0u, x1 = myblk == j ? b1 : 0u;
        const uint32_t* n = w + 4 * j;
        const uint32_t h0 = cr[2 * j], h1 = cr[2 * j + 1];  // crumbs of words 0, 1 / 2, 3
        // tile A (low nibbles) and tile B (high nibbles) operands of words i = 0..3
        const uint32_t A0 = ((n[0] << 2) & NM) | ((h0 << 6) & CM), B0 = ((n[0] >> 2) & NM) | ((h0 << 4) & CM);
        const uint32_t A1 = ((n[1] << 2) & NM) | ((h0 << 2) & CM), B1 = ((n[1] >> 2) & NM) | (h0 & CM);
        const uint32_t A2 = ((n[2] << 2) & NM) | ((h1 << 6) & CM), B2 = ((n[2] >> 2) & NM) | ((h1 << 4) & CM);
        const uint32_t A3 = ((n[3] << 2) & NM) | ((h1 << 2) & CM), B3 = ((n[3] >> 2) & NM) | (h1 & CM);
        mma_s8s8_k16(A0, A1, x0, a0);
        mma_s8s8_k16(A2, A3, x1, a1);
        mma_s8s8_k16(B0, B1, x0, c0);
        mma_s8s8_k16(B2, B3, x1, c1);
    }
    const float s = 0.25f * ia;
    auto sc = [](uint32_t v, int b) { return (float)(int8_t)(uint8_t)(v >> (8 * b)); };
    auto row = [&](float d, uint32_t scw, int b, const int (&h0)[4], const int (&h1)[4], int r) {
        const float s0 = (float)(h0[2 * r] * 256 + h0[2 * r + 1]);
        const float s1 = (float)(h1[2 * r] * 256 + h1[2 * r + 1]);
        return d * fmaf(sc(scw, b), s0, sc(scw, b + 1) * s1);
    };
    acc[0] = fmaf(row(jinf_h2f((uint16_t)(dlo & 0xffffu)), sca, 0, a0, a1, 0), s, acc[0]);
    acc[1] = fmaf(row(jinf_h2f((uint16_t)(dlo >> 16)), sca, 2, a0, a1, 1), s, acc[1]);
    acc[2] = fmaf(row(jinf_h2f((uint16_t)(dhi & 0xffffu)), scb, 0, c0, c1, 0), s, acc[2]);
    acc[3] = fmaf(row(jinf_h2f((uint16_t)(dhi >> 16)), scb, 2, c0, c1, 1), s, acc[3]);
    __syncwarp();  // every lane's reads of the slot precede the next copy into it
}

// unit_mma for a Q8_0 unit (q4m.cuh): the weight words are the int8 q themselves, one
// m16n8k32 step per block and tile, no zero point; block c of row r contributes
// d (256 D_hi + D_lo) / alpha.
__device__ __forceinline__ void unit_mma_q8(uint32_t sl, const XRecS& xr, int g, int lane, float (&acc)[4]) {
    uint32_t b0, b1, d01, d23;
    float ia;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(d01), "=r"(d23) : "r"(sl + Q4M_D_8 + lane * 8));
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(b0), "=r"(b1) : "r"(xr.dig + g * 256 + lane * 8));
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(ia) : "r"(xr.prm + (g * 4 + (lane & 3)) * 16 + 8));
    const int myblk = lane >> 3;
    int da[4] = {0, 0, 0, 0}, db[4] = {0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint32_t wa[4], wb[4];
        asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(wa[0]), "=r"(wa[1]), "=r"(wa[2]), "=r"(wa[3])
                     : "r"(sl + 1024 * j + lane * 16));
        asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(wb[0]), "=r"(wb[1]), "=r"(wb[2]), "=r"(wb[3])
                     : "r"(sl + 1024 * j + 512 + lane * 16));
        const uint32_t x0 = myblk == j ? b0 : 0u, x1 = myblk == j ? b1 : 0u;
        mma_s8s8(wa[0], wa[1], wa[2], wa[3], x0, x1, da);
        mma_s8s8(wb[0], wb[1], wb[2], wb[3], x0, x1, db);
    }
    acc[0] = fmaf(jinf_h2f((uint16_t)(d01 & 0xffffu)) * ia, (float)(da[0] * 256 + da[1]), acc[0]);
    acc[1] = fmaf(jinf_h2f((uint16_t)(d01 >> 16)) * ia, (float)(da[2] * 256 + da[3]), acc[1]);
    acc[2] = fmaf(jinf_h2f((uint16_t)(d23 & 0xffffu)) * ia, (float)(db[0] * 256 + db[1]), acc[2]);
    acc[3] = fmaf(jinf_h2f((uint16_t)(d23 >> 16)) * ia, (float)(db[2] * 256 + db[3]), acc[3]);
}

template <int FMT>
__device__ __forceinline__ void unit_mma_fmt(uint32_t sl, const XRecS& xr, int g, int lane, float (&acc)[4]) {
    if (FMT == Q4M_Q4_K) unit_mma_k(sl, xr, g, lane, acc);
    else if (FMT == Q4M_Q6_K) unit_mma_q6(sl, xr, g, lane, acc);
    else if (FMT == Q4M_Q8_0) unit_mma_q8(sl, xr, g, lane, acc);
    else unit_mma(sl, xr, g, lane, acc);
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

__device__ __forceinline__ float4 ld_f4(const float* p, int i, bool coherent) {
    return coherent ? __ldcg(reinterpret_cast<const float4*>(p) + i) : reinterpret_cast<const float4*>(p)[i];
}

// Digit records of one 32-element block held by an octet of lanes (lane q = lane & 7 of the
// octet holds elements 4q .. 4q+3 in v): `dig` is the group's 64 record words and `prm` its
// 4 block params (shared or global memory), j the block within the group. All 32 lanes of
// the warp call it (the octet reductions shuffle); only octets with `store` write. A block
// of zeros gives zero records.
__device__ __forceinline__ void octet_to_records(float4 v, int lane, int j, uint32_t* dig, float4* prm,
                                                 bool store = true) {
    const int q = lane & 7;
    float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    amax = fmaxf(amax, __shfl_xor_sync(JINF_FULL_MASK, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(JINF_FULL_MASK, amax, 2));
    amax = fmaxf(amax, __shfl_xor_sync(JINF_FULL_MASK, amax, 4));
    const float alpha = amax > 0.f ? XREC_DIGIT_MAX / amax : 0.f;
    const float e[4] = {v.x, v.y, v.z, v.w};
    uint32_t H = 0, L = 0;
    int sh = 0, sl = 0;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const int vi = __float2int_rn(e[t] * alpha);
        const int hi = (vi + 128) >> 8, lo = vi - (hi << 8);
        H |= (uint32_t)(hi & 0xff) << (8 * t);
        L |= (uint32_t)(lo & 0xff) << (8 * t);
        sh += hi;
        sl += lo;
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
        sh += __shfl_xor_sync(JINF_FULL_MASK, sh, o);
        sl += __shfl_xor_sync(JINF_FULL_MASK, sl, o);
    }
    // elements k = 4q .. 4q+3: word r = q >> 2 of record lanes 4 (2j + h) + (q & 3)
    const int r = q >> 2, c = q & 3;
    if (!store) return;
    dig[(8 * j + c) * 2 + r] = H;
    dig[(8 * j + 4 + c) * 2 + r] = L;
    if (q == 0) {
        const float ia = amax / XREC_DIGIT_MAX;
        prm[j] = make_float4(__int_as_float(-8 * sh), __int_as_float(-8 * sl), ia, ia * 0.0625f);
    }
}

// Load one group's input of the calling lane (elements 4 (g*32 + lane) .. +3) for stage_x;
// zero past cols.
__device__ __forceinline__ void stage_load(int xm, const void* x, const float* hsrc, const float* yres,
                                           const float* norm_w, int g, int G, int n4, int lane, bool coherent,
                                           float4& h, float4& gn) {
    const int i = g * 32 + lane;
    h = make_float4(0.f, 0.f, 0.f, 0.f);
    gn = h;
    if (g >= G || i >= n4) return;
    if (xm == X_PLAIN_F32) {
        h = ld_f4(reinterpret_cast<const float*>(x), i, coherent);
    } else if (xm == X_PLAIN_F16) {
        const uint2 hv = reinterpret_cast<const uint2*>(x)[i];
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&hv.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&hv.y));
        h = make_float4(a.x, a.y, b.x, b.y);
    } else {
        h = ld_f4(hsrc, i, coherent && xm != X_EMBED_NORM);
        if (xm == X_RMSNORM && yres) {
            const float4 r = ld_f4(yres, i, coherent);
            h.x += r.x;
            h.y += r.y;
            h.z += r.z;
            h.w += r.w;
        }
        gn = reinterpret_cast<const float4*>(norm_w)[i];
    }
}

// Groups g0, g0 + NW, ... (BG of them) of one warp: every load is issued before the first
// conversion, so the warp pays one L2 round trip per batch, not one per group.
template <int NW, int BG, bool NORM>
__device__ __forceinline__ void stage_batch(int xm, const void* x, const float* hsrc, const float* yres, float* hout,
                                            bool store_h, const float* norm_w, int g0, int G, int n4, int lane,
                                            bool coherent, uint32_t* dig, float4* prm, float& ss) {
    float4 h[BG], gn[BG];
#pragma unroll
    for (int b = 0; b < BG; ++b) stage_load(xm, x, hsrc, yres, norm_w, g0 + b * NW, G, n4, lane, coherent, h[b], gn[b]);
#pragma unroll
    for (int b = 0; b < BG; ++b) {
        const int g = g0 + b * NW;
        if (g >= G) break;
        float4 v = h[b];
        if (NORM) {
            if (store_h && g * 32 + lane < n4) reinterpret_cast<float4*>(hout)[g * 32 + lane] = v;
            ss = fmaf(v.x, v.x, ss);
            ss = fmaf(v.y, v.y, ss);
            ss = fmaf(v.z, v.z, ss);
            ss = fmaf(v.w, v.w, ss);
            v = make_float4(v.x * gn[b].x, v.y * gn[b].y, v.z * gn[b].z, v.w * gn[b].w);
        }
        octet_to_records(v, lane, lane >> 3, dig + g * 64, prm + g * 4);
    }
}

// Stage the GEMV input as digit records in shared memory (`rec`, xrec_bytes(G) bytes): each
// warp loads and converts whole groups (lane l: block l / 8, elements 4 (l % 8) .. +3), so
// no warp waits on another before converting; groups past cols (padding) get zero records.
// In the norm modes the records hold h * gain and the returned factor is
// 1 / sqrt(mean(h^2) + eps), which the epilogue applies (W (h g r) = r W (h g)); otherwise it
// is 1. Every thread of the CTA calls this; it ends with the CTA synchronised. `coherent`
// reads inputs written by other CTAs of a running grid through L2. In the norm modes `hsrc`
// is the residual stream (or the embedding row, X_EMBED_NORM) and h is also stored to `hout`
// when `store_h_cta` is set (exactly one CTA of the grid does it).
template <int NT>
__device__ __forceinline__ float stage_x(int xm, const void* x, const float* hsrc, const float* yres, float* hout,
                                         bool store_h_cta, const float* norm_w, float eps, int cols, uint8_t* rec,
                                         float* misc, bool coherent) {
    constexpr int NW = NT / 32;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const bool norm = xm == X_RMSNORM || xm == X_EMBED_NORM;
    const bool store_h = norm && store_h_cta && hout;
    const int G = (cols + Q4M_KG - 1) / Q4M_KG, n4 = cols / 4;
    uint32_t* dig = reinterpret_cast<uint32_t*>(rec);
    float4* prm = reinterpret_cast<float4*>(rec + (size_t)G * 256);
    float ss = 0.f;
    if (norm) {
        for (int g0 = warp; g0 < G; g0 += NW * 4)
            stage_batch<NW, 4, true>(xm, x, hsrc, yres, hout, store_h, norm_w, g0, G, n4, lane, coherent, dig, prm, ss);
    } else {
        for (int g0 = warp; g0 < G; g0 += NW * 8)
            stage_batch<NW, 8, false>(xm, x, hsrc, yres, hout, false, norm_w, g0, G, n4, lane, coherent, dig, prm, ss);
    }
    float fac = 1.0f;
    if (norm) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(JINF_FULL_MASK, ss, o);
        if (lane == 0) misc[warp] = ss;
    }
    __syncthreads();
    if (norm) {
        ss = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) ss += misc[w];
        fac = rsqrtf(ss / (float)cols + eps);
    }
    return fac;
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
    // Optional values prepared before the GEMV finished (shared memory, indexed by
    // row - pre_row0): EPI_RESID the current h of the row, EPI_QKV at the even row of a
    // q or k pair the RoPE cosine and at the odd row the sine (rope_pair). Null: computed here.
    const float* pre = nullptr;
    int pre_row0 = 0;
};

// RoPE rotation of the adjacent pair (row, row + 1) of a q or k head at position `pos`:
// theta = base^(-2i / hd), i = the pair's index in its head (reference cuda/rope_kernel.cu).
__device__ __forceinline__ void rope_pair(int rr, int pos, float base, int head_dim, float& cs, float& sn) {
    const int i = (rr % head_dim) >> 1;
    const float theta = powf(base, -2.0f * (float)i / (float)head_dim);
    const float ang = (float)pos * theta;
    cs = cosf(ang);
    sn = sinf(ang);
}

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
        const float h0 = a.pre ? a.pre[row - a.pre_row0] : a.coherent ? __ldcg(a.y + row) : a.y[row];
        a.y[row] = h0 + v0;
        if (row + 1 < a.rows) {
            const float h1 = a.pre ? a.pre[row + 1 - a.pre_row0] : a.coherent ? __ldcg(a.y + row + 1) : a.y[row + 1];
            a.y[row + 1] = h1 + v1;
        }
    } else if (a.epi == EPI_GATEUP) {
        a.y[row >> 1] = v0 / (1.0f + expf(-v0)) * v1;
    } else {  // EPI_QKV: rows are [q | k | v], each head_dim-aligned
        const int pos = a.pos;
        if (row < a.nq + a.nk) {
            const int rr = row < a.nq ? row : row - a.nq;
            float cs, sn;
            if (a.pre) {
                cs = a.pre[row - a.pre_row0];
                sn = a.pre[row + 1 - a.pre_row0];
            } else {
                rope_pair(rr, pos, a.rope_base, a.head_dim, cs, sn);
            }
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
