// Multi-vector fused GEMV over the Q4M layout (q4m.cuh) on the tensor cores, sm_100a:
// Y[v] = W x[v] for up to 8 input vectors with one pass over W. It serves the engine's
// multi-sequence decode step (multi.h: the same prologues and epilogues as the one-token
// kernel-per-operation form, per vector) and the jinf_b200_gemv_q4m_batch* entry points
// (BASELINE config C2 at batch 4 and 8). The reference has no batched form; at one vector
// its arithmetic is cuda/matmul_kernels.cu:8-43 (Q4_0) and :104-185 (Q4_K, Q6_K, Q8_0).
//
// Arithmetic. One mma.m16n8k16 (f16 x f16 -> f32) multiplies 16 rows by 16 columns of all 8
// vectors at once: the vectors are the MMA's 8 columns.
//   A (weights): each lane turns the 4-bit (6-, 8-bit) codes of its unit words straight into
//     fp16 fragments of the exact integer weights: the byte code q becomes the fp16 1024 + q
//     (0x64 as the high byte) minus the format's offset, with no rounding. A unit word holds
//     columns 4c .. 4c + 3 of rows gr or gr + 8 (low nibbles: tile A, high: tile B); the MMA's
//     logical columns (2c, 2c+1 | 2c+8, 2c+9) are mapped to them, and the B fragments follow
//     the same map.
//   B (inputs): the K part's columns of every vector in shared memory as two fp16 terms,
//     hi = fp16(x s) and lo = fp16(x s - hi) (about 22 significant bits together), each vector
//     scaled by a power of two s that puts its largest magnitude in [2^13, 2^14) (undone
//     exactly on the outputs); lane (gr, c) reads hi and lo of columns 4c .. 4c + 3 of
//     vector gr as one 16-byte load, and the MMA runs once per term.
//   The block's scale (per row, per 32 columns; Q6_K: per 16) multiplies its fp32 sums
//     after its MMAs, as the reference applies d to each block's sum
//     (cuda/matmul_kernels.cu:8-43); Q4_K subtracts dmin m times the block's input sum.
// So the weights are exact, the inputs carry ~22 bits relative to their maximum, and every
// sum is fp32.
//
// Scheduling. CTA c works on K part kp = c % kw only, so it stages just that part's inputs
// (n vectors x gk groups) in shared memory. Two ways to share out a part's work:
//   per warp (many tile pairs, e.g. an LM head): the CTA's warps take tile pairs, each warp
//     all of the part's groups of its pair; consecutive pairs go to different CTAs;
//   per CTA (p.local: at most a few pairs per CTA, the projections of a layer): the CTA takes
//     tile pairs and its 16 warps split the part's groups of each, meeting in shared memory in
//     warp order, so no warp idles for want of a pair and few partials leave the CTA.
// Each warp streams its units through a private cp.async ring that runs ahead across pairs;
// the first units are requested before the kernel waits on its producer (programmatic
// dependent launch). With kw > 1 each (pair, part) leaves its n x 32 partial rows in the
// workspace and the last one of a pair (arrival counter, reset by it) adds them in K order,
// so results are deterministic. The pair's rows are staged in shared memory and the
// epilogue runs on adjacent row pairs.
#include "common.cuh"
#include "gemv.h"
#include "jinf/b200.h"
#include "jinf/quant.h"
#include "multi.h"
#include "q4m.cuh"
#include "q4m_device.cuh"

#include <math.h>

namespace jinf {

using namespace q4mdev;

namespace {

constexpr int MT = 512;               // threads per CTA
constexpr int MNW = MT / 32;          // warps
constexpr int kMultiMaxKw = 32;
constexpr int EP_STRIDE = 33;         // floats per staged row block (32 rows, padded)

// Ring slots per warp: 2 in flight per warp keep HBM busy with 16 warps per SM, and leave
// room for the inputs (the larger Q6_K and Q8_0 units: 1 in flight).
__host__ __device__ constexpr inline int multi_nbuf(int fmt) { return fmt == Q4M_Q6_K || fmt == Q4M_Q8_0 ? 2 : 3; }

// Staged inputs: per vector a row of 16-byte records, one per 4 columns (hi of the 4, then lo),
// padded by 64 bytes so that the two rows one quarter-warp load reads fall in different
// banks; then the inputs' sums per 32-column block [gk * 4][MULTI_MAX] floats (Q4_K's min
// term).
__host__ __device__ inline int multi_xs_stride(int gk) { return gk * 512 + 64; }  // bytes per vector
__host__ __device__ inline size_t multi_xs_bytes(int n, int gk) {
    return (size_t)n * multi_xs_stride(gk) + (size_t)gk * 4 * MULTI_MAX * 4;
}
// epilogue staging [MNW][MULTI_MAX][EP_STRIDE] floats, 64 floats of per-vector factors (norm,
// input scale, maximum), the argmax keys [MNW][MULTI_MAX], the merged rows
// [MULTI_MAX][EP_STRIDE] (per-CTA split) and a flag
constexpr size_t MULTI_EP_BYTES =
    (size_t)MNW * MULTI_MAX * EP_STRIDE * 4 + 64 * 4 + MNW * MULTI_MAX * 8 + MULTI_MAX * EP_STRIDE * 4 + 16;

__host__ __device__ inline size_t multi_smem(int n, int gk, int fmt) {
    return multi_xs_bytes(n, gk) + MULTI_EP_BYTES + (size_t)MNW * multi_nbuf(fmt) * q4m_unit_bytes(fmt);
}

__device__ __forceinline__ void lds128(uint32_t a, uint32_t (&r)[4]) {
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}

__device__ __forceinline__ void mma_f16(const uint32_t (&a)[4], uint32_t b0, uint32_t b1, float (&d)[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ __half2 as_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }
__device__ __forceinline__ uint32_t as_u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
// bytes 0, 1 (lo) or 2, 3 (hi) of a word of 8-bit codes as the fp16 pair (1024 + b, 1024 + b')
__device__ __forceinline__ __half2 codes_lo(uint32_t t) { return as_h2(__byte_perm(t, 0x64646464u, 0x4140)); }
__device__ __forceinline__ __half2 codes_hi(uint32_t t) { return as_h2(__byte_perm(t, 0x64646464u, 0x4342)); }

// Lane (gr, c)'s inputs: vector gr's row of records + 16 c bytes (the lanes of vectors gr >= n
// take zeros), and its two vector columns' block sums (Q4_K).
struct XFrag {
    uint32_t row;   // shared address
    uint32_t sblk;  // shared address of block sums [block][MULTI_MAX] + vector 2c
    bool on;
};
// hi (b[0], b[1]) and lo (b[2], b[3]) terms of the B fragment of the 16 columns from `col`
__device__ __forceinline__ void xfrag(const XFrag& x, int col, uint32_t (&b)[4]) {
    b[0] = b[1] = b[2] = b[3] = 0u;
    if (x.on)
        asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(b[0]), "=r"(b[1]), "=r"(b[2]), "=r"(b[3])
                     : "r"(x.row + 4u * (uint32_t)col));
}
// the block sums of vector columns 2c, 2c + 1 at block `blk` of the part
__device__ __forceinline__ float2 xsums(const XFrag& x, int blk) {
    float2 r;
    asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(r.x), "=f"(r.y) : "r"(x.sblk + (uint32_t)blk * MULTI_MAX * 4));
    return r;
}
// the A fragment of one 16-column step from its two code words (row gr: t0, row gr + 8: t1;
// bytes = codes of columns 4c .. 4c + 3): code - off, exact
__device__ __forceinline__ void frag_exact(uint32_t t0, uint32_t t1, __half2 off, uint32_t (&a)[4]) {
    a[0] = as_u(__hsub2(codes_lo(t0), off));
    a[1] = as_u(__hsub2(codes_lo(t1), off));
    a[2] = as_u(__hsub2(codes_hi(t0), off));
    a[3] = as_u(__hsub2(codes_hi(t1), off));
}
// A times both input terms, into d
__device__ __forceinline__ void mma_hl(const uint32_t (&a)[4], const uint32_t (&b)[4], float (&d)[4]) {
    mma_f16(a, b[0], b[1], d);
    mma_f16(a, b[2], b[3], d);
}
// small non-negative integer -> float without the conversion unit (exact below 2^23)
__device__ __forceinline__ float small_u2f(uint32_t u) { return __uint_as_float(0x4B000000u | u) - 8388608.0f; }

// ---- one unit (32 rows x 128 columns) of local group gl against the 8 vector columns, per
// weight format. accA: rows gr, gr + 8 (tile A), accB: 16 + gr, 24 + gr (tile B), vector
// columns 2c, 2c + 1 (c0, c1: the first row; c2, c3: the second). The slot's scale words are
// read across lanes: the caller synchronises the warp before (after its copies landed) and
// after (before a lane copies the next unit into the slot).

__device__ __forceinline__ void unit_f16_q40(uint32_t sl, const XFrag& x, int gl, int lane, float (&accA)[4],
                                             float (&accB)[4]) {
    const int gr = lane >> 2;
    uint32_t w[16], sa[4], sb[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint32_t t[4];
        lds128(sl + 512 * j + lane * 16, t);
#pragma unroll
        for (int i = 0; i < 4; ++i) w[4 * j + i] = t[i];
    }
    lds128(sl + Q4M_SCALES + 16 * gr, sa);  // words 4 gr + j: d of rows gr (low), gr + 8 (high), block j
    lds128(sl + Q4M_SCALES + 128 + 16 * gr, sb);
    const __half2 off = __float2half2_rn(1032.f);  // 1024 + the zero point 8: codes q - 8
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        float bA[4] = {0.f, 0.f, 0.f, 0.f}, bB[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int s = 0; s < 2; ++s) {
            const uint32_t r0 = w[4 * j + 2 * s], r1 = w[4 * j + 2 * s + 1];
            uint32_t fa[4], fb[4], xb[4];
            frag_exact(r0 & 0x0F0F0F0Fu, r1 & 0x0F0F0F0Fu, off, fa);
            frag_exact((r0 >> 4) & 0x0F0F0F0Fu, (r1 >> 4) & 0x0F0F0F0Fu, off, fb);
            xfrag(x, gl * 128 + 32 * j + 16 * s, xb);
            mma_hl(fa, xb, bA);
            mma_hl(fb, xb, bB);
        }
        const float a0 = jinf_h2f((uint16_t)(sa[j] & 0xffffu)), a1 = jinf_h2f((uint16_t)(sa[j] >> 16));
        const float b0 = jinf_h2f((uint16_t)(sb[j] & 0xffffu)), b1 = jinf_h2f((uint16_t)(sb[j] >> 16));
        accA[0] = fmaf(a0, bA[0], accA[0]);
        accA[1] = fmaf(a0, bA[1], accA[1]);
        accA[2] = fmaf(a1, bA[2], accA[2]);
        accA[3] = fmaf(a1, bA[3], accA[3]);
        accB[0] = fmaf(b0, bB[0], accB[0]);
        accB[1] = fmaf(b0, bB[1], accB[1]);
        accB[2] = fmaf(b1, bB[2], accB[2]);
        accB[3] = fmaf(b1, bB[3], accB[3]);
    }
}

// Q4_K: weight d sc q - dmin m (reference src/quant.cpp:71-77): per row and 32-column block,
// d sc times the block's sum of q x, minus dmin m times the block's sum of x.
__device__ __forceinline__ void unit_f16_q4k(uint32_t sl, const XFrag& x, int gl, int lane, float (&accA)[4],
                                             float (&accB)[4]) {
    const int gr = lane >> 2;
    uint32_t w[16], sa[4], sb[4], dm[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint32_t t[4];
        lds128(sl + 512 * j + lane * 16, t);
#pragma unroll
        for (int i = 0; i < 4; ++i) w[4 * j + i] = t[i];
    }
    lds128(sl + Q4M_SCALES + 16 * gr, sa);  // sc | m << 8 of rows gr (low half), gr + 8, block j
    lds128(sl + Q4M_SCALES + 128 + 16 * gr, sb);
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(dm[0]) : "r"(sl + Q4M_DMIN_K + gr * 4));
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(dm[1]) : "r"(sl + Q4M_DMIN_K + (gr + 8) * 4));
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(dm[2]) : "r"(sl + Q4M_DMIN_K + 64 + gr * 4));
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(dm[3]) : "r"(sl + Q4M_DMIN_K + 64 + (gr + 8) * 4));
    float d[4], mn[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        d[i] = jinf_h2f((uint16_t)(dm[i] & 0xffffu));
        mn[i] = jinf_h2f((uint16_t)(dm[i] >> 16));
    }
    const __half2 off = __float2half2_rn(1024.f);  // codes q
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        float bA[4] = {0.f, 0.f, 0.f, 0.f}, bB[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int s = 0; s < 2; ++s) {
            const uint32_t r0 = w[4 * j + 2 * s], r1 = w[4 * j + 2 * s + 1];
            uint32_t fa[4], fb[4], xb[4];
            frag_exact(r0 & 0x0F0F0F0Fu, r1 & 0x0F0F0F0Fu, off, fa);
            frag_exact((r0 >> 4) & 0x0F0F0F0Fu, (r1 >> 4) & 0x0F0F0F0Fu, off, fb);
            xfrag(x, gl * 128 + 32 * j + 16 * s, xb);
            mma_hl(fa, xb, bA);
            mma_hl(fb, xb, bB);
        }
        const float2 S = xsums(x, gl * 4 + j);
        // the four rows' (d sc, dmin m) of block j
        const uint32_t qa = sa[j], qb = sb[j];
        const float ka0 = d[0] * small_u2f(qa & 63u), ma0 = mn[0] * small_u2f((qa >> 8) & 63u);
        const float ka1 = d[1] * small_u2f((qa >> 16) & 63u), ma1 = mn[1] * small_u2f((qa >> 24) & 63u);
        const float kb0 = d[2] * small_u2f(qb & 63u), mb0 = mn[2] * small_u2f((qb >> 8) & 63u);
        const float kb1 = d[3] * small_u2f((qb >> 16) & 63u), mb1 = mn[3] * small_u2f((qb >> 24) & 63u);
        accA[0] = fmaf(ka0, bA[0], fmaf(-ma0, S.x, accA[0]));
        accA[1] = fmaf(ka0, bA[1], fmaf(-ma0, S.y, accA[1]));
        accA[2] = fmaf(ka1, bA[2], fmaf(-ma1, S.x, accA[2]));
        accA[3] = fmaf(ka1, bA[3], fmaf(-ma1, S.y, accA[3]));
        accB[0] = fmaf(kb0, bB[0], fmaf(-mb0, S.x, accB[0]));
        accB[1] = fmaf(kb0, bB[1], fmaf(-mb0, S.y, accB[1]));
        accB[2] = fmaf(kb1, bB[2], fmaf(-mb1, S.x, accB[2]));
        accB[3] = fmaf(kb1, bB[3], fmaf(-mb1, S.y, accB[3]));
    }
}

// Q6_K: the 6-bit code as the int8 4 (q - 32) (nibble and flipped crumb, as the one-vector
// path builds it), exact in fp16 through the 0x80 flip; each 16-column half has its own scale,
// so a half's sums take d sc / 4 of their row (reference cuda/dequant_kernels.cu:82-110).
__device__ __forceinline__ void unit_f16_q6k(uint32_t sl, const XFrag& x, int gl, int lane, float (&accA)[4],
                                             float (&accB)[4]) {
    const int gr = lane >> 2;
    uint32_t w[16], cr[8], sc[8], dlo, dhi;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint32_t t[4];
        lds128(sl + 512 * j + lane * 16, t);
#pragma unroll
        for (int i = 0; i < 4; ++i) w[4 * j + i] = t[i];
    }
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
        uint32_t t[4];
        lds128(sl + Q4M_CRUMB_6 + 512 * jj + lane * 16, t);
#pragma unroll
        for (int i = 0; i < 4; ++i) cr[4 * jj + i] = t[i];
        lds128(sl + Q4M_SC_6 + 32 * gr + 16 * jj, t);  // blocks 2 jj, 2 jj + 1: tile A word, tile B word
#pragma unroll
        for (int i = 0; i < 4; ++i) sc[4 * jj + i] = t[i];
    }
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(dlo), "=r"(dhi) : "r"(sl + Q4M_D_6 + gr * 8));
    const float d0 = 0.25f * jinf_h2f((uint16_t)(dlo & 0xffffu)), d1 = 0.25f * jinf_h2f((uint16_t)(dlo >> 16));
    const float d2 = 0.25f * jinf_h2f((uint16_t)(dhi & 0xffffu)), d3 = 0.25f * jinf_h2f((uint16_t)(dhi >> 16));
    const __half2 off = __float2half2_rn(1152.f);  // 1024 + the 0x80 flip
    constexpr uint32_t NM = 0x3C3C3C3Cu, CM = 0xC0C0C0C0u, FL = 0x80808080u;
    auto scv = [](uint32_t v, int b) { return (float)(int8_t)(uint8_t)(v >> (8 * b)); };
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t* nw = w + 4 * j;
        const uint32_t h0 = cr[2 * j], h1 = cr[2 * j + 1];
        // int8 4 (q - 32) of tiles A (low nibbles) and B (high), words i = 0..3, flipped by 0x80
        const uint32_t A[4] = {(((nw[0] << 2) & NM) | ((h0 << 6) & CM)) ^ FL, (((nw[1] << 2) & NM) | ((h0 << 2) & CM)) ^ FL,
                               (((nw[2] << 2) & NM) | ((h1 << 6) & CM)) ^ FL, (((nw[3] << 2) & NM) | ((h1 << 2) & CM)) ^ FL};
        const uint32_t B[4] = {(((nw[0] >> 2) & NM) | ((h0 << 4) & CM)) ^ FL, (((nw[1] >> 2) & NM) | (h0 & CM)) ^ FL,
                               (((nw[2] >> 2) & NM) | ((h1 << 4) & CM)) ^ FL, (((nw[3] >> 2) & NM) | (h1 & CM)) ^ FL};
        const uint32_t sca = sc[2 * j], scb = sc[2 * j + 1];  // bytes 2u + h: row gr + 8u, half h
#pragma unroll
        for (int s = 0; s < 2; ++s) {
            float bA[4] = {0.f, 0.f, 0.f, 0.f}, bB[4] = {0.f, 0.f, 0.f, 0.f};
            uint32_t fa[4], fb[4], xb[4];
            frag_exact(A[2 * s], A[2 * s + 1], off, fa);
            frag_exact(B[2 * s], B[2 * s + 1], off, fb);
            xfrag(x, gl * 128 + 32 * j + 16 * s, xb);
            mma_hl(fa, xb, bA);
            mma_hl(fb, xb, bB);
            const float ka0 = d0 * scv(sca, s), ka1 = d1 * scv(sca, 2 + s);
            const float kb0 = d2 * scv(scb, s), kb1 = d3 * scv(scb, 2 + s);
            accA[0] = fmaf(ka0, bA[0], accA[0]);
            accA[1] = fmaf(ka0, bA[1], accA[1]);
            accA[2] = fmaf(ka1, bA[2], accA[2]);
            accA[3] = fmaf(ka1, bA[3], accA[3]);
            accB[0] = fmaf(kb0, bB[0], accB[0]);
            accB[1] = fmaf(kb0, bB[1], accB[1]);
            accB[2] = fmaf(kb1, bB[2], accB[2]);
            accB[3] = fmaf(kb1, bB[3], accB[3]);
        }
    }
}

// Q8_0: the int8 code, exact in fp16 through the 0x80 flip; the block's sums take the row's d.
__device__ __forceinline__ void unit_f16_q80(uint32_t sl, const XFrag& x, int gl, int lane, float (&accA)[4],
                                             float (&accB)[4]) {
    const int gr = lane >> 2;
    uint32_t dd[8];
    {
        uint32_t t[4];
        lds128(sl + Q4M_D_8 + 32 * gr, t);  // blocks 0, 1: (d of rows gr, gr + 8), (16 + gr, 24 + gr)
#pragma unroll
        for (int i = 0; i < 4; ++i) dd[i] = t[i];
        lds128(sl + Q4M_D_8 + 32 * gr + 16, t);
#pragma unroll
        for (int i = 0; i < 4; ++i) dd[4 + i] = t[i];
    }
    const __half2 off = __float2half2_rn(1152.f);
    constexpr uint32_t FL = 0x80808080u;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint32_t wa[4], wb[4];
        lds128(sl + 1024 * j + lane * 16, wa);
        lds128(sl + 1024 * j + 512 + lane * 16, wb);
        float bA[4] = {0.f, 0.f, 0.f, 0.f}, bB[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int s = 0; s < 2; ++s) {
            uint32_t fa[4], fb[4], xb[4];
            frag_exact(wa[2 * s] ^ FL, wa[2 * s + 1] ^ FL, off, fa);
            frag_exact(wb[2 * s] ^ FL, wb[2 * s + 1] ^ FL, off, fb);
            xfrag(x, gl * 128 + 32 * j + 16 * s, xb);
            mma_hl(fa, xb, bA);
            mma_hl(fb, xb, bB);
        }
        const float e0 = jinf_h2f((uint16_t)(dd[2 * j] & 0xffffu)), e1 = jinf_h2f((uint16_t)(dd[2 * j] >> 16));
        const float e2 = jinf_h2f((uint16_t)(dd[2 * j + 1] & 0xffffu)), e3 = jinf_h2f((uint16_t)(dd[2 * j + 1] >> 16));
        accA[0] = fmaf(e0, bA[0], accA[0]);
        accA[1] = fmaf(e0, bA[1], accA[1]);
        accA[2] = fmaf(e1, bA[2], accA[2]);
        accA[3] = fmaf(e1, bA[3], accA[3]);
        accB[0] = fmaf(e2, bB[0], accB[0]);
        accB[1] = fmaf(e2, bB[1], accB[1]);
        accB[2] = fmaf(e3, bB[2], accB[2]);
        accB[3] = fmaf(e3, bB[3], accB[3]);
    }
}

template <int FMT>
__device__ __forceinline__ void unit_f16(uint32_t sl, const XFrag& x, int gl, int lane, float (&accA)[4],
                                         float (&accB)[4]) {
    if (FMT == Q4M_Q4_K) unit_f16_q4k(sl, x, gl, lane, accA, accB);
    else if (FMT == Q4M_Q6_K) unit_f16_q6k(sl, x, gl, lane, accA, accB);
    else if (FMT == Q4M_Q8_0) unit_f16_q80(sl, x, gl, lane, accA, accB);
    else unit_f16_q40(sl, x, gl, lane, accA, accB);
}

// Input of vector v at elements 4 i .. 4 i + 3 (zero past cols).
template <int XM>
__device__ __forceinline__ float4 multi_load(const MultiParams& p, int v, int i, int n4) {
    if (i >= n4) return make_float4(0.f, 0.f, 0.f, 0.f);
    if (XM == MX_PLAIN_F16) {
        const uint2 hv = *reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(p.x) + (size_t)v * p.ldx + 4 * i);
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&hv.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&hv.y));
        return make_float4(a.x, a.y, b.x, b.y);
    }
    float4 h = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p.x) + (size_t)v * p.ldx + 4 * i);
    if (XM == MX_NORMED) {
        const float4 g = reinterpret_cast<const float4*>(p.norm_w)[i];
        h = make_float4(h.x * g.x, h.y * g.y, h.z * g.z, h.w * g.w);
    }
    return h;
}

// The power of two s that puts a positive maximum in [2^13, 2^14) (1 for a zero maximum):
// scaled by s, the vector's fp16 values keep 11 significant bits and stay far below the
// fp16 maximum.
__device__ __forceinline__ float pow2_scale(float amax) {
    if (!(amax > 0.f)) return 1.0f;
    int e = (int)((__float_as_uint(amax) >> 23) & 0xFFu) - 127;  // amax in [2^e, 2^(e+1)) (normal)
    e = 13 - e;
    e = e > 126 ? 126 : e < -126 ? -126 : e;
    return __uint_as_float((uint32_t)(e + 127) << 23);
}

// Epilogue of rows (row, row + 1) of tile pair q for vector v, values v0, v1 (valid: v < n).
// Every lane of the warp calls it with its own row pair of 16 (qq = lane & 15, one vector per
// half warp): ME_RESID adds the halves' sums of squares with shuffles.
template <int EPI>
__device__ __forceinline__ void multi_epilogue(const MultiParams& p, int q, int qq, int v, bool valid, float v0,
                                               float v1, float& lmax, int& lidx) {
    const int row = q * Q4M_PAIR_ROWS + 2 * qq;
    if (EPI == ME_RESID) {
        float s2 = 0.f;
        if (valid) {  // rows = the residual width (a multiple of 32): every row exists
            float* hy = p.y + (size_t)v * p.ldy + row;
            const float h0 = hy[0] + v0, h1 = hy[1] + v1;
            hy[0] = h0;
            hy[1] = h1;
            s2 = fmaf(h0, h0, h1 * h1);
        }
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) s2 += __shfl_xor_sync(JINF_FULL_MASK, s2, o);
        if (valid && qq == 0) p.ssq_out[(size_t)q * p.n + v] = s2;
        return;
    }
    if (!valid) return;
    EpiArgs ea;
    ea.rows = p.rows;
    ea.y = p.y + (size_t)v * p.ldy;
    ea.coherent = false;
    if (EPI == ME_QKV) {
        const size_t so = (size_t)p.ms->seq[v] * p.seq_stride;
        ea.epi = EPI_QKV;
        ea.kcache = p.kcache + so;
        ea.vcache = p.vcache + so;
        ea.nq = p.nq;
        ea.nk = p.nk;
        ea.head_dim = p.head_dim;
        ea.max_ctx = p.max_ctx;
        ea.pos = p.ms->pos[v];
        ea.rope_base = p.rope_base;
    } else {
        ea.epi = EPI == ME_GATEUP ? EPI_GATEUP : EPI == ME_LMHEAD ? EPI_LMHEAD : EPI_STORE;
        ea.pos = 0;
    }
    epilogue_pair(ea, row, v0, v1, lmax, lidx);
}


template <int XM, int EPI, int FMT>
__global__ void __launch_bounds__(MT, 1) k_gemv_multi(const MultiParams p) {
    constexpr int UB = q4m_unit_bytes(FMT);
    constexpr int NB = multi_nbuf(FMT);  // ring slots per warp
    extern __shared__ __align__(16) uint8_t smem_m[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = p.groups, kw = p.kw, gk = p.gk, n = p.n;
    const int kp = blockIdx.x % kw, cidx = blockIdx.x / kw;
    const int cg = ((int)gridDim.x - kp + kw - 1) / kw;  // CTAs of part kp
    const int g0 = kp * G / kw, g1 = (kp + 1) * G / kw, ng = g1 - g0;
    const int xsb = multi_xs_stride(gk);
    uint8_t* xs = smem_m;                                                     // [n][xsb] fp16 input records
    float* sblk = reinterpret_cast<float*>(xs + (size_t)n * xsb);             // [gk * 4][MULTI_MAX] block sums
    float* ep = reinterpret_cast<float*>(smem_m + multi_xs_bytes(n, gk));    // [MNW][MULTI_MAX][EP_STRIDE]
    float* fac = ep + MNW * MULTI_MAX * EP_STRIDE;  // [v] norm factor, [8 + v] 1 / s, [16 + v] max, [24 + v] s
    u64* keys = reinterpret_cast<u64*>(fac + 64);                            // [MNW][MULTI_MAX]
    float* fin = reinterpret_cast<float*>(keys + MNW * MULTI_MAX);          // [MULTI_MAX][EP_STRIDE]
    int* flag = reinterpret_cast<int*>(fin + MULTI_MAX * EP_STRIDE);
    const uint32_t ring = smem_u32(smem_m + multi_xs_bytes(n, gk) + MULTI_EP_BYTES) + (uint32_t)(warp * NB * UB);
    float* eps_w = ep + warp * MULTI_MAX * EP_STRIDE;

    // ---------------- weight stream: per warp, pairs cidx + cg (warp + MNW i) of K part kp,
    // groups [0, ng) of each; per CTA (local), pairs cidx + cg i, groups [lg0, lg1) of each
    const bool local = p.local != 0;
    const int lg0 = warp * ng / MNW, lg1 = (warp + 1) * ng / MNW;
    const int wstep = local ? cg : cg * MNW;
    const int cg0 = local ? lg0 : 0, cg1 = local ? lg1 : ng;
    int cq = local ? cidx : cidx + cg * warp, cgl = cg0;  // copy cursor
    auto issue = [&](int slot) {
        if (cq < p.pairs && cg0 < cg1) {
            copy_unit_fmt<FMT>(ring + slot * UB, p.w + ((size_t)cq * G + g0 + cgl) * UB, lane);
            if (++cgl == cg1) {
                cgl = cg0;
                cq += wstep;
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");  // possibly empty: uniform group counts
    };
#pragma unroll
    for (int i = 0; i < NB - 1; ++i) issue(i);
    if (tid == 0 && p.pf_bytes) {
        const uint64_t share = ((p.pf_bytes + gridDim.x - 1) / gridDim.x + 15) & ~15ull;
        const uint64_t off = share * blockIdx.x;
        if (off < p.pf_bytes) {
            const uint64_t len = share < p.pf_bytes - off ? share : p.pf_bytes - off;
            for (uint64_t o = 0; o < len; o += (1ull << 20))
                prefetch_l2(p.pf_ptr + off + o, (uint32_t)(len - o < (1ull << 20) ? len - o : (1ull << 20)));
        }
    }
    pdl_wait();
    pdl_trigger();

    // ---------------- prologue: norm factors (warp v < n adds vector v's partial sums of
    // squares, eight loads in flight per lane, then a fixed shuffle tree); the part's inputs as
    // fp16, each vector scaled by the power of two of its part's maximum (two passes over the
    // items (vector, group), a warp's loads of up to 8 items issued before any is used)
    if (tid < MULTI_MAX) reinterpret_cast<int*>(fac)[16 + tid] = 0;
    if (warp < MULTI_MAX) {
        float f = 1.0f;
        if (XM == MX_NORMED && warp < n) {
            float ss = 0.f;
            for (int q0 = lane; q0 < p.ssq_parts; q0 += 8 * 32) {
                float t[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int q = q0 + 32 * i;
                    t[i] = q < p.ssq_parts ? p.ssq[(size_t)q * n + warp] : 0.f;
                }
#pragma unroll
                for (int i = 0; i < 8; ++i) ss += t[i];
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(JINF_FULL_MASK, ss, o);
            f = rsqrtf(ss / (float)p.cols + p.eps);
        }
        if (lane == 0) fac[warp] = f;
    }
    __syncthreads();
    const int n4 = p.cols / 4, items = n * ng;
    for (int base = warp; base < items; base += 8 * MNW) {  // pass 1: the maxima
        float4 x4[8];
#pragma unroll
        for (int b = 0; b < 8; ++b) {
            const int it = base + b * MNW;
            if (it < items) x4[b] = multi_load<XM>(p, it / ng, (g0 + it % ng) * 32 + lane, n4);
        }
#pragma unroll
        for (int b = 0; b < 8; ++b) {
            const int it = base + b * MNW;  // warp-uniform
            if (it >= items) break;
            float m = fmaxf(fmaxf(fabsf(x4[b].x), fabsf(x4[b].y)), fmaxf(fabsf(x4[b].z), fabsf(x4[b].w)));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(JINF_FULL_MASK, m, o));
            if (lane == 0) atomicMax(reinterpret_cast<int*>(fac) + 16 + it / ng, __float_as_int(m));
        }
    }
    __syncthreads();
    if (tid < n) {
        const float s = pow2_scale(__int_as_float(reinterpret_cast<int*>(fac)[16 + tid]));
        fac[24 + tid] = s;
        fac[8 + tid] = 1.0f / s;  // a power of two: exact
    }
    __syncthreads();
    for (int base = warp; base < items; base += 8 * MNW) {  // pass 2: scaled fp16 inputs
        float4 x4[8];
#pragma unroll
        for (int b = 0; b < 8; ++b) {
            const int it = base + b * MNW;
            if (it < items) x4[b] = multi_load<XM>(p, it / ng, (g0 + it % ng) * 32 + lane, n4);
        }
#pragma unroll
        for (int b = 0; b < 8; ++b) {
            const int it = base + b * MNW;
            if (it >= items) break;
            const int v = it / ng, gl = it % ng;
            const float s = fac[24 + v];
            const float e0 = x4[b].x * s, e1 = x4[b].y * s, e2 = x4[b].z * s, e3 = x4[b].w * s;
            const __half2 h01 = __floats2half2_rn(e0, e1), h23 = __floats2half2_rn(e2, e3);
            const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
            const __half2 l01 = __floats2half2_rn(e0 - f01.x, e1 - f01.y), l23 = __floats2half2_rn(e2 - f23.x, e3 - f23.y);
            *reinterpret_cast<uint4*>(xs + (size_t)v * xsb + (size_t)(gl * 32 + lane) * 16) =
                make_uint4(as_u(h01), as_u(h23), as_u(l01), as_u(l23));
            // the block's sum (lanes 8 i .. 8 i + 7 hold block i of the group)
            float bs = (e0 + e1) + (e2 + e3);
            bs += __shfl_xor_sync(JINF_FULL_MASK, bs, 1);
            bs += __shfl_xor_sync(JINF_FULL_MASK, bs, 2);
            bs += __shfl_xor_sync(JINF_FULL_MASK, bs, 4);
            if ((lane & 7) == 0) sblk[(gl * 4 + (lane >> 3)) * MULTI_MAX + v] = bs;
        }
    }
    __syncthreads();
    const int gr = lane >> 2, c = lane & 3;
    const XFrag xf{smem_u32(xs) + (uint32_t)(gr * xsb + 16 * c), smem_u32(sblk) + (uint32_t)(8 * c), gr < n};
    // a lane's sums -> the warp's staging block (true scale): rows gr, gr + 8, 16 + gr, 24 + gr of
    // vector columns 2c, 2c + 1
    auto stage_rows = [&](const float (&aA)[4], const float (&aB)[4]) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int v = 2 * c + h;
            if (v < n) {
                const float is = fac[8 + v];
                eps_w[v * EP_STRIDE + gr] = aA[h] * is;
                eps_w[v * EP_STRIDE + gr + 8] = aA[2 + h] * is;
                eps_w[v * EP_STRIDE + gr + 16] = aB[h] * is;
                eps_w[v * EP_STRIDE + gr + 24] = aB[2 + h] * is;
            }
        }
    };
    // ---------------- main loop
    float lmax[4];
    int lidx[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        lmax[k] = -INFINITY;
        lidx[k] = 0;
    }
    int slot = 0;
    if (local) {
        // ---------------- per CTA: all warps on one pair, each its groups [lg0, lg1)
        for (int q = cidx; q < p.pairs; q += cg) {
            float accA[4] = {0.f, 0.f, 0.f, 0.f}, accB[4] = {0.f, 0.f, 0.f, 0.f};
            for (int gl = lg0; gl < lg1; ++gl) {
                issue(slot == 0 ? NB - 1 : slot - 1);
                asm volatile("cp.async.wait_group %0;" ::"n"(NB - 1) : "memory");
                __syncwarp();  // scale words are read across lanes
                unit_f16<FMT>(ring + slot * UB, xf, gl, lane, accA, accB);
                __syncwarp();  // every lane's reads of the slot precede the next copy into it
                slot = slot + 1 == NB ? 0 : slot + 1;
            }
            stage_rows(accA, accB);
            __syncthreads();
            // the warps' pieces in warp order (warps without groups wrote zeros)
            if (tid < n * 32) {
                const int v = tid >> 5, r = tid & 31;
                float sum = 0.f;
#pragma unroll
                for (int w2 = 0; w2 < MNW; ++w2) sum += ep[(w2 * MULTI_MAX + v) * EP_STRIDE + r];
                if (kw > 1) p.part[((size_t)q * kw + kp) * n * 32 + tid] = sum;
                else fin[v * EP_STRIDE + r] = sum;
            }
            if (kw > 1) {
                __threadfence();
                __syncthreads();
                if (tid == 0) {
                    const unsigned old = atomicAdd(p.cnt + q, 1u);
                    *flag = old == (unsigned)(kw - 1);
                    if (*flag) p.cnt[q] = 0u;  // ready for the next launch
                }
                __syncthreads();
                if (!*flag) continue;  // another K part finishes this pair
                __threadfence();
                if (tid < n * 32) {  // the parts in K order, eight loads in flight
                    const float* pb = p.part + (size_t)q * kw * n * 32 + tid;
                    const size_t kst = (size_t)n * 32;
                    float sum = 0.f;
                    for (int k0 = 0; k0 < kw; k0 += 8) {
                        float t[8];
#pragma unroll
                        for (int i = 0; i < 8; ++i) t[i] = k0 + i < kw ? __ldcg(pb + (size_t)(k0 + i) * kst) : 0.f;
#pragma unroll
                        for (int i = 0; i < 8; ++i) sum += t[i];
                    }
                    fin[(tid >> 5) * EP_STRIDE + (tid & 31)] = sum;
                }
            }
            __syncthreads();
            if (warp < (n + 1) / 2) {  // row pair qq of vector 2 warp + lane / 16
                const int qq = lane & 15, v = 2 * warp + (lane >> 4);
                const bool valid = v < n;
                const float f = valid ? fac[v] : 0.f;
                const float v0 = valid ? fin[v * EP_STRIDE + 2 * qq] * f : 0.f;
                const float v1 = valid ? fin[v * EP_STRIDE + 2 * qq + 1] * f : 0.f;
                float lm = -INFINITY;
                int li = 0;
                multi_epilogue<EPI>(p, q, qq, v, valid, v0, v1, lm, li);
            }
            __syncthreads();  // the staging blocks are rewritten by the next pair
        }
    }
    for (int q = local ? p.pairs : cidx + cg * warp; q < p.pairs && ng > 0; q += wstep) {
        float accA[4] = {0.f, 0.f, 0.f, 0.f}, accB[4] = {0.f, 0.f, 0.f, 0.f};
        for (int gl = 0; gl < ng; ++gl) {
            issue(slot == 0 ? NB - 1 : slot - 1);
            asm volatile("cp.async.wait_group %0;" ::"n"(NB - 1) : "memory");
            __syncwarp();  // scale words are read across lanes
            unit_f16<FMT>(ring + slot * UB, xf, gl, lane, accA, accB);
            __syncwarp();  // every lane's reads of the slot precede the next copy into it
            slot = slot + 1 == NB ? 0 : slot + 1;
        }
        stage_rows(accA, accB);
        __syncwarp();
        if (kw > 1) {
            float* pt = p.part + ((size_t)q * kw + kp) * n * 32;
            for (int e = lane; e < n * 32; e += 32) pt[e] = eps_w[(e >> 5) * EP_STRIDE + (e & 31)];
            __threadfence();
            __syncwarp();
            unsigned old = 0;
            if (lane == 0) old = atomicAdd(p.cnt + q, 1u);
            old = __shfl_sync(JINF_FULL_MASK, old, 0);
            if (old != (unsigned)(kw - 1)) continue;  // another K part finishes this pair
            __threadfence();
            if (lane == 0) p.cnt[q] = 0u;  // ready for the next launch
            // the parts in K order, eight loads in flight per lane
            const float* pb = p.part + (size_t)q * kw * n * 32;
            const size_t kst = (size_t)n * 32;
            for (int e = lane; e < n * 32; e += 32) {
                float s = 0.f;
                for (int k0 = 0; k0 < kw; k0 += 8) {
                    float t[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) t[i] = k0 + i < kw ? __ldcg(pb + (size_t)(k0 + i) * kst + e) : 0.f;
#pragma unroll
                    for (int i = 0; i < 8; ++i) s += t[i];
                }
                eps_w[(e >> 5) * EP_STRIDE + (e & 31)] = s;
            }
            __syncwarp();
        }
        // ---------------- epilogue: lane handles row pair (2 (lane & 15), +1) of vector
        // 2 k + lane / 16, k = 0 .. ceil(n / 2) - 1
        const int qq = lane & 15;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            if (2 * k >= n) break;
            const int v = 2 * k + (lane >> 4);
            const bool valid = v < n;
            const float f = valid ? fac[v] : 0.f;
            const float v0 = valid ? eps_w[v * EP_STRIDE + 2 * qq] * f : 0.f;
            const float v1 = valid ? eps_w[v * EP_STRIDE + 2 * qq + 1] * f : 0.f;
            multi_epilogue<EPI>(p, q, qq, v, valid, v0, v1, lmax[k], lidx[k]);
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");

    if (EPI == ME_LMHEAD) {
        // per vector: the warp's argmax (first index wins on ties), then the CTA's, then one
        // atomicMax per CTA and vector
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            if (2 * k >= n) break;
            const int v = 2 * k + (lane >> 4);
            u64 key = lmax[k] == -INFINITY ? 0ull : argmax_key(lmax[k], lidx[k] + p.vocab_offset);
#pragma unroll
            for (int o = 1; o < 16; o <<= 1) {
                const u64 other = __shfl_xor_sync(JINF_FULL_MASK, key, o);
                key = other > key ? other : key;
            }
            if ((lane & 15) == 0 && v < n) keys[warp * MULTI_MAX + v] = key;
        }
        __syncthreads();
        if (tid < n) {
            u64 best = 0ull;
            for (int w2 = 0; w2 < MNW; ++w2) best = keys[w2 * MULTI_MAX + tid] > best ? keys[w2 * MULTI_MAX + tid] : best;
            if (best) atomicMax(&p.ms->best[tid], best);
        }
    }
}

// ---------------------------------------------------------------- small steps of the multi step

// One warp per 32-element chunk of a vector: h (+)= source, and the chunk's sum of squares.
__global__ void k_multi_rows(const float* __restrict__ table, const MultiState* __restrict__ ms, float* h,
                             const float* __restrict__ y, int n, int d, float* __restrict__ ssq) {
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int chunks = d / 32;
    const int wid = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    if (wid >= n * chunks) return;
    const int v = wid / chunks, ch = wid % chunks;
    const size_t i = (size_t)v * d + ch * 32 + lane;
    float val;
    if (table) val = table[(size_t)ms->token[v] * d + ch * 32 + lane];  // the embedding row
    else val = h[i] + y[i];                                             // the residual add
    h[i] = val;
    const float s = warp_sum(val * val);
    if (lane == 0) ssq[(size_t)ch * n + v] = s;
}

__global__ void k_multi_finalize(MultiState* ms, int n) {
    const int v = threadIdx.x;
    if (v >= n) return;
    const u64 key = ms->best[v];
    const int tok = key ? (int)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull)) : 0;
    ms->out_token[v] = tok;
    ms->best[v] = 0ull;
    if (ms->feedback) {
        ms->token[v] = tok;
        ms->pos[v] += 1;
    }
}

cudaError_t launch_rows(const float* table, const MultiState* ms, float* h, const float* y, int n, int d, float* ssq,
                        cudaStream_t s, bool pdl) {
    if (n < 1 || n > MULTI_MAX || d % 32 || !h || !ssq || (!table && !y) || (table && !ms))
        return cudaErrorInvalidValue;
    const int warps = n * (d / 32);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((warps + 7) / 8));
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_multi_rows, table, ms, h, y, n, d, ssq);
}

// ---------------------------------------------------------------- dispatch

template <int XM, int EPI, int FMT>
cudaError_t launch_multi_t(const MultiParams& p, int grid, cudaStream_t s, bool pdl) {
    const size_t smem = multi_smem(p.n, p.gk, FMT);
    static size_t configured = 0;
    if (smem > configured) {
        const cudaError_t e =
            cudaFuncSetAttribute(k_gemv_multi<XM, EPI, FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        configured = smem;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(MT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_gemv_multi<XM, EPI, FMT>, p);
}

template <int FMT>
cudaError_t launch_multi_f(const MultiParams& p, int xm, int epi, int grid, cudaStream_t s, bool pdl) {
    switch (xm * 16 + epi) {
        case MX_PLAIN_F32 * 16 + ME_STORE: return launch_multi_t<MX_PLAIN_F32, ME_STORE, FMT>(p, grid, s, pdl);
        case MX_PLAIN_F16 * 16 + ME_STORE: return launch_multi_t<MX_PLAIN_F16, ME_STORE, FMT>(p, grid, s, pdl);
        case MX_PLAIN_F32 * 16 + ME_RESID: return launch_multi_t<MX_PLAIN_F32, ME_RESID, FMT>(p, grid, s, pdl);
        case MX_NORMED * 16 + ME_QKV: return launch_multi_t<MX_NORMED, ME_QKV, FMT>(p, grid, s, pdl);
        case MX_NORMED * 16 + ME_GATEUP: return launch_multi_t<MX_NORMED, ME_GATEUP, FMT>(p, grid, s, pdl);
        case MX_NORMED * 16 + ME_LMHEAD: return launch_multi_t<MX_NORMED, ME_LMHEAD, FMT>(p, grid, s, pdl);
        default: return cudaErrorInvalidValue;
    }
}

int device_sms() {
    static int sms[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (!sms[dev]) {
        int v = 148;
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        sms[dev] = v;
    }
    return sms[dev];
}

}  // namespace

int multi_grid(int num_sms) { return num_sms; }

// Estimated time, in units of one unit's streaming time per warp (at full HBM rate a warp
// streams one unit while the other 15 warps of its SM stream theirs; a dependent global round
// trip costs about the same):
//   per warp: the busiest warp's pairs x the part's groups, plus, with kw > 1, its partial rows,
//     the arrival and the final sums (n loads per lane per part, eight in flight);
//   per CTA: rounds of pairs x (the warp's share of the part's groups + the merge), plus, with
//     kw > 1, the arrival and the final sums (one load per thread per part, eight in flight).
void multi_plan(int pairs, int groups, int n, int fmt, int grid, int epi, int* kw_out, int* local_out) {
    *kw_out = 0;
    *local_out = 0;
    if (pairs < 1 || groups < 1 || n < 1 || n > MULTI_MAX || grid < 1) return;
    double best = 1e300;
    const int lim = groups < kMultiMaxKw ? groups : kMultiMaxKw;
    for (int kw = 1; kw <= lim; ++kw) {
        const int gk = (groups + kw - 1) / kw;
        if (multi_smem(n, gk, fmt) > 226 * 1024) continue;
        const int cg = grid / kw > 0 ? grid / kw : 1;  // CTAs of the least served part
        const long long warps = (long long)cg * MNW;
        const double pw = (double)((pairs + warps - 1) / warps);
        const double cost_w = pw * (gk + (kw > 1 ? 1.0 + n * ((kw + 7) / 8) : 0.0));
        if (cost_w < best - 1e-9) {
            best = cost_w;
            *kw_out = kw;
            *local_out = 0;
        }
        if (epi == ME_LMHEAD) continue;
        const double rounds = (double)((pairs + cg - 1) / cg);
        const double cost_l = rounds * ((gk + MNW - 1) / MNW + 0.5) + (kw > 1 ? 1.0 + (kw + 7) / 8 : 0.0);
        if (cost_l < best - 1e-9) {
            best = cost_l;
            *kw_out = kw;
            *local_out = 1;
        }
    }
}

int multi_pick_kw(int pairs, int groups, int n, int fmt, int grid) {
    int kw, local;
    multi_plan(pairs, groups, n, fmt, grid, ME_STORE, &kw, &local);
    return kw;
}

size_t multi_workspace_bytes(int pairs, int kw, int n) {
    return (size_t)pairs * kw * n * 32 * sizeof(float) + (size_t)pairs * sizeof(unsigned int);
}

cudaError_t multi_gemv_launch(const MultiParams& p, int xm, int epi, int grid, cudaStream_t s, bool pdl) {
    if (!p.w || !p.x || !p.y || p.n < 1 || p.n > MULTI_MAX || p.kw < 1 || p.kw > p.groups || grid < p.kw)
        return cudaErrorInvalidValue;
    if (p.gk != (p.groups + p.kw - 1) / p.kw || multi_smem(p.n, p.gk, p.fmt) > 226 * 1024) return cudaErrorInvalidValue;
    if (p.kw > 1 && (!p.part || !p.cnt || (size_t)p.pairs * p.kw * p.n * 32 > p.part_floats ||
                     (size_t)p.pairs > p.cnt_n))
        return cudaErrorInvalidValue;
    if (p.cols % 4 || p.ldx < p.cols) return cudaErrorInvalidValue;
    if (xm == MX_NORMED && (!p.norm_w || !p.ssq || p.ssq_parts < 1)) return cudaErrorInvalidValue;
    if (epi == ME_RESID && (!p.ssq_out || p.rows % 32)) return cudaErrorInvalidValue;
    if ((epi == ME_QKV || epi == ME_LMHEAD) && !p.ms) return cudaErrorInvalidValue;
    if (p.local && epi == ME_LMHEAD) return cudaErrorInvalidValue;
    if (epi == ME_QKV && (!p.kcache || !p.vcache)) return cudaErrorInvalidValue;
    switch (p.fmt) {
        case Q4M_Q4_0: return launch_multi_f<Q4M_Q4_0>(p, xm, epi, grid, s, pdl);
        case Q4M_Q4_K: return launch_multi_f<Q4M_Q4_K>(p, xm, epi, grid, s, pdl);
        case Q4M_Q6_K: return launch_multi_f<Q4M_Q6_K>(p, xm, epi, grid, s, pdl);
        case Q4M_Q8_0: return launch_multi_f<Q4M_Q8_0>(p, xm, epi, grid, s, pdl);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t multi_embed_launch(const float* table, const MultiState* ms, int n, int d, float* h, float* ssq,
                               cudaStream_t s, bool pdl) {
    if (!table) return cudaErrorInvalidValue;
    return launch_rows(table, ms, h, nullptr, n, d, ssq, s, pdl);
}

cudaError_t multi_resid_launch(float* h, const float* y, int n, int d, float* ssq, cudaStream_t s, bool pdl) {
    if (!y) return cudaErrorInvalidValue;
    return launch_rows(nullptr, nullptr, h, y, n, d, ssq, s, pdl);
}

cudaError_t multi_finalize_launch(MultiState* ms, int n, cudaStream_t s) {
    if (!ms || n < 1 || n > MULTI_MAX) return cudaErrorInvalidValue;
    k_multi_finalize<<<1, 32, 0, s>>>(ms, n);
    return cudaGetLastError();
}

}  // namespace jinf

using namespace jinf;

// ---------------------------------------------------------------- C-ABI (config C2 at batch 4 / 8)

extern "C" size_t jinf_b200_gemv_q4m_batch_workspace_bytes(int rows, int cols, int batch) {
    Q4MShape sh;
    if (!q4m_shape(rows, cols, &sh) || batch < 1 || batch > MULTI_MAX) return 0;
    return multi_workspace_bytes(sh.pairs, kMultiMaxKw, batch);
}

extern "C" size_t jinf_b200_gemv_q4m_batch_workspace_bytes_qt(int rows, int cols, int batch, int qtype) {
    Q4MShape sh;
    const int fmt = q4m_fmt_of_qtype(qtype);
    if (fmt < 0 || !q4m_shape(rows, cols, &sh, fmt) || batch < 1 || batch > MULTI_MAX) return 0;
    return multi_workspace_bytes(sh.pairs, kMultiMaxKw, batch);
}

extern "C" jinf_status jinf_b200_gemv_q4m_batch_qt(const void* q4m, int qtype, const void* x, int x_type, float* y,
                                                  int rows, int cols, int batch, void* workspace, int kw,
                                                  cudaStream_t stream) {
    Q4MShape sh;
    const int fmt = q4m_fmt_of_qtype(qtype);
    if (!q4m || !x || !y || fmt < 0 || !q4m_shape(rows, cols, &sh, fmt) || batch < 1 || batch > MULTI_MAX)
        return JINF_ERR_INVALID;
    if (x_type != JINF_TYPE_F32 && x_type != JINF_TYPE_F16) return JINF_ERR_INVALID;
    const int grid = multi_grid(device_sms());
    int local = 0;
    if (kw == 0) {
        multi_plan(sh.pairs, sh.groups, batch, fmt, grid, ME_STORE, &kw, &local);
    } else if (kw < 0) {  // a forced split with the per-CTA sharing
        kw = -kw;
        local = 1;
    }
    if (kw < 1 || kw > sh.groups || kw > kMultiMaxKw || multi_smem(batch, (sh.groups + kw - 1) / kw, fmt) > 226 * 1024)
        return JINF_ERR_INVALID;
    if (kw > 1 && !workspace) return JINF_ERR_INVALID;
    MultiParams p{};
    p.w = (const uint8_t*)q4m;
    p.rows = rows;
    p.cols = cols;
    p.pairs = sh.pairs;
    p.groups = sh.groups;
    p.fmt = fmt;
    p.n = batch;
    p.kw = kw;
    p.gk = (sh.groups + kw - 1) / kw;
    p.local = local;
    p.x = x;
    p.ldx = cols;
    p.y = y;
    p.ldy = rows;
    if (kw > 1) {
        p.part = (float*)workspace;
        p.cnt = (unsigned int*)((uint8_t*)workspace + (size_t)sh.pairs * kMultiMaxKw * batch * 32 * sizeof(float));
        p.part_floats = (size_t)sh.pairs * kMultiMaxKw * batch * 32;
        p.cnt_n = (size_t)sh.pairs;
    }
    const cudaError_t e =
        multi_gemv_launch(p, x_type == JINF_TYPE_F16 ? MX_PLAIN_F16 : MX_PLAIN_F32, ME_STORE, grid, stream, false);
    return e == cudaSuccess ? JINF_OK : JINF_ERR_CUDA;
}

extern "C" jinf_status jinf_b200_gemv_q4m_batch(const void* q4m, const void* x, int x_type, float* y, int rows,
                                               int cols, int batch, void* workspace, cudaStream_t stream) {
    return jinf_b200_gemv_q4m_batch_qt(q4m, JINF_TYPE_Q4_0, x, x_type, y, rows, cols, batch, workspace, 0, stream);
}
