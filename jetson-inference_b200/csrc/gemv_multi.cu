// Multi-vector fused GEMV over the Q4M layout (q4m.cuh) on the tensor cores, sm_100a:
// Y[v] = W x[v] for up to 8 input vectors with one pass over W. It serves the engine's
// multi-sequence decode step (multi.h: the same prologues and epilogues as the one-token
// kernel-per-operation form, per vector) and the jinf_b200_gemv_q4m_batch* entry points
// (BASELINE config C2 at batch 4 and 8). The reference has no batched form; at one vector
// its arithmetic is cuda/matmul_kernels.cu:8-43 (Q4_0) and :104-185 (Q4_K, Q6_K, Q8_0).
//
// Arithmetic (q4m_device.cuh for one vector). The inputs are int8 digit records per
// 32-element block (alpha = 32639 / max|x|, v = rint(x alpha) = 256 hi + lo). In one
// m16n8k32 step the B operand's 8 columns hold digit h of vector 4 vb + c in column 2c + h,
// so one step multiplies a block of 16 rows by four vectors' digits and the accumulator
// columns (2c, 2c + 1) of a lane are vector c's hi and lo sums. Each block is finished on its
// own (its scale differs per row, its digit scale per vector): the step starts from the
// vector's zero-point offsets (Q4_0) and the block adds d (256 D_hi + D_lo) / alpha to the
// lane's rows. Vectors 4..7 take a second step per block. A lane ends a task with complete
// sums of rows gr, gr + 8, 16 + gr, 24 + gr of the tile pair for its vector(s); no lane
// reduction is needed.
//
// Scheduling. CTA c works on K part kp = c % kw only, so it stages just that part's records
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
// room for the records of several vectors (the larger Q6_K and Q8_0 units: 1 in flight).
__host__ __device__ constexpr inline int multi_nbuf(int fmt) { return fmt == Q4M_Q6_K || fmt == Q4M_Q8_0 ? 2 : 3; }

// Staged records: digits [n][gk][256 B] then params [n][gk][4][16 B], each vector's run padded
// (digits +64 B, params +16 B) so that the lanes of one load that read different vectors fall
// in different shared-memory banks.
__host__ __device__ inline int multi_dig_stride(int gk) { return gk * 256 + 64; }
__host__ __device__ inline int multi_prm_stride(int gk) { return gk * 64 + 16; }
__host__ __device__ inline int multi_pad(int n) { return (n + 3) & ~3; }  // staged vectors: whole blocks of 4
__host__ __device__ inline size_t multi_rec_bytes(int n, int gk) {
    return (size_t)multi_pad(n) * (multi_dig_stride(gk) + multi_prm_stride(gk));
}
// epilogue staging [MNW][MULTI_MAX][EP_STRIDE] floats, 64 floats of norm factors, the argmax
// keys [MNW][MULTI_MAX], the merged rows [MULTI_MAX][EP_STRIDE] (per-CTA split) and a flag
constexpr size_t MULTI_EP_BYTES =
    (size_t)MNW * MULTI_MAX * EP_STRIDE * 4 + 64 * 4 + MNW * MULTI_MAX * 8 + MULTI_MAX * EP_STRIDE * 4 + 16;

__host__ __device__ inline size_t multi_smem(int n, int gk, int fmt) {
    return multi_rec_bytes(n, gk) + MULTI_EP_BYTES + (size_t)MNW * multi_nbuf(fmt) * q4m_unit_bytes(fmt);
}

__device__ __forceinline__ void lds128(uint32_t a, uint32_t (&r)[4]) {
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}

// Staged records of one vector block (4 vectors) for block j of local group gl: the lane's B
// fragment (digit h = gr & 1 of vector 4 vb + gr / 2) and the params of its accumulator vector
// 4 vb + c (zero-point offsets kh, kl and the digit scales ia, ia / 16). The staged vectors are
// padded to a multiple of 4 with zero records, so every lane loads unconditionally; the lane's
// addresses for group 0, block 0 are computed once per kernel.
struct MultiRec {
    uint32_t dig[2], prm[2];  // shared addresses of vector blocks 0 and 1
};
__device__ __forceinline__ MultiRec multi_rec(uint32_t dig, uint32_t prm, int dstride, int pstride, int lane) {
    const int gr = lane >> 2, c = lane & 3;
    MultiRec r;
#pragma unroll
    for (int vb = 0; vb < 2; ++vb) {
        r.dig[vb] = dig + (uint32_t)((4 * vb + (gr >> 1)) * dstride + ((gr & 1) * 4 + c) * 8);
        r.prm[vb] = prm + (uint32_t)((4 * vb + c) * pstride);
    }
    return r;
}
__device__ __forceinline__ void rec_frag(const MultiRec& r, int vb, int j, int gl, uint32_t& b0, uint32_t& b1) {
    asm("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(b0), "=r"(b1) : "r"(r.dig[vb] + (uint32_t)(gl * 256 + j * 64)));
}
__device__ __forceinline__ void rec_prm(const MultiRec& r, int vb, int j, int gl, int& kh, int& kl, float& ia,
                                        float& ib) {
    asm("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
        : "=r"(kh), "=r"(kl), "=f"(ia), "=f"(ib)
        : "r"(r.prm[vb] + (uint32_t)(gl * 64 + j * 16)));
}

// Integer MMAs with a zero accumulator input (no register initialisation per step).
__device__ __forceinline__ void mma_u8s8_z(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1,
                                           int (&d)[4]) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %10, %10, %10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}
__device__ __forceinline__ void mma_s8s8_z(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1,
                                           int (&d)[4]) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %10, %10, %10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}
__device__ __forceinline__ void mma_s8s8_k16_z(uint32_t a0, uint32_t a1, uint32_t b0, int (&d)[4]) {
    asm("mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5}, {%6}, {%7, %7, %7, %7};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(b0), "r"(0));
}

// ---- one unit (32 rows x 128 columns) against NVB vector blocks, per weight format.
// The slot's scale words are read across lanes: the caller synchronises the warp before
// (after its copies landed) and after (before a lane copies the next unit into the slot).

template <int NVB>
__device__ __forceinline__ void unit_multi_q40(uint32_t sl, const MultiRec& r, int gl, int lane, float (&acc)[NVB][4]) {
    const int gr = lane >> 2;
    uint32_t w[16], sa[4], sb[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint32_t t[4];
        lds128(sl + 512 * j + lane * 16, t);
#pragma unroll
        for (int i = 0; i < 4; ++i) w[4 * j + i] = t[i];
    }
    lds128(sl + Q4M_SCALES + 16 * gr, sa);        // words 4 gr + j: rows gr, gr + 8 of block j
    lds128(sl + Q4M_SCALES + 128 + 16 * gr, sb);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float dA0 = jinf_h2f((uint16_t)(sa[j] & 0xffffu)), dA1 = jinf_h2f((uint16_t)(sa[j] >> 16));
        const float dB0 = jinf_h2f((uint16_t)(sb[j] & 0xffffu)), dB1 = jinf_h2f((uint16_t)(sb[j] >> 16));
#pragma unroll
        for (int vb = 0; vb < NVB; ++vb) {
            uint32_t b0, b1;
            int kh, kl;
            float ia, ib;
            rec_frag(r, vb, j, gl, b0, b1);
            rec_prm(r, vb, j, gl, kh, kl, ia, ib);
            // the zero-point offsets (kh, kl: -8 x the digit sums) added after the MMAs: the
            // (hi, lo) pair of tile A gets 256 kh + kl, tile B's (its operand carries 16 q) 16 x that
            const int k = kh * 256 + kl, k16 = k * 16;
            int da[4], db[4];
            mma_u8s8_z(nib_lo(w[4 * j]), nib_lo(w[4 * j + 1]), nib_lo(w[4 * j + 2]), nib_lo(w[4 * j + 3]), b0, b1, da);
            mma_u8s8_z(nib_hi(w[4 * j]), nib_hi(w[4 * j + 1]), nib_hi(w[4 * j + 2]), nib_hi(w[4 * j + 3]), b0, b1, db);
            acc[vb][0] = fmaf(dA0 * ia, (float)(da[0] * 256 + da[1] + k), acc[vb][0]);
            acc[vb][1] = fmaf(dA1 * ia, (float)(da[2] * 256 + da[3] + k), acc[vb][1]);
            acc[vb][2] = fmaf(dB0 * ib, (float)(db[0] * 256 + db[1] + k16), acc[vb][2]);
            acc[vb][3] = fmaf(dB1 * ib, (float)(db[2] * 256 + db[3] + k16), acc[vb][3]);
        }
    }
}

// Q4_K: no zero point; block j of row r contributes (d sc (256 D_hi + D_lo) -
// dmin m (256 S_hi + S_lo)) / alpha, S the block's digit sums recovered from the record's
// zero-point params (-8 S). Tile B's sums carry the 16 of its high-nibble operand, so its min
// term is taken x16 and the row scaled by 1 / (16 alpha).
template <int NVB>
__device__ __forceinline__ void unit_multi_q4k(uint32_t sl, const MultiRec& r, int gl, int lane, float (&acc)[NVB][4]) {
    const int gr = lane >> 2;
    uint32_t w[16], sa[4], sb[4], dm[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint32_t t[4];
        lds128(sl + 512 * j + lane * 16, t);
#pragma unroll
        for (int i = 0; i < 4; ++i) w[4 * j + i] = t[i];
    }
    lds128(sl + Q4M_SCALES + 16 * gr, sa);        // sc | m << 8 of rows gr (low half), gr + 8, block j
    lds128(sl + Q4M_SCALES + 128 + 16 * gr, sb);
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(dm[0]) : "r"(sl + Q4M_DMIN_K + gr * 4));
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(dm[1]) : "r"(sl + Q4M_DMIN_K + (gr + 8) * 4));
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(dm[2]) : "r"(sl + Q4M_DMIN_K + 64 + gr * 4));
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(dm[3]) : "r"(sl + Q4M_DMIN_K + 64 + (gr + 8) * 4));
    float d[4], m[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        d[i] = jinf_h2f((uint16_t)(dm[i] & 0xffffu));
        m[i] = jinf_h2f((uint16_t)(dm[i] >> 16));
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t scm[4] = {sa[j] & 0xffffu, sa[j] >> 16, sb[j] & 0xffffu, sb[j] >> 16};
        float sd[4], sm[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            sd[i] = d[i] * (float)(scm[i] & 63u);
            sm[i] = m[i] * (float)((scm[i] >> 8) & 63u);
        }
#pragma unroll
        for (int vb = 0; vb < NVB; ++vb) {
            uint32_t b0, b1;
            int kh, kl;
            float ia, ib;
            rec_frag(r, vb, j, gl, b0, b1);
            rec_prm(r, vb, j, gl, kh, kl, ia, ib);
            int da[4], db[4];
            mma_u8s8_z(nib_lo(w[4 * j]), nib_lo(w[4 * j + 1]), nib_lo(w[4 * j + 2]), nib_lo(w[4 * j + 3]), b0, b1, da);
            mma_u8s8_z(nib_hi(w[4 * j]), nib_hi(w[4 * j + 1]), nib_hi(w[4 * j + 2]), nib_hi(w[4 * j + 3]), b0, b1, db);
            const float S = (float)(-((kh << 8) + kl) >> 3);  // 256 S_hi + S_lo of the block (exact)
            acc[vb][0] = fmaf(fmaf(sd[0], (float)(da[0] * 256 + da[1]), -sm[0] * S), ia, acc[vb][0]);
            acc[vb][1] = fmaf(fmaf(sd[1], (float)(da[2] * 256 + da[3]), -sm[1] * S), ia, acc[vb][1]);
            acc[vb][2] = fmaf(fmaf(sd[2], (float)(db[0] * 256 + db[1]), -sm[2] * 16.0f * S), ib, acc[vb][2]);
            acc[vb][3] = fmaf(fmaf(sd[3], (float)(db[2] * 256 + db[3]), -sm[3] * 16.0f * S), ib, acc[vb][3]);
        }
    }
}

// Q6_K: each weight byte is rebuilt as the int8 value 4 (q - 32) from its nibble and flipped
// crumb; a scale covers 16 elements, so every block is two m16n8k16 steps per tile, one per
// half, into their own accumulators; block j of row r contributes
// d (sc_0 (256 D0_hi + D0_lo) + sc_1 (256 D1_hi + D1_lo)) / (4 alpha).
template <int NVB>
__device__ __forceinline__ void unit_multi_q6k(uint32_t sl, const MultiRec& r, int gl, int lane, float (&acc)[NVB][4]) {
    const int gr = lane >> 2;
    uint32_t w[16], cr[8], sc[8];
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
    uint32_t dlo, dhi;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(dlo), "=r"(dhi) : "r"(sl + Q4M_D_6 + gr * 8));
    const float d0 = jinf_h2f((uint16_t)(dlo & 0xffffu)), d1 = jinf_h2f((uint16_t)(dlo >> 16));
    const float d2 = jinf_h2f((uint16_t)(dhi & 0xffffu)), d3 = jinf_h2f((uint16_t)(dhi >> 16));
    constexpr uint32_t NM = 0x3C3C3C3Cu, CM = 0xC0C0C0C0u;
    auto scv = [](uint32_t v, int b) { return (float)(int8_t)(uint8_t)(v >> (8 * b)); };
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t* nw = w + 4 * j;
        const uint32_t h0 = cr[2 * j], h1 = cr[2 * j + 1];
        const uint32_t A0 = ((nw[0] << 2) & NM) | ((h0 << 6) & CM), B0 = ((nw[0] >> 2) & NM) | ((h0 << 4) & CM);
        const uint32_t A1 = ((nw[1] << 2) & NM) | ((h0 << 2) & CM), B1 = ((nw[1] >> 2) & NM) | (h0 & CM);
        const uint32_t A2 = ((nw[2] << 2) & NM) | ((h1 << 6) & CM), B2 = ((nw[2] >> 2) & NM) | ((h1 << 4) & CM);
        const uint32_t A3 = ((nw[3] << 2) & NM) | ((h1 << 2) & CM), B3 = ((nw[3] >> 2) & NM) | (h1 & CM);
        const uint32_t sca = sc[2 * j], scb = sc[2 * j + 1];
        // per row: the two half-block scales times d
        const float a00 = d0 * scv(sca, 0), a01 = d0 * scv(sca, 1), a10 = d1 * scv(sca, 2), a11 = d1 * scv(sca, 3);
        const float b00 = d2 * scv(scb, 0), b01 = d2 * scv(scb, 1), b10 = d3 * scv(scb, 2), b11 = d3 * scv(scb, 3);
#pragma unroll
        for (int vb = 0; vb < NVB; ++vb) {
            uint32_t x0, x1;
            int kh, kl;
            float ia, ib;
            rec_frag(r, vb, j, gl, x0, x1);
            rec_prm(r, vb, j, gl, kh, kl, ia, ib);
            int p0[4], p1[4], q0[4], q1[4];
            mma_s8s8_k16_z(A0, A1, x0, p0);
            mma_s8s8_k16_z(A2, A3, x1, p1);
            mma_s8s8_k16_z(B0, B1, x0, q0);
            mma_s8s8_k16_z(B2, B3, x1, q1);
            const float s = 0.25f * ia;
            auto dsum = [](const int (&h)[4], int rr) { return (float)(h[2 * rr] * 256 + h[2 * rr + 1]); };
            acc[vb][0] = fmaf(fmaf(a00, dsum(p0, 0), a01 * dsum(p1, 0)), s, acc[vb][0]);
            acc[vb][1] = fmaf(fmaf(a10, dsum(p0, 1), a11 * dsum(p1, 1)), s, acc[vb][1]);
            acc[vb][2] = fmaf(fmaf(b00, dsum(q0, 0), b01 * dsum(q1, 0)), s, acc[vb][2]);
            acc[vb][3] = fmaf(fmaf(b10, dsum(q0, 1), b11 * dsum(q1, 1)), s, acc[vb][3]);
        }
    }
}

// Q8_0: the weight words are the int8 q themselves, one m16n8k32 step per block and tile, no
// zero point; block j of row r contributes d (256 D_hi + D_lo) / alpha.
template <int NVB>
__device__ __forceinline__ void unit_multi_q80(uint32_t sl, const MultiRec& r, int gl, int lane, float (&acc)[NVB][4]) {
    const int gr = lane >> 2;
    uint32_t dd[8];
    {
        uint32_t t[4];
        lds128(sl + Q4M_D_8 + 32 * gr, t);  // blocks 0, 1: (rows gr, gr + 8), (16 + gr, 24 + gr)
#pragma unroll
        for (int i = 0; i < 4; ++i) dd[i] = t[i];
        lds128(sl + Q4M_D_8 + 32 * gr + 16, t);
#pragma unroll
        for (int i = 0; i < 4; ++i) dd[4 + i] = t[i];
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint32_t wa[4], wb[4];
        lds128(sl + 1024 * j + lane * 16, wa);
        lds128(sl + 1024 * j + 512 + lane * 16, wb);
        const float e0 = jinf_h2f((uint16_t)(dd[2 * j] & 0xffffu)), e1 = jinf_h2f((uint16_t)(dd[2 * j] >> 16));
        const float e2 = jinf_h2f((uint16_t)(dd[2 * j + 1] & 0xffffu)), e3 = jinf_h2f((uint16_t)(dd[2 * j + 1] >> 16));
#pragma unroll
        for (int vb = 0; vb < NVB; ++vb) {
            uint32_t x0, x1;
            int kh, kl;
            float ia, ib;
            rec_frag(r, vb, j, gl, x0, x1);
            rec_prm(r, vb, j, gl, kh, kl, ia, ib);
            int da[4], db[4];
            mma_s8s8_z(wa[0], wa[1], wa[2], wa[3], x0, x1, da);
            mma_s8s8_z(wb[0], wb[1], wb[2], wb[3], x0, x1, db);
            acc[vb][0] = fmaf(e0 * ia, (float)(da[0] * 256 + da[1]), acc[vb][0]);
            acc[vb][1] = fmaf(e1 * ia, (float)(da[2] * 256 + da[3]), acc[vb][1]);
            acc[vb][2] = fmaf(e2 * ia, (float)(db[0] * 256 + db[1]), acc[vb][2]);
            acc[vb][3] = fmaf(e3 * ia, (float)(db[2] * 256 + db[3]), acc[vb][3]);
        }
    }
}

template <int FMT, int NVB>
__device__ __forceinline__ void unit_multi(uint32_t sl, const MultiRec& r, int gl, int lane, float (&acc)[NVB][4]) {
    if (FMT == Q4M_Q4_K) unit_multi_q4k<NVB>(sl, r, gl, lane, acc);
    else if (FMT == Q4M_Q6_K) unit_multi_q6k<NVB>(sl, r, gl, lane, acc);
    else if (FMT == Q4M_Q8_0) unit_multi_q80<NVB>(sl, r, gl, lane, acc);
    else unit_multi_q40<NVB>(sl, r, gl, lane, acc);
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

// Epilogue of rows (row, row + 1) of tile pair q for vector v, values v0, v1 (valid: v < n).
// Every lane of the warp calls it with its own row pair of 16 (qq = lane & 15, one vector per
// half warp): ME_RESID adds the halves' sums of squares with shuffles.
template <int EPI>
__device__ __forceinline__ void multi_epilogue(const MultiParams& p, int q, int qq, int v, bool valid, float v0,
                                               float v1, float& lmax, int& lidx) {
    const int row = q * Q4M_PAIR_ROWS + 2 * qq;
    if (EPI == ME_RESID) {
        float s2 = 0.f, h0v = 0.f, h1v = 0.f;
        if (valid) {  // rows = the residual width (a multiple of 32): every row exists
            float* hy = p.y + (size_t)v * p.ldy + row;
            h0v = hy[0] + v0;
            h1v = hy[1] + v1;
            hy[0] = h0v;
            hy[1] = h1v;
            s2 = fmaf(h0v, h0v, h1v * h1v);
        }
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) s2 += __shfl_xor_sync(JINF_FULL_MASK, s2, o);
        if (valid && qq == 0) p.ssq_out[(size_t)q * p.n + v] = s2;
        if (p.rec_out) {
            // the pair is block q of the next GEMV's input: its records of h * gain_out. Octet
            // lane L of lanes 0..7 (vector 2k) and 8..15 (vector 2k + 1) takes elements 4L .. 4L+3,
            // the rows of half-warp lanes 2L and 2L + 1
            const int lane = threadIdx.x & 31, hh = (lane >> 3) & 1, L = lane & 7;
            const int src = 16 * hh + 2 * L;
            const float e0 = __shfl_sync(JINF_FULL_MASK, h0v, src), e1 = __shfl_sync(JINF_FULL_MASK, h1v, src);
            const float e2 = __shfl_sync(JINF_FULL_MASK, h0v, src + 1), e3 = __shfl_sync(JINF_FULL_MASK, h1v, src + 1);
            const int vv = v - (lane >> 4) + hh;  // v of lane 0 is 2k
            const bool st = lane < 16 && vv < p.n;
            float4 g = make_float4(0.f, 0.f, 0.f, 0.f);
            if (st) g = reinterpret_cast<const float4*>(p.gain_out + (size_t)q * Q4M_PAIR_ROWS)[L];
            const int gout = p.rows / Q4M_KG;
            uint8_t* base = p.rec_out + (size_t)(st ? vv : 0) * xrec_bytes(gout);
            octet_to_records(make_float4(e0 * g.x, e1 * g.y, e2 * g.z, e3 * g.w), lane, q & 3,
                             reinterpret_cast<uint32_t*>(base) + (q >> 2) * 64,
                             reinterpret_cast<float4*>(base + (size_t)gout * 256) + (q >> 2) * 4, st);
        }
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

template <int XM, int EPI, int FMT, int NVB>
__global__ void __launch_bounds__(MT, 1) k_gemv_multi(const MultiParams p) {
    constexpr int UB = q4m_unit_bytes(FMT);
    constexpr int NB = multi_nbuf(FMT);  // ring slots per warp
    extern __shared__ __align__(16) uint8_t smem_m[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = p.groups, kw = p.kw, gk = p.gk, n = p.n;
    const int kp = blockIdx.x % kw, cidx = blockIdx.x / kw;
    const int cg = ((int)gridDim.x - kp + kw - 1) / kw;  // CTAs of part kp
    const int g0 = kp * G / kw, g1 = (kp + 1) * G / kw, ng = g1 - g0;
    uint8_t* rec = smem_m;
    uint32_t* dig = reinterpret_cast<uint32_t*>(rec);
    float4* prm = reinterpret_cast<float4*>(rec + (size_t)multi_pad(n) * multi_dig_stride(gk));
    float* ep = reinterpret_cast<float*>(rec + multi_rec_bytes(n, gk));  // [MNW][MULTI_MAX][EP_STRIDE]
    float* fac = ep + MNW * MULTI_MAX * EP_STRIDE;                       // [MULTI_MAX] (64 floats)
    u64* keys = reinterpret_cast<u64*>(fac + 64);                        // [MNW][MULTI_MAX]
    float* fin = reinterpret_cast<float*>(keys + MNW * MULTI_MAX);      // [MULTI_MAX][EP_STRIDE]
    int* flag = reinterpret_cast<int*>(fin + MULTI_MAX * EP_STRIDE);
    const uint32_t ring = smem_u32(rec + multi_rec_bytes(n, gk) + MULTI_EP_BYTES) + (uint32_t)(warp * NB * UB);
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
    if (EPI == ME_QKV && tid == 32 && p.nk > 0) {
        // the attention after this GEMV reads every vector's cache rows 0 .. pos - 1 of this
        // layer: bring them into L2 now, one (vector, kv head, K or V) region per CTA. The
        // positions and sequences of the step were written before the step began.
        const int nkvh = p.nk / p.head_dim;
        for (int r = blockIdx.x; r < n * nkvh * 2; r += gridDim.x) {
            const int v = r / (nkvh * 2), kvh = (r >> 1) % nkvh;
            const __half* base = ((r & 1) ? p.vcache : p.kcache) + (size_t)p.ms->seq[v] * p.seq_stride +
                                 (size_t)kvh * p.max_ctx * p.head_dim;
            const uint32_t bytes = (uint32_t)p.ms->pos[v] * (uint32_t)p.head_dim * 2u;
            for (uint32_t o = 0; o < bytes; o += (1u << 20))
                prefetch_l2(reinterpret_cast<const uint8_t*>(base) + o, bytes - o < (1u << 20) ? bytes - o : (1u << 20));
        }
    }
    pdl_wait();
    pdl_trigger();

    // ---------------- prologue: norm factors (warp v < n adds vector v's partial sums of
    // squares: lane l the parts l, l + 32, ..., then a fixed shuffle tree), then the part's
    // records (one group of one vector per warp pass: lane l converts block l / 8, elements
    // 4 (l % 8) .. +3)
    if (warp < MULTI_MAX) {
        float f = 1.0f;
        if ((XM == MX_NORMED || (XM == MX_RECORDS && p.ssq)) && warp < n) {
            float ss = 0.f;
            for (int q0 = lane; q0 < p.ssq_parts; q0 += 8 * 32) {  // eight loads in flight
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
    if (XM == MX_RECORDS) {
        // records written by the producer (xrec layout per vector, xrec_bytes(G) apart): the
        // part's digit words and params, 16 bytes per thread and copy
        const uint8_t* src = reinterpret_cast<const uint8_t*>(p.x);
        const size_t vstride = xrec_bytes(G);
        const int dchunks = ng * 16, pchunks = ng * 4;  // 16-byte pieces per vector
        for (int i = tid; i < n * (dchunks + pchunks); i += MT) {
            const int v = i / (dchunks + pchunks), r = i % (dchunks + pchunks);
            const uint8_t* g = src + (size_t)v * vstride;
            uint32_t dst;
            if (r < dchunks) {
                g += (size_t)g0 * 256 + (size_t)r * 16;
                dst = smem_u32(dig) + (uint32_t)(v * multi_dig_stride(gk) + r * 16);
            } else {
                g += (size_t)G * 256 + (size_t)g0 * 64 + (size_t)(r - dchunks) * 16;
                dst = smem_u32(prm) + (uint32_t)(v * multi_prm_stride(gk) + (r - dchunks) * 16);
            }
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(g) : "memory");
        }
        asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
    }
    // a warp issues the loads of up to 8 of its items before converting any, so it pays one
    // L2 round trip per 8 items, not one per item
    const int n4 = p.cols / 4, items = XM == MX_RECORDS ? 0 : n * ng;
    for (int base = warp; base < items; base += 8 * MNW) {
        float4 x4[8];
#pragma unroll
        for (int b = 0; b < 8; ++b) {
            const int it = base + b * MNW;
            if (it < items) x4[b] = multi_load<XM>(p, it / ng, (g0 + it % ng) * 32 + lane, n4);
        }
#pragma unroll
        for (int b = 0; b < 8; ++b) {
            const int it = base + b * MNW;  // warp-uniform: the conversion's shuffles see every lane
            if (it >= items) break;
            const int v = it / ng, gl = it % ng;
            octet_to_records(x4[b], lane, lane >> 3, dig + (v * multi_dig_stride(gk) + gl * 256) / 4,
                             prm + (v * multi_prm_stride(gk) + gl * 64) / 16);
        }
    }
    // zero records for the padding vectors n .. multi_pad(n) - 1 (they contribute nothing)
    for (int i = tid; i < (multi_pad(n) - n) * (multi_dig_stride(gk) + multi_prm_stride(gk)) / 16; i += MT) {
        const int per_d = (multi_pad(n) - n) * multi_dig_stride(gk) / 16;
        uint4* dst = i < per_d ? reinterpret_cast<uint4*>(rec + (size_t)n * multi_dig_stride(gk)) + i
                               : reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(prm) + (size_t)n * multi_prm_stride(gk)) +
                                     (i - per_d);
        *dst = make_uint4(0u, 0u, 0u, 0u);
    }
    __syncthreads();
    const MultiRec mr = multi_rec(smem_u32(dig), smem_u32(prm), multi_dig_stride(gk), multi_prm_stride(gk), lane);

    // ---------------- main loop
    const int gr = lane >> 2, c = lane & 3;
    float lmax[2 * NVB];
    int lidx[2 * NVB];
#pragma unroll
    for (int k = 0; k < 2 * NVB; ++k) {
        lmax[k] = -INFINITY;
        lidx[k] = 0;
    }
    int slot = 0;
    if (local) {
        // ---------------- per CTA: all warps on one pair, each its groups [lg0, lg1)
        for (int q = cidx; q < p.pairs; q += cg) {
            float acc[NVB][4];
#pragma unroll
            for (int vb = 0; vb < NVB; ++vb)
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[vb][i] = 0.f;
            for (int gl = lg0; gl < lg1; ++gl) {
                issue(slot == 0 ? NB - 1 : slot - 1);
                asm volatile("cp.async.wait_group %0;" ::"n"(NB - 1) : "memory");
                __syncwarp();  // scale words are read across lanes
                unit_multi<FMT, NVB>(ring + slot * UB, mr, gl, lane, acc);
                __syncwarp();  // every lane's reads of the slot precede the next copy into it
                slot = slot + 1 == NB ? 0 : slot + 1;
            }
#pragma unroll
            for (int vb = 0; vb < NVB; ++vb) {
                const int v = 4 * vb + c;
                if (v < n)
#pragma unroll
                    for (int i = 0; i < 4; ++i) eps_w[v * EP_STRIDE + gr + 8 * i] = acc[vb][i];
            }
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
        float acc[NVB][4];
#pragma unroll
        for (int vb = 0; vb < NVB; ++vb)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[vb][i] = 0.f;
        for (int gl = 0; gl < ng; ++gl) {
            issue(slot == 0 ? NB - 1 : slot - 1);
            asm volatile("cp.async.wait_group %0;" ::"n"(NB - 1) : "memory");
            __syncwarp();  // scale words are read across lanes
            unit_multi<FMT, NVB>(ring + slot * UB, mr, gl, lane, acc);
            __syncwarp();  // every lane's reads of the slot precede the next copy into it
            slot = slot + 1 == NB ? 0 : slot + 1;
        }
        // the pair's rows to the warp's staging block: lane (gr, c) holds vector 4 vb + c,
        // rows gr + 8 i
#pragma unroll
        for (int vb = 0; vb < NVB; ++vb) {
            const int v = 4 * vb + c;
            if (v < n)
#pragma unroll
                for (int i = 0; i < 4; ++i) eps_w[v * EP_STRIDE + gr + 8 * i] = acc[vb][i];
        }
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
        for (int k = 0; k < 2 * NVB; ++k) {
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
        for (int k = 0; k < 2 * NVB; ++k) {
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

// One warp per 32-element chunk of a vector: h (+)= source, and the chunk's sum of squares;
// with rec, the chunk is block ch of the next GEMV's input: its digit records of h * gain
// (octet lane L of lanes 0..7 converts elements 4L .. 4L+3, the values of lanes 4L .. 4L+3).
__global__ void k_multi_rows(const float* __restrict__ table, const MultiState* __restrict__ ms, float* h,
                             const float* __restrict__ y, int n, int d, float* __restrict__ ssq, uint8_t* rec,
                             const float* __restrict__ gain) {
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int chunks = d / 32;
    const int wid = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    if (wid >= n * chunks) return;  // whole warps: the shuffles below see every lane
    const int v = wid / chunks, ch = wid % chunks;
    const size_t i = (size_t)v * d + ch * 32 + lane;
    float val;
    if (table) val = table[(size_t)ms->token[v] * d + ch * 32 + lane];  // the embedding row
    else val = h[i] + y[i];                                             // the residual add
    h[i] = val;
    const float s = warp_sum(val * val);
    if (lane == 0) ssq[(size_t)ch * n + v] = s;
    if (rec) {
        const float gv = val * gain[ch * 32 + lane];
        const int src = 4 * (lane & 7);
        const float4 e = make_float4(__shfl_sync(JINF_FULL_MASK, gv, src), __shfl_sync(JINF_FULL_MASK, gv, src + 1),
                                     __shfl_sync(JINF_FULL_MASK, gv, src + 2), __shfl_sync(JINF_FULL_MASK, gv, src + 3));
        const int G = d / Q4M_KG;
        uint8_t* base = rec + (size_t)v * xrec_bytes(G);
        octet_to_records(e, lane, ch & 3, reinterpret_cast<uint32_t*>(base) + (ch >> 2) * 64,
                         reinterpret_cast<float4*>(base + (size_t)G * 256) + (ch >> 2) * 4, lane < 8);
    }
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
                        uint8_t* rec, const float* gain, cudaStream_t s, bool pdl) {
    if (n < 1 || n > MULTI_MAX || d % 32 || !h || !ssq || (!table && !y) || (table && !ms))
        return cudaErrorInvalidValue;
    if (rec && (!gain || d % Q4M_KG)) return cudaErrorInvalidValue;
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
    return cudaLaunchKernelEx(&cfg, k_multi_rows, table, ms, h, y, n, d, ssq, rec, gain);
}

// ---------------------------------------------------------------- dispatch

template <int XM, int EPI, int FMT, int NVB>
cudaError_t launch_multi_t(const MultiParams& p, int grid, cudaStream_t s, bool pdl) {
    const size_t smem = multi_smem(p.n, p.gk, FMT);
    static size_t configured = 0;
    if (smem > configured) {
        const cudaError_t e =
            cudaFuncSetAttribute(k_gemv_multi<XM, EPI, FMT, NVB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
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
    return cudaLaunchKernelEx(&cfg, k_gemv_multi<XM, EPI, FMT, NVB>, p);
}

template <int XM, int EPI, int FMT>
cudaError_t launch_multi_n(const MultiParams& p, int grid, cudaStream_t s, bool pdl) {
    return p.n <= 4 ? launch_multi_t<XM, EPI, FMT, 1>(p, grid, s, pdl) : launch_multi_t<XM, EPI, FMT, 2>(p, grid, s, pdl);
}

template <int FMT>
cudaError_t launch_multi_f(const MultiParams& p, int xm, int epi, int grid, cudaStream_t s, bool pdl) {
    switch (xm * 16 + epi) {
        case MX_PLAIN_F32 * 16 + ME_STORE: return launch_multi_n<MX_PLAIN_F32, ME_STORE, FMT>(p, grid, s, pdl);
        case MX_PLAIN_F16 * 16 + ME_STORE: return launch_multi_n<MX_PLAIN_F16, ME_STORE, FMT>(p, grid, s, pdl);
        case MX_PLAIN_F32 * 16 + ME_RESID: return launch_multi_n<MX_PLAIN_F32, ME_RESID, FMT>(p, grid, s, pdl);
        case MX_NORMED * 16 + ME_QKV: return launch_multi_n<MX_NORMED, ME_QKV, FMT>(p, grid, s, pdl);
        case MX_NORMED * 16 + ME_GATEUP: return launch_multi_n<MX_NORMED, ME_GATEUP, FMT>(p, grid, s, pdl);
        case MX_NORMED * 16 + ME_LMHEAD: return launch_multi_n<MX_NORMED, ME_LMHEAD, FMT>(p, grid, s, pdl);
        case MX_RECORDS * 16 + ME_QKV: return launch_multi_n<MX_RECORDS, ME_QKV, FMT>(p, grid, s, pdl);
        case MX_RECORDS * 16 + ME_GATEUP: return launch_multi_n<MX_RECORDS, ME_GATEUP, FMT>(p, grid, s, pdl);
        case MX_RECORDS * 16 + ME_LMHEAD: return launch_multi_n<MX_RECORDS, ME_LMHEAD, FMT>(p, grid, s, pdl);
        case MX_RECORDS * 16 + ME_RESID: return launch_multi_n<MX_RECORDS, ME_RESID, FMT>(p, grid, s, pdl);
        case MX_RECORDS * 16 + ME_STORE: return launch_multi_n<MX_RECORDS, ME_STORE, FMT>(p, grid, s, pdl);
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
// trip costs about the same), fitted to B200 measurements of the 8B and 70B layer shapes at
// 2, 4 and 8 vectors:
//   per warp: the busiest warp's pairs x (the part's groups, plus, with kw > 1, its partial
//     rows, the arrival and the final sums: n loads per lane per part, eight in flight, 1.2
//     units per round of loads);
//   per CTA, one K part only: 2.5 + rounds of pairs x (the warp's share of the groups + 0.9
//     for the three barriers and the 16-warp merge of each pair);
// both plus the CTA's input staging spread over its 16 warps (n x the part's groups: 0.7
// units each when converted from fp32, 0.15 when copied as records). The per-CTA form wins
// where the pairs are about as many as the CTAs and one part holds every group (the 8B QKV,
// o and gate|up projections); with several K parts it lost every measured case, so it is
// not considered there; the per-warp form with several K parts wins elsewhere.
void multi_plan(int pairs, int groups, int n, int fmt, int grid, int epi, int xm, int* kw_out, int* local_out) {
    *kw_out = 0;
    *local_out = 0;
    if (pairs < 1 || groups < 1 || n < 1 || n > MULTI_MAX || grid < 1) return;
    const double stage = xm == MX_RECORDS ? 0.15 : 0.7;
    double best = 1e300;
    const int lim = groups < kMultiMaxKw ? groups : kMultiMaxKw;
    for (int kw = 1; kw <= lim; ++kw) {
        const int gk = (groups + kw - 1) / kw;
        if (multi_smem(n, gk, fmt) > 226 * 1024) continue;
        const int cg = grid / kw > 0 ? grid / kw : 1;  // CTAs of the least served part
        const long long warps = (long long)cg * MNW;
        const double pw = (double)((pairs + warps - 1) / warps);
        const double st = stage * n * gk / MNW;
        const double cost_w = pw * (gk + (kw > 1 ? 1.0 + 1.2 * n * ((kw + 7) / 8) : 0.0)) + st;
        if (cost_w < best - 1e-9) {
            best = cost_w;
            *kw_out = kw;
            *local_out = 0;
        }
        if (epi == ME_LMHEAD || kw > 1) continue;
        const double rounds = (double)((pairs + cg - 1) / cg);
        const double cost_l = 2.5 + rounds * ((gk + MNW - 1) / MNW + 0.9) + st;
        if (cost_l < best - 1e-9) {
            best = cost_l;
            *kw_out = kw;
            *local_out = 1;
        }
    }
}

int multi_pick_kw(int pairs, int groups, int n, int fmt, int grid) {
    int kw, local;
    multi_plan(pairs, groups, n, fmt, grid, ME_STORE, MX_PLAIN_F32, &kw, &local);
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
    if (xm == MX_RECORDS && (p.cols % Q4M_KG || (p.ssq && p.ssq_parts < 1))) return cudaErrorInvalidValue;
    if (epi == ME_RESID && (!p.ssq_out || p.rows % 32)) return cudaErrorInvalidValue;
    if (p.rec_out && (epi != ME_RESID || !p.gain_out || p.rows % Q4M_KG)) return cudaErrorInvalidValue;
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
                               uint8_t* rec, const float* gain, cudaStream_t s, bool pdl) {
    if (!table) return cudaErrorInvalidValue;
    return launch_rows(table, ms, h, nullptr, n, d, ssq, rec, gain, s, pdl);
}

cudaError_t multi_resid_launch(float* h, const float* y, int n, int d, float* ssq, uint8_t* rec, const float* gain,
                               cudaStream_t s, bool pdl) {
    if (!y) return cudaErrorInvalidValue;
    return launch_rows(nullptr, nullptr, h, y, n, d, ssq, rec, gain, s, pdl);
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
        multi_plan(sh.pairs, sh.groups, batch, fmt, grid, ME_STORE, MX_PLAIN_F32, &kw, &local);
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
