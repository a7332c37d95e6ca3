// Q4M: the engine's HBM layout for Q4_0 weight matrices, shaped for the tensor-core GEMV
// (q4m_device.cuh: mma.sync m16n8k32, u8 weights x s8 input digits, s32 accumulation). It
// is a lossless repack of the reference's 18-byte AoS blocks (reference
// include/jinf/quant.h:31-35): every nibble and every fp16 scale is moved, none is
// re-quantised.
//
// Geometry. A matrix [rows][cols] is cut into tile pairs of 32 rows (two MMA tiles of 16:
// tile A = rows 0..15 of the pair, tile B = rows 16..31) and groups of 128 columns (four
// Q4_0 blocks j = 0..3). The bytes of one (pair P, group G) form one contiguous 2304-byte
// unit at byte (P * groups + G) * 2304, so a matrix streams front to back:
//   bytes    0 .. 2047   [4 blocks j][32 lanes][4 words i]   nibbles (word (j, i) of lane L
//                         at byte 512 j + 16 L + 4 i)
//   bytes 2048 .. 2175   [32 lanes][2 x fp16]   tile A: d(row gr, block c), d(row gr+8, block c)
//   bytes 2176 .. 2303   [32 lanes][2 x fp16]   tile B: the same for rows 16+gr, 24+gr
// for lane L = 4 gr + c (gr = 0..7, c = 0..3). Rows past `rows` and blocks past cols/32 are
// zero (nibbles 0, scale 0).
//
// MMA mapping. Word i of block j of lane (gr, c) is the lane's A register i of the
// m16n8k32 step that multiplies block j (k = element of the block):
//   i = 0: row gr,   k = 4c + b        i = 2: row gr,   k = 16 + 4c + b
//   i = 1: row gr+8, k = 4c + b        i = 3: row gr+8, k = 16 + 4c + b
// for byte b = 0..3 of the word. The byte's low nibble is q of that row of tile A, its high
// nibble q of the same row of tile B. So w & 0x0F0F0F0F is tile A's A register (u8 values
// q) and w & 0xF0F0F0F0 tile B's (u8 values 16 q): one lop3 decodes four weights.
//
// Block element e = 2i of the reference block is the low nibble of qs byte i, e = 2i+1 the
// high nibble (reference src/quant.cpp:49-60, cuda/matmul_kernels.cu:27-34).
//
// Q4_K matrices (reference include/jinf/quant.h:38-46: 256-element super-blocks, d and dmin
// in fp16, a 6-bit scale sc and min m per 32-element sub-block, w = d sc q - dmin m) use
// the same unit with a larger scale area (Q4M_UNIT_K = 2432 bytes): the four blocks of
// group G are sub-blocks 4 (G % 2) + j of super-block G / 2, their nibbles laid out as above,
// then
//   bytes 2048 .. 2175   [32 lanes][2 x u16]   tile A: sc | m << 8 of (row gr, block c), (row gr+8, block c)
//   bytes 2176 .. 2303   [32 lanes][2 x u16]   tile B: the same for rows 16+gr, 24+gr
//   bytes 2304 .. 2367   [16 rows][fp16 d, fp16 dmin]   tile A rows 0..15
//   bytes 2368 .. 2431   [16 rows][fp16 d, fp16 dmin]   tile B rows 16..31
// (d, dmin repeat in both units of a super-block). Q4_K columns are whole super-blocks.
//
// Q6_K matrices (reference include/jinf/quant.h:59-69: 256-element super-blocks, fp16 d, an
// int8 scale per 16-element sub-block, w = d sc (q - 32) with q = low4 | high2 << 4, low4 the
// low nibble of ql[e / 2] for even e, high2 bits 2 (e % 4) of qh[e / 4]) use 3392-byte units
// (Q4M_UNIT_6) of the same geometry (group G = elements 128 (G % 2) .. +127 of super-block
// G / 2, block j = 32 of them, k the element in the block):
//   bytes    0 .. 2047   the low nibbles of q, laid out exactly as the Q4_0 nibbles above
//   bytes 2048 .. 3071   [2 block pairs jj][32 lanes][4 words]: word 2 (j % 2) + h of lane L
//                         holds the high two bits of q for the words i = 2h, 2h + 1 of block
//                         j = 2 jj + (j % 2): byte b has, from bit 0, the crumbs of tile A
//                         word 2h, tile B word 2h, tile A word 2h + 1, tile B word 2h + 1,
//                         each with its top bit flipped (crumb ^ 2)
//   bytes 3072 .. 3327   [32 lanes][2 words]: tile A, tile B int8 sub-block scales of lane
//                         (gr, c): sc(row gr, block c, half 0), (gr, c, 1), (gr + 8, c, 0),
//                         (gr + 8, c, 1) (half = elements 0..15 / 16..31 of the block)
//   bytes 3328 .. 3391   [8 gr][4 x fp16]: d of rows gr, gr + 8, 16 + gr, 24 + gr
// With the flipped crumb, (low4 << 2) | (crumb ^ 2) << 6 is the byte of the int8 value
// 4 (q - 32), the s8 tensor-core operand (q4m_device.cuh).
//
// Q8_0 matrices (reference include/jinf/quant.h:50-56: 32-element blocks, fp16 d, int8 q,
// w = d q) use 4352-byte units (Q4M_UNIT_8):
//   bytes    0 .. 4095   [4 blocks j][2 tiles t][32 lanes][4 words i]: byte b of word i is q
//                         of row 16 t + gr + 8 (i & 1), element k = 16 (i >> 1) + 4 c + b
//   bytes 4096 .. 4351   [32 lanes][4 x fp16]: d of (row gr, block c), (gr + 8, c),
//                         (16 + gr, c), (24 + gr, c)
// Q6_K columns are whole super-blocks, Q8_0 columns whole blocks.
#pragma once

#include <stdint.h>

namespace jinf {

constexpr int Q4M_ROWS = 16;             // rows per MMA tile
constexpr int Q4M_KG = 128;              // columns per group
constexpr int Q4M_UNIT = 2304;           // bytes per (tile pair, group)
constexpr int Q4M_SCALES = 2048;         // byte offset of the scales in a unit
constexpr int Q4M_PAIR_ROWS = 2 * Q4M_ROWS;
constexpr int Q4M_UNIT_K = 2432;         // bytes per (tile pair, group) of a Q4_K matrix
constexpr int Q4M_DMIN_K = 2304;         // byte offset of the per-row d, dmin in a Q4_K unit
constexpr int Q4M_UNIT_6 = 3392;         // bytes per (tile pair, group) of a Q6_K matrix
constexpr int Q4M_CRUMB_6 = 2048;        // byte offsets in a Q6_K unit: high-bit crumbs,
constexpr int Q4M_SC_6 = 3072;           //   sub-block scales,
constexpr int Q4M_D_6 = 3328;            //   per-row d
constexpr int Q4M_UNIT_8 = 4352;         // bytes per (tile pair, group) of a Q8_0 matrix
constexpr int Q4M_D_8 = 4096;            // byte offset of the scales in a Q8_0 unit

// Weight formats of a Q4M matrix
enum Q4MFormat { Q4M_Q4_0 = 0, Q4M_Q4_K = 1, Q4M_Q6_K = 2, Q4M_Q8_0 = 3 };
constexpr int Q4M_NFMT = 4;
// Not a matrix format: the persistent step's instance for models whose matrices mix Q4_0,
// Q4_K and Q6_K, each phase with its own formats (its ring slots fit the largest unit).
constexpr int Q4M_MIX = 4;
__host__ __device__ constexpr inline int q4m_unit_bytes(int fmt) {
    return fmt == Q4M_Q4_K ? Q4M_UNIT_K
         : fmt == Q4M_Q6_K || fmt == Q4M_MIX ? Q4M_UNIT_6
         : fmt == Q4M_Q8_0 ? Q4M_UNIT_8
                           : Q4M_UNIT;
}
// Columns of a matrix of format fmt come in whole blocks (32) or super-blocks (256).
__host__ __device__ constexpr inline int q4m_col_align(int fmt) {
    return fmt == Q4M_Q4_K || fmt == Q4M_Q6_K ? 256 : 32;
}

// Bytes of one row of `cols` weights in the reference's AoS blocks of format fmt (Q4_0: 18
// per 32, Q4_K: 144 per 256, Q6_K: 210 per 256, Q8_0: 34 per 32).
__host__ __device__ inline uint64_t aos_row_bytes(int fmt, int64_t cols) {
    return fmt == Q4M_Q4_K ? (uint64_t)cols / 256 * 144
         : fmt == Q4M_Q6_K ? (uint64_t)cols / 256 * 210
         : fmt == Q4M_Q8_0 ? (uint64_t)cols / 32 * 34
                           : (uint64_t)cols / 32 * 18;
}

struct Q4MShape {
    int rows, cols;
    int pairs;   // ceil(rows / 32)
    int groups;  // ceil(cols / 128)
    int fmt;     // Q4MFormat
    uint64_t bytes;
};

// Input records of one GEMV (the x operand, q4m_device.cuh): digits [G][32 lanes][2 words]
// (256 bytes per group: lane 4 gr + c holds digit gr & 1 of block gr >> 1, word r = elements
// 16 r + 4c .. +3), then params [G][4 blocks] {-8 sum(hi), -8 sum(lo) (int bits), 1/alpha,
// 1/(16 alpha)}.
__host__ __device__ inline size_t xrec_bytes(int groups) { return (size_t)groups * 320; }

// Byte offset of the unit of pair p, group g.
__host__ __device__ inline uint64_t q4m_unit_offset(int p, int g, int groups, int fmt = Q4M_Q4_0) {
    return ((uint64_t)p * groups + g) * q4m_unit_bytes(fmt);
}

// cols must be whole Q4_0 blocks (a multiple of 32); the last group is padded with zero
// blocks (scale 0) when cols is not a multiple of 128, and the GEMV stages zero digits for
// x there.
inline bool q4m_shape(int rows, int cols, Q4MShape* s, int fmt = Q4M_Q4_0) {
    if (rows <= 0 || cols <= 0 || fmt < 0 || fmt >= Q4M_NFMT || cols % q4m_col_align(fmt)) return false;
    s->rows = rows;
    s->cols = cols;
    s->pairs = (rows + Q4M_PAIR_ROWS - 1) / Q4M_PAIR_ROWS;
    s->groups = (cols + Q4M_KG - 1) / Q4M_KG;
    s->fmt = fmt;
    s->bytes = (uint64_t)s->pairs * s->groups * q4m_unit_bytes(fmt);
    return true;
}

// Where element k (0..31) of block j of pair row r (0..31) lives inside a unit: the byte
// offset of its nibble and whether it is the high nibble.
__host__ __device__ inline int q4m_nibble_byte(int r, int j, int k) {
    const int rt = r & 15, gr = rt & 7, i = ((k >> 4) << 1) | (rt >> 3), c = (k >> 2) & 3;
    return 512 * j + 16 * (4 * gr + c) + 4 * i + (k & 3);
}
__host__ __device__ inline bool q4m_nibble_high(int r) { return r >= 16; }

}  // namespace jinf
