// Q4M: the engine's HBM layout for Q4_0 weight matrices, shaped for the tensor-core GEMV
// (gemv_q4m.cu, mma.sync m16n8k16, fp16 operands, fp32 accumulation). It is a lossless
// repack of the reference's 18-byte AoS blocks (reference include/jinf/quant.h:31-35): every
// nibble and every fp16 scale is moved, none is re-quantised.
//
// Geometry. A matrix [rows][cols] is cut into tiles of 16 rows (the MMA's M) and groups
// of 128 columns (4 Q4_0 blocks j = 0..3). The bytes of one (tile t, group G) form one
// contiguous chunk of 1152 bytes; the chunks of the two tiles of a tile pair (t = 2P, 2P+1)
// and one group are adjacent, forming a 2304-byte unit at byte (P * groups + G) * 2304, so
// one copy brings 32 rows x 128 columns and both tiles share the same x fragments. A chunk:
//   bytes    0 ..  511   piece 0: [32 lanes][4 words]   words 0..3 (MMA steps 0..3)
//   bytes  512 .. 1023   piece 1: [32 lanes][4 words]   words 4..7 (MMA steps 4..7)
//   bytes 1024 .. 1151   [32 lanes][2 x fp16]           d(row gr, block c), d(row gr+8, block c)
// for lane = 4*gr + c (gr = 0..7, c = 0..3), so every warp access is one contiguous 512-
// or 128-byte segment and a matrix streams front to back. Rows past `rows` and blocks past
// cols/32 are zero.
//
// MMA mapping. Step i (0..7) of a group multiplies a 16 x 16 A tile whose k index packs
// element e = 4i + c' of all four blocks: k = 2c' + (j & 1) + 8*(j >> 1). The A fragment
// of lane (gr, c) at step i therefore holds element e = 4i + c of
//   a0 = {row gr,   block 0 | block 1}      a2 = {row gr,   block 2 | block 3}
//   a1 = {row gr+8, block 0 | block 1}      a3 = {row gr+8, block 2 | block 3}
// and word i of the lane packs those eight nibbles (w = 4-bit q of row r, block j):
//   bits  0.. 3 q(gr,0)    4.. 7 q(gr,2)    8..11 q(gr+8,0)  12..15 q(gr+8,2)
//   bits 16..19 q(gr,1)   20..23 q(gr,3)   24..27 q(gr+8,1)  28..31 q(gr+8,3)
// One lop3 ((w & mask) | 0x64006400) turns a nibble pair at bits {0,16} into the fp16
// pair 1024 + q, at bits {4,20} into 1024 + 16q; a shift by 8 brings the row gr+8 nibbles
// to the same places. So blocks 0,1 decode with scale s = 1 and blocks 2,3 with s = 16.
//
// Block element e = 2i of the reference block is the low nibble of qs byte i, e = 2i+1
// the high nibble (reference src/quant.cpp:49-60, cuda/matmul_kernels.cu:27-34).
#pragma once

#include <stdint.h>

namespace jinf {

constexpr int Q4M_ROWS = 16;             // rows per tile
constexpr int Q4M_KG = 128;              // columns per group
constexpr int Q4M_CHUNK = 1152;          // bytes per (tile, group)
constexpr int Q4M_UNIT = 2 * Q4M_CHUNK;  // bytes per (tile pair, group)
constexpr int Q4M_PAIR_ROWS = 2 * Q4M_ROWS;

struct Q4MShape {
    int rows, cols;
    int tiles;   // 2 * pairs (rows padded to a multiple of 32)
    int pairs;   // ceil(rows / 32)
    int groups;  // ceil(cols / 128)
    uint64_t bytes;
};

// Byte offset of the chunk of tile t, group g.
__host__ __device__ inline uint64_t q4m_chunk_offset(int t, int g, int groups) {
    return ((uint64_t)(t >> 1) * groups + g) * Q4M_UNIT + (uint64_t)(t & 1) * Q4M_CHUNK;
}

// cols must be whole Q4_0 blocks (a multiple of 32); the last group is padded with zero
// blocks (scale 0) when cols is not a multiple of 128, and the GEMV stages zeros for x there.
inline bool q4m_shape(int rows, int cols, Q4MShape* s) {
    if (rows <= 0 || cols <= 0 || cols % 32) return false;
    s->rows = rows;
    s->cols = cols;
    s->pairs = (rows + Q4M_PAIR_ROWS - 1) / Q4M_PAIR_ROWS;
    s->tiles = 2 * s->pairs;
    s->groups = (cols + Q4M_KG - 1) / Q4M_KG;
    s->bytes = (uint64_t)s->pairs * s->groups * Q4M_UNIT;
    return true;
}

// Bit position, inside word i of lane 4*gr + c, of the nibble of tile row r (0..15) and
// block j (0..3); the word holds element e = 4i + c of the block.
__host__ __device__ inline int q4m_nibble_bit(int r, int j) {
    return ((j & 1) << 4) | ((r >> 3) << 3) | ((j >> 1) << 2);
}

}  // namespace jinf
