// Q4T: the engine's HBM layout for Q4_0 weight matrices (lossless repack of the
// reference's 18-byte AoS blocks), and the shared definitions of the GEMV kernels
// that stream it.
//
// Layout. A matrix [rows][cols] (nb = cols/32 blocks per row) is cut into warp tiles
// of RW = R * (32/LK) rows. A warp walks its tile in S = nb/LK steps; at each step
// lane `lam` = g*LK + l reads block (s*LK + l) of the R rows g*R .. g*R+R-1 of the tile.
// The bytes of one (tile, step) pair form a contiguous 'chunk' of R*576 bytes:
//   [R][32 lanes][16 B nibble words]   nibbles of block (row, blk) = the 16 AoS qs bytes
//   [32 lanes][R][fp16 scale]          d of the same blocks
// and chunk (t, s) sits at byte (t*S + s) * R*576. Every warp load is therefore one
// contiguous 512-byte (or 256-byte for the scales) segment, the stream of a whole
// matrix is contiguous, and rows past `rows` are zero padding (d = 0).
//
// Inside a 16-byte nibble group word w (little-endian qs bytes 4w..4w+3) holds block
// elements 8w..8w+7 at bit 4*(e%8), exactly the reference's pairing (byte i = elements
// 2i | 2i+1 << 4), so the repack moves bytes and never touches a nibble.
#pragma once

#include <stdint.h>

namespace jinf {

constexpr int Q4T_R = 4;                       // rows per thread
constexpr int Q4T_CHUNK = Q4T_R * 576;         // bytes per (tile, step)

struct Q4TShape {
    int rows, cols;   // logical
    int nb;           // cols / 32
    int lk;           // lanes along K (32, 16, 8 or 4)
    int rw;           // rows per tile
    int steps;        // nb / lk
    int tiles;        // ceil(rows / rw)
    uint64_t bytes;   // tiles * steps * Q4T_CHUNK
};

// Largest lane count along K in {32,16,8,4} dividing nb; 0 if nb % 4 != 0.
inline int q4t_pick_lk(int nb) {
    for (int lk = 32; lk >= 4; lk >>= 1)
        if (nb % lk == 0) return lk;
    return 0;
}

inline bool q4t_shape(int rows, int cols, Q4TShape* s) {
    if (rows <= 0 || cols <= 0 || cols % 128) return false;
    s->rows = rows;
    s->cols = cols;
    s->nb = cols / 32;
    s->lk = q4t_pick_lk(s->nb);
    if (!s->lk) return false;
    s->rw = Q4T_R * (32 / s->lk);
    s->steps = s->nb / s->lk;
    s->tiles = (rows + s->rw - 1) / s->rw;
    s->bytes = (uint64_t)s->tiles * s->steps * Q4T_CHUNK;
    return true;
}

// Device-side decode state shared by the engine kernels (one per engine, in HBM).
struct DeviceState {
    int pos;                  // position of the token being decoded (= n_past before the step)
    int token;                // input token id of the current step
    unsigned long long best;  // packed (ordered logit << 32 | ~index) argmax of the last LM head
    int argmax_token;         // decoded argmax of the last step
    int error;                // first device-side error code (0 = none)
    unsigned int attn_count[64];  // split-K arrival counters of the attention kernel (self-resetting)
};

}  // namespace jinf
