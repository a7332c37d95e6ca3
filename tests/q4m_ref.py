"""numpy statement of the Q4M layout and of the tensor-core GEMV arithmetic (test helper).

`pack` builds the Q4M image of AoS Q4_0 blocks exactly as the layout is documented in
jetson-inference_b200/csrc/q4m.cuh; `emulate_gemv` follows the kernel's arithmetic at matrix
level (nibbles decoded through the same bit patterns, x split into fp16 hi + lo with the
power-of-two pre-scale, block-diagonal B, accumulator offset) in fp32, so the derivation can
be checked against the oracle without a GPU.
"""
import numpy as np

ROWS, KG, CHUNK = 16, 128, 1152   # chunks of tiles 2P and 2P+1 (one group) are adjacent


def nibble_bit(r, j):
    return ((j & 1) << 4) | ((r >> 3) << 3) | ((j >> 1) << 2)


def pack(aos: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """AoS Q4_0 [rows][cols/32*18] uint8 -> Q4M bytes."""
    nb = cols // 32
    groups = (cols + KG - 1) // KG
    tiles = 2 * ((rows + 2 * ROWS - 1) // (2 * ROWS))
    blk = np.zeros((tiles * ROWS, groups * 4, 18), dtype=np.uint8)   # padded blocks: scale 0, nibbles 0
    blk[:rows, :nb] = aos.reshape(rows, nb, 18)
    qs = blk[:, :, 2:]
    # q[row, block, e]: element 2i = low nibble of byte i, 2i+1 = high nibble
    q = np.empty((tiles * ROWS, groups * 4, 32), dtype=np.uint32)
    q[:, :, 0::2] = qs & 15
    q[:, :, 1::2] = qs >> 4
    d = blk[:, :, 0].astype(np.uint32) | (blk[:, :, 1].astype(np.uint32) << 8)
    q = q.reshape(tiles, ROWS, groups, 4, 32)          # t, r, G, j, e
    d = d.reshape(tiles, ROWS, groups, 4)               # t, r, G, j
    out = np.zeros((tiles, groups, CHUNK), dtype=np.uint8)
    words = np.zeros((tiles, groups, 32, 8), dtype=np.uint32)  # lane, word i
    for lane in range(32):
        gr, c = lane >> 2, lane & 3
        for i in range(8):
            e = 4 * i + c
            w = np.zeros((tiles, groups), dtype=np.uint32)
            for half in range(2):
                r = gr + 8 * half
                for j in range(4):
                    w |= q[:, r, :, j, e] << nibble_bit(r, j)
            words[:, :, lane, i] = w
    wb = words.astype('<u4').view(np.uint8).reshape(tiles, groups, 32, 2, 16)  # lane, piece, 16 B
    out[:, :, 0:512] = wb[:, :, :, 0, :].reshape(tiles, groups, 512)
    out[:, :, 512:1024] = wb[:, :, :, 1, :].reshape(tiles, groups, 512)
    sc = np.zeros((tiles, groups, 32), dtype=np.uint32)
    for lane in range(32):
        gr, c = lane >> 2, lane & 3
        sc[:, :, lane] = d[:, gr, :, c] | (d[:, gr + 8, :, c] << 16)
    out[:, :, 1024:] = sc.astype('<u4').view(np.uint8).reshape(tiles, groups, 128)
    # memory order: (tile pair, group, tile in pair)
    return out.reshape(tiles // 2, 2, groups, CHUNK).transpose(0, 2, 1, 3).reshape(-1)


def unpack_words(img: np.ndarray, tiles: int, groups: int):
    ch = img.reshape(tiles // 2, groups, 2, CHUNK).transpose(0, 2, 1, 3).reshape(tiles, groups, CHUNK)
    w = np.concatenate([ch[:, :, 0:512].reshape(tiles, groups, 32, 16),
                        ch[:, :, 512:1024].reshape(tiles, groups, 32, 16)], axis=3)
    words = w.copy().view('<u4').reshape(tiles, groups, 32, 8)
    sc = ch[:, :, 1024:].copy().view('<u4').reshape(tiles, groups, 32)
    return words, sc


def _f16(bits):
    return np.asarray(bits, dtype=np.uint16).view(np.float16).astype(np.float32)


def emulate_gemv(img: np.ndarray, x: np.ndarray, rows: int, cols: int) -> np.ndarray:
    groups = (cols + KG - 1) // KG
    tiles = 2 * ((rows + 2 * ROWS - 1) // (2 * ROWS))
    words, sc = unpack_words(img, tiles, groups)
    # decode: a0 = (w & 0x000F000F) | 0x64006400, a2 = (w & 0x00F000F0) | ..., a1/a3 from w >> 8
    val = np.zeros((tiles, groups, ROWS, 4, 32), dtype=np.float32)  # decoded A value (1024 + s q)
    for lane in range(32):
        gr, c = lane >> 2, lane & 3
        for i in range(8):
            w = words[:, :, lane, i]
            u = w >> 8
            regs = {0: (w & 0x000F000F) | 0x64006400, 2: (w & 0x00F000F0) | 0x64006400,
                    1: (u & 0x000F000F) | 0x64006400, 3: (u & 0x00F000F0) | 0x64006400}
            e = 4 * i + c
            for reg, bits in regs.items():
                r = gr + 8 * (reg & 1)
                jlo = 0 if reg < 2 else 2
                val[:, :, r, jlo, e] = _f16(bits & 0xFFFF)
                val[:, :, r, jlo + 1, e] = _f16(bits >> 16)
    # B: power-of-two pre-scale, fp16 hi + lo, blocks 2,3 divided by 16
    amax = float(np.max(np.abs(x))) * 1.0001
    ex = int((np.float32(amax).view(np.uint32) >> 23) & 0xFF)
    k = min(max(268 - ex, 1), 254)
    alpha = np.uint32(k << 23).view(np.float32)
    xp = np.zeros(groups * KG, dtype=np.float32)
    xp[:cols] = x
    xs = xp.reshape(groups, 4, 32).astype(np.float32) * alpha
    xs[:, 2:, :] *= np.float32(0.0625)
    hi = xs.astype(np.float16).astype(np.float32)
    lo = (xs - hi).astype(np.float16).astype(np.float32)
    bsum = (hi + lo).sum(axis=2, dtype=np.float32)                     # [G][j]
    koff = -np.where(np.arange(4) < 2, 1032.0, 1152.0).astype(np.float32) * bsum
    # D[r, j] = sum_e val * (hi + lo) + koff   (the MMA's exact products, fp32 sums)
    dsum = (np.einsum('tgrje,gje->tgrj', val.astype(np.float64), (hi + lo).astype(np.float64))
            .astype(np.float32) + koff[None, :, None, :])
    dsc = np.zeros((tiles, groups, ROWS, 4), dtype=np.float32)
    for lane in range(32):
        gr, c = lane >> 2, lane & 3
        dsc[:, :, gr, c] = _f16(sc[:, :, lane] & 0xFFFF)
        dsc[:, :, gr + 8, c] = _f16(sc[:, :, lane] >> 16)
    y = (dsc * dsum).sum(axis=(1, 3)).reshape(-1)[:rows] / alpha
    return y.astype(np.float32)
