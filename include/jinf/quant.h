// jinf-b200: quantization types, on-disk block layouts, host dequantization.
//
// Drop-in for the reference's include/jinf/quant.h. The enum values are the
// GGUF/ggml type ids (reference include/jinf/quant.h:8-24) and the packed block
// structs keep the reference's byte layouts (reference include/jinf/quant.h:31-69),
// because every file, bundle and kernel argument on the decode path is made of them.
//
// Nibble convention (the reference's own, reference src/quant.cpp:49-93): inside a
// 16-byte group, byte i carries element 2i in its low nibble and element 2i+1 in its
// high nibble. This is NOT upstream ggml's "j / j+16" split; parity follows the
// reference.
#pragma once

#include <stddef.h>
#include <stdint.h>

enum jinf_qtype
#ifdef __cplusplus
    : int
#endif
{
    JINF_TYPE_F32  = 0,
    JINF_TYPE_F16  = 1,
    JINF_TYPE_Q4_0 = 2,
    JINF_TYPE_Q4_1 = 3,
    JINF_TYPE_Q5_0 = 6,
    JINF_TYPE_Q5_1 = 7,
    JINF_TYPE_Q8_0 = 8,
    JINF_TYPE_Q8_1 = 9,
    JINF_TYPE_Q2_K = 10,
    JINF_TYPE_Q3_K = 11,
    JINF_TYPE_Q4_K = 12,
    JINF_TYPE_Q5_K = 13,
    JINF_TYPE_Q6_K = 14,
    JINF_TYPE_Q8_K = 15,
    JINF_TYPE_COUNT,
};
#ifndef __cplusplus
typedef enum jinf_qtype jinf_qtype;
#endif

#pragma pack(push, 1)
// 32 weights: w = (q - 8) * d, q = 4-bit unsigned.
typedef struct jinf_block_q4_0 {
    uint16_t d;       // fp16 scale
    uint8_t  qs[16];  // 32 nibbles, byte i = elements (2i, 2i+1)
} jinf_block_q4_0;

// 256 weights in 8 sub-blocks of 32: w = d*sc[j]*q - dmin*mn[j].
typedef struct jinf_block_q4_K {
    uint16_t d;           // fp16 super-block scale
    uint16_t dmin;        // fp16 super-block min scale
    uint8_t  scales[12];  // 8 x 6-bit scales + 8 x 6-bit mins (packing: see jinf_q4k_scale_min)
    uint8_t  qs[128];     // sub-block j uses qs[16j .. 16j+15]
} jinf_block_q4_K;

// 32 weights: w = q * d, q = int8.
typedef struct jinf_block_q8_0 {
    uint16_t d;
    int8_t   qs[32];
} jinf_block_q8_0;

// 256 weights: w = d * scales[i/16] * (q6 - 32), q6 = ql nibble | (qh 2 bits << 4).
typedef struct jinf_block_q6_K {
    uint8_t  ql[128];     // element i: ql[i/2], low nibble for even i
    uint8_t  qh[64];      // element i: (qh[i/4] >> 2*(i%4)) & 3
    int8_t   scales[16];  // one per 16 elements
    uint16_t d;
} jinf_block_q6_K;
#pragma pack(pop)

#ifdef __cplusplus
static_assert(sizeof(jinf_block_q4_0) == 18, "Q4_0 block must be 18 bytes");
static_assert(sizeof(jinf_block_q4_K) == 144, "Q4_K block must be 144 bytes");
static_assert(sizeof(jinf_block_q8_0) == 34, "Q8_0 block must be 34 bytes");
static_assert(sizeof(jinf_block_q6_K) == 210, "Q6_K block must be 210 bytes");
#endif

// Weights per block (1 for plain float types, 0 for an unknown type).
static inline int jinf_qtype_block_size(jinf_qtype t) {
    switch (t) {
        case JINF_TYPE_F32: case JINF_TYPE_F16: return 1;
        case JINF_TYPE_Q4_0: case JINF_TYPE_Q4_1: case JINF_TYPE_Q5_0:
        case JINF_TYPE_Q5_1: case JINF_TYPE_Q8_0: case JINF_TYPE_Q8_1: return 32;
        case JINF_TYPE_Q2_K: case JINF_TYPE_Q3_K: case JINF_TYPE_Q4_K:
        case JINF_TYPE_Q5_K: case JINF_TYPE_Q6_K: case JINF_TYPE_Q8_K: return 256;
        default: return 0;
    }
}

// Bytes per block (ggml type sizes).
static inline size_t jinf_qtype_type_size(jinf_qtype t) {
    switch (t) {
        case JINF_TYPE_F32:  return 4;
        case JINF_TYPE_F16:  return 2;
        case JINF_TYPE_Q4_0: return 18;
        case JINF_TYPE_Q4_1: return 20;
        case JINF_TYPE_Q5_0: return 22;
        case JINF_TYPE_Q5_1: return 24;
        case JINF_TYPE_Q8_0: return 34;
        case JINF_TYPE_Q8_1: return 36;
        case JINF_TYPE_Q2_K: return 84;
        case JINF_TYPE_Q3_K: return 110;
        case JINF_TYPE_Q4_K: return 144;
        case JINF_TYPE_Q5_K: return 176;
        case JINF_TYPE_Q6_K: return 210;
        case JINF_TYPE_Q8_K: return 292;
        default: return 0;
    }
}

static inline const char* jinf_qtype_name(jinf_qtype t) {
    switch (t) {
        case JINF_TYPE_F32:  return "F32";
        case JINF_TYPE_F16:  return "F16";
        case JINF_TYPE_Q4_0: return "Q4_0";
        case JINF_TYPE_Q4_1: return "Q4_1";
        case JINF_TYPE_Q5_0: return "Q5_0";
        case JINF_TYPE_Q5_1: return "Q5_1";
        case JINF_TYPE_Q8_0: return "Q8_0";
        case JINF_TYPE_Q8_1: return "Q8_1";
        case JINF_TYPE_Q2_K: return "Q2_K";
        case JINF_TYPE_Q3_K: return "Q3_K";
        case JINF_TYPE_Q4_K: return "Q4_K";
        case JINF_TYPE_Q5_K: return "Q5_K";
        case JINF_TYPE_Q6_K: return "Q6_K";
        case JINF_TYPE_Q8_K: return "Q8_K";
        default: return "UNKNOWN";
    }
}

// Bytes of a tensor of n_elements values (whole blocks).
static inline size_t jinf_tensor_nbytes(jinf_qtype t, int64_t n_elements) {
    int bs = jinf_qtype_block_size(t);
    if (bs == 0) return 0;
    return (size_t)((n_elements + bs - 1) / bs) * jinf_qtype_type_size(t);
}

#ifdef __cplusplus
extern "C" {
#endif

// ---- Host dequantization (replaces reference src/quant.cpp:49-136) ----
// Outputs are fp32 with the reference's nibble order; Q4_K products and
// differences are computed without fused multiply-add, as the reference's host build does.
void jinf_dequantize_q4_0(const jinf_block_q4_0* blocks, float* out, int n_blocks);
void jinf_dequantize_q4_K(const jinf_block_q4_K* blocks, float* out, int n_blocks);
void jinf_dequantize_q8_0(const jinf_block_q8_0* blocks, float* out, int n_blocks);
// Declared but never defined by the reference (reference include/jinf/quant.h:149);
// defined here with the reference GPU kernel's layout (reference cuda/dequant_kernels.cu:82-112).
void jinf_dequantize_q6_K(const jinf_block_q6_K* blocks, float* out, int n_blocks);
// Type dispatcher (reference src/quant.cpp:108-136); unknown types leave `out` untouched.
void jinf_dequantize(const void* data, jinf_qtype type, float* out, int64_t n_elements);

// ---- New: host helpers used by the synthetic-model generator and tests ----
float    jinf_fp16_to_fp32(uint16_t h);
uint16_t jinf_fp32_to_fp16(float f);  // round-to-nearest-even
// Quantize n (multiple of 32) floats to Q4_0 blocks in the reference nibble order.
void jinf_quantize_q4_0(const float* x, jinf_block_q4_0* out, int64_t n);
// Quantize n (multiple of 256) floats to Q4_K blocks in the reference scale packing.
void jinf_quantize_q4_K(const float* x, jinf_block_q4_K* out, int64_t n);
// Quantize n (multiple of 32) floats to Q8_0 blocks: d = max|x| / 127, q = round(x / d).
void jinf_quantize_q8_0(const float* x, jinf_block_q8_0* out, int64_t n);
// Quantize n (multiple of 256) floats to Q6_K blocks in the reference GPU kernel's bit layout
// (ql[e/2] nibble, qh[e/4] bits 2 (e%4), int8 scale per 16, fp16 d last).
void jinf_quantize_q6_K(const float* x, jinf_block_q6_K* out, int64_t n);

#ifdef __cplusplus
}
#endif
