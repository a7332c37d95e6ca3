// Host-side quantization helpers: fp16 conversion, dequantizers with the reference's
// nibble/scale conventions (reference src/quant.cpp:49-136) and the quantizers the
// synthetic-model generator uses to produce blocks in those conventions.
#include "jinf/quant.h"
#include "synth_math.h"

#include <math.h>
#include <string.h>

extern "C" float jinf_fp16_to_fp32(uint16_t h) {
    // Exact for every fp16 value: normal, subnormal, zero, inf and NaN.
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t exp = (h >> 10) & 0x1f;
    uint32_t man = h & 0x3ff;
    uint32_t bits;
    if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (man << 13);
    } else if (exp != 0) {
        bits = sign | ((exp + 112) << 23) | (man << 13);
    } else if (man == 0) {
        bits = sign;
    } else {
        // subnormal: value = man * 2^-24; renormalise
        int e = -1;
        do { man <<= 1; ++e; } while ((man & 0x400) == 0);
        bits = sign | ((uint32_t)(112 - e) << 23) | ((man & 0x3ff) << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

extern "C" uint16_t jinf_fp32_to_fp16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) {  // inf / nan
        return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    }
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);  // rounds to inf
    if (ax < 0x38800000u) {
        // result is fp16 subnormal or zero: value / 2^-24, round to nearest even
        if (ax < 0x33000000u) return (uint16_t)sign;  // below half of the smallest subnormal
        uint32_t e = ax >> 23;
        uint32_t m = (ax & 0x7fffffu) | 0x800000u;
        uint32_t shift = 126 - e;  // e in [102, 112]: value = m * 2^(e-150); q = value/2^-24
        uint32_t q = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1))) ++q;
        return (uint16_t)(sign | q);
    }
    uint32_t e = (ax >> 23) - 112;
    uint32_t m = ax & 0x7fffffu;
    uint32_t h = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1))) ++h;  // may carry into the exponent: correct
    return (uint16_t)(sign | h);
}

// ---- dequantization ----

extern "C" void jinf_dequantize_q4_0(const jinf_block_q4_0* blocks, float* out, int n_blocks) {
    for (int b = 0; b < n_blocks; ++b) {
        const float d = jinf_fp16_to_fp32(blocks[b].d);
        float* o = out + (size_t)b * 32;
        for (int i = 0; i < 16; ++i) {
            const uint8_t v = blocks[b].qs[i];
            o[2 * i]     = (float)((int)(v & 15) - 8) * d;
            o[2 * i + 1] = (float)((int)(v >> 4) - 8) * d;
        }
    }
}

// Sub-block j (0..7) scale and min of a Q4_K block, reference packing
// (reference src/quant.cpp:72-78): j < 4 uses the low 6 bits of s[j] / s[j+4];
// j >= 4 puts the 4 bits of s[j+4] above the top 2 bits of s[j-4] / s[j].
static inline void q4k_scale_min(const uint8_t* s, int j, int* sc, int* mn) {
    if (j < 4) {
        *sc = s[j] & 63;
        *mn = s[j + 4] & 63;
    } else {
        *sc = ((s[j + 4] & 15) << 2) | (s[j - 4] >> 6);
        *mn = ((s[j + 4] >> 4) << 2) | (s[j] >> 6);
    }
}

extern "C" void jinf_dequantize_q4_K(const jinf_block_q4_K* blocks, float* out, int n_blocks) {
    for (int b = 0; b < n_blocks; ++b) {
        const float d = jinf_fp16_to_fp32(blocks[b].d);
        const float dmin = jinf_fp16_to_fp32(blocks[b].dmin);
        for (int j = 0; j < 8; ++j) {
            int sc, mn;
            q4k_scale_min(blocks[b].scales, j, &sc, &mn);
            // This file is built with -ffp-contract=off: the product and the difference
            // below round separately, like the reference's host build.
            const float sd = d * (float)sc;
            const float sm = dmin * (float)mn;
            float* o = out + (size_t)b * 256 + 32 * j;
            const uint8_t* q = blocks[b].qs + 16 * j;
            for (int i = 0; i < 16; ++i) {
                o[2 * i]     = sd * (float)(q[i] & 15) - sm;
                o[2 * i + 1] = sd * (float)(q[i] >> 4) - sm;
            }
        }
    }
}

extern "C" void jinf_dequantize_q8_0(const jinf_block_q8_0* blocks, float* out, int n_blocks) {
    for (int b = 0; b < n_blocks; ++b) {
        const float d = jinf_fp16_to_fp32(blocks[b].d);
        for (int i = 0; i < 32; ++i) out[(size_t)b * 32 + i] = (float)blocks[b].qs[i] * d;
    }
}

extern "C" void jinf_dequantize_q6_K(const jinf_block_q6_K* blocks, float* out, int n_blocks) {
    for (int b = 0; b < n_blocks; ++b) {
        const float d = jinf_fp16_to_fp32(blocks[b].d);
        for (int i = 0; i < 256; ++i) {
            const int lo = (blocks[b].ql[i >> 1] >> ((i & 1) * 4)) & 15;
            const int hi = (blocks[b].qh[i >> 2] >> (2 * (i & 3))) & 3;
            out[(size_t)b * 256 + i] = d * (float)blocks[b].scales[i >> 4] * (float)((lo | (hi << 4)) - 32);
        }
    }
}

extern "C" void jinf_dequantize(const void* data, jinf_qtype type, float* out, int64_t n_elements) {
    const int bs = jinf_qtype_block_size(type);
    if (bs == 0) return;
    const int nb = (int)((n_elements + bs - 1) / bs);
    switch (type) {
        case JINF_TYPE_Q4_0: jinf_dequantize_q4_0((const jinf_block_q4_0*)data, out, nb); break;
        case JINF_TYPE_Q4_K: jinf_dequantize_q4_K((const jinf_block_q4_K*)data, out, nb); break;
        case JINF_TYPE_Q8_0: jinf_dequantize_q8_0((const jinf_block_q8_0*)data, out, nb); break;
        case JINF_TYPE_Q6_K: jinf_dequantize_q6_K((const jinf_block_q6_K*)data, out, nb); break;
        case JINF_TYPE_F32: memcpy(out, data, (size_t)n_elements * sizeof(float)); break;
        case JINF_TYPE_F16: {
            const uint16_t* h = (const uint16_t*)data;
            for (int64_t i = 0; i < n_elements; ++i) out[i] = jinf_fp16_to_fp32(h[i]);
            break;
        }
        default: break;  // unknown types leave `out` untouched, as the reference does
    }
}

// ---- quantization ----

// Q4_0: d = (value of largest magnitude) / -8, q = clamp(trunc(x/d + 8.5), 0, 15).
// This is the common published Q4_0 rounding rule; nibbles are stored in the
// reference's pairing (byte i = elements 2i | 2i+1 << 4).
extern "C" void jinf_quantize_q4_0(const float* x, jinf_block_q4_0* out, int64_t n) {
    for (int64_t b = 0; b < n / 32; ++b) jinf_synth::quantize_q4_0_block(x + 32 * b, (uint8_t*)(out + b));
}

// Q8_0: d = max|x| / 127 (stored fp16), q = round-half-away(x / d) clamped to [-127, 127]
// against the stored d.
extern "C" void jinf_quantize_q8_0(const float* x, jinf_block_q8_0* out, int64_t n) {
    for (int64_t b = 0; b < n / 32; ++b) {
        const float* v = x + 32 * b;
        float amax = 0.f;
        for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
        const uint16_t dh = jinf_fp32_to_fp16(amax / 127.f);
        const float d = jinf_fp16_to_fp32(dh);
        out[b].d = dh;
        for (int i = 0; i < 32; ++i) {
            int q = d > 0.f ? (int)lroundf(v[i] / d) : 0;
            out[b].qs[i] = (int8_t)(q < -127 ? -127 : (q > 127 ? 127 : q));
        }
    }
}

// Q6_K: per 16-element sub-block a symmetric step s = max|x| / 31, the 16 steps quantised
// to int8 scales against the fp16 super-scale d = max(s) / 127, then q = round(x / (d sc)) + 32
// clamped to 0..63 against the stored parameters, packed in the reference GPU layout.
extern "C" void jinf_quantize_q6_K(const float* x, jinf_block_q6_K* out, int64_t n) {
    for (int64_t b = 0; b < n / 256; ++b) {
        const float* v = x + 256 * b;
        float st[16], smax = 0.f;
        for (int j = 0; j < 16; ++j) {
            float amax = 0.f;
            for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[16 * j + i]));
            st[j] = amax / 31.f;
            smax = fmaxf(smax, st[j]);
        }
        const uint16_t dh = jinf_fp32_to_fp16(smax / 127.f);
        const float d = jinf_fp16_to_fp32(dh);
        jinf_block_q6_K& o = out[b];
        memset(&o, 0, sizeof o);
        o.d = dh;
        for (int j = 0; j < 16; ++j) {
            int sc = d > 0.f ? (int)lrintf(st[j] / d) : 0;
            sc = sc > 127 ? 127 : sc;
            o.scales[j] = (int8_t)sc;
            const float step = d * (float)sc;
            for (int i = 0; i < 16; ++i) {
                const int e = 16 * j + i;
                int q = step > 0.f ? (int)lrintf(v[e] / step) + 32 : 32;
                q = q < 0 ? 0 : (q > 63 ? 63 : q);
                o.ql[e >> 1] |= (uint8_t)((q & 15) << (4 * (e & 1)));
                o.qh[e >> 2] |= (uint8_t)((q >> 4) << (2 * (e & 3)));
            }
        }
    }
}

// Q4_K: per 32-element sub-block an affine fit x ~ s*q - m (q in 0..15, m >= 0), the
// 8 scales and mins quantised to 6 bits against fp16 super-scales d = max(s)/63 and
// dmin = max(m)/63, then q re-derived from the stored (rounded) parameters. Packed in
// the reference's scale layout.
extern "C" void jinf_quantize_q4_K(const float* x, jinf_block_q4_K* out, int64_t n) {
    const int64_t nb = n / 256;
    for (int64_t b = 0; b < nb; ++b) {
        const float* v = x + b * 256;
        float s[8], m[8], smax = 0.f, mmax = 0.f;
        for (int j = 0; j < 8; ++j) {
            float lo = v[32 * j], hi = v[32 * j];
            for (int i = 1; i < 32; ++i) {
                lo = fminf(lo, v[32 * j + i]);
                hi = fmaxf(hi, v[32 * j + i]);
            }
            m[j] = lo < 0.f ? -lo : 0.f;
            s[j] = (hi + m[j]) / 15.f;
            smax = fmaxf(smax, s[j]);
            mmax = fmaxf(mmax, m[j]);
        }
        const uint16_t dh = jinf_fp32_to_fp16(smax / 63.f);
        const uint16_t mh = jinf_fp32_to_fp16(mmax / 63.f);
        const float d = jinf_fp16_to_fp32(dh), dmin = jinf_fp16_to_fp32(mh);
        int ls[8], lm[8];
        for (int j = 0; j < 8; ++j) {
            int a = d > 0.f ? (int)lrintf(s[j] / d) : 0;
            int c = dmin > 0.f ? (int)lrintf(m[j] / dmin) : 0;
            ls[j] = a < 0 ? 0 : (a > 63 ? 63 : a);
            lm[j] = c < 0 ? 0 : (c > 63 ? 63 : c);
        }
        out[b].d = dh;
        out[b].dmin = mh;
        uint8_t* sc = out[b].scales;
        for (int i = 0; i < 4; ++i) {
            sc[i]     = (uint8_t)((ls[i] & 63) | ((ls[i + 4] & 3) << 6));
            sc[i + 4] = (uint8_t)((lm[i] & 63) | ((lm[i + 4] & 3) << 6));
            sc[i + 8] = (uint8_t)(((ls[i + 4] >> 2) & 15) | (((lm[i + 4] >> 2) & 15) << 4));
        }
        for (int j = 0; j < 8; ++j) {
            const float step = d * (float)ls[j];
            const float off = dmin * (float)lm[j];
            for (int i = 0; i < 16; ++i) {
                int q[2];
                for (int t = 0; t < 2; ++t) {
                    const float val = v[32 * j + 2 * i + t];
                    int qq = step > 0.f ? (int)lrintf((val + off) / step) : 0;
                    q[t] = qq < 0 ? 0 : (qq > 15 ? 15 : qq);
                }
                out[b].qs[16 * j + i] = (uint8_t)(q[0] | (q[1] << 4));
            }
        }
    }
}
