// Deterministic synthetic-weight math shared by the host generator (synth.cpp) and the
// device generator (synth_gpu.cu).
//
// Only IEEE-754 basic operations (+ - * / sqrt, conversions) are used, every one written
// in a fixed evaluation order, and both translation units are compiled without
// multiply-add contraction (-ffp-contract=off on the host, -fmad=false on the device), so
// a value comes out bit-identical on the CPU and on the GPU. Box-Muller's log and
// sin/cos are evaluated with short series instead of the math library for that reason.
#pragma once

#include <math.h>
#include <stdint.h>

#ifdef __CUDACC__
#define JINF_HD __host__ __device__ __forceinline__
#else
#define JINF_HD inline
#endif

namespace jinf_synth {

JINF_HD uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// 53-bit uniform in (0, 1]
JINF_HD double to_unit(uint64_t x) {
    return (double)(x >> 11) * (1.0 / 9007199254740992.0) + (1.0 / 18014398509481984.0);
}

JINF_HD double bits_to_double(uint64_t b) {
    union { uint64_t u; double d; } v;
    v.u = b;
    return v.d;
}
JINF_HD uint64_t double_to_bits(double d) {
    union { uint64_t u; double d; } v;
    v.d = d;
    return v.u;
}

// ln(x), x in (0, 1]: x = m * 2^e, m in [sqrt(1/2), sqrt(2)), ln m = 2 atanh((m-1)/(m+1)).
JINF_HD double det_log(double x) {
    uint64_t bits = double_to_bits(x);
    int e = (int)((bits >> 52) & 0x7ff) - 1023;
    double m = bits_to_double((bits & 0x000fffffffffffffull) | 0x3ff0000000000000ull);
    if (m > 1.4142135623730951) {
        m = m * 0.5;
        e += 1;
    }
    const double s = (m - 1.0) / (m + 1.0);
    const double s2 = s * s;
    double t = 1.0 / 25.0;
    t = t * s2 + 1.0 / 23.0;
    t = t * s2 + 1.0 / 21.0;
    t = t * s2 + 1.0 / 19.0;
    t = t * s2 + 1.0 / 17.0;
    t = t * s2 + 1.0 / 15.0;
    t = t * s2 + 1.0 / 13.0;
    t = t * s2 + 1.0 / 11.0;
    t = t * s2 + 1.0 / 9.0;
    t = t * s2 + 1.0 / 7.0;
    t = t * s2 + 1.0 / 5.0;
    t = t * s2 + 1.0 / 3.0;
    t = t * s2 + 1.0;
    const double two_s = 2.0 * s;
    const double lm = two_s * t;
    const double le = (double)e * 0.69314718055994530942;
    return lm + le;
}

// sin / cos of 2*pi*u, u in [0, 1): quadrant reduction, Taylor series on [0, pi/2).
JINF_HD void det_sincos_2pi(double u, double* sn, double* cs) {
    const double f4 = u * 4.0;
    const int q = (int)f4;
    const double a = (f4 - (double)q) * 1.5707963267948966;
    const double a2 = a * a;
    const double cs_[12] = {1.0 / 600.0, 1.0 / 506.0, 1.0 / 420.0, 1.0 / 342.0, 1.0 / 272.0, 1.0 / 210.0,
                            1.0 / 156.0, 1.0 / 110.0, 1.0 / 72.0,  1.0 / 42.0,  1.0 / 20.0,  1.0 / 6.0};
    const double cc_[12] = {1.0 / 552.0, 1.0 / 462.0, 1.0 / 380.0, 1.0 / 306.0, 1.0 / 240.0, 1.0 / 182.0,
                            1.0 / 132.0, 1.0 / 90.0,  1.0 / 56.0,  1.0 / 30.0,  1.0 / 12.0,  1.0 / 2.0};
    double ts = 1.0, tc = 1.0;
#ifdef __CUDACC__
#pragma unroll
#endif
    for (int k = 0; k < 12; ++k) {
        const double ps = ts * a2;
        ts = 1.0 - ps * cs_[k];
        const double pc = tc * a2;
        tc = 1.0 - pc * cc_[k];
    }
    const double s = a * ts, c = tc;
    switch (q & 3) {
        case 0: *sn = s;  *cs = c;  break;
        case 1: *sn = c;  *cs = -s; break;
        case 2: *sn = -s; *cs = -c; break;
        default: *sn = -c; *cs = s; break;
    }
}

// The two normals of pair `pair` of stream `key`: element 2p -> r cos, 2p+1 -> r sin.
JINF_HD void normal_pair(uint64_t key, uint64_t pair, double* z0, double* z1) {
    const double u1 = to_unit(splitmix64(key + 2 * pair));
    const double u2 = to_unit(splitmix64(key + 2 * pair + 1));
    const double r = sqrt(-2.0 * det_log(u1));
    double sn, cs;
    det_sincos_2pi(u2, &sn, &cs);
    *z0 = r * cs;
    *z1 = r * sn;
}

// Element i of stream `key` scaled by stdv, rounded to fp32 first (same as the host path).
JINF_HD float normal_at(uint64_t key, uint64_t i, float stdv) {
    double z0, z1;
    normal_pair(key, i >> 1, &z0, &z1);
    return (float)((i & 1) ? z1 : z0) * stdv;
}

JINF_HD uint32_t f2u(float f) {
    union { uint32_t u; float f; } v;
    v.f = f;
    return v.u;
}
JINF_HD float u2f(uint32_t u) {
    union { uint32_t u; float f; } v;
    v.u = u;
    return v.f;
}

// fp32 -> fp16 bits, round to nearest even (bit manipulation only).
JINF_HD uint16_t fp32_to_fp16(float f) {
    const uint32_t x = f2u(f);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);
    if (ax < 0x38800000u) {
        if (ax < 0x33000000u) return (uint16_t)sign;
        const uint32_t e = ax >> 23;
        const uint32_t m = (ax & 0x7fffffu) | 0x800000u;
        const uint32_t shift = 126 - e;
        uint32_t q = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1);
        const uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1))) ++q;
        return (uint16_t)(sign | q);
    }
    const uint32_t e = (ax >> 23) - 112;
    const uint32_t m = ax & 0x7fffffu;
    uint32_t h = (e << 10) | (m >> 13);
    const uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1))) ++h;
    return (uint16_t)(sign | h);
}

JINF_HD float fabs_(float v) { return u2f(f2u(v) & 0x7fffffffu); }

// Streams of the sparse-FFN synthetic data: predictor matrix `which` (1: W1, 2: W2) of a
// layer, and a layer's fixed neuron mask.
JINF_HD uint64_t predictor_key(uint64_t seed, int layer, int which) {
    return splitmix64(seed ^ (0x5052454449435452ull + (uint64_t)layer * 0x9E3779B97F4A7C15ull +
                              (uint64_t)which * 0xD1B54A32D192ED03ull));
}
JINF_HD uint64_t mask_key(uint64_t seed, int layer) {
    return splitmix64(seed ^ (0x4D41534Bull + (uint64_t)layer * 0x9E3779B97F4A7C15ull));
}

// fp16 bits -> fp32 (exact: normal, subnormal, zero, inf, NaN).
JINF_HD float fp16_to_fp32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    const uint32_t exp = (h >> 10) & 0x1f;
    uint32_t man = h & 0x3ff;
    if (exp == 0x1f) return u2f(sign | 0x7f800000u | (man << 13));
    if (exp != 0) return u2f(sign | ((exp + 112) << 23) | (man << 13));
    if (man == 0) return u2f(sign);
    int e = -1;
    do {
        man <<= 1;
        ++e;
    } while ((man & 0x400) == 0);
    return u2f(sign | ((uint32_t)(112 - e) << 23) | ((man & 0x3ff) << 13));
}

// round to nearest, ties to even (lrintf in the default rounding mode)
JINF_HD int rint_i(float x) {
#ifdef __CUDA_ARCH__
    return __float2int_rn(x);
#else
    return (int)lrintf(x);
#endif
}

JINF_HD float fmin_(float a, float b) { return b < a ? b : a; }
JINF_HD float fmax_(float a, float b) { return b > a ? b : a; }

// Q4_K super-block from 256 floats, step for step the engine's host quantiser
// (jinf_quantize_q4_K, csrc/quant.cpp): per sub-block min m = -min(0, lo) and step
// s = (hi + m) / 15; d = max s / 63 and dmin = max m / 63 as fp16; 6-bit sc, m = rint(s / d),
// rint(m / dmin); q = clamp(rint((x + dmin m) / (d sc)), 0, 15). out: 144 bytes.
JINF_HD void quantize_q4_k_block(const float* v, uint8_t* out) {
    float s[8], m[8], smax = 0.f, mmax = 0.f;
    for (int j = 0; j < 8; ++j) {
        float lo = v[32 * j], hi = v[32 * j];
        for (int i = 1; i < 32; ++i) {
            lo = fmin_(lo, v[32 * j + i]);
            hi = fmax_(hi, v[32 * j + i]);
        }
        m[j] = lo < 0.f ? -lo : 0.f;
        s[j] = (hi + m[j]) / 15.f;
        smax = fmax_(smax, s[j]);
        mmax = fmax_(mmax, m[j]);
    }
    const uint16_t dh = fp32_to_fp16(smax / 63.f);
    const uint16_t mh = fp32_to_fp16(mmax / 63.f);
    const float d = fp16_to_fp32(dh), dmin = fp16_to_fp32(mh);
    int ls[8], lm[8];
    for (int j = 0; j < 8; ++j) {
        const int a = d > 0.f ? rint_i(s[j] / d) : 0;
        const int c = dmin > 0.f ? rint_i(m[j] / dmin) : 0;
        ls[j] = a < 0 ? 0 : (a > 63 ? 63 : a);
        lm[j] = c < 0 ? 0 : (c > 63 ? 63 : c);
    }
    out[0] = (uint8_t)(dh & 0xff);
    out[1] = (uint8_t)(dh >> 8);
    out[2] = (uint8_t)(mh & 0xff);
    out[3] = (uint8_t)(mh >> 8);
    uint8_t* sc = out + 4;
    for (int i = 0; i < 4; ++i) {
        sc[i] = (uint8_t)((ls[i] & 63) | ((ls[i + 4] & 3) << 6));
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
                const int qq = step > 0.f ? rint_i((val + off) / step) : 0;
                q[t] = qq < 0 ? 0 : (qq > 15 ? 15 : qq);
            }
            out[16 + 16 * j + i] = (uint8_t)(q[0] | (q[1] << 4));
        }
    }
}

// Q4_0 block from 32 floats: d = (value of largest magnitude)/-8, q = clamp(int(x/d+8.5)),
// reference nibble pairing (byte i = elements 2i | 2i+1 << 4). out: 18 bytes.
JINF_HD void quantize_q4_0_block(const float* v, uint8_t* out) {
    float amax = 0.f, vmax = 0.f;
    for (int i = 0; i < 32; ++i) {
        const float a = fabs_(v[i]);
        if (a > amax) {
            amax = a;
            vmax = v[i];
        }
    }
    const float d = vmax / -8.f;
    const float id = d != 0.f ? 1.f / d : 0.f;
    const uint16_t dh = fp32_to_fp16(d);
    out[0] = (uint8_t)(dh & 0xff);
    out[1] = (uint8_t)(dh >> 8);
    for (int i = 0; i < 16; ++i) {
        const float t0 = v[2 * i] * id, t1 = v[2 * i + 1] * id;
        int q0 = (int)(t0 + 8.5f), q1 = (int)(t1 + 8.5f);
        q0 = q0 < 0 ? 0 : (q0 > 15 ? 15 : q0);
        q1 = q1 < 0 ? 0 : (q1 > 15 ? 15 : q1);
        out[2 + i] = (uint8_t)(q0 | (q1 << 4));
    }
}

}  // namespace jinf_synth
