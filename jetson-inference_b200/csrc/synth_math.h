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
