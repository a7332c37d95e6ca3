// Engine decode attention over the fp16 KV cache, sm_100a.
//
// Math of reference cuda/attention_kernel.cu:45-98 (scores q.k / sqrt(hd), GQA head map
// h -> h / (H/Hkv), max-subtracted softmax, P.V), restated as split-K flash-decoding:
//   grid = n_kv_heads x n_split CTAs; CTA (h, s) covers positions [s*n/S, (s+1)*n/S)
//   for ALL query heads of kv head h, so each K/V row is read from HBM once (the
//   reference re-reads it once per query head). Each warp keeps an online-softmax
//   state per query head; lanes own positions for q.k and head dims for p.v.
//   The CTA's (m, l, acc) goes to a partial buffer; the last CTA of a kv head
//   (arrival counter, self-resetting for graph replay) merges the splits in fixed
//   order and writes the fp32 output [n_heads * hd].
// Cache layout: [n_kv_heads][max_ctx][hd] fp16 per layer; n = pos + 1 read from the
// device state, so one captured graph serves every position.
#include "common.cuh"
#include "q4t.cuh"
#include "attn_f16.h"

#include <math.h>

namespace jinf {

constexpr int AW = 4;       // warps per CTA
constexpr int AMAXG = 8;    // max query heads per kv head

template <int HD>
__global__ void __launch_bounds__(AW * 32) k_attn_f16(const AttnParams p) {
    constexpr int NJ = HD / 32;  // dims per lane in p.v
    const int kvh = blockIdx.x / p.n_split, split = blockIdx.x % p.n_split;
    const int G = p.n_heads / p.n_kv_heads;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;

    __shared__ __align__(16) float qs[AMAXG * HD];
    __shared__ float wacc[AW][AMAXG][HD];
    __shared__ float wm[AW][AMAXG], wl[AW][AMAXG];
    __shared__ int is_last;

    pdl_wait();
    pdl_trigger();
    const int n = p.st->pos + 1;
    const float scale = rsqrtf((float)HD);
    for (int i = threadIdx.x; i < G * HD; i += blockDim.x) qs[i] = p.q[(size_t)kvh * G * HD + i] * scale;
    __syncthreads();

    const int start = (int)((int64_t)n * split / p.n_split), end = (int)((int64_t)n * (split + 1) / p.n_split);
    const __half* kb = p.kcache + (size_t)kvh * p.max_ctx * HD;
    const __half* vb = p.vcache + (size_t)kvh * p.max_ctx * HD;

    float m[AMAXG], l[AMAXG], acc[AMAXG][NJ];
#pragma unroll
    for (int g = 0; g < AMAXG; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int j = 0; j < NJ; ++j) acc[g][j] = 0.f;
    }

    for (int t0 = start + 32 * wid; t0 < end; t0 += 32 * AW) {
        const int t = t0 + lane;
        const bool valid = t < end;
        float s[AMAXG];
#pragma unroll
        for (int g = 0; g < AMAXG; ++g) s[g] = 0.f;
        if (valid) {
            const uint4* kr = reinterpret_cast<const uint4*>(kb + (size_t)t * HD);
#pragma unroll 4
            for (int c = 0; c < HD / 8; ++c) {
                const uint4 raw = __ldg(kr + c);
                const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
                float kf[8];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = __half22float2(h2[e]);
                    kf[2 * e] = f.x;
                    kf[2 * e + 1] = f.y;
                }
#pragma unroll
                for (int g = 0; g < AMAXG; ++g) {
                    if (g < G) {
                        const float4 qa = *reinterpret_cast<const float4*>(qs + g * HD + 8 * c);
                        const float4 qb = *reinterpret_cast<const float4*>(qs + g * HD + 8 * c + 4);
                        s[g] = fmaf(qa.x, kf[0], s[g]); s[g] = fmaf(qa.y, kf[1], s[g]);
                        s[g] = fmaf(qa.z, kf[2], s[g]); s[g] = fmaf(qa.w, kf[3], s[g]);
                        s[g] = fmaf(qb.x, kf[4], s[g]); s[g] = fmaf(qb.y, kf[5], s[g]);
                        s[g] = fmaf(qb.z, kf[6], s[g]); s[g] = fmaf(qb.w, kf[7], s[g]);
                    }
                }
            }
        }
        float pr[AMAXG];
#pragma unroll
        for (int g = 0; g < AMAXG; ++g) {
            if (g >= G) { pr[g] = 0.f; continue; }
            const float sc = valid ? s[g] : -INFINITY;
            const float mn = fmaxf(m[g], warp_max(sc));
            const float corr = m[g] == -INFINITY ? 0.f : expf(m[g] - mn);
            pr[g] = valid ? expf(sc - mn) : 0.f;
            l[g] = l[g] * corr + warp_sum(pr[g]);
#pragma unroll
            for (int j = 0; j < NJ; ++j) acc[g][j] *= corr;
            m[g] = mn;
        }
        const int nt = min(32, end - t0);
        for (int tt = 0; tt < nt; ++tt) {
            const __half* vr = vb + (size_t)(t0 + tt) * HD + NJ * lane;
            float vv[NJ];
            if (NJ == 4) {
                const uint2 raw = __ldg(reinterpret_cast<const uint2*>(vr));
                const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
                const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
                vv[0] = a.x; vv[1] = a.y; vv[2 % NJ] = b.x; vv[3 % NJ] = b.y;
            } else {
#pragma unroll
                for (int j = 0; j < NJ; j += 2) {
                    const float2 a = __half22float2(__ldg(reinterpret_cast<const __half2*>(vr + j)));
                    vv[j] = a.x;
                    vv[j + 1] = a.y;
                }
            }
#pragma unroll
            for (int g = 0; g < AMAXG; ++g) {
                if (g >= G) continue;
                const float pg = __shfl_sync(JINF_FULL_MASK, pr[g], tt);
#pragma unroll
                for (int j = 0; j < NJ; ++j) acc[g][j] = fmaf(pg, vv[j], acc[g][j]);
            }
        }
    }

#pragma unroll
    for (int g = 0; g < AMAXG; ++g) {
        if (g >= G) continue;
#pragma unroll
        for (int j = 0; j < NJ; ++j) wacc[wid][g][NJ * lane + j] = acc[g][j];
        if (lane == 0) {
            wm[wid][g] = m[g];
            wl[wid][g] = l[g];
        }
    }
    __syncthreads();
    // CTA partial -> global
    float* part = p.partial + ((size_t)kvh * p.n_split + split) * (AMAXG * HD + 2 * AMAXG);
    for (int i = threadIdx.x; i < G * HD; i += blockDim.x) {
        const int g = i / HD, d = i % HD;
        float M = -INFINITY;
        for (int w = 0; w < AW; ++w) M = fmaxf(M, wm[w][g]);
        float a = 0.f, L = 0.f;
        if (M != -INFINITY) {
            for (int w = 0; w < AW; ++w) {
                if (wm[w][g] == -INFINITY) continue;
                const float f = expf(wm[w][g] - M);
                a = fmaf(wacc[w][g][d], f, a);
                L = fmaf(wl[w][g], f, L);
            }
        }
        part[g * HD + d] = a;
        if (d == 0) {
            part[AMAXG * HD + g] = M;
            part[AMAXG * HD + AMAXG + g] = L;
        }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned prev = atomicAdd(&p.st->attn_count[kvh], 1u);
        is_last = prev == (unsigned)(p.n_split - 1);
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    // merge the n_split partials of this kv head in split order
    const float* base = p.partial + (size_t)kvh * p.n_split * (AMAXG * HD + 2 * AMAXG);
    const size_t stride = AMAXG * HD + 2 * AMAXG;
    for (int i = threadIdx.x; i < G * HD; i += blockDim.x) {
        const int g = i / HD, d = i % HD;
        float M = -INFINITY;
        for (int s2 = 0; s2 < p.n_split; ++s2) M = fmaxf(M, __ldcg(base + s2 * stride + AMAXG * HD + g));
        float a = 0.f, L = 0.f;
        for (int s2 = 0; s2 < p.n_split; ++s2) {
            const float ms = __ldcg(base + s2 * stride + AMAXG * HD + g);
            if (ms == -INFINITY) continue;
            const float f = expf(ms - M);
            a = fmaf(__ldcg(base + s2 * stride + g * HD + d), f, a);
            L = fmaf(__ldcg(base + s2 * stride + AMAXG * HD + AMAXG + g), f, L);
        }
        p.out[(size_t)(kvh * G + g) * HD + d] = a / L;
    }
    if (threadIdx.x == 0) p.st->attn_count[kvh] = 0u;
}

size_t attn_partial_floats(int n_kv_heads, int n_split, int head_dim) {
    return (size_t)n_kv_heads * n_split * (AMAXG * head_dim + 2 * AMAXG);
}

cudaError_t attn_launch(const AttnParams& p, cudaStream_t s, bool pdl) {
    if (p.n_heads % p.n_kv_heads || p.n_heads / p.n_kv_heads > AMAXG || p.n_kv_heads > 64) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.n_kv_heads * p.n_split);
    cfg.blockDim = dim3(AW * 32);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    switch (p.head_dim) {
        case 64: return cudaLaunchKernelEx(&cfg, k_attn_f16<64>, p);
        case 128: return cudaLaunchKernelEx(&cfg, k_attn_f16<128>, p);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace jinf
