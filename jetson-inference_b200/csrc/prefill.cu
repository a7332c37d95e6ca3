// Batched prefill: the element-wise steps around the tensor-core projections
// (prefill_gemm.cu) and a causal attention over all prompt tokens at once, on the tensor
// cores (mma.sync m16n8k16, fp16 operands, fp32 accumulation and softmax).
//
// Per layer (reference src/engine.cpp:418-511, one token at a time there; every token of the
// prompt at once here):
//   rows_to_f16   RMSNorm(h) * gain (reference cuda/rmsnorm_kernel.cu:9-34: x * rsqrt(mean(x^2)
//                 + eps) * w) of every token row as fp16, prescaled by a power of two per row
//   [QKV GEMM]
//   rope_qkv      RoPE of q and k at the tokens' positions (cuda/rope_kernel.cu:8-50), K and V
//                 into the fp16 cache, q as fp16 scaled by 1/sqrt(hd)
//   attention     causal GQA attention of the prompt's queries over the cache
//                 (cuda/attention_kernel.cu:45-98 per token)
//   [o GEMM, residual add in its epilogue]
//   rows_to_f16   RMSNorm(h) * ffn gain
//   [gate|up GEMM]
//   silu_to_f16   SiLU(gate) * up (cuda/silu_kernel.cu:15-17) as fp16 rows
//   [down GEMM, residual add in its epilogue]
#include "common.cuh"
#include "mma_f16.cuh"
#include "prefill.h"
#include "q4m_device.cuh"

#include <cuda_fp16.h>

namespace jinf {
namespace {

constexpr int RT = 256;  // threads of the row kernels

__device__ __forceinline__ float block_sum(float v, float* sh) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(JINF_FULL_MASK, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) sh[w] = v;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < RT / 32; ++i) t += sh[i];
    return t;
}
__device__ __forceinline__ float block_max(float v, float* sh) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(JINF_FULL_MASK, v, o));
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) sh[w] = v;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < RT / 32; ++i) t = fmaxf(t, sh[i]);
    return t;
}

// Power of two s with amax * s in [2^13, 2^14) (1 for a zero row): the row's fp16 image keeps
// 11 significant bits at its largest elements whatever the row's range.
__device__ __forceinline__ float pow2_scale(float amax) {
    if (!(amax > 0.f)) return 1.f;
    int e;
    frexpf(amax, &e);  // amax in [2^(e-1), 2^e)
    return ldexpf(1.f, 14 - e);
}

// One token row per CTA: x = h * rsqrt(mean(h^2) + eps) * gain (norm) or x = h, as fp16 x * s,
// and tok_scale = 1 / s.
__global__ void __launch_bounds__(RT) k_rows_to_f16(const float* __restrict__ h, int ldh, int n,
                                                    const float* __restrict__ gain, float eps, int norm,
                                                    __half* __restrict__ x16, int ldx, float* __restrict__ tok_scale) {
    __shared__ float sh[RT / 32];
    const float* row = h + (size_t)blockIdx.x * ldh;
    float ss = 0.f, am = 0.f;
    for (int i = threadIdx.x; i < n; i += RT) {
        const float v = row[i];
        ss = fmaf(v, v, ss);
        am = fmaxf(am, fabsf(norm ? v * gain[i] : v));
    }
    const float r = norm ? rsqrtf(block_sum(ss, sh) / (float)n + eps) : 1.f;
    const float s = pow2_scale(block_max(am, sh) * r);
    __half* out = x16 + (size_t)blockIdx.x * ldx;
    for (int i = threadIdx.x; i < n; i += RT) {
        const float v = norm ? row[i] * r * gain[i] : row[i];
        out[i] = __float2half_rn(v * s);
    }
    if (threadIdx.x == 0) tok_scale[blockIdx.x] = 1.f / s;
}

// One token row per CTA: act = SiLU(g) * u over the interleaved gate|up row (g at 2i, u at
// 2i + 1), as fp16 act * s, tok_scale = 1 / s.
__global__ void __launch_bounds__(RT) k_silu_to_f16(const float* __restrict__ gu, int ldg, int ff,
                                                    __half* __restrict__ x16, int ldx, float* __restrict__ tok_scale) {
    __shared__ float sh[RT / 32];
    const float2* row = reinterpret_cast<const float2*>(gu + (size_t)blockIdx.x * ldg);
    float am = 0.f;
    for (int i = threadIdx.x; i < ff; i += RT) {
        const float2 p = row[i];
        am = fmaxf(am, fabsf(p.x / (1.0f + expf(-p.x)) * p.y));
    }
    const float s = pow2_scale(block_max(am, sh));
    __half* out = x16 + (size_t)blockIdx.x * ldx;
    for (int i = threadIdx.x; i < ff; i += RT) {
        const float2 p = row[i];
        out[i] = __float2half_rn(p.x / (1.0f + expf(-p.x)) * p.y * s);
    }
    if (threadIdx.x == 0) tok_scale[blockIdx.x] = 1.f / s;
}

// Embedding rows of the prompt tokens (f32 table) -> h [T][d].
__global__ void k_embed_rows(const float* __restrict__ table, const int* __restrict__ tokens, int d,
                             float* __restrict__ h) {
    const float4* src = reinterpret_cast<const float4*>(table + (size_t)tokens[blockIdx.x] * d);
    float4* dst = reinterpret_cast<float4*>(h + (size_t)blockIdx.x * d);
    for (int i = threadIdx.x; i < d / 4; i += blockDim.x) dst[i] = src[i];
}

// RoPE and the cache: thread (token t, adjacent pair i of the q|k|v row of Y). q and k pairs
// rotate at position p0 + t; q goes out as fp16 times 1/sqrt(hd), k and v into the cache.
__global__ void k_rope_qkv(const float* __restrict__ y, int ldy, int T, int p0, int nq, int nk, int hd, float base,
                           __half* __restrict__ q16, __half* __restrict__ kc, __half* __restrict__ vc, int max_ctx) {
    const int npair = (nq + 2 * nk) / 2;
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (long long)T * npair) return;
    const int t = (int)(idx / npair), pr = (int)(idx % npair), row = 2 * pr, pos = p0 + t;
    const float2 v = *reinterpret_cast<const float2*>(y + (size_t)t * ldy + row);
    float o0 = v.x, o1 = v.y;
    if (row < nq + nk) {
        float cs, sn;
        q4mdev::rope_pair(row < nq ? row : row - nq, pos, base, hd, cs, sn);
        o0 = v.x * cs - v.y * sn;
        o1 = v.x * sn + v.y * cs;
    }
    if (row < nq) {
        const float sc = rsqrtf((float)hd);
        *reinterpret_cast<__half2*>(q16 + (size_t)t * nq + row) = __floats2half2_rn(o0 * sc, o1 * sc);
    } else {
        const bool isk = row < nq + nk;
        const int rr = isk ? row - nq : row - nq - nk;
        const int kvh = rr / hd, dd = rr % hd;
        *reinterpret_cast<__half2*>((isk ? kc : vc) + ((size_t)kvh * max_ctx + pos) * hd + dd) = __floats2half2_rn(o0, o1);
    }
}

// ---------------------------------------------------------------- causal attention
//
// CTA (query block of 64 tokens, query head h) with 4 warps of 16 query rows; key blocks of 64
// positions of kv head h / (H / Hkv) staged in shared memory. S = Q K^T and O += P V on the
// tensor cores (m16n8k16, fp16 in, fp32 out), the online softmax in fp32 registers. Query
// token t (position p0 + t) sees positions 0 .. p0 + t.
constexpr int AQ = 64, AK = 64;

template <int HD>
__global__ void __launch_bounds__(128) k_prefill_attn(const __half* __restrict__ q16, int nq, int T, int p0,
                                                      const __half* __restrict__ kc, const __half* __restrict__ vc,
                                                      int max_ctx, int group, float* __restrict__ out) {
    constexpr int LD = HD + 8;  // padded row (halfs): 16-byte aligned rows, conflict-free ldmatrix
    extern __shared__ __align__(16) uint8_t sm[];
    __half* Qs = reinterpret_cast<__half*>(sm);
    __half* Ks = Qs + AQ * LD;
    __half* Vs = Ks + AK * LD;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, qd = lane & 3;
    const int qb = blockIdx.x * AQ, h = blockIdx.y, kvh = h / group;
    const __half* kbase = kc + (size_t)kvh * max_ctx * HD;
    const __half* vbase = vc + (size_t)kvh * max_ctx * HD;
    // Q tile (rows past T are zero)
    for (int i = tid; i < AQ * HD / 8; i += 128) {
        const int r = i / (HD / 8), c8 = i % (HD / 8);
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (qb + r < T) v = *reinterpret_cast<const uint4*>(q16 + (size_t)(qb + r) * nq + (size_t)h * HD + c8 * 8);
        *reinterpret_cast<uint4*>(Qs + r * LD + c8 * 8) = v;
    }
    __syncthreads();
    // this warp's Q fragments (16 rows x HD)
    uint32_t qa[HD / 16][4];
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
        const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, c = kk * 16 + (lane >> 4) * 8;
        ldsm_x4((uint32_t)__cvta_generic_to_shared(Qs + r * LD + c), qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3]);
    }
    float o[HD / 8][4];
#pragma unroll
    for (int j = 0; j < HD / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    const int qp0 = p0 + qb + warp * 16 + g, qp1 = qp0 + 8;  // positions of this thread's two rows
    const int kend = p0 + min(T, qb + AQ);                   // keys 0 .. kend - 1 can be seen
    for (int k0 = 0; k0 < kend; k0 += AK) {
        __syncthreads();  // the previous block's K and V are no longer read
        for (int i = tid; i < AK * HD / 8; i += 128) {
            const int r = i / (HD / 8), c8 = i % (HD / 8);
            uint4 kv = make_uint4(0u, 0u, 0u, 0u), vv = kv;
            if (k0 + r < kend) {
                kv = *reinterpret_cast<const uint4*>(kbase + (size_t)(k0 + r) * HD + c8 * 8);
                vv = *reinterpret_cast<const uint4*>(vbase + (size_t)(k0 + r) * HD + c8 * 8);
            }
            *reinterpret_cast<uint4*>(Ks + r * LD + c8 * 8) = kv;
            *reinterpret_cast<uint4*>(Vs + r * LD + c8 * 8) = vv;
        }
        __syncthreads();
        // S = Q K^T: 8 tiles of 8 keys
        float s[AK / 8][4];
#pragma unroll
        for (int j = 0; j < AK / 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
        for (int jj = 0; jj < AK / 16; ++jj) {
#pragma unroll
            for (int kk = 0; kk < HD / 16; ++kk) {
                uint32_t b0, b1, b2, b3;  // key tiles 2jj (b0, b1) and 2jj + 1 (b2, b3)
                const int r = jj * 16 + (lane & 7) + (lane >> 4) * 8, c = kk * 16 + ((lane >> 3) & 1) * 8;
                ldsm_x4((uint32_t)__cvta_generic_to_shared(Ks + r * LD + c), b0, b1, b2, b3);
                mma_f16(s[2 * jj], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b0, b1);
                mma_f16(s[2 * jj + 1], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b2, b3);
            }
        }
        // causal mask and the online softmax of the block (rows g and g + 8 of the warp)
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int j = 0; j < AK / 8; ++j) {
            const int kp = k0 + 8 * j + 2 * qd;
            if (kp > qp0 || kp >= kend) s[j][0] = -INFINITY;
            if (kp + 1 > qp0 || kp + 1 >= kend) s[j][1] = -INFINITY;
            if (kp > qp1 || kp >= kend) s[j][2] = -INFINITY;
            if (kp + 1 > qp1 || kp + 1 >= kend) s[j][3] = -INFINITY;
            mx0 = fmaxf(mx0, fmaxf(s[j][0], s[j][1]));
            mx1 = fmaxf(mx1, fmaxf(s[j][2], s[j][3]));
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(JINF_FULL_MASK, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(JINF_FULL_MASK, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(JINF_FULL_MASK, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(JINF_FULL_MASK, mx1, 2));
        const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
        // a row with no visible key in this block keeps its state (its max stays -inf here)
        const float c0 = n0 == -INFINITY ? 1.f : expf(m0 - n0), c1 = n1 == -INFINITY ? 1.f : expf(m1 - n1);
        float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
        for (int j = 0; j < AK / 8; ++j) {
            s[j][0] = s[j][0] == -INFINITY ? 0.f : expf(s[j][0] - n0);
            s[j][1] = s[j][1] == -INFINITY ? 0.f : expf(s[j][1] - n0);
            s[j][2] = s[j][2] == -INFINITY ? 0.f : expf(s[j][2] - n1);
            s[j][3] = s[j][3] == -INFINITY ? 0.f : expf(s[j][3] - n1);
            rs0 += s[j][0] + s[j][1];
            rs1 += s[j][2] + s[j][3];
        }
        rs0 += __shfl_xor_sync(JINF_FULL_MASK, rs0, 1);
        rs0 += __shfl_xor_sync(JINF_FULL_MASK, rs0, 2);
        rs1 += __shfl_xor_sync(JINF_FULL_MASK, rs1, 1);
        rs1 += __shfl_xor_sync(JINF_FULL_MASK, rs1, 2);
        l0 = l0 * c0 + rs0;
        l1 = l1 * c1 + rs1;
        m0 = n0;
        m1 = n1;
#pragma unroll
        for (int j = 0; j < HD / 8; ++j) {
            o[j][0] *= c0;
            o[j][1] *= c0;
            o[j][2] *= c1;
            o[j][3] *= c1;
        }
        // O += P V: k-steps of 16 keys, tiles of 8 head dims
#pragma unroll
        for (int ks = 0; ks < AK / 16; ++ks) {
            const uint32_t a0 = pack_h2(s[2 * ks][0], s[2 * ks][1]), a1 = pack_h2(s[2 * ks][2], s[2 * ks][3]);
            const uint32_t a2 = pack_h2(s[2 * ks + 1][0], s[2 * ks + 1][1]), a3 = pack_h2(s[2 * ks + 1][2], s[2 * ks + 1][3]);
#pragma unroll
            for (int jd = 0; jd < HD / 16; ++jd) {
                uint32_t b0, b1, b2, b3;  // dim tiles 2jd (b0, b1) and 2jd + 1 (b2, b3)
                const int r = ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, c = jd * 16 + (lane >> 4) * 8;
                ldsm_x4_t((uint32_t)__cvta_generic_to_shared(Vs + r * LD + c), b0, b1, b2, b3);
                mma_f16(o[2 * jd], a0, a1, a2, a3, b0, b1);
                mma_f16(o[2 * jd + 1], a0, a1, a2, a3, b2, b3);
            }
        }
    }
    // out = O / l for the rows inside the prompt
    const int t0r = qb + warp * 16 + g, t1r = t0r + 8;
    const float i0 = l0 > 0.f ? 1.f / l0 : 0.f, i1 = l1 > 0.f ? 1.f / l1 : 0.f;
#pragma unroll
    for (int j = 0; j < HD / 8; ++j) {
        const int d = j * 8 + 2 * qd;
        if (t0r < T)
            *reinterpret_cast<float2*>(out + (size_t)t0r * nq + (size_t)h * HD + d) = make_float2(o[j][0] * i0, o[j][1] * i0);
        if (t1r < T)
            *reinterpret_cast<float2*>(out + (size_t)t1r * nq + (size_t)h * HD + d) = make_float2(o[j][2] * i1, o[j][3] * i1);
    }
}

}  // namespace

cudaError_t prefill_rows_to_f16(const float* h, int ldh, int T, int n, const float* gain, float eps, __half* x16,
                                int ldx, float* tok_scale, cudaStream_t s) {
    k_rows_to_f16<<<T, RT, 0, s>>>(h, ldh, n, gain, eps, gain ? 1 : 0, x16, ldx, tok_scale);
    return cudaGetLastError();
}

cudaError_t prefill_silu_to_f16(const float* gu, int ldg, int T, int ff, __half* x16, int ldx, float* tok_scale,
                                cudaStream_t s) {
    k_silu_to_f16<<<T, RT, 0, s>>>(gu, ldg, ff, x16, ldx, tok_scale);
    return cudaGetLastError();
}

cudaError_t prefill_embed(const float* table, const int* tokens, int T, int d, float* h, cudaStream_t s) {
    k_embed_rows<<<T, 256, 0, s>>>(table, tokens, d, h);
    return cudaGetLastError();
}

cudaError_t prefill_rope_qkv(const float* y, int ldy, int T, int p0, int nq, int nk, int hd, float base, __half* q16,
                             __half* kc, __half* vc, int max_ctx, cudaStream_t s) {
    const long long n = (long long)T * ((nq + 2 * nk) / 2);
    k_rope_qkv<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(y, ldy, T, p0, nq, nk, hd, base, q16, kc, vc, max_ctx);
    return cudaGetLastError();
}

cudaError_t prefill_attention(const __half* q16, int n_heads, int n_kv_heads, int hd, int T, int p0, const __half* kc,
                              const __half* vc, int max_ctx, float* out, cudaStream_t s) {
    if (hd != 64 && hd != 128) return cudaErrorInvalidValue;
    const dim3 grid((unsigned)((T + AQ - 1) / AQ), (unsigned)n_heads);
    const size_t smem = (size_t)(AQ + 2 * AK) * (hd + 8) * sizeof(__half);
    const int group = n_heads / n_kv_heads;
    if (hd == 128) {
        static bool cfg = false;
        if (!cfg) {
            const cudaError_t e = cudaFuncSetAttribute(k_prefill_attn<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                       (int)smem);
            if (e != cudaSuccess) return e;
            cfg = true;
        }
        k_prefill_attn<128><<<grid, 128, smem, s>>>(q16, n_heads * hd, T, p0, kc, vc, max_ctx, group, out);
    } else {
        k_prefill_attn<64><<<grid, 128, smem, s>>>(q16, n_heads * hd, T, p0, kc, vc, max_ctx, group, out);
    }
    return cudaGetLastError();
}

}  // namespace jinf
