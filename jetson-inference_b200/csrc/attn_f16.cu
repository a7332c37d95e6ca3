// Engine decode attention over the fp16 KV cache, sm_100a.
//
// Math of reference cuda/attention_kernel.cu:45-98 (scores q.k / sqrt(hd), GQA head map
// h -> h / (H/Hkv), max-subtracted softmax, P.V), restated as split-K flash-decoding:
//   grid = n_kv_heads x n_split CTAs; of these, S = min(n_split, ceil(n / ATT_SPAN)) splits
//   hold positions (n = pos + 1 read at run time), CTA (h, s < S) covering [s*n/S,
//   (s+1)*n/S) for ALL query heads of kv head h, so each K/V row is read from HBM once (the
//   reference re-reads it once per query head), and every split has enough positions to
//   pay for its share of the merge.
//   Each warp takes 32-position tiles: the tile's K and V rows are copied into the
//   warp's shared memory with asynchronous 16-byte copies (all issued at once, one
//   wait), K chunk-swizzled so that lane-per-position reads are bank-conflict free.
//   Lanes own positions for q.k (online softmax per query head) and head dims for p.v.
//   The CTA's (m, l, acc) goes to a partial buffer; the last CTA of a kv head (arrival
//   counter, reset by that CTA for graph replay) merges the S splits in fixed order, every
//   load of a pass issued before the first is used.
// Cache layout: [n_kv_heads][max_ctx][hd] fp16 per layer; n = pos + 1 is read from the
// device state, so one captured graph serves every position.
#include "common.cuh"
#include "device_state.cuh"
#include "attn_f16.h"
#include "multi.h"

#include <math.h>

namespace jinf {

constexpr int AW = 4;      // warps per CTA
constexpr int AMAXG = 8;   // max query heads per kv head
constexpr int TP = 32;     // positions per warp tile
constexpr int ATT_SPAN = 64;  // fewest positions per split (more splits only for more positions)

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

template <int HD>
struct AttnSmem {
    static constexpr int CH = HD / 8;  // 16-byte chunks per K/V row
    float q[AMAXG * HD];
    __half k[AW][TP * HD];
    __half v[AW][TP * HD];
    float wacc[AW][AMAXG][HD];
    float wm[AW][AMAXG];
    float wl[AW][AMAXG];
    int is_last;
};

size_t attn_smem_bytes(int head_dim) {
    return head_dim == 64 ? sizeof(AttnSmem<64>) : sizeof(AttnSmem<128>);
}

template <int HD>
__global__ void __launch_bounds__(AW * 32) k_attn_f16(const AttnParams p) {
    constexpr int NJ = HD / 32;  // dims per lane in p.v
    constexpr int CH = HD / 8;
    extern __shared__ __align__(16) uint8_t smraw[];
    AttnSmem<HD>& sm = *reinterpret_cast<AttnSmem<HD>*>(smraw);
    const int kvh = blockIdx.x / p.n_split, split = blockIdx.x % p.n_split;
    const int G = p.n_heads / p.n_kv_heads;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;

    pdl_wait();
    pdl_trigger();
    // one sequence (st), or vector blockIdx.y of a multi-sequence step (ms)
    const int vec = blockIdx.y;
    const float* qv = p.q;
    float* outv = p.out;
    float* partv = p.partial;
    unsigned int* cntv = p.ms ? p.ms->attn_count + vec * MULTI_MAX_KV_HEADS : p.st->attn_count;
    size_t so = 0;
    int n;
    if (p.ms) {
        n = p.ms->pos[vec] + 1;
        so = (size_t)p.ms->seq[vec] * p.seq_stride;
        qv += (size_t)vec * p.q_stride;
        outv += (size_t)vec * p.q_stride;
        partv += (size_t)p.n_kv_heads * p.n_split * (AMAXG * HD + 2 * AMAXG) * vec;
    } else {
        n = p.st->pos + 1;
    }
    const float scale = rsqrtf((float)HD);
    {  // the kv head's query rows, float4 loads all in flight (G * HD / 4 <= 2 x 128 of them)
        const float4* q4 = reinterpret_cast<const float4*>(qv + (size_t)kvh * G * HD);
        float4 t[AMAXG * HD / 4 / (AW * 32)];
#pragma unroll
        for (int k = 0; k < AMAXG * HD / 4 / (AW * 32); ++k) {
            const int i = threadIdx.x + k * AW * 32;
            if (i < G * HD / 4) t[k] = q4[i];
        }
#pragma unroll
        for (int k = 0; k < AMAXG * HD / 4 / (AW * 32); ++k) {
            const int i = threadIdx.x + k * AW * 32;
            if (i < G * HD / 4)
                reinterpret_cast<float4*>(sm.q)[i] = make_float4(t[k].x * scale, t[k].y * scale, t[k].z * scale,
                                                                 t[k].w * scale);
        }
    }
    __syncthreads();

    const int ns = min(p.n_split, max(1, (n + ATT_SPAN - 1) / ATT_SPAN));  // splits with positions
    const int start = split < ns ? (int)((int64_t)n * split / ns) : n;
    const int end = split < ns ? (int)((int64_t)n * (split + 1) / ns) : n;
    const __half* kb = p.kcache + so + (size_t)kvh * p.max_ctx * HD;
    const __half* vb = p.vcache + so + (size_t)kvh * p.max_ctx * HD;
    __half* ksm = sm.k[wid];
    __half* vsm = sm.v[wid];

    float m[AMAXG], l[AMAXG], acc[AMAXG][NJ];
#pragma unroll
    for (int g = 0; g < AMAXG; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int j = 0; j < NJ; ++j) acc[g][j] = 0.f;
    }

    for (int t0 = start + TP * wid; t0 < end; t0 += TP * AW) {
        const int nt = min(TP, end - t0);
        // stage the tile: chunk c of row r lands at chunk (c ^ (r % CH)) of row r
        for (int i = lane; i < nt * CH; i += 32) {
            const int r = i / CH, c = i % CH;
            cp_async16(ksm + (r * CH + (c ^ (r % CH))) * 8, kb + (size_t)(t0 + r) * HD + c * 8);
            cp_async16(vsm + i * 8, vb + (size_t)(t0 + r) * HD + c * 8);
        }
        cp_async_wait_all();
        __syncwarp();

        const bool valid = lane < nt;
        float s[AMAXG];
#pragma unroll
        for (int g = 0; g < AMAXG; ++g) s[g] = 0.f;
        if (valid) {
#pragma unroll 4
            for (int c = 0; c < CH; ++c) {
                const uint4 raw = *reinterpret_cast<const uint4*>(ksm + (lane * CH + (c ^ (lane % CH))) * 8);
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
                        const float4 qa = *reinterpret_cast<const float4*>(sm.q + g * HD + 8 * c);
                        const float4 qb = *reinterpret_cast<const float4*>(sm.q + g * HD + 8 * c + 4);
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
            const float mn = fmaxf(m[g], warp_max(sc));  // finite: lane 0 is valid
            const float corr = m[g] == -INFINITY ? 0.f : expf(m[g] - mn);
            pr[g] = valid ? expf(sc - mn) : 0.f;
            l[g] = l[g] * corr + warp_sum(pr[g]);
#pragma unroll
            for (int j = 0; j < NJ; ++j) acc[g][j] *= corr;
            m[g] = mn;
        }
        for (int tt = 0; tt < nt; ++tt) {
            const __half* vr = vsm + tt * HD + NJ * lane;
            float vv[NJ];
#pragma unroll
            for (int j = 0; j < NJ; j += 2) {
                const float2 a = __half22float2(*reinterpret_cast<const __half2*>(vr + j));
                vv[j] = a.x;
                vv[j + 1] = a.y;
            }
#pragma unroll
            for (int g = 0; g < AMAXG; ++g) {
                if (g >= G) continue;
                const float pg = __shfl_sync(JINF_FULL_MASK, pr[g], tt);
#pragma unroll
                for (int j = 0; j < NJ; ++j) acc[g][j] = fmaf(pg, vv[j], acc[g][j]);
            }
        }
        __syncwarp();  // the next tile's copies overwrite this warp's K/V buffers
    }

#pragma unroll
    for (int g = 0; g < AMAXG; ++g) {
        if (g >= G) continue;
#pragma unroll
        for (int j = 0; j < NJ; ++j) sm.wacc[wid][g][NJ * lane + j] = acc[g][j];
        if (lane == 0) {
            sm.wm[wid][g] = m[g];
            sm.wl[wid][g] = l[g];
        }
    }
    __syncthreads();
    // CTA partial -> global
    const size_t stride = AMAXG * HD + 2 * AMAXG;
    float* part = partv + ((size_t)kvh * p.n_split + split) * stride;
    for (int i = threadIdx.x; i < G * HD; i += blockDim.x) {
        const int g = i / HD, d = i % HD;
        float M = -INFINITY;
        for (int w = 0; w < AW; ++w) M = fmaxf(M, sm.wm[w][g]);
        float a = 0.f, L = 0.f;
        if (M != -INFINITY) {
            for (int w = 0; w < AW; ++w) {
                if (sm.wm[w][g] == -INFINITY) continue;
                const float f = expf(sm.wm[w][g] - M);
                a = fmaf(sm.wacc[w][g][d], f, a);
                L = fmaf(sm.wl[w][g], f, L);
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
        const unsigned prev = atomicAdd(&cntv[kvh], 1u);
        sm.is_last = prev == (unsigned)(p.n_split - 1);
    }
    __syncthreads();
    if (!sm.is_last) return;
    __threadfence();
    // merge the ns partials of this kv head in split order. First every split's (m, l) of every
    // query head (one pass of loads), the weights f_s = exp(m_s - M) and L = sum f_s l_s; then
    // each thread adds float4s of the accumulators, eight splits' loads in flight at a time.
    const float* base = partv + (size_t)kvh * p.n_split * stride;
    float* fw = &sm.wacc[0][0][0];                  // [G][ns] m_s, then the weights
    float* fl = fw + AMAXG * p.n_split;             // [G][ns] l_s
    float* linv = &sm.wm[0][0];                     // [G] L
    for (int i = threadIdx.x; i < G * ns; i += blockDim.x) {
        const int g = i / ns, s2 = i % ns;
        fw[g * ns + s2] = __ldcg(base + s2 * stride + AMAXG * HD + g);
        fl[g * ns + s2] = __ldcg(base + s2 * stride + AMAXG * HD + AMAXG + g);
    }
    __syncthreads();
    if (threadIdx.x < G) {
        const int g = threadIdx.x;
        float M = -INFINITY;
        for (int s2 = 0; s2 < ns; ++s2) M = fmaxf(M, fw[g * ns + s2]);
        float L = 0.f;
        for (int s2 = 0; s2 < ns; ++s2) {
            const float ms = fw[g * ns + s2];
            const float f = ms == -INFINITY ? 0.f : expf(ms - M);
            fw[g * ns + s2] = f;
            L = fmaf(fl[g * ns + s2], f, L);
        }
        linv[g] = L;
    }
    __syncthreads();
    constexpr int D4 = HD / 4;
    for (int i = threadIdx.x; i < G * D4; i += blockDim.x) {
        const int g = i / D4, d4 = i % D4;
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int s0 = 0; s0 < ns; s0 += 8) {
            float4 t[8];
#pragma unroll
            for (int k = 0; k < 8; ++k)
                t[k] = s0 + k < ns ? __ldcg(reinterpret_cast<const float4*>(base + (s0 + k) * stride + g * HD) + d4)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float f = s0 + k < ns ? fw[g * ns + s0 + k] : 0.f;
                a.x = fmaf(t[k].x, f, a.x);
                a.y = fmaf(t[k].y, f, a.y);
                a.z = fmaf(t[k].z, f, a.z);
                a.w = fmaf(t[k].w, f, a.w);
            }
        }
        const float L = linv[g];
        *reinterpret_cast<float4*>(outv + (size_t)(kvh * G + g) * HD + 4 * d4) =
            make_float4(a.x / L, a.y / L, a.z / L, a.w / L);
    }
    if (threadIdx.x == 0) cntv[kvh] = 0u;
}

size_t attn_partial_floats(int n_kv_heads, int n_split, int head_dim) {
    return (size_t)n_kv_heads * n_split * (AMAXG * head_dim + 2 * AMAXG);
}

cudaError_t attn_launch(const AttnParams& p, cudaStream_t s, bool pdl) {
    if (p.n_heads % p.n_kv_heads || p.n_heads / p.n_kv_heads > AMAXG || p.n_kv_heads > 64) return cudaErrorInvalidValue;
    if (p.ms && (p.n_vec < 1 || p.n_vec > MULTI_MAX || p.n_kv_heads > MULTI_MAX_KV_HEADS)) return cudaErrorInvalidValue;
    // the merge keeps 2 x AMAXG x n_split floats in the CTA's accumulator scratch
    if (p.n_split < 1 || 2 * AMAXG * p.n_split > AW * AMAXG * p.head_dim) return cudaErrorInvalidValue;
    if (p.head_dim != 64 && p.head_dim != 128) return cudaErrorInvalidValue;
    const size_t smem = attn_smem_bytes(p.head_dim);
    static bool configured[2] = {false, false};
    const int which = p.head_dim == 64 ? 0 : 1;
    if (!configured[which]) {
        cudaError_t e = which == 0
            ? cudaFuncSetAttribute(k_attn_f16<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)
            : cudaFuncSetAttribute(k_attn_f16<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        configured[which] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.n_kv_heads * p.n_split, p.ms ? p.n_vec : 1);
    cfg.blockDim = dim3(AW * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return p.head_dim == 64 ? cudaLaunchKernelEx(&cfg, k_attn_f16<64>, p) : cudaLaunchKernelEx(&cfg, k_attn_f16<128>, p);
}

}  // namespace jinf
