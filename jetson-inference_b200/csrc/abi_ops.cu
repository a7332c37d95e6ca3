// Drop-in elementwise / normalisation / attention kernels of the reference C-ABI:
//   jinf_cuda_rmsnorm   (reference cuda/rmsnorm_kernel.cu)
//   jinf_cuda_rope      (reference cuda/rope_kernel.cu)
//   jinf_cuda_silu_mul  (reference cuda/silu_kernel.cu)
//   jinf_cuda_softmax   (reference cuda/softmax_kernel.cu)
//   jinf_cuda_attention (reference cuda/attention_kernel.cu)
//
// The attention entry point keeps the reference's fp32 cache layout
// [max_ctx][n_heads_kv * head_dim] but is split-K over positions: each kv head is
// served by one thread-block cluster, every CTA of the cluster covers a slice of the
// positions for all query heads of that kv head (the K/V rows are read once, not once
// per query head), and the partial softmax states are merged through distributed
// shared memory. No global scratch and no n_past-sized shared array are needed.
#include "common.cuh"
#include "jinf/kernels.h"

#include <cooperative_groups.h>
#include <math.h>

namespace cg = cooperative_groups;

// ------------------------------------------------------------------ rmsnorm

template <bool F16W>
__global__ void __launch_bounds__(1024) k_rmsnorm(float* out, const float* in, const void* w, int n, float eps) {
    __shared__ float red[32];
    float ss = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = in[i];
        ss = fmaf(v, v, ss);
    }
    ss = block_sum(ss, red);
    const float r = rsqrtf(ss / (float)n + eps);
    __syncthreads();  // all reads of `in` are done before an in-place write
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float wi = F16W ? jinf_h2f(reinterpret_cast<const uint16_t*>(w)[i]) : reinterpret_cast<const float*>(w)[i];
        out[i] = in[i] * r * wi;
    }
}

extern "C" void jinf_cuda_rmsnorm(float* output, const float* input, const void* weight, int n, float eps,
                                  int weight_type, cudaStream_t stream) {
    if (n <= 0) return;
    int threads = n < 1024 ? ((n + 31) / 32) * 32 : 1024;
    if (weight_type == 1)
        k_rmsnorm<true><<<1, threads, 0, stream>>>(output, input, weight, n, eps);
    else
        k_rmsnorm<false><<<1, threads, 0, stream>>>(output, input, weight, n, eps);
    jinf_check_launch("rmsnorm");
}

// ------------------------------------------------------------------ rope

__global__ void k_rope(float* q, float* k, int head_dim, int n_heads, int n_heads_kv, int pos, float base) {
    const int half = head_dim / 2;
    const int nq = n_heads * half, nk = n_heads_kv * half;
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= nq + nk) return;
    float* v = idx < nq ? q : k;
    const int p = idx < nq ? idx : idx - nq;
    const int head = p / half, i = p % half;
    const float theta = powf(base, -2.0f * (float)i / (float)head_dim);
    const float ang = (float)pos * theta;
    const float c = cosf(ang), s = sinf(ang);
    float* e = v + head * head_dim + 2 * i;
    const float x0 = e[0], x1 = e[1];
    e[0] = x0 * c - x1 * s;
    e[1] = x0 * s + x1 * c;
}

extern "C" void jinf_cuda_rope(float* q, float* k, int head_dim, int n_heads, int n_heads_kv, int pos,
                               float freq_base, cudaStream_t stream) {
    const int pairs = (n_heads + n_heads_kv) * (head_dim / 2);
    if (pairs <= 0) return;
    k_rope<<<(pairs + 255) / 256, 256, 0, stream>>>(q, k, head_dim, n_heads, n_heads_kv, pos, freq_base);
    jinf_check_launch("rope");
}

// ------------------------------------------------------------------ silu * up

__global__ void k_silu_mul(float* out, const float* g, const float* u, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float x = g[i];
    out[i] = x / (1.0f + expf(-x)) * u[i];
}

extern "C" void jinf_cuda_silu_mul(float* output, const float* gate, const float* up, int n, cudaStream_t stream) {
    if (n <= 0) return;
    k_silu_mul<<<(n + 255) / 256, 256, 0, stream>>>(output, gate, up, n);
    jinf_check_launch("silu_mul");
}

// ------------------------------------------------------------------ softmax

__global__ void __launch_bounds__(1024) k_softmax(float* out, const float* in, int n) {
    __shared__ float red[32];
    float m = -INFINITY;
    for (int i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, in[i]);
    m = block_max(m, red);
    float s = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s += expf(in[i] - m);
    s = block_sum(s, red);
    const float inv = 1.0f / s;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = expf(in[i] - m) * inv;
}

extern "C" void jinf_cuda_softmax(float* output, const float* input, int n, cudaStream_t stream) {
    if (n <= 0) return;
    int threads = n < 1024 ? ((n + 31) / 32) * 32 : 1024;
    k_softmax<<<1, threads, 0, stream>>>(output, input, n);
    jinf_check_launch("softmax");
}

// ------------------------------------------------------------------ attention (fp32 cache)

constexpr int ATT_WARPS = 4;
constexpr int ATT_CLUSTER = 8;
constexpr int ATT_MAXG = 8;  // query heads per kv head handled by one cluster pass

// Partial softmax state of one CTA: m, l per query head, acc per (head, dim).
struct AttnPartial {
    float m[ATT_MAXG];
    float l[ATT_MAXG];
};

// NJ = head_dim / 32 rounded up; lane owns dims lane + 32*j.
template <int NJ>
__global__ void __launch_bounds__(ATT_WARPS * 32) k_attention_f32(float* __restrict__ out, const float* __restrict__ q,
                                                                  const float* __restrict__ kc,
                                                                  const float* __restrict__ vc, int hd, int n_heads,
                                                                  int n_heads_kv, int n_past, int g0_base) {
    cg::cluster_group cluster = cg::this_cluster();
    const int crank = (int)cluster.block_rank();
    const int kvh = blockIdx.x / ATT_CLUSTER;
    const int G_all = n_heads / n_heads_kv;
    const int g0 = g0_base;  // first query head (within the group) of this pass
    const int G = min(ATT_MAXG, G_all - g0);
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int row_stride = n_heads_kv * hd;
    const float scale = rsqrtf((float)hd);

    extern __shared__ float sm[];
    float* qs = sm;                                      // [G][hd]
    float* wacc = qs + ATT_MAXG * hd;                    // [WARPS][G][hd]
    float* wml = wacc + ATT_WARPS * ATT_MAXG * hd;       // [WARPS][2][G]
    float* cacc = wml + ATT_WARPS * 2 * ATT_MAXG;        // [G][hd]   CTA partial (read remotely)
    float* cml = cacc + ATT_MAXG * hd;                   // [2][G]

    for (int i = threadIdx.x; i < G * hd; i += blockDim.x) {
        const int g = i / hd, d = i % hd;
        qs[i] = q[(size_t)(kvh * G_all + g0 + g) * hd + d];
    }
    __syncthreads();

    const int start = (int)((int64_t)n_past * crank / ATT_CLUSTER);
    const int end = (int)((int64_t)n_past * (crank + 1) / ATT_CLUSTER);

    float m[ATT_MAXG], l[ATT_MAXG], acc[ATT_MAXG][NJ];
#pragma unroll
    for (int g = 0; g < ATT_MAXG; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int j = 0; j < NJ; ++j) acc[g][j] = 0.f;
    }

    for (int t0 = start + 32 * wid; t0 < end; t0 += 32 * ATT_WARPS) {
        const int t = t0 + lane;
        const bool valid = t < end;
        float s[ATT_MAXG];
#pragma unroll
        for (int g = 0; g < ATT_MAXG; ++g) s[g] = 0.f;
        if (valid) {
            const float* kr = kc + (size_t)t * row_stride + (size_t)kvh * hd;
            for (int d = 0; d < hd; ++d) {
                const float kv = __ldg(kr + d);
#pragma unroll
                for (int g = 0; g < ATT_MAXG; ++g)
                    if (g < G) s[g] = fmaf(qs[g * hd + d], kv, s[g]);
            }
        }
        float p[ATT_MAXG];
#pragma unroll
        for (int g = 0; g < ATT_MAXG; ++g) {
            if (g >= G) { p[g] = 0.f; continue; }
            const float sc = valid ? s[g] * scale : -INFINITY;
            const float mt = warp_max(sc);
            const float mn = fmaxf(m[g], mt);  // finite: the tile has at least one valid lane
            const float corr = m[g] == -INFINITY ? 0.f : expf(m[g] - mn);
            p[g] = valid ? expf(sc - mn) : 0.f;
            l[g] = l[g] * corr + warp_sum(p[g]);
#pragma unroll
            for (int j = 0; j < NJ; ++j) acc[g][j] *= corr;
            m[g] = mn;
        }
        const int nt = min(32, end - t0);
        for (int tt = 0; tt < nt; ++tt) {
            const float* vr = vc + (size_t)(t0 + tt) * row_stride + (size_t)kvh * hd;
            float vv[NJ];
#pragma unroll
            for (int j = 0; j < NJ; ++j) {
                const int d = lane + 32 * j;
                vv[j] = d < hd ? __ldg(vr + d) : 0.f;
            }
#pragma unroll
            for (int g = 0; g < ATT_MAXG; ++g) {
                const float pg = __shfl_sync(JINF_FULL_MASK, p[g], tt);
#pragma unroll
                for (int j = 0; j < NJ; ++j) acc[g][j] = fmaf(pg, vv[j], acc[g][j]);
            }
        }
    }

    // warp partials -> shared
#pragma unroll
    for (int g = 0; g < ATT_MAXG; ++g) {
        if (g >= G) continue;
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
            const int d = lane + 32 * j;
            if (d < hd) wacc[(wid * ATT_MAXG + g) * hd + d] = acc[g][j];
        }
        if (lane == 0) {
            wml[(wid * 2 + 0) * ATT_MAXG + g] = m[g];
            wml[(wid * 2 + 1) * ATT_MAXG + g] = l[g];
        }
    }
    __syncthreads();
    // CTA combine
    for (int i = threadIdx.x; i < G * hd; i += blockDim.x) {
        const int g = i / hd, d = i % hd;
        float M = -INFINITY;
        for (int w = 0; w < ATT_WARPS; ++w) M = fmaxf(M, wml[(w * 2) * ATT_MAXG + g]);
        float a = 0.f, L = 0.f;
        if (M != -INFINITY) {
            for (int w = 0; w < ATT_WARPS; ++w) {
                const float mw = wml[(w * 2) * ATT_MAXG + g];
                if (mw == -INFINITY) continue;
                const float f = expf(mw - M);
                a = fmaf(wacc[(w * ATT_MAXG + g) * hd + d], f, a);
                L = fmaf(wml[(w * 2 + 1) * ATT_MAXG + g], f, L);
            }
        }
        cacc[g * hd + d] = a;
        if (d == 0) {
            cml[g] = M;
            cml[ATT_MAXG + g] = L;
        }
    }
    cluster.sync();
    if (crank == 0) {
        for (int i = threadIdx.x; i < G * hd; i += blockDim.x) {
            const int g = i / hd, d = i % hd;
            float M = -INFINITY;
            for (int r = 0; r < ATT_CLUSTER; ++r) M = fmaxf(M, cluster.map_shared_rank(cml, r)[g]);
            float a = 0.f, L = 0.f;
            for (int r = 0; r < ATT_CLUSTER; ++r) {
                const float mr = cluster.map_shared_rank(cml, r)[g];
                if (mr == -INFINITY) continue;
                const float f = expf(mr - M);
                a = fmaf(cluster.map_shared_rank(cacc, r)[g * hd + d], f, a);
                L = fmaf(cluster.map_shared_rank(cml, r)[ATT_MAXG + g], f, L);
            }
            out[(size_t)(kvh * G_all + g0 + g) * hd + d] = a / L;
        }
    }
    cluster.sync();  // keep every CTA's shared memory alive until rank 0 has read it
}

template <int NJ>
static cudaError_t launch_attention_f32(float* out, const float* q, const float* kc, const float* vc, int hd,
                                        int n_heads, int n_heads_kv, int n_past, int g0, cudaStream_t stream) {
    const size_t smem = sizeof(float) * (ATT_MAXG * hd + ATT_WARPS * ATT_MAXG * hd + ATT_WARPS * 2 * ATT_MAXG +
                                         ATT_MAXG * hd + 2 * ATT_MAXG);
    cudaFuncSetAttribute(k_attention_f32<NJ>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(n_heads_kv * ATT_CLUSTER);
    cfg.blockDim = dim3(ATT_WARPS * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = ATT_CLUSTER;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k_attention_f32<NJ>, out, q, kc, vc, hd, n_heads, n_heads_kv, n_past, g0);
}

extern "C" void jinf_cuda_attention(float* output, const float* q, const float* k_cache, const float* v_cache,
                                    int head_dim, int n_heads, int n_heads_kv, int n_past, int max_ctx,
                                    cudaStream_t stream) {
    if (n_past <= 0) return;
    if (head_dim <= 0 || head_dim > 256 || n_heads <= 0 || n_heads_kv <= 0 || n_heads % n_heads_kv ||
        n_past > max_ctx) {
        jinf_record_error(JINF_ERR_INVALID, "attention: bad arguments");
        return;
    }
    const int G = n_heads / n_heads_kv;
    const int nj = (head_dim + 31) / 32;
    for (int g0 = 0; g0 < G; g0 += ATT_MAXG) {
        cudaError_t e;
        if (nj <= 2) e = launch_attention_f32<2>(output, q, k_cache, v_cache, head_dim, n_heads, n_heads_kv, n_past, g0, stream);
        else if (nj <= 4) e = launch_attention_f32<4>(output, q, k_cache, v_cache, head_dim, n_heads, n_heads_kv, n_past, g0, stream);
        else e = launch_attention_f32<8>(output, q, k_cache, v_cache, head_dim, n_heads, n_heads_kv, n_past, g0, stream);
        if (e != cudaSuccess) {
            jinf_record_error(JINF_ERR_CUDA, "attention: launch");
            return;
        }
    }
    jinf_check_launch("attention");
}
