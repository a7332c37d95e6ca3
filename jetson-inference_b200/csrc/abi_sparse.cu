// jinf_cuda_sparse_ffn: FFN over the neuron bundles of the active neurons
// (reference cuda/sparse_matmul.cu:223-282, bundle layout tools/prepare_model.cpp:299-308).
//
// Phase 1: one warp per active neuron computes silu(gate . x) * (up . x) for Q4_0, Q8_0,
//          Q4_K or Q6_K rows (each format decoded as itself; Q4_0 through a vectorised path).
// Phase 2: output[d] = sum_i a_i * down_col_i[d]. A cluster of 8 CTAs splits the active
//          list; each thread owns 16 bytes of output rows and a subset of the columns, and
//          the partial sums are added in a fixed order through shared and distributed shared
//          memory: deterministic, no atomics, no memset, no scratch beyond the caller's
//          gate_up_tmp. It is launched as a programmatic dependent of phase 1, so its first
//          column loads overlap phase 1.
#include "common.cuh"
#include "jinf/quant.h"
#include "jinf/sparse_ops.h"
#include "sparse_engine.h"

#include <cooperative_groups.h>

namespace cg = cooperative_groups;

__device__ __forceinline__ uint32_t ld_u16(const uint8_t* p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8); }

// Dot product of one quantized row (hidden_dim weights) with x; result in every lane.
__device__ float warp_row_dot(const uint8_t* row, int qtype, const float* __restrict__ x, int n) {
    const int lane = threadIdx.x & 31;
    float acc = 0.f;
    if (qtype == JINF_TYPE_Q4_0 || qtype == JINF_TYPE_Q8_0) {
        const int bb = qtype == JINF_TYPE_Q4_0 ? 18 : 34;
        for (int b = lane; b < n / 32; b += 32) {
            const uint8_t* blk = row + (size_t)b * bb;
            const float d = jinf_h2f((uint16_t)ld_u16(blk));
            float s = 0.f;
            if (qtype == JINF_TYPE_Q4_0) {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const uint32_t v = blk[2 + i];
                    s = fmaf((float)((int)(v & 15) - 8), __ldg(x + 32 * b + 2 * i), s);
                    s = fmaf((float)((int)(v >> 4) - 8), __ldg(x + 32 * b + 2 * i + 1), s);
                }
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) s = fmaf((float)(int8_t)blk[2 + i], __ldg(x + 32 * b + i), s);
            }
            acc = fmaf(s, d, acc);
        }
    } else if (qtype == JINF_TYPE_Q4_K) {
        const int j = lane >> 2;
        for (int b = 0; b < n / 256; ++b) {
            const jinf_block_q4_K* blk = reinterpret_cast<const jinf_block_q4_K*>(row + (size_t)b * 144);
            int sc, mn;
            q4k_scale_min_dev(blk->scales, j, sc, mn);
            const float sd = __fmul_rn(jinf_h2f(blk->d), (float)sc), smn = __fmul_rn(jinf_h2f(blk->dmin), (float)mn);
            const uint8_t* q = blk->qs + 16 * j + 4 * (lane & 3);
            const float* xb = x + 256 * b + 8 * lane;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                acc = fmaf(__fsub_rn(__fmul_rn(sd, (float)(q[i] & 15)), smn), __ldg(xb + 2 * i), acc);
                acc = fmaf(__fsub_rn(__fmul_rn(sd, (float)(q[i] >> 4)), smn), __ldg(xb + 2 * i + 1), acc);
            }
        }
    } else {  // Q6_K
        for (int b = 0; b < n / 256; ++b) {
            const uint8_t* blk = row + (size_t)b * 210;
            const float d = jinf_h2f((uint16_t)ld_u16(blk + 208));
            const int e0 = 8 * lane;
            const float s = __fmul_rn(d, (float)(int8_t)blk[192 + (e0 >> 4)]);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int e = e0 + i;
                const int lo = (blk[e >> 1] >> ((e & 1) * 4)) & 15;
                const int hi = (blk[128 + (e >> 2)] >> (2 * (e & 3))) & 3;
                acc = fmaf(__fmul_rn(s, (float)((lo | (hi << 4)) - 32)), __ldg(x + 256 * b + e), acc);
            }
        }
    }
    return warp_sum(acc);
}

__global__ void k_sparse_gate_up(const uint8_t* __restrict__ bundles, const float* __restrict__ x,
                                 float* __restrict__ gu, const int* __restrict__ offs, int n_act, int hidden,
                                 int row_bytes, int qtype) {
    const int i = (int)(((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    if (i >= n_act) return;
    const uint8_t* b = bundles + offs[i];
    const float g = warp_row_dot(b, qtype, x, hidden);
    const float u = warp_row_dot(b + row_bytes, qtype, x, hidden);
    if ((threadIdx.x & 31) == 0) gu[i] = g / (1.0f + expf(-g)) * u;
}

// Q4_0 gate/up rows, the common case: x is staged transposed in shared memory, xs[e][b]
// (element e of block b), so that the x values of four consecutive blocks at one element are
// one conflict-free 16-byte load. Lane l covers blocks 4l..4l+3 (+128 per round): 72
// contiguous bytes per row, read as nine 8-byte loads, a warp's loads covering 2304
// contiguous bytes. Needs hidden % 128 == 0 and hidden <= 8192; rows off 8-byte alignment
// (checked per neuron) take a per-block path over the same staged x. With h_in set, x = RMSNorm(h_in + y_res) * gain
// is computed here by every CTA (CTA 0 stores h_out), which fuses the FFN prologue.
constexpr int SPG_WARPS = 8, SPG_THREADS = SPG_WARPS * 32, SPG_MAX_HIDDEN = 8192;

struct SpNorm {
    const float* h_in;  // nullptr: x is given
    const float* y_res;
    float* h_out;
    const float* gain;
    float eps;
};

__global__ void __launch_bounds__(SPG_THREADS)
    k_sparse_gate_up_q40(const uint8_t* __restrict__ bundles, const float* __restrict__ x, float* __restrict__ gu,
                         const int* __restrict__ offs, int n_act, int hidden, int row_bytes, SpNorm nm) {
    extern __shared__ float4 xs4[];
    __shared__ float red[32];
    pdl_trigger();  // the down kernel may start loading its columns
    const int tid = threadIdx.x;
    const int nb = hidden >> 5, nq = nb >> 2, n4 = hidden >> 2;
    constexpr int XU = SPG_MAX_HIDDEN / 4 / SPG_THREADS;  // 16-byte pieces of x per thread
    float4 v[XU];
    if (nm.h_in) {
        float ss = 0.f;
#pragma unroll
        for (int u = 0; u < XU; ++u) {
            const int i = tid + SPG_THREADS * u;
            v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (i < n4) {
                const float4 a = __ldg(reinterpret_cast<const float4*>(nm.h_in) + i);
                const float4 c = __ldg(reinterpret_cast<const float4*>(nm.y_res) + i);
                v[u] = make_float4(a.x + c.x, a.y + c.y, a.z + c.z, a.w + c.w);
                if (blockIdx.x == 0) reinterpret_cast<float4*>(nm.h_out)[i] = v[u];
                ss = fmaf(v[u].x, v[u].x, ss);
                ss = fmaf(v[u].y, v[u].y, ss);
                ss = fmaf(v[u].z, v[u].z, ss);
                ss = fmaf(v[u].w, v[u].w, ss);
            }
        }
        const float r = rsqrtf(block_sum(ss, red) / (float)hidden + nm.eps);
#pragma unroll
        for (int u = 0; u < XU; ++u) {
            const int i = tid + SPG_THREADS * u;
            if (i < n4) {
                const float4 g = __ldg(reinterpret_cast<const float4*>(nm.gain) + i);
                v[u] = make_float4(v[u].x * r * g.x, v[u].y * r * g.y, v[u].z * r * g.z, v[u].w * r * g.w);
            }
        }
    } else {
#pragma unroll
        for (int u = 0; u < XU; ++u) {
            const int i = tid + SPG_THREADS * u;
            v[u] = i < n4 ? __ldg(reinterpret_cast<const float4*>(x) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    float* xs = reinterpret_cast<float*>(xs4);
#pragma unroll
    for (int u = 0; u < XU; ++u) {
        const int i = tid + SPG_THREADS * u;
        if (i < n4) {  // elements 4i..4i+3: block (4i) >> 5, elements (4i & 31) + 0..3
            const int b = i >> 3, e = (4 * i) & 31;
            xs[e * nb + b] = v[u].x;
            xs[(e + 1) * nb + b] = v[u].y;
            xs[(e + 2) * nb + b] = v[u].z;
            xs[(e + 3) * nb + b] = v[u].w;
        }
    }
    __syncthreads();
    const int lane = tid & 31;
    const int n = blockIdx.x * SPG_WARPS + (tid >> 5);
    if (n >= n_act) return;
    const uint8_t* g = bundles + __ldg(offs + n);
    const uint8_t* u = g + row_bytes;
    float ag = 0.f, au = 0.f;
    if ((((uintptr_t)g | (uintptr_t)u) & 7) == 0) {
        for (int q = lane; q < nq; q += 32) {
            uint32_t wg[18], wu[18];
            const uint2* pg = reinterpret_cast<const uint2*>(g + 72 * q);
            const uint2* pu = reinterpret_cast<const uint2*>(u + 72 * q);
#pragma unroll
            for (int k = 0; k < 9; ++k) {
                const uint2 a = __ldg(pg + k), c = __ldg(pu + k);
                wg[2 * k] = a.x; wg[2 * k + 1] = a.y;
                wu[2 * k] = c.x; wu[2 * k + 1] = c.y;
            }
            // byte k of the 72-byte span
#define SP_BYTE(w, k) (((w)[(k) >> 2] >> (8 * ((k) & 3))) & 0xFFu)
            float sg[4] = {0.f, 0.f, 0.f, 0.f}, su[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int e = 0; e < 32; ++e) {
                const float4 xv4 = xs4[e * nq + q];
                const float xv[4] = {xv4.x, xv4.y, xv4.z, xv4.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int k = 18 * i + 2 + (e >> 1), sh = (e & 1) * 4;
                    // (q - 8) exactly: the nibble placed in the mantissa of 2^23, minus 2^23 + 8
                    const float qg = __int_as_float(0x4B000000 | ((SP_BYTE(wg, k) >> sh) & 15)) - 8388616.0f;
                    const float qu = __int_as_float(0x4B000000 | ((SP_BYTE(wu, k) >> sh) & 15)) - 8388616.0f;
                    sg[i] = fmaf(qg, xv[i], sg[i]);
                    su[i] = fmaf(qu, xv[i], su[i]);
                }
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t dg = SP_BYTE(wg, 18 * i) | (SP_BYTE(wg, 18 * i + 1) << 8);
                const uint32_t du = SP_BYTE(wu, 18 * i) | (SP_BYTE(wu, 18 * i + 1) << 8);
                ag = fmaf(sg[i], jinf_h2f((uint16_t)dg), ag);
                au = fmaf(su[i], jinf_h2f((uint16_t)du), au);
            }
#undef SP_BYTE
        }
        ag = warp_sum(ag);
        au = warp_sum(au);
    } else {
        // rows off 8-byte alignment: lane per block, byte loads, x from the staged copy
        for (int b = lane; b < nb; b += 32) {
            const uint8_t* bg = g + 18 * b;
            const uint8_t* bu = u + 18 * b;
            float sg = 0.f, su = 0.f;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const uint32_t vg = bg[2 + i], vu = bu[2 + i];
                const float x0 = xs[(2 * i) * nb + b], x1 = xs[(2 * i + 1) * nb + b];
                sg = fmaf((float)((int)(vg & 15) - 8), x0, sg);
                sg = fmaf((float)((int)(vg >> 4) - 8), x1, sg);
                su = fmaf((float)((int)(vu & 15) - 8), x0, su);
                su = fmaf((float)((int)(vu >> 4) - 8), x1, su);
            }
            ag = fmaf(sg, jinf_h2f((uint16_t)ld_u16(bg)), ag);
            au = fmaf(su, jinf_h2f((uint16_t)ld_u16(bu)), au);
        }
        ag = warp_sum(ag);
        au = warp_sum(au);
    }
    if (lane == 0) gu[n] = ag / (1.0f + expf(-ag)) * au;
}

constexpr int SP_CLUSTER = 8;

// Phase 2, vectorised: a CTA covers SPD_ROWS output rows as 16-byte slots; its threads are
// (slot, column subset) pairs. A thread loads the offsets of SPD_U of its columns, then 16
// bytes of each (the first batch before the dependency wait on the gate/up kernel), then
// accumulates. Partial sums are added in subset order in shared memory and in cluster-rank
// order through distributed shared memory.
constexpr int SPD_ROWS = 128, SPD_THREADS = 512, SPD_SLOTS = SPD_ROWS / 4, SPD_SUBS = SPD_THREADS / SPD_SLOTS,
              SPD_U = 8;

// 16 bytes of a down column at float index r: one 16-byte load when the address is 16-byte
// aligned, else four 4-byte loads. Predicated rather than branched, so that a thread's loads
// of a batch are all in flight together.
__device__ __forceinline__ float4 sp_col4(const uint8_t* col, int r) {
    const float* f = reinterpret_cast<const float*>(col) + r;
    const uint32_t al = (((uintptr_t)f) & 15) == 0;
    float4 v;
    asm("{\n\t.reg .pred p;\n\t"
        "setp.ne.u32 p, %4, 0;\n\t"
        "@p ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%5];\n\t"
        "@!p ld.global.nc.f32 %0, [%5];\n\t"
        "@!p ld.global.nc.f32 %1, [%5+4];\n\t"
        "@!p ld.global.nc.f32 %2, [%5+8];\n\t"
        "@!p ld.global.nc.f32 %3, [%5+12];\n\t}"
        : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
        : "r"(al), "l"(f));
    return v;
}

__global__ void __launch_bounds__(SPD_THREADS, 2)
    k_sparse_down_v4(const uint8_t* __restrict__ bundles, float* __restrict__ out, const float* __restrict__ gu,
                     const int* __restrict__ offs, int n_act, int hidden, int down_off) {
    cg::cluster_group cluster = cg::this_cluster();
    __shared__ float4 part[SPD_THREADS];
    const int rank = (int)cluster.block_rank();
    const int chunk = blockIdx.x / SP_CLUSTER;
    const int slot = threadIdx.x % SPD_SLOTS, sub = threadIdx.x / SPD_SLOTS;
    const int r = chunk * SPD_ROWS + 4 * slot;
    const bool live = r < hidden;
    const int r_ld = live ? r : 0;  // rows past the end load row 0 and weigh it by zero
    const int i0 = (int)((int64_t)n_act * rank / SP_CLUSTER), i1 = (int)((int64_t)n_act * (rank + 1) / SP_CLUSTER);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    bool waited = false;
    // every load below is unconditional (indices past the range read column 0, n_act >= 1, and
    // are weighed by zero), so a batch's loads issue back to back
    for (int i = i0 + sub; i < i1 || !waited; i += SPD_U * SPD_SUBS) {
        int ic[SPD_U];
        float4 v[SPD_U];
#pragma unroll
        for (int k = 0; k < SPD_U; ++k) {
            const int ii = i + k * SPD_SUBS;
            ic[k] = ii < i1 ? ii : 0;
        }
        int off[SPD_U];
#pragma unroll
        for (int k = 0; k < SPD_U; ++k) off[k] = __ldg(offs + ic[k]);
#pragma unroll
        for (int k = 0; k < SPD_U; ++k) v[k] = sp_col4(bundles + off[k] + down_off, r_ld);
        if (!waited) {
            pdl_wait();  // gate/up results, and the end of its reads of x (which `out` may alias)
            waited = true;
        }
        // gate/up results: written by the concurrent primary grid, so a coherent (L2) load that
        // cannot be hoisted above the wait, never the read-only path
        float a[SPD_U];
#pragma unroll
        for (int k = 0; k < SPD_U; ++k) a[k] = __ldcg(gu + ic[k]);
#pragma unroll
        for (int k = 0; k < SPD_U; ++k) {
            const float w = i + k * SPD_SUBS < i1 ? a[k] : 0.f;
            acc.x = fmaf(w, v[k].x, acc.x);
            acc.y = fmaf(w, v[k].y, acc.y);
            acc.z = fmaf(w, v[k].z, acc.z);
            acc.w = fmaf(w, v[k].w, acc.w);
        }
    }
    part[threadIdx.x] = acc;
    __syncthreads();
    if (threadIdx.x < SPD_SLOTS) {
        float4 t0 = part[threadIdx.x];
        for (int q = 1; q < SPD_SUBS; ++q) {
            const float4 t = part[q * SPD_SLOTS + threadIdx.x];
            t0.x += t.x; t0.y += t.y; t0.z += t.z; t0.w += t.w;
        }
        part[threadIdx.x] = t0;
    }
    cluster.sync();
    if (rank == 0 && threadIdx.x < SPD_SLOTS && live) {
        float4 t0 = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int q = 0; q < SP_CLUSTER; ++q) {
            const float4 t = cluster.map_shared_rank(part, q)[threadIdx.x];
            t0.x += t.x; t0.y += t.y; t0.z += t.z; t0.w += t.w;
        }
        *reinterpret_cast<float4*>(out + r) = t0;
    }
    cluster.sync();
}

// Phase 2 for hidden sizes that are not a multiple of 4: one thread per output row.
__global__ void __launch_bounds__(256) k_sparse_down(const uint8_t* __restrict__ bundles, float* __restrict__ out,
                                                     const float* __restrict__ gu, const int* __restrict__ offs,
                                                     int n_act, int hidden, int down_off) {
    cg::cluster_group cluster = cg::this_cluster();
    __shared__ float part[256];
    const int rank = (int)cluster.block_rank();
    const int chunk = blockIdx.x / SP_CLUSTER;
    const int d = chunk * 256 + threadIdx.x;
    const int i0 = (int)((int64_t)n_act * rank / SP_CLUSTER), i1 = (int)((int64_t)n_act * (rank + 1) / SP_CLUSTER);
    float acc = 0.f;
    pdl_wait();
    if (d < hidden) {
        for (int i = i0; i < i1; ++i) {
            const float* col = reinterpret_cast<const float*>(bundles + offs[i] + down_off);
            acc = fmaf(__ldcg(gu + i), __ldg(col + d), acc);
        }
    }
    part[threadIdx.x] = acc;
    cluster.sync();
    if (rank == 0 && d < hidden) {
        float s = 0.f;
        for (int r = 0; r < SP_CLUSTER; ++r) s += cluster.map_shared_rank(part, r)[threadIdx.x];
        out[d] = s;
    }
    cluster.sync();
}

// Both phases; nm.h_in set = fused prologue (fast gate/up path only). Returns the first launch
// error.
static cudaError_t sparse_ffn_run(const void* bundles, const float* input, float* output, const int* bundle_offsets,
                           int num_activated, int hidden_dim, int qtype, float* gate_up_tmp, const SpNorm& nm,
                           cudaStream_t stream) {
    const int bs = jinf_qtype_block_size((jinf_qtype)qtype);
    const int row_bytes = (int)((size_t)(hidden_dim / bs) * jinf_qtype_type_size((jinf_qtype)qtype));
    const bool fast_gu = qtype == JINF_TYPE_Q4_0 && hidden_dim % 128 == 0 && hidden_dim <= SPG_MAX_HIDDEN;
    if (fast_gu) {
        const size_t smem = sizeof(float) * (size_t)hidden_dim;
        k_sparse_gate_up_q40<<<(unsigned)((num_activated + SPG_WARPS - 1) / SPG_WARPS), SPG_THREADS, smem, stream>>>(
            (const uint8_t*)bundles, input, gate_up_tmp, bundle_offsets, num_activated, hidden_dim, row_bytes, nm);
    } else {
        const int64_t threads = (int64_t)num_activated * 32;
        k_sparse_gate_up<<<(unsigned)((threads + 255) / 256), 256, 0, stream>>>(
            (const uint8_t*)bundles, input, gate_up_tmp, bundle_offsets, num_activated, hidden_dim, row_bytes, qtype);
    }
    const cudaError_t ge = cudaGetLastError();
    if (ge != cudaSuccess) return ge;
    // The down kernel starts early (programmatic dependent launch) and waits on the gate/up
    // kernel before it reads gate_up_tmp or writes `output` (which may alias `input`).
    const bool vec = hidden_dim % 4 == 0;
    const int rows_per_cta = vec ? SPD_ROWS : 256;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(((hidden_dim + rows_per_cta - 1) / rows_per_cta) * SP_CLUSTER);
    cfg.blockDim = dim3(vec ? SPD_THREADS : 256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = SP_CLUSTER;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    const cudaError_t le =
        vec ? cudaLaunchKernelEx(&cfg, k_sparse_down_v4, (const uint8_t*)bundles, output, (const float*)gate_up_tmp,
                                 bundle_offsets, num_activated, hidden_dim, 2 * row_bytes)
            : cudaLaunchKernelEx(&cfg, k_sparse_down, (const uint8_t*)bundles, output, (const float*)gate_up_tmp,
                                 bundle_offsets, num_activated, hidden_dim, 2 * row_bytes);
    return le;
}

extern "C" void jinf_cuda_sparse_ffn(const void* bundles, const float* input, float* output,
                                     const int* bundle_offsets, int num_activated, int hidden_dim,
                                     int bundle_size, int qtype, float* gate_up_tmp, cudaStream_t stream) {
    (void)bundle_size;  // offsets are explicit; the size only bounds them on the caller side
    if (hidden_dim <= 0) return;
    const int bs = jinf_qtype_block_size((jinf_qtype)qtype);
    if (qtype != JINF_TYPE_Q4_0 && qtype != JINF_TYPE_Q8_0 && qtype != JINF_TYPE_Q4_K && qtype != JINF_TYPE_Q6_K) {
        jinf_record_error(JINF_ERR_INVALID, "sparse_ffn: unsupported qtype");
        return;
    }
    if (hidden_dim % bs) {
        jinf_record_error(JINF_ERR_INVALID, "sparse_ffn: hidden_dim not a multiple of the block size");
        return;
    }
    if (num_activated <= 0) {
        // No active neuron: the FFN contributes nothing.
        cudaMemsetAsync(output, 0, sizeof(float) * (size_t)hidden_dim, stream);
        return;
    }
    if (sparse_ffn_run(bundles, input, output, bundle_offsets, num_activated, hidden_dim, qtype, gate_up_tmp, SpNorm{},
                       stream) != cudaSuccess)
        jinf_record_error(JINF_ERR_CUDA, "sparse_ffn: launch");
}

namespace jinf {

bool sparse_ffn_fused_ok(int d, int qtype) {
    return qtype == JINF_TYPE_Q4_0 && d > 0 && d % 128 == 0 && d <= SPG_MAX_HIDDEN;
}

cudaError_t sparse_ffn_fused(const uint8_t* bundles, const float* h_in, const float* y_res, float* h_out,
                             const float* gain, float eps, float* out, const int* offs, int n_act, int d,
                             int bundle_size, float* gu_tmp, cudaStream_t s) {
    if (!sparse_ffn_fused_ok(d, JINF_TYPE_Q4_0) || n_act <= 0) return cudaErrorInvalidValue;
    return sparse_ffn_run(bundles, nullptr, out, offs, n_act, d, JINF_TYPE_Q4_0, gu_tmp,
                          SpNorm{h_in, y_res, h_out, gain, eps}, s);
}

}  // namespace jinf
