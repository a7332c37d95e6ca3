// The persistent decode step: one cooperative launch runs a whole token (every layer and
// the LM head) on one CTA of 16 warps per SM, sm_100a.
//
// Why. Batch-1 decode is a chain of ~5 dependent matrix-vector products per layer. As
// separate kernels each one pays a launch, an input prologue and a tail in which HBM idles
// (about 5-8 us per kernel on B200), more than the 1-10 us its weights take to stream.
// Here the weight stream does not stop at phase boundaries, and every dependency costs as
// few global round trips as possible (one round trip under load is ~0.75-1 us):
//   * CTA c owns a contiguous, balanced set of whole 32-row tile pairs of every matrix; its
//     16 warps split the CTA's 2304-byte Q4M units (q4m.cuh: a tile pair x 128 columns)
//     evenly, so a pair shared by several warps is merged through shared memory in warp
//     order (deterministic, no global atomics), and the CTA reports its finished pairs
//     with one counter add;
//   * each warp walks its unit ranges of all matrices in step order with a cp.async ring
//     (STEP_NBUF - 1 units in flight) feeding the tensor-core decode (q4m_device.cuh), so
//     while a CTA waits for the inputs of the next phase its first weights are already on
//     their way; the stream's geometry lives in shared memory;
//   * phases wait on completion counters instead of kernel boundaries (bounded spins:
//     DEV_ERR_TIMEOUT in the device state, never a hang).
// Per layer the phases are the reference's decode order (src/engine.cpp:418-511):
//   QKV GEMV     x = RMSNorm(h) * attn_norm (layer 0: the embedding row); epilogue RoPE,
//                q -> fp32, k/v -> fp16 KV cache at pos
//   attention    one CTA per kv head and up to 512 positions, warps of 32 positions,
//                merged in shared memory (and across CTAs for long contexts)
//   o GEMV       h += W_o attn            (residual fused into the epilogue)
//   gate|up      x = RMSNorm(h) * ffn_norm; epilogue silu(gate) * up
//   down GEMV    h += W_down act
// then the LM head (x = RMSNorm(h) * output_norm; logits + argmax). The last CTA to leave
// turns the argmax into the next input token, advances the position and clears the
// counters for the next launch.
#include "common.cuh"
#include "q4m_device.cuh"
#include "step.h"

#include <math.h>

namespace jinf {

using namespace q4mdev;

namespace {

constexpr int NW = STEP_THREADS / 32;

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Wait until *c >= target. Gives up after `limit` polls, or as soon as another CTA has
// recorded an error; a timeout records DEV_ERR_TIMEOUT.
__device__ bool wait_ge(const unsigned* c, unsigned target, DeviceState* st, unsigned long long limit) {
    for (unsigned long long it = 0;; ++it) {
        if (ld_acquire(c) >= target) return true;
        if (*(volatile int*)&st->error != DEV_OK) return false;
        if (it >= limit) {
            atomicCAS(&st->error, DEV_OK, DEV_ERR_TIMEOUT);
            return false;
        }
        __nanosleep(32);
    }
}

// Stream geometry of one phase, kept in shared memory (groups == 0: no weights).
struct PhaseInfo {
    const uint8_t* w;
    int pairs, groups;
};

// Unit range [c0, c1) of warp `warp` of CTA `cta` (of C) in a pairs x groups matrix
// (32-bit: a matrix has far fewer than 2^31 units).
__device__ __forceinline__ void warp_range(int cta, int C, int warp, int T, int G, int& c0, int& c1) {
    const int t0 = step_cta_tile(cta, C, T), t1 = step_cta_tile(cta + 1, C, T);
    const int n = (t1 - t0) * G;
    c0 = t0 * G + ((warp * n) >> 4);
    c1 = t0 * G + (((warp + 1) * n) >> 4);
}
static_assert(NW == 16, "warp_range divides by the warp count with a shift");

// Where a warp's weight stream continues: the first GEMV phase at or after `from` in which
// it has units, and that range. Out of line: it runs once per phase, and keeping it out of
// the copy loop keeps the loop's live state small.
struct StreamPos {
    const uint8_t* w;
    int ph, c, c1;
};
__device__ __noinline__ StreamPos stream_seek(const PhaseInfo* pinfo, int n, int from, int cta, int C, int warp) {
    StreamPos r;
    for (int i = from; i < n; ++i) {
        const int G = pinfo[i].groups;
        if (!G) continue;
        int c0, c1;
        warp_range(cta, C, warp, pinfo[i].pairs, G, c0, c1);
        if (c0 < c1) {
            r.w = pinfo[i].w;
            r.ph = i;
            r.c = c0;
            r.c1 = c1;
            return r;
        }
    }
    r.w = nullptr;
    r.ph = n;
    r.c = 0;
    r.c1 = 0;
    return r;
}

// Bring the units that CTA `cta` owns in GEMV phase `pi` (one contiguous byte range: whole
// tile pairs, all groups) into L2. Issued while the CTA would otherwise wait on a dependency,
// so that HBM keeps streaming weights through attention, input staging and merges.
__device__ __noinline__ void prefetch_cta_range(const PhaseInfo& pi, int cta, int C) {
    if (!pi.groups) return;
    const int t0 = step_cta_tile(cta, C, pi.pairs), t1 = step_cta_tile(cta + 1, C, pi.pairs);
    if (t0 >= t1) return;
    const uint8_t* b = pi.w + (size_t)t0 * pi.groups * Q4M_UNIT;
    const uint32_t bytes = (uint32_t)(t1 - t0) * (uint32_t)pi.groups * (uint32_t)Q4M_UNIT;  // multiple of 16
    for (uint32_t off = 0; off < bytes; off += (1u << 20))
        prefetch_l2(b + off, bytes - off < (1u << 20) ? bytes - off : (1u << 20));
}

// The weight stream of one warp between calls: ring slot of the next unit to consume and
// the copy position.
struct WarpStream {
    StreamPos sp;
    int slot;
};

struct PieceSum {
    float acc[4];
};

// Consume groups [gb, ge) of one tile pair from the ring (tensor-core decode, q4m_device.cuh),
// refilling it as it goes. Out of line so that the hot loop gets a register allocation of
// its own, independent of the rest of the step kernel.
__device__ __noinline__ PieceSum stream_piece(WarpStream& ws, uint32_t ring, const PhaseInfo* pinfo, int n_phases,
                                              int C, const XRecS xr, int gb, int ge) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    StreamPos sp = ws.sp;
    int slot = ws.slot;
    PieceSum r{{0.f, 0.f, 0.f, 0.f}};
    for (int g = gb; g < ge; ++g) {
        const int is = slot == 0 ? STEP_NBUF - 1 : slot - 1;
        if (sp.c < sp.c1) {
            copy_unit_async(ring + is * Q4M_UNIT, sp.w + (size_t)sp.c * Q4M_UNIT, lane);
            if (++sp.c == sp.c1) sp = stream_seek(pinfo, n_phases, sp.ph + 1, blockIdx.x, C, warp);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");  // possibly empty: uniform group counts
        asm volatile("cp.async.wait_group %0;" ::"n"(STEP_NBUF - 1) : "memory");
        unit_mma(ring + slot * Q4M_UNIT, xr, g, lane, r.acc);
        slot = slot + 1 == STEP_NBUF ? 0 : slot + 1;
    }
    ws.sp = sp;
    ws.slot = slot;
    return r;
}

__device__ __forceinline__ void unpack8(const uint4 v, float (&f)[8]) {
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 t = __half22float2(h[i]);
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}

template <int DPL>
__device__ __forceinline__ void load_vrow(const __half* vrow, int lane, bool ok, float (&v)[DPL]) {
    if constexpr (DPL == 4) {
        const uint2 raw = ok ? __ldcg(reinterpret_cast<const uint2*>(vrow) + lane) : make_uint2(0u, 0u);
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
        v[0] = a.x;
        v[1] = a.y;
        v[2] = b.x;
        v[3] = b.y;
    } else {
        const unsigned raw = ok ? __ldcg(reinterpret_cast<const unsigned*>(vrow) + lane) : 0u;
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw));
        v[0] = a.x;
        v[1] = a.y;
    }
}

// One warp's share of the decode attention (math of reference cuda/attention_kernel.cu:
// 45-98: scores q.k / sqrt(hd), GQA head map h -> h / (H/Hkv), max-subtracted softmax,
// P.V): positions [p0, p1) in blocks of 32, for all GQ query heads of one kv head, with an
// online softmax across the blocks. Lanes own positions for q.k and head dims for p.v; the
// (m, l, acc[hd]) of each query head goes to `part` ([GQ][HD + 2]). qs holds the
// pre-scaled q of the GQ heads.
template <int HD, int GQ>
__device__ __noinline__ void attn_warp(const float* qs, const __half* kb, const __half* vb, int p0, int p1, int lane,
                                       float* part) {
    constexpr int DPL = HD / 32;  // head dims per lane
    float m[GQ], l[GQ], acc[GQ][DPL];
#pragma unroll
    for (int g = 0; g < GQ; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int k = 0; k < DPL; ++k) acc[g][k] = 0.f;
    }
    for (int b0 = p0; b0 < p1; b0 += 32) {
        const int pp = b0 + lane;
        const bool valid = pp < p1;
        const int nj = p1 - b0 < 32 ? p1 - b0 : 32;
        float sc[GQ];
#pragma unroll
        for (int g = 0; g < GQ; ++g) sc[g] = 0.f;
        if (valid) {
            // this lane's K row, eight 16-byte loads in flight at a time
            const uint4* kr = reinterpret_cast<const uint4*>(kb + (size_t)pp * HD);
#pragma unroll
            for (int hb = 0; hb < HD / 64; ++hb) {
                uint4 kv[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) kv[u] = __ldcg(kr + hb * 8 + u);
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int c8 = hb * 8 + u;
                    float kf[8];
                    unpack8(kv[u], kf);
#pragma unroll
                    for (int g = 0; g < GQ; ++g) {
                        const float4 qa = reinterpret_cast<const float4*>(qs)[(g * HD) / 4 + 2 * c8];
                        const float4 qb = reinterpret_cast<const float4*>(qs)[(g * HD) / 4 + 2 * c8 + 1];
                        float a = sc[g];
                        a = fmaf(qa.x, kf[0], a);
                        a = fmaf(qa.y, kf[1], a);
                        a = fmaf(qa.z, kf[2], a);
                        a = fmaf(qa.w, kf[3], a);
                        a = fmaf(qb.x, kf[4], a);
                        a = fmaf(qb.y, kf[5], a);
                        a = fmaf(qb.z, kf[6], a);
                        a = fmaf(qb.w, kf[7], a);
                        sc[g] = a;
                    }
                }
            }
        }
        // the first 16 V rows are requested before the softmax (they do not depend on it)
        float v0[16][DPL];
#pragma unroll
        for (int u = 0; u < 16; ++u) load_vrow<DPL>(vb + (size_t)(b0 + u) * HD, lane, u < nj, v0[u]);
        float pr[GQ];
#pragma unroll
        for (int g = 0; g < GQ; ++g) {
            const float sv = valid ? sc[g] : -INFINITY;
            const float mn = fmaxf(m[g], warp_max(sv));
            const float corr = m[g] == -INFINITY ? 0.f : expf(m[g] - mn);
            pr[g] = valid ? expf(sv - mn) : 0.f;
            l[g] = l[g] * corr + warp_sum(pr[g]);
#pragma unroll
            for (int k = 0; k < DPL; ++k) acc[g][k] *= corr;
            m[g] = mn;
        }
#pragma unroll
        for (int u = 0; u < 16; ++u)
#pragma unroll
            for (int g = 0; g < GQ; ++g) {
                const float pj = __shfl_sync(JINF_FULL_MASK, pr[g], u);
#pragma unroll
                for (int k = 0; k < DPL; ++k) acc[g][k] = fmaf(pj, v0[u][k], acc[g][k]);
            }
        if (nj > 16) {
#pragma unroll
            for (int u = 0; u < 16; ++u) load_vrow<DPL>(vb + (size_t)(b0 + 16 + u) * HD, lane, 16 + u < nj, v0[u]);
#pragma unroll
            for (int u = 0; u < 16; ++u)
#pragma unroll
                for (int g = 0; g < GQ; ++g) {
                    const float pj = __shfl_sync(JINF_FULL_MASK, pr[g], 16 + u);
#pragma unroll
                    for (int k = 0; k < DPL; ++k) acc[g][k] = fmaf(pj, v0[u][k], acc[g][k]);
                }
        }
    }
#pragma unroll
    for (int g = 0; g < GQ; ++g) {
#pragma unroll
        for (int k = 0; k < DPL; ++k) part[g * (HD + 2) + lane * DPL + k] = acc[g][k];
        if (lane == 0) {
            part[g * (HD + 2) + HD] = m[g];
            part[g * (HD + 2) + HD + 1] = l[g];
        }
    }
}

template <int HD>
__device__ void attn_warp_dispatch(int gq, const float* qs, const __half* kb, const __half* vb, int p0, int p1,
                                   int lane, float* part) {
    switch (gq) {
        case 1: attn_warp<HD, 1>(qs, kb, vb, p0, p1, lane, part); break;
        case 2: attn_warp<HD, 2>(qs, kb, vb, p0, p1, lane, part); break;
        case 4: attn_warp<HD, 4>(qs, kb, vb, p0, p1, lane, part); break;
        default: attn_warp<HD, 8>(qs, kb, vb, p0, p1, lane, part); break;
    }
}

// Merge `n` partials (stride `stride` floats, [g][HD + 2] each; m = -inf marks an empty
// one) of query head g, dim dd: returns sum_i e^(m_i - M) acc_i and sets L (sum of weighted
// l_i) and M. Fixed order: deterministic.
__device__ __forceinline__ float merge_parts(const float* base, int n, size_t stride, int g, int dd, int hd,
                                             bool coherent, float& M, float& L) {
    auto ld = [&](const float* p) { return coherent ? __ldcg(p) : *p; };
    M = -INFINITY;
    for (int i = 0; i < n; ++i) M = fmaxf(M, ld(base + i * stride + g * (hd + 2) + hd));
    float a = 0.f;
    L = 0.f;
    for (int i = 0; i < n; ++i) {
        const float* r = base + i * stride + g * (hd + 2);
        const float mi = ld(r + hd);
        if (mi == -INFINITY) continue;
        const float f = expf(mi - M);
        L = fmaf(ld(r + hd + 1), f, L);
        a = fmaf(ld(r + dd), f, a);
    }
    return a;
}

}  // namespace

__global__ void __launch_bounds__(STEP_THREADS, 1) k_step(const StepParams P) {
    extern __shared__ __align__(16) uint8_t smem[];
    // shared memory: [xstage | misc 256 B | flags, keys, piece table 512 B | partial rows 4 KB |
    //                 phase descriptor 2 x 256 B | phase infos | rings]
    uint8_t* xbase = smem;
    float* misc = reinterpret_cast<float*>(smem + P.xstage_bytes);        // 64 floats of reductions
    int* flags = reinterpret_cast<int*>(smem + P.xstage_bytes + 256);     // [0..1] go, [2] attention last
    u64* wkeys = reinterpret_cast<u64*>(smem + P.xstage_bytes + 256 + 64);  // [NW] argmax keys
    int* ftile = reinterpret_cast<int*>(smem + P.xstage_bytes + 256 + 192);  // [NW] tile of a warp's first piece
    int* fmid = ftile + NW;                                                  // [NW] first piece starts mid-tile
    float* part_s = reinterpret_cast<float*>(smem + P.xstage_bytes + 768);   // [NW][2][32] partial rows
    StepPhase* dsm = reinterpret_cast<StepPhase*>(smem + P.xstage_bytes + 768 + 4096);  // [2] descriptors
    PhaseInfo* pinfo = reinterpret_cast<PhaseInfo*>(smem + P.xstage_bytes + 768 + 4096 + 512);
    const uint32_t ring_base = smem_u32(pinfo + ((P.n_phases + 1) & ~1));
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t ring = ring_base + (uint32_t)(warp * STEP_NBUF * Q4M_UNIT);
    const int C = gridDim.x;
    DeviceState* st = P.st;
    const int pos = *(volatile int*)&st->pos;

    // stream geometry of every phase -> shared memory
    for (int i = tid; i < P.n_phases; i += STEP_THREADS) {
        PhaseInfo pi;
        pi.w = P.phases[i].w;
        pi.pairs = P.phases[i].pairs;
        pi.groups = P.phases[i].kind == PH_GEMV ? P.phases[i].groups : 0;
        pinfo[i] = pi;
    }
    __syncthreads();

    // ---------------- weight stream: this warp's unit ranges of all GEMV phases, copied in
    // consumption order into the ring (STEP_NBUF - 1 units ahead of the arithmetic)
    WarpStream ws;
    ws.sp = stream_seek(pinfo, P.n_phases, 0, blockIdx.x, C, warp);
    ws.slot = 0;
    for (int i = 0; i < STEP_NBUF - 1; ++i) {
        if (ws.sp.c < ws.sp.c1) {
            copy_unit_async(ring + i * Q4M_UNIT, ws.sp.w + (size_t)ws.sp.c * Q4M_UNIT, lane);
            if (++ws.sp.c == ws.sp.c1) ws.sp = stream_seek(pinfo, P.n_phases, ws.sp.ph + 1, blockIdx.x, C, warp);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");  // possibly empty: uniform group counts
    }

    const int c4 = lane & 3;
    float lmax = -INFINITY;
    int lidx = 0;
    constexpr int DWORDS = (int)(sizeof(StepPhase) / 4);
    static_assert(sizeof(StepPhase) <= 256 && sizeof(StepPhase) % 4 == 0, "descriptor slot");
    for (int ph = 0; ph < P.n_phases; ++ph) {
        StepPhase& d = dsm[ph & 1];
        if (tid == 0) {
            const StepPhase& g = P.phases[ph];
            flags[ph & 1] = g.dep < 0 ? 1 : (wait_ge(P.done + g.dep, g.dep_target, st, P.spin_limit) ? 1 : 0);
        } else if (tid >= 32 && tid < 32 + DWORDS) {  // descriptor -> shared memory while warp 0 polls
            reinterpret_cast<uint32_t*>(&d)[tid - 32] = reinterpret_cast<const uint32_t*>(P.phases + ph)[tid - 32];
        } else if (tid == 32 * 9) {  // L2 prefetch of later weights while warp 0 polls
            for (int k = 0; k < 2; ++k) {
                const int j = P.phases[ph].pf[k];
                if (j > ph && j < P.n_phases) prefetch_cta_range(pinfo[j], blockIdx.x, C);
            }
        }
        __syncthreads();  // also: every warp is done with the previous phase's shared data
        if (!flags[ph & 1]) break;

        if (d.kind == PH_ATTN) {
            // ---------------- attention: CTA (kvh, split) covers up to ATTN_POS_PER_CTA positions
            const int hd = P.head_dim, gq = P.n_heads / P.n_kv_heads;
            const int n_pos = pos + 1;
            int cpk = (n_pos + ATTN_POS_PER_CTA - 1) / ATTN_POS_PER_CTA;
            cpk = cpk > ATTN_MAX_SPLIT ? ATTN_MAX_SPLIT : cpk;
            const int per = (n_pos + cpk - 1) / cpk;
            if ((int)blockIdx.x >= P.n_kv_heads * cpk) continue;
            const int kvh = blockIdx.x / cpk, sp = blockIdx.x % cpk;
            const int p0 = sp * per, p1 = min(n_pos, p0 + per);
            float* qs = reinterpret_cast<float*>(xbase);                   // [gq][hd], pre-scaled
            float* wp = qs + gq * hd;                                       // [NW][gq][hd + 2]
            const float scale = rsqrtf((float)hd);
            const float4* qsrc = reinterpret_cast<const float4*>(d.q + (size_t)kvh * gq * hd);
            for (int i = tid; i < gq * hd / 4; i += STEP_THREADS) {
                float4 v = __ldcg(qsrc + i);
                v.x *= scale;
                v.y *= scale;
                v.z *= scale;
                v.w *= scale;
                reinterpret_cast<float4*>(qs)[i] = v;
            }
            __syncthreads();
            float* mypart = wp + (size_t)warp * gq * (hd + 2);
            const int wp0 = p0 + warp * ATTN_POS_PER_WARP, wp1 = min(p1, wp0 + ATTN_POS_PER_WARP);
            const __half* kb = d.kcache + (size_t)kvh * P.max_ctx * hd;
            const __half* vb = d.vcache + (size_t)kvh * P.max_ctx * hd;
            if (wp0 < wp1) {
                if (hd == 64) attn_warp_dispatch<64>(gq, qs, kb, vb, wp0, wp1, lane, mypart);
                else attn_warp_dispatch<128>(gq, qs, kb, vb, wp0, wp1, lane, mypart);
            } else if (lane < gq) {
                mypart[lane * (hd + 2) + hd] = -INFINITY;  // empty
            }
            __syncthreads();
            // merge the warps (fixed order)
            float* gpart = P.attn_part + ((size_t)kvh * ATTN_MAX_SPLIT + sp) * ATTN_MAX_GROUP * (hd + 2);
            for (int i = tid; i < gq * hd; i += STEP_THREADS) {
                const int g = i / hd, dd = i % hd;
                float M, L;
                const float a = merge_parts(wp, NW, (size_t)gq * (hd + 2), g, dd, hd, false, M, L);
                if (cpk == 1) {
                    d.out[(size_t)(kvh * gq + g) * hd + dd] = a / L;
                } else {
                    gpart[g * (hd + 2) + dd] = a;
                    if (dd == 0) {
                        gpart[g * (hd + 2) + hd] = M;
                        gpart[g * (hd + 2) + hd + 1] = L;
                    }
                }
            }
            bool wrote = cpk == 1;
            if (cpk > 1) {
                // last CTA of this kv head merges the CTAs' partials (split order)
                __syncthreads();
                if (tid == 0) {
                    __threadfence();
                    const unsigned old = atomicAdd(&st->attn_count[kvh], 1u);
                    flags[2] = old == (unsigned)(cpk - 1);
                    if (flags[2]) {
                        __threadfence();
                        st->attn_count[kvh] = 0u;
                    }
                }
                __syncthreads();
                wrote = flags[2] != 0;
                if (wrote) {
                    const float* base = P.attn_part + (size_t)kvh * ATTN_MAX_SPLIT * ATTN_MAX_GROUP * (hd + 2);
                    for (int i = tid; i < gq * hd; i += STEP_THREADS) {
                        const int g = i / hd, dd = i % hd;
                        float M, L;
                        const float a =
                            merge_parts(base, cpk, (size_t)ATTN_MAX_GROUP * (hd + 2), g, dd, hd, true, M, L);
                        d.out[(size_t)(kvh * gq + g) * hd + dd] = a / L;
                    }
                }
            }
            if (wrote) {
                __syncthreads();
                if (tid == 0) {
                    __threadfence();
                    atomicAdd(P.done + ph, 1u);
                }
            }
            continue;
        }

        // ---------------- GEMV phase: this CTA's tile pairs [t0, t1)
        if (d.epi == EPI_QKV && tid == 0 && pos > 0 && (int)blockIdx.x < 2 * P.n_kv_heads) {
            // the attention after this phase reads this layer's K and V rows 0..pos-1 (one
            // region per CTA): bring them into L2 now, while the QKV weights stream
            const int kvh = blockIdx.x >> 1;
            const __half* base = ((blockIdx.x & 1) ? d.vcache : d.kcache) + (size_t)kvh * P.max_ctx * P.head_dim;
            const uint32_t bytes = (uint32_t)pos * (uint32_t)P.head_dim * 2u;
            for (uint32_t off = 0; off < bytes; off += (1u << 20))
                prefetch_l2(reinterpret_cast<const uint8_t*>(base) + off, bytes - off < (1u << 20) ? bytes - off : (1u << 20));
        }
        const int G = d.groups;
        const int t0 = step_cta_tile(blockIdx.x, C, d.pairs), t1 = step_cta_tile(blockIdx.x + 1, C, d.pairs);
        if (t0 >= t1) continue;
        const float* hsrc = d.xm == X_EMBED_NORM ? d.hsrc + (size_t)(*(volatile int*)&st->token) * d.cols : d.hsrc;
        // the CTA that owns pair 0 stores the embedding row as the residual stream
        const float fac = stage_x<STEP_THREADS>(d.xm, d.x, hsrc, nullptr, d.hout, t0 == 0, d.norm_w, P.eps, d.cols,
                                                xbase, misc, true);
        const XRecS xr{smem_u32(xbase), smem_u32(xbase + (size_t)G * 256)};
        // epilogue arguments are read from the shared descriptor when a tile finishes
        auto epilogue = [&](int row, float v0, float v1) {
            EpiArgs ea;
            ea.epi = d.epi;
            ea.rows = d.rows;
            ea.y = d.y;
            ea.kcache = d.kcache;
            ea.vcache = d.vcache;
            ea.nq = P.nq;
            ea.nk = P.nk;
            ea.head_dim = P.head_dim;
            ea.max_ctx = P.max_ctx;
            ea.pos = pos;
            ea.rope_base = P.rope_base;
            ea.coherent = true;
            epilogue_pair(ea, row, v0 * fac, v1 * fac, lmax, lidx);
        };
        int c, c1;
        warp_range(blockIdx.x, C, warp, d.pairs, G, c, c1);
        if (lane == 0) {
            ftile[warp] = -1;
            fmid[warp] = 0;
        }
        bool first_piece = true;
        int own_pair = -1, own_slot = 0;  // the split pair this warp finishes (its piece starts the pair)
        int pair = c / G, gb = c - pair * G;  // walked incrementally: no division per piece
        for (; c < c1; ++pair, gb = 0) {
            const int ge = c1 - c < G - gb ? gb + (c1 - c) : G;
            PieceSum ps = stream_piece(ws, ring, pinfo, P.n_phases, C, xr, gb, ge);
            c += ge - gb;
            if (first_piece && lane == 0) {
                ftile[warp] = pair;
                fmid[warp] = gb > 0;
            }
            unit_reduce(ps.acc);
            if (gb == 0 && ge == G) {
                const int q = lane & 15;
                const float v0 = unit_row(ps.acc, 2 * q), v1 = unit_row(ps.acc, 2 * q + 1);
                if (lane < 16) epilogue(pair * Q4M_PAIR_ROWS + 2 * q, v0, v1);
            } else {
                // a piece of a pair shared with the neighbouring warps: partial rows to shared memory
                const int sl = first_piece ? 0 : 1;
                if (c4 == 0) {
#pragma unroll
                    for (int i = 0; i < 4; ++i) part_s[(warp * 2 + sl) * 32 + unit_row_of(i, lane)] = ps.acc[i];
                }
                if (gb == 0) {
                    own_pair = pair;
                    own_slot = sl;
                }
            }
            first_piece = false;
        }
        __syncthreads();
        if (own_pair >= 0 && lane < 16) {
            // add the pieces of the following warps in warp order, then the epilogue
            float v0 = part_s[(warp * 2 + own_slot) * 32 + 2 * lane];
            float v1 = part_s[(warp * 2 + own_slot) * 32 + 2 * lane + 1];
            for (int w2 = warp + 1; w2 < NW; ++w2) {
                const int ft = ftile[w2];
                if (ft < 0) continue;                       // a warp with no units in this phase
                if (ft != own_pair || !fmid[w2]) break;     // the next pair starts
                v0 += part_s[(w2 * 2) * 32 + 2 * lane];
                v1 += part_s[(w2 * 2) * 32 + 2 * lane + 1];
            }
            epilogue(own_pair * Q4M_PAIR_ROWS + 2 * lane, v0, v1);
        }
        __syncthreads();  // every epilogue store of the CTA precedes the report
        if (tid == 0) {
            __threadfence();
            atomicAdd(P.done + ph, (unsigned)(t1 - t0));
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");

    // ---------------- leave: LM head argmax, then the last CTA finishes the step
    if (P.with_argmax) {
        u64 key = lmax == -INFINITY ? 0ull : argmax_key(lmax, lidx);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const u64 other = __shfl_xor_sync(JINF_FULL_MASK, key, o);
            key = other > key ? other : key;
        }
        if (lane == 0) wkeys[warp] = key;
    }
    __syncthreads();
    if (tid == 0) {
        if (P.with_argmax) {
            u64 best = 0ull;
            for (int w = 0; w < NW; ++w) best = wkeys[w] > best ? wkeys[w] : best;
            if (best) atomicMax(&st->best, best);
        }
        __threadfence();
        const unsigned old = atomicAdd(P.done + P.n_phases, 1u);
        if (old == gridDim.x - 1) {
            __threadfence();
            if (P.with_argmax) {
                const u64 b = atomicAdd(&st->best, 0ull);
                st->argmax_token = b ? (int)(0xFFFFFFFFu - (uint32_t)(b & 0xFFFFFFFFull)) : 0;
                st->token = st->argmax_token;
                st->best = 0ull;
            }
            st->pos = pos + 1;
            for (int i = 0; i <= P.n_phases; ++i) P.done[i] = 0u;
        }
    }
}

// ---------------------------------------------------------------- host side

unsigned int step_xstage_bytes(int max_cols, int group, int head_dim) {
    const size_t G = (size_t)(max_cols + Q4M_KG - 1) / Q4M_KG;
    const size_t gemv = xrec_bytes((int)G);
    const size_t attn = (size_t)group * head_dim * sizeof(float) + (size_t)NW * group * (head_dim + 2) * sizeof(float);
    const size_t b = gemv > attn ? gemv : attn;
    return (unsigned int)((b + 15) & ~(size_t)15);
}

size_t step_smem_bytes(unsigned int xstage_bytes, int n_phases) {
    const size_t infos = sizeof(PhaseInfo) * (size_t)((n_phases + 1) & ~1);
    return (size_t)xstage_bytes + 768 + 4096 + 512 + infos + (size_t)NW * STEP_NBUF * Q4M_UNIT;
}

static cudaError_t step_configure(size_t smem) {
    static size_t configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (smem <= configured[dev]) return cudaSuccess;
    const cudaError_t e = cudaFuncSetAttribute(k_step, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess) configured[dev] = smem;
    return e;
}

int step_occupancy(size_t smem) {
    if (step_configure(smem) != cudaSuccess) return 0;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_step, STEP_THREADS, smem) != cudaSuccess) return 0;
    return n;
}

cudaError_t step_launch(const StepParams& p, int grid, cudaStream_t s) {
    const size_t smem = step_smem_bytes(p.xstage_bytes, p.n_phases);
    cudaError_t e = step_configure(smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(STEP_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: the phase waits need it
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k_step, p);
}

}  // namespace jinf
