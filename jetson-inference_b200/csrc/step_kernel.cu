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
//     (NBUF - 1 units in flight) feeding the tensor-core decode (q4m_device.cuh), so
//     while a CTA waits for the inputs of the next phase its first weights are already on
//     their way; the stream's geometry lives in shared memory;
//   * phases wait on completion counters instead of kernel boundaries (bounded spins:
//     DEV_ERR_TIMEOUT in the device state, never a hang).
// Per layer the phases are the reference's decode order (src/engine.cpp:418-511):
//   QKV GEMV     x = RMSNorm(h) * attn_norm (layer 0: the embedding row); epilogue RoPE,
//                q -> fp32, k/v -> fp16 KV cache at pos
//   attention    each kv head's positions split over several CTAs (lanes on head dims,
//                cache rows read from L2 into registers), the splits merged by the CTAs
//                that own the output blocks, which write the o phase's input records
//   o GEMV       h += W_o attn            (residual fused into the epilogue)
//   gate|up      x = RMSNorm(h) * ffn_norm; epilogue silu(gate) * up -> down's input records
//   down GEMV    h += W_down act
// then the LM head (x = RMSNorm(h) * output_norm; logits + argmax). The last CTA to leave
// turns the argmax into the next input token, advances the position and clears the
// counters for the next launch.
// Tensor parallel (k_step<.., TP = true>, one rank per GPU): o and down write this rank's
// partial rows into every rank's exchange area over NVLink as flagged 8-byte words, and
// the next RMSNorm input adds all ranks' rows in rank order (stage_x_tp); the last CTA
// exchanges the argmax keys.
#include "common.cuh"
#include "mma_f16.cuh"
#include "multi.h"
#include "q4m_device.cuh"
#include "step.h"

#include <type_traits>

#include <algorithm>

#include <math.h>

namespace jinf {

using namespace q4mdev;

namespace {

constexpr int NW = STEP_THREADS / 32;

// Development timing (off unless built with -DJINF_STEP_TRACE): thread 0 of every CTA stamps
// %globaltimer at fixed points of every phase into g_step_trace[phase][cta][point]; the last
// launch's stamps are read with jinf_step_trace_read.
#ifdef JINF_STEP_TRACE
constexpr int TRACE_PTS = 6, TRACE_MAX_PH = 512, TRACE_MAX_CTA = 160;
__device__ unsigned long long g_step_trace[TRACE_MAX_PH * TRACE_MAX_CTA * TRACE_PTS];
__device__ __forceinline__ void trace_at(int ph, int pt) {
    if (threadIdx.x == 0 && ph < TRACE_MAX_PH && blockIdx.x < TRACE_MAX_CTA) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        g_step_trace[((size_t)ph * TRACE_MAX_CTA + blockIdx.x) * TRACE_PTS + pt] = t;
    }
}
#define JINF_TRACE(ph, pt) trace_at(ph, pt)
#else
#define JINF_TRACE(ph, pt) ((void)0)
#endif

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Wait until *c >= target. Gives up after `limit` polls, or as soon as another CTA has
// recorded an error; a timeout records DEV_ERR_TIMEOUT. The counter is polled back to back
// (one L2 round trip per poll, so a phase hand-off is seen within about one round trip);
// every 64th poll also reads the error word, checks the limit and sleeps briefly.
__device__ bool wait_ge(const unsigned* c, unsigned target, DeviceState* st, unsigned long long limit) {
    for (unsigned long long it = 0;; ++it) {
        if (ld_acquire(c) >= target) return true;
        if ((it & 63) == 63) {
            if (*(volatile int*)&st->error != DEV_OK) return false;
            if (it >= limit) {
                atomicCAS(&st->error, DEV_OK, DEV_ERR_TIMEOUT);
                return false;
            }
            __nanosleep(32);
        }
    }
}

// Tensor-parallel exchange (other ranks' kernels write this rank's exchange area over
// NVLink): system-scope acquire polls of a monotonic 64-bit counter, bounded like wait_ge.
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ bool wait_ge_sys(const unsigned long long* c, unsigned long long target, DeviceState* st,
                            unsigned long long limit) {
    for (unsigned long long it = 0;; ++it) {
        if (ld_acquire_sys(c) >= target) return true;
        if (*(volatile int*)&st->error != DEV_OK) return false;
        if (it >= limit) {
            atomicCAS(&st->error, DEV_OK, DEV_ERR_TIMEOUT);
            return false;
        }
        __nanosleep(32);
    }
}
// This step's slot of rank `src` at exchange point `point` in rank `rank`'s area: one 8-byte
// word per row, {value bits, flag} with flag = this step's epoch + 1 in the high half. An
// aligned 8-byte word is written and read whole, so a word whose flag matches carries this
// step's value: the consumer's load is also its wait, with no fence or counter on the way.
__device__ __forceinline__ unsigned long long* xchg_data(const StepParams& P, int rank, int point, unsigned par,
                                                         int src) {
    return reinterpret_cast<unsigned long long*>(P.xpeer[rank] + P.x_data + ((size_t)point * 2 + par) * P.x_point +
                                                 (size_t)src * P.x_slot);
}
__device__ __forceinline__ unsigned long long ll_word(float v, uint32_t flag) {
    return ((unsigned long long)flag << 32) | __float_as_uint(v);
}
__device__ __forceinline__ void st_ll2(unsigned long long* p, unsigned long long a, unsigned long long b) {
    asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ ulonglong2 ld_ll2(const unsigned long long* p) {
    ulonglong2 v;
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ bool ll_ok(const ulonglong2& w, uint32_t flag) {
    return (uint32_t)(w.x >> 32) == flag && (uint32_t)(w.y >> 32) == flag;
}

// ---------------------------------------------------------------- bulk copies
//
// Inputs staged once per phase (records, attention cache rows) come in by TMA bulk copy
// (cp.async.bulk, global -> shared) completing on an mbarrier, so waiting for them never
// waits on the weight rings' per-thread cp.async groups (which by then hold the next phase's
// first units).
__device__ __forceinline__ void mbar_init(uint32_t mbar) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(mbar) : "memory");
}
__device__ __forceinline__ void bulk_expect(uint32_t mbar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(mbar), "r"(bytes) : "memory");
}
// 16-byte aligned addresses, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t mbar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(mbar)
                 : "memory");
}
// Orders this thread's (and, after a barrier, its CTA's) generic-proxy accesses before its
// following bulk copies: the copied data was written through the generic proxy, and the
// shared destination was last read through it.
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async;" ::: "memory"); }
// Wait for phase `parity` of the mbarrier; gives up after `limit` polls (DEV_ERR_TIMEOUT).
__device__ __noinline__ bool mbar_wait(uint32_t mbar, uint32_t parity, DeviceState* st, unsigned long long limit) {
    for (unsigned long long it = 0;; ++it) {
        uint32_t ok;
        asm volatile(
            "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
            : "=r"(ok)
            : "r"(mbar), "r"(parity)
            : "memory");
        if (ok) return true;
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
    int pairs, groups, gran;
    int fmts;  // StepPhase::fmts
};

// Byte offset of tile pair t in a phase's matrix (pairs below fmts >> 8 in format fmts & 15,
// the rest in (fmts >> 4) & 15).
__device__ __forceinline__ size_t pair_offset(int fmts, int groups, int t) {
    const int ps = fmts >> 8;
    const size_t ua = (size_t)groups * q4m_unit_bytes(fmts & 15);
    return t <= ps ? (size_t)t * ua : (size_t)ps * ua + (size_t)(t - ps) * groups * q4m_unit_bytes((fmts >> 4) & 15);
}

// Tile pairs [t0, t1) of CTA `cta` (of C): balanced runs of `gran` pairs (T % gran == 0).
__device__ __forceinline__ void cta_range(int cta, int C, int T, int gran, int& t0, int& t1) {
    if (gran == 2) {
        t0 = 2 * step_cta_tile(cta, C, T >> 1);
        t1 = 2 * step_cta_tile(cta + 1, C, T >> 1);
    } else {
        t0 = step_cta_tile(cta, C, T);
        t1 = step_cta_tile(cta + 1, C, T);
    }
}

// Unit range [c0, c1) of warp `warp` of CTA `cta` (of C) in a pairs x groups matrix
// (32-bit: a matrix has far fewer than 2^31 units).
__device__ __forceinline__ void warp_range(int cta, int C, int warp, int T, int gran, int G, int& c0, int& c1) {
    int t0, t1;
    cta_range(cta, C, T, gran, t0, t1);
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
// The mixed-format instance's position (Q4M_MIX): units below cs are format fa from w, the
// rest fb from w2. Uniform instances keep the smaller StreamPos.
struct StreamPosMix : StreamPos {
    const uint8_t* w2;
    int cs, fa, fb;
};
template <bool M>
using StreamPosOf = typename std::conditional<M, StreamPosMix, StreamPos>::type;

template <bool M>
__device__ __noinline__ StreamPosOf<M> stream_seek(const PhaseInfo* pinfo, int n, int from, int cta, int C,
                                                   int warp) {
    StreamPosOf<M> r;
    for (int i = from; i < n; ++i) {
        const int G = pinfo[i].groups;
        if (!G) continue;
        int c0, c1;
        warp_range(cta, C, warp, pinfo[i].pairs, pinfo[i].gran, G, c0, c1);
        if (c0 < c1) {
            r.w = pinfo[i].w;
            r.ph = i;
            r.c = c0;
            r.c1 = c1;
            if constexpr (M) {
                const int fm = pinfo[i].fmts;
                r.cs = (fm >> 8) * G;
                r.fa = fm & 15;
                r.fb = (fm >> 4) & 15;
                r.w2 = r.w + (size_t)r.cs * q4m_unit_bytes(r.fa);
            }
            return r;
        }
    }
    r.w = nullptr;
    r.ph = n;
    r.c = 0;
    r.c1 = 0;
    if constexpr (M) {
        r.w2 = nullptr;
        r.cs = r.fa = r.fb = 0;
    }
    return r;
}

// Bring the units that CTA `cta` owns in GEMV phase `pi` (one contiguous byte range: whole
// tile pairs, all groups) into L2. Issued while the CTA would otherwise wait on a dependency,
// so that HBM keeps streaming weights through attention, input staging and merges.
__device__ __noinline__ void prefetch_cta_range(const PhaseInfo& pi, int cta, int C, int ub, bool mixed) {
    if (!pi.groups) return;
    int t0, t1;
    cta_range(cta, C, pi.pairs, pi.gran, t0, t1);
    if (t0 >= t1) return;
    const size_t o0 = mixed ? pair_offset(pi.fmts, pi.groups, t0) : (size_t)t0 * pi.groups * ub;
    const size_t o1 = mixed ? pair_offset(pi.fmts, pi.groups, t1) : (size_t)t1 * pi.groups * ub;
    const uint8_t* b = pi.w + o0;
    const uint32_t bytes = (uint32_t)(o1 - o0);  // multiple of 16
    for (uint32_t off = 0; off < bytes; off += (1u << 20))
        prefetch_l2(b + off, bytes - off < (1u << 20) ? bytes - off : (1u << 20));
}

// The weight stream of one warp between calls: ring slot of the next unit to consume and
// the copy position.
template <bool M>
struct WarpStream {
    StreamPosOf<M> sp;
    int slot;
};

struct PieceSum {
    float acc[4];
};

// Copy the unit at the stream position into ring slot `slot` (slots of SB bytes). In the
// mixed instance the unit's format and address follow the phase's split (StreamPos).
template <int FMT>
__device__ __forceinline__ void copy_stream_unit(uint32_t slot, const StreamPosOf<FMT == Q4M_MIX>& sp, int lane) {
    if constexpr (FMT == Q4M_MIX) {
        if (sp.c < sp.cs) {
            const uint8_t* u = sp.w + (size_t)sp.c * q4m_unit_bytes(sp.fa);
            if (sp.fa == Q4M_Q6_K) copy_unit_6_async(slot, u, lane);
            else if (sp.fa == Q4M_Q4_K) copy_unit_k_async(slot, u, lane);
            else copy_unit_async(slot, u, lane);
        } else {
            const uint8_t* u = sp.w2 + (size_t)(sp.c - sp.cs) * q4m_unit_bytes(sp.fb);
            if (sp.fb == Q4M_Q6_K) copy_unit_6_async(slot, u, lane);
            else if (sp.fb == Q4M_Q4_K) copy_unit_k_async(slot, u, lane);
            else copy_unit_async(slot, u, lane);
        }
    } else {
        copy_unit_fmt<FMT>(slot, sp.w + (size_t)sp.c * q4m_unit_bytes(FMT), lane);
    }
}

// Consume groups [gb, ge) of one tile pair from the ring (tensor-core decode, q4m_device.cuh),
// refilling it as it goes. Out of line so that the hot loop gets a register allocation of
// its own, independent of the rest of the step kernel. CF is the pair's weight format (FMT
// itself unless FMT is Q4M_MIX, whose ring may hold units of several formats: there the warp
// synchronises after each unit, so that no lane's copy into a slot overtakes another lane's
// reads of the unit it held).
template <int FMT, int NBUF, int CF>
__device__ __noinline__ PieceSum stream_piece(WarpStream<FMT == Q4M_MIX>& ws, uint32_t ring, const PhaseInfo* pinfo,
                                              int n_phases,
                                              int C, const XRecS xr, int gb, int ge) {
    constexpr int SB = q4m_unit_bytes(FMT);  // ring slot bytes
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    StreamPosOf<FMT == Q4M_MIX> sp = ws.sp;
    int slot = ws.slot;
    PieceSum r{{0.f, 0.f, 0.f, 0.f}};
    for (int g = gb; g < ge; ++g) {
        const int is = slot == 0 ? NBUF - 1 : slot - 1;
        if (sp.c < sp.c1) {
            copy_stream_unit<FMT>(ring + is * SB, sp, lane);
            if (++sp.c == sp.c1) sp = stream_seek<FMT == Q4M_MIX>(pinfo, n_phases, sp.ph + 1, blockIdx.x, C, warp);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");  // possibly empty: uniform group counts
        asm volatile("cp.async.wait_group %0;" ::"n"(NBUF - 1) : "memory");
        unit_mma_fmt<CF>(ring + slot * SB, xr, g, lane, r.acc);
        if constexpr (FMT == Q4M_MIX) __syncwarp();
        slot = slot + 1 == NBUF ? 0 : slot + 1;
    }
    ws.sp = sp;
    ws.slot = slot;
    return r;
}

// ---------------------------------------------------------------- tensor-parallel input
//
// RMSNorm input after a row-split GEMV on several ranks: h = hsrc + the ranks' partial rows
// of exchange point `point`, added in rank order (every rank adds the same words in the same
// order, so every rank holds the same h). Each warp converts whole groups as stage_x does;
// a lane loads its 4 elements of up to 4 ranks at a time and reloads the words whose flag is
// not yet this step's, at most `limit` times (then DEV_ERR_TIMEOUT; the step is discarded).
// h goes to `hout` from the CTA that owns pair 0; the records hold h * gain and the return
// value is 1 / sqrt(mean(h^2) + eps). Ends with the CTA synchronised.
// `base`: rank 0's slot of the point in this rank's area; `rs`: words from one slot to the next.
__device__ __noinline__ float stage_x_tp(const unsigned long long* base, size_t rs, int nranks, float eps,
                                         unsigned long long limit, const float* hsrc, float* hout, bool store_h,
                                         const float* norm_w, int cols, uint32_t flag, uint8_t* rec, float* misc,
                                         DeviceState* st) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = (cols + Q4M_KG - 1) / Q4M_KG, n4 = cols / 4;
    uint32_t* dig = reinterpret_cast<uint32_t*>(rec);
    float4* prm = reinterpret_cast<float4*>(rec + (size_t)G * 256);
    float ss = 0.f;
    for (int g = warp; g < G; g += NW) {
        const int i = g * 32 + lane;  // 16-byte piece of h: elements 4i .. 4i + 3
        float4 h = make_float4(0.f, 0.f, 0.f, 0.f), gn = h;
        if (i < n4) {
            h = __ldcg(reinterpret_cast<const float4*>(hsrc) + i);
            gn = reinterpret_cast<const float4*>(norm_w)[i];
            for (int r0 = 0; r0 < nranks; r0 += 4) {
                ulonglong2 w[4][2];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    if (r0 + k < nranks) {
                        const unsigned long long* p = base + (size_t)(r0 + k) * rs + 4 * (size_t)i;
                        w[k][0] = ld_ll2(p);
                        w[k][1] = ld_ll2(p + 2);
                    }
                }
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    if (r0 + k >= nranks) break;
                    const unsigned long long* p = base + (size_t)(r0 + k) * rs + 4 * (size_t)i;
                    for (unsigned long long it = 0; !(ll_ok(w[k][0], flag) && ll_ok(w[k][1], flag)); ++it) {
                        if (it >= limit || *(volatile int*)&st->error != DEV_OK) {
                            atomicCAS(&st->error, DEV_OK, DEV_ERR_TIMEOUT);
                            break;
                        }
                        __nanosleep(32);
                        w[k][0] = ld_ll2(p);
                        w[k][1] = ld_ll2(p + 2);
                    }
                    h.x += __uint_as_float((uint32_t)w[k][0].x);
                    h.y += __uint_as_float((uint32_t)w[k][0].y);
                    h.z += __uint_as_float((uint32_t)w[k][1].x);
                    h.w += __uint_as_float((uint32_t)w[k][1].y);
                }
            }
            if (store_h) reinterpret_cast<float4*>(hout)[i] = h;
            ss = fmaf(h.x, h.x, ss);
            ss = fmaf(h.y, h.y, ss);
            ss = fmaf(h.z, h.z, ss);
            ss = fmaf(h.w, h.w, ss);
        }
        const float4 v = make_float4(h.x * gn.x, h.y * gn.y, h.z * gn.z, h.w * gn.w);
        octet_to_records(v, lane, lane >> 3, dig + g * 64, prm + g * 4);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(JINF_FULL_MASK, ss, o);
    if (lane == 0) misc[warp] = ss;
    __syncthreads();
    ss = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) ss += misc[w];
    return rsqrtf(ss / (float)cols + eps);
}

// ---------------------------------------------------------------- input records
//
// A GEMV phase whose input was produced earlier in the step receives it as digit records
// (q4m_device.cuh) written by the producing phase's epilogue, so its CTAs only copy them
// (one L2 round trip) instead of each converting the whole input. For an RMSNorm input the
// records hold h * gain and the producer also leaves the sum of h^2 of every tile pair;
// every warp adds those up in the same fixed order (deterministic) for the norm factor.

// Copy the records (xrec_bytes(G)) into shared memory with one bulk copy on `mbar` (phase
// `parity`); returns the epilogue factor (1 / sqrt(mean(h^2) + eps) for a norm input, else
// 1). Every thread returns once the records are in shared memory.
__device__ __noinline__ float stage_records(const uint8_t* rec, const float* ssp, int n_ss, int cols, float eps,
                                           int G, uint8_t* xbase, uint32_t mbar, uint32_t parity, DeviceState* st,
                                           unsigned long long limit) {
    const int tid = threadIdx.x, lane = tid & 31;
    if (tid == 0) {
        fence_proxy_async();
        bulk_expect(mbar, (uint32_t)xrec_bytes(G));
        bulk_g2s(smem_u32(xbase), rec, (uint32_t)xrec_bytes(G), mbar);
    }
    float s = 0.f;
    if (ssp)
        for (int i0 = lane; i0 < n_ss; i0 += 8 * 32) {  // eight loads in flight per lane
            float t[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) t[k] = i0 + 32 * k < n_ss ? __ldcg(ssp + i0 + 32 * k) : 0.f;
#pragma unroll
            for (int k = 0; k < 8; ++k) s += t[k];
        }
    float fac = 1.0f;
    if (ssp) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(JINF_FULL_MASK, s, o);
        fac = rsqrtf(s / (float)cols + eps);
    }
    mbar_wait(mbar, parity, st, limit);
    return fac;
}

// EPI_RESID of one tile pair with records for the next phase, by a whole warp: lanes q < 16
// hold rows 2q, 2q+1 (v0, v1, already scaled). h += W x is stored; the pair's sum of h^2 and
// the records of h * gain (the pair is one 32-element block of the next input) are written.
__device__ __noinline__ void resid_records(const StepPhase& d, int pr, float v0, float v1) {
    const int lane = threadIdx.x & 31, q = lane & 15, row = pr * Q4M_PAIR_ROWS + 2 * q;
    float h0 = 0.f, h1 = 0.f;
    if (lane < 16 && row < d.rows) {
        h0 = __ldcg(d.y + row) + v0;
        d.y[row] = h0;
        if (row + 1 < d.rows) {
            h1 = __ldcg(d.y + row + 1) + v1;
            d.y[row + 1] = h1;
        }
    }
    float s = fmaf(h0, h0, h1 * h1);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) s += __shfl_xor_sync(JINF_FULL_MASK, s, o);
    if (lane == 0) d.ss_out[pr] = s;
    // octet layout: lane L < 8 takes elements 4L .. 4L+3 (rows of lanes 2L and 2L+1)
    const int src = 2 * (lane & 7);
    const float e0 = __shfl_sync(JINF_FULL_MASK, h0, src), e1 = __shfl_sync(JINF_FULL_MASK, h1, src);
    const float e2 = __shfl_sync(JINF_FULL_MASK, h0, src + 1), e3 = __shfl_sync(JINF_FULL_MASK, h1, src + 1);
    float4 gn = make_float4(0.f, 0.f, 0.f, 0.f);
    if (lane < 8 && pr * Q4M_PAIR_ROWS + 4 * lane < d.rows)
        gn = reinterpret_cast<const float4*>(d.gain_out + pr * Q4M_PAIR_ROWS)[lane];
    uint32_t* dig = reinterpret_cast<uint32_t*>(d.rec_out);
    float4* prm = reinterpret_cast<float4*>(d.rec_out + (size_t)d.groups_out * 256);
    octet_to_records(make_float4(e0 * gn.x, e1 * gn.y, e2 * gn.z, e3 * gn.w), lane, pr & 3, dig + (pr >> 2) * 64,
                     prm + (pr >> 2) * 4, lane < 8);
}

// Records of blocks [b0, b0 + nb) of the next input from fp32 values in shared memory
// (vals[32 * i] = first element of block b0 + i), by the whole CTA (4 blocks per warp pass).
__device__ __noinline__ void blocks_to_records(const float* vals, int b0, int nb, int groups_out, uint8_t* rec_out) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t* dig = reinterpret_cast<uint32_t*>(rec_out);
    float4* prm = reinterpret_cast<float4*>(rec_out + (size_t)groups_out * 256);
    for (int i0 = warp * 4; i0 < nb; i0 += NW * 4) {
        const int i = i0 + (lane >> 3);
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i < nb) v = reinterpret_cast<const float4*>(vals + 32 * i)[lane & 7];
        const int blk = b0 + i;
        octet_to_records(v, lane, blk & 3, dig + (blk >> 2) * 64, prm + (blk >> 2) * 4, i < nb);
    }
}

// ---------------------------------------------------------------- attention
//
// Decode attention over the fp16 cache (math of reference cuda/attention_kernel.cu:45-98:
// scores q.k / sqrt(hd), GQA head map h -> h / (H/Hkv), max-subtracted softmax, P.V). The
// positions of a kv head are split over S CTAs (S grows with the context, ATTN_SPLIT_POS
// positions per CTA, up to the CTAs available per kv head); the splits are merged in a
// fixed order by the CTAs that own the output blocks. Within a CTA the positions go in
// blocks of 16 warps x ATTN_PW: lanes own head dims, so a warp's load of a cache row is one
// contiguous 256-byte read (the rows were pulled into L2 during the QKV phase), every load
// of a block is issued before any arithmetic, and an online softmax joins the blocks.

struct AttnGeom {
    int kvh, sp, S, p0, p1;
};

// Split of CTA `cta` for a context of pos + 1 positions (false: no attention work).
__device__ __forceinline__ bool attn_geom(int pos, int n_kv_heads, int s_max, int cta, AttnGeom& a) {
    const int n_pos = pos + 1;
    int S = (n_pos + ATTN_SPLIT_POS - 1) / ATTN_SPLIT_POS;
    S = S > s_max ? s_max : S;
    if (cta >= n_kv_heads * S) return false;
    const int per = (n_pos + S - 1) / S;
    a.kvh = cta / S;
    a.sp = cta % S;
    a.S = S;
    a.p0 = a.sp * per;
    a.p1 = min(n_pos, a.p0 + per);
    if (a.p0 > a.p1) a.p0 = a.p1;
    return true;
}

template <int VD>
struct HalfVec;  // VD halves of one cache row, as loaded by one lane
template <>
struct HalfVec<4> {
    uint2 r;
    __device__ __forceinline__ void load(const __half* p) { r = __ldcg(reinterpret_cast<const uint2*>(p)); }
    __device__ __forceinline__ void zero() { r = make_uint2(0u, 0u); }
    __device__ __forceinline__ float get(int d) const {
        const __half2 h = *reinterpret_cast<const __half2*>(d < 2 ? &r.x : &r.y);
        return (d & 1) ? __high2float(h) : __low2float(h);
    }
};
template <>
struct HalfVec<2> {
    uint32_t r;
    __device__ __forceinline__ void load(const __half* p) { r = __ldcg(reinterpret_cast<const unsigned int*>(p)); }
    __device__ __forceinline__ void zero() { r = 0u; }
    __device__ __forceinline__ float get(int d) const {
        const __half2 h = *reinterpret_cast<const __half2*>(&r);
        return d ? __high2float(h) : __low2float(h);
    }
};

// One CTA's split [p0, p1) of kv head attention, after the QKV phase has finished: q of the
// GQ heads of the kv head at `q`, cache rows at kb / vb. Leaves either the normalised output
// in `outs` ([GQ][HD], shared memory; `part` null) or the split's partial (acc, m, l) in
// `part` ([GQ][HD + 2], global). Shared scratch at `xbase`: step_xstage_bytes covers it.
// PIPE: the next block's K and V rows are requested before this block's arithmetic (splits of
// several blocks; a split of one block, the persistent step's usual case, gains nothing).
template <int HD, int GQ, bool PIPE = false>
__device__ __noinline__ void attn_split(const float* q, const __half* kb, const __half* vb, int p0, int p1,
                                        uint8_t* xbase, float* part, float* outs) {
    constexpr int VD = HD / 32;                               // head dims per lane
    constexpr int PW = GQ * VD >= 32 ? ATTN_PW / 2 : ATTN_PW;  // positions per warp and block (registers)
    constexpr int BLK = NW * PW;                              // positions per block
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float* w_s = reinterpret_cast<float*>(xbase);  // [GQ][BLK] scores, then softmax weights
    float* ml_s = w_s + GQ * BLK;                   // [GQ][4]: m, l, correction
    float* red_s = ml_s + 4 * ATTN_MAX_GROUP;       // [NW][GQ][HD] per-warp p.v sums
    const float scale = rsqrtf((float)HD);
    float qr[GQ][VD];
#pragma unroll
    for (int g = 0; g < GQ; ++g) {
        if constexpr (VD == 4) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(q + g * HD) + lane);
            qr[g][0] = v.x * scale; qr[g][1] = v.y * scale; qr[g][2] = v.z * scale; qr[g][3] = v.w * scale;
        } else {
            const float2 v = __ldcg(reinterpret_cast<const float2*>(q + g * HD) + lane);
            qr[g][0] = v.x * scale; qr[g][1] = v.y * scale;
        }
    }
    if (tid < GQ) {
        ml_s[tid * 4] = -INFINITY;
        ml_s[tid * 4 + 1] = 0.f;
    }
    float acc[GQ][VD];
#pragma unroll
    for (int g = 0; g < GQ; ++g)
#pragma unroll
        for (int d = 0; d < VD; ++d) acc[g][d] = 0.f;
    // every K and V row piece of this warp's positions warp, warp + 16, ... of a block at once
    HalfVec<VD> kr[PW], vr[PW], kn[PW], vn[PW];
    auto fetch = [&](int b, HalfVec<VD>(&kk)[PW], HalfVec<VD>(&vv)[PW]) {
        const int nb = min(BLK, p1 - b);
#pragma unroll
        for (int k = 0; k < PW; ++k) {
            const int j = warp + NW * k;
            if (j < nb) {
                kk[k].load(kb + (size_t)(b + j) * HD + lane * VD);
                vv[k].load(vb + (size_t)(b + j) * HD + lane * VD);
            } else {
                kk[k].zero();
                vv[k].zero();
            }
        }
    };
    if (PIPE && p0 < p1) fetch(p0, kn, vn);
    for (int b0 = p0; b0 < p1; b0 += BLK) {
        const int n = min(BLK, p1 - b0);
        if (PIPE) {
#pragma unroll
            for (int k = 0; k < PW; ++k) {
                kr[k] = kn[k];
                vr[k] = vn[k];
            }
            if (b0 + BLK < p1) fetch(b0 + BLK, kn, vn);
        } else {
            fetch(b0, kr, vr);
        }
        // scores: each lane's dims, summed over the warp
#pragma unroll
        for (int k = 0; k < PW; ++k) {
            const int j = warp + NW * k;
#pragma unroll
            for (int g = 0; g < GQ; ++g) {
                float a = 0.f;
#pragma unroll
                for (int d = 0; d < VD; ++d) a = fmaf(qr[g][d], kr[k].get(d), a);
                a = warp_sum(a);
                if (lane == 0 && j < n) w_s[g * BLK + j] = a;
            }
        }
        __syncthreads();
        // online softmax of the block, one warp per query head
        if (warp < GQ) {
            float sv[BLK / 32];
            float mb = -INFINITY;
#pragma unroll
            for (int t = 0; t < BLK / 32; ++t) {
                const int j = lane + 32 * t;
                sv[t] = j < n ? w_s[warp * BLK + j] : -INFINITY;
                mb = fmaxf(mb, sv[t]);
            }
            const float mo = ml_s[warp * 4], mn = fmaxf(mo, warp_max(mb));
            float es = 0.f;
#pragma unroll
            for (int t = 0; t < BLK / 32; ++t) {
                const int j = lane + 32 * t;
                const float e = j < n ? expf(sv[t] - mn) : 0.f;
                if (j < BLK) w_s[warp * BLK + j] = e;
                es += e;
            }
            const float corr = mo == -INFINITY ? 0.f : expf(mo - mn);
            const float ln = fmaf(ml_s[warp * 4 + 1], corr, warp_sum(es));
            __syncwarp();
            if (lane == 0) {
                ml_s[warp * 4] = mn;
                ml_s[warp * 4 + 1] = ln;
                ml_s[warp * 4 + 2] = corr;
            }
        }
        __syncthreads();
        // p.v over this warp's positions, lanes own dims
#pragma unroll
        for (int g = 0; g < GQ; ++g) {
            const float c = ml_s[g * 4 + 2];
#pragma unroll
            for (int d = 0; d < VD; ++d) acc[g][d] *= c;
#pragma unroll
            for (int k = 0; k < PW; ++k) {
                const float e = w_s[g * BLK + warp + NW * k];  // 0 past the block's positions
#pragma unroll
                for (int d = 0; d < VD; ++d) acc[g][d] = fmaf(e, vr[k].get(d), acc[g][d]);
            }
        }
        __syncthreads();  // the next block overwrites the weights
    }
    // sum the warps' p.v in warp order
#pragma unroll
    for (int g = 0; g < GQ; ++g)
#pragma unroll
        for (int d = 0; d < VD; ++d) red_s[(warp * GQ + g) * HD + lane * VD + d] = acc[g][d];
    __syncthreads();
    for (int o = tid; o < GQ * HD; o += STEP_THREADS) {
        float a = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) a += red_s[w * GQ * HD + o];
        const int g = o / HD, dd = o % HD;
        if (part) {
            part[g * (HD + 2) + dd] = a;
            if (dd == 0) {
                part[g * (HD + 2) + HD] = p1 > p0 ? ml_s[g * 4] : -INFINITY;  // an empty split
                part[g * (HD + 2) + HD + 1] = ml_s[g * 4 + 1];
            }
        } else {
            outs[o] = a / ml_s[g * 4 + 1];
        }
    }
}

}  // namespace

template <int FMT, int NBUF, bool TP>
__global__ void __launch_bounds__(STEP_THREADS, 1) k_step(const StepParams P) {
    constexpr int UB = q4m_unit_bytes(FMT);  // ring slot bytes (the largest unit of a mixed model)
    constexpr bool MIXED = FMT == Q4M_MIX;
    extern __shared__ __align__(16) uint8_t smem[];
    // shared memory: [xstage | misc 256 B | flags, keys, piece table 512 B | partial rows 4 KB |
    //                 outputs to convert 4 KB | phase descriptor 2 x 256 B | phase infos | rings]
    uint8_t* xbase = smem;
    float* misc = reinterpret_cast<float*>(smem + P.xstage_bytes);        // 64 floats of reductions
    int* flags = reinterpret_cast<int*>(smem + P.xstage_bytes + 256);     // [0..1] go, [2] attention last
    u64* wkeys = reinterpret_cast<u64*>(smem + P.xstage_bytes + 256 + 64);  // [NW] argmax keys
    int* ftile = reinterpret_cast<int*>(smem + P.xstage_bytes + 256 + 192);  // [NW] tile of a warp's first piece
    int* fmid = ftile + NW;                                                  // [NW] first piece starts mid-tile
    float* part_s = reinterpret_cast<float*>(smem + P.xstage_bytes + 768);   // [NW][2][32] partial rows
    float* outs_s = reinterpret_cast<float*>(smem + P.xstage_bytes + 768 + 4096);  // [1024] outputs to convert
    const uint32_t mbar_rec = smem_u32(smem + P.xstage_bytes + 576);  // bulk copies of input records
    StepPhase* dsm = reinterpret_cast<StepPhase*>(smem + P.xstage_bytes + 768 + 8192);  // [2] descriptors
    PhaseInfo* pinfo = reinterpret_cast<PhaseInfo*>(smem + P.xstage_bytes + 768 + 8192 + 512);
    const uint32_t ring_base = smem_u32(pinfo + ((P.n_phases + 1) & ~1));
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t ring = ring_base + (uint32_t)(warp * NBUF * UB);
    const int C = gridDim.x;
    DeviceState* st = P.st;
    const int pos = *(volatile int*)&st->pos;
    // tensor parallel: this step's epoch (steps finished so far, the same on every rank; only
    // the finalizer advances it, after every CTA's last use). Re-read where needed rather
    // than kept live through the kernel.
    auto epoch = [&]() -> unsigned long long { return *(volatile unsigned long long*)P.xpeer[P.tp_rank]; };

    // stream geometry of every phase -> shared memory
    for (int i = tid; i < P.n_phases; i += STEP_THREADS) {
        PhaseInfo pi;
        pi.w = P.phases[i].w;
        pi.pairs = P.phases[i].pairs;
        pi.gran = P.phases[i].gran;
        pi.groups = P.phases[i].kind == PH_GEMV ? P.phases[i].groups : 0;
        pi.fmts = P.phases[i].fmts;
        pinfo[i] = pi;
    }
    if (tid == 0) {
        mbar_init(mbar_rec);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    uint32_t par_rec = 0;  // next phase of the records mbarrier (the same in every thread)
    __syncthreads();

    // ---------------- weight stream: this warp's unit ranges of all GEMV phases, copied in
    // consumption order into the ring (NBUF - 1 units ahead of the arithmetic)
    WarpStream<MIXED> ws;
    ws.sp = stream_seek<MIXED>(pinfo, P.n_phases, 0, blockIdx.x, C, warp);
    ws.slot = 0;
    for (int i = 0; i < NBUF - 1; ++i) {
        if (ws.sp.c < ws.sp.c1) {
            copy_stream_unit<FMT>(ring + i * UB, ws.sp, lane);
            if (++ws.sp.c == ws.sp.c1)
                ws.sp = stream_seek<MIXED>(pinfo, P.n_phases, ws.sp.ph + 1, blockIdx.x, C, warp);
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
        JINF_TRACE(ph, 0);
        if (tid == 0) {
            const StepPhase& g = P.phases[ph];
            // (a tensor-parallel input waits in its staging: the flagged words are the signal)
            flags[ph & 1] = g.dep < 0 || (TP && g.xin >= 0)
                                ? 1
                                : (wait_ge(P.done + g.dep, g.dep_target, st, P.spin_limit) ? 1 : 0);
        } else if (tid >= 32 && tid < 32 + DWORDS) {  // descriptor -> shared memory while warp 0 polls
            reinterpret_cast<uint32_t*>(&d)[tid - 32] = reinterpret_cast<const uint32_t*>(P.phases + ph)[tid - 32];
        } else if (tid >= 96) {
            if (tid == 32 * 9) {  // L2 prefetch of later weights while warp 0 polls
                for (int k = 0; k < 2; ++k) {
                    const int j = P.phases[ph].pf[k];
                    if (j > ph && j < P.n_phases) prefetch_cta_range(pinfo[j], blockIdx.x, C, UB, MIXED);
                }
            }
        }
        __syncthreads();  // also: every warp is done with the previous phase's shared data
        if (!flags[ph & 1]) break;
        JINF_TRACE(ph, 1);

        if (d.kind == PH_ATTN) {
            // ---------------- attention: CTA (kv head, split) of the context
            AttnGeom a;
            if (!attn_geom(pos, P.n_kv_heads, P.attn_smax, blockIdx.x, a)) continue;
            const int hd = P.head_dim, gq = P.n_heads / P.n_kv_heads;
            const float* qh = d.q + (size_t)a.kvh * gq * hd;
            const __half* kb = d.kcache + (size_t)a.kvh * P.max_ctx * hd;
            const __half* vb = d.vcache + (size_t)a.kvh * P.max_ctx * hd;
            float* gpart =
                a.S > 1 ? P.attn_part + ((size_t)a.kvh * ATTN_MAX_SPLIT + a.sp) * ATTN_MAX_GROUP * (hd + 2) : nullptr;
#define JINF_ATTN_SPLIT(HD_, GQ_) attn_split<HD_, GQ_>(qh, kb, vb, a.p0, a.p1, xbase, gpart, outs_s)
            if (hd == 64) {
                if (gq == 8) JINF_ATTN_SPLIT(64, 8);
                else if (gq == 4) JINF_ATTN_SPLIT(64, 4);
                else if (gq == 2) JINF_ATTN_SPLIT(64, 2);
                else JINF_ATTN_SPLIT(64, 1);
            } else {
                if (gq == 8) JINF_ATTN_SPLIT(128, 8);
                else if (gq == 4) JINF_ATTN_SPLIT(128, 4);
                else if (gq == 2) JINF_ATTN_SPLIT(128, 2);
                else JINF_ATTN_SPLIT(128, 1);
            }
#undef JINF_ATTN_SPLIT
            JINF_TRACE(ph, 2);
            const int nblk = gq * hd / 32;  // 32-element output blocks of this kv head
            if (a.S == 1) {
                __syncthreads();
                if (d.rec_out) {
                    blocks_to_records(outs_s, a.kvh * nblk, nblk, d.groups_out, d.rec_out);
                } else {
                    for (int i = tid; i < gq * hd; i += STEP_THREADS) d.out[(size_t)a.kvh * gq * hd + i] = outs_s[i];
                }
                __syncthreads();
                if (tid == 0) {
                    __threadfence();
                    atomicAdd(P.done + ph, (unsigned)nblk);
                }
                JINF_TRACE(ph, 5);
                continue;
            }
            // publish this split's partial; the splits that own output blocks (split sp owns
            // blocks sp, sp + S, ...) wait for all S partials of the kv head, then each merges its
            // blocks in split order (deterministic) and writes them as records
            __syncthreads();
            unsigned* cnt = P.attn_cnt + d.layer * P.n_kv_heads + a.kvh;
            if (tid == 0) {
                __threadfence();
                atomicAdd(cnt, 1u);
            }
            JINF_TRACE(ph, 3);
            if (a.sp >= nblk) continue;
            if (tid == 0) flags[2] = wait_ge(cnt, (unsigned)a.S, st, P.spin_limit) ? 1 : 0;
            __syncthreads();  // (a timeout is recorded in the device state; the step is then discarded)
            JINF_TRACE(ph, 4);
            const size_t stride = (size_t)ATTN_MAX_GROUP * (hd + 2);
            const float* base = P.attn_part + (size_t)a.kvh * ATTN_MAX_SPLIT * stride;
            float* ml = reinterpret_cast<float*>(xbase);  // [S][2] (m, l) of the block's query head
            float* av = ml + 2 * ATTN_MAX_SPLIT;           // [S][32] accumulators of the block
            float* ew = av + 32 * ATTN_MAX_SPLIT;          // [S] split weights e^(m_s - M)
            unsigned mine = 0;
            for (int b = a.sp; b < nblk; b += a.S, ++mine) {
                const int g = b * 32 / hd, dd0 = b * 32 % hd;
                {  // every partial load of the thread before any store (S <= 64: at most 4)
                    float t4[4];
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const int t = tid + k * STEP_THREADS;
                        t4[k] = t < a.S * 32 ? __ldcg(base + (t >> 5) * stride + g * (hd + 2) + dd0 + (t & 31)) : 0.f;
                    }
                    const float m0 = tid < a.S ? __ldcg(base + tid * stride + g * (hd + 2) + hd) : 0.f;
                    const float l0 = tid < a.S ? __ldcg(base + tid * stride + g * (hd + 2) + hd + 1) : 0.f;
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        if (tid + k * STEP_THREADS < a.S * 32) av[tid + k * STEP_THREADS] = t4[k];
                    if (tid < a.S) {
                        ml[2 * tid] = m0;
                        ml[2 * tid + 1] = l0;
                    }
                }
                __syncthreads();
                if (warp == 0) {
                    // lanes own splits lane, lane + 32: the max, the weights and their sum in parallel
                    const float ma = lane < a.S ? ml[2 * lane] : -INFINITY;
                    const float mb = lane + 32 < a.S ? ml[2 * (lane + 32)] : -INFINITY;
                    const float M = warp_max(fmaxf(ma, mb));
                    const float ea = ma == -INFINITY ? 0.f : expf(ma - M);  // 0: an empty split
                    const float eb = mb == -INFINITY ? 0.f : expf(mb - M);
                    const float L = warp_sum((lane < a.S ? ml[2 * lane + 1] * ea : 0.f) +
                                             (lane + 32 < a.S ? ml[2 * (lane + 32) + 1] * eb : 0.f));
                    if (lane < a.S) ew[lane] = ea;
                    if (lane + 32 < a.S) ew[lane + 32] = eb;
                    __syncwarp();
                    float v = 0.f;
                    for (int s2 = 0; s2 < a.S; ++s2) v = fmaf(ew[s2], av[s2 * 32 + lane], v);
                    v /= L;
                    const int blk = a.kvh * nblk + b;  // block of the o projection's input
                    if (d.rec_out) {
                        // octet layout: lane q < 8 takes elements 4q .. 4q+3
                        const int src = 4 * (lane & 7);
                        const float4 x = make_float4(__shfl_sync(JINF_FULL_MASK, v, src), __shfl_sync(JINF_FULL_MASK, v, src + 1),
                                                     __shfl_sync(JINF_FULL_MASK, v, src + 2), __shfl_sync(JINF_FULL_MASK, v, src + 3));
                        uint32_t* dig = reinterpret_cast<uint32_t*>(d.rec_out);
                        float4* prm = reinterpret_cast<float4*>(d.rec_out + (size_t)d.groups_out * 256);
                        octet_to_records(x, lane, blk & 3, dig + (blk >> 2) * 64, prm + (blk >> 2) * 4, lane < 8);
                    } else {
                        d.out[(size_t)blk * 32 + lane] = v;
                    }
                }
                __syncthreads();  // the scratch is reused by the next block
            }
            if (tid == 0) {
                __threadfence();
                atomicAdd(P.done + ph, mine);
            }
            JINF_TRACE(ph, 5);
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
        int t0, t1;
        cta_range(blockIdx.x, C, d.pairs, d.gran, t0, t1);
        if (t0 >= t1) continue;
        // Epilogue inputs that do not depend on this GEMV, prepared now by warps 1.. while
        // warp 0 starts the input staging (outs_s is free in these phases): the residual rows
        // of an EPI_RESID phase, the RoPE factors of an EPI_QKV phase. The staging ends with
        // the CTA synchronised, before any epilogue reads them.
        const int prow0 = t0 * Q4M_PAIR_ROWS, nprow = (t1 - t0) * Q4M_PAIR_ROWS;
        const bool pre = ((d.epi == EPI_RESID && !d.rec_out) || d.epi == EPI_QKV) && nprow <= 1024;
        if (pre && tid >= 32) {
            for (int i = tid - 32; i < nprow; i += STEP_THREADS - 32) {
                const int row = prow0 + i;
                if (d.epi == EPI_RESID) {
                    outs_s[i] = row < d.rows ? __ldcg(d.y + row) : 0.f;
                } else if ((i & 1) == 0 && row < P.nq + P.nk) {
                    float cs, sn;
                    rope_pair(row < P.nq ? row : row - P.nq, pos, P.rope_base, P.head_dim, cs, sn);
                    outs_s[i] = cs;
                    outs_s[i + 1] = sn;
                }
            }
        }
        float fac;
        if (d.xm == X_RECORDS) {
            fac = stage_records(d.rec, d.ssp, d.n_ss, d.cols, P.eps, G, xbase, mbar_rec, par_rec, st, P.spin_limit);
            par_rec ^= 1u;
        } else {
            const float* hsrc =
                d.xm == X_EMBED_NORM ? d.hsrc + (size_t)(*(volatile int*)&st->token) * d.cols : d.hsrc;
            // the CTA that owns pair 0 stores the embedding row as the residual stream
            if (TP && d.xm == X_RMSNORM_TP) {
                const unsigned long long ep = epoch();
                fac = stage_x_tp(xchg_data(P, P.tp_rank, d.xin, (unsigned)(ep & 1ull), 0), (size_t)(P.x_slot / 8),
                                 P.tp_size, P.eps, P.spin_limit, hsrc, d.hout, t0 == 0 && d.hout, d.norm_w, d.cols,
                                 (uint32_t)(ep + 1ull), xbase, misc, st);
            } else
                fac = stage_x<STEP_THREADS>(d.xm, d.x, hsrc, nullptr, d.hout, t0 == 0, d.norm_w, P.eps, d.cols,
                                            xbase, misc, true);
        }
        JINF_TRACE(ph, 2);
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
            ea.pre = pre ? outs_s : nullptr;
            ea.pre_row0 = prow0;
            epilogue_pair(ea, row, v0 * fac, v1 * fac, lmax, lidx);
        };
        // a finished pair, by the whole warp (lanes q < 16 hold rows 2q, 2q+1)
        auto finish_pair = [&](int pr, float v0, float v1) {
            const int q = lane & 15, row = pr * Q4M_PAIR_ROWS + 2 * q;
            if (TP && d.epi == EPI_PARTIAL) {
                // this rank's partial rows into its slot of every rank's exchange area
                if (lane < 16 && row < d.rows) {  // (rows: a multiple of 32)
                    const unsigned long long ep = epoch();
                    const uint32_t flag = (uint32_t)(ep + 1ull);
                    const unsigned long long w0 = ll_word(v0 * fac, flag), w1 = ll_word(v1 * fac, flag);
                    for (int r = 0; r < P.tp_size; ++r)
                        st_ll2(xchg_data(P, r, d.xout, (unsigned)(ep & 1ull), P.tp_rank) + row, w0, w1);
                }
            } else if (d.rec_out && d.epi == EPI_RESID) {
                resid_records(d, pr, v0 * fac, v1 * fac);
            } else if (d.rec_out && d.epi == EPI_GATEUP) {
                // the activation goes to shared memory; whole blocks become records below
                if (lane < 16) {
                    const float g = v0 * fac, u = v1 * fac;
                    outs_s[(pr - t0) * 16 + q] = row < d.rows ? g / (1.0f + expf(-g)) * u : 0.f;
                }
            } else if (lane < 16) {
                epilogue(row, v0, v1);
            }
        };
        int c, c1;
        warp_range(blockIdx.x, C, warp, d.pairs, d.gran, G, c, c1);
        if (lane == 0) {
            ftile[warp] = -1;
            fmid[warp] = 0;
        }
        bool first_piece = true;
        int own_pair = -1, own_slot = 0;  // the split pair this warp finishes (its piece starts the pair)
        int pair = c / G, gb = c - pair * G;  // walked incrementally: no division per piece
        for (; c < c1; ++pair, gb = 0) {
            const int ge = c1 - c < G - gb ? gb + (c1 - c) : G;
            PieceSum ps;
            if constexpr (MIXED) {
                const int f = pair < (d.fmts >> 8) ? (d.fmts & 15) : ((d.fmts >> 4) & 15);
                ps = f == Q4M_Q6_K   ? stream_piece<FMT, NBUF, Q4M_Q6_K>(ws, ring, pinfo, P.n_phases, C, xr, gb, ge)
                     : f == Q4M_Q4_K ? stream_piece<FMT, NBUF, Q4M_Q4_K>(ws, ring, pinfo, P.n_phases, C, xr, gb, ge)
                                     : stream_piece<FMT, NBUF, Q4M_Q4_0>(ws, ring, pinfo, P.n_phases, C, xr, gb, ge);
            } else {
                ps = stream_piece<FMT, NBUF, FMT>(ws, ring, pinfo, P.n_phases, C, xr, gb, ge);
            }
            c += ge - gb;
            if (first_piece && lane == 0) {
                ftile[warp] = pair;
                fmid[warp] = gb > 0;
            }
            unit_reduce(ps.acc);
            if (gb == 0 && ge == G) {
                const int q = lane & 15;
                const float v0 = unit_row(ps.acc, 2 * q), v1 = unit_row(ps.acc, 2 * q + 1);
                finish_pair(pair, v0, v1);
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
        JINF_TRACE(ph, 3);
        __syncthreads();
        JINF_TRACE(ph, 4);
        if (own_pair >= 0) {
            // add the pieces of the following warps in warp order, then the epilogue. The
            // contributing warps are the ones after this warp, up to the first warp with units
            // that does not continue this pair (warps without units skipped): found with two
            // ballots over the per-warp tile words, so the piece loads issue back to back.
            const int q = lane & 15;
            const int ftl = ftile[q], fml = fmid[q];
            const unsigned bad = __ballot_sync(JINF_FULL_MASK, lane < NW && lane > warp && ftl >= 0 &&
                                                                   (ftl != own_pair || !fml));
            const int stop = bad ? __ffs(bad) - 1 : NW;
            const unsigned good = __ballot_sync(JINF_FULL_MASK, lane < NW && lane > warp && lane < stop && ftl >= 0);
            float v0 = part_s[(warp * 2 + own_slot) * 32 + 2 * q];
            float v1 = part_s[(warp * 2 + own_slot) * 32 + 2 * q + 1];
            float p0[NW], p1[NW];
#pragma unroll
            for (int w2 = 0; w2 < NW; ++w2) {
                p0[w2] = (good >> w2) & 1u ? part_s[(w2 * 2) * 32 + 2 * q] : 0.f;
                p1[w2] = (good >> w2) & 1u ? part_s[(w2 * 2) * 32 + 2 * q + 1] : 0.f;
            }
#pragma unroll
            for (int w2 = 0; w2 < NW; ++w2) {
                if ((good >> w2) & 1u) {
                    v0 += p0[w2];
                    v1 += p1[w2];
                }
            }
            finish_pair(own_pair, v0, v1);
        }
        __syncthreads();  // every epilogue store of the CTA precedes the report
        if (d.rec_out && d.epi == EPI_GATEUP) {
            // pairs [t0, t1) hold activation blocks [t0 / 2, t1 / 2) (gran 2)
            blocks_to_records(outs_s, t0 >> 1, (t1 - t0) >> 1, d.groups_out, d.rec_out);
            __syncthreads();
        }
        if (tid == 0) {
            __threadfence();
            atomicAdd(P.done + ph, (unsigned)(t1 - t0));
        }
        JINF_TRACE(ph, 5);
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");

    // ---------------- leave: LM head argmax, then the last CTA finishes the step
    if (P.with_argmax) {
        u64 key = lmax == -INFINITY ? 0ull : argmax_key(lmax, lidx + P.vocab_off);
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
            u64 b = P.with_argmax ? atomicAdd(&st->best, 0ull) : 0ull;
            const bool tp = TP && P.tp_size > 1;
            const unsigned long long ep = tp ? epoch() : 0ull;
            const unsigned par = (unsigned)(ep & 1ull);
            if (tp) {
                // every rank's argmax key to every rank, then the largest (the key order puts the
                // lower global index first on ties). Steps without an LM head exchange a zero key,
                // so that every rank's step ends only after all writes into its area have landed.
                u64* keys = reinterpret_cast<u64*>(P.xpeer[P.tp_rank] + P.x_keys) + par * STEP_MAX_TP;
                for (int r = 0; r < P.tp_size; ++r)
                    reinterpret_cast<volatile u64*>(P.xpeer[r] + P.x_keys)[par * STEP_MAX_TP + P.tp_rank] = b;
                __threadfence_system();
                for (int r = 0; r < P.tp_size; ++r)
                    atomicAdd_system(reinterpret_cast<unsigned long long*>(P.xpeer[r] + P.x_keycnt), 1ull);
                if (wait_ge_sys(reinterpret_cast<const unsigned long long*>(P.xpeer[P.tp_rank] + P.x_keycnt),
                                (ep + 1ull) * (unsigned long long)P.tp_size, st, P.spin_limit)) {
                    for (int r = 0; r < P.tp_size; ++r) {
                        const u64 k = __ldcg(keys + r);
                        b = k > b ? k : b;
                    }
                }
            }
            if (P.with_argmax) {
                st->argmax_token = b ? (int)(0xFFFFFFFFu - (uint32_t)(b & 0xFFFFFFFFull)) : 0;
                st->token = st->argmax_token;
                st->best = 0ull;
            }
            st->pos = pos + 1;
            for (int i = 0; i <= P.n_phases; ++i) P.done[i] = 0u;
            for (int i = 0; i < P.n_attn_cnt; ++i) P.attn_cnt[i] = 0u;
            if (tp) *reinterpret_cast<volatile unsigned long long*>(P.xpeer[P.tp_rank]) = ep + 1ull;
        }
    }
}

// ---------------------------------------------------------------- host side

unsigned int step_xstage_bytes(int max_cols, int group, int head_dim) {
    const size_t G = (size_t)(max_cols + Q4M_KG - 1) / Q4M_KG;
    const size_t gemv = xrec_bytes((int)G);
    // attention: scores [group][NW * ATTN_PW], (m, l, correction) [ATTN_MAX_GROUP][4], p.v sums
    // [NW][group][head_dim]
    const size_t attn = sizeof(float) * ((size_t)group * NW * ATTN_PW + 4 * ATTN_MAX_GROUP + (size_t)NW * group * head_dim);
    const size_t merge = sizeof(float) * (size_t)(2 + 32 + 1) * ATTN_MAX_SPLIT;  // split merge scratch
    size_t b = gemv > attn ? gemv : attn;
    b = b > merge ? b : merge;
    return (unsigned int)((b + 15) & ~(size_t)15);
}

XchgLayout step_xchg_layout(int n_points, int tp_size, int d) {
    auto up = [](unsigned long long v) { return (v + 255ull) & ~255ull; };
    XchgLayout l;
    l.keycnt = 256;
    l.keys = l.keycnt + 256;
    l.data = up(l.keys + 2ull * STEP_MAX_TP * 8ull);
    l.slot = up(8ull * (unsigned long long)d);
    l.point = l.slot * (unsigned long long)tp_size;  // one parity of one point: every rank's slot
    l.total = l.data + (unsigned long long)n_points * 2ull * l.point;
    return l;
}

size_t step_smem_bytes(unsigned int xstage_bytes, int n_phases, int fmt, int nbuf) {
    const size_t infos = sizeof(PhaseInfo) * (size_t)((n_phases + 1) & ~1);
    return (size_t)xstage_bytes + 768 + 8192 + 512 + infos + (size_t)NW * nbuf * q4m_unit_bytes(fmt);
}

// The kernel instances: weight format x ring depth (STEP_NBUF, or 3 when a model's staged
// inputs leave no room for STEP_NBUF slots) x tensor parallel (the single-GPU instance
// carries none of the exchange code). Mixed-format models (Q4M_MIX) take 3 slots of the
// largest unit.
typedef void (*StepKernel)(const StepParams);
static StepKernel step_kernel_for(int fmt, int nbuf, bool tp) {
    if (fmt == Q4M_MIX) return tp ? k_step<Q4M_MIX, 3, true> : k_step<Q4M_MIX, 3, false>;
    if (tp) {
        if (fmt == Q4M_Q4_K) return nbuf == 3 ? k_step<Q4M_Q4_K, 3, true> : k_step<Q4M_Q4_K, STEP_NBUF, true>;
        return nbuf == 3 ? k_step<Q4M_Q4_0, 3, true> : k_step<Q4M_Q4_0, STEP_NBUF, true>;
    }
    if (fmt == Q4M_Q4_K) return nbuf == 3 ? k_step<Q4M_Q4_K, 3, false> : k_step<Q4M_Q4_K, STEP_NBUF, false>;
    return nbuf == 3 ? k_step<Q4M_Q4_0, 3, false> : k_step<Q4M_Q4_0, STEP_NBUF, false>;
}

static cudaError_t step_configure(size_t smem, int fmt, int nbuf, bool tp) {
    static size_t configured[64][12] = {{0}};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    const int slot = (fmt == Q4M_MIX ? 8 : fmt == Q4M_Q4_K ? 2 : 0) + (nbuf == 3 ? 1 : 0) + (tp ? 4 : 0) -
                     (fmt == Q4M_MIX && tp ? 2 : 0);  // mixed: 8 + nbuf3 (+ 2 for tp)
    if (smem <= configured[dev][slot]) return cudaSuccess;
    const cudaError_t e =
        cudaFuncSetAttribute(step_kernel_for(fmt, nbuf, tp), cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess) configured[dev][slot] = smem;
    return e;
}

int step_occupancy(size_t smem, int fmt, int nbuf) {
    int lo = 0;
    for (const bool tp : {false, true}) {
        if (step_configure(smem, fmt, nbuf, tp) != cudaSuccess) return 0;
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, step_kernel_for(fmt, nbuf, tp), STEP_THREADS, smem) !=
            cudaSuccess)
            return 0;
        lo = tp ? std::min(lo, n) : n;
    }
    return lo;
}

#ifdef JINF_STEP_TRACE
extern "C" int jinf_step_trace_read(unsigned long long* host, size_t n) {
    const size_t cap = (size_t)TRACE_MAX_PH * TRACE_MAX_CTA * TRACE_PTS;
    if (n > cap) n = cap;
    return cudaMemcpyFromSymbol(host, g_step_trace, n * sizeof(unsigned long long)) == cudaSuccess ? 0 : -1;
}
#endif

// ---------------------------------------------------------------- multi-sequence attention

namespace {

// The multi-sequence attention's split [p0, p1) of one kv head on the tensor cores
// (mma.sync, fp16 operands, fp32 accumulation), in CTAs of 8 warps, two per SM. K and V are
// the cache's fp16 values; q and the softmax weights p enter as fp16 hi + lo pairs (x = hi +
// lo to about 22 bits), so every product is the fp32 one to that rounding, and sums are fp32.
// The split is cut into 64-position blocks only to size the splits (TA_BLK); each warp
// streams chunks of 8 positions (attn_split_w). Leaves the split's partial (acc, m, l) in
// `part` ([GQ][HD + 2]), as attn_split does.
constexpr int TA_BLK = 64;
constexpr int TA_THREADS = 256;
constexpr int TA_NW = TA_THREADS / 32;
constexpr int TW_NST = 3;  // chunks in each warp's ring (attn_split_w)

// The split computed warp by warp, with no CTA barrier per chunk: warp w streams its own
// chunks of 8 positions (chunks w, w + 8, ... of the split) through a private cp.async ring of
// TW_NST chunks in shared memory, and keeps its own online softmax (m, l per head) and output
// accumulator; the 8 warps are merged once at the end, in warp order. Per chunk:
//   scores S = Q K^T (m16n8k16: the query heads as the MMA's rows, q hi + lo, the chunk's 8
//     positions as its columns), masked past p1;
//   the chunk's softmax weights stay in the registers that hold the scores: their layout
//     (head gid, positions 2 tig, 2 tig + 1) is the B fragment of the next MMA;
//   O^T += V^T P^T (m16n8k8: head dims as rows, the 8 positions as k, the heads as columns;
//     p hi + lo), V^T fragments by ldmatrix .trans.
template <int HD>
__host__ __device__ constexpr size_t tw_smem() {
    return (size_t)TA_NW * TW_NST * 16 * (HD + 8) * 2  // per warp: TW_NST chunks of K and V rows
           + (size_t)(HD / 16) * 32 * 16;              // q fragments [k-step][lane]
}

__device__ __forceinline__ void mma_f16_k8(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5}, {%6}, {%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(b0));
}

template <int HD, int GQ>
__device__ __forceinline__ void attn_split_w(const float* q, const __half* kb, const __half* vb, int p0, int p1,
                                             uint8_t* sm, float* part) {
    static_assert(GQ <= 8 && HD % 32 == 0 && HD <= 128, "heads are the MMA's 8 columns");
    constexpr int LD = HD + 8;               // padded row, halves
    constexpr int CHW = 16 * LD;             // halves per chunk: K rows 0..7, V rows 8..15
    constexpr int KS = HD / 16;              // score k-steps
    constexpr int MTL = HD / 16;             // p.v m-tiles
    constexpr int CH = HD / 8;               // 16-byte pieces per cache row
    static_assert((size_t)TA_NW * GQ * HD * 4 <= (size_t)TA_NW * TW_NST * CHW * 2, "the merge reuses the rings");
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, gid = lane >> 2, tig = lane & 3;
    __half* ring = reinterpret_cast<__half*>(sm) + (size_t)warp * TW_NST * CHW;
    uint4* qf = reinterpret_cast<uint4*>(sm + (size_t)TA_NW * TW_NST * CHW * 2);
    const int nc = (p1 - p0 + 7) / 8;                     // chunks of the split
    const int mine = nc > warp ? (nc - warp + TA_NW - 1) / TA_NW : 0;  // this warp's chunks

    // chunk k of this warp (positions p0 + 8 (warp + 8 k) ..) into ring slot k % TW_NST; rows
    // past p1 are zero-filled
    auto load_chunk = [&](int k) {
        __half* dst = ring + (k % TW_NST) * CHW;
        const int pos0 = p0 + 8 * (warp + TA_NW * k);
#pragma unroll
        for (int i = lane; i < 16 * CH; i += 32) {
            const int r = i / CH, c = i % CH, pr = r & 7;
            const bool in = pos0 + pr < p1;
            const __half* src = (r < 8 ? kb : vb) + (size_t)(in ? pos0 + pr : p0) * HD + c * 8;
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst + r * LD + c * 8)),
                         "l"(src), "r"(in ? 16 : 0)
                         : "memory");
        }
    };
#pragma unroll
    for (int k = 0; k < TW_NST - 1; ++k) {
        if (k < mine) load_chunk(k);
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    if (warp == 0) {  // the query fragments (the same for every warp): head gid, zero past GQ
        const float scale = rsqrtf((float)HD);
#pragma unroll
        for (int st = 0; st < KS; ++st) {
            uint32_t hi[2], lo[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                float2 t = make_float2(0.f, 0.f);
                if (gid < GQ) t = __ldcg(reinterpret_cast<const float2*>(q + gid * HD + st * 16 + h * 8 + tig * 2));
                split_h2(t.x * scale, t.y * scale, hi[h], lo[h]);
            }
            qf[st * 32 + lane] = make_uint4(hi[0], hi[1], lo[0], lo[1]);
        }
    }
    __syncthreads();  // the query fragments

    float m = -INFINITY, l = 0.f;  // head gid's running max and sum (the same in its 4 lanes)
    float acc[MTL][4];
#pragma unroll
    for (int t = 0; t < MTL; ++t)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[t][i] = 0.f;
    for (int k = 0; k < mine; ++k) {
        asm volatile("cp.async.wait_group %0;" ::"n"(TW_NST - 2) : "memory");
        __syncwarp();  // every lane's copies of chunk k landed; chunk k - 1's slot is free
        if (k + TW_NST - 1 < mine) load_chunk(k + TW_NST - 1);
        asm volatile("cp.async.commit_group;" ::: "memory");
        const __half* ck = ring + (k % TW_NST) * CHW;
        const __half* cv = ck + 8 * LD;
        const int pos0 = p0 + 8 * (warp + TA_NW * k);
        // scores: lane l addresses row (l & 7) of matrix l >> 3 (8 head dims each)
        float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int st = 0; st < KS; st += 2) {
            uint32_t b0, b1, b2, b3;
            ldsm_x4(smem_u32(ck + (lane & 7) * LD + st * 16 + (lane >> 3) * 8), b0, b1, b2, b3);
            const uint4 f0 = qf[st * 32 + lane], f1 = qf[(st + 1) * 32 + lane];
            mma_f16(c, f0.x, 0u, f0.y, 0u, b0, b1);
            mma_f16(c, f0.z, 0u, f0.w, 0u, b0, b1);
            mma_f16(c, f1.x, 0u, f1.y, 0u, b2, b3);
            mma_f16(c, f1.z, 0u, f1.w, 0u, b2, b3);
        }
        // online softmax of head gid over the chunk's positions 2 tig, 2 tig + 1
        const float s0 = pos0 + 2 * tig < p1 ? c[0] : -INFINITY, s1 = pos0 + 2 * tig + 1 < p1 ? c[1] : -INFINITY;
        float mc = fmaxf(s0, s1);
        mc = fmaxf(mc, __shfl_xor_sync(JINF_FULL_MASK, mc, 1));
        mc = fmaxf(mc, __shfl_xor_sync(JINF_FULL_MASK, mc, 2));
        const float mn = fmaxf(m, mc);  // finite: a chunk holds at least one position
        const float corr = m == -INFINITY ? 0.f : expf(m - mn);
        float e0 = expf(s0 - mn), e1 = expf(s1 - mn);
        if (gid >= GQ) e0 = e1 = 0.f;
        float es = e0 + e1;
        es += __shfl_xor_sync(JINF_FULL_MASK, es, 1);
        es += __shfl_xor_sync(JINF_FULL_MASK, es, 2);
        l = fmaf(l, corr, es);
        m = mn;
        uint32_t ph, pl;
        split_h2(e0, e1, ph, pl);
        // the accumulator's columns are heads 2 tig, 2 tig + 1: their corrections
        const float ca = __shfl_sync(JINF_FULL_MASK, corr, 8 * tig), cb = __shfl_sync(JINF_FULL_MASK, corr, 8 * tig + 4);
#pragma unroll
        for (int t = 0; t < MTL; t += 2) {
            // V^T fragments of head dims 16 t .. 16 t + 31: matrix l >> 3 covers dims 8 (l >> 3) ..
            uint32_t a0, a1, a2, a3;
            ldsm_x4_t(smem_u32(cv + (lane & 7) * LD + t * 16 + (lane >> 3) * 8), a0, a1, a2, a3);
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                float (&o)[4] = acc[t + u];
                o[0] *= ca;
                o[1] *= cb;
                o[2] *= ca;
                o[3] *= cb;
                mma_f16_k8(o, u ? a2 : a0, u ? a3 : a1, ph);
                mma_f16_k8(o, u ? a2 : a0, u ? a3 : a1, pl);
            }
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");  // the trailing groups are empty
    __syncthreads();  // every warp is done with its ring: the merge reuses them
    // per warp: m, l of each head, and its accumulator [GQ][HD], then merged in warp order
    float* wacc = reinterpret_cast<float*>(sm);                            // [TA_NW][GQ][HD]
    float* wml = reinterpret_cast<float*>(sm) + (size_t)TA_NW * GQ * HD;   // [TA_NW][GQ][2]
    if (tig == 0 && gid < GQ) {
        wml[(warp * GQ + gid) * 2] = m;
        wml[(warp * GQ + gid) * 2 + 1] = l;
    }
#pragma unroll
    for (int t = 0; t < MTL; ++t)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int g = 2 * tig + (i & 1), d = 16 * t + gid + 8 * (i >> 1);
            if (g < GQ) wacc[((size_t)warp * GQ + g) * HD + d] = acc[t][i];
        }
    __syncthreads();
    for (int o = tid; o < GQ * HD; o += TA_THREADS) {
        const int g = o / HD, dd = o % HD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < TA_NW; ++w) M = fmaxf(M, wml[(w * GQ + g) * 2]);
        float a = 0.f, L = 0.f;
#pragma unroll
        for (int w = 0; w < TA_NW; ++w) {
            const float mw = wml[(w * GQ + g) * 2];
            const float f = mw == -INFINITY ? 0.f : expf(mw - M);
            a = fmaf(f, wacc[((size_t)w * GQ + g) * HD + dd], a);
            L = fmaf(f, wml[(w * GQ + g) * 2 + 1], L);
        }
        part[g * (HD + 2) + dd] = a;
        if (dd == 0) {
            part[g * (HD + 2) + HD] = p1 > p0 ? M : -INFINITY;  // an empty split
            part[g * (HD + 2) + HD + 1] = L;
        }
    }
}

template <int HD, int GQ>
__global__ void __launch_bounds__(TA_THREADS, 2) k_attn_multi(const MultiAttnParams p) {
    extern __shared__ __align__(16) uint8_t smem_a[];
    __shared__ int is_last;
    const int tid = threadIdx.x;
    const int G = (int)gridDim.x / p.n_kv_heads;  // CTAs per (vector, kv head)
    const int v = blockIdx.y, kvh = blockIdx.x / G, sp = blockIdx.x % G;
    pdl_wait();
    pdl_trigger();
    const int n_pos = p.ms->pos[v] + 1;
    const int S = min(G, (n_pos + TA_BLK - 1) / TA_BLK);  // splits with positions
    const size_t pst = (size_t)GQ * (HD + 2);
    float* pbase = p.part + ((size_t)v * p.n_kv_heads + kvh) * p.s_max * pst;
    if (sp < S) {
        const int per = (n_pos + S - 1) / S;
        const int p0 = min(n_pos, sp * per), p1 = min(n_pos, p0 + per);
        const size_t so = (size_t)p.ms->seq[v] * p.seq_stride + (size_t)kvh * p.max_ctx * HD;
        attn_split_w<HD, GQ>(p.q + (size_t)v * p.q_stride + (size_t)kvh * GQ * HD, p.kcache + so, p.vcache + so, p0,
                              p1, smem_a, pbase + (size_t)sp * pst);
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const unsigned prev = atomicAdd(&p.ms->attn_count[v * MULTI_MAX_KV_HEADS + kvh], 1u);
        is_last = prev == (unsigned)(G - 1);
        if (is_last) p.ms->attn_count[v * MULTI_MAX_KV_HEADS + kvh] = 0u;  // ready for the next launch
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    // merge the S splits in order: every split's (m, l) of every head in one pass of loads, the
    // weights f_s = exp(m_s - M) and L = sum f_s l_s, then the outputs, eight splits' loads in
    // flight per thread
    float* fw = reinterpret_cast<float*>(smem_a);  // [GQ][S] m_s, then the weights
    float* fl = fw + GQ * S;                        // [GQ][S] l_s
    float* ls = fl + GQ * S;                        // [GQ] L
    for (int i = tid; i < GQ * S; i += TA_THREADS) {
        const int g = i / S, s2 = i % S;
        fw[i] = __ldcg(pbase + (size_t)s2 * pst + g * (HD + 2) + HD);
        fl[i] = __ldcg(pbase + (size_t)s2 * pst + g * (HD + 2) + HD + 1);
    }
    __syncthreads();
    if (tid < GQ) {
        float M = -INFINITY;
        for (int s2 = 0; s2 < S; ++s2) M = fmaxf(M, fw[tid * S + s2]);
        float L = 0.f;
        for (int s2 = 0; s2 < S; ++s2) {
            const float ms = fw[tid * S + s2];
            const float f = ms == -INFINITY ? 0.f : expf(ms - M);
            fw[tid * S + s2] = f;
            L = fmaf(fl[tid * S + s2], f, L);
        }
        ls[tid] = L;
    }
    __syncthreads();
    for (int o = tid; o < GQ * HD / 2; o += TA_THREADS) {
        const int g = o / (HD / 2), d2 = o % (HD / 2);
        float2 a = make_float2(0.f, 0.f);
        for (int s0 = 0; s0 < S; s0 += 8) {
            float2 t[8];
#pragma unroll
            for (int k = 0; k < 8; ++k)
                t[k] = s0 + k < S ? __ldcg(reinterpret_cast<const float2*>(pbase + (size_t)(s0 + k) * pst + g * (HD + 2)) + d2)
                                  : make_float2(0.f, 0.f);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float f = s0 + k < S ? fw[g * S + s0 + k] : 0.f;
                a.x = fmaf(t[k].x, f, a.x);
                a.y = fmaf(t[k].y, f, a.y);
            }
        }
        const float L = ls[g];
        const float ox = a.x / L, oy = a.y / L;
        *reinterpret_cast<float2*>(p.out + (size_t)v * p.q_stride + (size_t)(kvh * GQ + g) * HD + 2 * d2) =
            make_float2(ox, oy);
        if (p.rec) {
            // a warp holds 64 consecutive outputs (GQ * HD / 2 is a multiple of 32, so whole warps
            // take each pass), lane l elements 2l, 2l + 1: blocks 2w and 2w + 1, octet lane L of
            // lanes 0..7 and 8..15 takes elements 4L .. 4L+3 of its block
            const int lane = tid & 31, hh = (lane >> 3) & 1, src = 16 * hh + 2 * (lane & 7);
            const float4 e = make_float4(__shfl_sync(JINF_FULL_MASK, ox, src), __shfl_sync(JINF_FULL_MASK, oy, src),
                                         __shfl_sync(JINF_FULL_MASK, ox, src + 1), __shfl_sync(JINF_FULL_MASK, oy, src + 1));
            const int G = p.q_stride / Q4M_KG;
            const int blk = (kvh * GQ * HD + 2 * (o - lane)) / 32 + hh;
            uint8_t* base = p.rec + (size_t)v * xrec_bytes(G);
            octet_to_records(e, lane, blk & 3, reinterpret_cast<uint32_t*>(base) + (blk >> 2) * 64,
                             reinterpret_cast<float4*>(base + (size_t)G * 256) + (blk >> 2) * 4, lane < 16);
        }
    }
}

template <int HD, int GQ>
cudaError_t launch_attn_multi(const MultiAttnParams& p0, cudaStream_t s, bool pdl) {
    // the split's scratch (attn_split_w) or the merge's (2 x group x s_max + group floats)
    const size_t merge = sizeof(float) * ((size_t)2 * GQ * 64 + GQ);
    const size_t smem = (std::max(tw_smem<HD>(), merge) + 15) & ~(size_t)15;
    static int per_sm[64] = {0};  // resident CTAs per SM, per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!per_sm[dev]) {
        cudaError_t e = cudaFuncSetAttribute(k_attn_multi<HD, GQ>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        int k = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&k, k_attn_multi<HD, GQ>, TA_THREADS, smem);
        if (e != cudaSuccess) return e;
        per_sm[dev] = k > 0 ? k : 1;
    }
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const MultiAttnParams& p = p0;
    const int G = std::max(1, std::min(p.s_max, per_sm[dev] * sms / (p.n * p.n_kv_heads)));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(p.n_kv_heads * G), (unsigned)p.n);
    cfg.blockDim = dim3(TA_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_attn_multi<HD, GQ>, p);
}

}  // namespace

size_t multi_attn_part_floats(int n, int n_kv_heads, int s_max, int head_dim) {
    return (size_t)n * n_kv_heads * s_max * ATTN_MAX_GROUP * (head_dim + 2);
}

cudaError_t multi_attn_launch(const MultiAttnParams& p, cudaStream_t s, bool pdl) {
    if (!p.q || !p.kcache || !p.vcache || !p.out || !p.part || !p.ms || p.n < 1 || p.n > MULTI_MAX ||
        p.n_kv_heads < 1 || p.n_kv_heads > MULTI_MAX_KV_HEADS || p.n_heads % p.n_kv_heads || p.s_max < 1 ||
        p.s_max > 64)
        return cudaErrorInvalidValue;
    if (p.rec && (p.q_stride % Q4M_KG || p.q_stride < p.n_heads * p.head_dim)) return cudaErrorInvalidValue;
    const int gq = p.n_heads / p.n_kv_heads;
    if (p.head_dim == 64) {
        if (gq == 8) return launch_attn_multi<64, 8>(p, s, pdl);
        if (gq == 4) return launch_attn_multi<64, 4>(p, s, pdl);
        if (gq == 2) return launch_attn_multi<64, 2>(p, s, pdl);
        if (gq == 1) return launch_attn_multi<64, 1>(p, s, pdl);
    } else if (p.head_dim == 128) {
        if (gq == 8) return launch_attn_multi<128, 8>(p, s, pdl);
        if (gq == 4) return launch_attn_multi<128, 4>(p, s, pdl);
        if (gq == 2) return launch_attn_multi<128, 2>(p, s, pdl);
        if (gq == 1) return launch_attn_multi<128, 1>(p, s, pdl);
    }
    return cudaErrorInvalidValue;
}

cudaError_t step_launch(const StepParams& p, int grid, cudaStream_t s) {
    const size_t smem = step_smem_bytes(p.xstage_bytes, p.n_phases, p.fmt, p.nbuf);
    const bool tp = p.tp_size > 1;
    cudaError_t e = step_configure(smem, p.fmt, p.nbuf, tp);
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
    return cudaLaunchKernelEx(&cfg, step_kernel_for(p.fmt, p.nbuf, tp), p);
}

}  // namespace jinf
