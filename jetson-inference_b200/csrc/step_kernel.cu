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


// ---------------------------------------------------------------- flagged words
//
// Every tensor one phase hands to another travels as 8-byte words {value bits, flag}
// (step.h: step_flag). The producer stores them with plain stores and no fence; the
// consumer loads them and reloads the words whose flag is not yet the expected one, at
// most `limit` times (then DEV_ERR_TIMEOUT is recorded and the step is discarded). It also
// gives up as soon as another CTA has recorded an error, so a failed step ends quickly.
typedef unsigned long long u64w;

__device__ __forceinline__ u64w fword(float v, uint32_t flag) { return ((u64w)flag << 32) | __float_as_uint(v); }
__device__ __forceinline__ u64w fword_u(uint32_t v, uint32_t flag) { return ((u64w)flag << 32) | v; }
__device__ __forceinline__ void st_w(u64w* p, u64w w) {
    asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ u64w ld_w(const u64w* p) {
    u64w v;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ float fval(u64w w) { return __uint_as_float((uint32_t)w); }
__device__ __forceinline__ bool fw_ok(u64w w, uint32_t flag) { return (uint32_t)(w >> 32) == flag; }

__device__ __noinline__ void note_timeout(DeviceState* st) { atomicCAS(&st->error, DEV_OK, DEV_ERR_TIMEOUT); }

// Reload the word at p (whose last load gave w) until it carries `flag`. The check is inline;
// the reload loop is out of line, so that a word that is already there costs no call.
__device__ __noinline__ u64w wait_word_slow(const u64w* p, u64w w, uint32_t flag, DeviceState* st,
                                            unsigned long long limit) {
    for (unsigned long long it = 0; !fw_ok(w, flag); ++it) {
        if (it >= limit || *(volatile int*)&st->error != DEV_OK) {
            note_timeout(st);
            break;
        }
        __nanosleep(32);
        w = ld_w(p);
    }
    return w;
}
__device__ __forceinline__ u64w wait_word(const u64w* p, u64w w, uint32_t flag, DeviceState* st,
                                          unsigned long long limit) {
    return fw_ok(w, flag) ? w : wait_word_slow(p, w, flag, st, limit);
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
// Reload the 16-byte aligned pair of words at p (last loaded as w) until both carry `flag`
// (inline check, out-of-line reload loop).
__device__ __noinline__ ulonglong2 wait_pair_slow(const u64w* p, ulonglong2 w, uint32_t flag, DeviceState* st,
                                                  unsigned long long limit) {
    for (unsigned long long it = 0; !ll_ok(w, flag); ++it) {
        if (it >= limit || *(volatile int*)&st->error != DEV_OK) {
            note_timeout(st);
            break;
        }
        __nanosleep(32);
        w = ld_ll2(p);
    }
    return w;
}
__device__ __forceinline__ ulonglong2 wait_pair(const u64w* p, ulonglong2 w, uint32_t flag, DeviceState* st,
                                                unsigned long long limit) {
    return ll_ok(w, flag) ? w : wait_pair_slow(p, w, flag, st, limit);
}

// Stream geometry of one phase, kept in shared memory (groups == 0: no weights).
struct PhaseInfo {
    const uint8_t* w;
    int pairs, groups, gran;
    int fmts;  // StepPhase::fmts
};

// Unit range [c0, c1) of warp `warp` of CTA `cta` (of C) in a pairs x groups matrix: the
// CTA's equal share of the T * G units, split evenly over its warps (32-bit: a matrix has far
// fewer than 2^31 units).
__device__ __forceinline__ void warp_range(int cta, int C, int warp, int T, int G, int& c0, int& c1) {
    const int U = T * G, u0 = step_cta_unit(cta, C, U), n = step_cta_unit(cta + 1, C, U) - u0;
    c0 = u0 + ((warp * n) >> 4);
    c1 = u0 + (((warp + 1) * n) >> 4);
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
        warp_range(cta, C, warp, pinfo[i].pairs, G, c0, c1);
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
    const int U = pi.pairs * pi.groups, u0 = step_cta_unit(cta, C, U), u1 = step_cta_unit(cta + 1, C, U);
    if (u0 >= u1) return;
    // byte offset of unit u: mixed matrices hold the pairs below the split in format fa
    auto off = [&](int u) -> size_t {
        if (!mixed) return (size_t)u * ub;
        const int cs = (pi.fmts >> 8) * pi.groups;
        const size_t ua = q4m_unit_bytes(pi.fmts & 15), uw = q4m_unit_bytes((pi.fmts >> 4) & 15);
        return u <= cs ? (size_t)u * ua : (size_t)cs * ua + (size_t)(u - cs) * uw;
    };
    const size_t o0 = off(u0), o1 = off(u1);
    const uint8_t* b = pi.w + o0;
    const uint32_t bytes = (uint32_t)(o1 - o0);  // multiple of 16
    for (uint32_t off2 = 0; off2 < bytes; off2 += (1u << 20))
        prefetch_l2(b + off2, bytes - off2 < (1u << 20) ? bytes - off2 : (1u << 20));
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

// ---------------------------------------------------------------- RMSNorm inputs
//
// A GEMV input that is RMSNorm(h) * gain is staged by every CTA from the flagged words of h:
// the records hold h * gain and the returned factor is 1 / sqrt(mean(h^2) + eps), which the
// epilogue applies (W (h g r) = r W (h g)). Each warp converts whole groups of 128 columns
// (lane: elements 4 (g * 32 + lane) .. +3); a warp issues the loads of all its groups before
// its first wait, so it pays one round trip, not one per group. Ends with the CTA synchronised.
constexpr int STAGE_BG = 4;  // groups per warp in one batch of loads

// h from the flagged words fh (flag `flag`).
__device__ __noinline__ float stage_x_flag(const u64w* fh, uint32_t flag, const float* norm_w, float eps, int cols,
                                           uint8_t* rec, float* misc, DeviceState* st, unsigned long long limit) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = (cols + Q4M_KG - 1) / Q4M_KG, n4 = cols / 4;
    uint32_t* dig = reinterpret_cast<uint32_t*>(rec);
    float4* prm = reinterpret_cast<float4*>(rec + (size_t)G * 256);
    float ss = 0.f;
    for (int g0 = warp; g0 < G; g0 += NW * STAGE_BG) {
        ulonglong2 wa[STAGE_BG], wb[STAGE_BG];
        float4 gn[STAGE_BG];
#pragma unroll
        for (int k = 0; k < STAGE_BG; ++k) {
            const int i = (g0 + k * NW) * 32 + lane;
            if (g0 + k * NW < G && i < n4) {
                wa[k] = ld_ll2(fh + 4 * (size_t)i);
                wb[k] = ld_ll2(fh + 4 * (size_t)i + 2);
                gn[k] = reinterpret_cast<const float4*>(norm_w)[i];
            }
        }
#pragma unroll
        for (int k = 0; k < STAGE_BG; ++k) {
            const int g = g0 + k * NW;
            if (g >= G) break;
            const int i = g * 32 + lane;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (i < n4) {
                wa[k] = wait_pair(fh + 4 * (size_t)i, wa[k], flag, st, limit);
                wb[k] = wait_pair(fh + 4 * (size_t)i + 2, wb[k], flag, st, limit);
                const float4 h = make_float4(fval(wa[k].x), fval(wa[k].y), fval(wb[k].x), fval(wb[k].y));
                ss = fmaf(h.x, h.x, ss);
                ss = fmaf(h.y, h.y, ss);
                ss = fmaf(h.z, h.z, ss);
                ss = fmaf(h.w, h.w, ss);
                v = make_float4(h.x * gn[k].x, h.y * gn[k].y, h.z * gn[k].z, h.w * gn[k].w);
            }
            octet_to_records(v, lane, lane >> 3, dig + g * 64, prm + g * 4);
        }
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

// Tensor parallel: h = (the flagged h words fres, flag `flag_res`) + the ranks' partial rows
// of exchange point `point`, added in rank order (every rank adds the same words in the same
// order, so every rank holds the same h). A lane loads its 4 elements of up to 4 ranks at a
// time and reloads the words whose flag is not yet this step's exchange flag `xflag`.
// `base`: rank 0's slot of the point in this rank's area; `rs`: words from one slot to the
// next. `fhout` (may be null): where this CTA stores h (flag `flag_out`).
__device__ __noinline__ float stage_x_tp(const unsigned long long* base, size_t rs, int nranks, float eps,
                                         unsigned long long limit, const u64w* fres, uint32_t flag_res,
                                         u64w* fhout, uint32_t flag_out, const float* norm_w, int cols, uint32_t xflag,
                                         uint8_t* rec, float* misc, DeviceState* st) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = (cols + Q4M_KG - 1) / Q4M_KG, n4 = cols / 4;
    uint32_t* dig = reinterpret_cast<uint32_t*>(rec);
    float4* prm = reinterpret_cast<float4*>(rec + (size_t)G * 256);
    float ss = 0.f;
    for (int g = warp; g < G; g += NW) {
        const int i = g * 32 + lane;  // 16-byte piece of h: elements 4i .. 4i + 3
        float4 h = make_float4(0.f, 0.f, 0.f, 0.f), gn = h;
        if (i < n4) {
            ulonglong2 ha = ld_ll2(fres + 4 * (size_t)i), hb = ld_ll2(fres + 4 * (size_t)i + 2);
            gn = reinterpret_cast<const float4*>(norm_w)[i];
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
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
                    w[k][0] = wait_pair(p, w[k][0], xflag, st, limit);
                    w[k][1] = wait_pair(p + 2, w[k][1], xflag, st, limit);
                    acc.x += fval(w[k][0].x);
                    acc.y += fval(w[k][0].y);
                    acc.z += fval(w[k][1].x);
                    acc.w += fval(w[k][1].y);
                }
            }
            ha = wait_pair(fres + 4 * (size_t)i, ha, flag_res, st, limit);
            hb = wait_pair(fres + 4 * (size_t)i + 2, hb, flag_res, st, limit);
            h = make_float4(fval(ha.x) + acc.x, fval(ha.y) + acc.y, fval(hb.x) + acc.z, fval(hb.y) + acc.w);
            if (fhout) {
                st_ll2(fhout + 4 * (size_t)i, fword(h.x, flag_out), fword(h.y, flag_out));
                st_ll2(fhout + 4 * (size_t)i + 2, fword(h.z, flag_out), fword(h.w, flag_out));
            }
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
// A GEMV phase whose input was produced earlier in the step (the attention output, the FFN
// activation) receives it as digit records (q4m_device.cuh) written by the producing phase,
// as flagged words in the record layout (xrec_bytes(G) / 4 of them): its CTAs only copy them
// into shared memory instead of each converting the whole input.

// Block of word pair k of a G-group record buffer: pair k holds digit words 2k, 2k + 1
// (block 4 (2k / 64) + (2k % 64) / 16) while 2k < 64 G, then param words (block
// 4 (i / 16) + (i % 16) / 4, i = 2k - 64 G).
__device__ __forceinline__ int rec_pair_block(int k, int G) {
    const int w = 2 * k;
    if (w < 64 * G) return 4 * (w >> 6) + ((w & 63) >> 4);
    const int i = w - 64 * G;
    return 4 * (i >> 4) + ((i & 15) >> 2);
}

// Copy the records of G groups (nb real 32-element blocks; the padding blocks of the last
// group are never written and get zero records) from the flagged words fr into shared
// memory; every thread issues up to 8 pair loads before its first wait. Ends with the CTA
// synchronised.
__device__ __noinline__ void stage_records_flag(const u64w* fr, uint32_t flag, int G, int nb, uint8_t* xbase,
                                                DeviceState* st, unsigned long long limit) {
    constexpr int B = 8;
    const int n2 = G * 40;  // 16-byte pairs of words
    uint2* dst = reinterpret_cast<uint2*>(xbase);
    for (int k0 = threadIdx.x; k0 < n2; k0 += STEP_THREADS * B) {
        ulonglong2 w[B];
#pragma unroll
        for (int b = 0; b < B; ++b) {
            const int k = k0 + b * STEP_THREADS;
            if (k < n2 && rec_pair_block(k, G) < nb) w[b] = ld_ll2(fr + 2 * (size_t)k);
        }
#pragma unroll
        for (int b = 0; b < B; ++b) {
            const int k = k0 + b * STEP_THREADS;
            if (k < n2) {
                if (rec_pair_block(k, G) < nb) {
                    w[b] = wait_pair(fr + 2 * (size_t)k, w[b], flag, st, limit);
                    dst[k] = make_uint2((uint32_t)w[b].x, (uint32_t)w[b].y);
                } else {
                    dst[k] = make_uint2(0u, 0u);
                }
            }
        }
    }
    __syncthreads();
}

// Records of one 32-element block held by an octet of lanes (octet_digits), as flagged words:
// `fdig` is the group's 64 digit words and `fprm` its 16 param words in a record buffer of
// flagged words, j the block within the group. All 32 lanes call it; octets with `store` write.
__device__ __forceinline__ void octet_to_records_flag(float4 v, int lane, int j, u64w* fdig, u64w* fprm, uint32_t flag,
                                                      bool store) {
    const int q = lane & 7;
    const OctetDigits o = octet_digits(v);
    if (!store) return;
    st_w(fdig + rec_word_hi(j, q), fword_u(o.H, flag));
    st_w(fdig + rec_word_lo(j, q), fword_u(o.L, flag));
    if (q == 0) {
        const float ia = o.amax / XREC_DIGIT_MAX;
        st_ll2(fprm + 4 * j, fword_u((uint32_t)(-8 * o.sh), flag), fword_u((uint32_t)(-8 * o.sl), flag));
        st_ll2(fprm + 4 * j + 2, fword(ia, flag), fword(ia * 0.0625f, flag));
    }
}

// Flagged records of blocks [b0, b0 + nb) of the next input from fp32 values in shared memory
// (vals[32 * i] = first element of block b0 + i), by the whole CTA (4 blocks per warp pass).
// `fout`: the record buffer of a `groups_out`-group input.
__device__ __noinline__ void blocks_to_records_flag(const float* vals, int b0, int nb, int groups_out, u64w* fout,
                                                    uint32_t flag) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    u64w* fdig = fout;
    u64w* fprm = fout + (size_t)groups_out * 64;
    for (int i0 = warp * 4; i0 < nb; i0 += NW * 4) {
        const int i = i0 + (lane >> 3);
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i < nb) v = reinterpret_cast<const float4*>(vals + 32 * i)[lane & 7];
        const int blk = b0 + i;
        octet_to_records_flag(v, lane, blk & 3, fdig + (size_t)(blk >> 2) * 64, fprm + (size_t)(blk >> 2) * 16, flag,
                              i < nb);
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
// of a block is issued before any arithmetic, and an online softmax joins the blocks. The
// rows of earlier positions are in the cache since earlier steps; the row of the step's own
// position comes from the QKV phase's flagged words, and so does q.

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
    // the lane's dims of the step's own row: flagged words fw (two halves per word)
    __device__ __forceinline__ void load_flag(const u64w* fw, uint32_t flag, DeviceState* st, unsigned long long lim) {
        const ulonglong2 w = wait_pair(fw, ld_ll2(fw), flag, st, lim);
        r = make_uint2((uint32_t)w.x, (uint32_t)w.y);
    }
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
    __device__ __forceinline__ void load_flag(const u64w* fw, uint32_t flag, DeviceState* st, unsigned long long lim) {
        r = (uint32_t)wait_word(fw, ld_w(fw), flag, st, lim);
    }
    __device__ __forceinline__ void zero() { r = 0u; }
    __device__ __forceinline__ float get(int d) const {
        const __half2 h = *reinterpret_cast<const __half2*>(&r);
        return d ? __high2float(h) : __low2float(h);
    }
};

// The flagged inputs of one kv head's attention: q of its GQ heads and the K and V rows of the
// step's own position `pos` (the flag of the QKV phase).
struct AttnIn {
    const u64w* fq;  // [GQ][HD] q words of the kv head
    const u64w* fk;  // [HD / 2] K words of position pos
    const u64w* fv;  // [HD / 2] V words
    uint32_t flag;
    int pos;
    DeviceState* st;
    unsigned long long limit;
};

// One CTA's split [p0, p1) of kv head attention: cache rows at kb / vb (earlier positions)
// and the flagged inputs `in`. Leaves either the normalised output in `outs` ([GQ][HD],
// shared memory; `part` null) or the split's partial (acc, m, l) as flagged words (flag
// `pflag`) in `part` ([GQ][HD + 2]). Shared scratch at `xbase`: step_xstage_bytes covers it.
template <int HD, int GQ>
__device__ __noinline__ void attn_split(const AttnIn in, const __half* kb, const __half* vb, int p0, int p1,
                                        uint8_t* xbase, u64w* part, uint32_t pflag, float* outs) {
    constexpr int VD = HD / 32;                               // head dims per lane
    constexpr int PW = GQ * VD >= 32 ? ATTN_PW / 2 : ATTN_PW;  // positions per warp and block (registers)
    constexpr int BLK = NW * PW;                              // positions per block
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float* w_s = reinterpret_cast<float*>(xbase);  // [GQ][BLK] scores, then softmax weights
    float* ml_s = w_s + GQ * BLK;                   // [GQ][4]: m, l, correction
    float* red_s = ml_s + 4 * ATTN_MAX_GROUP;       // [NW][GQ][HD] per-warp p.v sums
    const float scale = rsqrtf((float)HD);
    // the first block's cache rows are requested before q is awaited
    HalfVec<VD> kr[PW], vr[PW];
    auto load_rows = [&](int b0, int n) {
#pragma unroll
        for (int k = 0; k < PW; ++k) {
            const int j = warp + NW * k;
            if (j < n && b0 + j != in.pos) {
                kr[k].load(kb + (size_t)(b0 + j) * HD + lane * VD);
                vr[k].load(vb + (size_t)(b0 + j) * HD + lane * VD);
            } else {
                kr[k].zero();
                vr[k].zero();
            }
        }
#pragma unroll
        for (int k = 0; k < PW; ++k) {
            const int j = warp + NW * k;
            if (j < n && b0 + j == in.pos) {
                kr[k].load_flag(in.fk + lane * VD / 2, in.flag, in.st, in.limit);
                vr[k].load_flag(in.fv + lane * VD / 2, in.flag, in.st, in.limit);
            }
        }
    };
    if (p0 < p1) load_rows(p0, min(BLK, p1 - p0));
    float qr[GQ][VD];
#pragma unroll
    for (int g = 0; g < GQ; ++g) {
        const u64w* fq = in.fq + (size_t)g * HD + lane * VD;
        if constexpr (VD == 4) {
            const ulonglong2 a = wait_pair(fq, ld_ll2(fq), in.flag, in.st, in.limit);
            const ulonglong2 b = wait_pair(fq + 2, ld_ll2(fq + 2), in.flag, in.st, in.limit);
            qr[g][0] = fval(a.x) * scale; qr[g][1] = fval(a.y) * scale; qr[g][2] = fval(b.x) * scale; qr[g][3] = fval(b.y) * scale;
        } else {
            const ulonglong2 a = wait_pair(fq, ld_ll2(fq), in.flag, in.st, in.limit);
            qr[g][0] = fval(a.x) * scale; qr[g][1] = fval(a.y) * scale;
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
    for (int b0 = p0; b0 < p1; b0 += BLK) {
        const int n = min(BLK, p1 - b0);
        if (b0 != p0) load_rows(b0, n);
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
            st_w(part + g * (HD + 2) + dd, fword(a, pflag));
            if (dd == 0)
                st_ll2(part + g * (HD + 2) + HD, fword(p1 > p0 ? ml_s[g * 4] : -INFINITY, pflag),  // an empty split
                       fword(ml_s[g * 4 + 1], pflag));
        } else {
            outs[o] = a / ml_s[g * 4 + 1];
        }
    }
}

// ---------------------------------------------------------------- phase pieces (out of line:
// each gets a register allocation of its own, and the kernel's loop keeps a small live state)

// Attention phase of one CTA: its split (kv head, positions) of the context, then, for the
// splits that own output blocks (split sp owns blocks sp, sp + S, ...), the merge of each of
// their blocks from all S partials of the kv head, in split order (deterministic), written as
// records of the o phase's input.
__device__ __noinline__ void attn_phase(const StepParams& P, const StepPhase& d, int pos, uint32_t fl_in,
                                        uint32_t fl_out, uint8_t* xbase, float* outs_s) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    DeviceState* st = P.st;
    AttnGeom a;
    if (!attn_geom(pos, P.n_kv_heads, P.attn_smax, blockIdx.x, a)) return;
    const int hd = P.head_dim, gq = P.n_heads / P.n_kv_heads;
    AttnIn in;
    in.fq = d.fin + (size_t)a.kvh * gq * hd;
    in.fk = d.fkv + (size_t)a.kvh * (hd / 2);
    in.fv = d.fkv + (size_t)P.nk / 2 + (size_t)a.kvh * (hd / 2);
    in.flag = fl_in;
    in.pos = pos;
    in.st = st;
    in.limit = P.spin_limit;
    const __half* kb = d.kcache + (size_t)a.kvh * P.max_ctx * hd;
    const __half* vb = d.vcache + (size_t)a.kvh * P.max_ctx * hd;
    const size_t stride = (size_t)ATTN_MAX_GROUP * (hd + 2);  // words per split
    u64w* gpart = a.S > 1 ? P.attn_part + ((size_t)a.kvh * ATTN_MAX_SPLIT + a.sp) * stride : nullptr;
#define JINF_ATTN_SPLIT(HD_, GQ_) attn_split<HD_, GQ_>(in, kb, vb, a.p0, a.p1, xbase, gpart, fl_out, outs_s)
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
    const int nblk = gq * hd / 32;  // 32-element output blocks of this kv head
    if (a.S == 1) {
        __syncthreads();
        blocks_to_records_flag(outs_s, a.kvh * nblk, nblk, d.groups_out, d.fout, fl_out);
        return;
    }
    if (a.sp >= nblk) return;
    __syncthreads();  // every thread is done with the split's scratch
    const u64w* base = P.attn_part + (size_t)a.kvh * ATTN_MAX_SPLIT * stride;
    float* ml = reinterpret_cast<float*>(xbase);  // [S][2] (m, l) of the block's query head
    float* av = ml + 2 * ATTN_MAX_SPLIT;           // [S][32] accumulators of the block
    float* ew = av + 32 * ATTN_MAX_SPLIT;          // [S] split weights e^(m_s - M)
    for (int b = a.sp; b < nblk; b += a.S) {
        const int g = b * 32 / hd, dd0 = b * 32 % hd;
        {  // every partial load of the thread before any wait (S <= 64: at most 4 + 2)
            u64w t4[4], mw = 0, lw = 0;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int t = tid + k * STEP_THREADS;
                t4[k] = t < a.S * 32 ? ld_w(base + (t >> 5) * stride + g * (hd + 2) + dd0 + (t & 31)) : 0ull;
            }
            if (tid < a.S) {
                mw = ld_w(base + tid * stride + g * (hd + 2) + hd);
                lw = ld_w(base + tid * stride + g * (hd + 2) + hd + 1);
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int t = tid + k * STEP_THREADS;
                if (t < a.S * 32) {
                    const u64w* pw = base + (t >> 5) * stride + g * (hd + 2) + dd0 + (t & 31);
                    av[t] = fval(wait_word(pw, t4[k], fl_out, st, P.spin_limit));
                }
            }
            if (tid < a.S) {
                ml[2 * tid] = fval(wait_word(base + tid * stride + g * (hd + 2) + hd, mw, fl_out, st, P.spin_limit));
                ml[2 * tid + 1] = fval(wait_word(base + tid * stride + g * (hd + 2) + hd + 1, lw, fl_out, st, P.spin_limit));
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
            // octet layout: lane q < 8 takes elements 4q .. 4q+3
            const int src = 4 * (lane & 7);
            const float4 x = make_float4(__shfl_sync(JINF_FULL_MASK, v, src), __shfl_sync(JINF_FULL_MASK, v, src + 1),
                                         __shfl_sync(JINF_FULL_MASK, v, src + 2), __shfl_sync(JINF_FULL_MASK, v, src + 3));
            octet_to_records_flag(x, lane, blk & 3, d.fout + (size_t)(blk >> 2) * 64,
                                  d.fout + (size_t)d.groups_out * 64 + (size_t)(blk >> 2) * 16, fl_out, lane < 8);
        }
        __syncthreads();  // the scratch is reused by the next block
    }
}

// Epilogue inputs that do not depend on the GEMV, by the threads from 32 up while warp 0
// starts the input staging: the residual rows of an EPI_RESID phase (flagged words of the
// phase d.tag_res), the RoPE factors of an EPI_QKV phase (cosine at the even row of a q or k
// pair, sine at the odd row). Rows [prow0, prow0 + nprow) -> outs_s.
__device__ __noinline__ void prepare_epilogue(const StepParams& P, const StepPhase& d, int pos, uint32_t fepoch,
                                              int prow0, int nprow, float* outs_s) {
    const int tid = threadIdx.x;
    if (d.epi == EPI_RESID) {
        const uint32_t fl_res = step_flag(fepoch, d.tag_res);
        for (int i = tid - 32; i < nprow; i += STEP_THREADS - 32) {
            const int row = prow0 + i;
            outs_s[i] = row < d.rows ? fval(wait_word(d.fres + row, ld_w(d.fres + row), fl_res, P.st, P.spin_limit)) : 0.f;
        }
    } else {
        for (int i = tid - 32; i < nprow; i += STEP_THREADS - 32) {
            const int row = prow0 + i;
            if ((i & 1) == 0 && row < P.nq + P.nk) {
                float cs, sn;
                rope_pair(row < P.nq ? row : row - P.nq, pos, P.rope_base, P.head_dim, cs, sn);
                outs_s[i] = cs;
                outs_s[i + 1] = sn;
            }
        }
    }
}

// The embedding row as flagged h words (the residual stream the first o phase adds to).
__device__ __noinline__ void store_h_flag(const float* emb, int cols, u64w* fout_h, uint32_t flag) {
    for (int i = threadIdx.x; i < cols / 2; i += STEP_THREADS) {
        const float2 e = reinterpret_cast<const float2*>(emb)[i];
        st_ll2(fout_h + 2 * (size_t)i, fword(e.x, flag), fword(e.y, flag));
    }
}

// Tensor-parallel RMSNorm input: the h of phase d.tag_res plus the ranks' partials of exchange
// point d.xin; the CTA that owns pair 0 stores the new h (flag fl_out).
__device__ __noinline__ float stage_tp(const StepParams& P, const StepPhase& d, int t0, uint32_t fepoch,
                                       uint32_t fl_out, uint8_t* xbase, float* misc) {
    const unsigned long long ep = *(volatile unsigned long long*)P.xpeer[P.tp_rank];
    return stage_x_tp(xchg_data(P, P.tp_rank, d.xin, (unsigned)(ep & 1ull), 0), (size_t)(P.x_slot / 8), P.tp_size,
                      P.eps, P.spin_limit, d.fres, step_flag(fepoch, d.tag_res), t0 == 0 ? d.fout_h : nullptr, fl_out,
                      d.norm_w, d.cols, (uint32_t)(ep + 1ull), xbase, misc, P.st);
}

// What a finished tile pair's epilogue needs besides the phase.
struct EpiCtx {
    float fac;        // 1 / rms of a normalised input, else 1
    int pos;
    uint32_t fepoch;  // the step's flag epoch
    uint32_t fl_out;  // flag of this phase's words
    int t0, prow0;    // the CTA's first pair and its first row
    bool pre;         // the epilogue inputs were prepared into outs_s (prepare_epilogue)
};

// The running argmax of the LM-head rows this warp finished.
struct ArgMax {
    float v;
    int i;
};

// The epilogue of a finished pair, by a whole warp: lanes q < 16 hold rows 2q, 2q + 1 (v0, v1,
// before the input's norm factor).
template <bool TP>
__device__ __noinline__ void finish_pair(const StepParams& P, const StepPhase& d, const EpiCtx& ec, int pr, float v0,
                                         float v1, float* outs_s, ArgMax& am) {
    const int lane = threadIdx.x & 31, q = lane & 15, row = pr * Q4M_PAIR_ROWS + 2 * q;
    v0 *= ec.fac;
    v1 *= ec.fac;
    if (TP && d.epi == EPI_PARTIAL) {
        // this rank's partial rows into its slot of every rank's exchange area
        if (lane < 16 && row < d.rows) {  // (rows: a multiple of 32)
            const unsigned long long ep = *(volatile unsigned long long*)P.xpeer[P.tp_rank];
            const uint32_t flag = (uint32_t)(ep + 1ull);
            const unsigned long long w0 = ll_word(v0, flag), w1 = ll_word(v1, flag);
            for (int r = 0; r < P.tp_size; ++r) st_ll2(xchg_data(P, r, d.xout, (unsigned)(ep & 1ull), P.tp_rank) + row, w0, w1);
        }
        return;
    }
    if (d.epi == EPI_GATEUP) {
        // the activation goes to shared memory; whole blocks become records after the phase
        if (lane < 16) outs_s[(pr - ec.t0) * 16 + q] = row < d.rows ? v0 / (1.0f + expf(-v0)) * v1 : 0.f;
        return;
    }
    if (lane >= 16 || row >= d.rows) return;
    if (d.epi == EPI_RESID) {
        // h += W x, the reference's residual add (src/engine.cpp:470-472, 505-507)
        float h0, h1;
        if (ec.pre) {
            h0 = outs_s[row - ec.prow0];
            h1 = outs_s[row + 1 - ec.prow0];
        } else {
            const ulonglong2 w = wait_pair(d.fres + row, ld_ll2(d.fres + row), step_flag(ec.fepoch, d.tag_res), P.st,
                                           P.spin_limit);
            h0 = fval(w.x);
            h1 = fval(w.y);
        }
        st_ll2(d.fout + row, fword(h0 + v0, ec.fl_out), fword(h1 + v1, ec.fl_out));
    } else if (d.epi == EPI_QKV) {
        // RoPE on q and k (reference cuda/rope_kernel.cu); q as flagged words, K and V into the
        // fp16 cache at pos and as flagged words for this step's attention
        float o0 = v0, o1 = v1;
        if (row < P.nq + P.nk) {
            float cs, sn;
            if (ec.pre) {
                cs = outs_s[row - ec.prow0];
                sn = outs_s[row + 1 - ec.prow0];
            } else {
                rope_pair(row < P.nq ? row : row - P.nq, ec.pos, P.rope_base, P.head_dim, cs, sn);
            }
            o0 = v0 * cs - v1 * sn;
            o1 = v0 * sn + v1 * cs;
        }
        if (row < P.nq) {
            st_ll2(d.fout + row, fword(o0, ec.fl_out), fword(o1, ec.fl_out));
        } else {
            const bool isk = row < P.nq + P.nk;
            const int rr = isk ? row - P.nq : row - P.nq - P.nk;
            const int kvh = rr / P.head_dim, dd = rr % P.head_dim;
            const __half2 hv = __floats2half2_rn(o0, o1);
            *reinterpret_cast<__half2*>((isk ? d.kcache : d.vcache) + ((size_t)kvh * P.max_ctx + ec.pos) * P.head_dim + dd) =
                hv;
            st_w(d.fkv + (isk ? 0 : P.nk / 2) + rr / 2, fword_u(*reinterpret_cast<const uint32_t*>(&hv), ec.fl_out));
        }
    } else {  // EPI_LMHEAD: logits and the running argmax (first maximum)
        d.y[row] = v0;
        if (v0 > am.v) {
            am.v = v0;
            am.i = row;
        }
        if (row + 1 < d.rows) {
            d.y[row + 1] = v1;
            if (v1 > am.v) {
                am.v = v1;
                am.i = row + 1;
            }
        }
    }
}

// A tile (gran pairs) whose units this CTA shares with neighbouring CTAs, by one warp: the CTA
// that holds the tile's last unit merges it (its own rows plus the flagged partial rows the
// earlier CTAs left in their slots, added in a fixed order) and runs the epilogue; the others
// leave their rows in their slot `slot` (0: their first tile, 1: their last). own: this CTA's
// rows of the tile ([gran][32], zero where it has no units).
template <bool TP>
__device__ __noinline__ void merge_split_tile(const StepParams& P, const StepPhase& d, const EpiCtx& ec, int t, int slot,
                                              int U, int TG, const float* own, float* outs_s, ArgMax& am) {
    const int lane = threadIdx.x & 31, C = gridDim.x, cta = blockIdx.x;
    const int nr = d.gran * 32;  // rows of the tile
    const int u1 = step_cta_unit(cta + 1, C, U);
    if ((t + 1) * TG > u1) {  // not the merging CTA: leave the rows
        u64w* dst = P.split_part + ((size_t)cta * 2 + slot) * 64;
        for (int r = lane; r < nr; r += 32) st_w(dst + r, fword(own[r], ec.fl_out));
        return;
    }
    float v[2] = {0.f, 0.f};  // rows lane, lane + 32
    for (int k = 0; k < d.gran; ++k) v[k] = own[lane + 32 * k];
    for (int c = cta - 1; c >= 0; --c) {  // the earlier CTAs that hold units of the tile
        const int cu0 = step_cta_unit(c, C, U), cu1 = step_cta_unit(c + 1, C, U);
        if (cu1 <= t * TG) break;
        if (cu0 >= cu1) continue;
        const u64w* src = P.split_part + ((size_t)c * 2 + (cu0 / TG == t ? 0 : 1)) * 64;
        for (int k = 0; k < d.gran; ++k)
            v[k] += fval(wait_word(src + lane + 32 * k, ld_w(src + lane + 32 * k), ec.fl_out, P.st, P.spin_limit));
    }
    if (d.epi == EPI_GATEUP) {
        // both pairs of the activation block: neuron q of pair k from rows 2q (gate), 2q + 1 (up)
        float* acts = outs_s + 1024 - 64 + 32 * slot;  // scratch past any pair's activations
        const float g0 = __shfl_sync(JINF_FULL_MASK, v[0], (2 * lane) & 31), u0v = __shfl_sync(JINF_FULL_MASK, v[0], (2 * lane + 1) & 31);
        const float g1 = __shfl_sync(JINF_FULL_MASK, v[1], (2 * lane) & 31), u1v = __shfl_sync(JINF_FULL_MASK, v[1], (2 * lane + 1) & 31);
        const float g = (lane < 16 ? g0 : g1) * ec.fac, u = (lane < 16 ? u0v : u1v) * ec.fac;
        const int nrow = 2 * (t * 32 + lane);  // the neuron's gate row
        acts[lane] = nrow < d.rows ? g / (1.0f + expf(-g)) * u : 0.f;
        __syncwarp();
        const float4 x = reinterpret_cast<const float4*>(acts)[lane & 7];
        octet_to_records_flag(x, lane, t & 3, d.fout + (size_t)(t >> 2) * 64,
                              d.fout + (size_t)d.groups_out * 64 + (size_t)(t >> 2) * 16, ec.fl_out, lane < 8);
        return;
    }
    // gran 1: lanes q < 16 take rows 2q, 2q + 1
    const int q = lane & 15;
    const float r0 = __shfl_sync(JINF_FULL_MASK, v[0], 2 * q), r1 = __shfl_sync(JINF_FULL_MASK, v[0], 2 * q + 1);
    finish_pair<TP>(P, d, ec, t, r0, r1, outs_s, am);
}

// The last CTA to leave finishes the step: the argmax (tensor parallel: exchanged with every
// rank) becomes the next input token, the position and the flag epoch advance, the exit
// counter is cleared for the next launch.
template <bool TP>
__device__ __noinline__ void finish_step(const StepParams& P, int pos, uint32_t fepoch) {
    DeviceState* st = P.st;
    __threadfence();
    u64 b = P.with_argmax ? atomicAdd(&st->best, 0ull) : 0ull;
    const bool tp = TP && P.tp_size > 1;
    const unsigned long long ep = tp ? *(volatile unsigned long long*)P.xpeer[P.tp_rank] : 0ull;
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
    st->epoch = fepoch + 1u;
    P.done[0] = 0u;
    if (tp) *reinterpret_cast<volatile unsigned long long*>(P.xpeer[P.tp_rank]) = ep + 1ull;
}

}  // namespace

template <int FMT, int NBUF, bool TP>
__global__ void __launch_bounds__(STEP_THREADS, 1) k_step(const __grid_constant__ StepParams P) {
    constexpr int UB = q4m_unit_bytes(FMT);  // ring slot bytes (the largest unit of a mixed model)
    constexpr bool MIXED = FMT == Q4M_MIX;
    extern __shared__ __align__(16) uint8_t smem[];
    // shared memory: [xstage | misc 256 B | flags, keys, piece table 512 B | partial rows 4 KB |
    //                 outputs to convert 4 KB | phase descriptor 2 x 256 B | phase infos | rings]
    uint8_t* xbase = smem;
    float* misc = reinterpret_cast<float*>(smem + P.xstage_bytes);        // 64 floats of reductions
    int* flags = reinterpret_cast<int*>(smem + P.xstage_bytes + 256);     // [0..1] go
    u64* wkeys = reinterpret_cast<u64*>(smem + P.xstage_bytes + 256 + 64);  // [NW] argmax keys
    int* ftile = reinterpret_cast<int*>(smem + P.xstage_bytes + 256 + 192);  // [NW] tile of a warp's first piece
    int* fmid = ftile + NW;                                                  // [NW] first piece starts mid-tile
    float* part_s = reinterpret_cast<float*>(smem + P.xstage_bytes + 768);   // [NW][2][32] partial rows
    float* outs_s = reinterpret_cast<float*>(smem + P.xstage_bytes + 768 + 4096);  // [1024] outputs to convert
    float* split_s = reinterpret_cast<float*>(smem + P.xstage_bytes + 768 + 8192);   // [2 tiles][64] rows of
                                                                                     // the shared tiles
    StepPhase* dsm = reinterpret_cast<StepPhase*>(smem + P.xstage_bytes + 768 + 8192 + 512);  // [2] descriptors
    PhaseInfo* pinfo = reinterpret_cast<PhaseInfo*>(smem + P.xstage_bytes + 768 + 8192 + 1024);
    const uint32_t ring_base = smem_u32(pinfo + ((P.n_phases + 1) & ~1));
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t ring = ring_base + (uint32_t)(warp * NBUF * UB);
    const int C = gridDim.x;
    DeviceState* st = P.st;
    const int pos = *(volatile int*)&st->pos;
    // the flag epoch of this step (only the last CTA to leave advances it, after every CTA's
    // last use)
    const uint32_t fepoch = *(volatile unsigned*)&st->epoch;

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
    ArgMax am{-INFINITY, 0};
    constexpr int DWORDS = (int)(sizeof(StepPhase) / 4);
    static_assert(sizeof(StepPhase) <= 256 && sizeof(StepPhase) % 4 == 0, "descriptor slot");
    for (int ph = 0; ph < P.n_phases; ++ph) {
        StepPhase& d = dsm[ph & 1];
        JINF_TRACE(ph, 0);
        if (tid == 0) {
            flags[ph & 1] = *(volatile int*)&st->error == DEV_OK ? 1 : 0;
        } else if (tid >= 32 && tid < 32 + DWORDS) {  // descriptor -> shared memory
            reinterpret_cast<uint32_t*>(&d)[tid - 32] = reinterpret_cast<const uint32_t*>(P.phases + ph)[tid - 32];
        } else if (tid == 32 * 9) {  // L2 prefetch of later weights
            for (int k = 0; k < 2; ++k) {
                const int j = P.phases[ph].pf[k];
                if (j > ph && j < P.n_phases) prefetch_cta_range(pinfo[j], blockIdx.x, C, UB, MIXED);
            }
        }
        __syncthreads();  // also: every warp is done with the previous phase's shared data
        if (!flags[ph & 1]) break;
        JINF_TRACE(ph, 1);
        const uint32_t fl_in = step_flag(fepoch, d.tag_in), fl_out = step_flag(fepoch, ph);

        if (d.kind == PH_ATTN) {
            attn_phase(P, d, pos, fl_in, fl_out, xbase, outs_s);
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
        // this CTA's equal share [u0, u1) of the phase's units; the pairs [t0, t1) it touches; its
        // first and last tile (gran pairs), which it may share with its neighbours
        const int U = d.pairs * G, u0 = step_cta_unit(blockIdx.x, C, U), u1 = step_cta_unit(blockIdx.x + 1, C, U);
        if (u0 >= u1) continue;
        const int t0 = u0 / G, t1 = (u1 - 1) / G + 1, TG = d.gran * G;
        const int tf = u0 / TG, tl = (u1 - 1) / TG;
        const bool split_f = tf * TG < u0 || (tf + 1) * TG > u1;
        const bool split_l = tl != tf && (tl + 1) * TG > u1;
        if (tid < 128) split_s[tid] = 0.f;  // rows of a shared tile this CTA has no units of stay 0
        // Epilogue inputs that do not depend on this GEMV, prepared now by warps 1.. while
        // warp 0 starts the input staging (outs_s is free in these phases): the residual rows
        // of an EPI_RESID phase, the RoPE factors of an EPI_QKV phase. The staging ends with
        // the CTA synchronised, before any epilogue reads them.
        const int prow0 = t0 * Q4M_PAIR_ROWS, nprow = (t1 - t0) * Q4M_PAIR_ROWS;
        const bool pre = (d.epi == EPI_RESID || d.epi == EPI_QKV) && nprow <= 1024;
        if (pre && tid >= 32) prepare_epilogue(P, d, pos, fepoch, prow0, nprow, outs_s);
        float fac;
        if (d.xm == X_RECORDS) {
            stage_records_flag(d.fin, fl_in, G, d.cols / 32, xbase, st, P.spin_limit);
            fac = 1.0f;
        } else if (d.xm == X_EMBED_NORM) {
            // the embedding row; the CTA that owns pair 0 also stores it as the residual stream
            const float* emb = d.hsrc + (size_t)(*(volatile int*)&st->token) * d.cols;
            fac = stage_x<STEP_THREADS>(X_EMBED_NORM, nullptr, emb, nullptr, nullptr, false, d.norm_w, P.eps, d.cols,
                                        xbase, misc, true);
            if (t0 == 0 && d.fout_h) store_h_flag(emb, d.cols, d.fout_h, fl_out);
        } else if (TP && d.xm == X_RMSNORM_TP) {
            fac = stage_tp(P, d, t0, fepoch, fl_out, xbase, misc);
        } else {
            fac = stage_x_flag(d.fin, fl_in, d.norm_w, P.eps, d.cols, xbase, misc, st, P.spin_limit);
        }
        JINF_TRACE(ph, 2);
        const XRecS xr{smem_u32(xbase), smem_u32(xbase + (size_t)G * 256)};
        const EpiCtx ec{fac, pos, fepoch, fl_out, t0, prow0, pre};
        // a pair's rows: finished here when its tile lies inside this CTA's units, else kept in
        // shared memory for the tile's merge with the neighbouring CTAs' partial rows
        auto deliver = [&](int pr, float v0, float v1) {
            const int t = pr / d.gran;
            if (t * TG >= u0 && (t + 1) * TG <= u1) {
                finish_pair<TP>(P, d, ec, pr, v0, v1, outs_s, am);
            } else if (lane < 16) {
                float* sp = split_s + (t == tf ? 0 : 64) + (pr - t * d.gran) * 32 + 2 * (lane & 15);
                sp[0] = v0;
                sp[1] = v1;
            }
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
                deliver(pair, v0, v1);
            } else {
                // a piece of a pair shared with the neighbouring warps: partial rows to shared memory
                const int sl = first_piece ? 0 : 1;
                if (c4 == 0) {
#pragma unroll
                    for (int i = 0; i < 4; ++i) part_s[(warp * 2 + sl) * 32 + unit_row_of(i, lane)] = ps.acc[i];
                }
                if (gb == 0 || pair * G + gb == u0) {  // the piece starts the pair's units in this CTA
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
            deliver(own_pair, v0, v1);
        }
        if (split_f || split_l || d.epi == EPI_GATEUP) __syncthreads();  // split_s and outs_s are complete
        if ((warp == 0 && split_f) || (warp == 1 && split_l))
            merge_split_tile<TP>(P, d, ec, warp == 0 ? tf : tl, warp, U, TG, split_s + 64 * warp, outs_s, am);
        if (d.epi == EPI_GATEUP) {
            // tiles inside this CTA's units are whole activation blocks, their activations in
            // outs_s from pair t0 on (the shared tiles' blocks are written by their merge)
            const int b0 = (u0 + TG - 1) / TG, b1 = u1 / TG;
            if (b1 > b0) blocks_to_records_flag(outs_s + (2 * b0 - t0) * 16, b0, b1 - b0, d.groups_out, d.fout, fl_out);
        }
        JINF_TRACE(ph, 5);
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");

    // ---------------- leave: LM head argmax, then the last CTA finishes the step
    if (P.with_argmax) {
        u64 key = am.v == -INFINITY ? 0ull : argmax_key(am.v, am.i + P.vocab_off);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const u64 other = __shfl_xor_sync(JINF_FULL_MASK, key, o);
            key = other > key ? other : key;
        }
        if (lane == 0) wkeys[warp] = key;
    }
    __syncthreads();
    if (tid == 0) {
        u64 best = 0ull;
        if (P.with_argmax) {
            for (int w = 0; w < NW; ++w) best = wkeys[w] > best ? wkeys[w] : best;
            if (best) atomicMax(&st->best, best);
        }
        __threadfence();
        const unsigned old = atomicAdd(P.done, 1u);
        if (old == gridDim.x - 1) finish_step<TP>(P, pos, fepoch);
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
    return (size_t)xstage_bytes + 768 + 8192 + 1024 + infos + (size_t)NW * nbuf * q4m_unit_bytes(fmt);
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
