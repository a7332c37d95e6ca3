// Stand-alone fused Q4_0 GEMV over the Q4M layout (q4m.cuh) on the tensor cores, sm_100a;
// the arithmetic is described in q4m_device.cuh. It serves the jinf_b200_gemv_q4m* entry
// points and the engine's kernel-per-operation step (tensor parallel runs, the FFN hook).
//
//   prologue  X_PLAIN        x given (fp32 or fp16)
//             X_RMSNORM      h = h_in + y_pending; x = rmsnorm(h) * gain   (CTA 0 stores h)
//             X_EMBED_NORM   h = token_embd[token];  x = rmsnorm(h) * gain (CTA 0 stores h)
//   epilogue  EPI_STORE      y[row]
//             EPI_QKV        RoPE on q/k pairs, q -> fp32, k/v -> fp16 KV cache at pos
//             EPI_GATEUP     rows interleaved (gate_n, up_n): h[n] = silu(gate_n) * up_n
//             EPI_LMHEAD     logits[row] and a packed (value, index) atomicMax argmax
//
// Scheduling. Tasks are (tile pair, K part): a pair's groups are split over `kw` tasks so
// that every SM gets about the same work. Each warp streams its tasks' units through a
// private cp.async ring (gemvm_nbuf(fmt) - 1 units in flight) that runs ahead
// across task boundaries; the first units are requested before the kernel waits on its
// producer (programmatic dependent launch), because weights never depend on it. With kw > 1
// each task writes its 32 partial sums to a workspace and the last task of a pair (arrival
// counter, reset by that task) adds them in K order, so results are deterministic.
#include "common.cuh"
#include "gemv.h"
#include "q4m.cuh"
#include "q4m_device.cuh"

#include <math.h>

namespace jinf {

using namespace q4mdev;

namespace {

constexpr int NW = GEMV_M_THREADS / 32;

__device__ __forceinline__ void l2_prefetch(const uint8_t* p, uint64_t bytes) {
    uint64_t off = 0;
    while (off < bytes) {
        const uint64_t rem = bytes - off;
        const uint32_t n = (uint32_t)(rem < (1ull << 20) ? rem : (1ull << 20));
        prefetch_l2(p + off, n);
        off += n;
    }
}

}  // namespace

template <int XM, int EPI, int FMT>
__global__ void __launch_bounds__(GEMV_M_THREADS) k_gemv_q4m(const GemvParams p) {
    constexpr int UB = q4m_unit_bytes(FMT);  // unit bytes
    extern __shared__ __align__(16) uint8_t smem_raw[];
    const int G = p.groups;
    uint8_t* rec = smem_raw;                                                     // input digit records
    float* misc = reinterpret_cast<float*>(smem_raw + xrec_bytes(G));           // 64 floats
    float* part_s = misc + 64;                                                   // [NW][32] (local_k)
    const uint32_t ring0 = smem_u32(part_s + NW * Q4M_PAIR_ROWS);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NB = gemvm_nbuf(FMT);       // ring slots per warp
    const uint32_t ring = ring0 + (uint32_t)(warp * NB * UB);
    const int kw = p.kw;
    const int T = p.pairs * kw;  // tasks: (tile pair, K part)
    const int W = gridDim.x * NW;

    // ---------------- weight stream: tasks gw, gw + W, ... (consecutive tasks on different SMs)
    const int gw = warp * gridDim.x + blockIdx.x;
    int ctask = gw, cg = 0, cge = 0;  // copy cursor
    if (ctask < T) {
        const int kp = ctask % kw;
        cg = kp * G / kw;
        cge = (kp + 1) * G / kw;
    }
    // CTA-local K split (p.local_k): CTA c takes tile pairs c, c + grid, ...; warp w takes
    // groups [w G / NW, (w + 1) G / NW) of each; the warps' partial rows meet in shared memory
    const bool local = p.local_k != 0;
    const int lg0 = warp * G / NW, lg1 = (warp + 1) * G / NW;
    int lpair = blockIdx.x, lcg = lg0;  // copy cursor (local_k)
    auto issue = [&](int slot) {
        if (local) {
            if (lg0 < lg1 && lpair < p.pairs) {
                copy_unit_fmt<FMT>(ring + slot * UB, p.w + ((size_t)lpair * G + lcg) * UB, lane);
                if (++lcg == lg1) {
                    lcg = lg0;
                    lpair += gridDim.x;
                }
            }
        } else if (ctask < T) {
            const int pair = ctask / kw;
            copy_unit_fmt<FMT>(ring + slot * UB, p.w + ((size_t)pair * G + cg) * UB, lane);
            if (++cg == cge) {
                ctask += W;
                if (ctask < T) {
                    const int kp = ctask % kw;
                    cg = kp * G / kw;
                    cge = (kp + 1) * G / kw;
                }
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");  // possibly empty: uniform group counts
    };
#pragma unroll
    for (int i = 0; i < NB - 1; ++i) issue(i);

    if (tid == 0 && p.pf_bytes) {
        const uint64_t share = ((p.pf_bytes + gridDim.x - 1) / gridDim.x + 15) & ~15ull;
        const uint64_t off = share * blockIdx.x;
        if (off < p.pf_bytes) l2_prefetch(p.pf_ptr + off, share < p.pf_bytes - off ? share : p.pf_bytes - off);
    }
    pdl_wait();
    pdl_trigger();

    // ---------------- prologue: x -> int8 digit records in shared memory
    const float* hsrc = XM == X_EMBED_NORM ? p.embed + (size_t)p.st->token * p.cols : p.hin;
    const float fac = stage_x<GEMV_M_THREADS>(XM, p.x, hsrc, p.yres, p.hout, blockIdx.x == 0, p.norm_w, p.eps, p.cols,
                                              rec, misc, false);
    const XRecS xr{smem_u32(rec), smem_u32(rec + (size_t)G * 256)};

    // ---------------- main loop
    const int c = lane & 3;
    EpiArgs ea;
    ea.epi = EPI;
    ea.rows = p.rows;
    ea.y = p.y;
    ea.kcache = p.kcache;
    ea.vcache = p.vcache;
    ea.nq = p.nq;
    ea.nk = p.nk;
    ea.head_dim = p.head_dim;
    ea.max_ctx = p.max_ctx;
    ea.pos = EPI == EPI_QKV ? p.st->pos : 0;
    ea.rope_base = p.rope_base;
    ea.coherent = false;
    float lmax = -INFINITY;
    int lidx = 0;
    int slot = 0;
    if (local) {
        for (int pair = blockIdx.x; pair < p.pairs; pair += gridDim.x) {
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            for (int g = lg0; g < lg1; ++g) {
                issue(slot == 0 ? NB - 1 : slot - 1);
                asm volatile("cp.async.wait_group %0;" ::"n"(NB - 1) : "memory");
                unit_mma_fmt<FMT>(ring + slot * UB, xr, g, lane, acc);
                slot = slot + 1 == NB ? 0 : slot + 1;
            }
            unit_reduce(acc);
            if (c == 0) {
#pragma unroll
                for (int i = 0; i < 4; ++i) part_s[warp * Q4M_PAIR_ROWS + unit_row_of(i, lane)] = acc[i];
            }
            __syncthreads();
            if (warp == 0) {  // rows 2q, 2q+1: the warps' pieces added in warp order
                const int r0 = 2 * (lane & 15);
                float v0 = 0.f, v1 = 0.f;
#pragma unroll
                for (int w = 0; w < NW; ++w) {
                    v0 += part_s[w * Q4M_PAIR_ROWS + r0];
                    v1 += part_s[w * Q4M_PAIR_ROWS + r0 + 1];
                }
                if (lane < 16) epilogue_pair(ea, pair * Q4M_PAIR_ROWS + r0, v0 * fac, v1 * fac, lmax, lidx);
            }
            __syncthreads();  // part_s is rewritten by the next pair
        }
    }
    for (int task = local ? T : gw; task < T; task += W) {
        const int pair = task / kw, kp = task % kw;
        const int g0 = kp * G / kw, g1 = (kp + 1) * G / kw;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int g = g0; g < g1; ++g) {
            issue(slot == 0 ? NB - 1 : slot - 1);
            asm volatile("cp.async.wait_group %0;" ::"n"(NB - 1) : "memory");
            unit_mma_fmt<FMT>(ring + slot * UB, xr, g, lane, acc);
            slot = slot + 1 == NB ? 0 : slot + 1;
        }
        unit_reduce(acc);
        // lane q < 16 finishes rows 2q, 2q+1 of the pair's 32
        const int r0 = 2 * (lane & 15);
        float v0, v1;
        if (kw == 1) {
            v0 = unit_row(acc, r0);
            v1 = unit_row(acc, r0 + 1);
        } else {
            float* pt = p.part + (size_t)task * Q4M_PAIR_ROWS;
            if (c == 0)
#pragma unroll
                for (int i = 0; i < 4; ++i) pt[unit_row_of(i, lane)] = acc[i];
            __threadfence();
            __syncwarp();
            unsigned old = 0;
            if (lane == 0) old = atomicAdd(p.cnt + pair, 1u);
            old = __shfl_sync(JINF_FULL_MASK, old, 0);
            if (old != (unsigned)(kw - 1)) continue;  // another task of this pair finishes it
            __threadfence();
            if (lane == 0) p.cnt[pair] = 0u;  // ready for the next launch
            v0 = 0.f;
            v1 = 0.f;
            // the parts in K order, eight row pairs in flight per lane
            const float* pb = p.part + (size_t)pair * kw * Q4M_PAIR_ROWS;
            for (int q0 = 0; q0 < kw; q0 += 8) {
                float2 t[8];
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    t[i] = q0 + i < kw ? __ldcg(reinterpret_cast<const float2*>(pb + (q0 + i) * Q4M_PAIR_ROWS + r0))
                                       : make_float2(0.f, 0.f);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    v0 += t[i].x;
                    v1 += t[i].y;
                }
            }
        }
        if (lane < 16) epilogue_pair(ea, pair * Q4M_PAIR_ROWS + r0, v0 * fac, v1 * fac, lmax, lidx);
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");

    if (EPI == EPI_LMHEAD) {
        // CTA argmax (first index wins on ties), then one atomicMax per CTA
        u64 key = lmax == -INFINITY ? 0ull : argmax_key(lmax, lidx + p.vocab_offset);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const u64 other = __shfl_xor_sync(JINF_FULL_MASK, key, o);
            key = other > key ? other : key;
        }
        __shared__ u64 wkeys[NW];
        if (lane == 0) wkeys[warp] = key;
        __syncthreads();
        if (tid == 0) {
            u64 best = 0ull;
            for (int w = 0; w < NW; ++w) best = wkeys[w] > best ? wkeys[w] : best;
            if (best) atomicMax(&p.st->best, best);
        }
    }
}

// ---------------------------------------------------------------- repack

// One thread per (pair, group, lane): its 16 nibble words and 2 scale words (q4m.cuh),
// gathered from the AoS blocks ([rows][nb] blocks of 18 bytes). Rows past `rows` and
// blocks past nb read as zero.
__host__ __device__ inline void pack_lane_q40(const uint8_t* __restrict__ aos, uint8_t* __restrict__ dst, int rows,
                                      int groups, int nb, int p, int G, int lane) {
    const int gr = lane >> 2, c = lane & 3;
    auto block = [&](int r, int j) -> const uint8_t* {  // pair row r, block j of the group
        const int row = p * Q4M_PAIR_ROWS + r;
        return row < rows && G * 4 + j < nb ? aos + ((size_t)row * nb + (size_t)G * 4 + j) * 18 : nullptr;
    };
    auto nib = [](const uint8_t* blk, int k) -> uint32_t {  // element k: byte k/2, low nibble if k even
        if (!blk) return 0u;
        const uint8_t byte = blk[2 + (k >> 1)];
        return (k & 1) ? (uint32_t)(byte >> 4) : (uint32_t)(byte & 15);
    };
    uint8_t* unit = dst + q4m_unit_offset(p, G, groups);
    for (int j = 0; j < 4; ++j)
        for (int i = 0; i < 4; ++i) {
            const int rt = gr + 8 * (i & 1);
            const uint8_t* a = block(rt, j);
            const uint8_t* b = block(16 + rt, j);
            uint32_t word = 0;
            for (int t = 0; t < 4; ++t) {
                const int k = 16 * (i >> 1) + 4 * c + t;
                word |= (nib(a, k) | (nib(b, k) << 4)) << (8 * t);
            }
            *reinterpret_cast<uint32_t*>(unit + 512 * j + 16 * lane + 4 * i) = word;
        }
    for (int t = 0; t < 2; ++t) {
        const uint8_t* b0 = block(16 * t + gr, c);
        const uint8_t* b1 = block(16 * t + gr + 8, c);
        const uint32_t d0 = b0 ? (uint32_t)b0[0] | ((uint32_t)b0[1] << 8) : 0u;
        const uint32_t d1 = b1 ? (uint32_t)b1[0] | ((uint32_t)b1[1] << 8) : 0u;
        *reinterpret_cast<uint32_t*>(unit + Q4M_SCALES + 128 * t + 4 * lane) = d0 | (d1 << 16);
    }
}
__global__ void k_repack_q4m(const uint8_t* __restrict__ aos, uint8_t* __restrict__ dst, int rows, int groups,
                             int pairs, int nb) {
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (int64_t)pairs * groups * 32) return;
    const int lane = (int)(gid & 31);
    const int64_t pg = gid >> 5;
    const int p = (int)(pg / groups), G = (int)(pg % groups);
    pack_lane_q40(aos, dst, rows, groups, nb, p, G, lane);
}

// One thread per (pair, group, lane) of a Q4_K matrix (AoS super-blocks of 144 bytes,
// [rows][nsb]): the unit's nibble words (group G = sub-blocks 4 (G % 2) + j of super-block
// G / 2), the lane's sc | m words, and lanes 0..15 / 16..31 the d, dmin of tile A / B row
// lane % 16 (q4m.cuh). The 6-bit sc and m unpacking follows reference src/quant.cpp:71-77.
__host__ __device__ inline void pack_lane_q4k(const uint8_t* __restrict__ aos, uint8_t* __restrict__ dst, int rows,
                                      int groups, int nsb, int p, int G, int lane) {
    const int gr = lane >> 2, c = lane & 3, sbk = G >> 1, half = G & 1;
    auto block = [&](int r) -> const uint8_t* {  // super-block sbk of pair row r
        const int row = p * Q4M_PAIR_ROWS + r;
        return row < rows && sbk < nsb ? aos + ((size_t)row * nsb + sbk) * 144 : nullptr;
    };
    auto nib = [&](const uint8_t* blk, int sb, int k) -> uint32_t {
        if (!blk) return 0u;
        const uint8_t byte = blk[16 + sb * 16 + (k >> 1)];
        return (k & 1) ? (uint32_t)(byte >> 4) : (uint32_t)(byte & 15);
    };
    auto scm = [&](const uint8_t* blk, int sb) -> uint32_t {  // sc | m << 8 of sub-block sb
        if (!blk) return 0u;
        const uint8_t* s = blk + 4;
        uint32_t sc, m;
        if (sb < 4) {
            sc = s[sb] & 0x3F;
            m = s[sb + 4] & 0x3F;
        } else {
            sc = (uint32_t)((s[sb + 4] & 0x0F) << 2) | (uint32_t)(s[sb - 4] >> 6);
            m = (uint32_t)((s[sb + 4] >> 4) << 2) | (uint32_t)(s[sb] >> 6);
        }
        return sc | (m << 8);
    };
    uint8_t* unit = dst + q4m_unit_offset(p, G, groups, Q4M_Q4_K);
    for (int j = 0; j < 4; ++j)
        for (int i = 0; i < 4; ++i) {
            const int rt = gr + 8 * (i & 1);
            const uint8_t* a = block(rt);
            const uint8_t* b = block(16 + rt);
            const int sb = 4 * half + j;
            uint32_t word = 0;
            for (int t = 0; t < 4; ++t) {
                const int k = 16 * (i >> 1) + 4 * c + t;
                word |= (nib(a, sb, k) | (nib(b, sb, k) << 4)) << (8 * t);
            }
            *reinterpret_cast<uint32_t*>(unit + 512 * j + 16 * lane + 4 * i) = word;
        }
    for (int t = 0; t < 2; ++t)
        *reinterpret_cast<uint32_t*>(unit + Q4M_SCALES + 128 * t + 4 * lane) =
            scm(block(16 * t + gr), 4 * half + c) | (scm(block(16 * t + gr + 8), 4 * half + c) << 16);
    const uint8_t* own = block(lane);  // tile A rows 0..15, tile B rows 16..31
    const uint32_t dd = own ? (uint32_t)own[0] | ((uint32_t)own[1] << 8) | ((uint32_t)own[2] << 16) |
                                  ((uint32_t)own[3] << 24)
                            : 0u;
    *reinterpret_cast<uint32_t*>(unit + Q4M_DMIN_K + 4 * lane) = dd;
}
__global__ void k_repack_q4mk(const uint8_t* __restrict__ aos, uint8_t* __restrict__ dst, int rows, int groups,
                              int pairs, int nsb) {
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (int64_t)pairs * groups * 32) return;
    const int lane = (int)(gid & 31);
    const int64_t pg = gid >> 5;
    const int p = (int)(pg / groups), G = (int)(pg % groups);
    pack_lane_q4k(aos, dst, rows, groups, nsb, p, G, lane);
}

// One thread per (pair, group, lane) of a Q6_K matrix (AoS super-blocks of 210 bytes,
// [rows][nsb]): the lane's nibble words and crumb words, its two scale words, and lanes with
// c = 0 the d record of row group gr (q4m.cuh). Element e of a super-block is
// low4 | high2 << 4 with low4 from ql[e / 2] (low nibble for even e) and high2 from bits
// 2 (e % 4) of qh[e / 4] (reference cuda/dequant_kernels.cu:82-110). Rows past `rows` pack
// as q = 32 with d = 0 (weight 0).
__host__ __device__ inline void pack_lane_q6k(const uint8_t* __restrict__ aos, uint8_t* __restrict__ dst, int rows,
                                      int groups, int nsb, int p, int G, int lane) {
    const int gr = lane >> 2, c = lane & 3, sbk = G >> 1, half = G & 1;
    auto block = [&](int r) -> const uint8_t* {  // super-block sbk of pair row r
        const int row = p * Q4M_PAIR_ROWS + r;
        return row < rows && sbk < nsb ? aos + ((size_t)row * nsb + sbk) * 210 : nullptr;
    };
    // low nibble and flipped crumb of element k of block j (of this group) of a super-block
    auto low4 = [&](const uint8_t* blk, int j, int k) -> uint32_t {
        if (!blk) return 0u;
        const int e = 128 * half + 32 * j + k;
        const uint8_t byte = blk[e >> 1];
        return (e & 1) ? (uint32_t)(byte >> 4) : (uint32_t)(byte & 15);
    };
    auto crumb = [&](const uint8_t* blk, int j, int k) -> uint32_t {
        if (!blk) return 0u;
        const int e = 128 * half + 32 * j + k;
        return (((uint32_t)blk[128 + (e >> 2)] >> (2 * (e & 3))) & 3u) ^ 2u;
    };
    uint8_t* unit = dst + q4m_unit_offset(p, G, groups, Q4M_Q6_K);
    for (int j = 0; j < 4; ++j) {
        for (int i = 0; i < 4; ++i) {
            const int rt = gr + 8 * (i & 1);
            const uint8_t* a = block(rt);
            const uint8_t* b = block(16 + rt);
            uint32_t word = 0;
            for (int t = 0; t < 4; ++t) {
                const int k = 16 * (i >> 1) + 4 * c + t;
                word |= (low4(a, j, k) | (low4(b, j, k) << 4)) << (8 * t);
            }
            *reinterpret_cast<uint32_t*>(unit + 512 * j + 16 * lane + 4 * i) = word;
        }
        for (int h = 0; h < 2; ++h) {
            uint32_t word = 0;
            for (int t = 0; t < 4; ++t) {
                uint32_t byte = 0;
                for (int u = 0; u < 2; ++u) {  // words i = 2h + u: rows gr + 8u of tiles A and B
                    const int k = 16 * h + 4 * c + t;
                    byte |= (crumb(block(gr + 8 * u), j, k) | (crumb(block(16 + gr + 8 * u), j, k) << 2)) << (4 * u);
                }
                word |= byte << (8 * t);
            }
            *reinterpret_cast<uint32_t*>(unit + Q4M_CRUMB_6 + 512 * (j >> 1) + 16 * lane + 4 * (2 * (j & 1) + h)) =
                word;
        }
    }
    for (int t = 0; t < 2; ++t) {
        uint32_t word = 0;
        for (int u = 0; u < 2; ++u) {
            const uint8_t* blk = block(16 * t + gr + 8 * u);
            for (int h = 0; h < 2; ++h) {
                const uint32_t sc = blk ? (uint32_t)blk[192 + 8 * half + 2 * c + h] : 0u;
                word |= sc << (8 * (2 * u + h));
            }
        }
        *reinterpret_cast<uint32_t*>(unit + Q4M_SC_6 + 8 * lane + 4 * t) = word;
    }
    if (c == 0) {
        uint16_t d4[4];
        for (int q = 0; q < 4; ++q) {
            const uint8_t* blk = block(gr + 8 * q);  // rows gr, gr + 8, 16 + gr, 24 + gr
            d4[q] = blk ? (uint16_t)(blk[208] | (blk[209] << 8)) : (uint16_t)0;
        }
        uint32_t* o = reinterpret_cast<uint32_t*>(unit + Q4M_D_6 + 8 * gr);
        o[0] = d4[0] | ((uint32_t)d4[1] << 16);
        o[1] = d4[2] | ((uint32_t)d4[3] << 16);
    }
}
__global__ void k_repack_q6k(const uint8_t* __restrict__ aos, uint8_t* __restrict__ dst, int rows, int groups,
                             int pairs, int nsb) {
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (int64_t)pairs * groups * 32) return;
    const int lane = (int)(gid & 31);
    const int64_t pg = gid >> 5;
    const int p = (int)(pg / groups), G = (int)(pg % groups);
    pack_lane_q6k(aos, dst, rows, groups, nsb, p, G, lane);
}

// One thread per (pair, group, lane) of a Q8_0 matrix (AoS blocks of 34 bytes: fp16 d, 32
// int8 q; [rows][nb], reference include/jinf/quant.h:50-56): the lane's eight weight words
// and its scale record. Rows past `rows` and blocks past nb pack as zeros.
__host__ __device__ inline void pack_lane_q80(const uint8_t* __restrict__ aos, uint8_t* __restrict__ dst, int rows,
                                      int groups, int nb, int p, int G, int lane) {
    const int gr = lane >> 2, c = lane & 3;
    auto block = [&](int r, int j) -> const uint8_t* {
        const int row = p * Q4M_PAIR_ROWS + r;
        return row < rows && G * 4 + j < nb ? aos + ((size_t)row * nb + (size_t)G * 4 + j) * 34 : nullptr;
    };
    uint8_t* unit = dst + q4m_unit_offset(p, G, groups, Q4M_Q8_0);
    for (int j = 0; j < 4; ++j)
        for (int t = 0; t < 2; ++t)
            for (int i = 0; i < 4; ++i) {
                const uint8_t* blk = block(16 * t + gr + 8 * (i & 1), j);
                uint32_t word = 0;
                if (blk)
                    for (int b = 0; b < 4; ++b) word |= (uint32_t)blk[2 + 16 * (i >> 1) + 4 * c + b] << (8 * b);
                *reinterpret_cast<uint32_t*>(unit + 1024 * j + 512 * t + 16 * lane + 4 * i) = word;
            }
    uint16_t d4[4];
    for (int q = 0; q < 4; ++q) {
        const uint8_t* blk = block(gr + 8 * q, c);  // rows gr, gr + 8, 16 + gr, 24 + gr
        d4[q] = blk ? (uint16_t)(blk[0] | (blk[1] << 8)) : (uint16_t)0;
    }
    uint32_t* o = reinterpret_cast<uint32_t*>(unit + Q4M_D_8 + 8 * lane);
    o[0] = d4[0] | ((uint32_t)d4[1] << 16);
    o[1] = d4[2] | ((uint32_t)d4[3] << 16);
}
__global__ void k_repack_q80(const uint8_t* __restrict__ aos, uint8_t* __restrict__ dst, int rows, int groups,
                             int pairs, int nb) {
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (int64_t)pairs * groups * 32) return;
    const int lane = (int)(gid & 31);
    const int64_t pg = gid >> 5;
    const int p = (int)(pg / groups), G = (int)(pg % groups);
    pack_lane_q80(aos, dst, rows, groups, nb, p, G, lane);
}

// ---------------------------------------------------------------- host side

size_t gemvm_smem_bytes(int cols, int fmt) {
    const int G = (cols + Q4M_KG - 1) / Q4M_KG;
    return xrec_bytes(G) + sizeof(float) * (64 + NW * Q4M_PAIR_ROWS) + (size_t)NW * gemvm_nbuf(fmt) * q4m_unit_bytes(fmt);
}

bool gemvm_use_local(int pairs, int grid) { return pairs <= 4 * grid; }

int gemvm_local_grid(int pairs, int grid) {
    const int rounds = (pairs + grid - 1) / grid;  // pairs per CTA, the same for every CTA
    return (pairs + rounds - 1) / rounds;
}

int gemvm_max_cols(int fmt) {
    // largest multiple of 128 whose staging fits next to the ring in the 227 KB per CTA
    int c = 128;
    while (gemvm_smem_bytes(c + 128, fmt) <= 226 * 1024) c += 128;  // static shared memory rides along
    return c;
}

template <int XM, int EPI, int FMT>
struct GemvMKernelInfo {
    static cudaError_t ensure_smem(size_t smem) {
        static size_t configured = 0;
        if (smem <= configured) return cudaSuccess;
        const size_t want = gemvm_smem_bytes(gemvm_max_cols(FMT), FMT);
        cudaError_t e =
            cudaFuncSetAttribute(k_gemv_q4m<XM, EPI, FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)want);
        if (e == cudaSuccess) configured = want;
        return e;
    }
    static int occupancy(int cols) {
        static int cached_cols = -1, cached_occ = 1;
        if (cached_cols != cols) {
            const size_t smem = gemvm_smem_bytes(cols, FMT);
            ensure_smem(smem);
            int n = 0;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_gemv_q4m<XM, EPI, FMT>, GEMV_M_THREADS, smem) !=
                    cudaSuccess ||
                n < 1)
                n = 1;
            cached_cols = cols;
            cached_occ = n;
        }
        return cached_occ;
    }
    static cudaError_t launch(const GemvParams& p, int grid, cudaStream_t s, bool pdl) {
        const size_t smem = gemvm_smem_bytes(p.cols, FMT);
        cudaError_t e = ensure_smem(smem);
        if (e != cudaSuccess) return e;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(grid);
        cfg.blockDim = dim3(GEMV_M_THREADS);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = pdl ? 1 : 0;
        return cudaLaunchKernelEx(&cfg, k_gemv_q4m<XM, EPI, FMT>, p);
    }
};

template <int XM, int EPI, int FMT>
static int occ_m(int cols) { return GemvMKernelInfo<XM, EPI, FMT>::occupancy(cols); }
template <int XM, int EPI, int FMT>
static cudaError_t launch_m(const GemvParams& p, int grid, cudaStream_t s, bool pdl) {
    return GemvMKernelInfo<XM, EPI, FMT>::launch(p, grid, s, pdl);
}

#define JINF_GEMVM_CASES(FN, F, ...)                                                                   \
    switch (xm * 16 + epi) {                                                                           \
        case X_PLAIN_F32 * 16 + EPI_STORE:   return FN<X_PLAIN_F32, EPI_STORE, F>(__VA_ARGS__);   \
        case X_PLAIN_F16 * 16 + EPI_STORE:   return FN<X_PLAIN_F16, EPI_STORE, F>(__VA_ARGS__);   \
        case X_RMSNORM * 16 + EPI_STORE:     return FN<X_RMSNORM, EPI_STORE, F>(__VA_ARGS__);     \
        case X_RMSNORM * 16 + EPI_QKV:       return FN<X_RMSNORM, EPI_QKV, F>(__VA_ARGS__);       \
        case X_EMBED_NORM * 16 + EPI_QKV:    return FN<X_EMBED_NORM, EPI_QKV, F>(__VA_ARGS__);    \
        case X_RMSNORM * 16 + EPI_GATEUP:    return FN<X_RMSNORM, EPI_GATEUP, F>(__VA_ARGS__);    \
        case X_PLAIN_F32 * 16 + EPI_GATEUP:  return FN<X_PLAIN_F32, EPI_GATEUP, F>(__VA_ARGS__);  \
        case X_RMSNORM * 16 + EPI_LMHEAD:    return FN<X_RMSNORM, EPI_LMHEAD, F>(__VA_ARGS__);    \
        case X_PLAIN_F32 * 16 + EPI_LMHEAD:  return FN<X_PLAIN_F32, EPI_LMHEAD, F>(__VA_ARGS__);  \
        default: break;                                                                                \
    }
#define JINF_GEMVM_DISPATCH(FMTV, FN, ...)                  \
    if ((FMTV) == Q4M_Q4_K) {                               \
        JINF_GEMVM_CASES(FN, Q4M_Q4_K, __VA_ARGS__)         \
    } else if ((FMTV) == Q4M_Q6_K) {                        \
        JINF_GEMVM_CASES(FN, Q4M_Q6_K, __VA_ARGS__)         \
    } else if ((FMTV) == Q4M_Q8_0) {                        \
        JINF_GEMVM_CASES(FN, Q4M_Q8_0, __VA_ARGS__)         \
    } else {                                                \
        JINF_GEMVM_CASES(FN, Q4M_Q4_0, __VA_ARGS__)         \
    }

int gemvm_grid(int cols, int xm, int epi, int num_sms, int fmt) {
    auto occ_fn = [&]() -> int {
        JINF_GEMVM_DISPATCH(fmt, occ_m, cols)
        return 1;
    };
    return occ_fn() * num_sms;
}

// K split per tile pair: the smallest cost ceil(tasks / grid) * (groups per task + overhead),
// with at least 8 busy warps per CTA where the matrix allows it.
int gemvm_pick_kw(int pairs, int groups, int grid, int max_kw) {
    int best = 1;
    double best_cost = 1e300;
    const int lim = groups < max_kw ? groups : max_kw;
    for (int kw = 1; kw <= lim; ++kw) {
        const long long T = (long long)pairs * kw;
        const bool busy = T >= (long long)grid * 8;
        const double per_cta = (double)((T + grid - 1) / grid);
        const double cost = per_cta * ((double)((groups + kw - 1) / kw) + (kw > 1 ? 0.6 : 0.1)) + (busy ? 0.0 : 1e9 / (double)T);
        if (cost < best_cost - 1e-9) {
            best_cost = cost;
            best = kw;
        }
    }
    return best;
}

cudaError_t gemvm_launch(const GemvParams& p, int xm, int epi, int grid, cudaStream_t s, bool pdl) {
    if (p.kw < 1 || p.kw > p.groups || (p.kw > 1 && (!p.part || !p.cnt))) return cudaErrorInvalidValue;
    if (p.cols > gemvm_max_cols(p.fmt)) return cudaErrorInvalidValue;
    JINF_GEMVM_DISPATCH(p.fmt, launch_m, p, grid, s, pdl)
    return cudaErrorInvalidValue;
}

// The same repack on the host (the lane functions the kernels run), for tools that write
// pre-packed matrices without a GPU.
void q4m_repack_host(const void* aos, void* dst, const Q4MShape& sh) {
    const int64_t n = (int64_t)sh.pairs * sh.groups;
    const uint8_t* a = (const uint8_t*)aos;
    uint8_t* d = (uint8_t*)dst;
#pragma omp parallel for schedule(static)
    for (int64_t pg = 0; pg < n; ++pg) {
        const int p = (int)(pg / sh.groups), G = (int)(pg % sh.groups);
        for (int lane = 0; lane < 32; ++lane) {
            if (sh.fmt == Q4M_Q6_K) pack_lane_q6k(a, d, sh.rows, sh.groups, sh.cols / 256, p, G, lane);
            else if (sh.fmt == Q4M_Q8_0) pack_lane_q80(a, d, sh.rows, sh.groups, sh.cols / 32, p, G, lane);
            else if (sh.fmt == Q4M_Q4_K) pack_lane_q4k(a, d, sh.rows, sh.groups, sh.cols / 256, p, G, lane);
            else pack_lane_q40(a, d, sh.rows, sh.groups, sh.cols / 32, p, G, lane);
        }
    }
}

cudaError_t q4m_repack(const void* aos, void* dst, const Q4MShape& sh, cudaStream_t s) {
    const int64_t n = (int64_t)sh.pairs * sh.groups * 32;
    if (sh.fmt == Q4M_Q6_K)
        k_repack_q6k<<<(unsigned)((n + 255) / 256), 256, 0, s>>>((const uint8_t*)aos, (uint8_t*)dst, sh.rows,
                                                                 sh.groups, sh.pairs, sh.cols / 256);
    else if (sh.fmt == Q4M_Q8_0)
        k_repack_q80<<<(unsigned)((n + 255) / 256), 256, 0, s>>>((const uint8_t*)aos, (uint8_t*)dst, sh.rows,
                                                                 sh.groups, sh.pairs, sh.cols / 32);
    else if (sh.fmt == Q4M_Q4_K)
        k_repack_q4mk<<<(unsigned)((n + 255) / 256), 256, 0, s>>>((const uint8_t*)aos, (uint8_t*)dst, sh.rows,
                                                                  sh.groups, sh.pairs, sh.cols / 256);
    else
        k_repack_q4m<<<(unsigned)((n + 255) / 256), 256, 0, s>>>((const uint8_t*)aos, (uint8_t*)dst, sh.rows,
                                                                 sh.groups, sh.pairs, sh.cols / 32);
    return cudaGetLastError();
}

}  // namespace jinf
