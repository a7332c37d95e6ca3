// Fused Q4_0 GEMV over the Q4M layout (q4m.cuh) on the tensor cores, sm_100a.
//
// Same prologue / epilogue modes as the Q4T kernel (gemv_q4t.cu): plain x, RMSNorm of the
// residual stream, embedding row + RMSNorm; plain store, QKV with RoPE and fp16 KV write,
// gate|up with silu(gate)*up, LM head with the packed argmax.
//
// Why tensor cores for a batch-1 GEMV. The reference computes y = sum_b d_b sum_e (q-8) x_e
// in fp32 (cuda/matmul_kernels.cu:8-43). Streaming 4-bit weights at HBM speed leaves about
// three issue slots per weight on the CUDA cores, and an exact fp32 decode needs about that
// many (decode, bias, multiply-add). Here the decode is one lop3 per two weights and the
// multiply-add is retired by mma.sync.m16n8k16: the weight tile is the A operand, decoded
// in registers to the exact fp16 values 1024 + s*q (s = 1 or 16); the B operand holds x
// split into fp16 hi + lo parts (22 significant bits), pre-scaled by 2^k / s. B is block
// diagonal: its column 2j+h carries part h of block j of the group, so one m16n8k16 step
// advances 16 rows x 4 blocks at once and the accumulator column pair (2c, 2c+1) of a lane
// is exactly one block's dot product for rows gr and gr+8. Products are exact in fp32; the
// constant 1024 + 8s offset of every weight is removed by initialising the accumulator with
// -(1024 + 8s) * sum(B) of the block, and the block scale d multiplies the block sum once.
//
// Scheduling. Tasks are (tile, K part) pairs: a tile's groups are split over `kw` tasks so
// that every SM gets the same amount of work. Each warp streams its tasks' chunks through
// a private cp.async ring (GEMV_M_NBUF - 1 chunks of 1152 bytes in flight) that runs ahead
// across task boundaries; the first chunks are requested before the kernel waits on its
// producer (programmatic dependent launch), because weights never depend on it. With kw > 1
// each task writes its 16 partial sums to a workspace and the last task of a tile (arrival
// counter, reset by that task) adds them in K order, so results are deterministic.
#include "common.cuh"
#include "q4m.cuh"
#include "gemv_q4t.h"

#include <math.h>

namespace jinf {

namespace {

typedef unsigned long long u64;
constexpr int NW = GEMV_M_THREADS / 32;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// This lane's 36 bytes of a chunk: nibble words of piece 0 and 1 and its two scales. Each
// lane reads back only what it copied, so the ring needs no warp synchronisation.
__device__ __forceinline__ void copy_chunk_async(uint32_t slot, const uint8_t* chunk, int lane) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(slot + lane * 16), "l"(chunk + lane * 16)
                 : "memory");
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(slot + 512 + lane * 16),
                 "l"(chunk + 512 + lane * 16)
                 : "memory");
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(slot + 1024 + lane * 4), "l"(chunk + 1024 + lane * 4)
                 : "memory");
}

// One MMA step: decode the lane's word (eight nibbles -> four fp16x2 A registers) and
// accumulate A x B into d. The lop3 immediate 0xEA is (a & b) | c.
__device__ __forceinline__ void mma_step(uint32_t w, uint32_t b0, uint32_t b1, float (&d)[4]) {
    asm("{\n\t"
        ".reg .b32 a0, a1, a2, a3, u;\n\t"
        "shr.u32 u, %4, 8;\n\t"
        "lop3.b32 a0, %4, 0x000F000F, 0x64006400, 0xEA;\n\t"
        "lop3.b32 a2, %4, 0x00F000F0, 0x64006400, 0xEA;\n\t"
        "lop3.b32 a1, u, 0x000F000F, 0x64006400, 0xEA;\n\t"
        "lop3.b32 a3, u, 0x00F000F0, 0x64006400, 0xEA;\n\t"
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {a0, a1, a2, a3}, {%5, %6}, "
        "{%0, %1, %2, %3};\n\t"
        "}"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(w), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t ordered_bits(float v) {
    const uint32_t b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ void l2_prefetch(const uint8_t* p, uint64_t bytes) {
    uint64_t off = 0;
    while (off < bytes) {
        const uint64_t rem = bytes - off;
        const uint32_t n = (uint32_t)(rem < (1ull << 20) ? rem : (1ull << 20));
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p + off), "r"(n) : "memory");
        off += n;
    }
}

// Power-of-two pre-scale 2^k putting amax * 2^k in [2^14, 2^15): the fp16 hi part of
// every scaled x stays finite and the lo part keeps its precision.
__device__ __forceinline__ float pow2_prescale(float amax) {
    int e = (int)((__float_as_uint(amax) >> 23) & 0xff);  // biased exponent of amax
    int k = 127 + 14 - (e - 127);                           // biased exponent of 2^(14 - E)
    k = k < 1 ? 1 : (k > 254 ? 254 : k);
    return __uint_as_float((uint32_t)k << 23);
}

}  // namespace

template <int XM, int EPI>
__global__ void __launch_bounds__(GEMV_M_THREADS) k_gemv_q4m(const GemvParams p) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    const int G = p.groups, nb = p.cols / 32;
    uint16_t* xb = reinterpret_cast<uint16_t*>(smem_raw);                   // [G][32 lanes][8] fp16 B values
    float* xk = reinterpret_cast<float*>(smem_raw + (size_t)G * 512);      // [nb] accumulator offsets
    float* misc = xk + nb;                                                  // 64 floats
    const uint32_t ring0 = smem_u32(misc + 64);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t ring = ring0 + (uint32_t)(warp * GEMV_M_NBUF * Q4M_CHUNK);
    const int kw = p.kw;
    const int T = p.tiles * kw;
    const int W = gridDim.x * NW;

    // ---------------- weight stream: tasks gw, gw + W, ... (consecutive tasks on different SMs)
    const int gw = warp * gridDim.x + blockIdx.x;
    int ctask = gw, cg = 0, cge = 0;  // copy cursor
    if (ctask < T) {
        const int kp = ctask % kw;
        cg = kp * G / kw;
        cge = (kp + 1) * G / kw;
    }
    auto issue = [&](int slot) {
        if (ctask < T) {
            const int tile = ctask / kw;
            copy_chunk_async(ring + slot * Q4M_CHUNK, p.w + ((size_t)tile * G + cg) * Q4M_CHUNK, lane);
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
    for (int i = 0; i < GEMV_M_NBUF - 1; ++i) issue(i);

    if (tid == 0 && p.pf_bytes) {
        const uint64_t share = ((p.pf_bytes + gridDim.x - 1) / gridDim.x + 15) & ~15ull;
        const uint64_t off = share * blockIdx.x;
        if (off < p.pf_bytes) l2_prefetch(p.pf_ptr + off, share < p.pf_bytes - off ? share : p.pf_bytes - off);
    }
    pdl_wait();
    pdl_trigger();

    // ---------------- prologue: x -> block-diagonal fp16 hi/lo B values in shared memory.
    // One round trip to global memory: the fp32 input (x, or h * gain in the norm modes) is
    // staged in the B region itself, sum(h^2) and max|x| are reduced in one pass, then each
    // warp converts whole 128-column groups in place.
    constexpr bool NORM = XM == X_RMSNORM || XM == X_EMBED_NORM;
    float* xf = reinterpret_cast<float*>(smem_raw);  // [cols] fp32, group g at bytes [512 g, 512 g + 512)
    const float* hsrc = p.hin;
    if (XM == X_EMBED_NORM) hsrc = p.embed + (size_t)p.st->token * p.cols;
    const bool store_h = NORM && blockIdx.x == 0 && p.hout;
    float ss = 0.f, amax = 0.f;
#pragma unroll 4
    for (int i = tid; i < p.cols / 4; i += GEMV_M_THREADS) {
        float4 v;
        if (XM == X_PLAIN_F32) {
            v = reinterpret_cast<const float4*>(p.x)[i];
        } else if (XM == X_PLAIN_F16) {
            const uint2 hv = reinterpret_cast<const uint2*>(p.x)[i];
            const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&hv.x));
            const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&hv.y));
            v = make_float4(a.x, a.y, b.x, b.y);
        } else {
            float4 h = reinterpret_cast<const float4*>(hsrc)[i];
            if (XM == X_RMSNORM && p.yres) {
                const float4 r = reinterpret_cast<const float4*>(p.yres)[i];
                h.x += r.x;
                h.y += r.y;
                h.z += r.z;
                h.w += r.w;
            }
            if (store_h) reinterpret_cast<float4*>(p.hout)[i] = h;
            ss = fmaf(h.x, h.x, ss);
            ss = fmaf(h.y, h.y, ss);
            ss = fmaf(h.z, h.z, ss);
            ss = fmaf(h.w, h.w, ss);
            const float4 g = reinterpret_cast<const float4*>(p.norm_w)[i];
            v = make_float4(h.x * g.x, h.y * g.y, h.z * g.z, h.w * g.w);
        }
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        reinterpret_cast<float4*>(xf)[i] = v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        ss += __shfl_xor_sync(JINF_FULL_MASK, ss, o);
        amax = fmaxf(amax, __shfl_xor_sync(JINF_FULL_MASK, amax, o));
    }
    if (lane == 0) {
        misc[warp] = ss;
        misc[32 + warp] = amax;
    }
    __syncthreads();
    ss = 0.f;
    amax = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
        ss += misc[w];
        amax = fmaxf(amax, misc[32 + w]);
    }
    const float rnorm = NORM ? rsqrtf(ss / (float)p.cols + p.eps) : 1.0f;
    const float alpha = pow2_prescale(amax * rnorm * 1.0001f);
    const float inv_alpha = 1.0f / alpha;  // exact: alpha is a power of two
    for (int g = warp; g < G; g += NW) {
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = xf[g * 128 + j * 32 + lane];
        __syncwarp();  // the whole group is in registers before it is overwritten
        float s[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float x = NORM ? v[j] * rnorm : v[j];
            const float sv = x * alpha * (j < 2 ? 1.0f : 0.0625f);
            const __half hi = __float2half_rn(sv);
            const __half lo = __float2half_rn(sv - __half2float(hi));
            // element e = lane of block j: lane record 4*(2j + h) + (e & 3), half e >> 2
            uint16_t* rec = xb + (size_t)g * 256 + (8 * j + (lane & 3)) * 8 + (lane >> 2);
            rec[0] = __half_as_ushort(hi);
            rec[32] = __half_as_ushort(lo);  // h = 1: four lane records further
            s[j] = __half2float(hi) + __half2float(lo);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int j = 0; j < 4; ++j) s[j] += __shfl_xor_sync(JINF_FULL_MASK, s[j], o);
        if (lane < 4) {
            float sj = s[0];
#pragma unroll
            for (int j = 1; j < 4; ++j)
                if (lane == j) sj = s[j];
            xk[g * 4 + lane] = -(lane < 2 ? 1032.0f : 1152.0f) * sj;
        }
    }
    __syncthreads();

    // ---------------- main loop
    const int gr = lane >> 2, c = lane & 3, jn = lane >> 3;
    // B fragment byte selectors: this lane's value goes to half (jn & 1) of b0 (jn < 2)
    // or b1 (jn >= 2); even steps take bytes 0-1 of the staged word, odd steps bytes 2-3.
    const uint32_t s0e = jn == 0 ? 0x4410u : jn == 1 ? 0x1044u : 0x4444u;
    const uint32_t s0o = jn == 0 ? 0x4432u : jn == 1 ? 0x3244u : 0x4444u;
    const uint32_t s1e = jn == 2 ? 0x4410u : jn == 3 ? 0x1044u : 0x4444u;
    const uint32_t s1o = jn == 2 ? 0x4432u : jn == 3 ? 0x3244u : 0x4444u;
    float lmax = -INFINITY;
    int lidx = 0;
    int slot = 0;
    for (int task = gw; task < T; task += W) {
        const int tile = task / kw, kp = task % kw;
        const int g0 = kp * G / kw, g1 = (kp + 1) * G / kw;
        float acc0 = 0.f, acc1 = 0.f;
        for (int g = g0; g < g1; ++g) {
            issue(slot == 0 ? GEMV_M_NBUF - 1 : slot - 1);
            asm volatile("cp.async.wait_group %0;" ::"n"(GEMV_M_NBUF - 1) : "memory");
            const uint32_t sl = ring + slot * Q4M_CHUNK;
            uint32_t w[8], sc;
            asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]) : "r"(sl + lane * 16));
            asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(w[4]), "=r"(w[5]), "=r"(w[6]), "=r"(w[7]) : "r"(sl + 512 + lane * 16));
            asm volatile("ld.shared.u32 %0, [%1];" : "=r"(sc) : "r"(sl + 1024 + lane * 4));
            const uint4 xv = *reinterpret_cast<const uint4*>(xb + (size_t)g * 256 + lane * 8);
            const float k = xk[g * 4 + c];
            float da[4] = {k, 0.f, k, 0.f}, db[4] = {0.f, 0.f, 0.f, 0.f};
            const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
            for (int i = 0; i < 8; i += 2) {
                mma_step(w[i], __byte_perm(xw[i >> 1], 0u, s0e), __byte_perm(xw[i >> 1], 0u, s1e), da);
                mma_step(w[i + 1], __byte_perm(xw[i >> 1], 0u, s0o), __byte_perm(xw[i >> 1], 0u, s1o), db);
            }
            const float t0 = (da[0] + da[1]) + (db[0] + db[1]);
            const float t1 = (da[2] + da[3]) + (db[2] + db[3]);
            acc0 = fmaf(jinf_h2f((uint16_t)(sc & 0xffffu)), t0, acc0);
            acc1 = fmaf(jinf_h2f((uint16_t)(sc >> 16)), t1, acc1);
            slot = slot + 1 == GEMV_M_NBUF ? 0 : slot + 1;
        }
        // blocks c = 0..3 of the lanes of a row group
        acc0 += __shfl_xor_sync(JINF_FULL_MASK, acc0, 1);
        acc1 += __shfl_xor_sync(JINF_FULL_MASK, acc1, 1);
        acc0 += __shfl_xor_sync(JINF_FULL_MASK, acc0, 2);
        acc1 += __shfl_xor_sync(JINF_FULL_MASK, acc1, 2);
        // lane q < 8 finishes rows 2q, 2q+1 of the tile
        const int r0 = 2 * (lane & 7), r1 = r0 + 1;
        float v0, v1;
        if (kw == 1) {
            const float a0 = __shfl_sync(JINF_FULL_MASK, acc0, 4 * (r0 & 7));
            const float b0 = __shfl_sync(JINF_FULL_MASK, acc1, 4 * (r0 & 7));
            const float a1 = __shfl_sync(JINF_FULL_MASK, acc0, 4 * (r1 & 7));
            const float b1 = __shfl_sync(JINF_FULL_MASK, acc1, 4 * (r1 & 7));
            v0 = r0 < 8 ? a0 : b0;
            v1 = r1 < 8 ? a1 : b1;
        } else {
            float* pt = p.part + (size_t)task * 16;
            if (c == 0) {
                pt[gr] = acc0;
                pt[gr + 8] = acc1;
            }
            __threadfence();
            __syncwarp();
            unsigned old = 0;
            if (lane == 0) old = atomicAdd(p.cnt + tile, 1u);
            old = __shfl_sync(JINF_FULL_MASK, old, 0);
            if (old != (unsigned)(kw - 1)) continue;  // another task of this tile finishes it
            __threadfence();
            if (lane == 0) p.cnt[tile] = 0u;  // ready for the next launch
            v0 = 0.f;
            v1 = 0.f;
            const float* pb = p.part + (size_t)tile * kw * 16;
            for (int q = 0; q < kw; ++q) {
                v0 += __ldcg(pb + q * 16 + r0);
                v1 += __ldcg(pb + q * 16 + r1);
            }
        }
        v0 *= inv_alpha;
        v1 *= inv_alpha;
        const int row = tile * Q4M_ROWS + r0;
        if (lane < 8 && row < p.rows) {
            if (EPI == EPI_STORE || EPI == EPI_LMHEAD) {
                p.y[row] = v0;
                if (EPI == EPI_LMHEAD && v0 > lmax) { lmax = v0; lidx = row; }
                if (row + 1 < p.rows) {
                    p.y[row + 1] = v1;
                    if (EPI == EPI_LMHEAD && v1 > lmax) { lmax = v1; lidx = row + 1; }
                }
            } else if (EPI == EPI_GATEUP) {
                p.y[row >> 1] = v0 / (1.0f + expf(-v0)) * v1;
            } else {  // EPI_QKV: rows are [q | k | v], each head_dim-aligned
                const int pos = p.st->pos;
                if (row < p.nq + p.nk) {
                    const int rr = row < p.nq ? row : row - p.nq;
                    const int i = (rr % p.head_dim) >> 1;
                    const float theta = powf(p.rope_base, -2.0f * (float)i / (float)p.head_dim);
                    const float ang = (float)pos * theta;
                    const float cs = cosf(ang), sn = sinf(ang);
                    const float o0 = v0 * cs - v1 * sn, o1 = v0 * sn + v1 * cs;
                    if (row < p.nq) {
                        p.y[row] = o0;
                        p.y[row + 1] = o1;
                    } else {
                        const int kvh = rr / p.head_dim, dd = rr % p.head_dim;
                        __half* dst = p.kcache + ((size_t)kvh * p.max_ctx + pos) * p.head_dim + dd;
                        *reinterpret_cast<__half2*>(dst) = __floats2half2_rn(o0, o1);
                    }
                } else {
                    const int rr = row - p.nq - p.nk;
                    const int kvh = rr / p.head_dim, dd = rr % p.head_dim;
                    __half* dst = p.vcache + ((size_t)kvh * p.max_ctx + pos) * p.head_dim + dd;
                    *reinterpret_cast<__half2*>(dst) = __floats2half2_rn(v0, v1);
                }
            }
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");

    if (EPI == EPI_LMHEAD) {
        // CTA argmax (first index wins on ties), then one atomicMax per CTA
        u64 key = lmax == -INFINITY ? 0ull
                : ((u64)ordered_bits(lmax) << 32) | (u64)(0xFFFFFFFFu - (uint32_t)(lidx + p.vocab_offset));
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

// One thread per (tile, group, lane): its 8 nibble words and 2 scales, gathered from the
// AoS blocks. Rows past `rows` read as zero.
__global__ void k_repack_q4m(const uint8_t* __restrict__ aos, uint8_t* __restrict__ dst, int rows, int groups,
                             int tiles) {
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (int64_t)tiles * groups * 32) return;
    const int lane = (int)(gid & 31);
    const int64_t tg = gid >> 5;
    const int t = (int)(tg / groups), G = (int)(tg % groups);
    const int gr = lane >> 2, c = lane & 3;
    const int nb = groups * 4;
    auto block = [&](int r, int j) -> const uint8_t* {
        const int row = t * Q4M_ROWS + r;
        return row < rows ? aos + ((size_t)row * nb + (size_t)G * 4 + j) * 18 : nullptr;
    };
    uint8_t* chunk = dst + (size_t)tg * Q4M_CHUNK;
    for (int i = 0; i < 8; ++i) {
        const int e = 4 * i + c;
        uint32_t word = 0;
        for (int half = 0; half < 2; ++half)
            for (int j = 0; j < 4; ++j) {
                const int r = gr + 8 * half;
                const uint8_t* blk = block(r, j);
                if (!blk) continue;
                const uint8_t byte = blk[2 + (e >> 1)];
                const uint32_t q = (e & 1) ? (byte >> 4) : (byte & 15);
                word |= q << q4m_nibble_bit(r, j);
            }
        *reinterpret_cast<uint32_t*>(chunk + (i >> 2) * 512 + lane * 16 + (i & 3) * 4) = word;
    }
    const uint8_t* b0 = block(gr, c);
    const uint8_t* b1 = block(gr + 8, c);
    const uint32_t d0 = b0 ? (uint32_t)b0[0] | ((uint32_t)b0[1] << 8) : 0u;
    const uint32_t d1 = b1 ? (uint32_t)b1[0] | ((uint32_t)b1[1] << 8) : 0u;
    *reinterpret_cast<uint32_t*>(chunk + 1024 + lane * 4) = d0 | (d1 << 16);
}

// ---------------------------------------------------------------- host side

size_t gemvm_smem_bytes(int cols) {
    const int G = cols / Q4M_KG;
    return (size_t)G * 512 + sizeof(float) * ((size_t)(cols / 32) + 64) + (size_t)NW * GEMV_M_NBUF * Q4M_CHUNK;
}

int gemvm_max_cols() {
    // largest multiple of 128 whose staging fits next to the ring in the 227 KB per CTA
    int c = 128;
    while (gemvm_smem_bytes(c + 128) <= 226 * 1024) c += 128;  // static shared memory rides along
    return c;
}

template <int XM, int EPI>
struct GemvMKernelInfo {
    static cudaError_t ensure_smem(size_t smem) {
        static size_t configured = 0;
        if (smem <= configured) return cudaSuccess;
        const size_t want = gemvm_smem_bytes(gemvm_max_cols());
        cudaError_t e = cudaFuncSetAttribute(k_gemv_q4m<XM, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)want);
        if (e == cudaSuccess) configured = want;
        return e;
    }
    static int occupancy(int cols) {
        static int cached_cols = -1, cached_occ = 1;
        if (cached_cols != cols) {
            const size_t smem = gemvm_smem_bytes(cols);
            ensure_smem(smem);
            int n = 0;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_gemv_q4m<XM, EPI>, GEMV_M_THREADS, smem) !=
                    cudaSuccess ||
                n < 1)
                n = 1;
            cached_cols = cols;
            cached_occ = n;
        }
        return cached_occ;
    }
    static cudaError_t launch(const GemvParams& p, int grid, cudaStream_t s, bool pdl) {
        const size_t smem = gemvm_smem_bytes(p.cols);
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
        return cudaLaunchKernelEx(&cfg, k_gemv_q4m<XM, EPI>, p);
    }
};

template <int XM, int EPI>
static int occ_m(int cols) { return GemvMKernelInfo<XM, EPI>::occupancy(cols); }
template <int XM, int EPI>
static cudaError_t launch_m(const GemvParams& p, int grid, cudaStream_t s, bool pdl) {
    return GemvMKernelInfo<XM, EPI>::launch(p, grid, s, pdl);
}

#define JINF_GEMVM_DISPATCH(FN, ...)                                                    \
    switch (xm * 16 + epi) {                                                            \
        case X_PLAIN_F32 * 16 + EPI_STORE:   return FN<X_PLAIN_F32, EPI_STORE>(__VA_ARGS__);   \
        case X_PLAIN_F16 * 16 + EPI_STORE:   return FN<X_PLAIN_F16, EPI_STORE>(__VA_ARGS__);   \
        case X_RMSNORM * 16 + EPI_STORE:     return FN<X_RMSNORM, EPI_STORE>(__VA_ARGS__);     \
        case X_RMSNORM * 16 + EPI_QKV:       return FN<X_RMSNORM, EPI_QKV>(__VA_ARGS__);       \
        case X_EMBED_NORM * 16 + EPI_QKV:    return FN<X_EMBED_NORM, EPI_QKV>(__VA_ARGS__);    \
        case X_RMSNORM * 16 + EPI_GATEUP:    return FN<X_RMSNORM, EPI_GATEUP>(__VA_ARGS__);    \
        case X_PLAIN_F32 * 16 + EPI_GATEUP:  return FN<X_PLAIN_F32, EPI_GATEUP>(__VA_ARGS__);  \
        case X_RMSNORM * 16 + EPI_LMHEAD:    return FN<X_RMSNORM, EPI_LMHEAD>(__VA_ARGS__);    \
        case X_PLAIN_F32 * 16 + EPI_LMHEAD:  return FN<X_PLAIN_F32, EPI_LMHEAD>(__VA_ARGS__);  \
        default: break;                                                                 \
    }

int gemvm_grid(int cols, int xm, int epi, int num_sms) {
    auto occ_fn = [&]() -> int {
        JINF_GEMVM_DISPATCH(occ_m, cols)
        return 1;
    };
    return occ_fn() * num_sms;
}

// K split per tile: the smallest cost ceil(tasks / grid) * (groups per task + overhead),
// with at least 8 busy warps per CTA where the matrix allows it.
int gemvm_pick_kw(int tiles, int groups, int grid, int max_kw) {
    int best = 1;
    double best_cost = 1e300;
    const int lim = groups < max_kw ? groups : max_kw;
    for (int kw = 1; kw <= lim; ++kw) {
        const long long T = (long long)tiles * kw;
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
    if (p.cols > gemvm_max_cols()) return cudaErrorInvalidValue;
    JINF_GEMVM_DISPATCH(launch_m, p, grid, s, pdl)
    return cudaErrorInvalidValue;
}

cudaError_t q4m_repack(const void* aos, void* dst, const Q4MShape& sh, cudaStream_t s) {
    const int64_t n = (int64_t)sh.tiles * sh.groups * 32;
    k_repack_q4m<<<(unsigned)((n + 255) / 256), 256, 0, s>>>((const uint8_t*)aos, (uint8_t*)dst, sh.rows, sh.groups,
                                                             sh.tiles);
    return cudaGetLastError();
}

}  // namespace jinf
