// Fused Q4_0 GEMV kernels over the Q4T layout (see q4t.cuh), sm_100a.
//
// One kernel template covers every projection of the decode step:
//   prologue  X_PLAIN        x given (fp32 or fp16)
//             X_RMSNORM      h = h_in + y_pending; x = rmsnorm(h) * gain   (CTA 0 stores h)
//             X_EMBED_NORM   h = token_embd[token];  x = rmsnorm(h) * gain (CTA 0 stores h)
//   epilogue  EPI_STORE      y[row]
//             EPI_QKV        RoPE on q/k pairs, q -> fp32, k/v -> fp16 KV cache at pos
//             EPI_GATEUP     rows interleaved (gate_n, up_n): h[n] = silu(gate_n) * up_n
//             EPI_LMHEAD     logits[row] and a packed (value, index) atomicMax argmax
//
// Arithmetic (reference cuda/matmul_kernels.cu:8-43 computes sum (q-8)*d*x in fp32):
// nibble q at bit position p of a word becomes the float 2^23 + q*2^p by OR-ing in the
// exponent of 2^23 (one LOP3), subtracting 2^23 + 8*2^p gives (q-8)*2^p exactly, and x
// is pre-scaled by 2^-p when it is staged in shared memory, so each product equals the
// fp32 product (q-8)*x. Adds and FMAs run two lanes at a time with sm_100's packed
// add.f32x2 / fma.rn.f32x2. The block scale multiplies the per-block sum once.
#include "common.cuh"
#include "q4t.cuh"
#include "gemv_q4t.h"

#include <math.h>

namespace jinf {

namespace {

typedef unsigned long long u64;

__device__ __forceinline__ u64 pk(uint32_t a, uint32_t b) {
    u64 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(a), "r"(b));
    return r;
}
__device__ __forceinline__ u64 pkf(float a, float b) { return pk(__float_as_uint(a), __float_as_uint(b)); }
__device__ __forceinline__ void upk(u64 v, float& a, float& b) {
    uint32_t x, y;
    asm("mov.b64 {%0, %1}, %2;" : "=r"(x), "=r"(y) : "l"(v));
    a = __uint_as_float(x);
    b = __uint_as_float(y);
}
__device__ __forceinline__ u64 add2(u64 a, u64 b) {
    u64 r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ u64 fma2(u64 a, u64 b, u64 c) {
    u64 r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}

constexpr uint32_t MAGIC = 0x4B000000u;  // exponent bits of 2^23
// bit position of nibble n (0..7) after the decode shifts: n<5 in place, n>=5 after >>12
__host__ __device__ constexpr int nib_shift(int n) { return n < 5 ? 4 * n : 4 * n - 12; }

struct Frag {
    uint4 q[Q4T_R];
    uint2 sc;
};

__device__ __forceinline__ void load_frag(const uint8_t* chunk, int lane, Frag& f) {
#pragma unroll
    for (int i = 0; i < Q4T_R; ++i) f.q[i] = ldg_stream_u4(chunk + (i * 32 + lane) * 16);
    f.sc = ldg_stream_u2(chunk + Q4T_R * 512 + lane * (Q4T_R * 2));
}

// acc[i] += d_i * sum_e (q_ie - 8) * x_e for one block; xb points at the prescaled,
// padded shared copy of the block's 32 inputs.
__device__ __forceinline__ void mac_frag(const Frag& f, const float* xb, float (&acc)[Q4T_R]) {
    const u64 c01 = pkf(-(8388608.f + 8.f * (1 << nib_shift(0))), -(8388608.f + 8.f * (1 << nib_shift(1))));
    const u64 c23 = pkf(-(8388608.f + 8.f * (1 << nib_shift(2))), -(8388608.f + 8.f * (1 << nib_shift(3))));
    const u64 c45 = pkf(-(8388608.f + 8.f * (1 << nib_shift(4))), -(8388608.f + 8.f * (1 << nib_shift(5))));
    const u64 c67 = pkf(-(8388608.f + 8.f * (1 << nib_shift(6))), -(8388608.f + 8.f * (1 << nib_shift(7))));
    u64 bacc[Q4T_R];
#pragma unroll
    for (int i = 0; i < Q4T_R; ++i) bacc[i] = 0ull;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        const float4 xa = *reinterpret_cast<const float4*>(xb + 8 * w);
        const float4 xc = *reinterpret_cast<const float4*>(xb + 8 * w + 4);
        const u64 x01 = pkf(xa.x, xa.y), x23 = pkf(xa.z, xa.w), x45 = pkf(xc.x, xc.y), x67 = pkf(xc.z, xc.w);
#pragma unroll
        for (int i = 0; i < Q4T_R; ++i) {
            const uint32_t wd = w == 0 ? f.q[i].x : w == 1 ? f.q[i].y : w == 2 ? f.q[i].z : f.q[i].w;
            const uint32_t hi = wd >> 12;
            const u64 v01 = pk((wd & 0xFu) | MAGIC, (wd & 0xF0u) | MAGIC);
            const u64 v23 = pk((wd & 0xF00u) | MAGIC, (wd & 0xF000u) | MAGIC);
            const u64 v45 = pk((wd & 0xF0000u) | MAGIC, (hi & 0xF00u) | MAGIC);
            const u64 v67 = pk((hi & 0xF000u) | MAGIC, (hi & 0xF0000u) | MAGIC);
            bacc[i] = fma2(add2(v01, c01), x01, bacc[i]);
            bacc[i] = fma2(add2(v23, c23), x23, bacc[i]);
            bacc[i] = fma2(add2(v45, c45), x45, bacc[i]);
            bacc[i] = fma2(add2(v67, c67), x67, bacc[i]);
        }
    }
    const uint32_t s01 = f.sc.x, s23 = f.sc.y;
#pragma unroll
    for (int i = 0; i < Q4T_R; ++i) {
        const uint32_t sw = i < 2 ? s01 : s23;
        const float d = jinf_h2f((uint16_t)((i & 1) ? (sw >> 16) : (sw & 0xffff)));
        float a, b;
        upk(bacc[i], a, b);
        acc[i] = fmaf(d, a + b, acc[i]);
    }
}

__device__ __forceinline__ float prescale(int e) {
    // 2^-p for block element e (p = nibble bit position after decode)
    const int n = e & 7;
    return n == 0 ? 1.f : n == 1 ? 0.0625f : (n == 2 || n == 5) ? 0.00390625f
         : (n == 3 || n == 6) ? 0.000244140625f : 0.0000152587890625f;
}

__device__ __forceinline__ uint32_t ordered_bits(float v) {
    const uint32_t b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ void l2_prefetch(const uint8_t* p, uint64_t bytes) {
    // bulk L2 prefetch, 16-byte granules, pieces of <= 1 MB
    uint64_t off = 0;
    while (off < bytes) {
        const uint64_t rem = bytes - off;
        const uint32_t n = (uint32_t)(rem < (1ull << 20) ? rem : (1ull << 20));
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p + off), "r"(n) : "memory");
        off += n;
    }
}

}  // namespace

template <int LK, int XM, int EPI>
__global__ void __launch_bounds__(GEMV_THREADS) k_gemv_q4t(const GemvParams p) {
    constexpr int R = Q4T_R;
    constexpr int G = 32 / LK;
    constexpr int RW = R * G;
    constexpr int NW = GEMV_THREADS / 32;
    extern __shared__ __align__(16) float smem[];
    const int nb = p.cols / 32;
    float* xs = smem;                 // [nb][36]
    float* red = smem + nb * 36;      // [NW][RW]
    float* misc = red + NW * RW;      // scratch for reductions (64 floats)
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    // Weights do not depend on the previous kernel: start streaming the next
    // projection's bytes into L2 before waiting for our inputs.
    if (tid == 0 && p.pf_bytes) {
        const uint64_t share = ((p.pf_bytes + gridDim.x - 1) / gridDim.x + 15) & ~15ull;
        const uint64_t off = share * blockIdx.x;
        if (off < p.pf_bytes) l2_prefetch(p.pf_ptr + off, share < p.pf_bytes - off ? share : p.pf_bytes - off);
    }
    pdl_wait();
    pdl_trigger();

    // ---------------- prologue: stage x (prescaled, 36-float stride per block)
    if (XM == X_PLAIN_F32 || XM == X_PLAIN_F16) {
        for (int i = tid; i < p.cols; i += GEMV_THREADS) {
            const float v = XM == X_PLAIN_F32 ? reinterpret_cast<const float*>(p.x)[i]
                                              : __half2float(reinterpret_cast<const __half*>(p.x)[i]);
            xs[(i >> 5) * 36 + (i & 31)] = v * prescale(i);
        }
    } else {
        const float* hsrc = p.hin;
        if (XM == X_EMBED_NORM) hsrc = p.embed + (size_t)p.st->token * p.cols;
        float ss = 0.f;
        for (int i = tid; i < p.cols; i += GEMV_THREADS) {
            float h = hsrc[i];
            if (XM == X_RMSNORM && p.yres) h += p.yres[i];
            ss = fmaf(h, h, ss);
        }
        ss = block_sum(ss, misc);
        const float r = rsqrtf(ss / (float)p.cols + p.eps);
        const bool store_h = blockIdx.x == 0 && p.hout;
        for (int i = tid; i < p.cols; i += GEMV_THREADS) {
            float h = hsrc[i];
            if (XM == X_RMSNORM && p.yres) h += p.yres[i];
            if (store_h) p.hout[i] = h;
            xs[(i >> 5) * 36 + (i & 31)] = h * r * p.norm_w[i] * prescale(i);
        }
    }
    __syncthreads();

    // ---------------- main loop: CTA = TPC tiles x KS step-lanes of warps
    const int S = p.steps;
    const int KS = S >= 8 ? 8 : S >= 4 ? 4 : S >= 2 ? 2 : 1;
    const int TPC = NW / KS;
    const int ti = warp / KS, ks = warp % KS;
    const int g = lane / LK, l = lane % LK;
    float lmax = -INFINITY;
    int lidx = 0;

    for (int tg = blockIdx.x; tg * TPC < p.tiles; tg += gridDim.x) {
        const int t = tg * TPC + ti;
        float acc[R];
#pragma unroll
        for (int i = 0; i < R; ++i) acc[i] = 0.f;
        if (t < p.tiles) {
            const uint8_t* tb = p.w + (size_t)t * S * Q4T_CHUNK;
            int s = ks;
            for (; s + KS < S; s += 2 * KS) {
                Frag f0, f1;
                load_frag(tb + (size_t)s * Q4T_CHUNK, lane, f0);
                load_frag(tb + (size_t)(s + KS) * Q4T_CHUNK, lane, f1);
                mac_frag(f0, xs + (s * LK + l) * 36, acc);
                mac_frag(f1, xs + ((s + KS) * LK + l) * 36, acc);
            }
            if (s < S) {
                Frag f0;
                load_frag(tb + (size_t)s * Q4T_CHUNK, lane, f0);
                mac_frag(f0, xs + (s * LK + l) * 36, acc);
            }
        }
#pragma unroll
        for (int o = LK / 2; o >= 1; o >>= 1)
#pragma unroll
            for (int i = 0; i < R; ++i) acc[i] += __shfl_xor_sync(JINF_FULL_MASK, acc[i], o);
        if (l == 0) {
#pragma unroll
            for (int i = 0; i < R; ++i) red[warp * RW + g * R + i] = acc[i];
        }
        __syncthreads();

        // ---------------- epilogue (fixed-order sum over the KS warps of a tile)
        const int nrows = TPC * RW;
        if (EPI == EPI_STORE || EPI == EPI_LMHEAD) {
            for (int j = tid; j < nrows; j += GEMV_THREADS) {
                const int tj = j / RW, r = j % RW;
                const int row = (tg * TPC + tj) * RW + r;
                float v = 0.f;
                for (int k = 0; k < KS; ++k) v += red[(tj * KS + k) * RW + r];
                if (row < p.rows) {
                    p.y[row] = v;
                    if (EPI == EPI_LMHEAD && v > lmax) { lmax = v; lidx = row; }
                }
            }
        } else {
            for (int j = tid; j < nrows / 2; j += GEMV_THREADS) {
                const int tj = (2 * j) / RW, r = (2 * j) % RW;
                const int row = (tg * TPC + tj) * RW + r;
                float v0 = 0.f, v1 = 0.f;
                for (int k = 0; k < KS; ++k) {
                    v0 += red[(tj * KS + k) * RW + r];
                    v1 += red[(tj * KS + k) * RW + r + 1];
                }
                if (row >= p.rows) continue;
                if (EPI == EPI_GATEUP) {
                    p.y[row >> 1] = v0 / (1.0f + expf(-v0)) * v1;
                } else {  // EPI_QKV
                    const int pos = p.st->pos;
                    if (row < p.nq + p.nk) {
                        const int rr = row < p.nq ? row : row - p.nq;
                        const int i = (rr % p.head_dim) >> 1;
                        const float theta = powf(p.rope_base, -2.0f * (float)i / (float)p.head_dim);
                        const float ang = (float)pos * theta;
                        const float c = cosf(ang), sn = sinf(ang);
                        const float o0 = v0 * c - v1 * sn, o1 = v0 * sn + v1 * c;
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
        __syncthreads();
    }

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

// One thread per (row, block) of the AoS source: 16 nibble bytes + the fp16 scale move
// to their Q4T positions. Padding rows must be zeroed by the caller beforehand.
__global__ void k_repack_q4t(const uint8_t* __restrict__ aos, uint8_t* __restrict__ dst, int rows, int nb,
                             int lk, int steps) {
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (int64_t)rows * nb) return;
    const int r = (int)(gid / nb), b = (int)(gid % nb);
    const int rw = Q4T_R * (32 / lk);
    const int t = r / rw, g = (r % rw) / Q4T_R, i = r % Q4T_R;
    const int s = b / lk, l = b % lk;
    const int lam = g * lk + l;
    uint8_t* chunk = dst + ((size_t)t * steps + s) * Q4T_CHUNK;
    const uint8_t* src = aos + gid * 18;
    uint8_t* nib = chunk + (i * 32 + lam) * 16;
#pragma unroll
    for (int k = 0; k < 16; ++k) nib[k] = src[2 + k];
    uint8_t* sc = chunk + Q4T_R * 512 + (lam * Q4T_R + i) * 2;
    sc[0] = src[0];
    sc[1] = src[1];
}

// ---------------------------------------------------------------- host side

size_t gemv_smem_bytes(int cols, int lk) {
    const int nb = cols / 32;
    const int rw = Q4T_R * (32 / lk);
    return sizeof(float) * ((size_t)nb * 36 + (GEMV_THREADS / 32) * rw + 64);
}

template <int LK, int XM, int EPI>
static cudaError_t launch_t(const GemvParams& p, int grid, cudaStream_t s, bool pdl) {
    const size_t smem = gemv_smem_bytes(p.cols, LK);
    cudaError_t e = cudaFuncSetAttribute(k_gemv_q4t<LK, XM, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(GEMV_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_gemv_q4t<LK, XM, EPI>, p);
}

template <int XM, int EPI>
static cudaError_t launch_lk(const GemvParams& p, int grid, cudaStream_t s, bool pdl) {
    switch (p.lk) {
        case 32: return launch_t<32, XM, EPI>(p, grid, s, pdl);
        case 16: return launch_t<16, XM, EPI>(p, grid, s, pdl);
        case 8:  return launch_t<8, XM, EPI>(p, grid, s, pdl);
        case 4:  return launch_t<4, XM, EPI>(p, grid, s, pdl);
        default: return cudaErrorInvalidValue;
    }
}

template <int LK, int XM, int EPI>
static int occupancy_t(int cols) {
    const size_t smem = gemv_smem_bytes(cols, LK);
    cudaFuncSetAttribute(k_gemv_q4t<LK, XM, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_gemv_q4t<LK, XM, EPI>, GEMV_THREADS, smem) != cudaSuccess)
        return 1;
    return n > 0 ? n : 1;
}

template <int XM, int EPI>
static int occupancy_lk(int lk, int cols) {
    switch (lk) {
        case 32: return occupancy_t<32, XM, EPI>(cols);
        case 16: return occupancy_t<16, XM, EPI>(cols);
        case 8:  return occupancy_t<8, XM, EPI>(cols);
        default: return occupancy_t<4, XM, EPI>(cols);
    }
}

#define JINF_GEMV_DISPATCH(FN, ...)                                                    \
    switch (xm * 16 + epi) {                                                           \
        case X_PLAIN_F32 * 16 + EPI_STORE:   return FN<X_PLAIN_F32, EPI_STORE>(__VA_ARGS__);   \
        case X_PLAIN_F16 * 16 + EPI_STORE:   return FN<X_PLAIN_F16, EPI_STORE>(__VA_ARGS__);   \
        case X_RMSNORM * 16 + EPI_STORE:     return FN<X_RMSNORM, EPI_STORE>(__VA_ARGS__);     \
        case X_RMSNORM * 16 + EPI_QKV:       return FN<X_RMSNORM, EPI_QKV>(__VA_ARGS__);       \
        case X_EMBED_NORM * 16 + EPI_QKV:    return FN<X_EMBED_NORM, EPI_QKV>(__VA_ARGS__);    \
        case X_RMSNORM * 16 + EPI_GATEUP:    return FN<X_RMSNORM, EPI_GATEUP>(__VA_ARGS__);    \
        case X_PLAIN_F32 * 16 + EPI_GATEUP:  return FN<X_PLAIN_F32, EPI_GATEUP>(__VA_ARGS__);  \
        case X_RMSNORM * 16 + EPI_LMHEAD:    return FN<X_RMSNORM, EPI_LMHEAD>(__VA_ARGS__);    \
        case X_PLAIN_F32 * 16 + EPI_LMHEAD:  return FN<X_PLAIN_F32, EPI_LMHEAD>(__VA_ARGS__);  \
        default: break;                                                                \
    }

int gemv_grid(const GemvParams& p, int xm, int epi, int num_sms) {
    const int S = p.steps;
    const int KS = S >= 8 ? 8 : S >= 4 ? 4 : S >= 2 ? 2 : 1;
    const int tpc = (GEMV_THREADS / 32) / KS;
    const int groups = (p.tiles + tpc - 1) / tpc;
    int occ = 1;
    auto occ_fn = [&]() -> int {
        JINF_GEMV_DISPATCH(occupancy_lk, p.lk, p.cols)
        return 1;
    };
    occ = occ_fn();
    const int persistent = occ * num_sms;
    return groups < persistent ? groups : persistent;
}

cudaError_t gemv_launch(const GemvParams& p, int xm, int epi, int grid, cudaStream_t s, bool pdl) {
    JINF_GEMV_DISPATCH(launch_lk, p, grid, s, pdl)
    return cudaErrorInvalidValue;
}

cudaError_t q4t_repack(const void* aos, void* dst, const Q4TShape& sh, cudaStream_t s) {
    cudaError_t e = cudaMemsetAsync(dst, 0, sh.bytes, s);
    if (e != cudaSuccess) return e;
    const int64_t n = (int64_t)sh.rows * sh.nb;
    k_repack_q4t<<<(unsigned)((n + 255) / 256), 256, 0, s>>>((const uint8_t*)aos, (uint8_t*)dst, sh.rows, sh.nb,
                                                             sh.lk, sh.steps);
    return cudaGetLastError();
}

}  // namespace jinf
