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
struct Frag {
    uint4 q[Q4T_R];
    uint2 sc;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Asynchronous copy of this lane's share of a chunk (its R 16-byte nibble groups and its
// R fp16 scales) into the same offsets of a shared-memory slot. Each lane later reads
// back only the bytes it copied itself, so no warp-level synchronisation is needed.
__device__ __forceinline__ void copy_frag_async(uint32_t slot, const uint8_t* chunk, int lane) {
#pragma unroll
    for (int i = 0; i < Q4T_R; ++i) {
        const int off = (i * 32 + lane) * 16;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(slot + off), "l"(chunk + off) : "memory");
    }
    const int so = Q4T_R * 512 + lane * (Q4T_R * 2);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(slot + so), "l"(chunk + so) : "memory");
}

__device__ __forceinline__ void read_frag(uint32_t slot, int lane, Frag& f) {
#pragma unroll
    for (int i = 0; i < Q4T_R; ++i)
        asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(f.q[i].x), "=r"(f.q[i].y), "=r"(f.q[i].z), "=r"(f.q[i].w)
                     : "r"(slot + (i * 32 + lane) * 16));
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(f.sc.x), "=r"(f.sc.y)
                 : "r"(slot + Q4T_R * 512 + lane * (Q4T_R * 2)));
}

// Nibble pairs. A 16-byte group of a block is four words {w0, w1, w2, w3}; word j holds
// block elements 8j..8j+7 at bits 4*(e%8). The words are decoded two at a time:
// (w & (0xF << 4n)) | magic on w0 and on w1 gives the floats 2^23 + q*2^(4n) of elements
// (n, n+8) (n = 0..3); the same on {w0, w1} >> 16 (a 64-bit shift: only the low 16 bits
// of each half are used afterwards) gives elements (n+4, n+12). Subtracting
// 2^23 + 8*2^(4n) leaves (q-8)*2^(4n) exactly; x is staged pre-multiplied by 2^-(4n) in
// the same pair order, so each fma.f32x2 adds the fp32 products (q-8)*x of two elements.
template <int N>
__device__ __forceinline__ u64 bias_pair() {
    constexpr float c = -(8388608.f + 8.f * (float)(1 << (4 * N)));
    return ((u64)__float_as_uint(c) << 32) | (u64)__float_as_uint(c);
}

// The 8 element pairs of one word pair {wa, wb} (x pairs xp[0..7]), written as one PTX
// block so that each nibble costs exactly one lop3 ((w & mask) | magic) and each pair one
// add.f32x2 and one fma.f32x2.
#define JINF_PAIR(ACC, SRC_LO, SRC_HI, MASK, BIAS, XP)                   \
    "lop3.b32 t0, " SRC_LO ", " MASK ", 0x4B000000, 0xEA;\n\t"          \
    "lop3.b32 t1, " SRC_HI ", " MASK ", 0x4B000000, 0xEA;\n\t"          \
    "mov.b64 v, {t0, t1};\n\t"                                         \
    "add.rn.f32x2 v, v, " BIAS ";\n\t"                                 \
    "fma.rn.f32x2 " ACC ", v, " XP ", " ACC ";\n\t"

// Two independent accumulator chains (low and high nibble halves), summed by the caller.
__device__ __forceinline__ void mac_words(u64 w, const u64* xp, u64& acc0, u64& acc1) {
    const u64 b0 = bias_pair<0>(), b1 = bias_pair<1>(), b2 = bias_pair<2>(), b3 = bias_pair<3>();
    asm("{\n\t"
        ".reg .b32 wl, wh, hl, hh, t0, t1;\n\t"
        ".reg .b64 v, h;\n\t"
        "mov.b64 {wl, wh}, %2;\n\t"
        "shr.b64 h, %2, 16;\n\t"
        "mov.b64 {hl, hh}, h;\n\t"
        JINF_PAIR("%0", "wl", "wh", "0xF", "%11", "%3")
        JINF_PAIR("%1", "hl", "hh", "0xF", "%11", "%7")
        JINF_PAIR("%0", "wl", "wh", "0xF0", "%12", "%4")
        JINF_PAIR("%1", "hl", "hh", "0xF0", "%12", "%8")
        JINF_PAIR("%0", "wl", "wh", "0xF00", "%13", "%5")
        JINF_PAIR("%1", "hl", "hh", "0xF00", "%13", "%9")
        JINF_PAIR("%0", "wl", "wh", "0xF000", "%14", "%6")
        JINF_PAIR("%1", "hl", "hh", "0xF000", "%14", "%10")
        "}"
        : "+l"(acc0), "+l"(acc1)
        : "l"(w), "l"(xp[0]), "l"(xp[1]), "l"(xp[2]), "l"(xp[3]), "l"(xp[4]), "l"(xp[5]), "l"(xp[6]),
          "l"(xp[7]), "l"(b0), "l"(b1), "l"(b2), "l"(b3));
}
#undef JINF_PAIR

// acc[i] += d_i * sum_e (q_ie - 8) * x_e for one block of R rows; xb points at the
// block's 16 staged x pairs (36-float stride per block, see the prologue).
__device__ __forceinline__ void mac_frag(const Frag& f, const float* xb, float (&acc)[Q4T_R]) {
    u64 xp[16];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const float4 v = *reinterpret_cast<const float4*>(xb + 4 * j);
        xp[2 * j] = pkf(v.x, v.y);
        xp[2 * j + 1] = pkf(v.z, v.w);
    }
#pragma unroll
    for (int i = 0; i < Q4T_R; ++i) {
        u64 a0 = 0ull, a1 = 0ull;
        mac_words(pk(f.q[i].x, f.q[i].y), xp, a0, a1);
        mac_words(pk(f.q[i].z, f.q[i].w), xp + 8, a0, a1);
        const uint32_t sw = i < 2 ? f.sc.x : f.sc.y;
        const float d = jinf_h2f((uint16_t)((i & 1) ? (sw >> 16) : (sw & 0xffff)));
        float l0, h0, l1, h1;
        upk(a0, l0, h0);
        upk(a1, l1, h1);
        acc[i] = fmaf(d, (l0 + h0) + (l1 + h1), acc[i]);
    }
}

// Shared-memory slot (0..31) and pre-scale of block element e (0..31): element e of
// word j = e/8, nibble n = e%8, goes to pair k = 8*(j/2) + n, half j%2, scaled 2^-4(n%4).
__device__ __forceinline__ int x_slot(int e) {
    const int j = e >> 3, n = e & 7;
    return 2 * (8 * (j >> 1) + n) + (j & 1);
}
__device__ __forceinline__ float prescale(int e) {
    const int n = e & 3;
    return n == 0 ? 1.f : n == 1 ? 0.0625f : n == 2 ? 0.00390625f : 0.000244140625f;
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

// One warp owns one tile (RW rows x all columns) at a time and walks its S steps. The
// weight chunks stream through a per-warp ring of GEMV_NBUF shared-memory slots filled
// with cp.async (GEMV_NBUF - 1 chunks of 2304 bytes in flight per warp, no registers
// held), and no block-wide barrier is needed after the prologue. Lanes of a row group sum
// their partial dot products with xor shuffles; the lane with l == 0 runs the epilogue.
template <int LK, int XM, int EPI>
__global__ void __launch_bounds__(GEMV_THREADS) k_gemv_q4t(const GemvParams p) {
    constexpr int R = Q4T_R;
    constexpr int G = 32 / LK;
    constexpr int RW = R * G;
    constexpr int NW = GEMV_THREADS / 32;
    extern __shared__ __align__(16) float smem[];
    const int nb = p.cols / 32;
    float* xs = smem;               // [nb][36]
    float* misc = smem + nb * 36;   // scratch for reductions (64 floats)
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // per-warp ring of GEMV_NBUF chunk slots for the asynchronous weight stream
    const uint32_t ring = smem_u32(misc + 64) + (uint32_t)(warp * GEMV_NBUF * Q4T_CHUNK);

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
            xs[(i >> 5) * 36 + x_slot(i & 31)] = v * prescale(i);
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
            xs[(i >> 5) * 36 + x_slot(i & 31)] = h * r * p.norm_w[i] * prescale(i);
        }
    }
    __syncthreads();

    // ---------------- main loop: warp per tile, chunks streamed through a cp.async ring
    // The warp walks the chunk sequence of its tiles (tile t, steps 0..S-1, then tile
    // t + wstride, ...); the copy cursor runs GEMV_NBUF - 1 chunks ahead of the compute
    // cursor, across tile boundaries.
    const int S = p.steps;
    const int g = lane / LK, l = lane % LK;
    float lmax = -INFINITY;
    int lidx = 0;
    const int wstride = gridDim.x * NW;
    int tp = blockIdx.x * NW + warp, sp = 0;  // copy cursor
    auto issue = [&](int slot) {
        if (tp < p.tiles) {
            copy_frag_async(ring + slot * Q4T_CHUNK, p.w + ((size_t)tp * S + sp) * Q4T_CHUNK, lane);
            if (++sp == S) {
                sp = 0;
                tp += wstride;
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");  // possibly empty: keeps group counts uniform
    };
#pragma unroll
    for (int i = 0; i < GEMV_NBUF - 1; ++i) issue(i);
    float acc[R];
#pragma unroll
    for (int i = 0; i < R; ++i) acc[i] = 0.f;
    int slot = 0, sc = 0;
    for (int t = blockIdx.x * NW + warp; t < p.tiles;) {
        issue(slot == 0 ? GEMV_NBUF - 1 : slot - 1);
        asm volatile("cp.async.wait_group %0;" ::"n"(GEMV_NBUF - 1) : "memory");
        Frag f;
        read_frag(ring + slot * Q4T_CHUNK, lane, f);
        mac_frag(f, xs + (sc * LK + l) * 36, acc);
        slot = slot + 1 == GEMV_NBUF ? 0 : slot + 1;
        if (++sc < S) continue;

        // ---------------- tile done: reduce over the LK lanes of each row group
#pragma unroll
        for (int o = LK / 2; o >= 1; o >>= 1)
#pragma unroll
            for (int i = 0; i < R; ++i) acc[i] += __shfl_xor_sync(JINF_FULL_MASK, acc[i], o);
        if (l == 0) {
            // ---------------- epilogue: rows row0 .. row0+R-1 (R = 4 consecutive rows)
            const int row0 = t * RW + g * R;
            if (EPI == EPI_STORE || EPI == EPI_LMHEAD) {
#pragma unroll
                for (int i = 0; i < R; ++i) {
                    const int row = row0 + i;
                    if (row < p.rows) {
                        p.y[row] = acc[i];
                        if (EPI == EPI_LMHEAD && acc[i] > lmax) { lmax = acc[i]; lidx = row; }
                    }
                }
            } else {
#pragma unroll
                for (int pr = 0; pr < R / 2; ++pr) {
                    const int row = row0 + 2 * pr;
                    const float v0 = acc[2 * pr], v1 = acc[2 * pr + 1];
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
        }
#pragma unroll
        for (int i = 0; i < R; ++i) acc[i] = 0.f;
        sc = 0;
        t += wstride;
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
    (void)lk;
    return sizeof(float) * ((size_t)(cols / 32) * 36 + 64) + (size_t)(GEMV_THREADS / 32) * GEMV_NBUF * Q4T_CHUNK;
}

// Per-instantiation launch set-up (max dynamic shared memory, occupancy) is done once and
// cached, so repeated launches cost only the launch itself.
template <int LK, int XM, int EPI>
struct GemvKernelInfo {
    static int occupancy(int cols) {
        static int cached_cols = -1, cached_occ = 1;
        if (cached_cols != cols) {
            const size_t smem = gemv_smem_bytes(cols, LK);
            ensure_smem(smem);
            int n = 0;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_gemv_q4t<LK, XM, EPI>, GEMV_THREADS, smem) !=
                cudaSuccess || n < 1)
                n = 1;
            cached_cols = cols;
            cached_occ = n;
        }
        return cached_occ;
    }
    static cudaError_t ensure_smem(size_t smem) {
        static size_t configured = 0;
        if (smem <= configured) return cudaSuccess;
        // configure for the largest possible x staging once (cols <= 32768)
        const size_t want = smem > gemv_smem_bytes(32768, LK) ? smem : gemv_smem_bytes(32768, LK);
        cudaError_t e = cudaFuncSetAttribute(k_gemv_q4t<LK, XM, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)want);
        if (e == cudaSuccess) configured = want;
        return e;
    }
};

template <int LK, int XM, int EPI>
static cudaError_t launch_t(const GemvParams& p, int grid, cudaStream_t s, bool pdl) {
    const size_t smem = gemv_smem_bytes(p.cols, LK);
    cudaError_t e = GemvKernelInfo<LK, XM, EPI>::ensure_smem(smem);
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
    return GemvKernelInfo<LK, XM, EPI>::occupancy(cols);
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
    const int ctas = (p.tiles + GEMV_THREADS / 32 - 1) / (GEMV_THREADS / 32);
    auto occ_fn = [&]() -> int {
        JINF_GEMV_DISPATCH(occupancy_lk, p.lk, p.cols)
        return 1;
    };
    const int persistent = occ_fn() * num_sms;
    return ctas < persistent ? ctas : persistent;
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
