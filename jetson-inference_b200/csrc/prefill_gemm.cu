// Batched prefill GEMM on the 5th-generation tensor cores (sm_100a: tcgen05.mma with the
// accumulator in tensor memory, B operand by TMA).
//
//   Y[t][m] = tok_scale[t] * sum_k X[t][k] * W[m][k]      t < T tokens, m < M rows, k < K
//
// W is a Q4M matrix (q4m.cuh: the lossless repack of the reference's Q4_0 blocks, reference
// include/jinf/quant.h:31-35, value (q - 8) * d, src/quant.cpp:49-60). X is fp16 [T][K], each
// token's row prescaled by a power of two (prefill.cu) so that fp16 keeps its precision
// whatever the activation's range, and tok_scale undoes it. This replaces the reference's
// prompt loop, which runs every prompt token through the whole model one at a time
// (src/engine.cpp:690-751), by one contraction per projection over all prompt tokens.
//
// One CTA computes a 128-row x 128-token tile of Y over all of K, 128 columns (one Q4M group)
// per pipeline stage, 3 stages:
//   warp 0 (one lane)  copies the stage's four raw 2304-byte Q4M units (cp.async.bulk) and
//                      the two 64-column boxes of X (TMA tiled load, 128B swizzle) into
//                      shared memory, completing on the stage's `full` mbarrier;
//   warps 2..15        dequantise the raw units into the fp16 A tile (K-major, 128B swizzle,
//                      the canonical UMMA layout), then arrive on `aready`;
//   warp 1             allocates 128 TMEM columns; one lane issues 8 tcgen05.mma (M 128,
//                      N 128, K 16, f16 x f16 -> f32) per stage and commits each stage's MMAs
//                      to its `empty` mbarrier, which frees the stage for the next copies;
//   warps 4..7         after the last stage, read the accumulator (tcgen05.ld, one TMEM lane
//                      quarter per warp) and store Y (or add it to Y: the residual add).
// Every mbarrier wait is bounded: a wait that runs out records an error in *err, the CTA
// stops issuing work, lets its copies and MMAs in flight finish (bounded again), frees its
// tensor memory and returns.
#include "common.cuh"
#include "q4m.cuh"
#include "prefill.h"

#include <cuda.h>
#include <cuda_fp16.h>

namespace jinf {
namespace {

constexpr int PG_BM = 128, PG_BN = 128, PG_BK = 128, PG_STAGES = 3, PG_THREADS = 512;
constexpr int PG_ATOM = 16384;                        // one 64-column swizzle atom of a 128-row tile
constexpr int PG_A_BYTES = 2 * PG_ATOM;               // 128 rows x 128 columns fp16
constexpr int PG_B_BYTES = 2 * PG_ATOM;               // 128 tokens x 128 columns fp16
constexpr int PG_RAW_BYTES = 4 * Q4M_UNIT;            // four tile pairs of one group
constexpr int PG_DQ_THREADS = 448;                    // warps 2..15
constexpr unsigned long long PG_SPIN = 1ull << 22;    // polls of a wait before it gives up

// shared memory offsets from the 1024-aligned base
constexpr int PG_OFF_A = 0;
constexpr int PG_OFF_B = PG_OFF_A + PG_STAGES * PG_A_BYTES;
constexpr int PG_OFF_RAW = PG_OFF_B + PG_STAGES * PG_B_BYTES;
constexpr int PG_OFF_BAR = PG_OFF_RAW + PG_STAGES * PG_RAW_BYTES;
constexpr int PG_SMEM = PG_OFF_BAR + 256 + 1024;      // + barriers + alignment slack

__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mb_init(uint32_t b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(b), "r"(count) : "memory");
}
__device__ __forceinline__ void mb_expect(uint32_t b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(b), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mb_arrive(uint32_t b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(b) : "memory");
}
// Bounded wait for phase `parity` of the mbarrier; false when it ran out.
__device__ __forceinline__ bool mb_wait(uint32_t b, uint32_t parity) {
    for (unsigned long long it = 0; it < PG_SPIN; ++it) {
        uint32_t ok;
        asm volatile(
            "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
            : "=r"(ok)
            : "r"(b), "r"(parity)
            : "memory");
        if (ok) return true;
        if (it > 64) __nanosleep(64);
    }
    return false;
}

// raw bytes global -> shared on an mbarrier (16-byte aligned, a multiple of 16 bytes)
__device__ __forceinline__ void bulk_copy(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
// one box of the 2-D tensor map (x: column, y: token) into shared memory, this GPU's own memory
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"(map), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

// UMMA shared-memory descriptor of a K-major, 128B-swizzled operand: start address, leading
// byte offset 16 (unused with this swizzle), stride byte offset 1024 (eight 128-byte rows),
// descriptor version 1, swizzle mode 2 (128B).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor of kind::f16: f32 accumulator, f16 A and B, both K-major, N 128, M 128.
constexpr uint32_t PG_IDESC = (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(PG_BN >> 3) << 17) |
                              ((uint32_t)(PG_BM >> 4) << 24);

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(PG_IDESC), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// (q - 8) * d for the four bytes of a word, low nibbles (tile A row) or high nibbles (tile B
// row): two half2 in k order. 0x6400 | q is the fp16 1024 + q, so subtracting 1032 gives q - 8
// exactly; the product with d is rounded once, to fp16.
__device__ __forceinline__ void nib_to_half(uint32_t nib, __half2 d2, __half2& h01, __half2& h23) {
    const uint32_t a = __byte_perm(nib, 0x64646464u, 0x4140);  // bytes q0, 0x64, q1, 0x64
    const uint32_t b = __byte_perm(nib, 0x64646464u, 0x4342);  // q2, 0x64, q3, 0x64
    const __half2 off = __float2half2_rn(1032.f);
    h01 = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&a), off), d2);
    h23 = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&b), off), d2);
}

// Dequantise one stage: the raw units of pairs pp = 0..3 (raw + 2304 pp, `npairs` valid) into
// the A tile (two 64-column atoms). Item (pp, rr, kc) covers rows rr and 16 + rr of pair pp
// (tile A and tile B) at columns 8 kc .. 8 kc + 7 of the group: two nibble words of the unit
// and the two rows' block scales (q4m.cuh: word i of block j of lane 4 gr + c holds rows gr
// (i even) or gr + 8 (i odd), columns 4c .. 4c + 3 (+16 for i >= 2)).
__device__ __forceinline__ void dequant_stage(const uint8_t* raw, uint8_t* A, int npairs, int t) {
    for (int item = t; item < 4 * 16 * 16; item += PG_DQ_THREADS) {
        const int pp = item >> 8, rr = (item >> 4) & 15, kc = item & 15;
        const int gr = rr & 7, h8 = rr >> 3, j = kc >> 2, kq = kc & 3;
        const int i = ((kq >> 1) << 1) | h8, c0 = (kq & 1) << 1;
        uint4 va = make_uint4(0u, 0u, 0u, 0u), vb = va;
        if (pp < npairs) {
            const uint8_t* u = raw + pp * Q4M_UNIT;
            const uint32_t w0 = *reinterpret_cast<const uint32_t*>(u + 512 * j + 16 * (4 * gr + c0) + 4 * i);
            const uint32_t w1 = *reinterpret_cast<const uint32_t*>(u + 512 * j + 16 * (4 * gr + c0 + 1) + 4 * i);
            const __half da = *reinterpret_cast<const __half*>(u + Q4M_SCALES + 4 * (4 * gr + j) + 2 * h8);
            const __half db = *reinterpret_cast<const __half*>(u + Q4M_SCALES + 128 + 4 * (4 * gr + j) + 2 * h8);
            const __half2 da2 = __halves2half2(da, da), db2 = __halves2half2(db, db);
            __half2 a0, a1, a2, a3, b0, b1, b2, b3;
            nib_to_half(w0 & 0x0F0F0F0Fu, da2, a0, a1);
            nib_to_half(w1 & 0x0F0F0F0Fu, da2, a2, a3);
            nib_to_half((w0 >> 4) & 0x0F0F0F0Fu, db2, b0, b1);
            nib_to_half((w1 >> 4) & 0x0F0F0F0Fu, db2, b2, b3);
            va = make_uint4(*reinterpret_cast<uint32_t*>(&a0), *reinterpret_cast<uint32_t*>(&a1),
                            *reinterpret_cast<uint32_t*>(&a2), *reinterpret_cast<uint32_t*>(&a3));
            vb = make_uint4(*reinterpret_cast<uint32_t*>(&b0), *reinterpret_cast<uint32_t*>(&b1),
                            *reinterpret_cast<uint32_t*>(&b2), *reinterpret_cast<uint32_t*>(&b3));
        }
        // rows RA (tile A) and RA + 16 (tile B); 16-byte chunk cc of atom kk, swizzled by row % 8
        const int ra = 32 * pp + gr + 8 * h8, rb = ra + 16, kk = kc >> 3, cc = kc & 7;
        uint8_t* atom = A + kk * PG_ATOM;
        *reinterpret_cast<uint4*>(atom + (ra >> 3) * 1024 + (ra & 7) * 128 + ((cc ^ (ra & 7)) << 4)) = va;
        *reinterpret_cast<uint4*>(atom + (rb >> 3) * 1024 + (rb & 7) * 128 + ((cc ^ (rb & 7)) << 4)) = vb;
    }
}

__global__ void __launch_bounds__(PG_THREADS, 1)
    k_prefill_gemm(const __grid_constant__ CUtensorMap tmx, const uint8_t* __restrict__ w, int rows, int pairs,
                   int groups, int T, float* __restrict__ y, int ldy, const float* __restrict__ tok_scale, int accum, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* sA = smem + PG_OFF_A;
    uint8_t* sB = smem + PG_OFF_B;
    uint8_t* sRaw = smem + PG_OFF_RAW;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + PG_OFF_BAR);  // full[3] aready[3] empty[3] acc drain
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
    int* abort_flag = reinterpret_cast<int*>(bars + 17);
    const uint32_t b_full = su32(bars), b_aready = su32(bars + 3), b_empty = su32(bars + 6), b_acc = su32(bars + 9),
                   b_drain = su32(bars + 10);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t0 = blockIdx.x * PG_BN, p0 = blockIdx.y * 4;
    const int npairs = min(4, pairs - p0);

    if (tid == 0) {
        for (int s = 0; s < PG_STAGES; ++s) {
            mb_init(b_full + 8 * s, 1);
            mb_init(b_aready + 8 * s, PG_DQ_THREADS);
            mb_init(b_empty + 8 * s, 1);
        }
        mb_init(b_acc, 1);
        mb_init(b_drain, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {  // 128 fp32 columns of tensor memory: the 128 x 128 accumulator
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 128;" ::"r"(su32(tmem_slot))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    auto fail = [&]() {
        atomicExch(abort_flag, 1);
        atomicCAS(err, 0, 1);
    };

    if (warp == 0) {
        if (lane == 0) {  // ---- copies
            const uint32_t tx = (uint32_t)npairs * Q4M_UNIT + PG_B_BYTES;
            for (int kt = 0; kt < groups; ++kt) {
                const int s = kt % PG_STAGES;
                if (kt >= PG_STAGES && !mb_wait(b_empty + 8 * s, ((kt / PG_STAGES) - 1) & 1)) {
                    fail();
                    break;
                }
                if (*(volatile int*)abort_flag) break;
                mb_expect(b_full + 8 * s, tx);
                for (int pp = 0; pp < npairs; ++pp)
                    bulk_copy(su32(sRaw + s * PG_RAW_BYTES + pp * Q4M_UNIT),
                              w + ((size_t)(p0 + pp) * groups + kt) * Q4M_UNIT, Q4M_UNIT, b_full + 8 * s);
                tma_load_2d(su32(sB + s * PG_B_BYTES), &tmx, kt * PG_BK, t0, b_full + 8 * s);
                tma_load_2d(su32(sB + s * PG_B_BYTES + PG_ATOM), &tmx, kt * PG_BK + 64, t0, b_full + 8 * s);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {  // ---- MMAs
            int issued = 0;
            for (int kt = 0; kt < groups; ++kt) {
                const int s = kt % PG_STAGES;
                // the stage's X box (TMA) and its dequantised weights
                if (!mb_wait(b_full + 8 * s, (kt / PG_STAGES) & 1) || !mb_wait(b_aready + 8 * s, (kt / PG_STAGES) & 1)) {
                    fail();
                    break;
                }
                if (*(volatile int*)abort_flag) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t a0 = su32(sA + s * PG_A_BYTES), bb0 = su32(sB + s * PG_B_BYTES);
#pragma unroll
                for (int kk = 0; kk < PG_BK / 16; ++kk) {
                    const uint32_t off = (uint32_t)((kk >> 2) * PG_ATOM + (kk & 3) * 32);
                    umma_f16(tmem, umma_desc(a0 + off), umma_desc(bb0 + off), (kt | kk) ? 1u : 0u);
                }
                umma_commit(b_empty + 8 * s);
                ++issued;
            }
            if (issued == groups) {
                umma_commit(b_acc);
            } else {
                umma_commit(b_drain);  // the MMAs already issued finish before the memory goes
                mb_wait(b_drain, 0);
            }
        }
    } else {
        // ---- dequantisation (warps 2..15)
        const int t = tid - 64;
        for (int kt = 0; kt < groups; ++kt) {
            const int s = kt % PG_STAGES;
            if (!mb_wait(b_full + 8 * s, (kt / PG_STAGES) & 1)) {
                fail();
                break;
            }
            if (*(volatile int*)abort_flag) break;
            dequant_stage(sRaw + s * PG_RAW_BYTES, sA + s * PG_A_BYTES, npairs, t);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor core reads
            mb_arrive(b_aready + 8 * s);
        }
        // ---- epilogue (warps 4..7: TMEM lane quarter warp % 4)
        if (warp >= 4 && warp < 8) {
            const bool ok = !*(volatile int*)abort_flag && mb_wait(b_acc, 0);
            if (!ok) {
                fail();
            } else {
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const int q = warp & 3;
                const int row = p0 * 32 + 32 * q + lane;
                for (int c0 = 0; c0 < PG_BN; c0 += 32) {
                    uint32_t v[32];
                    const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0;
                    asm volatile(
                        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
                        "%13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, "
                        "[%32];"
                        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
                          "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]),
                          "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]),
                          "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
                        : "r"(taddr));
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                    if (row < rows) {
#pragma unroll
                        for (int jj = 0; jj < 32; ++jj) {
                            const int tok = t0 + c0 + jj;
                            if (tok < T) {
                                float* py = y + (size_t)tok * ldy + row;
                                const float val = __uint_as_float(v[jj]) * tok_scale[tok];
                                *py = accum ? *py + val : val;
                            }
                        }
                    }
                }
            }
        }
    }
    // leave: the copies of the stages the copier armed have landed (a CTA that gave up waits for
    // them, bounded) and the MMAs are done (accumulator read or drained), then free the memory
    __syncthreads();
    if (tid == 0 && *(volatile int*)abort_flag) {
        for (int s = 0; s < PG_STAGES; ++s) {
            const int last = ((groups - 1 - s) / PG_STAGES);  // phases armed on stage s (at most)
            if (s < groups) mb_wait(b_full + 8 * s, last & 1);
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 128;" ::"r"(tmem) : "memory");
    }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
    }
    return fn;
}

}  // namespace

size_t prefill_gemm_smem_bytes() { return PG_SMEM; }

cudaError_t prefill_gemm_launch(const uint8_t* w, int rows, int cols, const __half* x, int T, const float* tok_scale,
                                float* y, int ldy, int accum, int* err, cudaStream_t s) {
    Q4MShape sh;
    if (!w || !x || !y || !tok_scale || !err || T <= 0 || !q4m_shape(rows, cols, &sh) || ldy < rows)
        return cudaErrorInvalidValue;
    // TMA: the global base 16-byte aligned, the row stride a multiple of 16 bytes
    if (((uintptr_t)x & 15) || (cols * 2) % 16) return cudaErrorInvalidValue;
    EncodeTiledFn enc = encode_tiled();
    if (!enc) return cudaErrorNotSupported;
    CUtensorMap map;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)T};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)PG_BN};
    const cuuint32_t estr[2] = {1, 1};
    if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void*)x, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    static int configured = 0;
    if (!configured) {
        const cudaError_t e = cudaFuncSetAttribute(k_prefill_gemm, cudaFuncAttributeMaxDynamicSharedMemorySize, PG_SMEM);
        if (e != cudaSuccess) return e;
        configured = 1;
    }
    const dim3 grid((unsigned)((T + PG_BN - 1) / PG_BN), (unsigned)((sh.pairs + 3) / 4));
    k_prefill_gemm<<<grid, PG_THREADS, PG_SMEM, s>>>(map, w, rows, sh.pairs, sh.groups, T, y, ldy, tok_scale, accum,
                                                     err);
    return cudaGetLastError();
}

}  // namespace jinf
