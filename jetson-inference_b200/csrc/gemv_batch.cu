// Batched Q4_0 GEMV over the Q4M layout (BASELINE config C2 at batch 4 and 8): Y[b] = W x[b]
// for up to 8 input vectors with one pass over W. The reference has no batched form; at
// batch 1 this is jinf_b200_gemv_q4m.
//
// Arithmetic as in q4m_device.cuh, with the B operand's 8 columns holding (vector v, digit
// h) of 4 vectors (column 2v + h) instead of (block, digit) of 4 blocks: one m16n8k32 step
// multiplies a block of both tiles' rows by 4 vectors' digits, and the accumulator columns
// (2c, 2c+1) of a lane are vector c's hi and lo block sums. Each block is finished on its
// own (its scale differs per row and its digit scale per vector): the step starts from the
// vector's zero-point offsets and the block adds d (256 D_hi + D_lo) / alpha to the lane's
// rows. Batches of 5..8 take a second step per block for vectors 4..7. A lane ends a task
// with complete sums for rows gr, gr+8, 16+gr, 24+gr of the tile pair for its vector(s).
//
// Scheduling: CTA c works on K part kp = c % kw only (so it stages just that part's input
// records, B x ceil(G / kw) groups) and its warps take tile pairs round-robin; with kw > 1
// each task leaves B x 32 partial sums in the workspace and the last K part of a pair (arrival
// counter, reset by it) adds them in K order: deterministic.
#include "common.cuh"
#include "gemv.h"
#include "jinf/b200.h"
#include "jinf/quant.h"
#include "q4m.cuh"
#include "q4m_device.cuh"

namespace jinf {

using namespace q4mdev;

namespace {

constexpr int BT = 512;        // threads per CTA
constexpr int BNW = BT / 32;
constexpr int BNBUF = 4;       // ring slots per warp
constexpr int kBatchMaxKw = 32;

struct BatchParams {
    const uint8_t* w;
    int rows, cols, pairs, groups, batch, kw, gk;  // gk: groups per K part (max)
    const void* x;  // [batch][cols] fp32 or fp16
    int x_f16;
    float* y;       // [batch][rows]
    float* part;    // [pairs][kw][batch][32]
    unsigned* cnt;  // [pairs]
};

// Staged records: digits [batch][gk][256 B] then params [batch][gk][4][16 B], each vector's
// run padded (digits +64 B, params +16 B) so that the lanes of one load that read different
// vectors fall in different shared-memory banks.
__host__ __device__ inline int batch_dig_stride(int gk) { return gk * 256 + 64; }  // bytes per vector
__host__ __device__ inline int batch_prm_stride(int gk) { return gk * 64 + 16; }
__host__ __device__ inline size_t batch_rec_bytes(int batch, int gk) {
    return (size_t)batch * (batch_dig_stride(gk) + batch_prm_stride(gk));
}

// One unit against the staged groups `gl` (local index) of vectors 4 vb .. 4 vb + 3:
// lane (gr, c) adds vector 4 vb + c's block sums of rows gr, gr+8 (tile A) and 16+gr, 24+gr
// (tile B) into acc.
__device__ __forceinline__ void unit_batch(const uint32_t (&w)[16], const uint32_t (&sa)[4], const uint32_t (&sb)[4],
                                           uint32_t dig, uint32_t prm, int gk, int gl, int vb, int batch, int lane,
                                           float (&acc)[4]) {
    const int gr = lane >> 2, c = lane & 3;
    const int v = 4 * vb + (gr >> 1), h = gr & 1;  // this lane's B column: digit h of vector v
    const int vo = 4 * vb + c;                     // this lane's accumulator vector
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint32_t b0 = 0u, b1 = 0u;
        if (v < batch)
            asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];"
                         : "=r"(b0), "=r"(b1)
                         : "r"(dig + (uint32_t)(v * batch_dig_stride(gk) + gl * 256 + ((2 * j + h) * 4 + c) * 8)));
        int kh = 0, kl = 0;
        float ia = 0.f, ib = 0.f;
        if (vo < batch)
            asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(kh), "=r"(kl), "=f"(ia), "=f"(ib)
                         : "r"(prm + (uint32_t)(vo * batch_prm_stride(gk) + (gl * 4 + j) * 16)));
        int da[4] = {kh, kl, kh, kl};
        int db[4] = {kh * 16, kl * 16, kh * 16, kl * 16};
        mma_u8s8(nib_lo(w[4 * j]), nib_lo(w[4 * j + 1]), nib_lo(w[4 * j + 2]), nib_lo(w[4 * j + 3]), b0, b1, da);
        mma_u8s8(nib_hi(w[4 * j]), nib_hi(w[4 * j + 1]), nib_hi(w[4 * j + 2]), nib_hi(w[4 * j + 3]), b0, b1, db);
        acc[0] = fmaf(jinf_h2f((uint16_t)(sa[j] & 0xffffu)) * ia, (float)(da[0] * 256 + da[1]), acc[0]);
        acc[1] = fmaf(jinf_h2f((uint16_t)(sa[j] >> 16)) * ia, (float)(da[2] * 256 + da[3]), acc[1]);
        acc[2] = fmaf(jinf_h2f((uint16_t)(sb[j] & 0xffffu)) * ib, (float)(db[0] * 256 + db[1]), acc[2]);
        acc[3] = fmaf(jinf_h2f((uint16_t)(sb[j] >> 16)) * ib, (float)(db[2] * 256 + db[3]), acc[3]);
    }
}

template <int NVB>  // vector blocks of 4 (1: batch <= 4, 2: batch <= 8)
__global__ void __launch_bounds__(BT, 1) k_gemv_q4m_batch(const BatchParams p) {
    extern __shared__ __align__(16) uint8_t smem_b[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = p.groups, kw = p.kw, gk = p.gk;
    const int kp = blockIdx.x % kw, cgrid = gridDim.x / kw, cidx = blockIdx.x / kw;
    const int g0 = kp * G / kw, g1 = (kp + 1) * G / kw, ng = g1 - g0;
    uint8_t* rec = smem_b;  // digits, then params (batch_rec_bytes)
    uint32_t* dig = reinterpret_cast<uint32_t*>(rec);
    float4* prm = reinterpret_cast<float4*>(rec + (size_t)p.batch * batch_dig_stride(gk));
    const uint32_t ring = smem_u32(rec + batch_rec_bytes(p.batch, gk)) + (uint32_t)(warp * BNBUF * Q4M_UNIT);

    // tasks of this warp: tile pairs q = cidx + (warp + BNW i) cgrid, all ng groups of K part kp
    int tq = cidx + warp * cgrid, cg = 0;  // copy cursor
    auto issue = [&](int slot) {
        if (tq < p.pairs) {
            copy_unit_async(ring + slot * Q4M_UNIT, p.w + ((size_t)tq * G + g0 + cg) * Q4M_UNIT, lane);
            if (++cg == ng) {
                cg = 0;
                tq += BNW * cgrid;
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
#pragma unroll
    for (int i = 0; i < BNBUF - 1; ++i) issue(i);

    // records of groups [g0, g1) of every vector (one octet per block, 4 blocks per warp pass)
    const int n4 = p.cols / 4;
    for (int it = warp; it < p.batch * ng; it += BNW) {
        const int b = it / ng, gl = it % ng, g = g0 + gl;
        const int i4 = g * 32 + lane;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i4 < n4) {
            if (p.x_f16) {
                const uint2 hv = reinterpret_cast<const uint2*>(p.x)[(size_t)b * n4 + i4];
                const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&hv.x));
                const float2 c2 = __half22float2(*reinterpret_cast<const __half2*>(&hv.y));
                v = make_float4(a.x, a.y, c2.x, c2.y);
            } else {
                v = reinterpret_cast<const float4*>(p.x)[(size_t)b * n4 + i4];
            }
        }
        octet_to_records(v, lane, lane >> 3, dig + (b * batch_dig_stride(gk) + gl * 256) / 4,
                         prm + (b * batch_prm_stride(gk) + gl * 64) / 16);
    }
    __syncthreads();
    const uint32_t dig_s = smem_u32(dig), prm_s = smem_u32(prm);

    int slot = 0;
    const int gr = lane >> 2, c = lane & 3;
    for (int q = cidx + warp * cgrid; q < p.pairs; q += BNW * cgrid) {
        float acc[NVB][4];
#pragma unroll
        for (int vb = 0; vb < NVB; ++vb)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[vb][i] = 0.f;
        for (int gl = 0; gl < ng; ++gl) {
            issue(slot == 0 ? BNBUF - 1 : slot - 1);
            asm volatile("cp.async.wait_group %0;" ::"n"(BNBUF - 1) : "memory");
            __syncwarp();  // the block scales of every block are read across lanes
            const uint32_t sl = ring + slot * Q4M_UNIT;
            uint32_t w[16], sa[4], sb[4];
#pragma unroll
            for (int j = 0; j < 4; ++j)
                asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                             : "=r"(w[4 * j]), "=r"(w[4 * j + 1]), "=r"(w[4 * j + 2]), "=r"(w[4 * j + 3])
                             : "r"(sl + 512 * j + lane * 16));
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                asm volatile("ld.shared.u32 %0, [%1];" : "=r"(sa[j]) : "r"(sl + Q4M_SCALES + (4 * gr + j) * 4));
                asm volatile("ld.shared.u32 %0, [%1];" : "=r"(sb[j]) : "r"(sl + Q4M_SCALES + 128 + (4 * gr + j) * 4));
            }
            __syncwarp();  // every lane's reads of the slot precede the next copy into it
#pragma unroll
            for (int vb = 0; vb < NVB; ++vb) unit_batch(w, sa, sb, dig_s, prm_s, gk, gl, vb, p.batch, lane, acc[vb]);
            slot = slot + 1 == BNBUF ? 0 : slot + 1;
        }
        // lane (gr, c): vectors 4 vb + c, rows gr + 8 i of the pair
        if (kw == 1) {
#pragma unroll
            for (int vb = 0; vb < NVB; ++vb) {
                const int v = 4 * vb + c;
                if (v >= p.batch) continue;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int row = q * Q4M_PAIR_ROWS + gr + 8 * i;
                    if (row < p.rows) p.y[(size_t)v * p.rows + row] = acc[vb][i];
                }
            }
            continue;
        }
        float* pt = p.part + ((size_t)q * kw + kp) * p.batch * 32;
#pragma unroll
        for (int vb = 0; vb < NVB; ++vb) {
            const int v = 4 * vb + c;
            if (v >= p.batch) continue;
#pragma unroll
            for (int i = 0; i < 4; ++i) pt[v * 32 + gr + 8 * i] = acc[vb][i];
        }
        __threadfence();
        __syncwarp();
        unsigned old = 0;
        if (lane == 0) old = atomicAdd(p.cnt + q, 1u);
        old = __shfl_sync(JINF_FULL_MASK, old, 0);
        if (old != (unsigned)(kw - 1)) continue;  // another K part finishes this pair
        __threadfence();
        if (lane == 0) p.cnt[q] = 0u;
        const float* pb = p.part + (size_t)q * kw * p.batch * 32;
        for (int e = lane; e < p.batch * 32; e += 32) {
            const int v = e / 32, r = e % 32, row = q * Q4M_PAIR_ROWS + r;
            float s = 0.f;
            for (int k2 = 0; k2 < kw; ++k2) s += __ldcg(pb + (size_t)k2 * p.batch * 32 + e);
            if (row < p.rows) p.y[(size_t)v * p.rows + row] = s;
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
}

size_t batch_smem(int batch, int gk) { return batch_rec_bytes(batch, gk) + (size_t)BNW * BNBUF * Q4M_UNIT; }

int batch_sms() {
    static int sms[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (!sms[dev]) {
        int n = 148;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        sms[dev] = n;
    }
    return sms[dev];
}

// K parts: enough tasks to keep about 8 warps per SM streaming, and the CTA's records in
// shared memory next to the ring.
int batch_kw(int pairs, int groups, int batch, int sms) {
    const size_t budget = 226 * 1024 - (size_t)BNW * BNBUF * Q4M_UNIT;
    for (int kw = 1; kw <= kBatchMaxKw && kw <= groups; ++kw) {
        const int gk = (groups + kw - 1) / kw;
        if (batch_rec_bytes(batch, gk) > budget) continue;
        if ((long long)pairs * kw >= 8LL * sms || kw == groups || kw == kBatchMaxKw) return kw;
    }
    return 0;
}

}  // namespace

}  // namespace jinf

using namespace jinf;

extern "C" size_t jinf_b200_gemv_q4m_batch_workspace_bytes(int rows, int cols, int batch) {
    Q4MShape sh;
    if (!q4m_shape(rows, cols, &sh) || batch < 1 || batch > 8) return 0;
    return (size_t)sh.pairs * kBatchMaxKw * batch * 32 * sizeof(float) + (size_t)sh.pairs * sizeof(unsigned);
}

extern "C" jinf_status jinf_b200_gemv_q4m_batch(const void* q4m, const void* x, int x_type, float* y, int rows,
                                               int cols, int batch, void* workspace, cudaStream_t stream) {
    Q4MShape sh;
    if (!q4m || !x || !y || !q4m_shape(rows, cols, &sh) || batch < 1 || batch > 8) return JINF_ERR_INVALID;
    if (x_type != JINF_TYPE_F32 && x_type != JINF_TYPE_F16) return JINF_ERR_INVALID;
    const int sms = batch_sms();
    const int kw = batch_kw(sh.pairs, sh.groups, batch, sms);
    if (kw < 1 || (kw > 1 && !workspace)) return JINF_ERR_INVALID;
    BatchParams p{};
    p.w = (const uint8_t*)q4m;
    p.rows = rows;
    p.cols = cols;
    p.pairs = sh.pairs;
    p.groups = sh.groups;
    p.batch = batch;
    p.kw = kw;
    p.gk = (sh.groups + kw - 1) / kw;
    p.x = x;
    p.x_f16 = x_type == JINF_TYPE_F16;
    p.y = y;
    if (kw > 1) {
        p.part = (float*)workspace;
        p.cnt = (unsigned*)((uint8_t*)workspace + (size_t)sh.pairs * kBatchMaxKw * batch * 32 * sizeof(float));
    }
    const int grid = kw * (sms / kw > 0 ? sms / kw : 1);
    const size_t smem = batch_smem(batch, p.gk);
    cudaError_t e;
    if (batch <= 4) {
        e = cudaFuncSetAttribute(k_gemv_q4m_batch<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess) k_gemv_q4m_batch<1><<<grid, BT, smem, stream>>>(p);
    } else {
        e = cudaFuncSetAttribute(k_gemv_q4m_batch<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess) k_gemv_q4m_batch<2><<<grid, BT, smem, stream>>>(p);
    }
    if (e == cudaSuccess) e = cudaGetLastError();
    return e == cudaSuccess ? JINF_OK : JINF_ERR_CUDA;
}
