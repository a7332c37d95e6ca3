// Host interface of the fused Q4M tensor-core GEMV kernels (gemv_q4m.cu).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "device_state.cuh"
#include "q4m.cuh"

namespace jinf {

// One CTA of 16 warps per SM (persistent), each warp with a private ring of GEMV_M_NBUF
// unit slots (2304-byte tile-pair units).
#ifndef JINF_GEMV_M_NBUF
#define JINF_GEMV_M_NBUF 4
#endif
constexpr int GEMV_M_THREADS = 512;
constexpr int GEMV_M_NBUF = JINF_GEMV_M_NBUF;
// Ring slots per warp for a weight format: the larger Q6_K and Q8_0 units take 2, so that
// the ring still leaves room for the input records of 28672 columns (a 70B down projection).
#ifndef JINF_GEMV_M_NBUF_WIDE
#define JINF_GEMV_M_NBUF_WIDE 2
#endif
__host__ __device__ constexpr inline int gemvm_nbuf(int fmt) {
    return fmt == Q4M_Q6_K || fmt == Q4M_Q8_0 ? JINF_GEMV_M_NBUF_WIDE : GEMV_M_NBUF;
}

// X_RECORDS (persistent step only): the input is already staged as digit records in global
// memory by the phase that produced it (q4m_device.cuh, xrec_bytes).
// X_RMSNORM_TP (persistent step, tensor parallel): x = RMSNorm(h + the sum of the ranks'
// partial outputs of the previous row-split GEMV, added in rank order).
enum XMode { X_PLAIN_F32 = 0, X_PLAIN_F16 = 1, X_RMSNORM = 2, X_EMBED_NORM = 3, X_RECORDS = 4, X_RMSNORM_TP = 5 };
// EPI_PARTIAL (persistent step, tensor parallel): the rank's partial W x is stored to every
// rank's exchange slot for it.
enum EpiMode { EPI_STORE = 0, EPI_QKV = 1, EPI_GATEUP = 2, EPI_LMHEAD = 3, EPI_RESID = 4, EPI_PARTIAL = 5 };

struct GemvParams {
    const uint8_t* w;  // Q4M stream of the matrix
    int rows, cols, pairs, groups;
    int fmt;                // Q4MFormat of w
    int kw;                 // K parts per tile pair (tasks per pair)
    int local_k;            // 1: CTA c takes pairs c, c + grid, ... and its warps split K, merging in
                            // shared memory (kw unused, no workspace); for matrices of at most
                            // `grid` tile pairs (gemvm_use_local)
    float* part;            // kw > 1: [pairs * kw][32] partial row sums
    unsigned int* cnt;      // kw > 1: [pairs] arrival counters, zero before the first launch (self-resetting)
    // prologue
    const void* x;          // X_PLAIN_*: input vector
    const float* hin;       // X_RMSNORM: residual stream
    const float* yres;      // X_RMSNORM: pending residual added to hin (may be null)
    float* hout;            // X_RMSNORM / X_EMBED_NORM: CTA 0 stores h here (may be null)
    const float* norm_w;    // RMSNorm gain [cols]
    float eps;
    const float* embed;     // X_EMBED_NORM: token_embd [n_vocab][cols] (row read at st->token)
    // epilogue
    float* y;               // STORE: y[rows]; QKV: q[nq]; GATEUP: h[rows/2]; LMHEAD: logits[rows]
    __half* kcache;         // QKV: this layer's K cache [n_kv_heads][max_ctx][head_dim]
    __half* vcache;
    int nq, nk, head_dim, max_ctx;
    float rope_base;
    int vocab_offset;       // LMHEAD: global id of row 0
    DeviceState* st;
    // L2 prefetch of the bytes the next kernel will stream
    const uint8_t* pf_ptr;
    uint64_t pf_bytes;
};

inline void gemvm_params_for(GemvParams& p, const void* w, const Q4MShape& sh) {
    p.w = (const uint8_t*)w;
    p.rows = sh.rows;
    p.cols = sh.cols;
    p.pairs = sh.pairs;
    p.groups = sh.groups;
    p.fmt = sh.fmt;
    p.kw = 1;
}
size_t gemvm_smem_bytes(int cols, int fmt = Q4M_Q4_0);
int gemvm_max_cols(int fmt = Q4M_Q4_0);
// Persistent grid: resident CTAs per SM * num_sms.
int gemvm_grid(int cols, int xm, int epi, int num_sms, int fmt = Q4M_Q4_0);
// K parts per tile pair for a grid of `grid` CTAs (1 <= kw <= min(groups, max_kw)).
int gemvm_pick_kw(int pairs, int groups, int grid, int max_kw);
// The CTA-local K split serves matrices of at most 4 `grid` tile pairs: no global partial
// sums, no arrival counters. It runs on gemvm_local_grid CTAs, each taking the same number of
// pairs.
bool gemvm_use_local(int pairs, int grid);
int gemvm_local_grid(int pairs, int grid);
cudaError_t gemvm_launch(const GemvParams& p, int xm, int epi, int grid, cudaStream_t s, bool pdl);
// Q4M format of a reference block type (jinf_qtype: Q4_0 = 2, Q8_0 = 8, Q4_K = 12,
// Q6_K = 14); -1 for types the Q4M GEMV does not stream.
inline int q4m_fmt_of_qtype(int qtype) {
    return qtype == 2 ? Q4M_Q4_0 : qtype == 12 ? Q4M_Q4_K : qtype == 14 ? Q4M_Q6_K : qtype == 8 ? Q4M_Q8_0 : -1;
}
// AoS Q4_0, Q4_K, Q6_K or Q8_0 (sh.fmt) [rows][cols] (device) -> Q4M (device, sh.bytes).
cudaError_t q4m_repack(const void* aos, void* dst, const Q4MShape& sh, cudaStream_t s);
// The same on the host (host pointers; every byte of the image is written).
void q4m_repack_host(const void* aos, void* dst, const Q4MShape& sh);

}  // namespace jinf
