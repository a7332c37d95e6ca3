// Host interface of the persistent decode-step kernel (step_kernel.cu).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "device_state.cuh"
#include "gemv.h"

namespace jinf {

#ifndef JINF_STEP_NBUF
#define JINF_STEP_NBUF 4
#endif
// L2 prefetch schedule of the persistent step (engine.cu, build_step): 0 none; 1 o and
// gate|up during attention; 2 also down during gate|up; 3 also the next layer's QKV during down.
#ifndef JINF_STEP_PF_MODE
#define JINF_STEP_PF_MODE 1
#endif
constexpr int STEP_THREADS = 512;              // 16 warps, one CTA per SM
constexpr int STEP_NBUF = JINF_STEP_NBUF;      // ring slots per warp (STEP_NBUF - 1 units in flight)
constexpr int ATTN_PW = 4;             // attention positions per warp in one block (16 warps: 64)
#ifndef JINF_ATTN_SPLIT_POS
#define JINF_ATTN_SPLIT_POS 16
#endif
constexpr int ATTN_SPLIT_POS = JINF_ATTN_SPLIT_POS;  // positions per CTA below which fewer CTAs split a kv head

constexpr int ATTN_MAX_SPLIT = 64;     // CTAs per kv head
constexpr int ATTN_MAX_GROUP = 8;      // query heads per kv head
constexpr int STEP_MAX_TP = 8;         // ranks of the tensor-parallel persistent step

enum PhaseKind { PH_GEMV = 0, PH_ATTN = 1 };

// One phase of the decode step. A phase starts (on every CTA) once phase `dep` has
// reported `dep_target` finished units: GEMV phases count finished 32-row tile pairs,
// attention counts finished kv heads.
struct StepPhase {
    int kind;
    int dep;                 // -1: no dependency
    unsigned int dep_target;
    int gran;                // a CTA owns whole runs of `gran` tile pairs (2: its gate|up rows
                             // make whole 32-element blocks of the activation)
    int layer;               // PH_ATTN: layer index (selects its split arrival counters)
    int pf[2];               // GEMV phases (-1: none) whose weights this CTA owns are prefetched
                             // into L2 when the CTA reaches this phase (before its wait)
    int xin;                 // tensor parallel: exchange point this phase reads (X_RMSNORM_TP; its
                             // staging waits for the flagged words, in place of `dep`), -1: none
    int xout;                // exchange point this phase writes (EPI_PARTIAL), -1: none
    // PH_GEMV
    int xm, epi;
    int fmts;                // weight formats: pairs below fmts >> 8 are format fmts & 15, the
                             // rest (fmts >> 4) & 15 (a QKV of [q|k] in one type, v in another)
    const uint8_t* w;        // Q4M matrix
    int rows, cols, pairs, groups;
    const float* x;          // X_PLAIN_F32: input (written earlier in the step)
    const float* hsrc;       // X_RMSNORM: residual stream; X_EMBED_NORM: token_embd [V][cols]
    float* hout;             // X_EMBED_NORM: residual stream (CTA 0 stores the embedding row)
    const float* norm_w;     // RMSNorm gain
    float* y;                // epilogue output; EPI_RESID: the residual stream (h += W x)
    __half* kcache;          // EPI_QKV and PH_ATTN: this layer's cache [Hkv][max_ctx][hd]
    __half* vcache;
    // X_RECORDS input: the digit records written by the producing phase and, for an RMSNorm
    // input, the producer's per-pair sums of h^2 (n_ss of them) that give the norm factor
    const uint8_t* rec;
    const float* ssp;
    int n_ss;
    // records this phase writes for the next GEMV phase (null: none), that phase's group
    // count, and for EPI_RESID the per-pair sums of h^2 and the next RMSNorm gain (the
    // records then hold h * gain)
    int groups_out;
    uint8_t* rec_out;
    float* ss_out;
    const float* gain_out;
    // PH_ATTN
    const float* q;          // [n_heads * hd], RoPE applied
    float* out;              // [n_heads * hd]
};

struct StepParams {
    const StepPhase* phases;  // device array
    int n_phases;
    unsigned int* done;       // [n_phases + 1] zero at launch; [n_phases] counts exiting CTAs
    float* attn_part;         // [Hkv][ATTN_MAX_SPLIT][ATTN_MAX_GROUP][hd + 2] per-CTA attention partials
    unsigned int* attn_cnt;   // [layers][Hkv] split arrival counters, zero at launch (cleared at the end)
    int n_attn_cnt;
    DeviceState* st;
    int nq, nk, head_dim, max_ctx, n_heads, n_kv_heads;
    float rope_base, eps;
    int attn_smax;            // CTAs per kv head at most (grid / kv heads, <= ATTN_MAX_SPLIT)
    int with_argmax;          // the last phase is the LM head: finish the argmax, feed it back
    int fmt;                  // Q4MFormat of every weight matrix of the step
    int nbuf;                 // weight ring slots per warp: STEP_NBUF, or 3 for wide models
    unsigned int xstage_bytes;  // shared bytes for the staged GEMV input / attention scratch
    unsigned long long spin_limit;  // polls before a dependency wait gives up (DEV_ERR_TIMEOUT)
    // tensor parallel (tp_size > 1): the exchange area of every rank, mapped into this
    // process (xpeer[tp_rank] is this rank's own), laid out as step_xchg_layout says
    int tp_rank, tp_size;
    int vocab_off;           // global id of this rank's first LM-head row
    uint8_t* xpeer[STEP_MAX_TP];
    unsigned long long x_keycnt, x_keys, x_data, x_point, x_slot;
};

// Exchange area of one rank for the tensor-parallel persistent step (same layout on every
// rank; all offsets 256-byte aligned):
//   [0, 8)     epoch: steps this rank's persistent kernel has finished (its parity selects
//              the data and key halves of a step, so a step never overwrites the previous)
//   keycnt     u64 arrival counter of the LM-head argmax keys, monotonic (a step's target is
//              (epoch + 1) * ranks)
//   keys       [2 parities][STEP_MAX_TP] packed argmax keys
//   data       [n_points][2 parities][ranks][slot] the ranks' partial outputs: per row one
//              8-byte word {value bits, epoch + 1} (slot = 8 d bytes)
struct XchgLayout {
    unsigned long long keycnt, keys, data, point, slot, total;
};
XchgLayout step_xchg_layout(int n_points, int tp_size, int d);

// CTA c of C owns tile pairs [step_cta_tile(c), step_cta_tile(c + 1)) of every GEMV phase.
// (c * T stays far below 2^32: at most a few hundred CTAs times tens of thousands of pairs.)
__host__ __device__ inline int step_cta_tile(int c, int C, int T) { return (int)((unsigned)(c * T) / (unsigned)C); }

// Shared bytes of the staged input for the widest GEMV phase, or of the attention scratch
// (q of one kv head's query heads + per-warp partials), whichever is larger.
unsigned int step_xstage_bytes(int max_cols, int group, int head_dim);
size_t step_smem_bytes(unsigned int xstage_bytes, int n_phases, int fmt, int nbuf);
// Launches the step on `grid` CTAs (one per SM) as a cooperative launch.
cudaError_t step_launch(const StepParams& p, int grid, cudaStream_t s);
// Resident CTAs per SM for this shared-memory size (must be >= 1).
int step_occupancy(size_t smem, int fmt, int nbuf);

}  // namespace jinf
