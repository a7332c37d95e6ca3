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

// One phase of the decode step. Phases hand their outputs on as flagged words (8 bytes:
// the value's 32 bits, then a 32-bit flag): the flag of a word written by phase `ph` during the
// step with epoch e is step_flag(e, ph), so a consumer's load of the word is also its wait
// (it reloads until the flag is the one it expects), with no counter and no fence on the way.
// An aligned 8-byte word is written and read whole.
struct StepPhase {
    int kind;
    int tag_in;              // phase whose flagged output this phase's input is (-1: none)
    int tag_res;             // EPI_RESID: phase that wrote the residual rows `fres`; tensor parallel:
                             //   phase that wrote the h of `fres` the ranks' partials are added to
    int gran;                // a CTA owns whole runs of `gran` tile pairs (2: its gate|up rows
                             // make whole 32-element blocks of the activation)
    int layer;               // layer index
    int pf[2];               // GEMV phases (-1: none) whose weights this CTA owns are prefetched
                             // into L2 when the CTA reaches this phase
    int xin;                 // tensor parallel: exchange point this phase reads (X_RMSNORM_TP), -1: none
    int xout;                // exchange point this phase writes (EPI_PARTIAL), -1: none
    // PH_GEMV
    int xm, epi;
    int fmts;                // weight formats: pairs below fmts >> 8 are format fmts & 15, the
                             // rest (fmts >> 4) & 15 (a QKV of [q|k] in one type, v in another)
    const uint8_t* w;        // Q4M matrix
    int rows, cols, pairs, groups;
    const float* hsrc;       // X_EMBED_NORM: token_embd [V][cols]
    const float* norm_w;     // RMSNorm gain
    float* y;                // EPI_LMHEAD: logits
    __half* kcache;          // EPI_QKV and PH_ATTN: this layer's cache [Hkv][max_ctx][hd]
    __half* vcache;
    // flagged words (step_flag): the input (X_RMSNORM: h [cols]; X_RECORDS: digit records as
    // xrec_bytes(groups) / 4 words; PH_ATTN: q [n_heads * hd]), the residual rows EPI_RESID
    // adds to (and the tensor-parallel h the partials are added to), the output (EPI_RESID:
    // h [rows]; EPI_QKV: q; EPI_GATEUP and PH_ATTN: the next phase's records, groups_out
    // groups), and the new K and V rows of the step's position (EPI_QKV writes, PH_ATTN
    // reads: [nk / 2] K words then [nk / 2] V words, two halves per word)
    const unsigned long long* fin;
    const unsigned long long* fres;
    unsigned long long* fout;
    unsigned long long* fkv;
    unsigned long long* fout_h;  // X_EMBED_NORM and X_RMSNORM_TP: the CTA that owns pair 0 stores
                                 // the phase's h here (flag of this phase), or null
    int groups_out;
};

struct StepParams {
    const StepPhase* phases;  // device array
    int n_phases;
    unsigned int* done;       // [1] CTAs that have left the step (zero at launch, cleared by the last)
    unsigned long long* attn_part;  // [Hkv][ATTN_MAX_SPLIT][ATTN_MAX_GROUP][hd + 2] flagged per-split
                                    // attention partials (acc, m, l)
    unsigned long long* split_part;  // [grid][2][64] flagged partial rows of the (at most two) tiles a
                                     // CTA shares with its neighbours in a GEMV phase
    DeviceState* st;
    int nq, nk, head_dim, max_ctx, n_heads, n_kv_heads;
    float rope_base, eps;
    int attn_smax;            // CTAs per kv head at most (grid / kv heads, <= ATTN_MAX_SPLIT)
    int with_argmax;          // the last phase is the LM head: finish the argmax, feed it back
    int fmt;                  // Q4MFormat of every weight matrix of the step
    int nbuf;                 // weight ring slots per warp: STEP_NBUF, or 3 for wide models
    unsigned int xstage_bytes;  // shared bytes for the staged GEMV input / attention scratch
    unsigned long long spin_limit;  // polls before a wait gives up (DEV_ERR_TIMEOUT)
    // tensor parallel (tp_size > 1): the exchange area of every rank, mapped into this
    // process (xpeer[tp_rank] is this rank's own), laid out as step_xchg_layout says
    int tp_rank, tp_size;
    int vocab_off;           // global id of this rank's first LM-head row
    uint8_t* xpeer[STEP_MAX_TP];
    unsigned long long x_keycnt, x_keys, x_data, x_point, x_slot;
};

// Flag of the words phase `ph` writes during the step whose epoch is `epoch` (steps the
// engine's persistent kernel has finished; never reset, so no stale word of an earlier step
// carries a current flag: the flag repeats only after 2^22 steps, and every word a step reads
// is rewritten by that step). Never 0, so zeroed buffers hold no valid word.
__host__ __device__ inline uint32_t step_flag(uint32_t epoch, int ph) { return epoch * 1024u + (uint32_t)ph + 1u; }
constexpr int STEP_MAX_PHASES = 1023;  // phase indices (and tags) below 1024; 1023 is never written

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

// CTA c of C owns units [step_cta_unit(c), step_cta_unit(c + 1)) of every GEMV phase of U
// units (pair-major: unit p * groups + g), an equal share whatever the shape; a tile of
// `gran` pairs that crosses a CTA boundary is merged by the CTA that holds its last unit.
__host__ __device__ inline int step_cta_unit(int c, int C, int U) {
    return (int)((unsigned long long)c * (unsigned long long)U / (unsigned long long)C);
}

// Shared bytes of the staged input for the widest GEMV phase, or of the attention scratch
// (q of one kv head's query heads + per-warp partials), whichever is larger.
unsigned int step_xstage_bytes(int max_cols, int group, int head_dim);
size_t step_smem_bytes(unsigned int xstage_bytes, int n_phases, int fmt, int nbuf);
// Launches the step on `grid` CTAs (one per SM) as a cooperative launch.
cudaError_t step_launch(const StepParams& p, int grid, cudaStream_t s);
// Resident CTAs per SM for this shared-memory size (must be >= 1).
int step_occupancy(size_t smem, int fmt, int nbuf);

}  // namespace jinf
