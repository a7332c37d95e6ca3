// Multi-sequence decode (gemv_multi.cu, the attention in attn_f16.cu): one step advances up to
// MULTI_MAX sequences by one token each, every sequence with its own KV cache and position.
// The reference decodes one sequence (src/engine.cpp:691-751); here the weights of each
// projection are streamed once per step for all the sequences, so the step costs about what
// one token costs and the throughput grows with the number of sequences.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace jinf {

constexpr int MULTI_MAX = 8;           // sequences per step
constexpr int MULTI_MAX_KV_HEADS = 64;

// Device-side state of a multi-sequence step (one per engine, in HBM). The host writes the
// first three arrays before each step; the kernels read them, so one captured graph per
// sequence count serves every step.
struct MultiState {
    int token[MULTI_MAX];  // input token of vector v
    int pos[MULTI_MAX];    // its position (the sequence's n_past)
    int seq[MULTI_MAX];    // its sequence (KV cache slot)
    int feedback;          // 1: the finaliser feeds each argmax back as the vector's next token
                           // and advances its position (resident decode, no host round trip)
    int out_token[MULTI_MAX];           // greedy argmax of the step (first maximum wins)
    unsigned long long best[MULTI_MAX];  // packed argmax keys of the LM head (reset by the finaliser)
    unsigned int attn_count[MULTI_MAX * MULTI_MAX_KV_HEADS];  // attention split arrivals (self-resetting)
};

// Input of a multi GEMV: fp32 or fp16 vectors x[v][ldx], or MX_NORMED: x = h * gain with the
// RMSNorm factor of vector v, 1 / sqrt(sum of its ssq partials / cols + eps), applied to the
// outputs (W (h g r) = r W (h g)).
// MX_RECORDS: x holds the inputs already as digit records (q4m_device.cuh, xrec_bytes(groups)
// bytes per vector, written by the producer: records of h * gain with ssq set, the RMSNorm
// factor then applied as for MX_NORMED; of plain values with ssq null).
enum MultiX { MX_PLAIN_F32 = 0, MX_PLAIN_F16 = 1, MX_NORMED = 2, MX_RECORDS = 3 };
// Output: ME_STORE y[v][row]; ME_QKV RoPE on the q and k rows at the vector's position, q to
// y[v], k and v rows into its sequence's cache; ME_GATEUP rows interleaved (gate_n, up_n):
// y[v][n] = SiLU(gate_n) up_n; ME_LMHEAD y[v][row] and the vector's argmax key; ME_RESID
// h[v][row] += (W x)[row] (y is h) and the sum of squares of each 32 new rows to
// ssq_out[pair][v].
enum MultiEpi { ME_STORE = 0, ME_QKV = 1, ME_GATEUP = 2, ME_LMHEAD = 3, ME_RESID = 4 };

struct MultiParams {
    const uint8_t* w;  // Q4M image of the matrix
    int rows, cols, pairs, groups, fmt;
    int n;             // vectors (1..MULTI_MAX)
    int kw, gk;        // K parts per tile pair; groups per part (the largest)
    int local;         // 1: a CTA's 16 warps split each of its tile pairs (not with ME_LMHEAD)
    const void* x;     // [n][ldx]
    int ldx;
    const float* norm_w;  // MX_NORMED: gain [cols]
    const float* ssq;     // MX_NORMED: [ssq_parts][n] partial sums of squares of h
    int ssq_parts;
    float eps;
    float* y;          // [n][ldy]
    int ldy;
    float* ssq_out;    // ME_RESID: [pairs][n]
    uint8_t* rec_out;  // ME_RESID, optional: records of h * gain_out for the next GEMV (per vector
    const float* gain_out;  //   xrec_bytes(rows / 128) bytes apart; one 32-row pair is one block)
    __half* kcache;    // ME_QKV: this layer's K cache of sequence 0 ([n_kv_heads][max_ctx][hd])
    __half* vcache;
    size_t seq_stride;  // elements from one sequence's cache to the next
    int nq, nk, head_dim, max_ctx;
    float rope_base;
    int vocab_offset;  // ME_LMHEAD: global id of row 0
    MultiState* ms;    // ME_QKV (positions, sequences), ME_LMHEAD (argmax keys)
    float* part;       // kw > 1: [pairs][kw][n][32] partial rows
    unsigned int* cnt;  // kw > 1: [pairs] arrival counters, zero before the first launch (self-resetting)
    size_t part_floats, cnt_n;  // their sizes (checked at launch)
    const uint8_t* pf_ptr;  // L2 prefetch of the next kernel's weights
    uint64_t pf_bytes;
};

// How an n-vector GEMV of this shape and input kind (xm) runs on `grid` CTAs: the K parts (the
// part's records within shared memory next to the weight rings) and whether a CTA's warps
// split each tile pair (*local), by the smallest estimated time; kw 0 when no split fits.
void multi_plan(int pairs, int groups, int n, int fmt, int grid, int epi, int xm, int* kw, int* local);
int multi_pick_kw(int pairs, int groups, int n, int fmt, int grid);
int multi_grid(int num_sms);
size_t multi_workspace_bytes(int pairs, int kw, int n);
cudaError_t multi_gemv_launch(const MultiParams& p, int xm, int epi, int grid, cudaStream_t s, bool pdl);

// Decode attention of a multi-sequence step (step_kernel.cu, one kernel per layer): vector v's
// query heads over positions 0 .. ms->pos[v] of sequence ms->seq[v]'s cache, the positions of
// each (vector, kv head) split over S = min(G, position blocks) CTAs of 16 warps, G = the
// resident CTA slots / (n x n_kv_heads) (at least 1, at most s_max): one wave of CTAs, each
// with one contiguous range of positions, the next block's K and V rows requested before the
// current block's arithmetic. The last CTA of each (vector, kv head) merges the splits in order.
struct MultiAttnParams {
    const float* q;         // [n][q_stride], RoPE applied
    int q_stride;
    const __half* kcache;   // this layer's cache of sequence 0: [n_kv_heads][max_ctx][head_dim]
    const __half* vcache;
    size_t seq_stride;      // elements from one sequence's cache to the next
    float* out;             // [n][q_stride]
    float* part;            // multi_attn_part_floats floats of scratch
    uint8_t* rec;           // optional: the output's digit records (xrec_bytes(q_stride / 128) per vector)
    int n, n_heads, n_kv_heads, head_dim, max_ctx, s_max;
    MultiState* ms;
};
size_t multi_attn_part_floats(int n, int n_kv_heads, int s_max, int head_dim);
cudaError_t multi_attn_launch(const MultiAttnParams& p, cudaStream_t s, bool pdl);

// h[v] = table[token_v] and its sums of squares per 32 elements (ssq [d / 32][n]).
// rec (optional): the digit records of h * gain (xrec_bytes(d / 128) bytes per vector).
cudaError_t multi_embed_launch(const float* table, const MultiState* ms, int n, int d, float* h, float* ssq,
                               uint8_t* rec, const float* gain, cudaStream_t s, bool pdl);
// h[v] += y[v] and the new sums of squares per 32 elements (tensor parallel: after the
// allreduce of the row-split partial outputs).
cudaError_t multi_resid_launch(float* h, const float* y, int n, int d, float* ssq, uint8_t* rec, const float* gain,
                               cudaStream_t s, bool pdl);
// out_token[v] from the argmax keys, which are reset for the next step (and, with feedback,
// fed back as the next step's tokens, positions advanced).
cudaError_t multi_finalize_launch(MultiState* ms, int n, cudaStream_t s);

}  // namespace jinf
