// jinf-b200: the decode engine (reference include/jinf/engine.h:161-176 API).
//
// Kept from the reference:
//   - jinf_engine_create/destroy/forward/generate/reset/get_stats with the same
//     argument meaning and error contract (null arguments -> JINF_ERR_INVALID, a
//     failed create leaves *e untouched, reference tests/test_engine.cpp:29-63);
//   - forward() returns an engine-owned DEVICE pointer to fp32 logits [n_vocab],
//     valid until the next call (reference src/engine.cpp:755);
//   - generate() is greedy, first maximum wins, and stops after emitting token 2
//     (reference src/engine.cpp:783-795);
//   - the public fields that tools read (n_layers, n_ff, n_vocab, ffn_hook, ...).
// Changed for B200:
//   - all weights live in HBM (no NVMe tier); the layer loop is fused kernels
//     replayed as one CUDA graph per token; argmax runs on the GPU and 4 bytes
//     cross to the host per generated token instead of the full logits;
//   - the KV cache is fp16 by default ([layer][kv_head][max_ctx][head_dim]);
//   - tensor parallelism over several GPUs (one process per GPU, NCCL allreduce),
//     selected through jinf_engine_create_ex().
#pragma once

#include "jinf/common.h"
#include "jinf/gguf.h"
#include "jinf/nvmw.h"

typedef struct CUstream_st* cudaStream_t;

typedef struct jinf_perf_stats {
    double total_ms;
    double nvme_read_ms;     // always 0 on B200 (no streaming tier)
    double gpu_compute_ms;   // device time of forward() calls (CUDA events)
    double attention_ms;
    double ffn_ms;
    int    tokens_generated;
    double nvme_bytes_read;  // always 0 on B200
} jinf_perf_stats;

typedef struct jinf_engine_config {
    const char* model_path;         // .nvmw file
    size_t      gpu_memory_budget;  // kept for API compatibility; every tensor is placed in HBM
    size_t      buffer_capacity;    // kept for API compatibility; unused (no double buffer)
    int         max_context;
    int         io_queue_depth;     // kept for API compatibility; unused
    const char* predictor_path;     // static activation profile (reference format) or NULL
    float       sparsity_threshold;
} jinf_engine_config;

static inline jinf_engine_config jinf_engine_config_default(void) {
    jinf_engine_config c;
    c.model_path = 0;
    c.gpu_memory_budget = (size_t)4500 * 1024 * 1024;
    c.buffer_capacity = (size_t)128 * 1024 * 1024;
    c.max_context = 512;
    c.io_queue_depth = 64;
    c.predictor_path = 0;
    c.sparsity_threshold = 0.5f;
    return c;
}

typedef void (*jinf_ffn_hook_fn)(void* user_data, int layer, const float* gate_output, int n_ff);

struct jinf_engine_impl;

typedef struct jinf_engine {
    // Model parameters (same names as the reference struct).
    int     n_layers;
    int     n_embd;
    int     n_heads;
    int     n_heads_kv;
    int     n_ff;
    int     n_vocab;
    int     max_context;
    int     head_dim;
    float   rms_norm_eps;
    float   rope_freq_base;
    int32_t primary_type;

    int n_past;  // tokens already in the KV cache

    // FFN profiling hook: when set, forward() runs layer by layer (no graph) and hands
    // the device pointer of the raw gate pre-activation [n_ff] of each layer to the hook.
    // Under tensor parallelism the pointer covers this rank's n_ff / tp_size neurons.
    jinf_ffn_hook_fn ffn_hook;
    void*            ffn_hook_data;

    float*       logits_buf;      // device fp32 [n_vocab]
    cudaStream_t compute_stream;  // the stream every engine kernel runs on
    jinf_perf_stats perf;

    struct jinf_engine_impl* impl;  // B200 internals (arenas, graphs, communicator)
} jinf_engine;

// ---- B200 options (new) ----
typedef struct jinf_b200_options {
    int   device;           // CUDA device ordinal (the reference always used 0)
    int   tp_rank;          // tensor-parallel rank of this process
    int   tp_size;          // 1, 2, 4 or 8
    const void* nccl_id;    // ncclUniqueId bytes (128), required when tp_size > 1
    int   kv_type;          // JINF_TYPE_F16 (default) or JINF_TYPE_F32
    int   use_graph;        // capture the per-token step in a CUDA graph (default 1)
    int   eos_token;        // generate() stops after this id (default 2; -1 = never)
    int   sparse_mode;      // 0 dense FFN (default), 1 predictor top-k, 2 fixed mask
    float sparse_keep;      // fraction of FFN neurons kept in sparse modes (default 0.15)
    uint64_t sparse_seed;   // seed of the predictor weights / fixed masks
    int   persistent;       // tp_size 1: run each token as one persistent kernel (default 1)
    int   prefill;          // forward() of several tokens runs all but the last through the batched
                            // prefill (tensor-core projections over all tokens at once) where the
                            // model allows it: one GPU, Q4_0 weights, dense FFN (default 1)
    int   max_seqs;         // sequences with a KV cache of their own for jinf_engine_decode_batch
                            // (1..8, default 1; sequence 0 is the one forward()/generate() use)
} jinf_b200_options;

static inline jinf_b200_options jinf_b200_options_default(void) {
    jinf_b200_options o;
    o.device = 0;
    o.tp_rank = 0;
    o.tp_size = 1;
    o.nccl_id = 0;
    o.kv_type = 1;  // JINF_TYPE_F16
    o.use_graph = 1;
    o.eos_token = 2;
    o.sparse_mode = 0;
    o.sparse_keep = 0.15f;
    o.sparse_seed = 0;
    o.persistent = 1;
    o.prefill = 1;
    o.max_seqs = 1;
    return o;
}

// ---- Synthetic Llama model (new; seeded, counter-based, deterministic) ----
typedef struct jinf_synth_config {
    jinf_model_hparams hp;  // arch "llama"; n_ctx_train is informative only
    uint64_t seed;
    int      weight_type;   // JINF_TYPE_Q4_0, Q4_K, Q6_K or Q8_0 for the 7 projections + output
    float    weight_std;    // 0.02
    float    embed_std;     // 0.02 (token_embd is f32)
    int      mix_type;      // 0, or a second type for attn_v and ffn_down of the even layers and
                            // for output (the pattern of a Q4_K_M file: mix_type Q6_K)
} jinf_synth_config;

typedef struct jinf_synth_model jinf_synth_model;

#ifdef __cplusplus
extern "C" {
#endif

// ---- Reference API ----
jinf_status jinf_engine_create(jinf_engine** e, const jinf_engine_config* config);
void        jinf_engine_destroy(jinf_engine* e);
jinf_status jinf_engine_forward(jinf_engine* e, const int32_t* tokens, int n_tokens, float** logits);
jinf_status jinf_engine_generate(jinf_engine* e, const int32_t* prompt, int n_prompt,
                                 int32_t* output, int max_tokens, int* n_generated);
void        jinf_engine_reset(jinf_engine* e);
const jinf_perf_stats* jinf_engine_get_stats(const jinf_engine* e);

// ---- New ----
jinf_status jinf_engine_create_ex(jinf_engine** e, const jinf_engine_config* config,
                                  const jinf_b200_options* options);
// Build an engine straight from a synthetic model (no file round trip).
jinf_status jinf_engine_create_synthetic(jinf_engine** e, const jinf_engine_config* config,
                                         const jinf_synth_model* model,
                                         const jinf_b200_options* options);
// Greedy step entirely on the device: runs `n_steps` decode tokens starting from the
// engine's last argmax, without host round trips (token feedback stays in HBM).
// Used to measure resident throughput; out_tokens (host, may be NULL) receives the ids.
jinf_status jinf_engine_decode_resident(jinf_engine* e, int n_steps, int32_t* out_tokens);
// Argmax of the last forward() logits (device computed, first maximum wins).
jinf_status jinf_engine_last_argmax(jinf_engine* e, int32_t* token);
// Fill the KV cache positions [0, n_pos) of every layer with seeded N(0,1) fp16 values
// and set n_past = n_pos (timing-only shortcut for long contexts).
jinf_status jinf_engine_fill_kv_random(jinf_engine* e, int n_pos, uint64_t seed);
// Copy positions [0, n_pos) of this rank's fp16 KV cache to host memory, as
// [layer][kv_head of this rank][n_pos][head_dim] fp16 for K and for V (each
// n_layers * n_heads_kv_of_rank * n_pos * head_dim values). Lets a checker start from the
// engine's cache (e.g. after jinf_engine_fill_kv_random). Synchronous.
jinf_status jinf_engine_kv_read(jinf_engine* e, int n_pos, uint16_t* k_host, uint16_t* v_host);
// 1 when each decode token runs as one persistent kernel, 0 for one kernel per operation.
int         jinf_engine_is_persistent(const jinf_engine* e);
// Sparse FFN modes: the active neurons of `layer` used by the last forward (ids ascending,
// at most `max` written to the host array `ids`); *n their count. JINF_ERR_INVALID in
// dense mode.
jinf_status jinf_engine_sparse_ids(jinf_engine* e, int layer, int32_t* ids, int max, int* n);
// Calibration (reference tools/profile_activations.cpp): forward `n_tokens` tokens from the
// current position and add to counts[l * n_ff + n] (host) one for every token on which
// |SiLU(gate_n)| of layer l exceeds `threshold`. Counted on the device, no host copy per
// layer. Dense FFN, one GPU. jinf_activation_profile_write turns the counts into the
// profile that jinf_engine_config.predictor_path reads.
jinf_status jinf_engine_count_activations(jinf_engine* e, const int32_t* tokens, int n_tokens, float threshold,
                                          int32_t* counts);
// Failure-path check of the persistent step (one GPU): runs one step whose attention phase
// waits for a count that nothing reaches, with `spin_limit` polls per wait. Every CTA gives
// up, the step returns JINF_ERR_TIMEOUT and the context stays usable; the engine's state is
// then undefined until jinf_engine_reset.
jinf_status jinf_engine_debug_step_timeout(jinf_engine* e, unsigned long long spin_limit);
// Bytes of quantized weights this rank streams per token (algorithmic weight traffic).
uint64_t    jinf_engine_weight_bytes_per_token(const jinf_engine* e);
// Time one launch of each fused kernel kind on its own (CUDA events, `reps` repetitions
// rotated over the layers). times_us receives 7 values: qkv, attention, o_proj, gate_up,
// down, lm_head, sparse_ffn (sparse modes: the whole FFN of a layer; 0 in dense mode, where
// gate_up and down are the FFN). bytes receives the algorithmic bytes of one launch of each.
jinf_status jinf_engine_profile_kernels(jinf_engine* e, int reps, double* times_us, double* bytes);
// The same for the kernels of an n-vector multi-sequence step (times_us, bytes: 8 entries:
// QKV, attention, o, gate|up, down, LM head, embedding/residual rows, finaliser). Leaves the
// sequences' state undefined.
jinf_status jinf_engine_profile_multi(jinf_engine* e, int n, int reps, double* times_us, double* bytes);

// ---- Multi-sequence decode (new; the reference decodes one sequence) ----
// Sequences 0 .. max_seqs - 1 each have a KV cache and a position of their own; sequence 0 is
// the one forward(), generate() and e->n_past describe. decode_batch advances n distinct
// sequences (1 <= n <= max_seqs) by one token in one step, every projection's weights streamed
// once for all of them: tokens[i] is fed to sequence seqs[i] at its position, next_tokens[i]
// (host, may be NULL) receives that sequence's greedy argmax (first maximum wins) and logits
// (host, may be NULL; one GPU only) the fp32 logits [n][n_vocab]. Dense FFN models. Under
// tensor parallelism every rank makes the same call. The prompt of a sequence is fed the same
// way, one token per call (its argmax ignored).
jinf_status jinf_engine_decode_batch(jinf_engine* e, int n, const int32_t* seqs, const int32_t* tokens,
                                     int32_t* next_tokens, float* logits);
// n_steps greedy steps of the same n sequences without host round trips: step 0 feeds tokens,
// every later step the previous step's argmax of each sequence (fed back on the device).
// out_tokens (host, may be NULL) receives the ids [n_steps][n]. Used to measure resident
// multi-sequence throughput.
jinf_status jinf_engine_decode_batch_resident(jinf_engine* e, int n, const int32_t* seqs, const int32_t* tokens,
                                              int n_steps, int32_t* out_tokens);
// Tokens in the KV cache of sequence `seq` (-1 for an invalid sequence).
int         jinf_engine_seq_n_past(const jinf_engine* e, int seq);
// Forget sequence `seq` (its position returns to 0).
jinf_status jinf_engine_seq_reset(jinf_engine* e, int seq);
// jinf_engine_fill_kv_random / jinf_engine_kv_read for the cache of sequence `seq`.
jinf_status jinf_engine_seq_fill_kv_random(jinf_engine* e, int seq, int n_pos, uint64_t seed);
jinf_status jinf_engine_seq_kv_read(jinf_engine* e, int seq, int n_pos, uint16_t* k_host, uint16_t* v_host);

// nccl unique id (128 bytes) for tensor-parallel set-up; rank 0 creates it and the
// caller distributes it. Returns JINF_ERR_CUDA if NCCL cannot be loaded.
jinf_status jinf_nccl_get_unique_id(void* out128);

jinf_status jinf_synth_create(jinf_synth_model** m, const jinf_synth_config* cfg);
void        jinf_synth_destroy(jinf_synth_model* m);
const jinf_synth_config* jinf_synth_get_config(const jinf_synth_model* m);
// Number of tensors and their names in file order (GGUF Llama naming).
int         jinf_synth_n_tensors(const jinf_synth_model* m);
const char* jinf_synth_tensor_name(const jinf_synth_model* m, int i);
// Tensor shape in ggml order (shape[0] = input features / fastest), type and bytes.
jinf_status jinf_synth_tensor_info(const jinf_synth_model* m, const char* name, int* type,
                                   int64_t* shape4, int* n_dims, uint64_t* n_bytes);
// Generate rows [row0, row0 + n_rows) of a tensor into `dst` (blocks / floats in file layout).
jinf_status jinf_synth_read_rows(const jinf_synth_model* m, const char* name, int64_t row0,
                                 int64_t n_rows, void* dst);
// Same rows generated on the GPU straight into device memory `dst` (asynchronous on
// `stream`); the bytes are identical to jinf_synth_read_rows.
jinf_status jinf_synth_read_rows_device(const jinf_synth_model* m, const char* name, int64_t row0,
                                        int64_t n_rows, void* dst, cudaStream_t stream);
// Write the model as a GGUF v3 file or as an all-hot .nvmw v1 file.
jinf_status jinf_synth_write_gguf(const jinf_synth_model* m, const char* path);
jinf_status jinf_synth_write_nvmw(const jinf_synth_model* m, const char* path);

#ifdef __cplusplus
}
#endif
