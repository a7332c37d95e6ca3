// The B200 decode engine behind the reference's jinf_engine_* API
// (reference src/engine.cpp:41-804, include/jinf/engine.h:161-176).
//
// Per token and per layer the reference issues 16 stream operations (7 GEMVs, 2
// RMSNorms, RoPE, 2 KV memcpys, attention, SiLU-mul, 2 residual adds,
// reference src/engine.cpp:418-511). On one GPU the whole token is ONE persistent
// cooperative kernel (step_kernel.cu) that streams every layer's weights without stopping
// at phase boundaries. Tensor-parallel runs (NCCL allreduce between phases) and the FFN
// hook use the kernel-per-operation form, where a layer is 5 fused kernels:
//   1. QKV GEMV   prologue: h = h + y_down (residual), RMSNorm(attn_norm)
//                 epilogue: RoPE(q,k) at pos, q -> fp32, k/v -> fp16 KV cache
//   2. attention  split-K GQA over positions 0..pos
//   3. o GEMV     -> y_o                       (tensor parallel: allreduce y_o)
//   4. gate|up    prologue: h = h + y_o, RMSNorm(ffn_norm); epilogue: silu(g)*u
//   5. down GEMV  -> y_down                    (tensor parallel: allreduce y_down)
// then LM head (prologue: final residual + output_norm; epilogue: logits + argmax) and
// a 1-thread finalize (argmax -> token, pos++). The whole step is captured once as a
// CUDA graph and replayed every token: the position and the token live in device
// memory. Residual adds are folded into the next prologue (ping-pong h buffers), so the
// reference's fp32 order "h += proj; rmsnorm(h)" is kept exactly.
//
// Weights: every projection is repacked (losslessly) into the Q4M layout (q4m.cuh) in one
// HBM arena laid out in consumption order; in the kernel-per-operation form each GEMV
// prefetches the next matrix into L2 (cp.async.bulk.prefetch.L2) before it waits on its
// inputs, so HBM keeps streaming across kernel boundaries.
#include "jinf/b200.h"
#include "jinf/engine.h"
#include "jinf/kernels.h"
#include "jinf/quant.h"
#include "jinf/sparse_ops.h"
#include "jinf/splitter.h"

#include "attn_f16.h"
#include "common.cuh"
#include "device_state.cuh"
#include "gemv.h"
#include "multi.h"
#include "nccl_shim.h"
#include "prefill.h"
#include "q4m.cuh"
#include "sparse_engine.h"
#include "step.h"
#include "synth_internal.h"

#include <fcntl.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include <algorithm>
#include <array>
#include <memory>
#include <string>
#include <vector>

using namespace jinf;

// ------------------------------------------------------------------ model sources

namespace {

struct TensorMeta {
    int type = -1;
    int n_dims = 0;
    int64_t shape[4] = {1, 1, 1, 1};
    int64_t rows() const { return n_dims > 1 ? shape[1] : 1; }
    int64_t cols() const { return shape[0]; }
    uint64_t row_bytes() const { return jinf_tensor_nbytes((jinf_qtype)type, cols()); }
};

// Host-side view of a model: tensor metadata + row reads in file (AoS) layout.
struct ModelSource {
    virtual ~ModelSource() {}
    virtual bool meta(const char* name, TensorMeta* m) const = 0;
    virtual jinf_status read_rows(const char* name, int64_t row0, int64_t n, void* dst) const = 0;
    // Optional device-side generation (synthetic models): Q4_0 or Q4_K rows [r0, r0+nr) x
    // columns [c0, c0+nc) into device rows dst_row0 + i*dst_step of pitch dst_row_bytes, or
    // the whole f32 tensor. Return false when the source has no device path.
    virtual bool device_quant(const char*, int64_t, int64_t, int64_t, int64_t, uint8_t*, int64_t, int64_t, int64_t,
                              cudaStream_t, jinf_status*) const { return false; }
    virtual bool device_f32(const char*, float*, cudaStream_t, jinf_status*) const { return false; }
    // B200-layout files (NVMW version 3): the projections are stored as the engine's Q4M
    // images; read_packed copies one into device memory (exactly `bytes` long).
    virtual bool prepacked() const { return false; }
    // Select the images of tensor-parallel rank `rank` of `size` in a pre-packed file; false
    // when the file holds none for that split.
    virtual bool select_shard(int, int) const { return false; }
    virtual jinf_status read_packed(const char*, uint8_t*, uint64_t) const { return JINF_ERR_INVALID; }
    jinf_model_hparams hp{};
    int primary_type = JINF_TYPE_Q4_0;
};

struct SynthSource : ModelSource {
    const jinf_synth_model* m;
    explicit SynthSource(const jinf_synth_model* mm) : m(mm) {
        hp = jinf_synth_get_config(m)->hp;
        primary_type = jinf_synth_get_config(m)->weight_type;
    }
    bool meta(const char* name, TensorMeta* t) const override {
        uint64_t nbytes;
        return jinf_synth_tensor_info(m, name, &t->type, t->shape, &t->n_dims, &nbytes) == JINF_OK;
    }
    jinf_status read_rows(const char* name, int64_t row0, int64_t n, void* dst) const override {
        return jinf_synth_read_rows(m, name, row0, n, dst);
    }
    bool device_quant(const char* name, int64_t r0, int64_t nr, int64_t c0, int64_t nc, uint8_t* dst,
                      int64_t dst_row_bytes, int64_t dst_row0, int64_t dst_step, cudaStream_t s,
                      jinf_status* st) const override {
        uint64_t key;
        float stdv;
        int role;
        TensorMeta t;
        if (!synth_tensor_params(m, name, &key, &stdv, &role) || !meta(name, &t) ||
            (t.type != JINF_TYPE_Q4_0 && t.type != JINF_TYPE_Q4_K))
            return false;
        const cudaError_t e =
            t.type == JINF_TYPE_Q4_K
                ? synth_fill_q4_k(key, stdv, t.cols(), r0, nr, c0, nc, dst, dst_row_bytes, dst_row0, dst_step, s)
                : synth_fill_q4_0(key, stdv, t.cols(), r0, nr, c0, nc, dst, dst_row_bytes, dst_row0, dst_step, s);
        *st = e == cudaSuccess ? JINF_OK : JINF_ERR_CUDA;
        return true;
    }
    bool device_f32(const char* name, float* dst, cudaStream_t s, jinf_status* st) const override {
        uint64_t key;
        float stdv;
        int role;
        TensorMeta t;
        if (!synth_tensor_params(m, name, &key, &stdv, &role) || !meta(name, &t) || t.type != JINF_TYPE_F32)
            return false;
        const int64_t n = t.rows() * t.cols();
        cudaError_t e = role == 1 ? fill_f32(dst, n, 1.0f, s) : synth_fill_f32(key, stdv, t.cols(), 0, t.rows(), dst, s);
        *st = e == cudaSuccess ? JINF_OK : JINF_ERR_CUDA;
        return true;
    }
};

struct NvmwSource : ModelSource {
    jinf_nvmw_reader* r = nullptr;
    int fd = -1;
    ~NvmwSource() override {
        if (fd >= 0) close(fd);
        if (r) jinf_nvmw_close(r);
    }
    bool b200 = false;  // version 3: pre-packed projections
    mutable std::string pfx;  // "tp<size>.<rank>." when a tensor-parallel rank reads its images
    bool prepacked() const override { return b200; }
    bool select_shard(int rank, int size) const override {
        pfx = size > 1 ? "tp" + std::to_string(size) + "." + std::to_string(rank) + "." : "";
        return b200 && jinf_nvmw_find_tensor(r, (pfx + "output.q4m").c_str()) != nullptr;
    }
    // In a B200-layout file a projection's type is that of the Q4M image that holds it.
    const jinf_nvmw_tensor_entry* packed_entry_for(const char* name) const {
        int l = -1;
        char part[64] = {0};
        std::string img;
        if (sscanf(name, "blk.%d.%63[a-z_].weight", &l, part) == 2) {
            const std::string p(part);
            const std::string pre = "blk." + std::to_string(l) + ".";
            if (p == "attn_q" || p == "attn_k") img = pre + "qkv.q4m";
            else if (p == "attn_v") img = jinf_nvmw_find_tensor(r, (pfx + pre + "v.q4m").c_str()) ? pre + "v.q4m" : pre + "qkv.q4m";
            else if (p == "attn_output") img = pre + "o.q4m";
            else if (p == "ffn_gate" || p == "ffn_up") img = pre + "gu.q4m";
            else if (p == "ffn_down") img = pre + "down.q4m";
        } else if (!strcmp(name, "output.weight")) {
            img = "output.q4m";
        }
        return img.empty() ? nullptr : jinf_nvmw_find_tensor(r, (pfx + img).c_str());
    }
    bool meta(const char* name, TensorMeta* t) const override {
        const jinf_nvmw_tensor_entry* te = jinf_nvmw_find_tensor(r, name);
        if (!te && b200) {
            const jinf_nvmw_tensor_entry* pe = packed_entry_for(name);
            if (!pe || (int)pe->type < JINF_NVMW_TYPE_Q4M) return false;
            t->type = qtype_of_q4m_format((int)pe->type - JINF_NVMW_TYPE_Q4M);
            t->n_dims = 2;
            t->shape[0] = pe->shape[0];
            t->shape[1] = pe->shape[1];
            t->shape[2] = t->shape[3] = 1;
            return true;
        }
        if (!te) return false;
        t->type = te->type;
        t->n_dims = (int)te->n_dims;
        for (int i = 0; i < 4; ++i) t->shape[i] = i < (int)te->n_dims ? te->shape[i] : 1;
        return true;
    }
    jinf_status read_packed(const char* name, uint8_t* dst_dev, uint64_t bytes) const override {
        const jinf_nvmw_tensor_entry* te = jinf_nvmw_find_tensor(r, (pfx + name).c_str());
        if (!te || (int)te->type < JINF_NVMW_TYPE_Q4M || te->n_bytes != bytes) {
            JINF_LOG("tensor %s: no pre-packed image of %llu bytes in this file", name, (unsigned long long)bytes);
            return JINF_ERR_INVALID;
        }
        std::vector<uint8_t> buf((size_t)std::min<uint64_t>(bytes, 64ull << 20));
        uint64_t off = jinf_nvmw_tensor_file_offset(r, te), done = 0;
        while (done < bytes) {
            const size_t n = (size_t)std::min<uint64_t>(bytes - done, buf.size());
            size_t got = 0;
            while (got < n) {
                const ssize_t k = pread(fd, buf.data() + got, n - got, (off_t)(off + done + got));
                if (k <= 0) return JINF_ERR_IO;
                got += (size_t)k;
            }
            JINF_CUDA_CHECK(cudaMemcpy(dst_dev + done, buf.data(), n, cudaMemcpyHostToDevice));
            done += n;
        }
        return JINF_OK;
    }
    jinf_status read_rows(const char* name, int64_t row0, int64_t n, void* dst) const override {
        const jinf_nvmw_tensor_entry* te = jinf_nvmw_find_tensor(r, name);
        if (!te) return JINF_ERR_INVALID;
        TensorMeta t;
        meta(name, &t);
        const uint64_t rb = t.row_bytes();
        if ((uint64_t)(row0 + n) * rb > te->n_bytes) return JINF_ERR_PARSE;
        uint64_t off = jinf_nvmw_tensor_file_offset(r, te) + (uint64_t)row0 * rb;
        uint64_t left = (uint64_t)n * rb;
        uint8_t* p = (uint8_t*)dst;
        while (left) {
            const ssize_t got = pread(fd, p, left > (1u << 30) ? (1u << 30) : left, (off_t)off);
            if (got <= 0) return JINF_ERR_IO;
            p += got;
            off += (uint64_t)got;
            left -= (uint64_t)got;
        }
        return JINF_OK;
    }
};

jinf_status open_nvmw_source(const char* path, std::unique_ptr<ModelSource>* out) {
    auto s = std::make_unique<NvmwSource>();
    JINF_CHECK(jinf_nvmw_open(&s->r, path), "open .nvmw");
    const jinf_nvmw_header* h = jinf_nvmw_get_header(s->r);
    s->fd = open(path, O_RDONLY);
    if (s->fd < 0) return JINF_ERR_IO;
    memset(&s->hp, 0, sizeof s->hp);
    strcpy(s->hp.arch, "llama");
    s->hp.n_layers = h->n_layers;
    s->hp.n_embd = h->n_embd;
    s->hp.n_heads = h->n_heads;
    s->hp.n_heads_kv = h->n_heads_kv ? h->n_heads_kv : h->n_heads;
    s->hp.n_ff = h->n_ff;
    s->hp.n_vocab = h->n_vocab;
    s->hp.n_ctx_train = h->n_ctx_train;
    s->hp.rope_freq_base = h->rope_freq_base;
    s->hp.rms_norm_eps = h->rms_norm_eps;
    s->primary_type = h->primary_type;
    s->b200 = h->version == JINF_NVMW_VERSION_B200;
    *out = std::move(s);
    return JINF_OK;
}

// ------------------------------------------------------------------ small kernels

__global__ void k_finalize(DeviceState* st, int with_argmax) {
    if (with_argmax) {
        const unsigned long long b = st->best;
        st->argmax_token = b ? (int)(0xFFFFFFFFu - (uint32_t)(b & 0xFFFFFFFFull)) : 0;
        st->token = st->argmax_token;
        st->best = 0ull;
    }
    st->pos += 1;
}

__global__ void k_fill_kv_random(__half* k, __half* v, int n_layers, int hkv, int max_ctx, int hd, int n_pos,
                                 unsigned long long seed) {
    const int64_t total = (int64_t)n_layers * hkv * n_pos * hd;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t d = i % hd;
        int64_t r = i / hd;
        const int64_t p = r % n_pos;
        r /= n_pos;  // = layer * hkv + head
        const size_t off = ((size_t)r * max_ctx + p) * hd + d;
        // two uniforms from a counter hash, Box-Muller
        unsigned long long z = seed + 0x9E3779B97F4A7C15ull * (unsigned long long)(2 * i + 1);
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        z ^= z >> 31;
        const float u1 = ((float)(z >> 40) + 0.5f) * (1.0f / 16777216.0f);
        const float u2 = ((float)((z >> 16) & 0xFFFFFF) + 0.5f) * (1.0f / 16777216.0f);
        const float rr = sqrtf(-2.0f * logf(u1));
        float s, c;
        sincospif(2.0f * u2, &s, &c);
        k[off] = __float2half(rr * c);
        v[off] = __float2half(rr * s);
    }
}

__global__ void k_even_rows(const float* in, float* out, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = in[2 * i];
}

// Calibration: counts[n] += 1 where |SiLU(gate[n])| > thr (reference
// tools/profile_activations.cpp:56-68, counted on the device instead of after a host copy).
__global__ void k_count_active(const float* __restrict__ gate, int n, float thr, int32_t* __restrict__ counts) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float g = gate[i];
    if (fabsf(g / (1.0f + expf(-g))) > thr) counts[i] += 1;
}

// Sparse FFN in the persistent step (fixed masks): dst row i = src row idx[i] of an AoS
// matrix (row_bytes each); idx[i] < 0 gives a zero row (scale 0: the row contributes 0).
__global__ void k_gather_rows(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, const int* __restrict__ idx,
                              int n, int row_bytes) {
    const int64_t total = (int64_t)n * row_bytes;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int i = (int)(t / row_bytes), b = (int)(t % row_bytes);
        const int r = idx[i];
        dst[t] = r < 0 ? 0 : src[(int64_t)r * row_bytes + b];
    }
}

// dst[r][j] = src[r][blk[j]]: the listed column blocks (bb bytes each) of every row.
__global__ void k_gather_blocks(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, const int* __restrict__ blk,
                                int rows, int nb_src, int nb, int bb) {
    const int64_t total = (int64_t)rows * nb * bb;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = t / ((int64_t)nb * bb);
        const int j = (int)((t / bb) % nb), b = (int)(t % bb);
        dst[t] = src[(r * nb_src + blk[j]) * bb + b];
    }
}


enum OpKind { OP_GEMV = 0, OP_ATTN = 1, OP_ALLREDUCE_F32 = 2, OP_ALLREDUCE_MAXU64 = 3, OP_FINALIZE = 4,
              OP_SPARSE_FFN = 5,
              // multi-sequence step (multi.h)
              OP_MGEMV = 6, OP_MEMBED = 7, OP_MRESID = 8, OP_MFINAL = 9, OP_MATTN = 10 };
enum GemvRole { ROLE_QKV = 0, ROLE_O = 1, ROLE_GATEUP = 2, ROLE_DOWN = 3, ROLE_LM = 4, ROLE_NONE = 5 };

struct Op {
    int kind;
    int role = ROLE_NONE;
    int layer = -1;
    GemvParams gp{};
    int xm = 0, epi = 0, grid = 1;
    AttnParams ap{};
    void* buf = nullptr;
    size_t count = 0;
    int with_argmax = 0;
    uint64_t bytes = 0;  // algorithmic bytes of the op (weights + vectors)
    MultiParams mp{};    // OP_MGEMV (xm, epi, grid as above)
    MultiAttnParams map{};  // OP_MATTN
    int n_vec = 0;       // multi-sequence ops: vectors of the step
    uint8_t* rec = nullptr;      // OP_MEMBED, OP_MRESID: records of h * gain for the next GEMV
    const float* gain = nullptr;
};

}  // namespace

struct jinf_engine_impl {
    int device = 0;
    int tp_rank = 0, tp_size = 1;
    int num_sms = 148;
    int wfmt = Q4M_Q4_0;       // Q4MFormat of the weight matrices when they share one (uniform),
                               // else Q4M_MIX (the persistent step's mixed instance)
    bool uniform = true;       // every projection and the output head of one type, Q4_0 or Q4_K
    bool step_formats = true;  // every matrix Q4_0, Q4_K or Q6_K: the persistent step can stream it
    int wtype = JINF_TYPE_Q4_0;
    cudaStream_t stream = nullptr;
    bool use_graph = true;
    int eos = 2;
    // global and local dims
    int d = 0, hd = 0, H = 0, Hkv = 0, ff = 0, V = 0, L = 0;
    int Hl = 0, Hkvl = 0, ffl = 0, Vl = 0, vocab_off = 0;
    float eps = 1e-5f, rope_base = 10000.f;
    int max_ctx = 0;
    // weights
    uint8_t* arena = nullptr;
    uint64_t arena_bytes = 0;
    uint64_t weight_bytes_token = 0;  // algorithmic quantized bytes per token (this rank)
    struct Layer {
        uint8_t* qkv; Q4MShape qkv_sh;  // [q | k | v] rows, or [q | k] when v has its own type
        uint8_t* v = nullptr; Q4MShape v_sh{};  // v rows of another weight type (Q4_K_M files)
        uint8_t* o; Q4MShape o_sh;
        uint8_t* gu; Q4MShape gu_sh;
        uint8_t* down; Q4MShape down_sh;
        float* attn_norm;
        float* ffn_norm;
    };
    std::vector<Layer> layers;
    uint8_t* lm = nullptr;
    Q4MShape lm_sh{};
    float* out_norm = nullptr;
    float* norms = nullptr;  // all norm gains
    float* embed = nullptr;  // [V][d] f32
    // KV cache [L][Hkvl][max_ctx][hd] fp16
    __half* kc = nullptr;
    __half* vc = nullptr;
    // activations
    float* hA = nullptr;
    float* hB = nullptr;
    float* y_o = nullptr;
    float* y_down = nullptr;
    float* q = nullptr;
    float* attn = nullptr;
    float* act = nullptr;
    float* gate_raw = nullptr;  // FFN hook buffer
    // sparse FFN mode (0 dense, 1 predictor top-k, 2 fixed mask; tp_size 1, kernel per operation)
    int sparse_mode = 0;
    int sparse_k = 0;                // neurons kept per layer (mode 1)
    int pred_r = 0;                  // predictor rank (mode 1)
    int bundle_size = 0;
    uint8_t* bundles = nullptr;      // [L][ff][bundle_size]
    __half* pred_w1 = nullptr;       // [L][r][d] fp16
    __half* pred_w2 = nullptr;       // [L][ff][r] fp16
    int32_t* sparse_ids = nullptr;   // [L][ff] active neuron ids (ascending)
    int32_t* sparse_offs = nullptr;  // [L][ff] their bundle byte offsets
    std::vector<int> sparse_n;       // active neurons per layer
    // fixed masks in the persistent step: per layer the 32-neuron blocks that hold an active
    // neuron (ascending) and the active flags; gate|up and down are stored compacted to them
    bool sparse_persistent = false;
    std::vector<std::vector<int32_t>> static_ids;  // mode 2: the active neurons of each layer
    // calibration (jinf_engine_count_activations): device counters [L][ffl] while counting
    int32_t* count_dev = nullptr;
    float count_thr = 0.f;
    std::vector<std::vector<int>> sparse_blocks;
    std::vector<std::vector<uint8_t>> sparse_active;
    float* sparse_x = nullptr;       // [d] normalised FFN input
    float* sparse_scratch = nullptr; // [r + ff] predictor scores
    float* gate_up_tmp = nullptr;    // [ff]
    float* logits = nullptr;    // local shard [Vl]
    float* logits_full = nullptr;  // [V] (== logits when tp_size == 1)
    float* attn_partial = nullptr;
    int n_split = 1;
    DeviceState* st = nullptr;
    int32_t* pinned = nullptr;  // [0] token in, [1] token out
    int32_t* dev_tokens = nullptr;  // prompt tokens of the current forward() [max_ctx]
    // split-K workspace of the stand-alone GEMV kernels
    float* gemv_part = nullptr;
    unsigned int* gemv_cnt = nullptr;
    // persistent step: phase tables on the device, counters, partials
    bool persistent = false;
    // tensor-parallel persistent step: this rank's exchange area and every rank's, mapped
    // (xpeer[tp_rank] == xchg; the others are IPC mappings of the peers' areas)
    uint8_t* xchg = nullptr;
    uint8_t* xpeer[STEP_MAX_TP] = {};
    XchgLayout xl{};
    int step_grid = 0;
    StepPhase* d_phases = nullptr;  // [n_full + n_body]
    unsigned int* step_done = nullptr;
    float* step_attn_part = nullptr;
    // input records of the GEMV phases (inputs of o, gate|up, down, qkv / LM head), written by
    // the producing phase, and the per-pair sums of h^2 behind the RMSNorm inputs
    uint8_t* step_rec[4] = {nullptr, nullptr, nullptr, nullptr};
    float* step_ss = nullptr;
    unsigned int* step_attn_cnt = nullptr;  // [layers][Hkv] attention split arrival counters
    StepParams sp_full{}, sp_body{};
    // batched prefill (prefill.h): enabled for one GPU, Q4_0 weights, dense FFN; buffers for a
    // chunk of up to pf_cap tokens, allocated at the first long forward()
    bool prefill = false;
    int pf_cap = 0;
    float *pf_h = nullptr, *pf_y = nullptr, *pf_att = nullptr, *pf_sc = nullptr;
    __half *pf_x16 = nullptr, *pf_q16 = nullptr;
    int* pf_err = nullptr;
    // multi-sequence decode (multi.h): n_seqs KV caches of seq_stride elements each (sequence
    // 0 = the one-sequence cache), the positions of sequences 1.. (sequence 0's is e->n_past),
    // the step's vectors [n_seqs][...], and one op list / graph per vector count
    int n_seqs = 1;
    size_t seq_stride = 0;
    std::vector<int> seq_past;
    MultiState* ms = nullptr;
    int32_t* ms_pinned = nullptr;  // [3 * MULTI_MAX] step inputs (token, pos, seq), then [MULTI_MAX] outputs
    float *m_h = nullptr, *m_y = nullptr, *m_q = nullptr, *m_attn = nullptr, *m_act = nullptr, *m_logits = nullptr,
          *m_ssq = nullptr, *m_attn_part = nullptr, *m_part = nullptr;
    // the GEMV inputs as digit records, written by their producers (n_seqs vectors each): h *
    // the next norm's gain, and the attention output; null when a width is not a whole number
    // of 128-element groups (the GEMVs then convert their inputs themselves)
    uint8_t *m_rec_h = nullptr, *m_rec_a = nullptr;
    unsigned int* m_cnt = nullptr;
    size_t m_part_floats = 0, m_cnt_n = 0;  // their sizes
    int32_t* m_out = nullptr;  // [max_ctx][MULTI_MAX] argmax ids of resident multi steps
    int m_split = 1;  // attention splits of a multi step
    std::vector<Op> m_ops[MULTI_MAX + 1];
    cudaGraphExec_t m_exec[MULTI_MAX + 1] = {};
    // ops and graphs
    std::vector<Op> ops_full, ops_body;
    cudaGraphExec_t exec_full = nullptr, exec_body = nullptr;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    ncclComm_t comm = nullptr;
    bool logits_valid = false;
};

namespace {

jinf_status run_op(jinf_engine_impl* I, const Op& op, cudaStream_t s) {
    cudaError_t e = cudaSuccess;
    switch (op.kind) {
        case OP_GEMV: e = gemvm_launch(op.gp, op.xm, op.epi, op.grid, s, true); break;
        case OP_ATTN: e = attn_launch(op.ap, s, true); break;
        case OP_FINALIZE: k_finalize<<<1, 1, 0, s>>>(I->st, op.with_argmax); e = cudaGetLastError(); break;
        case OP_MGEMV: e = multi_gemv_launch(op.mp, op.xm, op.epi, op.grid, s, true); break;
        case OP_MEMBED:
            e = multi_embed_launch(I->embed, I->ms, op.n_vec, I->d, I->m_h, I->m_ssq, op.rec, op.gain, s, true);
            break;
        case OP_MRESID:
            e = multi_resid_launch(I->m_h, I->m_y, op.n_vec, I->d, I->m_ssq, op.rec, op.gain, s, true);
            break;
        case OP_MFINAL: e = multi_finalize_launch(I->ms, op.n_vec, s); break;
        case OP_MATTN: e = multi_attn_launch(op.map, s, true); break;
        case OP_SPARSE_FFN: {
            // h = h + y_o; x = RMSNorm(h) * ffn_norm; [predictor]; y_down = FFN over the active
            // neurons (the next layer's QKV prologue adds y_down to h)
            const int L = op.layer;
            const size_t ff = (size_t)I->ffl;
            int32_t* ids = I->sparse_ids + (size_t)L * ff;
            int32_t* offs = I->sparse_offs + (size_t)L * ff;
            const uint8_t* bund = I->bundles + (size_t)L * ff * I->bundle_size;
            if (I->sparse_mode == 2 && sparse_ffn_fused_ok(I->d, I->wtype) && I->sparse_n[L] > 0) {
                // fixed mask: the prologue runs inside the gate/up kernel
                e = sparse_ffn_fused(bund, I->hA, I->y_o, I->hB, I->layers[L].ffn_norm, I->eps, I->y_down, offs,
                                     I->sparse_n[L], I->d, I->bundle_size, I->gate_up_tmp, s);
                break;
            }
            if (I->sparse_mode == 1)  // predictor: the prologue runs inside its first GEMV
                e = sparse_predict_norm(I->pred_w1 + (size_t)L * I->pred_r * I->d,
                                        I->pred_w2 + (size_t)L * ff * I->pred_r, I->hA, I->y_o, I->hB,
                                        I->layers[L].ffn_norm, I->eps, I->sparse_x, I->d, I->pred_r, I->ffl,
                                        I->sparse_k, I->bundle_size, ids, offs, I->sparse_scratch, s);
            else
                e = sparse_ffn_prologue(I->hA, I->y_o, I->hB, I->layers[L].ffn_norm, I->eps, I->d, I->sparse_x, s);
            if (e == cudaSuccess) {
                jinf_cuda_sparse_ffn(bund, I->sparse_x, I->y_down, offs,
                                     I->sparse_n[L], I->d, I->bundle_size, I->wtype, I->gate_up_tmp, s);
                e = cudaGetLastError();
            }
            break;
        }
        case OP_ALLREDUCE_F32:
        case OP_ALLREDUCE_MAXU64: {
            const NcclApi* n = nccl_api();
            if (!n || !I->comm) return JINF_ERR_CUDA;
            const ncclResult_t r =
                op.kind == OP_ALLREDUCE_F32
                    ? n->AllReduce(op.buf, op.buf, op.count, ncclFloat32, ncclSum, I->comm, s)
                    : n->AllReduce(op.buf, op.buf, op.count, ncclUint64, ncclMax, I->comm, s);
            if (r != ncclSuccess) {
                JINF_LOG("NCCL allreduce failed: %s", n->GetErrorString(r));
                return JINF_ERR_CUDA;
            }
            break;
        }
        default: return JINF_ERR_INVALID;
    }
    if (e != cudaSuccess) {
        JINF_LOG("launch failed (op %d): %s", op.kind, cudaGetErrorString(e));
        return JINF_ERR_CUDA;
    }
    return JINF_OK;
}

jinf_status run_ops(jinf_engine_impl* I, const std::vector<Op>& ops, cudaStream_t s) {
    for (const Op& op : ops) JINF_CHECK(run_op(I, op, s), "step op");
    return JINF_OK;
}

jinf_status capture(jinf_engine_impl* I, const std::vector<Op>& ops, cudaGraphExec_t* exec) {
    cudaGraph_t g = nullptr;
    JINF_CUDA_CHECK(cudaStreamBeginCapture(I->stream, cudaStreamCaptureModeThreadLocal));
    jinf_status st = run_ops(I, ops, I->stream);
    cudaError_t e = cudaStreamEndCapture(I->stream, &g);
    if (st != JINF_OK) {
        if (g) cudaGraphDestroy(g);
        return st;
    }
    JINF_CUDA_CHECK(e);
    e = cudaGraphInstantiate(exec, g, 0);
    cudaGraphDestroy(g);
    JINF_CUDA_CHECK(e);
    return JINF_OK;
}

constexpr int kEngineMaxKw = 16;  // K parts per tile of the stand-alone GEMVs

// Build the op list of one decode step. `with_head` adds the LM head + argmax.
void build_ops(jinf_engine_impl* I, bool with_head, std::vector<Op>& ops) {
    ops.clear();
    auto gemv_bytes = [](const Q4MShape& sh, int in_elems, int out_elems) -> uint64_t {
        return (uint64_t)sh.rows * aos_row_bytes(sh.fmt, sh.cols) + 4ull * in_elems + 4ull * out_elems;
    };
    // grid and K split of a stand-alone GEMV
    auto finish = [&](Op& op) {
        op.grid = gemvm_grid(op.gp.cols, op.xm, op.epi, I->num_sms, op.gp.fmt);
        op.gp.kw = gemvm_pick_kw(op.gp.pairs, op.gp.groups, op.grid, kEngineMaxKw);
        op.gp.part = I->gemv_part;
        op.gp.cnt = I->gemv_cnt;
        if (gemvm_use_local(op.gp.pairs, op.grid)) {
            op.gp.kw = 1;
            op.gp.local_k = 1;
            op.grid = gemvm_local_grid(op.gp.pairs, op.grid);
        }
    };
    for (int L = 0; L < I->L; ++L) {
        const auto& ly = I->layers[L];
        const auto* next_qkv = L + 1 < I->L ? &I->layers[L + 1] : nullptr;
        Op qkv{OP_GEMV};
        qkv.role = ROLE_QKV;
        qkv.layer = L;
        gemvm_params_for(qkv.gp, ly.qkv, ly.qkv_sh);
        qkv.xm = L == 0 ? X_EMBED_NORM : X_RMSNORM;
        qkv.epi = EPI_QKV;
        qkv.gp.hin = I->hB;
        qkv.gp.yres = L == 0 ? nullptr : I->y_down;
        qkv.gp.hout = I->hA;
        qkv.gp.embed = I->embed;
        qkv.gp.norm_w = ly.attn_norm;
        qkv.gp.eps = I->eps;
        qkv.gp.y = I->q;
        qkv.gp.kcache = I->kc + (size_t)L * I->Hkvl * I->max_ctx * I->hd;
        qkv.gp.vcache = I->vc + (size_t)L * I->Hkvl * I->max_ctx * I->hd;
        qkv.gp.nq = I->Hl * I->hd;
        qkv.gp.nk = I->Hkvl * I->hd;
        qkv.gp.head_dim = I->hd;
        qkv.gp.max_ctx = I->max_ctx;
        qkv.gp.rope_base = I->rope_base;
        qkv.gp.st = I->st;
        qkv.gp.pf_ptr = ly.v ? ly.v : ly.o;
        qkv.gp.pf_bytes = ly.v ? ly.v_sh.bytes : ly.o_sh.bytes;
        finish(qkv);
        qkv.bytes = gemv_bytes(ly.qkv_sh, I->d, ly.qkv_sh.rows);
        ops.push_back(qkv);
        if (ly.v) {
            // v of another weight type: a GEMV of its own over the same input, every row a v
            // row (nq = nk = 0); both GEMVs store the same h
            Op v = qkv;
            gemvm_params_for(v.gp, ly.v, ly.v_sh);
            v.gp.local_k = 0;
            v.gp.nq = 0;
            v.gp.nk = 0;
            v.gp.pf_ptr = ly.o;
            v.gp.pf_bytes = ly.o_sh.bytes;
            finish(v);
            v.bytes = gemv_bytes(ly.v_sh, I->d, ly.v_sh.rows);
            ops.push_back(v);
        }

        Op at{OP_ATTN};
        at.layer = L;
        at.ap.q = I->q;
        at.ap.kcache = qkv.gp.kcache;
        at.ap.vcache = qkv.gp.vcache;
        at.ap.out = I->attn;
        at.ap.partial = I->attn_partial;
        at.ap.n_heads = I->Hl;
        at.ap.n_kv_heads = I->Hkvl;
        at.ap.head_dim = I->hd;
        at.ap.max_ctx = I->max_ctx;
        at.ap.n_split = I->n_split;
        at.ap.st = I->st;
        ops.push_back(at);

        Op o{OP_GEMV};
        o.role = ROLE_O;
        o.layer = L;
        gemvm_params_for(o.gp, ly.o, ly.o_sh);
        o.xm = X_PLAIN_F32;
        o.epi = EPI_STORE;
        o.gp.x = I->attn;
        o.gp.y = I->y_o;
        o.gp.st = I->st;
        // the dense gate|up matrix is next, unless the FFN runs over sparse bundles
        o.gp.pf_ptr = I->sparse_mode ? nullptr : ly.gu;
        o.gp.pf_bytes = I->sparse_mode ? 0 : ly.gu_sh.bytes;
        finish(o);
        o.bytes = gemv_bytes(ly.o_sh, ly.o_sh.cols, ly.o_sh.rows);
        ops.push_back(o);
        if (I->tp_size > 1) {
            Op ar{OP_ALLREDUCE_F32};
            ar.buf = I->y_o;
            ar.count = (size_t)I->d;
            ops.push_back(ar);
        }

        if (I->sparse_mode) {
            Op sp{OP_SPARSE_FFN};
            sp.layer = L;
            sp.bytes = (uint64_t)I->sparse_n[L] * I->bundle_size;
            if (I->sparse_mode == 1)  // fp16 predictor W1 [r][d] and W2 [ff][r]
                sp.bytes += 2ull * I->pred_r * ((uint64_t)I->d + I->ffl);
            ops.push_back(sp);
            continue;
        }

        Op gu{OP_GEMV};
        gu.role = ROLE_GATEUP;
        gu.layer = L;
        gemvm_params_for(gu.gp, ly.gu, ly.gu_sh);
        gu.xm = X_RMSNORM;
        gu.epi = EPI_GATEUP;
        gu.gp.hin = I->hA;
        gu.gp.yres = I->y_o;
        gu.gp.hout = I->hB;
        gu.gp.norm_w = ly.ffn_norm;
        gu.gp.eps = I->eps;
        gu.gp.y = I->act;
        gu.gp.st = I->st;
        gu.gp.pf_ptr = ly.down;
        gu.gp.pf_bytes = ly.down_sh.bytes;
        finish(gu);
        gu.bytes = gemv_bytes(ly.gu_sh, I->d, ly.gu_sh.rows / 2);
        ops.push_back(gu);

        Op dn{OP_GEMV};
        dn.role = ROLE_DOWN;
        dn.layer = L;
        gemvm_params_for(dn.gp, ly.down, ly.down_sh);
        dn.xm = X_PLAIN_F32;
        dn.epi = EPI_STORE;
        dn.gp.x = I->act;
        dn.gp.y = I->y_down;
        dn.gp.st = I->st;
        if (next_qkv) {
            dn.gp.pf_ptr = next_qkv->qkv;
            dn.gp.pf_bytes = next_qkv->qkv_sh.bytes;
        } else if (with_head) {
            dn.gp.pf_ptr = I->lm;
            dn.gp.pf_bytes = I->lm_sh.bytes;
        }
        finish(dn);
        dn.bytes = gemv_bytes(ly.down_sh, ly.down_sh.cols, ly.down_sh.rows);
        ops.push_back(dn);
        if (I->tp_size > 1) {
            Op ar{OP_ALLREDUCE_F32};
            ar.buf = I->y_down;
            ar.count = (size_t)I->d;
            ops.push_back(ar);
        }
    }
    if (with_head) {
        Op lm{OP_GEMV};
        lm.role = ROLE_LM;
        gemvm_params_for(lm.gp, I->lm, I->lm_sh);
        lm.xm = X_RMSNORM;
        lm.epi = EPI_LMHEAD;
        lm.gp.hin = I->hB;
        lm.gp.yres = I->y_down;
        lm.gp.hout = nullptr;
        lm.gp.norm_w = I->out_norm;
        lm.gp.eps = I->eps;
        lm.gp.y = I->logits;
        lm.gp.vocab_offset = I->vocab_off;
        lm.gp.st = I->st;
        lm.gp.pf_ptr = I->layers[0].qkv;
        lm.gp.pf_bytes = I->layers[0].qkv_sh.bytes;
        finish(lm);
        lm.bytes = gemv_bytes(I->lm_sh, I->d, I->lm_sh.rows);
        ops.push_back(lm);
        if (I->tp_size > 1) {
            Op ar{OP_ALLREDUCE_MAXU64};
            ar.buf = &I->st->best;
            ar.count = 1;
            ops.push_back(ar);
        }
    }
    Op fin{OP_FINALIZE};
    fin.with_argmax = with_head ? 1 : 0;
    ops.push_back(fin);
}

// Op list of one multi-sequence step over n vectors (vector v = a sequence's token). Per layer:
//   [embedding rows (layer 0)] -> QKV (x = RMSNorm(h), RoPE at each vector's position, k/v
//   into each vector's sequence cache) -> attention (vector v over its sequence's positions)
//   -> o (h += W attn, and the new h's sums of squares for the next RMSNorm) -> gate|up
//   (x = RMSNorm(h), SiLU(gate) up) -> down (h += W act)
// then the LM head (x = RMSNorm(h), logits and each vector's argmax) and the finaliser. Tensor
// parallel: o and down store their partial outputs, which an allreduce sums before the residual
// add, and the argmax keys are reduced across the ranks.
Op multi_gemv_op(jinf_engine_impl* I, int n, const uint8_t* w, const Q4MShape& sh, int xm, int epi) {
    Op op{OP_MGEMV};
    op.xm = xm;
    op.epi = epi;
    op.n_vec = n;
    op.grid = multi_grid(I->num_sms);
    MultiParams& p = op.mp;
    p.w = w;
    p.rows = sh.rows;
    p.cols = sh.cols;
    p.pairs = sh.pairs;
    p.groups = sh.groups;
    p.fmt = sh.fmt;
    p.n = n;
    multi_plan(sh.pairs, sh.groups, n, sh.fmt, op.grid, epi, xm, &p.kw, &p.local);
    p.gk = p.kw > 0 ? (sh.groups + p.kw - 1) / p.kw : 0;
    p.part = I->m_part;
    p.cnt = I->m_cnt;
    p.part_floats = I->m_part_floats;
    p.cnt_n = I->m_cnt_n;
    p.ms = I->ms;
    p.eps = I->eps;
    p.ssq = I->m_ssq;
    p.ssq_parts = I->d / 32;
    op.bytes = (uint64_t)sh.rows * aos_row_bytes(sh.fmt, sh.cols);
    return op;
}

void build_multi_ops(jinf_engine_impl* I, int n, std::vector<Op>& ops) {
    ops.clear();
    const int d = I->d, nq = I->Hl * I->hd, nk = I->Hkvl * I->hd;
    const bool tp = I->tp_size > 1;
    const bool rec = I->m_rec_h != nullptr;
    const int xm_h = rec ? MX_RECORDS : MX_NORMED;  // inputs normalised from h
    auto from_h = [&](Op& g, const float* gain) {
        g.mp.x = rec ? static_cast<const void*>(I->m_rec_h) : static_cast<const void*>(I->m_h);
        g.mp.ldx = d;
        g.mp.norm_w = gain;
    };
    // o / down: residual add (one GPU) or partial + allreduce + add; the new h's records with
    // the gain of the norm after it
    auto resid = [&](Op& g, const float* next_gain) {
        if (!tp) {
            g.epi = ME_RESID;
            g.mp.y = I->m_h;
            g.mp.ldy = d;
            g.mp.ssq_out = I->m_ssq;
            if (rec) {
                g.mp.rec_out = I->m_rec_h;
                g.mp.gain_out = next_gain;
            }
            ops.push_back(g);
            return;
        }
        g.epi = ME_STORE;
        g.mp.y = I->m_y;
        g.mp.ldy = d;
        ops.push_back(g);
        Op ar{OP_ALLREDUCE_F32};
        ar.buf = I->m_y;
        ar.count = (size_t)n * d;
        ops.push_back(ar);
        Op ad{OP_MRESID};
        ad.n_vec = n;
        if (rec) {
            ad.rec = I->m_rec_h;
            ad.gain = next_gain;
        }
        ops.push_back(ad);
    };
    Op em{OP_MEMBED};
    em.n_vec = n;
    if (rec) {
        em.rec = I->m_rec_h;
        em.gain = I->layers[0].attn_norm;
    }
    ops.push_back(em);
    for (int L = 0; L < I->L; ++L) {
        const auto& ly = I->layers[L];
        __half* kc = I->kc + (size_t)L * I->Hkvl * I->max_ctx * I->hd;
        __half* vc = I->vc + (size_t)L * I->Hkvl * I->max_ctx * I->hd;
        Op qkv = multi_gemv_op(I, n, ly.qkv, ly.qkv_sh, xm_h, ME_QKV);
        qkv.role = ROLE_QKV;
        qkv.layer = L;
        MultiParams& qp = qkv.mp;
        from_h(qkv, ly.attn_norm);
        qp.y = I->m_q;
        qp.ldy = nq;
        qp.kcache = kc;
        qp.vcache = vc;
        qp.seq_stride = I->seq_stride;
        qp.nq = nq;
        qp.nk = nk;
        qp.head_dim = I->hd;
        qp.max_ctx = I->max_ctx;
        qp.rope_base = I->rope_base;
        qp.pf_ptr = ly.v ? ly.v : ly.o;
        qp.pf_bytes = ly.v ? ly.v_sh.bytes : ly.o_sh.bytes;
        ops.push_back(qkv);
        if (ly.v) {  // v of another weight type: every row a v row
            Op v = multi_gemv_op(I, n, ly.v, ly.v_sh, xm_h, ME_QKV);
            v.mp = qp;
            v.mp.w = ly.v;
            v.mp.rows = ly.v_sh.rows;
            v.mp.pairs = ly.v_sh.pairs;
            v.mp.groups = ly.v_sh.groups;
            v.mp.fmt = ly.v_sh.fmt;
            multi_plan(ly.v_sh.pairs, ly.v_sh.groups, n, ly.v_sh.fmt, v.grid, ME_QKV, xm_h, &v.mp.kw, &v.mp.local);
            v.mp.gk = v.mp.kw > 0 ? (ly.v_sh.groups + v.mp.kw - 1) / v.mp.kw : 0;
            v.mp.nq = 0;
            v.mp.nk = 0;
            v.mp.pf_ptr = ly.o;
            v.mp.pf_bytes = ly.o_sh.bytes;
            v.bytes = (uint64_t)ly.v_sh.rows * aos_row_bytes(ly.v_sh.fmt, ly.v_sh.cols);
            ops.push_back(v);
        }
        Op at{OP_MATTN};
        at.layer = L;
        at.n_vec = n;
        at.map.q = I->m_q;
        at.map.q_stride = nq;
        at.map.kcache = kc;
        at.map.vcache = vc;
        at.map.seq_stride = I->seq_stride;
        at.map.out = I->m_attn;
        at.map.part = I->m_attn_part;
        at.map.n = n;
        at.map.n_heads = I->Hl;
        at.map.n_kv_heads = I->Hkvl;
        at.map.head_dim = I->hd;
        at.map.max_ctx = I->max_ctx;
        at.map.s_max = I->m_split;
        at.map.ms = I->ms;
        at.map.rec = rec ? I->m_rec_a : nullptr;
        ops.push_back(at);

        Op o = multi_gemv_op(I, n, ly.o, ly.o_sh, rec ? MX_RECORDS : MX_PLAIN_F32, ME_RESID);
        o.role = ROLE_O;
        o.layer = L;
        o.mp.x = rec ? static_cast<const void*>(I->m_rec_a) : static_cast<const void*>(I->m_attn);
        o.mp.ldx = nq;
        o.mp.ssq = nullptr;  // plain values: no norm factor
        o.mp.pf_ptr = ly.gu;
        o.mp.pf_bytes = ly.gu_sh.bytes;
        resid(o, ly.ffn_norm);

        Op gu = multi_gemv_op(I, n, ly.gu, ly.gu_sh, xm_h, ME_GATEUP);
        gu.role = ROLE_GATEUP;
        gu.layer = L;
        from_h(gu, ly.ffn_norm);
        gu.mp.y = I->m_act;
        gu.mp.ldy = I->ffl;
        gu.mp.pf_ptr = ly.down;
        gu.mp.pf_bytes = ly.down_sh.bytes;
        ops.push_back(gu);

        Op dn = multi_gemv_op(I, n, ly.down, ly.down_sh, MX_PLAIN_F32, ME_RESID);
        dn.role = ROLE_DOWN;
        dn.layer = L;
        dn.mp.x = I->m_act;
        dn.mp.ldx = I->ffl;
        dn.mp.pf_ptr = L + 1 < I->L ? I->layers[L + 1].qkv : I->lm;
        dn.mp.pf_bytes = L + 1 < I->L ? I->layers[L + 1].qkv_sh.bytes : I->lm_sh.bytes;
        resid(dn, L + 1 < I->L ? I->layers[L + 1].attn_norm : I->out_norm);
    }
    Op lm = multi_gemv_op(I, n, I->lm, I->lm_sh, xm_h, ME_LMHEAD);
    lm.role = ROLE_LM;
    from_h(lm, I->out_norm);
    lm.mp.y = I->m_logits;
    lm.mp.ldy = I->Vl;
    lm.mp.vocab_offset = I->vocab_off;
    lm.mp.pf_ptr = I->layers[0].qkv;
    lm.mp.pf_bytes = I->layers[0].qkv_sh.bytes;
    ops.push_back(lm);
    if (tp) {
        Op ar{OP_ALLREDUCE_MAXU64};
        ar.buf = I->ms->best;
        ar.count = (size_t)n;
        ops.push_back(ar);
    }
    Op fin{OP_MFINAL};
    fin.n_vec = n;
    ops.push_back(fin);
}

// Phase table of the persistent step (tp_size == 1). Every phase
// waits for the one before it; the residual stream is hA, updated in place by the o and
// down epilogues.
void build_step(jinf_engine_impl* I, bool with_head, std::vector<StepPhase>& ph) {
    ph.clear();
    auto add_gemv = [&](const uint8_t* w, const Q4MShape& sh, int xm, int epi) -> StepPhase& {
        StepPhase p{};
        p.kind = PH_GEMV;
        p.xm = xm;
        p.epi = epi;
        p.w = w;
        p.rows = sh.rows;
        p.cols = sh.cols;
        p.pairs = sh.pairs;
        p.groups = sh.groups;
        p.fmts = sh.fmt | (sh.fmt << 4) | (sh.pairs << 8);
        p.gran = 1;
        p.xin = p.xout = -1;
        ph.push_back(p);
        return ph.back();
    };
    // tensor parallel: o and down store partials into exchange points 2L and 2L + 1 of every
    // rank; the next RMSNorm input adds them up (h ping-pongs between hA and hB, so that no
    // CTA overwrites the h another CTA is still reading)
    const bool tp = I->tp_size > 1;
    float* hcur = I->hA;
    auto tp_input = [&](StepPhase& p, int point) {
        p.xm = X_RMSNORM_TP;
        p.xin = point;
        p.hsrc = hcur;
        p.hout = hcur == I->hA ? I->hB : I->hA;
        hcur = p.hout;
    };
    for (int L = 0; L < I->L; ++L) {
        const auto& ly = I->layers[L];
        __half* kc = I->kc + (size_t)L * I->Hkvl * I->max_ctx * I->hd;
        __half* vc = I->vc + (size_t)L * I->Hkvl * I->max_ctx * I->hd;
        // The attention output and the activation arrive as records from their producing
        // phase (attention -> o: rec 0, gate|up -> down: rec 2). The RMSNorm inputs are staged
        // by every CTA from h (records of h * gain would cost the o and down epilogues an
        // extra dependent round trip each, more than they save; step_rec[1], [3] and
        // step_ss stay available for that form).
        StepPhase& qkv = add_gemv(ly.qkv, ly.qkv_sh, L == 0 ? X_EMBED_NORM : X_RMSNORM, EPI_QKV);
        if (ly.v) {  // [q | k] rows, then the v rows of their own type right after them
            qkv.rows = ly.qkv_sh.rows + ly.v_sh.rows;
            qkv.pairs = ly.qkv_sh.pairs + ly.v_sh.pairs;
            qkv.fmts = ly.qkv_sh.fmt | (ly.v_sh.fmt << 4) | (ly.qkv_sh.pairs << 8);
        }
        qkv.hsrc = L == 0 ? I->embed : I->hA;
        qkv.hout = L == 0 ? I->hA : nullptr;
        if (tp && L > 0) tp_input(qkv, 2 * (L - 1) + 1);
        qkv.norm_w = ly.attn_norm;
        qkv.y = I->q;
        qkv.kcache = kc;
        qkv.vcache = vc;
        StepPhase at{};
        at.kind = PH_ATTN;
        at.xin = at.xout = -1;
        at.q = I->q;
        at.out = I->attn;
        at.kcache = kc;
        at.vcache = vc;
        at.layer = L;
        at.rec_out = I->step_rec[0];
        at.groups_out = ly.o_sh.groups;
        ph.push_back(at);
        StepPhase& o = add_gemv(ly.o, ly.o_sh, X_RECORDS, tp ? EPI_PARTIAL : EPI_RESID);
        o.rec = I->step_rec[0];
        o.y = I->hA;
        if (tp) o.xout = 2 * L;
        StepPhase& gu = add_gemv(ly.gu, ly.gu_sh, X_RMSNORM, EPI_GATEUP);
        gu.hsrc = I->hA;
        if (tp) tp_input(gu, 2 * L);
        gu.norm_w = ly.ffn_norm;
        gu.gran = 2;
        gu.rec_out = I->step_rec[2];
        gu.groups_out = ly.down_sh.groups;
        StepPhase& dn = add_gemv(ly.down, ly.down_sh, X_RECORDS, tp ? EPI_PARTIAL : EPI_RESID);
        dn.rec = I->step_rec[2];
        dn.y = I->hA;
        if (tp) dn.xout = 2 * L + 1;
    }
    if (with_head) {
        StepPhase& lm = add_gemv(I->lm, I->lm_sh, X_RMSNORM, EPI_LMHEAD);
        lm.hsrc = I->hA;
        if (tp) {
            tp_input(lm, 2 * (I->L - 1) + 1);
            lm.hout = nullptr;  // the step's last h is not needed
        }
        lm.norm_w = I->out_norm;
        lm.y = I->logits;
    }
    for (size_t i = 0; i < ph.size(); ++i) {
        ph[i].dep = (int)i - 1;
        // GEMV phases report tile pairs, attention its 32-element output blocks
        ph[i].dep_target = i == 0                      ? 0u
                           : ph[i - 1].kind == PH_GEMV ? (unsigned)ph[i - 1].pairs
                                                       : (unsigned)(I->Hl * I->hd / 32);
        ph[i].pf[0] = ph[i].pf[1] = -1;
    }
    // L2 prefetch schedule (phase order per layer: qkv, attention, o, gate|up, down). HBM
    // would idle while attention runs and while CTAs stage inputs and merge rows; in those
    // windows each CTA pulls the weights it owns in a later phase into L2, and the later
    // ring copies hit L2. At most ~80 MB are outstanding at any time (L2: 126 MB).
    const int n = (int)ph.size();
    for (int i = 0; i < n; ++i) {
        const bool gemv_next = i + 1 < n && ph[i + 1].kind == PH_GEMV;
        if (ph[i].kind == PH_ATTN) {
            if (JINF_STEP_PF_MODE >= 1 && i + 2 < n) {
                ph[i].pf[0] = i + 1;  // o
                ph[i].pf[1] = i + 2;  // gate|up
            }
        } else if (ph[i].epi == EPI_GATEUP) {
            if (JINF_STEP_PF_MODE >= 2 && gemv_next) ph[i].pf[0] = i + 1;  // down
        } else if (ph[i].epi == EPI_RESID && i > 0 && ph[i - 1].epi == EPI_GATEUP) {
            if (JINF_STEP_PF_MODE >= 3 && gemv_next && ph[i + 1].epi == EPI_QKV) ph[i].pf[0] = i + 1;  // next qkv
        }
    }
}

// Tensor-parallel persistent step: allocate this rank's exchange area (zeroed), share its
// IPC handle with every rank over NCCL and map the peers' areas. Returns false (and logs)
// when peer mappings are not available; the engine then runs one kernel per operation.
bool setup_exchange(jinf_engine_impl* I) {
    const int tp = I->tp_size, rank = I->tp_rank;
    const NcclApi* n = nccl_api();
    if (tp > STEP_MAX_TP || !n || !I->comm) return false;
    I->xl = step_xchg_layout(2 * I->L, tp, I->d);
    if (cudaMalloc(&I->xchg, I->xl.total) != cudaSuccess) return false;
    cudaMemset(I->xchg, 0, I->xl.total);
    cudaDeviceSynchronize();  // zero before any peer can have the handle
    cudaIpcMemHandle_t mine;
    if (cudaIpcGetMemHandle(&mine, I->xchg) != cudaSuccess) {
        JINF_LOG("tensor-parallel persistent step: no IPC handle for the exchange area");
        cudaGetLastError();
        return false;
    }
    std::vector<cudaIpcMemHandle_t> all(tp);
    uint8_t* dev = nullptr;
    if (cudaMalloc(&dev, sizeof(cudaIpcMemHandle_t) * tp) != cudaSuccess) return false;
    cudaMemcpy(dev + sizeof(cudaIpcMemHandle_t) * rank, &mine, sizeof mine, cudaMemcpyHostToDevice);
    const bool ok = n->AllGather(dev + sizeof(cudaIpcMemHandle_t) * rank, dev, sizeof(cudaIpcMemHandle_t), ncclUint8,
                                 I->comm, I->stream) == ncclSuccess &&
                    cudaStreamSynchronize(I->stream) == cudaSuccess &&
                    cudaMemcpy(all.data(), dev, sizeof(cudaIpcMemHandle_t) * tp, cudaMemcpyDeviceToHost) == cudaSuccess;
    cudaFree(dev);
    if (!ok) return false;
    bool mapped = true;
    for (int r = 0; r < tp; ++r) {
        if (r == rank) {
            I->xpeer[r] = I->xchg;
            continue;
        }
        void* p = nullptr;
        if (cudaIpcOpenMemHandle(&p, all[r], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            JINF_LOG("tensor-parallel persistent step: rank %d's exchange area cannot be mapped", r);
            cudaGetLastError();
            mapped = false;
            break;
        }
        I->xpeer[r] = (uint8_t*)p;
    }
    // every rank must agree: all ranks take the persistent form or none does
    int* flag = nullptr;
    int v = mapped ? 1 : 0;
    if (cudaMalloc(&flag, sizeof(int)) != cudaSuccess) return false;
    cudaMemcpy(flag, &v, sizeof v, cudaMemcpyHostToDevice);
    const bool agreed = n->AllReduce(flag, flag, 1, ncclInt32, ncclMin, I->comm, I->stream) == ncclSuccess &&
                        cudaStreamSynchronize(I->stream) == cudaSuccess &&
                        cudaMemcpy(&v, flag, sizeof v, cudaMemcpyDeviceToHost) == cudaSuccess && v == 1;
    cudaFree(flag);
    return agreed;
}

void free_exchange(jinf_engine_impl* I) {
    for (int r = 0; r < STEP_MAX_TP; ++r)
        if (I->xpeer[r] && I->xpeer[r] != I->xchg) cudaIpcCloseMemHandle(I->xpeer[r]);
    for (int r = 0; r < STEP_MAX_TP; ++r) I->xpeer[r] = nullptr;
    if (I->xchg) cudaFree(I->xchg);
    I->xchg = nullptr;
}

// Set up the persistent step: phase tables on the device, counters and partial buffers.
// Returns JINF_OK with I->persistent = false when the shape does not fit the kernel.
jinf_status setup_persistent(jinf_engine_impl* I) {
    I->persistent = false;
    const int G = I->Hl / I->Hkvl;
    int max_cols = I->d;
    for (const auto& ly : I->layers)
        for (const Q4MShape* sh : {&ly.qkv_sh, &ly.o_sh, &ly.gu_sh, &ly.down_sh}) max_cols = std::max(max_cols, sh->cols);
    const unsigned xs = step_xstage_bytes(max_cols, G, I->hd);
    // ring depth: STEP_NBUF slots per warp when they fit next to the staged inputs, else 3
    int nbuf = I->wfmt == Q4M_MIX ? 3 : STEP_NBUF;
    size_t smem = step_smem_bytes(xs, 5 * I->L + 1, I->wfmt, nbuf);
    if (smem > 227 * 1024) {
        nbuf = 3;
        smem = step_smem_bytes(xs, 5 * I->L + 1, I->wfmt, nbuf);
    }
    // input records: a tile pair of h is one 32-element block, a CTA's gate|up rows are whole
    // activation blocks and fit the 1024-float conversion buffer, as do a kv head's outputs
    const int gu_pairs = I->layers.empty() ? 0 : I->layers[0].gu_sh.pairs;
    const int gu_per_cta = 2 * ((gu_pairs / 2 + I->num_sms - 1) / I->num_sms);
    const bool records_ok = I->d % 32 == 0 && (I->Hl * I->hd) % 32 == 0 && gu_pairs % 2 == 0 &&
                            gu_per_cta * 16 <= 1024 && G * I->hd <= 1024;
    if (G > ATTN_MAX_GROUP || (G & (G - 1)) || I->Hkvl > 64 || (I->hd != 64 && I->hd != 128) || smem > 227 * 1024 ||
        step_occupancy(smem, I->wfmt, nbuf) < 1 || !records_ok) {
        JINF_LOG("persistent step unavailable for this shape (%zu bytes of shared memory); using one kernel per "
                 "operation", smem);
        return JINF_OK;
    }
    I->step_grid = I->num_sms;
    {
        const auto& ly = I->layers[0];
        const int rec_groups[4] = {ly.o_sh.groups, ly.gu_sh.groups, ly.down_sh.groups,
                                   std::max(ly.qkv_sh.groups, I->lm_sh.groups)};
        for (int i = 0; i < 4; ++i) {
            // zero once: padding blocks past the real columns are never written and stay zero
            JINF_CUDA_CHECK(cudaMalloc(&I->step_rec[i], xrec_bytes(rec_groups[i])));
            JINF_CUDA_CHECK(cudaMemset(I->step_rec[i], 0, xrec_bytes(rec_groups[i])));
        }
        JINF_CUDA_CHECK(cudaMalloc(&I->step_ss, sizeof(float) * (size_t)(I->d / 32)));
        JINF_CUDA_CHECK(cudaMalloc(&I->step_attn_cnt, sizeof(unsigned int) * (size_t)I->L * I->Hkvl));
        JINF_CUDA_CHECK(cudaMemset(I->step_attn_cnt, 0, sizeof(unsigned int) * (size_t)I->L * I->Hkvl));
    }
    std::vector<StepPhase> full, body;
    build_step(I, true, full);
    build_step(I, false, body);
    const size_t attn_floats = (size_t)I->Hkvl * ATTN_MAX_SPLIT * ATTN_MAX_GROUP * (I->hd + 2);
    std::vector<StepPhase> all(full);
    all.insert(all.end(), body.begin(), body.end());
    JINF_CUDA_CHECK(cudaMalloc(&I->d_phases, sizeof(StepPhase) * all.size()));
    JINF_CUDA_CHECK(cudaMalloc(&I->step_done, sizeof(unsigned int) * (full.size() + 1)));
    JINF_CUDA_CHECK(cudaMalloc(&I->step_attn_part, sizeof(float) * attn_floats));
    JINF_CUDA_CHECK(cudaMemcpy(I->d_phases, all.data(), sizeof(StepPhase) * all.size(), cudaMemcpyHostToDevice));
    JINF_CUDA_CHECK(cudaMemset(I->step_done, 0, sizeof(unsigned int) * (full.size() + 1)));
    StepParams sp{};
    sp.done = I->step_done;
    sp.attn_part = I->step_attn_part;
    sp.attn_cnt = I->step_attn_cnt;
    sp.n_attn_cnt = I->L * I->Hkvl;
    sp.st = I->st;
    sp.nq = I->Hl * I->hd;
    sp.nk = I->Hkvl * I->hd;
    sp.head_dim = I->hd;
    sp.max_ctx = I->max_ctx;
    sp.n_heads = I->Hl;
    sp.n_kv_heads = I->Hkvl;
    sp.rope_base = I->rope_base;
    sp.eps = I->eps;
    sp.attn_smax = std::max(1, std::min(ATTN_MAX_SPLIT, I->num_sms / I->Hkvl));
    sp.fmt = I->wfmt;
    sp.nbuf = nbuf;
    sp.xstage_bytes = xs;
    sp.spin_limit = 4000000ull;  // about a second of polling: far beyond any phase, never a hang
    sp.tp_rank = I->tp_rank;
    sp.tp_size = I->tp_size;
    sp.vocab_off = I->vocab_off;
    if (I->tp_size > 1) {
        for (int r = 0; r < I->tp_size; ++r) sp.xpeer[r] = I->xpeer[r];
        sp.x_keycnt = I->xl.keycnt;
        sp.x_keys = I->xl.keys;
        sp.x_data = I->xl.data;
        sp.x_point = I->xl.point;
        sp.x_slot = I->xl.slot;
    }
    I->sp_full = sp;
    I->sp_full.phases = I->d_phases;
    I->sp_full.n_phases = (int)full.size();
    I->sp_full.with_argmax = 1;
    I->sp_body = sp;
    I->sp_body.phases = I->d_phases + full.size();
    I->sp_body.n_phases = (int)body.size();
    I->sp_body.with_argmax = 0;
    I->persistent = true;
    return JINF_OK;
}

// ---------------------------------------------------------------- loading

struct Loader {
    jinf_engine_impl* I;
    const ModelSource* src;
    std::vector<uint8_t> host;  // AoS staging on the host
    uint8_t* dstage = nullptr;  // AoS staging on the device
    size_t dstage_bytes = 0;

    ~Loader() {
        if (dstage) cudaFree(dstage);
    }

    jinf_status ensure_dstage(size_t n) {
        if (n <= dstage_bytes) return JINF_OK;
        if (dstage) cudaFree(dstage);
        dstage = nullptr;
        JINF_CUDA_CHECK(cudaMalloc(&dstage, n));
        dstage_bytes = n;
        return JINF_OK;
    }

    // Replace the staged matrix by a gather of it (via a scratch buffer of the same size).
    jinf_status gather_rows(const std::vector<int>& idx, int row_bytes) {
        uint8_t* tmp = nullptr;
        int* didx = nullptr;
        JINF_CUDA_CHECK(cudaMalloc(&tmp, (size_t)idx.size() * row_bytes));
        JINF_CUDA_CHECK(cudaMalloc(&didx, sizeof(int) * idx.size()));
        JINF_CUDA_CHECK(cudaMemcpy(didx, idx.data(), sizeof(int) * idx.size(), cudaMemcpyHostToDevice));
        k_gather_rows<<<1184, 256, 0, I->stream>>>(dstage, tmp, didx, (int)idx.size(), row_bytes);
        JINF_CUDA_CHECK(cudaGetLastError());
        JINF_CUDA_CHECK(cudaMemcpyAsync(dstage, tmp, (size_t)idx.size() * row_bytes, cudaMemcpyDeviceToDevice, I->stream));
        JINF_CUDA_CHECK(cudaStreamSynchronize(I->stream));
        cudaFree(tmp);
        cudaFree(didx);
        return JINF_OK;
    }
    jinf_status gather_blocks(const std::vector<int>& blk, int rows, int nb_src, int bb) {
        uint8_t* tmp = nullptr;
        int* dblk = nullptr;
        const size_t bytes = (size_t)rows * blk.size() * bb;
        JINF_CUDA_CHECK(cudaMalloc(&tmp, bytes));
        JINF_CUDA_CHECK(cudaMalloc(&dblk, sizeof(int) * blk.size()));
        JINF_CUDA_CHECK(cudaMemcpy(dblk, blk.data(), sizeof(int) * blk.size(), cudaMemcpyHostToDevice));
        k_gather_blocks<<<1184, 256, 0, I->stream>>>(dstage, tmp, dblk, rows, nb_src, (int)blk.size(), bb);
        JINF_CUDA_CHECK(cudaGetLastError());
        JINF_CUDA_CHECK(cudaMemcpyAsync(dstage, tmp, bytes, cudaMemcpyDeviceToDevice, I->stream));
        JINF_CUDA_CHECK(cudaStreamSynchronize(I->stream));
        cudaFree(tmp);
        cudaFree(dblk);
        return JINF_OK;
    }

    // Stage rows [r0, r0+nr) x columns [c0, c0+nc) of Q4_0 tensor `name` as AoS blocks into
    // the device staging buffer, row i at staging row dst_row0 + i*dst_step (pitch
    // dst_row_bytes). Synthetic models are generated in place on the device; files are
    // read on the host and copied with one pitched copy.
    jinf_status stage(const char* name, int64_t r0, int64_t nr, int64_t c0, int64_t nc, int64_t dst_row_bytes,
                      int64_t dst_row0, int64_t dst_step) {
        TensorMeta m;
        if (!src->meta(name, &m)) {
            JINF_LOG("tensor %s missing", name);
            return JINF_ERR_PARSE;
        }
        if (q4m_fmt_of_qtype(m.type) < 0) {
            JINF_LOG("tensor %s: type %s has no Q4M form", name, jinf_qtype_name((jinf_qtype)m.type));
            return JINF_ERR_INVALID;
        }
        const int bs = jinf_qtype_block_size((jinf_qtype)m.type), bb = (int)jinf_qtype_type_size((jinf_qtype)m.type);
        if (r0 < 0 || c0 < 0 || r0 + nr > m.rows() || c0 + nc > m.cols() || c0 % bs || nc % bs) {
            JINF_LOG("tensor %s: slice [%lld+%lld, %lld+%lld) out of range", name, (long long)r0, (long long)nr,
                     (long long)c0, (long long)nc);
            return JINF_ERR_INVALID;
        }
        jinf_status st = JINF_OK;
        if (src->device_quant(name, r0, nr, c0, nc, dstage, dst_row_bytes, dst_row0, dst_step, I->stream, &st))
            return st;
        const uint64_t rb = m.row_bytes();
        host.resize((size_t)(nr * rb));
        JINF_CHECK(src->read_rows(name, r0, nr, host.data()), name);
        JINF_CUDA_CHECK(cudaMemcpy2DAsync(dstage + dst_row0 * dst_row_bytes, (size_t)(dst_step * dst_row_bytes),
                                          host.data() + (c0 / bs) * bb, (size_t)rb, (size_t)(nc / bs) * bb,
                                          (size_t)nr, cudaMemcpyHostToDevice, I->stream));
        JINF_CUDA_CHECK(cudaStreamSynchronize(I->stream));  // `host` is reused by the next call
        return JINF_OK;
    }

    // Stage this rank's tensor-parallel slice of `name` (jinf_tp_shard), which must be
    // want_rows x want_cols.
    jinf_status stage_shard(const char* name, int64_t want_rows, int64_t want_cols, int64_t dst_row_bytes,
                            int64_t dst_row0, int64_t dst_step) {
        TensorMeta m;
        if (!src->meta(name, &m)) {
            JINF_LOG("tensor %s missing", name);
            return JINF_ERR_PARSE;
        }
        int64_t r0, nr, c0, nc;
        if (jinf_tp_shard(name, m.rows(), m.cols(), I->tp_rank, I->tp_size, &r0, &nr, &c0, &nc) != JINF_OK ||
            nr != want_rows || nc != want_cols) {
            JINF_LOG("tensor %s: shard of rank %d/%d does not match the model shape", name, I->tp_rank, I->tp_size);
            return JINF_ERR_INVALID;
        }
        return stage(name, r0, nr, c0, nc, dst_row_bytes, dst_row0, dst_step);
    }

    // Repack the staged AoS matrix into the arena.
    jinf_status pack(uint8_t* dst, const Q4MShape& sh) {
        JINF_CUDA_CHECK(q4m_repack(dstage, dst, sh, I->stream));
        JINF_CUDA_CHECK(cudaStreamSynchronize(I->stream));
        return JINF_OK;
    }

    jinf_status read_f32(const char* name, float* dst_dev, int64_t n_expect) {
        TensorMeta m;
        if (!src->meta(name, &m)) {
            JINF_LOG("tensor %s missing", name);
            return JINF_ERR_PARSE;
        }
        const int64_t n = m.rows() * m.cols();
        if (n != n_expect) {
            JINF_LOG("tensor %s: %lld elements, expected %lld", name, (long long)n, (long long)n_expect);
            return JINF_ERR_PARSE;
        }
        jinf_status dst_status = JINF_OK;
        if (src->device_f32(name, dst_dev, I->stream, &dst_status)) {
            if (dst_status == JINF_OK) JINF_CUDA_CHECK(cudaStreamSynchronize(I->stream));
            return dst_status;
        }
        const uint64_t bytes = m.row_bytes() * (uint64_t)m.rows();
        // read in slabs of rows to bound host memory
        const int64_t rows = m.rows();
        const int64_t slab = rows > 4096 ? 4096 : rows;
        std::vector<uint8_t> buf((size_t)(slab * m.row_bytes()));
        std::vector<float> f32;
        for (int64_t r = 0; r < rows; r += slab) {
            const int64_t nr = r + slab <= rows ? slab : rows - r;
            JINF_CHECK(src->read_rows(name, r, nr, buf.data()), name);
            const int64_t ne = nr * m.cols();
            float* dst = dst_dev + r * m.cols();
            if (m.type == JINF_TYPE_F32) {
                JINF_CUDA_CHECK(cudaMemcpy(dst, buf.data(), (size_t)ne * 4, cudaMemcpyHostToDevice));
            } else {
                f32.resize((size_t)ne);
                jinf_dequantize(buf.data(), (jinf_qtype)m.type, f32.data(), ne);
                if (m.type != JINF_TYPE_F16 && m.type != JINF_TYPE_Q4_0 && m.type != JINF_TYPE_Q4_K &&
                    m.type != JINF_TYPE_Q8_0 && m.type != JINF_TYPE_Q6_K) {
                    JINF_LOG("tensor %s: unsupported type %d", name, m.type);
                    return JINF_ERR_INVALID;
                }
                JINF_CUDA_CHECK(cudaMemcpy(dst, f32.data(), (size_t)ne * 4, cudaMemcpyHostToDevice));
            }
        }
        (void)bytes;
        return JINF_OK;
    }
};

void free_impl(jinf_engine_impl* I) {
    if (!I) return;
    if (I->device >= 0) cudaSetDevice(I->device);
    if (I->exec_full) cudaGraphExecDestroy(I->exec_full);
    if (I->exec_body) cudaGraphExecDestroy(I->exec_body);
    for (cudaGraphExec_t& g : I->m_exec)
        if (g) cudaGraphExecDestroy(g);
    if (I->stream) cudaStreamSynchronize(I->stream);
    free_exchange(I);  // every write of a peer into this area landed before our last step ended
    if (I->comm) {
        const NcclApi* n = nccl_api();
        if (n) n->CommDestroy(I->comm);
    }
    void* ptrs[] = {I->arena, I->norms, I->embed, I->kc, I->vc, I->hA, I->hB, I->y_o, I->y_down, I->q, I->attn,
                    I->act, I->gate_raw, I->logits, I->attn_partial, I->st, I->dev_tokens, I->gemv_part,
                    I->gemv_cnt, I->d_phases, I->step_done, I->step_attn_part, I->step_rec[0], I->step_rec[1], I->step_rec[2], I->step_rec[3], I->step_ss, I->step_attn_cnt, I->pf_h, I->pf_y,
                    I->pf_att, I->pf_sc, I->pf_x16, I->pf_q16, I->pf_err, I->bundles, I->pred_w1,
                    I->pred_w2, I->sparse_ids, I->sparse_offs, I->sparse_x, I->sparse_scratch, I->gate_up_tmp,
                    I->ms, I->m_h, I->m_y, I->m_q, I->m_attn, I->m_act, I->m_logits, I->m_ssq, I->m_attn_part,
                    I->m_part, I->m_cnt, I->m_out, I->m_rec_h, I->m_rec_a};
    for (void* p : ptrs)
        if (p) cudaFree(p);
    if (I->logits_full && I->logits_full != I->logits) cudaFree(I->logits_full);
    if (I->pinned) cudaFreeHost(I->pinned);
    if (I->ms_pinned) cudaFreeHost(I->ms_pinned);
    if (I->ev0) cudaEventDestroy(I->ev0);
    if (I->ev1) cudaEventDestroy(I->ev1);
    if (I->stream) cudaStreamDestroy(I->stream);
    delete I;
}

jinf_status create_from_source(jinf_engine** out, const jinf_engine_config* cfg, const ModelSource& src,
                               const jinf_b200_options* opt_in) {
    jinf_b200_options opt = opt_in ? *opt_in : jinf_b200_options_default();
    const jinf_model_hparams& hp = src.hp;
    if (hp.n_layers == 0 || hp.n_embd == 0 || hp.n_heads == 0 || hp.n_ff == 0 || hp.n_vocab == 0) {
        JINF_LOG("model hyper-parameters incomplete");
        return JINF_ERR_PARSE;
    }
    const int tp = opt.tp_size > 0 ? opt.tp_size : 1;
    const int hkv = hp.n_heads_kv ? (int)hp.n_heads_kv : (int)hp.n_heads;
    if ((int)hp.n_heads % tp || hkv % tp || (int)hp.n_ff % tp || (int)hp.n_vocab % tp || opt.tp_rank < 0 ||
        opt.tp_rank >= tp) {
        JINF_LOG("tensor-parallel size %d does not divide the model (heads %u/%d, ff %u, vocab %u)", tp, hp.n_heads,
                 hkv, hp.n_ff, hp.n_vocab);
        return JINF_ERR_INVALID;
    }
    if (cfg->max_context <= 0) return JINF_ERR_INVALID;
    if (opt.kv_type != JINF_TYPE_F16) {
        JINF_LOG("only the fp16 KV cache is implemented on B200");
        return JINF_ERR_INVALID;
    }

    jinf_engine_impl* I = new jinf_engine_impl();
    I->device = opt.device;
    I->tp_rank = opt.tp_rank;
    I->tp_size = tp;
    I->use_graph = opt.use_graph != 0;
    I->prefill = opt.prefill != 0;
    I->eos = opt.eos_token;
    I->d = (int)hp.n_embd;
    I->H = (int)hp.n_heads;
    I->Hkv = hkv;
    I->hd = I->d / I->H;
    I->ff = (int)hp.n_ff;
    I->V = (int)hp.n_vocab;
    I->L = (int)hp.n_layers;
    I->Hl = I->H / tp;
    I->Hkvl = I->Hkv / tp;
    I->ffl = I->ff / tp;
    I->Vl = I->V / tp;
    I->vocab_off = I->Vl * opt.tp_rank;
    I->eps = hp.rms_norm_eps;
    I->rope_base = hp.rope_freq_base;
    I->max_ctx = cfg->max_context;
    auto fail = [&](jinf_status s) {
        free_impl(I);
        return s;
    };
    if (I->hd != 64 && I->hd != 128) {
        JINF_LOG("head_dim %d not supported (64 or 128)", I->hd);
        return fail(JINF_ERR_INVALID);
    }
    // the projections' quantisation, per matrix: Q4_0, Q4_K, Q6_K or Q8_0 (Q4_K_M files
    // keep attn_v, ffn_down of some layers and the output head in Q6_K); q and k, and gate
    // and up, must share a type (they are fused). The persistent step serves models whose
    // matrices are all Q4_0 or all Q4_K; others run one kernel per operation.
    std::vector<std::array<int, 5>> lfmt((size_t)I->L);  // per layer: q|k, v, o, gate|up, down
    int lm_fmt = -1;
    // a pre-packed file: this rank's images (a tensor-parallel file holds one set per rank)
    if (src.prepacked() && tp > 1 && !src.select_shard(opt.tp_rank, tp)) {
        JINF_LOG("this B200-layout model file holds no images for %d GPUs (jinf_prepare_model_b200_tp)", tp);
        return fail(JINF_ERR_INVALID);
    }
    {
        TensorMeta m;
        if (src.meta("blk.0.attn_q.weight", &m)) I->wtype = m.type;
        auto fmt_of = [&](const char* nm, int* fmt) -> bool {
            TensorMeta t;
            if (!src.meta(nm, &t)) {
                JINF_LOG("tensor %s missing", nm);
                return false;
            }
            *fmt = q4m_fmt_of_qtype(t.type);
            if (*fmt < 0) {
                JINF_LOG("tensor %s: weights of type %s are not supported by the B200 engine (Q4_0, Q4_K, Q6_K or "
                         "Q8_0)", nm, jinf_qtype_name((jinf_qtype)t.type));
                return false;
            }
            return true;
        };
        char nm[128];
        for (int L = 0; L < I->L; ++L) {
            int f[7];
            const char* parts[7] = {"attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"};
            for (int i = 0; i < 7; ++i) {
                snprintf(nm, sizeof nm, "blk.%d.%s.weight", L, parts[i]);
                if (!fmt_of(nm, &f[i])) return fail(JINF_ERR_INVALID);
            }
            if (f[0] != f[1] || f[4] != f[5]) {
                JINF_LOG("layer %d: attn_q and attn_k, and ffn_gate and ffn_up, must share a weight type", L);
                return fail(JINF_ERR_INVALID);
            }
            lfmt[L] = {f[0], f[2], f[3], f[4], f[6]};
        }
        if (!fmt_of("output.weight", &lm_fmt)) return fail(JINF_ERR_INVALID);
        I->step_formats = lm_fmt != Q4M_Q8_0;
        for (const auto& lf : lfmt)
            for (const int f : lf) {
                I->uniform = I->uniform && f == lm_fmt;
                I->step_formats = I->step_formats && f != Q4M_Q8_0;
            }
        I->uniform = I->uniform && (lm_fmt == Q4M_Q4_0 || lm_fmt == Q4M_Q4_K);
        I->wfmt = I->uniform ? lm_fmt : Q4M_MIX;
        if (I->uniform) I->wtype = lm_fmt == Q4M_Q4_K ? JINF_TYPE_Q4_K : JINF_TYPE_Q4_0;
        if (src.prepacked() && opt.sparse_mode) {
            JINF_LOG("a B200-layout model file is prepared for the dense FFN");
            return fail(JINF_ERR_INVALID);
        }
        if (!I->uniform && opt.sparse_mode) {
            JINF_LOG("sparse FFN modes need every projection in one type, Q4_0 or Q4_K");
            return fail(JINF_ERR_INVALID);
        }
    }
    if (I->H / I->Hkv > 8) {
        JINF_LOG("more than 8 query heads per kv head are not supported");
        return fail(JINF_ERR_INVALID);
    }
    I->sparse_mode = opt.sparse_mode;
    if (I->sparse_mode < 0 || I->sparse_mode > 2 || (I->sparse_mode && (tp > 1 || !(opt.sparse_keep > 0.f) ||
                                                                       opt.sparse_keep > 1.f || I->d % 32 ||
                                                                       I->d > 8192 ||
                                                                       (I->sparse_mode == 1 &&
                                                                        I->ff > JINF_TOPK_MAX_N)))) {
        JINF_LOG("sparse_mode %d (keep %.3f) not supported: modes 0-2, keep in (0, 1], one GPU, d <= 8192, "
                 "predictor n_ff <= %d",
                 opt.sparse_mode, opt.sparse_keep, JINF_TOPK_MAX_N);
        return fail(JINF_ERR_INVALID);
    }
    if (cudaSetDevice(I->device) != cudaSuccess) {
        JINF_LOG("cannot select CUDA device %d", I->device);
        return fail(JINF_ERR_CUDA);
    }
    cudaDeviceGetAttribute(&I->num_sms, cudaDevAttrMultiProcessorCount, I->device);
    if (cudaStreamCreateWithFlags(&I->stream, cudaStreamNonBlocking) != cudaSuccess) return fail(JINF_ERR_CUDA);
    cudaEventCreate(&I->ev0);
    cudaEventCreate(&I->ev1);

    // ---- fixed masks in the persistent step: gate|up and down compacted to the 32-neuron
    // blocks that hold an active neuron (Q4_0 only: its blocks are 32 columns wide)
    // the static active sets of mode 2: the reference's activation profile when the config
    // names one (reference src/engine.cpp:228-252: a profile that cannot be read leaves the
    // FFN dense), else the seeded fixed masks
    if (cfg->predictor_path && src.prepacked()) {
        // a B200-layout file holds the dense gate|up and down images only (as the reference
        // runs a dense FFN for a model without neuron bundles, src/engine.cpp:253-255)
        JINF_LOG("Warning: predictor path set but the B200-layout model holds no sparse FFN form; dense FFN");
    } else if (cfg->predictor_path && tp == 1 && I->d <= 8192) {
        std::vector<int32_t> ids((size_t)I->L * I->ffl), cnt(I->L);
        const jinf_status ps = jinf_activation_profile_read(cfg->predictor_path, cfg->sparsity_threshold, I->L, I->ffl,
                                                            ids.data(), cnt.data());
        if (ps == JINF_OK) {
            I->sparse_mode = 2;
            I->static_ids.assign(I->L, {});
            for (int L = 0; L < I->L; ++L)
                I->static_ids[L].assign(ids.begin() + (size_t)L * I->ffl, ids.begin() + (size_t)L * I->ffl + cnt[L]);
            JINF_LOG("static predictor %s (threshold %.2f): sparse FFN", cfg->predictor_path, cfg->sparsity_threshold);
        } else {
            JINF_LOG("Warning: cannot use the activation profile %s (%s); dense FFN", cfg->predictor_path,
                     jinf_status_str(ps));
        }
    } else if (I->sparse_mode == 2) {
        std::vector<int32_t> ids(I->ffl);
        I->static_ids.assign(I->L, {});
        for (int L = 0; L < I->L; ++L) {
            const int n = jinf_sparse_fixed_mask(opt.sparse_seed, L, I->ffl, opt.sparse_keep, ids.data());
            I->static_ids[L].assign(ids.begin(), ids.begin() + n);
        }
    }
    I->sparse_persistent = I->sparse_mode == 2 && opt.persistent && tp == 1 && I->wtype == JINF_TYPE_Q4_0 &&
                           I->ffl % 32 == 0;
    if (I->sparse_persistent) {
        I->sparse_blocks.assign(I->L, {});
        I->sparse_active.assign(I->L, std::vector<uint8_t>(I->ffl, 0));
        for (int L = 0; L < I->L; ++L) {
            const std::vector<int32_t>& ids = I->static_ids[L];
            const int n = (int)ids.size();
            for (int i = 0; i < n; ++i) {
                I->sparse_active[L][ids[i]] = 1;
                const int b = ids[i] / 32;
                if (I->sparse_blocks[L].empty() || I->sparse_blocks[L].back() != b) I->sparse_blocks[L].push_back(b);
            }
            if (I->sparse_blocks[L].empty()) I->sparse_blocks[L].push_back(0);  // keep a non-empty (all-zero) FFN
        }
    }

    // ---- shapes and arena layout (consumption order)
    const int d = I->d, hd = I->hd;
    const int qkv_rows = (I->Hl + 2 * I->Hkvl) * hd;
    I->layers.resize(I->L);
    uint64_t off = 0;
    auto place = [&](Q4MShape& sh, int rows, int cols, uint8_t*& ptr, int fmt) -> bool {
        if (!q4m_shape(rows, cols, &sh, fmt) || cols > gemvm_max_cols(fmt)) {
            JINF_LOG("a %d x %d matrix is not supported by the Q4M layout of its type (columns must be whole "
                     "%d-element blocks, at most %d)", rows, cols, q4m_col_align(fmt), gemvm_max_cols(fmt));
            return false;
        }
        ptr = (uint8_t*)(uintptr_t)off;  // offset for now
        off += (sh.bytes + 255) & ~255ull;
        I->weight_bytes_token += (uint64_t)rows * aos_row_bytes(fmt, cols);
        return true;
    };
    for (int L = 0; L < I->L; ++L) {
        auto& ly = I->layers[L];
        const auto& lf = lfmt[L];
        const int ffc = I->sparse_persistent ? 32 * (int)I->sparse_blocks[L].size() : I->ffl;  // FFN width stored
        const int qk_rows = (I->Hl + I->Hkvl) * hd;
        const bool split_v = lf[1] != lf[0];
        if (!place(ly.qkv_sh, split_v ? qk_rows : qkv_rows, d, ly.qkv, lf[0]) ||
            (split_v && !place(ly.v_sh, I->Hkvl * hd, d, ly.v, lf[1])) || !place(ly.o_sh, d, I->Hl * hd, ly.o, lf[2]) ||
            !place(ly.gu_sh, 2 * ffc, d, ly.gu, lf[3]) || !place(ly.down_sh, d, ffc, ly.down, lf[4]))
            return fail(JINF_ERR_INVALID);
    }
    if (!place(I->lm_sh, I->Vl, d, I->lm, lm_fmt)) return fail(JINF_ERR_INVALID);
    I->arena_bytes = off;
    if (cudaMalloc(&I->arena, I->arena_bytes) != cudaSuccess) {
        JINF_LOG("cannot allocate %.1f MB of weights", I->arena_bytes / 1048576.0);
        return fail(JINF_ERR_OOM);
    }
    for (auto& ly : I->layers) {
        ly.qkv = I->arena + (uintptr_t)ly.qkv;
        if (ly.v) ly.v = I->arena + (uintptr_t)ly.v;
        ly.o = I->arena + (uintptr_t)ly.o;
        ly.gu = I->arena + (uintptr_t)ly.gu;
        ly.down = I->arena + (uintptr_t)ly.down;
    }
    I->lm = I->arena + (uintptr_t)I->lm;

    // ---- other buffers
    const size_t kv_elems = (size_t)I->L * I->Hkvl * I->max_ctx * hd;  // one sequence's cache
    I->n_seqs = opt.max_seqs < 1 ? 1 : opt.max_seqs;
    if (I->n_seqs > MULTI_MAX || (I->n_seqs > 1 && I->sparse_mode)) {
        JINF_LOG("max_seqs must be 1..%d (dense FFN for more than one sequence)", MULTI_MAX);
        return fail(JINF_ERR_INVALID);
    }
    I->seq_stride = kv_elems;
    I->seq_past.assign(I->n_seqs, 0);
    // attention splits (the kernel uses one per 64 positions at run time, up to this many)
    I->n_split = std::max(1, std::min(64, (I->max_ctx + 63) / 64));
    bool ok = cudaMalloc(&I->norms, sizeof(float) * (size_t)(2 * I->L + 1) * d) == cudaSuccess &&
              cudaMalloc(&I->embed, sizeof(float) * (size_t)I->V * d) == cudaSuccess &&
              cudaMalloc(&I->kc, sizeof(__half) * kv_elems * I->n_seqs) == cudaSuccess &&
              cudaMalloc(&I->vc, sizeof(__half) * kv_elems * I->n_seqs) == cudaSuccess &&
              cudaMalloc(&I->hA, sizeof(float) * d) == cudaSuccess &&
              cudaMalloc(&I->hB, sizeof(float) * d) == cudaSuccess &&
              cudaMalloc(&I->y_o, sizeof(float) * d) == cudaSuccess &&
              cudaMalloc(&I->y_down, sizeof(float) * d) == cudaSuccess &&
              cudaMalloc(&I->q, sizeof(float) * (size_t)I->Hl * hd) == cudaSuccess &&
              cudaMalloc(&I->attn, sizeof(float) * (size_t)I->Hl * hd) == cudaSuccess &&
              cudaMalloc(&I->act, sizeof(float) * (size_t)I->ffl) == cudaSuccess &&
              cudaMalloc(&I->logits, sizeof(float) * (size_t)I->Vl) == cudaSuccess &&
              cudaMalloc(&I->attn_partial, sizeof(float) * attn_partial_floats(I->Hkvl, I->n_split, hd)) == cudaSuccess &&
              cudaMalloc(&I->st, sizeof(DeviceState)) == cudaSuccess &&
              cudaMalloc(&I->dev_tokens, sizeof(int32_t) * (size_t)I->max_ctx) == cudaSuccess &&
              cudaHostAlloc(&I->pinned, 4 * sizeof(int32_t), cudaHostAllocDefault) == cudaSuccess;
    if (ok) I->pinned[2] = DEV_OK;
    if (ok && tp > 1) ok = cudaMalloc(&I->logits_full, sizeof(float) * (size_t)I->V) == cudaSuccess;
    if (!ok) return fail(JINF_ERR_OOM);
    if (tp == 1) I->logits_full = I->logits;
    cudaMemset(I->kc, 0, sizeof(__half) * kv_elems * I->n_seqs);
    cudaMemset(I->vc, 0, sizeof(__half) * kv_elems * I->n_seqs);
    cudaMemset(I->st, 0, sizeof(DeviceState));
    cudaMemset(I->y_o, 0, sizeof(float) * d);
    cudaMemset(I->y_down, 0, sizeof(float) * d);

    // ---- sparse FFN mode: neuron bundles (filled while loading), predictor or fixed masks
    if (I->sparse_mode) {
        const size_t ff = (size_t)I->ffl;
        I->bundle_size = sparse_bundle_bytes(d, I->wtype);
        I->sparse_n.assign(I->L, 0);
        std::vector<int32_t> ids(ff * I->L, 0), offs(ff * I->L, 0);
        if (I->sparse_mode == 1) {
            I->pred_r = d / 4;
            I->sparse_k = (int)std::floor((double)opt.sparse_keep * (double)I->ffl);
            if (I->sparse_k < 1) I->sparse_k = 1;
            for (int L = 0; L < I->L; ++L) I->sparse_n[L] = I->sparse_k;
        } else {
            for (int L = 0; L < I->L; ++L) {
                I->sparse_n[L] = (int)I->static_ids[L].size();
                for (int i = 0; i < I->sparse_n[L]; ++i) {
                    ids[L * ff + i] = I->static_ids[L][i];
                    offs[L * ff + i] = ids[L * ff + i] * I->bundle_size;
                }
            }
        }
        bool sok = cudaMalloc(&I->bundles, (size_t)I->L * ff * I->bundle_size) == cudaSuccess &&
                   cudaMalloc(&I->sparse_ids, sizeof(int32_t) * ff * I->L) == cudaSuccess &&
                   cudaMalloc(&I->sparse_offs, sizeof(int32_t) * ff * I->L) == cudaSuccess &&
                   cudaMalloc(&I->sparse_x, sizeof(float) * (size_t)d) == cudaSuccess &&
                   cudaMalloc(&I->gate_up_tmp, sizeof(float) * ff) == cudaSuccess;
        if (sok && I->sparse_mode == 1)
            sok = cudaMalloc(&I->pred_w1, sizeof(__half) * (size_t)I->L * I->pred_r * d) == cudaSuccess &&
                  cudaMalloc(&I->pred_w2, sizeof(__half) * (size_t)I->L * ff * I->pred_r) == cudaSuccess &&
                  cudaMalloc(&I->sparse_scratch, sizeof(float) * ((size_t)I->pred_r + ff)) == cudaSuccess;
        if (!sok) {
            JINF_LOG("cannot allocate the sparse-FFN buffers (%.1f MB of bundles)",
                     (double)I->L * ff * I->bundle_size / 1048576.0);
            return fail(JINF_ERR_OOM);
        }
        cudaMemset(I->bundles, 0, (size_t)I->L * ff * I->bundle_size);
        JINF_CUDA_CHECK(cudaMemcpy(I->sparse_ids, ids.data(), sizeof(int32_t) * ids.size(), cudaMemcpyHostToDevice));
        JINF_CUDA_CHECK(cudaMemcpy(I->sparse_offs, offs.data(), sizeof(int32_t) * offs.size(), cudaMemcpyHostToDevice));
        if (I->sparse_mode == 1)
            for (int L = 0; L < I->L; ++L) {
                JINF_CUDA_CHECK(sparse_fill_predictor(opt.sparse_seed, L, 1, (int64_t)I->pred_r * d,
                                                      I->pred_w1 + (size_t)L * I->pred_r * d, I->stream));
                JINF_CUDA_CHECK(sparse_fill_predictor(opt.sparse_seed, L, 2, (int64_t)ff * I->pred_r,
                                                      I->pred_w2 + (size_t)L * ff * I->pred_r, I->stream));
            }
    }

    // ---- load weights (per matrix: stage AoS rows in HBM, then repack into the arena)
    {
        Loader ld{I, &src};
        size_t max_stage = 0;
        for (const auto& ly : I->layers)
            for (const Q4MShape* sh : {&ly.qkv_sh, &ly.v_sh, &ly.o_sh, &ly.gu_sh, &ly.down_sh})
                if (sh->rows > 0) max_stage = std::max(max_stage, (size_t)sh->rows * aos_row_bytes(sh->fmt, sh->cols));
        max_stage = std::max(max_stage, (size_t)I->lm_sh.rows * aos_row_bytes(I->lm_sh.fmt, I->lm_sh.cols));
        if (ld.ensure_dstage(max_stage) != JINF_OK) return fail(JINF_ERR_OOM);
        // AoS row bytes of a d-column Q4_0 / Q4_K matrix (both take 9/16 byte per weight): the
        // sparse FFN bundles, built from uniform Q4 models only
        const int64_t rb_d = (int64_t)(d / 32) * 18;
        char nm[128];
        jinf_status s = JINF_OK;
        for (int L = 0; L < I->L && s == JINF_OK; ++L) {
            auto& ly = I->layers[L];
            ly.attn_norm = I->norms + (size_t)(2 * L) * d;
            ly.ffn_norm = I->norms + (size_t)(2 * L + 1) * d;
            snprintf(nm, sizeof nm, "blk.%d.attn_norm.weight", L);
            s = ld.read_f32(nm, ly.attn_norm, d);
            if (s != JINF_OK) break;
            snprintf(nm, sizeof nm, "blk.%d.ffn_norm.weight", L);
            s = ld.read_f32(nm, ly.ffn_norm, d);
            if (s != JINF_OK) break;
            if (src.prepacked()) {  // the file holds this layer's matrices as Q4M images
                const std::pair<const char*, std::pair<uint8_t*, uint64_t>> imgs[5] = {
                    {"qkv", {ly.qkv, ly.qkv_sh.bytes}}, {"v", {ly.v, ly.v ? ly.v_sh.bytes : 0}},
                    {"o", {ly.o, ly.o_sh.bytes}}, {"gu", {ly.gu, ly.gu_sh.bytes}}, {"down", {ly.down, ly.down_sh.bytes}}};
                for (const auto& im : imgs) {
                    if (!im.second.first || s != JINF_OK) continue;
                    snprintf(nm, sizeof nm, "blk.%d.%s.q4m", L, im.first);
                    s = src.read_packed(nm, im.second.first, im.second.second);
                }
                continue;
            }
            // QKV: this rank's q heads, then its k heads, then its v heads
            const int64_t nq = (int64_t)I->Hl * hd, nk = (int64_t)I->Hkvl * hd;
            const int64_t rb_qk = (int64_t)aos_row_bytes(ly.qkv_sh.fmt, d);
            snprintf(nm, sizeof nm, "blk.%d.attn_q.weight", L);
            s = ld.stage_shard(nm, nq, d, rb_qk, 0, 1);
            if (s == JINF_OK) {
                snprintf(nm, sizeof nm, "blk.%d.attn_k.weight", L);
                s = ld.stage_shard(nm, nk, d, rb_qk, nq, 1);
            }
            if (s == JINF_OK && !ly.v) {
                snprintf(nm, sizeof nm, "blk.%d.attn_v.weight", L);
                s = ld.stage_shard(nm, nk, d, rb_qk, nq + nk, 1);
            }
            if (s == JINF_OK) s = ld.pack(ly.qkv, ly.qkv_sh);
            if (s == JINF_OK && ly.v) {  // v of its own type: a matrix of its own
                snprintf(nm, sizeof nm, "blk.%d.attn_v.weight", L);
                s = ld.stage_shard(nm, nk, d, (int64_t)aos_row_bytes(ly.v_sh.fmt, d), 0, 1);
                if (s == JINF_OK) s = ld.pack(ly.v, ly.v_sh);
            }
            // o: every output row, this rank's input columns (row split)
            if (s == JINF_OK) {
                snprintf(nm, sizeof nm, "blk.%d.attn_output.weight", L);
                s = ld.stage_shard(nm, d, nq, (int64_t)aos_row_bytes(ly.o_sh.fmt, nq), 0, 1);
            }
            if (s == JINF_OK) s = ld.pack(ly.o, ly.o_sh);
            // gate|up interleaved by neuron: gate_n -> row 2n, up_n -> row 2n+1
            const int64_t rb_gu = (int64_t)aos_row_bytes(ly.gu_sh.fmt, d);
            if (s == JINF_OK) {
                snprintf(nm, sizeof nm, "blk.%d.ffn_gate.weight", L);
                s = ld.stage_shard(nm, I->ffl, d, rb_gu, 0, 2);
            }
            if (s == JINF_OK) {
                snprintf(nm, sizeof nm, "blk.%d.ffn_up.weight", L);
                s = ld.stage_shard(nm, I->ffl, d, rb_gu, 1, 2);
            }
            uint8_t* bl = I->bundles ? I->bundles + (size_t)L * I->ffl * I->bundle_size : nullptr;
            if (s == JINF_OK && bl && sparse_bundle_gate_up(ld.dstage, I->ffl, (int)rb_d, bl, I->bundle_size,
                                                            I->stream) != cudaSuccess)
                s = JINF_ERR_CUDA;
            if (s == JINF_OK && I->sparse_persistent) {
                // the gate and up rows of every neuron of the kept blocks; inactive ones zeroed
                std::vector<int> idx;
                for (const int b : I->sparse_blocks[L])
                    for (int k = 0; k < 32; ++k) {
                        const int n = 32 * b + k;
                        idx.push_back(I->sparse_active[L][n] ? 2 * n : -1);
                        idx.push_back(I->sparse_active[L][n] ? 2 * n + 1 : -1);
                    }
                s = ld.gather_rows(idx, (int)rb_d);
            }
            if (s == JINF_OK) s = ld.pack(ly.gu, ly.gu_sh);
            // down: every output row, this rank's neuron columns (row split)
            if (s == JINF_OK) {
                snprintf(nm, sizeof nm, "blk.%d.ffn_down.weight", L);
                s = ld.stage_shard(nm, d, I->ffl, (int64_t)aos_row_bytes(ly.down_sh.fmt, I->ffl), 0, 1);
            }
            if (s == JINF_OK && bl && sparse_bundle_down(ld.dstage, d, I->ffl, I->wtype, bl, I->bundle_size,
                                                         (int)(2 * rb_d), I->stream) != cudaSuccess)
                s = JINF_ERR_CUDA;
            if (s == JINF_OK && I->sparse_persistent)  // the kept blocks' columns (whole Q4_0 blocks)
                s = ld.gather_blocks(I->sparse_blocks[L], d, I->ffl / 32, 18);
            if (s == JINF_OK) s = ld.pack(ly.down, ly.down_sh);
        }
        I->out_norm = I->norms + (size_t)(2 * I->L) * d;
        if (s == JINF_OK) s = ld.read_f32("output_norm.weight", I->out_norm, d);
        if (s == JINF_OK && src.prepacked()) {
            s = src.read_packed("output.q4m", I->lm, I->lm_sh.bytes);
        } else {
            if (s == JINF_OK)
                s = ld.stage_shard("output.weight", I->Vl, d, (int64_t)aos_row_bytes(I->lm_sh.fmt, d), 0, 1);
            if (s == JINF_OK) s = ld.pack(I->lm, I->lm_sh);
        }
        if (s == JINF_OK) s = ld.read_f32("token_embd.weight", I->embed, (int64_t)I->V * d);
        if (s != JINF_OK) return fail(s);
    }
    if (cudaDeviceSynchronize() != cudaSuccess) return fail(JINF_ERR_CUDA);

    // ---- communicator
    if (tp > 1) {
        const NcclApi* n = nccl_api();
        if (!n || !opt.nccl_id) {
            JINF_LOG("tensor parallelism needs NCCL and a unique id");
            return fail(n ? JINF_ERR_INVALID : JINF_ERR_CUDA);
        }
        ncclUniqueId id;
        memcpy(&id, opt.nccl_id, sizeof id);
        const ncclResult_t r = n->CommInitRank(&I->comm, tp, id, opt.tp_rank);
        if (r != ncclSuccess) {
            JINF_LOG("ncclCommInitRank failed: %s", n->GetErrorString(r));
            I->comm = nullptr;
            return fail(JINF_ERR_CUDA);
        }
    }

    // ---- split-K workspace of the stand-alone GEMVs (counters zero, self-resetting)
    {
        size_t pairs = I->lm_sh.pairs;
        for (const auto& ly : I->layers)
            for (const Q4MShape* sh : {&ly.qkv_sh, &ly.v_sh, &ly.o_sh, &ly.gu_sh, &ly.down_sh})
                pairs = std::max(pairs, (size_t)sh->pairs);
        if (cudaMalloc(&I->gemv_part, sizeof(float) * pairs * kEngineMaxKw * Q4M_PAIR_ROWS) != cudaSuccess ||
            cudaMalloc(&I->gemv_cnt, sizeof(unsigned int) * pairs) != cudaSuccess)
            return fail(JINF_ERR_OOM);
        cudaMemset(I->gemv_cnt, 0, sizeof(unsigned int) * pairs);
    }
    // ---- multi-sequence step buffers (the GEMV workspace sized for the K splits every vector
    // count picks; arrival counters zero, self-resetting)
    if (!I->sparse_mode) {
        const int S = I->n_seqs, nq = I->Hl * hd;
        const int grid = multi_grid(I->num_sms);
        size_t ws = 0, pairs = 0;
        for (int n = 1; n <= S; ++n) {
            auto need = [&](const Q4MShape& sh, int epi) {  // the plans the step's op can make
                if (!sh.rows) return;
                for (int xm : {MX_PLAIN_F32, MX_RECORDS}) {
                    int kw = 0, local = 0;
                    multi_plan(sh.pairs, sh.groups, n, sh.fmt, grid, epi, xm, &kw, &local);
                    ws = std::max(ws, (size_t)sh.pairs * std::max(kw, 1) * n * 32);
                }
                pairs = std::max(pairs, (size_t)sh.pairs);
            };
            need(I->lm_sh, ME_LMHEAD);
            for (const auto& ly : I->layers)
                for (const Q4MShape* sh : {&ly.qkv_sh, &ly.v_sh, &ly.o_sh, &ly.gu_sh, &ly.down_sh}) need(*sh, ME_STORE);
        }
        // attention splits: one per 64 positions at run time, up to this many
        I->m_split = I->n_split;
        const size_t attn_part = multi_attn_part_floats(S, I->Hkvl, I->m_split, hd);
        I->m_part_floats = std::max(ws, (size_t)1);
        I->m_cnt_n = std::max(pairs, (size_t)1);
        bool mok = cudaMalloc(&I->ms, sizeof(MultiState)) == cudaSuccess &&
                   cudaHostAlloc(&I->ms_pinned, sizeof(int32_t) * 4 * MULTI_MAX, cudaHostAllocDefault) == cudaSuccess &&
                   cudaMalloc(&I->m_h, sizeof(float) * (size_t)S * d) == cudaSuccess &&
                   cudaMalloc(&I->m_y, sizeof(float) * (size_t)S * d) == cudaSuccess &&
                   cudaMalloc(&I->m_q, sizeof(float) * (size_t)S * nq) == cudaSuccess &&
                   cudaMalloc(&I->m_attn, sizeof(float) * (size_t)S * nq) == cudaSuccess &&
                   cudaMalloc(&I->m_act, sizeof(float) * (size_t)S * I->ffl) == cudaSuccess &&
                   cudaMalloc(&I->m_logits, sizeof(float) * (size_t)S * I->Vl) == cudaSuccess &&
                   cudaMalloc(&I->m_ssq, sizeof(float) * (size_t)S * (d / 32)) == cudaSuccess &&
                   cudaMalloc(&I->m_attn_part, sizeof(float) * attn_part) == cudaSuccess &&
                   cudaMalloc(&I->m_part, sizeof(float) * std::max(ws, (size_t)1)) == cudaSuccess &&
                   cudaMalloc(&I->m_cnt, sizeof(unsigned int) * std::max(pairs, (size_t)1)) == cudaSuccess &&
                   cudaMalloc(&I->m_out, sizeof(int32_t) * (size_t)I->max_ctx * MULTI_MAX) == cudaSuccess;
        if (mok && d % Q4M_KG == 0 && nq % Q4M_KG == 0)
            mok = cudaMalloc(&I->m_rec_h, (size_t)S * xrec_bytes(d / Q4M_KG)) == cudaSuccess &&
                  cudaMalloc(&I->m_rec_a, (size_t)S * xrec_bytes(nq / Q4M_KG)) == cudaSuccess;
        if (!mok) return fail(JINF_ERR_OOM);
        cudaMemset(I->ms, 0, sizeof(MultiState));
        cudaMemset(I->m_cnt, 0, sizeof(unsigned int) * std::max(pairs, (size_t)1));
    }
    // mixed models in the persistent step: a v of its own type must follow its [q | k] rows
    // directly (one phase streams both) and start on a tile pair
    bool step_ok = I->uniform || I->step_formats;
    for (const auto& ly : I->layers)
        if (ly.v && (ly.v != ly.qkv + ly.qkv_sh.bytes || ly.qkv_sh.rows % Q4M_PAIR_ROWS)) step_ok = false;
    if (opt.persistent && !step_ok)
        JINF_LOG("weight types not streamed by the persistent step (Q8_0 in a mixed model): one kernel per operation");
    if (opt.persistent && step_ok && (!I->sparse_mode || I->sparse_persistent)) {
        // tensor parallel: the exchange areas first (every rank decides the same way)
        bool ok = tp == 1 || setup_exchange(I);
        if (!ok) {
            JINF_LOG("tensor-parallel persistent step unavailable; using one kernel per operation");
            free_exchange(I);
        } else {
            const jinf_status s = setup_persistent(I);
            if (s != JINF_OK) return fail(s);
        }
    }

    // ---- step programs
    build_ops(I, true, I->ops_full);
    build_ops(I, false, I->ops_body);
    if (I->use_graph) {
        jinf_status s = capture(I, I->ops_full, &I->exec_full);
        if (s == JINF_OK) s = capture(I, I->ops_body, &I->exec_body);
        if (s != JINF_OK) return fail(s);
    }

    jinf_engine* e = (jinf_engine*)calloc(1, sizeof(jinf_engine));
    if (!e) return fail(JINF_ERR_OOM);
    e->n_layers = I->L;
    e->n_embd = I->d;
    e->n_heads = I->H;
    e->n_heads_kv = I->Hkv;
    e->n_ff = I->ff;
    e->n_vocab = I->V;
    e->max_context = I->max_ctx;
    e->head_dim = hd;
    e->rms_norm_eps = I->eps;
    e->rope_freq_base = I->rope_base;
    e->primary_type = src.primary_type;
    e->logits_buf = I->logits_full;
    e->compute_stream = I->stream;
    e->impl = I;
    *out = e;
    JINF_LOG("engine ready: %d layers, d=%d, heads %d/%d, ff=%d, vocab=%d, tp %d/%d, weights %.1f MB/rank, %s",
             I->L, I->d, I->H, I->Hkv, I->ff, I->V, I->tp_rank, tp, I->arena_bytes / 1048576.0,
             I->persistent ? "persistent step kernel" : "one kernel per operation");
    return JINF_OK;
}

// One decode step for the token already in st->token (device).
jinf_status step(jinf_engine* e, bool with_head) {
    jinf_engine_impl* I = e->impl;
    if (e->n_past >= I->max_ctx) {
        JINF_LOG("context full (%d positions)", I->max_ctx);
        return JINF_ERR_INVALID;
    }
    if (e->ffn_hook || I->count_dev) {
        // Layer-by-layer path that exposes the raw gate pre-activation of each layer.
        const std::vector<Op>& ops = with_head ? I->ops_full : I->ops_body;
        for (const Op& op : ops) {
            Op o2 = op;
            JINF_CHECK(run_op(I, o2, I->stream), "op");
            if (op.kind == OP_GEMV && op.role == ROLE_GATEUP) {
                // The fused kernel never materialises the raw gate. Re-run the same matrix
                // as a plain GEMV: its prologue input is hB (= h after the o residual, which
                // the fused kernel just stored), gate rows are the even interleaved rows.
                if (!I->gate_raw) JINF_CUDA_CHECK(cudaMalloc(&I->gate_raw, sizeof(float) * 3 * (size_t)I->ffl));
                GemvParams gp = op.gp;
                gp.hin = I->hB;
                gp.yres = nullptr;
                gp.hout = nullptr;
                gp.y = I->gate_raw + I->ffl;  // [2*ffl] interleaved gate/up
                gp.pf_bytes = 0;
                JINF_CUDA_CHECK(gemvm_launch(gp, X_RMSNORM, EPI_STORE, op.grid, I->stream, false));
                k_even_rows<<<(I->ffl + 255) / 256, 256, 0, I->stream>>>(I->gate_raw + I->ffl, I->gate_raw, I->ffl);
                JINF_CUDA_CHECK(cudaGetLastError());
                if (I->count_dev) {
                    k_count_active<<<(I->ffl + 255) / 256, 256, 0, I->stream>>>(
                        I->gate_raw, I->ffl, I->count_thr, I->count_dev + (size_t)op.layer * I->ffl);
                    JINF_CUDA_CHECK(cudaGetLastError());
                } else {
                    JINF_CUDA_CHECK(cudaStreamSynchronize(I->stream));
                    e->ffn_hook(e->ffn_hook_data, op.layer, I->gate_raw, I->ffl);
                }
            }
        }
    } else if (I->persistent) {
        JINF_CUDA_CHECK(step_launch(with_head ? I->sp_full : I->sp_body, I->step_grid, I->stream));
    } else if (I->use_graph) {
        JINF_CUDA_CHECK(cudaGraphLaunch(with_head ? I->exec_full : I->exec_body, I->stream));
    } else {
        JINF_CHECK(run_ops(I, with_head ? I->ops_full : I->ops_body, I->stream), "step");
    }
    e->n_past += 1;
    return JINF_OK;
}

// ---------------------------------------------------------------- batched prefill
//
// The reference runs every prompt token through the whole model one at a time
// (src/engine.cpp:690-751). Here the tokens [0, T) of a forward() (all but its last, whose
// logits the caller reads) go through each layer together: the projections are tensor-core
// contractions over all T tokens (prefill_gemm.cu), RMSNorm, RoPE, the KV store, a causal
// attention and SiLU * up run once per layer over all rows (prefill.cu). Chunks of up to 512
// tokens; each chunk's attention also sees the positions before it.
constexpr int PF_CHUNK = 512;
constexpr int PF_MIN_TOKENS = 8;  // shorter prompts run token by token

bool prefill_usable(const jinf_engine* e, int T) {
    const jinf_engine_impl* I = e->impl;
    return I->prefill && T >= PF_MIN_TOKENS && I->persistent && I->tp_size == 1 && I->uniform &&
           I->wfmt == Q4M_Q4_0 && !I->sparse_mode && !e->ffn_hook && !I->count_dev && (I->hd == 64 || I->hd == 128) &&
           I->d % 64 == 0 && I->ffl % 64 == 0;
}

jinf_status prefill_alloc(jinf_engine_impl* I) {
    if (I->pf_cap) return JINF_OK;
    const size_t C = PF_CHUNK, nq = (size_t)I->Hl * I->hd, nk = (size_t)I->Hkvl * I->hd;
    const size_t ny = std::max(nq + 2 * nk, 2 * (size_t)I->ffl), nx = std::max(std::max((size_t)I->d, (size_t)I->ffl), nq);
    JINF_CUDA_CHECK(cudaMalloc(&I->pf_h, sizeof(float) * C * I->d));
    JINF_CUDA_CHECK(cudaMalloc(&I->pf_y, sizeof(float) * C * ny));
    JINF_CUDA_CHECK(cudaMalloc(&I->pf_att, sizeof(float) * C * nq));
    JINF_CUDA_CHECK(cudaMalloc(&I->pf_sc, sizeof(float) * C));
    JINF_CUDA_CHECK(cudaMalloc(&I->pf_x16, sizeof(__half) * C * nx));
    JINF_CUDA_CHECK(cudaMalloc(&I->pf_q16, sizeof(__half) * C * nq));
    JINF_CUDA_CHECK(cudaMalloc(&I->pf_err, sizeof(int)));
    JINF_CUDA_CHECK(cudaMemset(I->pf_err, 0, sizeof(int)));
    I->pf_cap = PF_CHUNK;
    return JINF_OK;
}

// Tokens dev_tokens[0, T) at positions n_past .. n_past + T - 1; afterwards n_past += T and
// the device position follows (the last token of the forward() then runs as a decode step).
jinf_status prefill_tokens(jinf_engine* e, int T) {
    jinf_engine_impl* I = e->impl;
    JINF_CHECK(prefill_alloc(I), "prefill buffers");
    cudaStream_t s = I->stream;
    const int d = I->d, nq = I->Hl * I->hd, nk = I->Hkvl * I->hd, ff = I->ffl, nqkv = nq + 2 * nk;
    for (int c0 = 0; c0 < T; c0 += PF_CHUNK) {
        const int Tc = std::min(PF_CHUNK, T - c0), p0 = e->n_past + c0;
        JINF_CUDA_CHECK(prefill_embed(I->embed, I->dev_tokens + c0, Tc, d, I->pf_h, s));
        for (int L = 0; L < I->L; ++L) {
            const auto& ly = I->layers[L];
            __half* kc = I->kc + (size_t)L * I->Hkvl * I->max_ctx * I->hd;
            __half* vc = I->vc + (size_t)L * I->Hkvl * I->max_ctx * I->hd;
            JINF_CUDA_CHECK(prefill_rows_to_f16(I->pf_h, d, Tc, d, ly.attn_norm, I->eps, I->pf_x16, d, I->pf_sc, s));
            JINF_CUDA_CHECK(prefill_gemm_launch(ly.qkv, nqkv, d, I->pf_x16, Tc, I->pf_sc, I->pf_y, nqkv, 0, I->pf_err, s));
            JINF_CUDA_CHECK(prefill_rope_qkv(I->pf_y, nqkv, Tc, p0, nq, nk, I->hd, I->rope_base, I->pf_q16, kc, vc,
                                             I->max_ctx, s));
            JINF_CUDA_CHECK(prefill_attention(I->pf_q16, I->Hl, I->Hkvl, I->hd, Tc, p0, kc, vc, I->max_ctx, I->pf_att, s));
            JINF_CUDA_CHECK(prefill_rows_to_f16(I->pf_att, nq, Tc, nq, nullptr, 0.f, I->pf_x16, nq, I->pf_sc, s));
            JINF_CUDA_CHECK(prefill_gemm_launch(ly.o, d, nq, I->pf_x16, Tc, I->pf_sc, I->pf_h, d, 1, I->pf_err, s));
            JINF_CUDA_CHECK(prefill_rows_to_f16(I->pf_h, d, Tc, d, ly.ffn_norm, I->eps, I->pf_x16, d, I->pf_sc, s));
            JINF_CUDA_CHECK(
                prefill_gemm_launch(ly.gu, 2 * ff, d, I->pf_x16, Tc, I->pf_sc, I->pf_y, 2 * ff, 0, I->pf_err, s));
            JINF_CUDA_CHECK(prefill_silu_to_f16(I->pf_y, 2 * ff, Tc, ff, I->pf_x16, ff, I->pf_sc, s));
            JINF_CUDA_CHECK(prefill_gemm_launch(ly.down, d, ff, I->pf_x16, Tc, I->pf_sc, I->pf_h, d, 1, I->pf_err, s));
        }
    }
    e->n_past += T;
    I->pinned[3] = e->n_past;
    JINF_CUDA_CHECK(cudaMemcpyAsync(&I->st->pos, &I->pinned[3], sizeof(int32_t), cudaMemcpyHostToDevice, s));
    // a pipeline wait of the tensor-core GEMM that ran out is reported like a step timeout
    JINF_CUDA_CHECK(cudaMemcpyAsync(&I->pinned[2], I->pf_err, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
    JINF_CUDA_CHECK(cudaStreamSynchronize(s));
    if (I->pinned[2] != 0) {
        JINF_LOG("prefill: a tensor-core pipeline wait ran out");
        cudaMemsetAsync(I->pf_err, 0, sizeof(int), s);
        I->pinned[2] = DEV_ERR_TIMEOUT;
        return JINF_ERR_TIMEOUT;
    }
    return JINF_OK;
}

// Device-side error recorded by a step (pinned[2], copied after the step): a dependency
// wait of the persistent kernel that gave up.
jinf_status device_error(jinf_engine_impl* I) {
    if (I->pinned[2] == DEV_OK) return JINF_OK;
    JINF_LOG("device error %d: a phase of the persistent step timed out waiting for its inputs", I->pinned[2]);
    return JINF_ERR_TIMEOUT;
}

jinf_status gather_logits(jinf_engine* e) {
    jinf_engine_impl* I = e->impl;
    if (I->tp_size == 1) return JINF_OK;
    const NcclApi* n = nccl_api();
    if (!n) return JINF_ERR_CUDA;
    if (n->AllGather(I->logits, I->logits_full, (size_t)I->Vl, ncclFloat32, I->comm, I->stream) != ncclSuccess)
        return JINF_ERR_CUDA;
    return JINF_OK;
}

}  // namespace

// ================================================================== public API

extern "C" jinf_status jinf_engine_create_ex(jinf_engine** e, const jinf_engine_config* config,
                                             const jinf_b200_options* options) {
    if (!e || !config || !config->model_path) return JINF_ERR_INVALID;
    std::unique_ptr<ModelSource> src;
    JINF_CHECK(open_nvmw_source(config->model_path, &src), "model");
    return create_from_source(e, config, *src, options);
}

extern "C" jinf_status jinf_engine_create(jinf_engine** e, const jinf_engine_config* config) {
    return jinf_engine_create_ex(e, config, nullptr);
}

extern "C" jinf_status jinf_engine_create_synthetic(jinf_engine** e, const jinf_engine_config* config,
                                                    const jinf_synth_model* model, const jinf_b200_options* options) {
    if (!e || !config || !model) return JINF_ERR_INVALID;
    SynthSource src(model);
    return create_from_source(e, config, src, options);
}

extern "C" void jinf_engine_destroy(jinf_engine* e) {
    if (!e) return;
    free_impl(e->impl);
    free(e);
}

extern "C" void jinf_engine_reset(jinf_engine* e) {
    if (!e || !e->impl) return;
    jinf_engine_impl* I = e->impl;
    cudaSetDevice(I->device);
    cudaStreamSynchronize(I->stream);
    const size_t kv_elems = (size_t)I->L * I->Hkvl * I->max_ctx * I->hd;
    cudaMemsetAsync(I->kc, 0, sizeof(__half) * kv_elems, I->stream);
    cudaMemsetAsync(I->vc, 0, sizeof(__half) * kv_elems, I->stream);
    cudaMemsetAsync(I->st, 0, sizeof(DeviceState), I->stream);
    cudaStreamSynchronize(I->stream);
    e->n_past = 0;
    std::fill(I->seq_past.begin(), I->seq_past.end(), 0);
    I->logits_valid = false;
    memset(&e->perf, 0, sizeof e->perf);
}

extern "C" const jinf_perf_stats* jinf_engine_get_stats(const jinf_engine* e) { return e ? &e->perf : nullptr; }

extern "C" jinf_status jinf_engine_forward(jinf_engine* e, const int32_t* tokens, int n_tokens, float** logits) {
    if (!e || !tokens || n_tokens <= 0 || !logits || !e->impl) return JINF_ERR_INVALID;
    jinf_engine_impl* I = e->impl;
    for (int t = 0; t < n_tokens; ++t)
        if (tokens[t] < 0 || tokens[t] >= I->V) return JINF_ERR_INVALID;
    if (e->n_past + n_tokens > I->max_ctx) return JINF_ERR_INVALID;
    JINF_CUDA_CHECK(cudaSetDevice(I->device));
    jinf_timer timer;
    JINF_CUDA_CHECK(cudaEventRecord(I->ev0, I->stream));
    if (n_tokens == 1) {
        I->pinned[0] = tokens[0];
        JINF_CUDA_CHECK(cudaMemcpyAsync(&I->st->token, &I->pinned[0], sizeof(int32_t), cudaMemcpyHostToDevice,
                                        I->stream));
    } else {
        JINF_CUDA_CHECK(cudaMemcpyAsync(I->dev_tokens, tokens, sizeof(int32_t) * (size_t)n_tokens,
                                        cudaMemcpyHostToDevice, I->stream));
    }
    int t_first = 0;
    if (n_tokens > 1 && prefill_usable(e, n_tokens - 1)) {
        JINF_CHECK(prefill_tokens(e, n_tokens - 1), "prefill");
        t_first = n_tokens - 1;
    }
    for (int t = t_first; t < n_tokens; ++t) {
        if (n_tokens > 1)
            JINF_CUDA_CHECK(cudaMemcpyAsync(&I->st->token, I->dev_tokens + t, sizeof(int32_t),
                                            cudaMemcpyDeviceToDevice, I->stream));
        // Only the last token's logits are observable: earlier tokens skip the LM head.
        JINF_CHECK(step(e, t == n_tokens - 1), "decode step");
    }
    JINF_CHECK(gather_logits(e), "logits gather");
    JINF_CUDA_CHECK(cudaMemcpyAsync(&I->pinned[2], &I->st->error, sizeof(int32_t), cudaMemcpyDeviceToHost, I->stream));
    JINF_CUDA_CHECK(cudaEventRecord(I->ev1, I->stream));
    JINF_CUDA_CHECK(cudaStreamSynchronize(I->stream));
    JINF_CHECK(device_error(I), "decode step");
    float ms = 0.f;
    cudaEventElapsedTime(&ms, I->ev0, I->ev1);
    *logits = I->logits_full;
    I->logits_valid = true;
    e->perf.total_ms += timer.elapsed_ms();
    e->perf.gpu_compute_ms += ms;
    e->perf.tokens_generated += n_tokens;
    return JINF_OK;
}

extern "C" jinf_status jinf_engine_last_argmax(jinf_engine* e, int32_t* token) {
    if (!e || !token || !e->impl || !e->impl->logits_valid) return JINF_ERR_INVALID;
    jinf_engine_impl* I = e->impl;
    JINF_CUDA_CHECK(cudaSetDevice(I->device));
    // argmax_token and error are adjacent in the device state: one 8-byte read
    JINF_CUDA_CHECK(cudaMemcpyAsync(&I->pinned[1], &I->st->argmax_token, 2 * sizeof(int32_t), cudaMemcpyDeviceToHost,
                                    I->stream));
    JINF_CUDA_CHECK(cudaStreamSynchronize(I->stream));
    JINF_CHECK(device_error(I), "decode step");
    *token = I->pinned[1];
    return JINF_OK;
}

extern "C" jinf_status jinf_engine_generate(jinf_engine* e, const int32_t* prompt, int n_prompt, int32_t* output,
                                            int max_tokens, int* n_generated) {
    if (!e || !output || !n_generated || !e->impl) return JINF_ERR_INVALID;
    jinf_engine_impl* I = e->impl;
    float* logits = nullptr;
    if (n_prompt > 0) {
        if (!prompt) return JINF_ERR_INVALID;
        JINF_CHECK(jinf_engine_forward(e, prompt, n_prompt, &logits), "prompt");
    } else if (e->n_past == 0 || !I->logits_valid) {
        return JINF_ERR_INVALID;
    }
    // Same loop as the reference (reference src/engine.cpp:779-800): emit the argmax of
    // the current logits, stop after EOS, otherwise feed the token back through forward().
    // Per token 4 bytes cross each way (the reference copied all n_vocab logits D2H).
    int gen = 0;
    for (int i = 0; i < max_tokens; ++i) {
        int32_t best;
        JINF_CHECK(jinf_engine_last_argmax(e, &best), "argmax");
        output[gen++] = best;
        if (I->eos >= 0 && best == I->eos) break;
        if (jinf_engine_forward(e, &best, 1, &logits) != JINF_OK) break;
    }
    *n_generated = gen;
    return JINF_OK;
}

extern "C" jinf_status jinf_engine_decode_resident(jinf_engine* e, int n_steps, int32_t* out_tokens) {
    if (!e || !e->impl || n_steps < 0) return JINF_ERR_INVALID;
    jinf_engine_impl* I = e->impl;
    if (!I->logits_valid || e->n_past + n_steps > I->max_ctx) return JINF_ERR_INVALID;
    JINF_CUDA_CHECK(cudaSetDevice(I->device));
    // st->token already holds the argmax of the last step (finalize feeds it back)
    for (int i = 0; i < n_steps; ++i) {
        JINF_CHECK(step(e, true), "decode step");
        if (out_tokens)
            JINF_CUDA_CHECK(cudaMemcpyAsync(&out_tokens[i], &I->st->argmax_token, sizeof(int32_t),
                                            cudaMemcpyDeviceToHost, I->stream));
    }
    JINF_CUDA_CHECK(cudaMemcpyAsync(&I->pinned[2], &I->st->error, sizeof(int32_t), cudaMemcpyDeviceToHost, I->stream));
    JINF_CUDA_CHECK(cudaStreamSynchronize(I->stream));
    JINF_CHECK(device_error(I), "decode step");
    return JINF_OK;
}

extern "C" jinf_status jinf_engine_seq_fill_kv_random(jinf_engine* e, int seq, int n_pos, uint64_t seed) {
    if (!e || !e->impl || n_pos < 0 || n_pos > e->impl->max_ctx || seq < 0 || seq >= e->impl->n_seqs)
        return JINF_ERR_INVALID;
    jinf_engine_impl* I = e->impl;
    JINF_CUDA_CHECK(cudaSetDevice(I->device));
    const size_t so = (size_t)seq * I->seq_stride;
    if (n_pos > 0) {
        k_fill_kv_random<<<4 * I->num_sms, 256, 0, I->stream>>>(I->kc + so, I->vc + so, I->L, I->Hkvl, I->max_ctx, I->hd,
                                                               n_pos, (unsigned long long)seed);
        JINF_CUDA_CHECK(cudaGetLastError());
    }
    if (seq == 0) {  // set the device position; the token stays whatever was last fed
        JINF_CUDA_CHECK(cudaMemcpyAsync(&I->st->pos, &n_pos, sizeof(int), cudaMemcpyHostToDevice, I->stream));
        e->n_past = n_pos;
    } else {
        I->seq_past[seq] = n_pos;
    }
    JINF_CUDA_CHECK(cudaStreamSynchronize(I->stream));
    return JINF_OK;
}

extern "C" jinf_status jinf_engine_fill_kv_random(jinf_engine* e, int n_pos, uint64_t seed) {
    return jinf_engine_seq_fill_kv_random(e, 0, n_pos, seed);
}

extern "C" jinf_status jinf_engine_seq_kv_read(jinf_engine* e, int seq, int n_pos, uint16_t* k_host, uint16_t* v_host) {
    if (!e || !e->impl || !k_host || !v_host || n_pos <= 0 || n_pos > e->impl->max_ctx || seq < 0 ||
        seq >= e->impl->n_seqs)
        return JINF_ERR_INVALID;
    jinf_engine_impl* I = e->impl;
    JINF_CUDA_CHECK(cudaSetDevice(I->device));
    // the cache is [layer][kv head][max_ctx][hd]: one strided copy per cache, rows of n_pos * hd
    const size_t so = (size_t)seq * I->seq_stride;
    const size_t w = (size_t)n_pos * I->hd * sizeof(__half), pitch = (size_t)I->max_ctx * I->hd * sizeof(__half);
    const size_t h = (size_t)I->L * I->Hkvl;
    JINF_CUDA_CHECK(cudaMemcpy2DAsync(k_host, w, I->kc + so, pitch, w, h, cudaMemcpyDeviceToHost, I->stream));
    JINF_CUDA_CHECK(cudaMemcpy2DAsync(v_host, w, I->vc + so, pitch, w, h, cudaMemcpyDeviceToHost, I->stream));
    JINF_CUDA_CHECK(cudaStreamSynchronize(I->stream));
    return JINF_OK;
}

extern "C" jinf_status jinf_engine_kv_read(jinf_engine* e, int n_pos, uint16_t* k_host, uint16_t* v_host) {
    return jinf_engine_seq_kv_read(e, 0, n_pos, k_host, v_host);
}

extern "C" int jinf_engine_seq_n_past(const jinf_engine* e, int seq) {
    if (!e || !e->impl || seq < 0 || seq >= e->impl->n_seqs) return -1;
    return seq == 0 ? e->n_past : e->impl->seq_past[seq];
}

extern "C" jinf_status jinf_engine_seq_reset(jinf_engine* e, int seq) {
    if (!e || !e->impl || seq < 0 || seq >= e->impl->n_seqs) return JINF_ERR_INVALID;
    if (seq == 0) {
        jinf_engine_reset(e);
        return JINF_OK;
    }
    e->impl->seq_past[seq] = 0;
    return JINF_OK;
}

namespace {

// Validate a multi-sequence call and stage its inputs (tokens, positions, sequences) in the
// pinned buffer; n_steps positions must fit in every sequence's cache.
jinf_status multi_inputs(jinf_engine* e, int n, const int32_t* seqs, const int32_t* tokens, int n_steps, bool* has0) {
    jinf_engine_impl* I = e->impl;
    if (!I->ms || n < 1 || n > I->n_seqs || n_steps < 1) return JINF_ERR_INVALID;
    int32_t* in = I->ms_pinned;
    *has0 = false;
    for (int i = 0; i < n; ++i) {
        const int sq = seqs[i];
        if (sq < 0 || sq >= I->n_seqs || tokens[i] < 0 || tokens[i] >= I->V) return JINF_ERR_INVALID;
        for (int j = 0; j < i; ++j)
            if (seqs[j] == sq) return JINF_ERR_INVALID;
        const int pos = sq == 0 ? e->n_past : I->seq_past[sq];
        if (pos + n_steps > I->max_ctx) {
            JINF_LOG("context full (%d positions) for sequence %d", I->max_ctx, sq);
            return JINF_ERR_INVALID;
        }
        in[i] = tokens[i];
        in[MULTI_MAX + i] = pos;
        in[2 * MULTI_MAX + i] = sq;
        *has0 |= sq == 0;
    }
    return JINF_OK;
}

// The graph of an n-vector step (captured at its first use) on the engine's stream.
jinf_status multi_launch(jinf_engine_impl* I, int n) {
    if (I->m_ops[n].empty()) build_multi_ops(I, n, I->m_ops[n]);
    if (I->use_graph) {
        if (!I->m_exec[n]) JINF_CHECK(capture(I, I->m_ops[n], &I->m_exec[n]), "multi-sequence step capture");
        JINF_CUDA_CHECK(cudaGraphLaunch(I->m_exec[n], I->stream));
    } else {
        JINF_CHECK(run_ops(I, I->m_ops[n], I->stream), "multi-sequence step");
    }
    return JINF_OK;
}

// After n_steps steps: positions advance; sequence 0's also on the one-sequence device state.
jinf_status multi_advance(jinf_engine* e, int n, const int32_t* seqs, int n_steps, bool has0) {
    jinf_engine_impl* I = e->impl;
    if (has0) {
        I->pinned[3] = e->n_past + n_steps;
        JINF_CUDA_CHECK(cudaMemcpyAsync(&I->st->pos, &I->pinned[3], sizeof(int32_t), cudaMemcpyHostToDevice, I->stream));
    }
    JINF_CUDA_CHECK(cudaEventRecord(I->ev1, I->stream));
    JINF_CUDA_CHECK(cudaStreamSynchronize(I->stream));
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, I->ev0, I->ev1) == cudaSuccess) e->perf.gpu_compute_ms += ms;
    for (int i = 0; i < n; ++i) {
        if (seqs[i] == 0) {
            e->n_past += n_steps;
            I->logits_valid = false;
        } else {
            I->seq_past[seqs[i]] += n_steps;
        }
    }
    e->perf.tokens_generated += n * n_steps;
    return JINF_OK;
}

}  // namespace

// One multi-sequence step: the inputs go to the device state in one copy, the step's graph for
// this vector count runs, and the argmax ids (and, if asked, the logits) come back. Sequence
// 0's new position is also written to the one-sequence state.
extern "C" jinf_status jinf_engine_decode_batch(jinf_engine* e, int n, const int32_t* seqs, const int32_t* tokens,
                                               int32_t* next_tokens, float* logits) {
    if (!e || !e->impl || !seqs || !tokens) return JINF_ERR_INVALID;
    jinf_engine_impl* I = e->impl;
    if (logits && I->tp_size > 1) return JINF_ERR_INVALID;
    bool has0 = false;
    JINF_CHECK(multi_inputs(e, n, seqs, tokens, 1, &has0), "decode_batch arguments");
    JINF_CUDA_CHECK(cudaSetDevice(I->device));
    int32_t* in = I->ms_pinned;
    JINF_CUDA_CHECK(cudaEventRecord(I->ev0, I->stream));
    JINF_CUDA_CHECK(cudaMemcpyAsync(I->ms, in, sizeof(int32_t) * 3 * MULTI_MAX, cudaMemcpyHostToDevice, I->stream));
    JINF_CHECK(multi_launch(I, n), "decode_batch");
    JINF_CUDA_CHECK(cudaMemcpyAsync(in + 3 * MULTI_MAX, I->ms->out_token, sizeof(int32_t) * n, cudaMemcpyDeviceToHost,
                                    I->stream));
    if (logits)  // one GPU: the vocabulary is whole, rows [n][n_vocab]
        JINF_CUDA_CHECK(cudaMemcpyAsync(logits, I->m_logits, sizeof(float) * (size_t)n * I->Vl, cudaMemcpyDeviceToHost,
                                        I->stream));
    JINF_CHECK(multi_advance(e, n, seqs, 1, has0), "decode_batch");
    if (next_tokens)
        for (int i = 0; i < n; ++i) next_tokens[i] = in[3 * MULTI_MAX + i];
    return JINF_OK;
}

// n_steps multi-sequence steps back to back with the argmax fed back on the device: the
// host copies the inputs once and, at the end, the ids of every step.
extern "C" jinf_status jinf_engine_decode_batch_resident(jinf_engine* e, int n, const int32_t* seqs,
                                                        const int32_t* tokens, int n_steps, int32_t* out_tokens) {
    if (!e || !e->impl || !seqs || !tokens) return JINF_ERR_INVALID;
    jinf_engine_impl* I = e->impl;
    bool has0 = false;
    JINF_CHECK(multi_inputs(e, n, seqs, tokens, n_steps, &has0), "decode_batch_resident arguments");
    JINF_CUDA_CHECK(cudaSetDevice(I->device));
    int32_t* in = I->ms_pinned;
    in[3 * MULTI_MAX] = 1;  // feedback on (the word after the three input arrays)
    JINF_CUDA_CHECK(cudaEventRecord(I->ev0, I->stream));
    JINF_CUDA_CHECK(cudaMemcpyAsync(I->ms, in, sizeof(int32_t) * (3 * MULTI_MAX + 1), cudaMemcpyHostToDevice, I->stream));
    for (int t = 0; t < n_steps; ++t) {
        JINF_CHECK(multi_launch(I, n), "decode_batch_resident");
        if (out_tokens)
            JINF_CUDA_CHECK(cudaMemcpyAsync(I->m_out + (size_t)t * MULTI_MAX, I->ms->out_token, sizeof(int32_t) * n,
                                            cudaMemcpyDeviceToDevice, I->stream));
    }
    in[3 * MULTI_MAX] = 0;
    JINF_CUDA_CHECK(cudaMemcpyAsync(&I->ms->feedback, in + 3 * MULTI_MAX, sizeof(int32_t), cudaMemcpyHostToDevice,
                                    I->stream));
    JINF_CHECK(multi_advance(e, n, seqs, n_steps, has0), "decode_batch_resident");
    if (out_tokens) {
        std::vector<int32_t> buf((size_t)n_steps * MULTI_MAX);
        JINF_CUDA_CHECK(cudaMemcpy(buf.data(), I->m_out, sizeof(int32_t) * buf.size(), cudaMemcpyDeviceToHost));
        for (int t = 0; t < n_steps; ++t)
            for (int i = 0; i < n; ++i) out_tokens[(size_t)t * n + i] = buf[(size_t)t * MULTI_MAX + i];
    }
    return JINF_OK;
}

extern "C" int jinf_engine_is_persistent(const jinf_engine* e) {
    return e && e->impl && e->impl->persistent ? 1 : 0;
}

extern "C" jinf_status jinf_engine_debug_step_timeout(jinf_engine* e, unsigned long long spin_limit) {
    if (!e || !e->impl || spin_limit == 0) return JINF_ERR_INVALID;
    jinf_engine_impl* I = e->impl;
    if (!I->persistent || I->tp_size != 1) return JINF_ERR_INVALID;
    cudaSetDevice(I->device);
    // a copy of the phase table whose attention phase waits for more finished QKV tile
    // pairs than exist: nothing ever sets what it waits for
    StepParams sp = I->sp_full;
    std::vector<StepPhase> ph((size_t)sp.n_phases);
    JINF_CUDA_CHECK(cudaMemcpy(ph.data(), sp.phases, sizeof(StepPhase) * ph.size(), cudaMemcpyDeviceToHost));
    for (auto& p : ph)
        if (p.kind == PH_ATTN) {
            p.dep_target = 0xFFFFFFFFu;
            break;
        }
    StepPhase* dph = nullptr;
    JINF_CUDA_CHECK(cudaMalloc(&dph, sizeof(StepPhase) * ph.size()));
    JINF_CUDA_CHECK(cudaMemcpy(dph, ph.data(), sizeof(StepPhase) * ph.size(), cudaMemcpyHostToDevice));
    sp.phases = dph;
    sp.spin_limit = spin_limit;
    const cudaError_t le = step_launch(sp, I->step_grid, I->stream);
    int32_t err = DEV_OK;
    const cudaError_t ce = cudaStreamSynchronize(I->stream);
    cudaMemcpy(&err, &I->st->error, sizeof err, cudaMemcpyDeviceToHost);
    cudaFree(dph);
    if (le != cudaSuccess || ce != cudaSuccess) return JINF_ERR_CUDA;
    // the step is discarded: clear the recorded error; the caller resets the engine
    cudaMemset(&I->st->error, 0, sizeof(int32_t));
    return err == DEV_ERR_TIMEOUT ? JINF_ERR_TIMEOUT : err == DEV_OK ? JINF_OK : JINF_ERR_CUDA;
}

extern "C" jinf_status jinf_engine_count_activations(jinf_engine* e, const int32_t* tokens, int n_tokens,
                                                    float threshold, int32_t* counts) {
    if (!e || !e->impl || !tokens || n_tokens <= 0 || !counts) return JINF_ERR_INVALID;
    jinf_engine_impl* I = e->impl;
    if (I->tp_size != 1 || I->sparse_mode) {
        JINF_LOG("activation counting needs the dense FFN on one GPU");
        return JINF_ERR_INVALID;
    }
    cudaSetDevice(I->device);
    const size_t n = (size_t)I->L * I->ffl;
    int32_t* dev = nullptr;
    JINF_CUDA_CHECK(cudaMalloc(&dev, sizeof(int32_t) * n));
    if (cudaMemset(dev, 0, sizeof(int32_t) * n) != cudaSuccess) {
        cudaFree(dev);
        return JINF_ERR_CUDA;
    }
    I->count_dev = dev;  // counting on for this forward only
    I->count_thr = threshold;
    float* logits = nullptr;
    const jinf_status s = jinf_engine_forward(e, tokens, n_tokens, &logits);
    std::vector<int32_t> add(n);
    const bool copied = cudaMemcpy(add.data(), I->count_dev, sizeof(int32_t) * n, cudaMemcpyDeviceToHost) == cudaSuccess;
    cudaFree(I->count_dev);
    I->count_dev = nullptr;
    if (s != JINF_OK) return s;
    if (!copied) return JINF_ERR_CUDA;
    for (size_t i = 0; i < n; ++i) counts[i] += add[i];
    return JINF_OK;
}

extern "C" jinf_status jinf_engine_sparse_ids(jinf_engine* e, int layer, int32_t* ids, int max, int* n) {
    if (!e || !e->impl || !n || !e->impl->sparse_mode || layer < 0 || layer >= e->impl->L) return JINF_ERR_INVALID;
    jinf_engine_impl* I = e->impl;
    if (I->device >= 0) cudaSetDevice(I->device);
    *n = I->sparse_n[layer];
    if (ids && max > 0) {
        JINF_CUDA_CHECK(cudaStreamSynchronize(I->stream));
        JINF_CUDA_CHECK(cudaMemcpy(ids, I->sparse_ids + (size_t)layer * I->ffl,
                                   sizeof(int32_t) * (size_t)std::min(max, *n), cudaMemcpyDeviceToHost));
    }
    return JINF_OK;
}

extern "C" uint64_t jinf_engine_weight_bytes_per_token(const jinf_engine* e) {
    return e && e->impl ? e->impl->weight_bytes_token : 0;
}

// The kernels of an n-vector multi-sequence step, each kind launched back to back over the
// layers (as jinf_engine_profile_kernels): QKV, attention, o, gate|up, down, LM head, the
// embedding / residual rows and the finaliser; the exchange steps of tensor parallelism are not
// timed. Leaves the multi-sequence state undefined (callers reset the sequences afterwards).
extern "C" jinf_status jinf_engine_profile_multi(jinf_engine* e, int n, int reps, double* times_us, double* bytes) {
    if (!e || !e->impl || reps <= 0 || !times_us || !bytes || n < 1 || n > e->impl->n_seqs || e->impl->sparse_mode)
        return JINF_ERR_INVALID;
    jinf_engine_impl* I = e->impl;
    JINF_CUDA_CHECK(cudaSetDevice(I->device));
    if (I->m_ops[n].empty()) build_multi_ops(I, n, I->m_ops[n]);
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    const int roles[6] = {ROLE_QKV, -1, ROLE_O, ROLE_GATEUP, ROLE_DOWN, ROLE_LM};
    for (int k = 0; k < 8; ++k) {
        std::vector<const Op*> sel;
        for (const Op& op : I->m_ops[n]) {
            const bool pick = k == 1   ? op.kind == OP_MATTN
                              : k == 6 ? (op.kind == OP_MEMBED || op.kind == OP_MRESID)
                              : k == 7 ? op.kind == OP_MFINAL
                                       : (op.kind == OP_MGEMV && op.role == roles[k]);
            if (pick) sel.push_back(&op);
        }
        times_us[k] = 0;
        bytes[k] = 0;
        if (sel.empty()) continue;
        // each GEMV streams its own weights only (no L2 prefetch of the next matrix, which the
        // next launch here would not use)
        auto launch = [&](int r) {
            Op op = *sel[r % sel.size()];
            if (op.kind == OP_MGEMV) op.mp.pf_bytes = 0;
            run_op(I, op, I->stream);
        };
        for (int r = 0; r < 3; ++r) launch(r);
        cudaEventRecord(a, I->stream);
        for (int r = 0; r < reps; ++r) launch(r);
        cudaEventRecord(b, I->stream);
        cudaEventSynchronize(b);
        float ms = 0.f;
        cudaEventElapsedTime(&ms, a, b);
        times_us[k] = 1000.0 * ms / reps;
        bytes[k] = (double)sel[0]->bytes;
    }
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    JINF_CUDA_CHECK(cudaMemsetAsync(I->ms->best, 0, sizeof(I->ms->best), I->stream));
    JINF_CUDA_CHECK(cudaStreamSynchronize(I->stream));
    JINF_CUDA_CHECK(cudaGetLastError());
    return JINF_OK;
}

extern "C" jinf_status jinf_engine_profile_kernels(jinf_engine* e, int reps, double* times_us, double* bytes) {
    if (!e || !e->impl || reps <= 0 || !times_us || !bytes) return JINF_ERR_INVALID;
    jinf_engine_impl* I = e->impl;
    JINF_CUDA_CHECK(cudaSetDevice(I->device));
    const int roles[7] = {ROLE_QKV, -1 /* attention */, ROLE_O, ROLE_GATEUP, ROLE_DOWN, ROLE_LM, -2 /* sparse FFN */};
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    for (int k = 0; k < 7; ++k) {
        std::vector<const Op*> sel;
        for (const Op& op : I->ops_full) {
            if (k == 1 ? op.kind == OP_ATTN
                       : k == 6 ? op.kind == OP_SPARSE_FFN : (op.kind == OP_GEMV && op.role == roles[k]))
                sel.push_back(&op);
        }
        times_us[k] = 0;
        bytes[k] = 0;
        if (sel.empty()) continue;
        // back-to-back launches rotating over the layers (launch overhead overlapped,
        // weights of consecutive launches distinct, so every launch streams from HBM)
        for (int r = 0; r < 3; ++r) {
            Op op = *sel[r % sel.size()];
            if (op.kind == OP_GEMV) op.gp.pf_bytes = 0;
            run_op(I, op, I->stream);
        }
        cudaEventRecord(a, I->stream);
        for (int r = 0; r < reps; ++r) {
            Op op = *sel[r % sel.size()];
            if (op.kind == OP_GEMV) op.gp.pf_bytes = 0;  // time the kernel's own stream only
            run_op(I, op, I->stream);
        }
        cudaEventRecord(b, I->stream);
        cudaEventSynchronize(b);
        float ms = 0.f;
        cudaEventElapsedTime(&ms, a, b);
        const double total = ms;
        times_us[k] = 1000.0 * total / reps;
        bytes[k] = (double)sel[0]->bytes;
        if (k == 1) {
            // K and V rows of positions 0..pos for this rank's kv heads
            int pos = 0;
            cudaMemcpy(&pos, &I->st->pos, sizeof(int), cudaMemcpyDeviceToHost);
            bytes[k] = 2.0 * (pos + 1) * I->Hkvl * I->hd * 2.0;
        }
    }
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    // The kernels above rewrote the residual stream and the argmax accumulator: the
    // sequence state is no longer meaningful (callers reset before decoding again).
    JINF_CUDA_CHECK(cudaMemsetAsync(&I->st->best, 0, sizeof(unsigned long long), I->stream));
    JINF_CUDA_CHECK(cudaStreamSynchronize(I->stream));
    I->logits_valid = false;
    return JINF_OK;
}
