// Seeded synthetic Llama models.
//
// Every value is a pure function of (seed, tensor name, element index): a splitmix64
// counter hash gives two uniforms, Box-Muller turns them into two normals (synth_math.h).
// Only basic IEEE operations are used, so the same bits come out on any x86-64 host, at
// any thread count, for any row range, and on the GPU (synth_gpu.cu): the engine, the CPU
// oracle and a tensor-parallel rank each generate exactly the slice they need.
//
// Tensor set and naming follow the GGUF Llama convention the reference engine binds
// by name (reference src/engine.cpp:150-158, :170-190).
#include "jinf/engine.h"
#include "jinf/quant.h"
#include "jinf/gguf.h"
#include "jinf/nvmw.h"
#include "synth_math.h"
#include "synth_internal.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <string>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

using jinf_synth::splitmix64;

uint64_t fnv1a64(const char* s) {
    uint64_t h = 0xcbf29ce484222325ull;
    for (; *s; ++s) { h ^= (uint8_t)*s; h *= 0x100000001b3ull; }
    return h;
}

// Fill out[0..n) with N(0,1)*stdv for element indices [i0, i0 + n) of stream `key`.
void gen_normals(uint64_t key, uint64_t i0, int64_t n, float stdv, float* out) {
    int64_t k = 0;
    uint64_t i = i0;
    while (k < n) {
        double z0, z1;
        jinf_synth::normal_pair(key, i >> 1, &z0, &z1);
        if ((i & 1) == 0) {
            out[k++] = (float)z0 * stdv;
            ++i;
            if (k < n) { out[k++] = (float)z1 * stdv; ++i; }
        } else {
            out[k++] = (float)z1 * stdv;
            ++i;
        }
    }
}

struct SynthTensor {
    std::string name;
    int type;
    int n_dims;
    int64_t shape[4];  // ggml order: shape[0] = columns (input features)
    int role;          // 0 = projection (normal, quantized), 1 = norm (ones), 2 = embedding (normal f32)
    int64_t rows() const { return n_dims > 1 ? shape[1] : 1; }
    int64_t cols() const { return shape[0]; }
    uint64_t row_bytes() const { return jinf_tensor_nbytes((jinf_qtype)type, cols()); }
    uint64_t n_bytes() const { return row_bytes() * (uint64_t)rows(); }
};

}  // namespace

struct jinf_synth_model {
    jinf_synth_config cfg;
    std::vector<SynthTensor> tensors;
    const SynthTensor* find(const char* name) const {
        for (auto& t : tensors) if (t.name == name) return &t;
        return nullptr;
    }
};

extern "C" jinf_status jinf_synth_create(jinf_synth_model** out, const jinf_synth_config* cfg) {
    if (!out || !cfg) return JINF_ERR_INVALID;
    const jinf_model_hparams& hp = cfg->hp;
    if (hp.n_layers == 0 || hp.n_embd == 0 || hp.n_heads == 0 || hp.n_ff == 0 || hp.n_vocab == 0)
        return JINF_ERR_INVALID;
    const uint32_t hkv = hp.n_heads_kv ? hp.n_heads_kv : hp.n_heads;
    if (hp.n_embd % hp.n_heads || hp.n_heads % hkv) return JINF_ERR_INVALID;
    const int wt = cfg->weight_type, mt = cfg->mix_type ? cfg->mix_type : cfg->weight_type;
    auto quant_ok = [](int t) {
        return t == JINF_TYPE_Q4_0 || t == JINF_TYPE_Q4_K || t == JINF_TYPE_Q6_K || t == JINF_TYPE_Q8_0;
    };
    if (!quant_ok(wt) || !quant_ok(mt)) return JINF_ERR_INVALID;
    for (const int t : {wt, mt}) {
        const int bs = jinf_qtype_block_size((jinf_qtype)t);
        if (hp.n_embd % bs || hp.n_ff % bs) return JINF_ERR_INVALID;
    }

    jinf_synth_model* m = new jinf_synth_model();
    m->cfg = *cfg;
    m->cfg.hp.n_heads_kv = hkv;
    if (m->cfg.hp.arch[0] == 0) strcpy(m->cfg.hp.arch, "llama");
    const int64_t d = hp.n_embd, kv = (int64_t)(hp.n_embd / hp.n_heads) * hkv, ff = hp.n_ff, V = hp.n_vocab;
    auto add = [&](const std::string& name, int type, int nd, int64_t s0, int64_t s1, int role) {
        SynthTensor t;
        t.name = name; t.type = type; t.n_dims = nd;
        t.shape[0] = s0; t.shape[1] = nd > 1 ? s1 : 1; t.shape[2] = 1; t.shape[3] = 1;
        t.role = role;
        m->tensors.push_back(t);
    };
    add("token_embd.weight", JINF_TYPE_F32, 2, d, V, 2);
    char buf[96];
    for (uint32_t L = 0; L < hp.n_layers; ++L) {
        snprintf(buf, sizeof buf, "blk.%u.attn_norm.weight", L);   add(buf, JINF_TYPE_F32, 1, d, 1, 1);
        snprintf(buf, sizeof buf, "blk.%u.attn_q.weight", L);      add(buf, wt, 2, d, d, 0);
        snprintf(buf, sizeof buf, "blk.%u.attn_k.weight", L);      add(buf, wt, 2, d, kv, 0);
        const int lt = L % 2 == 0 ? mt : wt;  // attn_v and ffn_down of the even layers
        snprintf(buf, sizeof buf, "blk.%u.attn_v.weight", L);      add(buf, lt, 2, d, kv, 0);
        snprintf(buf, sizeof buf, "blk.%u.attn_output.weight", L); add(buf, wt, 2, d, d, 0);
        snprintf(buf, sizeof buf, "blk.%u.ffn_norm.weight", L);    add(buf, JINF_TYPE_F32, 1, d, 1, 1);
        snprintf(buf, sizeof buf, "blk.%u.ffn_gate.weight", L);    add(buf, wt, 2, d, ff, 0);
        snprintf(buf, sizeof buf, "blk.%u.ffn_up.weight", L);      add(buf, wt, 2, d, ff, 0);
        snprintf(buf, sizeof buf, "blk.%u.ffn_down.weight", L);    add(buf, lt, 2, ff, d, 0);
    }
    add("output_norm.weight", JINF_TYPE_F32, 1, d, 1, 1);
    add("output.weight", mt, 2, d, V, 0);
    *out = m;
    return JINF_OK;
}

extern "C" void jinf_synth_destroy(jinf_synth_model* m) { delete m; }

extern "C" const jinf_synth_config* jinf_synth_get_config(const jinf_synth_model* m) {
    return m ? &m->cfg : nullptr;
}

extern "C" int jinf_synth_n_tensors(const jinf_synth_model* m) { return m ? (int)m->tensors.size() : 0; }

extern "C" const char* jinf_synth_tensor_name(const jinf_synth_model* m, int i) {
    if (!m || i < 0 || i >= (int)m->tensors.size()) return nullptr;
    return m->tensors[i].name.c_str();
}

extern "C" jinf_status jinf_synth_tensor_info(const jinf_synth_model* m, const char* name, int* type,
                                              int64_t* shape4, int* n_dims, uint64_t* n_bytes) {
    if (!m || !name) return JINF_ERR_INVALID;
    const SynthTensor* t = m->find(name);
    if (!t) return JINF_ERR_INVALID;
    if (type) *type = t->type;
    if (shape4) memcpy(shape4, t->shape, sizeof t->shape);
    if (n_dims) *n_dims = t->n_dims;
    if (n_bytes) *n_bytes = t->n_bytes();
    return JINF_OK;
}

extern "C" jinf_status jinf_synth_read_rows(const jinf_synth_model* m, const char* name, int64_t row0,
                                           int64_t n_rows, void* dst) {
    if (!m || !name || !dst || row0 < 0 || n_rows < 0) return JINF_ERR_INVALID;
    const SynthTensor* t = m->find(name);
    if (!t || row0 + n_rows > t->rows()) return JINF_ERR_INVALID;
    const int64_t cols = t->cols();
    const uint64_t rb = t->row_bytes();
    const uint64_t key = splitmix64(m->cfg.seed ^ fnv1a64(t->name.c_str()));
    if (t->role == 1) {
        float* o = (float*)dst;
        for (int64_t i = 0; i < n_rows * cols; ++i) o[i] = 1.0f;
        return JINF_OK;
    }
    const float stdv = t->role == 2 ? m->cfg.embed_std : m->cfg.weight_std;
#pragma omp parallel
    {
        std::vector<float> row((size_t)cols);
#pragma omp for schedule(static)
        for (int64_t r = 0; r < n_rows; ++r) {
            const uint64_t idx0 = (uint64_t)(row0 + r) * (uint64_t)cols;
            uint8_t* o = (uint8_t*)dst + (uint64_t)r * rb;
            if (t->type == JINF_TYPE_F32) {
                gen_normals(key, idx0, cols, stdv, (float*)o);
            } else {
                gen_normals(key, idx0, cols, stdv, row.data());
                if (t->type == JINF_TYPE_Q4_0)
                    jinf_quantize_q4_0(row.data(), (jinf_block_q4_0*)o, cols);
                else if (t->type == JINF_TYPE_Q4_K)
                    jinf_quantize_q4_K(row.data(), (jinf_block_q4_K*)o, cols);
                else if (t->type == JINF_TYPE_Q6_K)
                    jinf_quantize_q6_K(row.data(), (jinf_block_q6_K*)o, cols);
                else
                    jinf_quantize_q8_0(row.data(), (jinf_block_q8_0*)o, cols);
            }
        }
    }
    return JINF_OK;
}

extern "C" jinf_status jinf_synth_write_gguf(const jinf_synth_model* m, const char* path) {
    if (!m || !path) return JINF_ERR_INVALID;
    jinf_gguf_writer* w = nullptr;
    JINF_CHECK(jinf_gguf_writer_create(&w, path), "gguf writer");
    const jinf_model_hparams& hp = m->cfg.hp;
    jinf_gguf_writer_add_kv_str(w, "general.architecture", hp.arch);
    std::string p = std::string(hp.arch) + ".";
    jinf_gguf_writer_add_kv_u32(w, (p + "block_count").c_str(), hp.n_layers);
    jinf_gguf_writer_add_kv_u32(w, (p + "embedding_length").c_str(), hp.n_embd);
    jinf_gguf_writer_add_kv_u32(w, (p + "attention.head_count").c_str(), hp.n_heads);
    jinf_gguf_writer_add_kv_u32(w, (p + "attention.head_count_kv").c_str(), hp.n_heads_kv);
    jinf_gguf_writer_add_kv_u32(w, (p + "feed_forward_length").c_str(), hp.n_ff);
    jinf_gguf_writer_add_kv_u32(w, (p + "vocab_size").c_str(), hp.n_vocab);
    jinf_gguf_writer_add_kv_u32(w, (p + "context_length").c_str(), hp.n_ctx_train ? hp.n_ctx_train : 8192);
    jinf_gguf_writer_add_kv_f32(w, (p + "rope.freq_base").c_str(), hp.rope_freq_base);
    jinf_gguf_writer_add_kv_f32(w, (p + "attention.layer_norm_rms_epsilon").c_str(), hp.rms_norm_eps);
    for (auto& t : m->tensors) {
        std::vector<uint8_t> buf(t.n_bytes());
        jinf_synth_read_rows(m, t.name.c_str(), 0, t.rows(), buf.data());
        jinf_status s = jinf_gguf_writer_add_tensor(w, t.name.c_str(), t.n_dims, t.shape,
                                                    (jinf_qtype)t.type, buf.data(), buf.size());
        if (s != JINF_OK) return s;
    }
    return jinf_gguf_writer_finish(w);
}

extern "C" jinf_status jinf_synth_write_nvmw(const jinf_synth_model* m, const char* path) {
    if (!m || !path) return JINF_ERR_INVALID;
    const jinf_model_hparams& hp = m->cfg.hp;
    jinf_nvmw_writer* w = nullptr;
    JINF_CHECK(jinf_nvmw_writer_create(&w, path), "nvmw writer");
    jinf_nvmw_header hdr;
    memset(&hdr, 0, sizeof hdr);
    hdr.magic = JINF_NVMW_MAGIC;
    hdr.version = JINF_NVMW_VERSION;
    hdr.n_layers = hp.n_layers;
    hdr.n_tensors = (uint32_t)m->tensors.size();
    hdr.n_embd = hp.n_embd;
    hdr.n_heads = hp.n_heads;
    hdr.n_heads_kv = hp.n_heads_kv;
    hdr.n_ff = hp.n_ff;
    hdr.n_vocab = hp.n_vocab;
    hdr.n_ctx_train = hp.n_ctx_train ? hp.n_ctx_train : 8192;
    hdr.rope_freq_base = hp.rope_freq_base;
    hdr.rms_norm_eps = hp.rms_norm_eps;
    hdr.primary_type = m->cfg.weight_type;
    const size_t index_size = (size_t)hp.n_layers * sizeof(jinf_nvmw_layer_desc) +
                              m->tensors.size() * sizeof(jinf_nvmw_tensor_entry);
    hdr.index_offset = 4096;
    hdr.index_size = index_size;
    hdr.hot_offset = JINF_ALIGN_4K(4096 + index_size);
    uint64_t cursor = 0;
    for (auto& t : m->tensors) {
        jinf_nvmw_tensor_entry te;
        memset(&te, 0, sizeof te);
        strncpy(te.name, t.name.c_str(), sizeof te.name - 1);
        te.type = (jinf_qtype)t.type;
        memcpy(te.shape, t.shape, sizeof te.shape);
        te.n_dims = (uint32_t)t.n_dims;
        te.offset = cursor;
        te.n_bytes = t.n_bytes();
        te.layer_index = -1;
        if (strncmp(t.name.c_str(), "blk.", 4) == 0) te.layer_index = atoi(t.name.c_str() + 4);
        te.is_hot = 1;
        jinf_nvmw_writer_add_tensor_entry(w, &te);
        cursor += JINF_ALIGN_4K(t.n_bytes());
    }
    hdr.hot_size = cursor;
    hdr.cold_start_offset = JINF_ALIGN_4K(hdr.hot_offset + cursor);
    hdr.cold_total_size = 0;
    for (uint32_t L = 0; L < hp.n_layers; ++L) {
        jinf_nvmw_layer_desc ld;
        memset(&ld, 0, sizeof ld);
        ld.cold_start_offset = hdr.cold_start_offset;
        jinf_nvmw_writer_add_layer_desc(w, (int)L, &ld);
    }
    jinf_nvmw_writer_set_header(w, &hdr);
    jinf_status s = jinf_nvmw_writer_finalize(w);
    if (s != JINF_OK) { jinf_nvmw_writer_destroy(w); return s; }
    for (auto& t : m->tensors) {
        std::vector<uint8_t> buf(JINF_ALIGN_4K(t.n_bytes()), 0);
        jinf_synth_read_rows(m, t.name.c_str(), 0, t.rows(), buf.data());
        s = jinf_nvmw_writer_write_hot(w, buf.data(), buf.size());
        if (s != JINF_OK) { jinf_nvmw_writer_destroy(w); return s; }
    }
    jinf_nvmw_writer_destroy(w);
    return JINF_OK;
}

bool jinf::synth_tensor_params(const jinf_synth_model* m, const char* name, uint64_t* key, float* stdv, int* role) {
    if (!m || !name) return false;
    const SynthTensor* t = m->find(name);
    if (!t) return false;
    *key = splitmix64(m->cfg.seed ^ fnv1a64(t->name.c_str()));
    *stdv = t->role == 2 ? m->cfg.embed_std : m->cfg.weight_std;
    *role = t->role;
    return true;
}

// ---------------------------------------------------------------- sparse-FFN synthetic data

// Fixed neuron mask of a layer: runs of 8 consecutive neurons, each kept with probability
// `keep` (seeded). Writes the kept ids ascending (when `ids` is not NULL); returns the count.
extern "C" int jinf_sparse_fixed_mask(uint64_t seed, int layer, int n_ff, float keep, int32_t* ids) {
    if (n_ff <= 0 || layer < 0) return 0;
    int n = 0;
    const uint64_t base = jinf_synth::mask_key(seed, layer);
    for (int run = 0; run < (n_ff + 7) / 8; ++run) {
        const double u = jinf_synth::to_unit(jinf_synth::splitmix64(base + (uint64_t)run));
        if (u > (double)keep) continue;  // u in (0, 1]: kept with probability `keep`
        for (int i = 8 * run; i < 8 * run + 8 && i < n_ff; ++i) {
            if (ids) ids[n] = i;
            ++n;
        }
    }
    return n;
}

// Predictor weights of a layer (which 1: W1 [r][d], 2: W2 [n_ff][r]) as fp16 bits ~ N(0, 0.02):
// the same values the engine generates on the device.
extern "C" void jinf_sparse_predictor_weights(uint64_t seed, int layer, int which, int64_t n, uint16_t* out) {
    const uint64_t key = jinf_synth::predictor_key(seed, layer, which);
    for (int64_t i = 0; i < n; ++i) out[i] = jinf_synth::fp32_to_fp16(jinf_synth::normal_at(key, (uint64_t)i, 0.02f));
}
