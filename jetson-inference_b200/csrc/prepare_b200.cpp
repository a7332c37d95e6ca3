// GGUF -> B200-layout NVMW (version 3): the engine's weight arena written ahead of time. New,
// with no counterpart in the reference, whose tools/prepare_model.cpp copies the GGUF blocks
// (this library writes that format too: prepare_model.cpp).
//
// Every projection is stored the way the engine streams it on one GPU: per layer the fused
// QKV (q, k, v rows; when v has another type than q and k, [q | k] and v as two matrices),
// o, gate|up with rows interleaved gate_n, up_n, down, and the output head, each already
// repacked into its Q4M image (q4m.cuh, by the same lane functions as the device repack).
// Such a tensor has type JINF_NVMW_TYPE_Q4M + its Q4M format and shape [cols, rows]. The
// embedding table and the norm gains are copied as they are. Everything lies in the hot
// region (on B200 the whole model is in HBM), 4 KB aligned; the cold regions are empty.
// The engine copies each image into its arena without staging or repacking. The file is
// prepared for the dense FFN and for one GPU, or (jinf_prepare_model_b200_tp) for tensor
// parallelism over tp_size GPUs: then every rank r has its own images, named
// "tp<size>.<r>." + the one-GPU name, each the rank's slice in the engine's split
// (jinf_tp_shard: q, k, v, gate, up and the output head by rows, o and down by whole column
// blocks), so a rank reads exactly its shard.
#include "jinf/b200.h"
#include "jinf/common.h"
#include "jinf/gguf.h"
#include "jinf/nvmw.h"
#include "jinf/quant.h"
#include "jinf/splitter.h"

#include <stdio.h>
#include <string.h>

#include <string>
#include <vector>

namespace {

struct Item {
    std::string name;
    int layer;
    // a copied tensor (src) or a packed matrix assembled from up to 3 sources
    const jinf_gguf_tensor_info* src = nullptr;
    const jinf_gguf_tensor_info* parts[3] = {nullptr, nullptr, nullptr};
    int64_t r0[3] = {0, 0, 0}, nr[3] = {0, 0, 0}, c0[3] = {0, 0, 0};  // each part's slice (rows, first column)
    bool interleave = false;  // gate|up: rows alternate parts[0], parts[1]
    int qtype = 0;
    int64_t rows = 0, cols = 0;
    uint64_t bytes = 0, offset = 0;
};

const jinf_gguf_tensor_info* find(const jinf_gguf_file* g, const std::string& name) {
    for (uint64_t i = 0; i < g->tensor_count; ++i)
        if (name == g->tensor_infos[i].name) return &g->tensor_infos[i];
    return nullptr;
}

bool read_at(FILE* in, uint64_t off, void* dst, size_t n) {
    return fseeko(in, (off_t)off, SEEK_SET) == 0 && fread(dst, 1, n, in) == n;
}

}  // namespace

extern "C" jinf_status jinf_prepare_model_b200_tp(const char* gguf_path, const char* nvmw_path, int tp_size) {
    if (!gguf_path || !nvmw_path || (tp_size != 1 && tp_size != 2 && tp_size != 4 && tp_size != 8))
        return JINF_ERR_INVALID;
    jinf_gguf_file* g = nullptr;
    JINF_CHECK(jinf_gguf_open(&g, gguf_path), "gguf");
    const jinf_model_hparams hp = g->hparams;
    const int L = (int)hp.n_layers;
    std::vector<Item> items;
    jinf_status st = JINF_OK;
    auto fail = [&](const char* what, const std::string& name) {
        JINF_LOG("prepare_model_b200: %s: %s", what, name.c_str());
        st = JINF_ERR_INVALID;
    };
    auto copy_item = [&](const std::string& name, int layer) {
        const jinf_gguf_tensor_info* t = find(g, name);
        if (!t) return fail("tensor missing", name);
        Item it;
        it.name = name;
        it.layer = layer;
        it.src = t;
        it.bytes = t->n_bytes;
        items.push_back(it);
    };
    // one image per rank: the fused slices of the sources
    auto packed_item = [&](const std::string& name, int layer, std::vector<std::string> srcs, bool interleave) {
        for (int rank = 0; rank < tp_size && st == JINF_OK; ++rank) {
            Item it;
            it.name = tp_size == 1 ? name : "tp" + std::to_string(tp_size) + "." + std::to_string(rank) + "." + name;
            it.layer = layer;
            it.interleave = interleave;
            for (size_t i = 0; i < srcs.size(); ++i) {
                const jinf_gguf_tensor_info* t = find(g, srcs[i]);
                if (!t || t->n_dims != 2) return fail("matrix missing", srcs[i]);
                if (i > 0 && (t->type != it.parts[0]->type || t->shape[0] != it.parts[0]->shape[0]))
                    return fail("fused matrices of different types or widths", srcs[i]);
                int64_t r0, nr, c0, nc;
                if (jinf_tp_shard(srcs[i].c_str(), t->shape[1], t->shape[0], rank, tp_size, &r0, &nr, &c0, &nc) !=
                    JINF_OK)
                    return fail("no tensor-parallel split of this shape", srcs[i]);
                if (c0 % jinf_qtype_block_size(t->type) || nc % jinf_qtype_block_size(t->type))
                    return fail("column split inside a block", srcs[i]);
                if (i > 0 && nc != it.cols) return fail("fused matrices split to different widths", srcs[i]);
                it.parts[i] = t;
                it.r0[i] = r0;
                it.nr[i] = nr;
                it.c0[i] = c0;
                it.cols = nc;
                it.rows += nr;
            }
            it.qtype = it.parts[0]->type;
            it.bytes = jinf_b200_q4m_bytes_qt((int)it.rows, (int)it.cols, it.qtype);
            if (!it.bytes) return fail("no Q4M form for this type or width", it.name);
            items.push_back(it);
        }
    };
    copy_item("token_embd.weight", -1);
    char b[160];
    for (int l = 0; l < L && st == JINF_OK; ++l) {
        auto nm = [&](const char* part) {
            snprintf(b, sizeof b, "blk.%d.%s", l, part);
            return std::string(b);
        };
        copy_item(nm("attn_norm.weight"), l);
        copy_item(nm("ffn_norm.weight"), l);
        const jinf_gguf_tensor_info* tq = find(g, nm("attn_q.weight"));
        const jinf_gguf_tensor_info* tv = find(g, nm("attn_v.weight"));
        if (!tq || !tv) {
            fail("attention matrices missing", nm("attn_q.weight"));
            break;
        }
        if (tv->type == tq->type) {
            packed_item(nm("qkv.q4m"), l, {nm("attn_q.weight"), nm("attn_k.weight"), nm("attn_v.weight")}, false);
        } else {
            packed_item(nm("qkv.q4m"), l, {nm("attn_q.weight"), nm("attn_k.weight")}, false);
            packed_item(nm("v.q4m"), l, {nm("attn_v.weight")}, false);
        }
        packed_item(nm("o.q4m"), l, {nm("attn_output.weight")}, false);
        packed_item(nm("gu.q4m"), l, {nm("ffn_gate.weight"), nm("ffn_up.weight")}, true);
        packed_item(nm("down.q4m"), l, {nm("ffn_down.weight")}, false);
    }
    if (st == JINF_OK) {
        copy_item("output_norm.weight", -1);
        packed_item("output.q4m", -1, {"output.weight"}, false);
    }
    FILE* in = st == JINF_OK ? fopen(gguf_path, "rb") : nullptr;
    if (st != JINF_OK || !in) {
        jinf_gguf_close(g);
        return st != JINF_OK ? st : JINF_ERR_IO;
    }

    // header and index: every tensor in the hot region, 4 KB aligned
    jinf_nvmw_header h;
    memset(&h, 0, sizeof h);
    h.magic = JINF_NVMW_MAGIC;
    h.version = JINF_NVMW_VERSION_B200;
    h.n_layers = hp.n_layers;
    h.n_tensors = (uint32_t)items.size();
    h.n_embd = hp.n_embd;
    h.n_heads = hp.n_heads;
    h.n_heads_kv = hp.n_heads_kv;
    h.n_ff = hp.n_ff;
    h.n_vocab = hp.n_vocab;
    h.n_ctx_train = hp.n_ctx_train;
    h.rope_freq_base = hp.rope_freq_base;
    h.rms_norm_eps = hp.rms_norm_eps;
    h.primary_type = items.size() > 3 ? items[3].qtype : 0;  // the first layer's QKV type
    uint64_t cursor = 0;
    for (auto& it : items) {
        it.offset = cursor;
        cursor += JINF_ALIGN_4K(it.bytes);
    }
    const size_t index_size =
        (size_t)h.n_layers * sizeof(jinf_nvmw_layer_desc) + (size_t)h.n_tensors * sizeof(jinf_nvmw_tensor_entry);
    h.index_offset = 4096;
    h.index_size = index_size;
    h.hot_offset = JINF_ALIGN_4K(4096 + index_size);
    h.hot_size = cursor;
    h.cold_start_offset = h.hot_offset + cursor;
    h.cold_total_size = 0;
    jinf_nvmw_writer* w = nullptr;
    if (jinf_nvmw_writer_create(&w, nvmw_path) != JINF_OK) {
        fclose(in);
        jinf_gguf_close(g);
        return JINF_ERR_IO;
    }
    for (const auto& it : items) {
        jinf_nvmw_tensor_entry e;
        memset(&e, 0, sizeof e);
        strncpy(e.name, it.name.c_str(), sizeof(e.name) - 1);
        if (it.src) {
            e.type = it.src->type;
            memcpy(e.shape, it.src->shape, sizeof(e.shape));
            e.n_dims = it.src->n_dims;
        } else {
            e.type = (jinf_qtype)(JINF_NVMW_TYPE_Q4M + q4m_format_of_qtype(it.qtype));
            e.shape[0] = it.cols;
            e.shape[1] = it.rows;
            e.shape[2] = e.shape[3] = 1;
            e.n_dims = 2;
        }
        e.offset = it.offset;
        e.n_bytes = it.bytes;
        e.layer_index = it.layer;
        e.is_hot = 1;
        jinf_nvmw_writer_add_tensor_entry(w, &e);
    }
    for (int l = 0; l < L; ++l) {
        jinf_nvmw_layer_desc ld;
        memset(&ld, 0, sizeof ld);
        ld.cold_start_offset = h.cold_start_offset;
        jinf_nvmw_writer_add_layer_desc(w, l, &ld);
    }
    jinf_nvmw_writer_set_header(w, &h);
    st = jinf_nvmw_writer_finalize(w);
    jinf_nvmw_writer_destroy(w);

    // tensor data
    FILE* out = st == JINF_OK ? fopen(nvmw_path, "r+b") : nullptr;
    if (st == JINF_OK && !out) st = JINF_ERR_IO;
    std::vector<uint8_t> aos, img;
    for (size_t k = 0; k < items.size() && st == JINF_OK; ++k) {
        const Item& it = items[k];
        if (it.src) {
            img.assign(JINF_ALIGN_4K(it.bytes), 0);
            if (!read_at(in, g->data_offset + it.src->offset, img.data(), it.bytes)) st = JINF_ERR_IO;
        } else {
            // the fused slices in the reference's blocks, then their Q4M image
            const jinf_qtype qt = (jinf_qtype)it.qtype;
            const size_t bb = jinf_qtype_type_size(qt);
            const int64_t bs = jinf_qtype_block_size(qt);
            const size_t rb = (size_t)(it.cols / bs) * bb;  // bytes of one row of the slice
            aos.assign(rb * (size_t)it.rows, 0);
            size_t row0 = 0;
            for (int i = 0; i < 3 && it.parts[i] && st == JINF_OK; ++i) {
                const jinf_gguf_tensor_info* t = it.parts[i];
                const size_t srb = t->n_bytes / (size_t)t->shape[1];  // bytes of one source row
                std::vector<uint8_t> tmp((size_t)it.nr[i] * srb);
                if (!read_at(in, g->data_offset + t->offset + (uint64_t)it.r0[i] * srb, tmp.data(), tmp.size())) {
                    st = JINF_ERR_IO;
                    break;
                }
                const size_t coff = (size_t)(it.c0[i] / bs) * bb;
                for (int64_t r = 0; r < it.nr[i]; ++r) {
                    const size_t dst_row = it.interleave ? (size_t)(2 * r + i) : row0 + (size_t)r;
                    memcpy(aos.data() + dst_row * rb, tmp.data() + (size_t)r * srb + coff, rb);
                }
                row0 += (size_t)it.nr[i];
            }
            img.assign(JINF_ALIGN_4K(it.bytes), 0);
            if (st == JINF_OK)
                st = jinf_b200_q4m_pack_host(aos.data(), it.qtype, img.data(), (int)it.rows, (int)it.cols);
        }
        if (st == JINF_OK && (fseeko(out, (off_t)(h.hot_offset + it.offset), SEEK_SET) != 0 ||
                              fwrite(img.data(), 1, img.size(), out) != img.size()))
            st = JINF_ERR_IO;
    }
    if (out) fclose(out);
    fclose(in);
    jinf_gguf_close(g);
    return st;
}

extern "C" jinf_status jinf_prepare_model_b200(const char* gguf_path, const char* nvmw_path) {
    return jinf_prepare_model_b200_tp(gguf_path, nvmw_path, 1);
}
