// GGUF -> NVMW conversion, the format producer of reference tools/prepare_model.cpp (the
// file it writes, byte for byte): header and index at 4096, the split plan's hot tensors
// then each layer's cold tensors, every tensor 4 KB padded, and with `bundled` the neuron
// bundles (gate row, up row, down column as fp32 dequantised like the reference's
// src/quant.cpp) followed by the bundle index, the header then marking version 2.
//
// Layout steps (reference tools/prepare_model.cpp:99-214 header, plan and offsets;
// :228-288 data; :293-492 bundles):
//   index        = n_layers layer descs + n_tensors entries, at 4096
//   hot region   = align4K(4096 + index), the hot tensors in plan order, each align4K
//   cold         = from align4K(hot end), per layer: its cold tensors in plan order, each
//                  align4K, offsets relative to the layer's start
//   bundles      = align4K(end of cold); per layer n_ff bundles of
//                  align4K(2 row_bytes(primary type) + 4 n_embd) bytes; then align4K and
//                  the bundle header + per-layer descs
#include "jinf/gguf.h"
#include "jinf/nvmw.h"
#include "jinf/quant.h"
#include "jinf/splitter.h"

#include <stdio.h>
#include <string.h>

#include <string>
#include <vector>

namespace {

struct Out {
    FILE* fp = nullptr;
    bool ok = true;
    void write(const void* p, size_t n) {
        if (ok && n && fwrite(p, 1, n, fp) != n) ok = false;
    }
    void pad_4k() {
        const long pos = ftell(fp);
        if (pos < 0) {
            ok = false;
            return;
        }
        const size_t to = JINF_ALIGN_4K((size_t)pos);
        std::vector<uint8_t> z(to - (size_t)pos, 0);
        write(z.data(), z.size());
    }
};

bool read_tensor(FILE* in, const jinf_gguf_file* g, const jinf_gguf_tensor_info* t, std::vector<uint8_t>& buf,
                 size_t size) {
    buf.assign(size, 0);
    if (fseek(in, (long)(g->data_offset + t->offset), SEEK_SET) != 0) return false;
    return fread(buf.data(), 1, (size_t)t->n_bytes, in) == (size_t)t->n_bytes;
}

size_t row_bytes_of(jinf_qtype t, uint32_t n) {
    const int bs = jinf_qtype_block_size(t);
    return (size_t)((n + bs - 1) / bs) * jinf_qtype_type_size(t);
}

// The FFN tensors of a layer, matched by name as the reference does (last match wins).
void ffn_tensors(const jinf_gguf_file* g, int layer, const jinf_gguf_tensor_info** gate,
                 const jinf_gguf_tensor_info** up, const jinf_gguf_tensor_info** down) {
    char prefix[64];
    snprintf(prefix, sizeof prefix, "blk.%d.", layer);
    *gate = *up = *down = nullptr;
    for (uint64_t i = 0; i < g->tensor_count; ++i) {
        const jinf_gguf_tensor_info* t = &g->tensor_infos[i];
        if (!strstr(t->name, prefix)) continue;
        if (strstr(t->name, "ffn_gate.weight")) *gate = t;
        else if (strstr(t->name, "ffn_up.weight")) *up = t;
        else if (strstr(t->name, "ffn_down.weight")) *down = t;
    }
}

}  // namespace

extern "C" jinf_status jinf_prepare_model(const char* gguf_path, const char* nvmw_path, size_t gpu_budget_mb,
                                          int bundled) {
    if (!gguf_path || !nvmw_path) return JINF_ERR_INVALID;
    jinf_gguf_file* g = nullptr;
    JINF_CHECK(jinf_gguf_open(&g, gguf_path), "gguf");
    jinf_split_config sc;
    memset(&sc, 0, sizeof sc);
    sc.gpu_memory_budget = gpu_budget_mb * 1024 * 1024;
    jinf_split_plan* plan = nullptr;
    jinf_status s = jinf_split_analyze(g, &sc, &plan);
    if (s != JINF_OK) {
        jinf_gguf_close(g);
        return s;
    }
    FILE* in = fopen(gguf_path, "rb");
    jinf_nvmw_writer* w = nullptr;
    if (!in || jinf_nvmw_writer_create(&w, nvmw_path) != JINF_OK) {
        if (in) fclose(in);
        jinf_split_plan_free(plan);
        jinf_gguf_close(g);
        return JINF_ERR_IO;
    }

    jinf_nvmw_header h;
    memset(&h, 0, sizeof h);
    h.magic = JINF_NVMW_MAGIC;
    h.version = JINF_NVMW_VERSION;
    h.n_layers = g->hparams.n_layers;
    h.n_tensors = (uint32_t)g->tensor_count;
    h.n_embd = g->hparams.n_embd;
    h.n_heads = g->hparams.n_heads;
    h.n_heads_kv = g->hparams.n_heads_kv;
    h.n_ff = g->hparams.n_ff;
    h.n_vocab = g->hparams.n_vocab;
    h.n_ctx_train = g->hparams.n_ctx_train;
    h.rope_freq_base = g->hparams.rope_freq_base;
    h.rms_norm_eps = g->hparams.rms_norm_eps;
    for (uint64_t i = 0; i < g->tensor_count; ++i)  // primary type: the first tensor above 1 MB
        if (g->tensor_infos[i].n_bytes > 1024 * 1024) {
            h.primary_type = (int32_t)g->tensor_infos[i].type;
            break;
        }

    // hot tensors in plan order, cold ones per layer in plan order (non-layer cold dropped)
    std::vector<const jinf_weight_assignment*> hot;
    std::vector<std::vector<const jinf_weight_assignment*>> cold(h.n_layers);
    for (int i = 0; i < plan->count; ++i) {
        const jinf_weight_assignment* a = &plan->assignments[i];
        if (a->placement == JINF_PLACE_HOT) hot.push_back(a);
        else if (a->layer_index >= 0 && a->layer_index < (int)h.n_layers) cold[a->layer_index].push_back(a);
    }
    size_t hot_total = 0;
    for (const auto* a : hot) hot_total += JINF_ALIGN_4K(a->tensor->n_bytes);
    const size_t index_size =
        (size_t)h.n_layers * sizeof(jinf_nvmw_layer_desc) + (size_t)h.n_tensors * sizeof(jinf_nvmw_tensor_entry);
    h.index_offset = 4096;
    h.index_size = index_size;
    h.hot_offset = JINF_ALIGN_4K(4096 + index_size);
    h.hot_size = hot_total;
    h.cold_start_offset = JINF_ALIGN_4K(h.hot_offset + hot_total);

    auto entry_of = [&](const jinf_weight_assignment* a, uint64_t offset, int layer, int is_hot) {
        jinf_nvmw_tensor_entry e;
        memset(&e, 0, sizeof e);
        strncpy(e.name, a->tensor->name, sizeof(e.name) - 1);
        e.type = a->tensor->type;
        memcpy(e.shape, a->tensor->shape, sizeof(e.shape));
        e.n_dims = a->tensor->n_dims;
        e.offset = offset;
        e.n_bytes = a->tensor->n_bytes;
        e.layer_index = layer;
        e.is_hot = (uint8_t)is_hot;
        return e;
    };
    uint64_t cursor = 0;
    for (const auto* a : hot) {
        const jinf_nvmw_tensor_entry e = entry_of(a, cursor, a->layer_index, 1);
        jinf_nvmw_writer_add_tensor_entry(w, &e);
        cursor += JINF_ALIGN_4K(a->tensor->n_bytes);
    }
    uint64_t cold_cursor = h.cold_start_offset;
    for (int l = 0; l < (int)h.n_layers; ++l) {
        const uint64_t start = JINF_ALIGN_4K(cold_cursor);
        uint64_t off = 0;
        for (const auto* a : cold[l]) {
            const jinf_nvmw_tensor_entry e = entry_of(a, off, l, 0);
            jinf_nvmw_writer_add_tensor_entry(w, &e);
            off += JINF_ALIGN_4K(a->tensor->n_bytes);
        }
        jinf_nvmw_layer_desc ld;
        memset(&ld, 0, sizeof ld);
        ld.cold_start_offset = start;
        ld.cold_total_size = off;
        ld.n_cold_tensors = (uint32_t)cold[l].size();
        jinf_nvmw_writer_add_layer_desc(w, l, &ld);
        cold_cursor = start + off;
    }
    h.cold_total_size = cold_cursor - h.cold_start_offset;
    jinf_nvmw_writer_set_header(w, &h);
    s = jinf_nvmw_writer_finalize(w);
    jinf_nvmw_writer_destroy(w);

    Out o;
    if (s == JINF_OK) {
        o.fp = fopen(nvmw_path, "r+b");
        if (!o.fp) s = JINF_ERR_IO;
    }
    std::vector<uint8_t> buf;
    if (s == JINF_OK) {
        fseek(o.fp, (long)h.hot_offset, SEEK_SET);
        // Hot tensors go through one reused copy buffer whose padding is not cleared, so a
        // tensor's padding holds what the buffer last held there (bytes it gains are zero). The
        // reference writes the same bytes (tools/prepare_model.cpp:246-255); no reader looks
        // at them, but keeping them makes the two files identical.
        std::vector<uint8_t> reuse;
        for (const auto* a : hot) {
            const size_t al = JINF_ALIGN_4K(a->tensor->n_bytes);
            reuse.resize(al, 0);  // shrinking drops bytes; growing adds zeros
            if (fseek(in, (long)(g->data_offset + a->tensor->offset), SEEK_SET) != 0 ||
                fread(reuse.data(), 1, (size_t)a->tensor->n_bytes, in) != (size_t)a->tensor->n_bytes)
                s = JINF_ERR_IO;
            o.write(reuse.data(), al);
        }
        for (int l = 0; l < (int)h.n_layers && s == JINF_OK; ++l) {
            if (cold[l].empty()) continue;
            for (const auto* a : cold[l]) {
                if (!read_tensor(in, g, a->tensor, buf, JINF_ALIGN_4K(a->tensor->n_bytes))) s = JINF_ERR_IO;
                o.write(buf.data(), buf.size());
            }
            o.pad_4k();
        }
    }
    if (s == JINF_OK && bundled) {
        const jinf_qtype qt = (jinf_qtype)h.primary_type;
        const size_t bundle = JINF_ALIGN_4K(2 * row_bytes_of(qt, h.n_embd) + (size_t)h.n_embd * sizeof(float));
        std::vector<jinf_nvmw_bundle_layer_desc> descs(h.n_layers);
        memset(descs.data(), 0, sizeof(jinf_nvmw_bundle_layer_desc) * descs.size());
        o.pad_4k();
        std::vector<uint8_t> gate, up, down, b(bundle);
        std::vector<float> downf;
        for (int l = 0; l < (int)h.n_layers && s == JINF_OK && o.ok; ++l) {
            const jinf_gguf_tensor_info *gt, *ut, *dt;
            ffn_tensors(g, l, &gt, &ut, &dt);
            if (!gt || !ut || !dt) continue;  // no FFN: an all-zero descriptor
            descs[l].bundles_offset = (uint64_t)ftell(o.fp);
            descs[l].n_neurons = h.n_ff;
            descs[l].bundle_size = (uint32_t)bundle;
            const size_t grb = row_bytes_of(gt->type, h.n_embd), urb = row_bytes_of(ut->type, h.n_embd);
            if (!read_tensor(in, g, gt, gate, gt->n_bytes) || !read_tensor(in, g, ut, up, ut->n_bytes) ||
                !read_tensor(in, g, dt, down, dt->n_bytes)) {
                s = JINF_ERR_IO;
                break;
            }
            downf.assign((size_t)h.n_embd * h.n_ff, 0.f);  // [n_embd][n_ff], as the reference dequantises
            jinf_dequantize(down.data(), dt->type, downf.data(), (int64_t)h.n_embd * h.n_ff);
            for (uint32_t n = 0; n < h.n_ff; ++n) {
                memset(b.data(), 0, bundle);
                memcpy(b.data(), gate.data() + (size_t)n * grb, grb);
                memcpy(b.data() + grb, up.data() + (size_t)n * urb, urb);
                float* col = reinterpret_cast<float*>(b.data() + grb + urb);
                for (uint32_t r = 0; r < h.n_embd; ++r) col[r] = downf[(size_t)r * h.n_ff + n];
                o.write(b.data(), bundle);
            }
            descs[l].bundles_total_size = (uint64_t)h.n_ff * bundle;
        }
        if (s == JINF_OK) {
            jinf_nvmw_bundle_header bh;
            memset(&bh, 0, sizeof bh);
            bh.n_bundle_layers = h.n_layers;
            bh.bundle_size = (uint32_t)bundle;
            bh.n_ff = h.n_ff;
            o.pad_4k();
            const long idx = ftell(o.fp);
            o.write(&bh, sizeof bh);
            o.write(descs.data(), sizeof(jinf_nvmw_bundle_layer_desc) * descs.size());
            // the header on disk: the bundle index and the bundled version
            jinf_nvmw_header hd;
            fseek(o.fp, 0, SEEK_SET);
            if (fread(&hd, sizeof hd, 1, o.fp) != 1) o.ok = false;
            hd.bundle_index_offset = (uint64_t)idx;
            hd.version = JINF_NVMW_VERSION_BUNDLED;
            fseek(o.fp, 0, SEEK_SET);
            o.write(&hd, sizeof hd);
        }
    }
    if (o.fp && fclose(o.fp) != 0) o.ok = false;
    if (s == JINF_OK && !o.ok) s = JINF_ERR_IO;
    fclose(in);
    jinf_split_plan_free(plan);
    jinf_gguf_close(g);
    return s;
}
