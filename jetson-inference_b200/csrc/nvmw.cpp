// .nvmw container reader/writer with the reference's file layout
// (reference include/jinf/nvmw.h:8-17, src/nvmw.cpp). The writer API and its call
// order are the reference's: finalize() writes the header and the index and leaves
// the stream at the 4K-aligned hot region, region bytes are appended after it.
#include "jinf/nvmw.h"

#include <stdlib.h>
#include <string.h>
#include <string>
#include <vector>

struct jinf_nvmw_writer {
    FILE* fp = nullptr;
    jinf_nvmw_header header{};
    std::vector<jinf_nvmw_layer_desc> layers;
    std::vector<jinf_nvmw_tensor_entry> entries;
};

struct jinf_nvmw_reader {
    std::string path;
    jinf_nvmw_header header{};
    std::vector<jinf_nvmw_layer_desc> layers;
    std::vector<jinf_nvmw_tensor_entry> entries;
    bool has_bundles = false;
    jinf_nvmw_bundle_header bundle_header{};
    std::vector<jinf_nvmw_bundle_layer_desc> bundle_layers;
};

static jinf_status pad_stream_4k(FILE* fp) {
    const long pos = ftell(fp);
    if (pos < 0) return JINF_ERR_IO;
    size_t pad = JINF_ALIGN_4K((size_t)pos) - (size_t)pos;
    static const uint8_t zeros[4096] = {0};
    while (pad) {
        const size_t n = pad < sizeof zeros ? pad : sizeof zeros;
        if (fwrite(zeros, 1, n, fp) != n) return JINF_ERR_IO;
        pad -= n;
    }
    return JINF_OK;
}

extern "C" jinf_status jinf_nvmw_writer_create(jinf_nvmw_writer** w, const char* path) {
    if (!w || !path) return JINF_ERR_INVALID;
    FILE* fp = fopen(path, "wb");
    if (!fp) {
        JINF_LOG("cannot create %s", path);
        return JINF_ERR_IO;
    }
    jinf_nvmw_writer* wr = new jinf_nvmw_writer();
    wr->fp = fp;
    *w = wr;
    return JINF_OK;
}

extern "C" void jinf_nvmw_writer_destroy(jinf_nvmw_writer* w) {
    if (!w) return;
    if (w->fp) fclose(w->fp);
    delete w;
}

extern "C" jinf_status jinf_nvmw_writer_set_header(jinf_nvmw_writer* w, const jinf_nvmw_header* hdr) {
    if (!w || !hdr) return JINF_ERR_INVALID;
    w->header = *hdr;
    return JINF_OK;
}

extern "C" jinf_status jinf_nvmw_writer_add_layer_desc(jinf_nvmw_writer* w, int layer,
                                                      const jinf_nvmw_layer_desc* desc) {
    if (!w || !desc || layer < 0) return JINF_ERR_INVALID;
    if ((size_t)layer >= w->layers.size()) w->layers.resize((size_t)layer + 1);
    w->layers[(size_t)layer] = *desc;
    return JINF_OK;
}

extern "C" jinf_status jinf_nvmw_writer_add_tensor_entry(jinf_nvmw_writer* w,
                                                        const jinf_nvmw_tensor_entry* entry) {
    if (!w || !entry) return JINF_ERR_INVALID;
    w->entries.push_back(*entry);
    return JINF_OK;
}

extern "C" jinf_status jinf_nvmw_writer_write_hot(jinf_nvmw_writer* w, const void* data, size_t size) {
    if (!w || !w->fp || !data) return JINF_ERR_INVALID;
    return fwrite(data, 1, size, w->fp) == size ? JINF_OK : JINF_ERR_IO;
}

extern "C" jinf_status jinf_nvmw_writer_write_cold_layer(jinf_nvmw_writer* w, int layer,
                                                        const void* data, size_t size) {
    if (!w || !w->fp || !data) return JINF_ERR_INVALID;
    JINF_CHECK(pad_stream_4k(w->fp), "pad");
    const long pos = ftell(w->fp);
    if (layer >= 0 && (size_t)layer < w->layers.size()) {
        w->layers[(size_t)layer].cold_start_offset = (uint64_t)pos;
        w->layers[(size_t)layer].cold_total_size = size;
    }
    return fwrite(data, 1, size, w->fp) == size ? JINF_OK : JINF_ERR_IO;
}

extern "C" jinf_status jinf_nvmw_writer_finalize(jinf_nvmw_writer* w) {
    if (!w || !w->fp) return JINF_ERR_INVALID;
    rewind(w->fp);
    const size_t index_size = w->layers.size() * sizeof(jinf_nvmw_layer_desc) +
                              w->entries.size() * sizeof(jinf_nvmw_tensor_entry);
    jinf_nvmw_header& h = w->header;
    h.magic = JINF_NVMW_MAGIC;
    if (h.version == 0) h.version = JINF_NVMW_VERSION;
    h.n_tensors = (uint32_t)w->entries.size();
    h.index_offset = 4096;
    h.index_size = index_size;
    h.hot_offset = JINF_ALIGN_4K(4096 + index_size);
    if (fwrite(&h, sizeof h, 1, w->fp) != 1) return JINF_ERR_IO;
    if (!w->layers.empty() &&
        fwrite(w->layers.data(), sizeof(jinf_nvmw_layer_desc), w->layers.size(), w->fp) != w->layers.size())
        return JINF_ERR_IO;
    if (!w->entries.empty() &&
        fwrite(w->entries.data(), sizeof(jinf_nvmw_tensor_entry), w->entries.size(), w->fp) != w->entries.size())
        return JINF_ERR_IO;
    JINF_CHECK(pad_stream_4k(w->fp), "pad");
    fflush(w->fp);
    return JINF_OK;
}

extern "C" jinf_status jinf_nvmw_writer_write_bundle_section(jinf_nvmw_writer* w,
                                                            const jinf_nvmw_bundle_header* bh,
                                                            const jinf_nvmw_bundle_layer_desc* descs,
                                                            int n_layers) {
    if (!w || !w->fp || !bh || !descs || n_layers < 0) return JINF_ERR_INVALID;
    JINF_CHECK(pad_stream_4k(w->fp), "pad");
    const long pos = ftell(w->fp);
    if (fwrite(bh, sizeof *bh, 1, w->fp) != 1) return JINF_ERR_IO;
    if (n_layers && fwrite(descs, sizeof *descs, (size_t)n_layers, w->fp) != (size_t)n_layers)
        return JINF_ERR_IO;
    // Record the index position and the bundled version in the header on disk.
    w->header.bundle_index_offset = (uint64_t)pos;
    w->header.version = JINF_NVMW_VERSION_BUNDLED;
    const long end = ftell(w->fp);
    fseek(w->fp, 0, SEEK_SET);
    if (fwrite(&w->header, sizeof w->header, 1, w->fp) != 1) return JINF_ERR_IO;
    fseek(w->fp, end, SEEK_SET);
    return JINF_OK;
}

extern "C" jinf_status jinf_nvmw_open(jinf_nvmw_reader** r, const char* path) {
    if (!r || !path) return JINF_ERR_INVALID;
    FILE* fp = fopen(path, "rb");
    if (!fp) {
        JINF_LOG("cannot open %s", path);
        return JINF_ERR_IO;
    }
    jinf_nvmw_reader* rd = new jinf_nvmw_reader();
    rd->path = path;
    jinf_status st = JINF_OK;
    if (fread(&rd->header, sizeof rd->header, 1, fp) != 1) st = JINF_ERR_PARSE;
    if (st == JINF_OK && rd->header.magic != JINF_NVMW_MAGIC) {
        JINF_LOG("bad NVMW magic 0x%08X in %s", rd->header.magic, path);
        st = JINF_ERR_PARSE;
    }
    // Bound the index so a corrupt header cannot ask for absurd allocations.
    if (st == JINF_OK && (rd->header.n_layers > 100000 || rd->header.n_tensors > 10000000))
        st = JINF_ERR_PARSE;
    if (st == JINF_OK && fseek(fp, (long)rd->header.index_offset, SEEK_SET) != 0) st = JINF_ERR_PARSE;
    if (st == JINF_OK) {
        rd->layers.resize(rd->header.n_layers);
        rd->entries.resize(rd->header.n_tensors);
        if (rd->header.n_layers &&
            fread(rd->layers.data(), sizeof(jinf_nvmw_layer_desc), rd->layers.size(), fp) != rd->layers.size())
            st = JINF_ERR_PARSE;
        if (st == JINF_OK && rd->header.n_tensors &&
            fread(rd->entries.data(), sizeof(jinf_nvmw_tensor_entry), rd->entries.size(), fp) != rd->entries.size())
            st = JINF_ERR_PARSE;
    }
    if (st == JINF_OK && rd->header.bundle_index_offset != 0) {
        if (fseek(fp, (long)rd->header.bundle_index_offset, SEEK_SET) == 0 &&
            fread(&rd->bundle_header, sizeof rd->bundle_header, 1, fp) == 1 &&
            rd->bundle_header.n_bundle_layers <= 100000) {
            rd->bundle_layers.resize(rd->bundle_header.n_bundle_layers);
            rd->has_bundles = rd->bundle_layers.empty() ||
                              fread(rd->bundle_layers.data(), sizeof(jinf_nvmw_bundle_layer_desc),
                                    rd->bundle_layers.size(), fp) == rd->bundle_layers.size();
            if (!rd->has_bundles) rd->bundle_layers.clear();
        }
    }
    fclose(fp);
    if (st != JINF_OK) {
        delete rd;
        return st;
    }
    *r = rd;
    return JINF_OK;
}

extern "C" void jinf_nvmw_close(jinf_nvmw_reader* r) { delete r; }

extern "C" const jinf_nvmw_header* jinf_nvmw_get_header(const jinf_nvmw_reader* r) {
    return r ? &r->header : nullptr;
}

extern "C" const jinf_nvmw_layer_desc* jinf_nvmw_get_layer_desc(const jinf_nvmw_reader* r, int layer) {
    if (!r || layer < 0 || (size_t)layer >= r->layers.size()) return nullptr;
    return &r->layers[(size_t)layer];
}

extern "C" const jinf_nvmw_tensor_entry* jinf_nvmw_get_tensor_entries(const jinf_nvmw_reader* r, int* count) {
    if (!r) {
        if (count) *count = 0;
        return nullptr;
    }
    if (count) *count = (int)r->entries.size();
    return r->entries.data();
}

extern "C" jinf_status jinf_nvmw_get_layer_cold_range(const jinf_nvmw_reader* r, int layer,
                                                     uint64_t* offset, uint64_t* size) {
    if (!r || !offset || !size) return JINF_ERR_INVALID;
    const jinf_nvmw_layer_desc* ld = jinf_nvmw_get_layer_desc(r, layer);
    if (!ld) return JINF_ERR_INVALID;
    *offset = ld->cold_start_offset;
    *size = ld->cold_total_size;
    return JINF_OK;
}

extern "C" jinf_status jinf_nvmw_get_hot_range(const jinf_nvmw_reader* r, uint64_t* offset, uint64_t* size) {
    if (!r || !offset || !size) return JINF_ERR_INVALID;
    *offset = r->header.hot_offset;
    *size = r->header.hot_size;
    return JINF_OK;
}

extern "C" const jinf_nvmw_tensor_entry* jinf_nvmw_find_tensor(const jinf_nvmw_reader* r, const char* name) {
    if (!r || !name) return nullptr;
    for (const auto& te : r->entries)
        if (strncmp(te.name, name, sizeof te.name) == 0) return &te;
    return nullptr;
}

extern "C" bool jinf_nvmw_has_bundles(const jinf_nvmw_reader* r) { return r && r->has_bundles; }

extern "C" const jinf_nvmw_bundle_header* jinf_nvmw_get_bundle_header(const jinf_nvmw_reader* r) {
    return r && r->has_bundles ? &r->bundle_header : nullptr;
}

extern "C" const jinf_nvmw_bundle_layer_desc* jinf_nvmw_get_bundle_layer_desc(const jinf_nvmw_reader* r, int layer) {
    if (!r || !r->has_bundles || layer < 0 || (size_t)layer >= r->bundle_layers.size()) return nullptr;
    return &r->bundle_layers[(size_t)layer];
}

extern "C" uint64_t jinf_nvmw_get_neuron_bundle_offset(const jinf_nvmw_reader* r, int layer, int neuron_id) {
    const jinf_nvmw_bundle_layer_desc* d = jinf_nvmw_get_bundle_layer_desc(r, layer);
    return d ? d->bundles_offset + (uint64_t)neuron_id * d->bundle_size : 0;
}

extern "C" uint64_t jinf_nvmw_tensor_file_offset(const jinf_nvmw_reader* r, const jinf_nvmw_tensor_entry* te) {
    if (!r || !te) return 0;
    if (te->is_hot) return r->header.hot_offset + te->offset;
    const jinf_nvmw_layer_desc* ld = jinf_nvmw_get_layer_desc(r, te->layer_index);
    return ld ? ld->cold_start_offset + te->offset : 0;
}

extern "C" const char* jinf_nvmw_get_path(const jinf_nvmw_reader* r) { return r ? r->path.c_str() : nullptr; }
