// GGUF v2/v3 reader and a minimal v3 writer.
//
// Reader behaviour follows reference src/gguf.cpp:143-311: scalar and string KVs are
// kept, array KVs are skipped (their element type and count recorded), the data
// section starts at the next `general.alignment` boundary (default 32), and the
// Llama hyper-parameters are read from "<arch>.*" keys with the reference's defaults
// (n_heads_kv := n_heads, n_vocab from token_embd when the key is missing).
#include "jinf/gguf.h"

#include <errno.h>
#include <stdlib.h>
#include <string.h>
#include <string>
#include <vector>

namespace {

struct Reader {
    FILE* fp;
    bool ok = true;
    template <class T> T get() {
        T v{};
        if (ok && fread(&v, sizeof v, 1, fp) != 1) ok = false;
        return v;
    }
    char* str() {
        const uint64_t n = get<uint64_t>();
        if (!ok || n > (1u << 20)) { ok = false; return nullptr; }
        char* s = (char*)malloc(n + 1);
        if (!s || (n && fread(s, 1, n, fp) != n)) { free(s); ok = false; return nullptr; }
        s[n] = 0;
        return s;
    }
    bool skip(uint64_t n) { return ok = ok && fseek(fp, (long)n, SEEK_CUR) == 0; }
};

int scalar_size(uint32_t t) {
    switch (t) {
        case JINF_GGUF_TYPE_UINT8: case JINF_GGUF_TYPE_INT8: case JINF_GGUF_TYPE_BOOL: return 1;
        case JINF_GGUF_TYPE_UINT16: case JINF_GGUF_TYPE_INT16: return 2;
        case JINF_GGUF_TYPE_UINT32: case JINF_GGUF_TYPE_INT32: case JINF_GGUF_TYPE_FLOAT32: return 4;
        case JINF_GGUF_TYPE_UINT64: case JINF_GGUF_TYPE_INT64: case JINF_GGUF_TYPE_FLOAT64: return 8;
        default: return 0;
    }
}

bool skip_value(Reader& rd, uint32_t type, int depth) {
    if (depth > 4) return false;
    if (int sz = scalar_size(type)) return rd.skip((uint64_t)sz);
    if (type == JINF_GGUF_TYPE_STRING) {
        const uint64_t n = rd.get<uint64_t>();
        return rd.ok && rd.skip(n);
    }
    if (type == JINF_GGUF_TYPE_ARRAY) {
        const uint32_t et = rd.get<uint32_t>();
        const uint64_t cnt = rd.get<uint64_t>();
        if (!rd.ok) return false;
        if (int sz = scalar_size(et)) return rd.skip((uint64_t)sz * cnt);
        for (uint64_t i = 0; i < cnt; ++i)
            if (!skip_value(rd, et, depth + 1)) return false;
        return true;
    }
    return false;
}

bool read_kv(Reader& rd, jinf_gguf_kv* kv) {
    kv->key = rd.str();
    if (!rd.ok) return false;
    const uint32_t t = rd.get<uint32_t>();
    if (!rd.ok) return false;
    kv->type = (jinf_gguf_value_type)t;
    switch (t) {
        case JINF_GGUF_TYPE_UINT8:   kv->val_u8 = rd.get<uint8_t>(); break;
        case JINF_GGUF_TYPE_INT8:    kv->val_i8 = rd.get<int8_t>(); break;
        case JINF_GGUF_TYPE_UINT16:  kv->val_u16 = rd.get<uint16_t>(); break;
        case JINF_GGUF_TYPE_INT16:   kv->val_i16 = rd.get<int16_t>(); break;
        case JINF_GGUF_TYPE_UINT32:  kv->val_u32 = rd.get<uint32_t>(); break;
        case JINF_GGUF_TYPE_INT32:   kv->val_i32 = rd.get<int32_t>(); break;
        case JINF_GGUF_TYPE_FLOAT32: kv->val_f32 = rd.get<float>(); break;
        case JINF_GGUF_TYPE_BOOL:    kv->val_bool = rd.get<uint8_t>() != 0; break;
        case JINF_GGUF_TYPE_UINT64:  kv->val_u64 = rd.get<uint64_t>(); break;
        case JINF_GGUF_TYPE_INT64:   kv->val_i64 = rd.get<int64_t>(); break;
        case JINF_GGUF_TYPE_FLOAT64: kv->val_f64 = rd.get<double>(); break;
        case JINF_GGUF_TYPE_STRING: {
            // length is re-derived from the string itself
            kv->val_str.data = rd.str();
            kv->val_str.length = kv->val_str.data ? strlen(kv->val_str.data) : 0;
            break;
        }
        case JINF_GGUF_TYPE_ARRAY: {
            const uint32_t et = rd.get<uint32_t>();
            const uint64_t cnt = rd.get<uint64_t>();
            kv->val_arr.elem_type = (jinf_gguf_value_type)et;
            kv->val_arr.count = cnt;
            kv->val_arr.data = nullptr;
            if (!rd.ok) return false;
            if (int sz = scalar_size(et)) return rd.skip((uint64_t)sz * cnt);
            for (uint64_t i = 0; i < cnt; ++i)
                if (!skip_value(rd, et, 1)) return false;
            break;
        }
        default: return false;
    }
    return rd.ok;
}

jinf_qtype map_type(uint32_t t) {
    switch (t) {
        case 0: case 1: case 2: case 3: case 6: case 7: case 8: case 9:
        case 10: case 11: case 12: case 13: case 14: case 15: return (jinf_qtype)t;
        default: return JINF_TYPE_F32;  // the reference maps unknown ids to F32
    }
}

}  // namespace

extern "C" void jinf_gguf_close(jinf_gguf_file* f) {
    if (!f) return;
    if (f->kvs) {
        for (uint64_t i = 0; i < f->kv_count; ++i) {
            free(f->kvs[i].key);
            if (f->kvs[i].type == JINF_GGUF_TYPE_STRING) free(f->kvs[i].val_str.data);
        }
        free(f->kvs);
    }
    if (f->tensor_infos) {
        for (uint64_t i = 0; i < f->tensor_count; ++i) free(f->tensor_infos[i].name);
        free(f->tensor_infos);
    }
    free(f);
}

extern "C" const jinf_gguf_kv* jinf_gguf_find_kv(const jinf_gguf_file* f, const char* key) {
    if (!f || !key) return nullptr;
    for (uint64_t i = 0; i < f->kv_count; ++i)
        if (f->kvs[i].key && strcmp(f->kvs[i].key, key) == 0) return &f->kvs[i];
    return nullptr;
}

extern "C" const jinf_gguf_tensor_info* jinf_gguf_find_tensor(const jinf_gguf_file* f, const char* name) {
    if (!f || !name) return nullptr;
    for (uint64_t i = 0; i < f->tensor_count; ++i)
        if (f->tensor_infos[i].name && strcmp(f->tensor_infos[i].name, name) == 0) return &f->tensor_infos[i];
    return nullptr;
}

extern "C" const char* jinf_gguf_get_str(const jinf_gguf_file* f, const char* key, const char* def) {
    const jinf_gguf_kv* kv = jinf_gguf_find_kv(f, key);
    return kv && kv->type == JINF_GGUF_TYPE_STRING && kv->val_str.data ? kv->val_str.data : def;
}

extern "C" uint32_t jinf_gguf_get_u32(const jinf_gguf_file* f, const char* key, uint32_t def) {
    const jinf_gguf_kv* kv = jinf_gguf_find_kv(f, key);
    if (!kv) return def;
    switch (kv->type) {
        case JINF_GGUF_TYPE_UINT32:  return kv->val_u32;
        case JINF_GGUF_TYPE_INT32:   return (uint32_t)kv->val_i32;
        case JINF_GGUF_TYPE_UINT64:  return (uint32_t)kv->val_u64;
        case JINF_GGUF_TYPE_INT64:   return (uint32_t)kv->val_i64;
        case JINF_GGUF_TYPE_FLOAT32: return (uint32_t)kv->val_f32;
        default: return def;
    }
}

extern "C" float jinf_gguf_get_f32(const jinf_gguf_file* f, const char* key, float def) {
    const jinf_gguf_kv* kv = jinf_gguf_find_kv(f, key);
    if (!kv) return def;
    switch (kv->type) {
        case JINF_GGUF_TYPE_FLOAT32: return kv->val_f32;
        case JINF_GGUF_TYPE_FLOAT64: return (float)kv->val_f64;
        case JINF_GGUF_TYPE_UINT32:  return (float)kv->val_u32;
        case JINF_GGUF_TYPE_INT32:   return (float)kv->val_i32;
        default: return def;
    }
}

extern "C" jinf_status jinf_gguf_open(jinf_gguf_file** out, const char* path) {
    if (!out || !path) return JINF_ERR_INVALID;
    FILE* fp = fopen(path, "rb");
    if (!fp) {
        JINF_LOG("cannot open %s: %s", path, strerror(errno));
        return JINF_ERR_IO;
    }
    Reader rd{fp};
    const uint32_t magic = rd.get<uint32_t>();
    const uint32_t version = rd.get<uint32_t>();
    if (!rd.ok || magic != JINF_GGUF_MAGIC) {
        JINF_LOG("not a GGUF file: %s", path);
        fclose(fp);
        return JINF_ERR_PARSE;
    }
    if (version != JINF_GGUF_VERSION_2 && version != JINF_GGUF_VERSION_3) {
        JINF_LOG("unsupported GGUF version %u", version);
        fclose(fp);
        return JINF_ERR_PARSE;
    }
    const uint64_t n_tensors = rd.get<uint64_t>();
    const uint64_t n_kv = rd.get<uint64_t>();
    if (!rd.ok || n_tensors > (1u << 24) || n_kv > (1u << 24)) {
        fclose(fp);
        return JINF_ERR_PARSE;
    }
    jinf_gguf_file* gf = (jinf_gguf_file*)calloc(1, sizeof(jinf_gguf_file));
    if (!gf) { fclose(fp); return JINF_ERR_OOM; }
    gf->version = version;
    gf->alignment = JINF_GGUF_DEFAULT_ALIGNMENT;
    gf->kvs = (jinf_gguf_kv*)calloc(n_kv ? n_kv : 1, sizeof(jinf_gguf_kv));
    gf->tensor_infos = (jinf_gguf_tensor_info*)calloc(n_tensors ? n_tensors : 1, sizeof(jinf_gguf_tensor_info));
    if (!gf->kvs || !gf->tensor_infos) { jinf_gguf_close(gf); fclose(fp); return JINF_ERR_OOM; }
    gf->kv_count = n_kv;
    gf->tensor_count = n_tensors;
    for (uint64_t i = 0; i < n_kv; ++i) {
        if (!read_kv(rd, &gf->kvs[i])) {
            JINF_LOG("GGUF: bad KV %llu", (unsigned long long)i);
            jinf_gguf_close(gf);
            fclose(fp);
            return JINF_ERR_PARSE;
        }
        if (gf->kvs[i].key && strcmp(gf->kvs[i].key, "general.alignment") == 0 &&
            gf->kvs[i].type == JINF_GGUF_TYPE_UINT32 && gf->kvs[i].val_u32 > 0)
            gf->alignment = gf->kvs[i].val_u32;
    }
    for (uint64_t i = 0; i < n_tensors; ++i) {
        jinf_gguf_tensor_info* ti = &gf->tensor_infos[i];
        ti->name = rd.str();
        ti->n_dims = rd.get<uint32_t>();
        if (!rd.ok || ti->n_dims > 4) {
            jinf_gguf_close(gf);
            fclose(fp);
            return JINF_ERR_PARSE;
        }
        ti->n_elements = 1;  // dims past n_dims stay 0, as in the reference's parser
        for (uint32_t d = 0; d < ti->n_dims; ++d) {
            ti->shape[d] = rd.get<int64_t>();
            ti->n_elements *= ti->shape[d];
        }
        ti->type = map_type(rd.get<uint32_t>());
        ti->offset = rd.get<uint64_t>();
        if (!rd.ok) {
            jinf_gguf_close(gf);
            fclose(fp);
            return JINF_ERR_PARSE;
        }
        ti->n_bytes = jinf_tensor_nbytes(ti->type, ti->n_elements);
    }
    const long pos = ftell(fp);
    fclose(fp);
    gf->data_offset = ((size_t)pos + gf->alignment - 1) / gf->alignment * gf->alignment;

    jinf_model_hparams* hp = &gf->hparams;
    memset(hp, 0, sizeof *hp);
    strncpy(hp->arch, jinf_gguf_get_str(gf, "general.architecture", "llama"), sizeof hp->arch - 1);
    const std::string p = std::string(hp->arch) + ".";
    hp->n_layers = jinf_gguf_get_u32(gf, (p + "block_count").c_str(), 0);
    hp->n_embd = jinf_gguf_get_u32(gf, (p + "embedding_length").c_str(), 0);
    hp->n_heads = jinf_gguf_get_u32(gf, (p + "attention.head_count").c_str(), 0);
    hp->n_heads_kv = jinf_gguf_get_u32(gf, (p + "attention.head_count_kv").c_str(), 0);
    hp->n_ff = jinf_gguf_get_u32(gf, (p + "feed_forward_length").c_str(), 0);
    hp->n_vocab = jinf_gguf_get_u32(gf, (p + "vocab_size").c_str(), 0);
    hp->n_ctx_train = jinf_gguf_get_u32(gf, (p + "context_length").c_str(), 2048);
    hp->rope_freq_base = jinf_gguf_get_f32(gf, (p + "rope.freq_base").c_str(), 10000.0f);
    hp->rms_norm_eps = jinf_gguf_get_f32(gf, (p + "attention.layer_norm_rms_epsilon").c_str(), 1e-5f);
    if (hp->n_heads_kv == 0) hp->n_heads_kv = hp->n_heads;
    if (hp->n_vocab == 0) {
        const jinf_gguf_tensor_info* e = jinf_gguf_find_tensor(gf, "token_embd.weight");
        if (e && e->n_dims >= 2) hp->n_vocab = (uint32_t)e->shape[1];
    }
    *out = gf;
    return JINF_OK;
}

// ---- writer ----

struct jinf_gguf_writer {
    std::string path;
    std::vector<uint8_t> kv_bytes;
    uint64_t n_kv = 0;
    struct T { std::string name; int n_dims; int64_t shape[4]; uint32_t type; std::vector<uint8_t> data; };
    std::vector<T> tensors;
    void put(const void* p, size_t n) {
        const uint8_t* b = (const uint8_t*)p;
        kv_bytes.insert(kv_bytes.end(), b, b + n);
    }
    void put_str(const char* s) {
        const uint64_t n = strlen(s);
        put(&n, 8);
        put(s, n);
    }
};

extern "C" jinf_status jinf_gguf_writer_create(jinf_gguf_writer** w, const char* path) {
    if (!w || !path) return JINF_ERR_INVALID;
    *w = new jinf_gguf_writer();
    (*w)->path = path;
    return JINF_OK;
}

extern "C" jinf_status jinf_gguf_writer_add_kv_u32(jinf_gguf_writer* w, const char* key, uint32_t v) {
    if (!w || !key) return JINF_ERR_INVALID;
    const uint32_t t = JINF_GGUF_TYPE_UINT32;
    w->put_str(key); w->put(&t, 4); w->put(&v, 4); ++w->n_kv;
    return JINF_OK;
}

extern "C" jinf_status jinf_gguf_writer_add_kv_f32(jinf_gguf_writer* w, const char* key, float v) {
    if (!w || !key) return JINF_ERR_INVALID;
    const uint32_t t = JINF_GGUF_TYPE_FLOAT32;
    w->put_str(key); w->put(&t, 4); w->put(&v, 4); ++w->n_kv;
    return JINF_OK;
}

extern "C" jinf_status jinf_gguf_writer_add_kv_str(jinf_gguf_writer* w, const char* key, const char* v) {
    if (!w || !key || !v) return JINF_ERR_INVALID;
    const uint32_t t = JINF_GGUF_TYPE_STRING;
    w->put_str(key); w->put(&t, 4); w->put_str(v); ++w->n_kv;
    return JINF_OK;
}

extern "C" jinf_status jinf_gguf_writer_add_tensor(jinf_gguf_writer* w, const char* name, int n_dims,
                                                  const int64_t* shape, jinf_qtype type,
                                                  const void* data, size_t n_bytes) {
    if (!w || !name || !shape || n_dims < 1 || n_dims > 4 || (!data && n_bytes)) return JINF_ERR_INVALID;
    jinf_gguf_writer::T t;
    t.name = name;
    t.n_dims = n_dims;
    for (int i = 0; i < 4; ++i) t.shape[i] = i < n_dims ? shape[i] : 1;
    t.type = (uint32_t)type;
    t.data.assign((const uint8_t*)data, (const uint8_t*)data + n_bytes);
    w->tensors.push_back(std::move(t));
    return JINF_OK;
}

extern "C" jinf_status jinf_gguf_writer_finish(jinf_gguf_writer* w) {
    if (!w) return JINF_ERR_INVALID;
    FILE* fp = fopen(w->path.c_str(), "wb");
    if (!fp) { delete w; return JINF_ERR_IO; }
    const uint32_t align = JINF_GGUF_DEFAULT_ALIGNMENT;
    bool ok = true;
    auto put = [&](const void* p, size_t n) { ok = ok && fwrite(p, 1, n, fp) == n; };
    const uint32_t magic = JINF_GGUF_MAGIC, version = 3;
    const uint64_t nt = w->tensors.size();
    put(&magic, 4); put(&version, 4); put(&nt, 8); put(&w->n_kv, 8);
    put(w->kv_bytes.data(), w->kv_bytes.size());
    uint64_t off = 0;
    for (auto& t : w->tensors) {
        const uint64_t n = t.name.size();
        put(&n, 8); put(t.name.data(), n);
        const uint32_t nd = (uint32_t)t.n_dims;
        put(&nd, 4);
        put(t.shape, 8 * (size_t)t.n_dims);
        put(&t.type, 4);
        put(&off, 8);
        off += (t.data.size() + align - 1) / align * align;
    }
    static const uint8_t zeros[64] = {0};
    long pos = ftell(fp);
    put(zeros, (size_t)((align - (uint64_t)pos % align) % align));
    for (auto& t : w->tensors) {
        put(t.data.data(), t.data.size());
        put(zeros, (size_t)((align - t.data.size() % align) % align));
    }
    fclose(fp);
    delete w;
    return ok ? JINF_OK : JINF_ERR_IO;
}
