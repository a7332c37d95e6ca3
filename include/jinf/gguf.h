// jinf-b200: GGUF v2/v3 reader (and a writer for synthetic models).
//
// Drop-in for reference include/jinf/gguf.h. The in-memory structs keep the
// reference's field names and types, because callers (the splitter and its tests,
// reference tests/test_splitter.cpp:13-74) build jinf_gguf_file values by hand.
// Array-valued KVs are skipped on read, as the reference does (reference src/gguf.cpp:100-113).
#pragma once

#include "jinf/common.h"
#include "jinf/quant.h"

#define JINF_GGUF_MAGIC             0x46554747u  // "GGUF"
#define JINF_GGUF_VERSION_2         2
#define JINF_GGUF_VERSION_3         3
#define JINF_GGUF_DEFAULT_ALIGNMENT 32

enum jinf_gguf_value_type
#ifdef __cplusplus
    : int
#endif
{
    JINF_GGUF_TYPE_UINT8   = 0,
    JINF_GGUF_TYPE_INT8    = 1,
    JINF_GGUF_TYPE_UINT16  = 2,
    JINF_GGUF_TYPE_INT16   = 3,
    JINF_GGUF_TYPE_UINT32  = 4,
    JINF_GGUF_TYPE_INT32   = 5,
    JINF_GGUF_TYPE_FLOAT32 = 6,
    JINF_GGUF_TYPE_BOOL    = 7,
    JINF_GGUF_TYPE_STRING  = 8,
    JINF_GGUF_TYPE_ARRAY   = 9,
    JINF_GGUF_TYPE_UINT64  = 10,
    JINF_GGUF_TYPE_INT64   = 11,
    JINF_GGUF_TYPE_FLOAT64 = 12,
};
#ifndef __cplusplus
typedef enum jinf_gguf_value_type jinf_gguf_value_type;
#endif

typedef struct jinf_gguf_kv {
    char*                key;
    jinf_gguf_value_type type;
    union {
        uint8_t  val_u8;
        int8_t   val_i8;
        uint16_t val_u16;
        int16_t  val_i16;
        uint32_t val_u32;
        int32_t  val_i32;
        float    val_f32;
        bool     val_bool;
        uint64_t val_u64;
        int64_t  val_i64;
        double   val_f64;
        struct { char* data; uint64_t length; } val_str;
        struct { jinf_gguf_value_type elem_type; uint64_t count; void* data; } val_arr;
    };
} jinf_gguf_kv;

typedef struct jinf_gguf_tensor_info {
    char*      name;
    uint32_t   n_dims;
    int64_t    shape[4];    // shape[0] is the fastest-varying dimension (ggml ne0)
    jinf_qtype type;
    uint64_t   offset;      // relative to the data section
    int64_t    n_elements;
    size_t     n_bytes;
} jinf_gguf_tensor_info;

typedef struct jinf_model_hparams {
    char     arch[64];
    uint32_t n_layers;
    uint32_t n_embd;
    uint32_t n_heads;
    uint32_t n_heads_kv;
    uint32_t n_ff;
    uint32_t n_vocab;
    uint32_t n_ctx_train;
    float    rope_freq_base;
    float    rms_norm_eps;
} jinf_model_hparams;

typedef struct jinf_gguf_file {
    uint32_t               version;
    uint64_t               tensor_count;
    uint64_t               kv_count;
    uint32_t               alignment;
    jinf_gguf_kv*          kvs;
    jinf_gguf_tensor_info* tensor_infos;
    size_t                 data_offset;  // absolute file offset of the data section
    jinf_model_hparams     hparams;
} jinf_gguf_file;

#ifdef __cplusplus
extern "C" {
#endif

// Parse header, KVs and tensor infos (reference src/gguf.cpp:143-311). On failure
// *file is left untouched and an error status is returned.
jinf_status jinf_gguf_open(jinf_gguf_file** file, const char* path);
void        jinf_gguf_close(jinf_gguf_file* file);

const jinf_gguf_kv*          jinf_gguf_find_kv(const jinf_gguf_file* file, const char* key);
const jinf_gguf_tensor_info* jinf_gguf_find_tensor(const jinf_gguf_file* file, const char* name);
const char* jinf_gguf_get_str(const jinf_gguf_file* file, const char* key, const char* def);
uint32_t    jinf_gguf_get_u32(const jinf_gguf_file* file, const char* key, uint32_t def);
float       jinf_gguf_get_f32(const jinf_gguf_file* file, const char* key, float def);

// ---- New: GGUF v3 writer (used to emit synthetic Llama models) ----
typedef struct jinf_gguf_writer jinf_gguf_writer;
jinf_status jinf_gguf_writer_create(jinf_gguf_writer** w, const char* path);
jinf_status jinf_gguf_writer_add_kv_u32(jinf_gguf_writer* w, const char* key, uint32_t v);
jinf_status jinf_gguf_writer_add_kv_f32(jinf_gguf_writer* w, const char* key, float v);
jinf_status jinf_gguf_writer_add_kv_str(jinf_gguf_writer* w, const char* key, const char* v);
// `shape` uses ggml order (shape[0] fastest). The data is copied when the file is finished.
jinf_status jinf_gguf_writer_add_tensor(jinf_gguf_writer* w, const char* name, int n_dims,
                                        const int64_t* shape, jinf_qtype type,
                                        const void* data, size_t n_bytes);
jinf_status jinf_gguf_writer_finish(jinf_gguf_writer* w);  // writes and frees the writer

#ifdef __cplusplus
}
#endif
