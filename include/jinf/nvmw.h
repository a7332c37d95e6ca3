// jinf-b200: the .nvmw model container (reader and writer).
//
// Drop-in for reference include/jinf/nvmw.h. The on-disk structs keep the
// reference's exact byte layouts (reference include/jinf/nvmw.h:25-103), so files
// written by the reference's tools/prepare_model open here and vice versa:
//   [4 KB header][layer descs + tensor entries][hot region (4K aligned)]
//   [cold layer regions (4K aligned)][optional v2 bundle section + bundle index]
// On B200 every region is loaded into HBM; "cold" only describes the file layout.
#pragma once

#include "jinf/common.h"
#include "jinf/quant.h"

#define JINF_NVMW_MAGIC           0x574D564Eu  // "NVMW"
#define JINF_NVMW_VERSION         1
#define JINF_NVMW_VERSION_BUNDLED 2
// New (no counterpart in the reference): the B200 layout, projections pre-packed into the
// engine's Q4M images (jinf_prepare_model_b200); such a tensor's type is
// JINF_NVMW_TYPE_Q4M + its Q4M format (0 Q4_0, 1 Q4_K, 2 Q6_K, 3 Q8_0).
#define JINF_NVMW_VERSION_B200    3
#define JINF_NVMW_TYPE_Q4M        0x40
static inline int q4m_format_of_qtype(int qtype) {
    return qtype == 2 ? 0 : qtype == 12 ? 1 : qtype == 14 ? 2 : qtype == 8 ? 3 : -1;
}
static inline int qtype_of_q4m_format(int fmt) { return fmt == 0 ? 2 : fmt == 1 ? 12 : fmt == 2 ? 14 : fmt == 3 ? 8 : -1; }

// Tensor entry: natural (unpacked) alignment, 200 bytes.
typedef struct jinf_nvmw_tensor_entry {
    char       name[128];
    jinf_qtype type;
    int64_t    shape[4];
    uint32_t   n_dims;
    uint64_t   offset;       // hot: from the hot region start; cold: from the layer's cold start
    uint64_t   n_bytes;
    int32_t    layer_index;  // -1 for non-layer tensors
    uint8_t    is_hot;
    uint8_t    _pad[3];
} jinf_nvmw_tensor_entry;

typedef struct jinf_nvmw_layer_desc {
    uint64_t cold_start_offset;  // absolute file offset
    uint64_t cold_total_size;
    uint32_t n_cold_tensors;
    uint32_t _pad;
} jinf_nvmw_layer_desc;

#pragma pack(push, 1)
typedef struct jinf_nvmw_bundle_header {
    uint32_t n_bundle_layers;
    uint32_t bundle_size;  // bytes per neuron bundle (4K padded)
    uint32_t n_ff;
    uint32_t _pad;
} jinf_nvmw_bundle_header;

typedef struct jinf_nvmw_bundle_layer_desc {
    uint64_t bundles_offset;      // absolute file offset of this layer's bundles
    uint64_t bundles_total_size;  // n_ff * bundle_size
    uint32_t n_neurons;
    uint32_t bundle_size;
} jinf_nvmw_bundle_layer_desc;

typedef struct jinf_nvmw_header {
    uint32_t magic;
    uint32_t version;
    uint32_t n_layers;
    uint32_t n_tensors;
    uint64_t index_offset;
    uint64_t index_size;
    uint64_t hot_offset;
    uint64_t hot_size;
    uint64_t cold_start_offset;
    uint64_t cold_total_size;
    uint32_t n_embd;
    uint32_t n_heads;
    uint32_t n_heads_kv;
    uint32_t n_ff;
    uint32_t n_vocab;
    uint32_t n_ctx_train;
    float    rope_freq_base;
    float    rms_norm_eps;
    int32_t  primary_type;
    uint32_t _pad0;
    uint64_t bundle_index_offset;  // 0 = no bundle section
    uint8_t  _reserved[4096 - 112];
} jinf_nvmw_header;
#pragma pack(pop)

#ifdef __cplusplus
static_assert(sizeof(jinf_nvmw_tensor_entry) == 200, "tensor entry layout");
static_assert(offsetof(jinf_nvmw_tensor_entry, shape) == 136, "tensor entry layout");
static_assert(offsetof(jinf_nvmw_tensor_entry, offset) == 176, "tensor entry layout");
static_assert(offsetof(jinf_nvmw_tensor_entry, layer_index) == 192, "tensor entry layout");
static_assert(sizeof(jinf_nvmw_layer_desc) == 24, "layer desc layout");
static_assert(sizeof(jinf_nvmw_bundle_header) == 16, "bundle header layout");
static_assert(sizeof(jinf_nvmw_bundle_layer_desc) == 24, "bundle layer desc layout");
static_assert(sizeof(jinf_nvmw_header) == 4096, "NVMW header must be 4 KB");
#endif

typedef struct jinf_nvmw_reader jinf_nvmw_reader;
typedef struct jinf_nvmw_writer jinf_nvmw_writer;

#ifdef __cplusplus
extern "C" {
#endif

// ---- Writer (reference src/nvmw.cpp:10-164) ----
// Usage as in the reference's prepare_model: set header, add layer descs and tensor
// entries, finalize (writes header + index and leaves the file positioned at the
// hot region), then write region bytes.
jinf_status jinf_nvmw_writer_create(jinf_nvmw_writer** w, const char* path);
void        jinf_nvmw_writer_destroy(jinf_nvmw_writer* w);
jinf_status jinf_nvmw_writer_set_header(jinf_nvmw_writer* w, const jinf_nvmw_header* hdr);
jinf_status jinf_nvmw_writer_add_layer_desc(jinf_nvmw_writer* w, int layer, const jinf_nvmw_layer_desc* desc);
jinf_status jinf_nvmw_writer_add_tensor_entry(jinf_nvmw_writer* w, const jinf_nvmw_tensor_entry* entry);
jinf_status jinf_nvmw_writer_write_hot(jinf_nvmw_writer* w, const void* data, size_t size);
jinf_status jinf_nvmw_writer_write_cold_layer(jinf_nvmw_writer* w, int layer, const void* data, size_t size);
jinf_status jinf_nvmw_writer_finalize(jinf_nvmw_writer* w);

// GGUF -> NVMW conversion as the reference's tools/prepare_model writes it (the same file,
// byte for byte): the split plan for `gpu_budget_mb`, hot and per-layer cold tensors 4 KB
// padded, and with `bundled` the neuron bundles (gate row, up row, fp32 down column) and
// their index (version 2). New: the reference has it only as a command-line tool.
jinf_status jinf_prepare_model(const char* gguf_path, const char* nvmw_path, size_t gpu_budget_mb, int bundled);
// GGUF -> B200-layout NVMW (version 3) for one GPU and the dense FFN: every projection stored
// as the engine's fused Q4M image (qkv, o, gate|up interleaved, down, output head), so the
// engine copies it into HBM without repacking; the embedding and norms as in the GGUF. New:
// no counterpart in the reference.
jinf_status jinf_prepare_model_b200(const char* gguf_path, const char* nvmw_path);
// The same for tensor parallelism over tp_size GPUs (1, 2, 4 or 8): every rank's shard of
// every projection as an image of its own, named "tp<tp_size>.<rank>." + the one-GPU name;
// an engine created with that tp_size reads its rank's images.
jinf_status jinf_prepare_model_b200_tp(const char* gguf_path, const char* nvmw_path, int tp_size);
jinf_status jinf_nvmw_writer_write_bundle_section(jinf_nvmw_writer* w,
                                                  const jinf_nvmw_bundle_header* bh,
                                                  const jinf_nvmw_bundle_layer_desc* layer_descs,
                                                  int n_layers);

// ---- Reader (reference src/nvmw.cpp:180-313) ----
jinf_status jinf_nvmw_open(jinf_nvmw_reader** r, const char* path);
void        jinf_nvmw_close(jinf_nvmw_reader* r);
const jinf_nvmw_header*       jinf_nvmw_get_header(const jinf_nvmw_reader* r);
const jinf_nvmw_layer_desc*   jinf_nvmw_get_layer_desc(const jinf_nvmw_reader* r, int layer);
const jinf_nvmw_tensor_entry* jinf_nvmw_get_tensor_entries(const jinf_nvmw_reader* r, int* count);
jinf_status jinf_nvmw_get_layer_cold_range(const jinf_nvmw_reader* r, int layer,
                                           uint64_t* offset, uint64_t* size);
jinf_status jinf_nvmw_get_hot_range(const jinf_nvmw_reader* r, uint64_t* offset, uint64_t* size);
const jinf_nvmw_tensor_entry* jinf_nvmw_find_tensor(const jinf_nvmw_reader* r, const char* name);
bool jinf_nvmw_has_bundles(const jinf_nvmw_reader* r);
const jinf_nvmw_bundle_header*     jinf_nvmw_get_bundle_header(const jinf_nvmw_reader* r);
const jinf_nvmw_bundle_layer_desc* jinf_nvmw_get_bundle_layer_desc(const jinf_nvmw_reader* r, int layer);
uint64_t jinf_nvmw_get_neuron_bundle_offset(const jinf_nvmw_reader* r, int layer, int neuron_id);

// ---- New: absolute file offset of a tensor's bytes (hot or cold), 0 if unknown ----
uint64_t jinf_nvmw_tensor_file_offset(const jinf_nvmw_reader* r, const jinf_nvmw_tensor_entry* te);
const char* jinf_nvmw_get_path(const jinf_nvmw_reader* r);

#ifdef __cplusplus
}
#endif
