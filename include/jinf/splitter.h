// jinf-b200: hot/cold weight placement planner.
//
// Drop-in for reference include/jinf/splitter.h. Placement semantics are the
// reference's (reference src/splitter.cpp:37-157): norms, embeddings and the output
// head are always hot; the rest is promoted layer by layer, attention before FFN,
// until the budget is exhausted. On B200 the default engine budget covers the whole
// model, so every tensor ends up hot in HBM; the planner additionally reports each
// tensor's tensor-parallel split role (jinf_split_tp_role).
#pragma once

#include "jinf/common.h"
#include "jinf/gguf.h"

enum jinf_weight_placement
#ifdef __cplusplus
    : int
#endif
{
    JINF_PLACE_HOT  = 0,
    JINF_PLACE_COLD = 1,
};
#ifndef __cplusplus
typedef enum jinf_weight_placement jinf_weight_placement;
#endif

typedef struct jinf_split_config {
    size_t gpu_memory_budget;
    size_t kv_cache_budget;
    size_t buffer_budget;
} jinf_split_config;

typedef struct jinf_weight_assignment {
    const jinf_gguf_tensor_info* tensor;
    jinf_weight_placement        placement;
    int                          layer_index;  // -1 for non-layer tensors
} jinf_weight_assignment;

typedef struct jinf_split_plan {
    jinf_weight_assignment* assignments;
    int                     count;
    size_t                  total_hot_bytes;
    size_t                  total_cold_bytes;
} jinf_split_plan;

// Tensor-parallel role of a tensor (new).
enum jinf_tp_role
#ifdef __cplusplus
    : int
#endif
{
    JINF_TP_REPLICATED = 0,  // norms, embeddings
    JINF_TP_COLUMN     = 1,  // output rows split: q, k, v, gate, up, output (vocab)
    JINF_TP_ROW        = 2,  // input columns split: attn_output, ffn_down
};
#ifndef __cplusplus
typedef enum jinf_tp_role jinf_tp_role;
#endif

#ifdef __cplusplus
extern "C" {
#endif

jinf_status jinf_split_analyze(const jinf_gguf_file* model, const jinf_split_config* config,
                               jinf_split_plan** plan);
void        jinf_split_plan_free(jinf_split_plan* plan);
void        jinf_split_plan_print(const jinf_split_plan* plan);

// New: split role of a tensor by name.
jinf_tp_role jinf_split_tp_role(const char* tensor_name);
// New: the slice of a rows x cols tensor that tensor-parallel rank `rank` of `size` holds,
// from its role: JINF_TP_COLUMN tensors are split by rows, JINF_TP_ROW tensors by columns
// (whole 32-element blocks), others are whole. JINF_ERR_INVALID when the split dimension
// does not divide evenly. The engine loads each rank's weights with it.
jinf_status jinf_tp_shard(const char* name, int64_t rows, int64_t cols, int rank, int size, int64_t* row0,
                          int64_t* n_rows, int64_t* col0, int64_t* n_cols);

#ifdef __cplusplus
}
#endif
