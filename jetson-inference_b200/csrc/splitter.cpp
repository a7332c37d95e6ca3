// Hot/cold placement planner with the reference's promotion rule
// (reference src/splitter.cpp:37-157), plus the tensor-parallel role of each tensor.
#include "jinf/splitter.h"

#include <stdlib.h>
#include <string.h>
#include <algorithm>
#include <map>
#include <vector>

namespace {

enum Role { EMBED, OUTPUT, OUTPUT_NORM, ATTN_NORM, FFN_NORM, ATTN_Q, ATTN_K, ATTN_V, ATTN_OUT,
            FFN_GATE, FFN_UP, FFN_DOWN, OTHER };

Role role_of(const char* n) {
    if (!strcmp(n, "token_embd.weight")) return EMBED;
    if (!strcmp(n, "output.weight")) return OUTPUT;
    if (!strcmp(n, "output_norm.weight")) return OUTPUT_NORM;
    if (strstr(n, "attn_norm.weight")) return ATTN_NORM;
    if (strstr(n, "ffn_norm.weight")) return FFN_NORM;
    if (strstr(n, "attn_q.weight")) return ATTN_Q;
    if (strstr(n, "attn_k.weight")) return ATTN_K;
    if (strstr(n, "attn_v.weight")) return ATTN_V;
    if (strstr(n, "attn_output.weight")) return ATTN_OUT;
    if (strstr(n, "ffn_gate.weight")) return FFN_GATE;
    if (strstr(n, "ffn_up.weight")) return FFN_UP;
    if (strstr(n, "ffn_down.weight")) return FFN_DOWN;
    return OTHER;
}

int layer_of(const char* n) {
    const char* p = strstr(n, "blk.");
    return p ? atoi(p + 4) : -1;
}

}  // namespace

extern "C" jinf_tp_role jinf_split_tp_role(const char* name) {
    if (!name) return JINF_TP_REPLICATED;
    switch (role_of(name)) {
        case ATTN_Q: case ATTN_K: case ATTN_V: case FFN_GATE: case FFN_UP: case OUTPUT: return JINF_TP_COLUMN;
        case ATTN_OUT: case FFN_DOWN: return JINF_TP_ROW;
        default: return JINF_TP_REPLICATED;
    }
}

extern "C" jinf_status jinf_tp_shard(const char* name, int64_t rows, int64_t cols, int rank, int size,
                                     int64_t* row0, int64_t* n_rows, int64_t* col0, int64_t* n_cols) {
    if (!name || !row0 || !n_rows || !col0 || !n_cols || rows <= 0 || cols <= 0 || size <= 0 || rank < 0 ||
        rank >= size)
        return JINF_ERR_INVALID;
    *row0 = 0;
    *n_rows = rows;
    *col0 = 0;
    *n_cols = cols;
    switch (jinf_split_tp_role(name)) {
        case JINF_TP_COLUMN:  // output rows split evenly: every rank a contiguous slice
            if (rows % size) return JINF_ERR_INVALID;
            *n_rows = rows / size;
            *row0 = (int64_t)rank * *n_rows;
            break;
        case JINF_TP_ROW:  // input columns split evenly, on whole 32-element blocks
            if (cols % ((int64_t)size * 32)) return JINF_ERR_INVALID;
            *n_cols = cols / size;
            *col0 = (int64_t)rank * *n_cols;
            break;
        default: break;
    }
    return JINF_OK;
}

extern "C" jinf_status jinf_split_analyze(const jinf_gguf_file* model, const jinf_split_config* cfg,
                                          jinf_split_plan** out) {
    if (!model || !cfg || !out) return JINF_ERR_INVALID;
    const int n = (int)model->tensor_count;
    jinf_split_plan* plan = (jinf_split_plan*)calloc(1, sizeof(jinf_split_plan));
    if (!plan) return JINF_ERR_OOM;
    plan->assignments = (jinf_weight_assignment*)calloc(n > 0 ? n : 1, sizeof(jinf_weight_assignment));
    if (!plan->assignments) { free(plan); return JINF_ERR_OOM; }
    plan->count = n;

    size_t hot = 0, cold = 0;
    // Phase 1: norms, embeddings and the output head are always hot; everything else starts cold.
    struct Group { size_t attn_bytes = 0, ffn_bytes = 0; std::vector<int> attn, ffn; };
    std::map<int, Group> layers;  // ordered by layer index
    for (int i = 0; i < n; ++i) {
        const jinf_gguf_tensor_info* t = &model->tensor_infos[i];
        const Role r = role_of(t->name);
        jinf_weight_assignment& a = plan->assignments[i];
        a.tensor = t;
        a.layer_index = layer_of(t->name);
        if (r == EMBED || r == OUTPUT || r == OUTPUT_NORM || r == ATTN_NORM || r == FFN_NORM) {
            a.placement = JINF_PLACE_HOT;
            hot += t->n_bytes;
            continue;
        }
        a.placement = JINF_PLACE_COLD;
        cold += t->n_bytes;
        if (a.layer_index < 0) continue;
        Group& g = layers[a.layer_index];
        if (r >= ATTN_Q && r <= ATTN_OUT) { g.attn.push_back(i); g.attn_bytes += t->n_bytes; }
        else { g.ffn.push_back(i); g.ffn_bytes += t->n_bytes; }
    }
    // Phase 2: promote layer by layer, attention before FFN. The walk ends at the first
    // layer whose attention block no longer fits; a layer whose FFN does not fit keeps it
    // cold and the walk goes on to the next layer's attention (reference behaviour).
    auto promote = [&](const std::vector<int>& idx) {
        for (int i : idx) {
            plan->assignments[i].placement = JINF_PLACE_HOT;
            hot += model->tensor_infos[i].n_bytes;
            cold -= model->tensor_infos[i].n_bytes;
        }
    };
    for (auto& kv : layers) {
        Group& g = kv.second;
        if (hot + g.attn_bytes > cfg->gpu_memory_budget) break;
        promote(g.attn);
        if (hot + g.ffn_bytes <= cfg->gpu_memory_budget) promote(g.ffn);
    }
    plan->total_hot_bytes = hot;
    plan->total_cold_bytes = cold;
    *out = plan;
    return JINF_OK;
}

extern "C" void jinf_split_plan_free(jinf_split_plan* plan) {
    if (!plan) return;
    free(plan->assignments);
    free(plan);
}

extern "C" void jinf_split_plan_print(const jinf_split_plan* plan) {
    if (!plan) return;
    int nh = 0;
    for (int i = 0; i < plan->count; ++i) nh += plan->assignments[i].placement == JINF_PLACE_HOT;
    JINF_LOG("split plan: %d tensors (%d hot, %d cold), hot %.1f MB, cold %.1f MB", plan->count, nh,
             plan->count - nh, plan->total_hot_bytes / 1048576.0, plan->total_cold_bytes / 1048576.0);
    for (int i = 0; i < plan->count; ++i) {
        const jinf_weight_assignment* a = &plan->assignments[i];
        JINF_LOG("  %-48s %s %9.2f MB layer=%d tp=%d", a->tensor->name,
                 a->placement == JINF_PLACE_HOT ? "HOT " : "COLD", a->tensor->n_bytes / 1048576.0,
                 a->layer_index, (int)jinf_split_tp_role(a->tensor->name));
    }
}
