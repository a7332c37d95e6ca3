// C-linkage entry points into the reference's own host code, compiled (unmodified, from
// its source tree) into _ref/libjinf_ref.so by this folder's Makefile. Test
// infrastructure only: it lets the tests and the golden-vector script call the
// reference's dequantizer, GGUF parser and splitter, whose symbols have C++ linkage.
#include "jinf/gguf.h"
#include "jinf/quant.h"
#include "jinf/splitter.h"

#include <stdio.h>
#include <string.h>

extern "C" {

void ref_dequantize_q4_0(const void* b, float* out, int n) { jinf_dequantize_q4_0((const jinf_block_q4_0*)b, out, n); }
void ref_dequantize_q4_K(const void* b, float* out, int n) { jinf_dequantize_q4_K((const jinf_block_q4_K*)b, out, n); }
void ref_dequantize_q8_0(const void* b, float* out, int n) { jinf_dequantize_q8_0((const jinf_block_q8_0*)b, out, n); }
void ref_dequantize(const void* data, int type, float* out, long long n) {
    jinf_dequantize(data, (jinf_qtype)type, out, (int64_t)n);
}

// Parse a GGUF file with the reference parser; writes a compact text summary:
// "status version n_tensors n_kv alignment data_offset\n" then hparams, then one line per tensor.
int ref_gguf_summary(const char* path, char* out, int cap) {
    jinf_gguf_file* f = nullptr;
    jinf_status s = jinf_gguf_open(&f, path);
    if (s != JINF_OK) return snprintf(out, cap, "status %d\n", (int)s);
    int n = snprintf(out, cap, "status 0 %u %llu %llu %u %zu\n", f->version, (unsigned long long)f->tensor_count,
                     (unsigned long long)f->kv_count, f->alignment, f->data_offset);
    const jinf_model_hparams* h = &f->hparams;
    n += snprintf(out + n, cap - n, "hp %s %u %u %u %u %u %u %u %.9g %.9g\n", h->arch, h->n_layers, h->n_embd,
                  h->n_heads, h->n_heads_kv, h->n_ff, h->n_vocab, h->n_ctx_train, h->rope_freq_base,
                  h->rms_norm_eps);
    for (uint64_t i = 0; i < f->tensor_count && n < cap; ++i) {
        const jinf_gguf_tensor_info* t = &f->tensor_infos[i];
        n += snprintf(out + n, cap - n, "t %s %u %lld %lld %d %llu %lld %zu\n", t->name, t->n_dims,
                      (long long)t->shape[0], (long long)t->shape[1], (int)t->type, (unsigned long long)t->offset,
                      (long long)t->n_elements, t->n_bytes);
    }
    jinf_gguf_close(f);
    return n;
}

// Run the reference splitter on a GGUF file; placements[i] = 0 hot / 1 cold per tensor,
// totals[0..1] = hot / cold bytes. Returns the tensor count or -status.
int ref_split(const char* path, unsigned long long budget, int* placements, unsigned long long* totals) {
    jinf_gguf_file* f = nullptr;
    jinf_status s = jinf_gguf_open(&f, path);
    if (s != JINF_OK) return -(int)s;
    jinf_split_config cfg = {(size_t)budget, 0, 0};
    jinf_split_plan* plan = nullptr;
    s = jinf_split_analyze(f, &cfg, &plan);
    if (s != JINF_OK) {
        jinf_gguf_close(f);
        return -(int)s;
    }
    for (int i = 0; i < plan->count; ++i) placements[i] = (int)plan->assignments[i].placement;
    totals[0] = plan->total_hot_bytes;
    totals[1] = plan->total_cold_bytes;
    const int n = plan->count;
    jinf_split_plan_free(plan);
    jinf_gguf_close(f);
    return n;
}

}  // extern "C"
