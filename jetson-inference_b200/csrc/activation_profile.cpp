// Activation profiles in the reference's file format (the static predictor's input):
//   int32 n_layers, int32 n_ff, int32 total_tokens, then n_layers x n_ff float32
//   frequencies (the fraction of calibration tokens on which |SiLU(gate_n)| exceeded the
//   profiling threshold).
// Writer: reference tools/profile_activations.cpp:143-162. Reader and the static predictor
// rule (a neuron is active when its frequency is above the threshold): reference
// src/activation_predictor.cpp:226-300.
#include "jinf/b200.h"

#include <stdio.h>

#include <vector>

extern "C" jinf_status jinf_activation_profile_write(const char* path, int n_layers, int n_ff, int total_tokens,
                                                     const int32_t* counts) {
    if (!path || n_layers <= 0 || n_ff <= 0 || total_tokens < 0 || !counts) return JINF_ERR_INVALID;
    FILE* fp = fopen(path, "wb");
    if (!fp) return JINF_ERR_IO;
    bool ok = fwrite(&n_layers, sizeof(int), 1, fp) == 1 && fwrite(&n_ff, sizeof(int), 1, fp) == 1 &&
              fwrite(&total_tokens, sizeof(int), 1, fp) == 1;
    std::vector<float> freq((size_t)n_ff);
    for (int l = 0; ok && l < n_layers; ++l) {
        for (int n = 0; n < n_ff; ++n)
            freq[n] = total_tokens > 0 ? (float)counts[(size_t)l * n_ff + n] / (float)total_tokens : 0.0f;
        ok = fwrite(freq.data(), sizeof(float), (size_t)n_ff, fp) == (size_t)n_ff;
    }
    if (fclose(fp) != 0) ok = false;
    return ok ? JINF_OK : JINF_ERR_IO;
}

extern "C" jinf_status jinf_activation_profile_read(const char* path, float threshold, int n_layers, int n_ff,
                                                    int32_t* ids, int32_t* n_active) {
    if (!path || n_layers <= 0 || n_ff <= 0 || !ids || !n_active) return JINF_ERR_INVALID;
    FILE* fp = fopen(path, "rb");
    if (!fp) return JINF_ERR_IO;
    int hdr[3] = {0, 0, 0};
    jinf_status s = JINF_OK;
    if (fread(hdr, sizeof(int), 3, fp) != 3 || hdr[0] <= 0 || hdr[1] <= 0) {
        s = JINF_ERR_PARSE;
    } else if (hdr[0] != n_layers || hdr[1] != n_ff) {
        s = JINF_ERR_INVALID;  // a profile of another model
    } else {
        std::vector<float> freq((size_t)n_ff);
        for (int l = 0; l < n_layers && s == JINF_OK; ++l) {
            if (fread(freq.data(), sizeof(float), (size_t)n_ff, fp) != (size_t)n_ff) {
                s = JINF_ERR_PARSE;
                break;
            }
            int k = 0;
            for (int n = 0; n < n_ff; ++n)
                if (freq[n] > threshold) ids[(size_t)l * n_ff + k++] = n;
            n_active[l] = k;
        }
    }
    fclose(fp);
    return s;
}
