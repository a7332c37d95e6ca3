// TEST INFRASTRUCTURE: a command-line driver around the reference's own engine and CUDA
// kernels, compiled unmodified from the reference tree by oracle/Makefile (target
// _ref/ref_engine; the NVMe reader is replaced by ref_io_pread.cpp). It produces the
// outputs that pin the CPU oracle's forward restatement, and it times the reference's
// dequant-matvec kernel recompiled for this GPU. Nothing in the product links it.
//
//   ref_engine decode  <model.nvmw> <out.bin> <max_ctx> <n_gen> <tok>...
//       jinf_engine_create + one jinf_engine_forward per prompt token (reference
//       src/engine.cpp:684-760), then n_gen greedy steps (first maximum, as
//       src/engine.cpp:783-790, without the EOS stop so every step is recorded).
//       out.bin: int32 n_prompt, n_gen, n_vocab; int32 tokens[n_prompt + n_gen];
//       float logits[n_prompt + n_gen][n_vocab] (the logits after each forward).
//   ref_engine kernels <in.bin> <out.bin>
//       runs jinf_cuda_dequant_matvec, jinf_cuda_rmsnorm, jinf_cuda_rope,
//       jinf_cuda_attention and jinf_cuda_silu_mul on the cases in in.bin (layout below,
//       written by tests/golden/make_ref_engine_golden.py) and writes their outputs.
//   ref_engine gemv    <out.json>
//       jinf_cuda_dequant_matvec (Q4_0) on the Llama-3-8B projection shapes, weight copies
//       rotated over more than 4x L2, CUDA events over 50 launches per shape.
#include "jinf/engine.h"
#include "jinf/quant.h"

#include <cuda_runtime.h>

#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <string>
#include <vector>

extern "C" {
void jinf_cuda_rmsnorm(float* output, const float* input, const void* weight, int n, float eps, int weight_type,
                       cudaStream_t stream);
void jinf_cuda_rope(float* q, float* k, int head_dim, int n_heads, int n_heads_kv, int pos, float freq_base,
                    cudaStream_t stream);
void jinf_cuda_silu_mul(float* output, const float* gate, const float* up, int n, cudaStream_t stream);
void jinf_cuda_dequant_matvec(const void* weight, const float* input, float* output, int rows, int cols, int qtype,
                              cudaStream_t stream);
void jinf_cuda_attention(float* output, const float* q, const float* k_cache, const float* v_cache, int head_dim,
                         int n_heads, int n_heads_kv, int n_past, int max_ctx, cudaStream_t stream);
}

#define CK(x)                                                                                      \
    do {                                                                                           \
        cudaError_t e_ = (x);                                                                      \
        if (e_ != cudaSuccess) {                                                                   \
            fprintf(stderr, "ref_engine: %s failed: %s\n", #x, cudaGetErrorString(e_));            \
            exit(2);                                                                               \
        }                                                                                          \
    } while (0)

static void put(FILE* f, const void* p, size_t n) {
    if (fwrite(p, 1, n, f) != n) {
        fprintf(stderr, "ref_engine: short write\n");
        exit(2);
    }
}

static int decode(int argc, char** argv) {
    if (argc < 7) return 1;
    const char* model = argv[2];
    const char* out = argv[3];
    const int max_ctx = atoi(argv[4]), n_gen = atoi(argv[5]);
    std::vector<int32_t> toks;
    toks.reserve((size_t)argc + 4096);
    for (int i = 6; i < argc; ++i) toks.push_back(atoi(argv[i]));
    const int n_prompt = (int)toks.size();
    if (n_prompt + n_gen > max_ctx) return 1;

    jinf_engine_config cfg = jinf_engine_config_default();
    cfg.model_path = model;
    cfg.max_context = max_ctx;
    cfg.buffer_capacity = (size_t)16 << 20;
    jinf_engine* e = nullptr;
    if (jinf_engine_create(&e, &cfg) != JINF_OK) {
        fprintf(stderr, "ref_engine: jinf_engine_create failed\n");
        return 2;
    }
    const int V = e->n_vocab;
    std::vector<float> logits((size_t)(n_prompt + n_gen) * V);
    for (int t = 0; t < n_prompt + n_gen; ++t) {
        float* dl = nullptr;
        if (jinf_engine_forward(e, &toks[t], 1, &dl) != JINF_OK) {
            fprintf(stderr, "ref_engine: jinf_engine_forward failed at step %d\n", t);
            return 2;
        }
        CK(cudaMemcpy(&logits[(size_t)t * V], dl, (size_t)V * sizeof(float), cudaMemcpyDeviceToHost));
        if (t + 1 >= n_prompt && (int)toks.size() < n_prompt + n_gen) {
            const float* l = &logits[(size_t)t * V];
            int best = 0;
            for (int j = 1; j < V; ++j)
                if (l[j] > l[best]) best = j;
            toks.push_back(best);
        }
    }
    FILE* f = fopen(out, "wb");
    if (!f) return 2;
    const int32_t hdr[3] = {n_prompt, n_gen, V};
    put(f, hdr, sizeof(hdr));
    put(f, toks.data(), toks.size() * sizeof(int32_t));
    put(f, logits.data(), logits.size() * sizeof(float));
    fclose(f);
    jinf_engine_destroy(e);
    return 0;
}

// ---------------------------------------------------------------- kernel cases
//
// in.bin, a sequence of little-endian records:
//   matvec:    int32 rows, cols, qtype, n_weight_bytes; u8 weight[n]; float x[cols]
//   rmsnorm:   int32 n; float eps; float x[n]; float w[n]
//   rope:      int32 hd, nh, nkv, pos; float base; float q[nh*hd]; float k[nkv*hd]
//   attention: int32 hd, nh, nkv, n_past, max_ctx; float q[nh*hd];
//              float kc[max_ctx*nkv*hd]; float vc[max_ctx*nkv*hd]
//   silu:      int32 n; float g[n]; float u[n]
// each preceded by an int32 kind (1..5); kind 0 ends the file. out.bin holds, per record,
// the kernel's output floats (rope: q then k).
struct Reader {
    FILE* f;
    int32_t i32() {
        int32_t v;
        if (fread(&v, 4, 1, f) != 1) exit(3);
        return v;
    }
    float f32() {
        float v;
        if (fread(&v, 4, 1, f) != 1) exit(3);
        return v;
    }
    template <class T>
    std::vector<T> vec(size_t n) {
        std::vector<T> v(n);
        if (n && fread(v.data(), sizeof(T), n, f) != n) exit(3);
        return v;
    }
};

template <class T>
static T* dev(const std::vector<T>& h) {
    T* d = nullptr;
    CK(cudaMalloc(&d, h.size() * sizeof(T) + 16));
    CK(cudaMemcpy(d, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice));
    return d;
}

static std::vector<float> back(const float* d, size_t n) {
    std::vector<float> h(n);
    CK(cudaDeviceSynchronize());
    CK(cudaMemcpy(h.data(), d, n * sizeof(float), cudaMemcpyDeviceToHost));
    return h;
}

static int kernels(int argc, char** argv) {
    if (argc < 4) return 1;
    Reader r{fopen(argv[2], "rb")};
    FILE* out = fopen(argv[3], "wb");
    if (!r.f || !out) return 2;
    for (;;) {
        const int kind = r.i32();
        if (kind == 0) break;
        std::vector<float> res;
        if (kind == 1) {
            const int rows = r.i32(), cols = r.i32(), qt = r.i32(), nb = r.i32();
            auto w = r.vec<uint8_t>((size_t)nb);
            auto x = r.vec<float>((size_t)cols);
            uint8_t* dw = dev(w);
            float* dx = dev(x);
            float* dy = nullptr;
            CK(cudaMalloc(&dy, (size_t)rows * 4));
            jinf_cuda_dequant_matvec(dw, dx, dy, rows, cols, qt, 0);
            res = back(dy, (size_t)rows);
            cudaFree(dw), cudaFree(dx), cudaFree(dy);
        } else if (kind == 2) {
            const int n = r.i32();
            const float eps = r.f32();
            auto x = r.vec<float>((size_t)n);
            auto w = r.vec<float>((size_t)n);
            float *dx = dev(x), *dw = dev(w), *dy = nullptr;
            CK(cudaMalloc(&dy, (size_t)n * 4));
            jinf_cuda_rmsnorm(dy, dx, dw, n, eps, 0, 0);
            res = back(dy, (size_t)n);
            cudaFree(dx), cudaFree(dw), cudaFree(dy);
        } else if (kind == 3) {
            const int hd = r.i32(), nh = r.i32(), nkv = r.i32(), pos = r.i32();
            const float base = r.f32();
            auto q = r.vec<float>((size_t)nh * hd);
            auto k = r.vec<float>((size_t)nkv * hd);
            float *dq = dev(q), *dk = dev(k);
            jinf_cuda_rope(dq, dk, hd, nh, nkv, pos, base, 0);
            res = back(dq, q.size());
            const auto kk = back(dk, k.size());
            res.insert(res.end(), kk.begin(), kk.end());
            cudaFree(dq), cudaFree(dk);
        } else if (kind == 4) {
            const int hd = r.i32(), nh = r.i32(), nkv = r.i32(), n_past = r.i32(), max_ctx = r.i32();
            auto q = r.vec<float>((size_t)nh * hd);
            auto kc = r.vec<float>((size_t)max_ctx * nkv * hd);
            auto vc = r.vec<float>((size_t)max_ctx * nkv * hd);
            float *dq = dev(q), *dk = dev(kc), *dv = dev(vc), *dy = nullptr;
            CK(cudaMalloc(&dy, (size_t)nh * hd * 4));
            jinf_cuda_attention(dy, dq, dk, dv, hd, nh, nkv, n_past, max_ctx, 0);
            res = back(dy, (size_t)nh * hd);
            cudaFree(dq), cudaFree(dk), cudaFree(dv), cudaFree(dy);
        } else if (kind == 5) {
            const int n = r.i32();
            auto g = r.vec<float>((size_t)n);
            auto u = r.vec<float>((size_t)n);
            float *dg = dev(g), *du = dev(u), *dy = nullptr;
            CK(cudaMalloc(&dy, (size_t)n * 4));
            jinf_cuda_silu_mul(dy, dg, du, n, 0);
            res = back(dy, (size_t)n);
            cudaFree(dg), cudaFree(du), cudaFree(dy);
        } else {
            fprintf(stderr, "ref_engine: unknown case kind %d\n", kind);
            return 2;
        }
        CK(cudaGetLastError());
        put(out, res.data(), res.size() * sizeof(float));
    }
    fclose(r.f);
    fclose(out);
    return 0;
}

// ---------------------------------------------------------------- GEMV timing

static uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static int gemv(int argc, char** argv) {
    if (argc < 3) return 1;
    const int shapes[5][2] = {{4096, 4096}, {1024, 4096}, {14336, 4096}, {4096, 14336}, {128256, 4096}};
    FILE* out = fopen(argv[2], "w");
    if (!out) return 2;
    cudaDeviceProp prop;
    CK(cudaGetDeviceProperties(&prop, 0));
    fprintf(out, "{\"device\": \"%s\", \"kernel\": \"reference jinf_cuda_dequant_matvec (Q4_0), sm_100a build\", \"shapes\": {",
            prop.name);
    cudaStream_t s;
    CK(cudaStreamCreate(&s));
    for (int si = 0; si < 5; ++si) {
        const int rows = shapes[si][0], cols = shapes[si][1];
        const size_t wbytes = (size_t)rows * (cols / 32) * sizeof(jinf_block_q4_0);
        const int copies = (int)std::max<size_t>(2, (size_t)(4.0 * 126e6 / (double)wbytes) + 1);
        // one host image: random nibbles, scales 2^-7 .. 2^-6 (finite, like N(0, 0.02) weights)
        std::vector<uint8_t> h(wbytes);
        for (size_t b = 0; b < wbytes / sizeof(jinf_block_q4_0); ++b) {
            jinf_block_q4_0* blk = (jinf_block_q4_0*)h.data() + b;
            const uint64_t z = mix64(b);
            blk->d = (uint16_t)(0x2000u | (uint16_t)(z & 0x3FFu));
            for (int i = 0; i < 16; ++i) blk->qs[i] = (uint8_t)(mix64(z + i) & 0xFF);
        }
        std::vector<void*> dw(copies);
        for (int c = 0; c < copies; ++c) {
            CK(cudaMalloc(&dw[c], wbytes));
            CK(cudaMemcpy(dw[c], h.data(), wbytes, cudaMemcpyHostToDevice));
        }
        std::vector<float> x(cols);
        for (int i = 0; i < cols; ++i) x[i] = (float)((double)(mix64(1000003 + i) >> 11) / 9007199254740992.0 * 2 - 1);
        float* dx = dev(x);
        float* dy = nullptr;
        CK(cudaMalloc(&dy, (size_t)rows * 4));
        for (int i = 0; i < 3; ++i) jinf_cuda_dequant_matvec(dw[i % copies], dx, dy, rows, cols, JINF_TYPE_Q4_0, s);
        CK(cudaStreamSynchronize(s));
        const int n = 50;
        cudaEvent_t e0, e1;
        CK(cudaEventCreate(&e0));
        CK(cudaEventCreate(&e1));
        CK(cudaEventRecord(e0, s));
        for (int i = 0; i < n; ++i) jinf_cuda_dequant_matvec(dw[i % copies], dx, dy, rows, cols, JINF_TYPE_Q4_0, s);
        CK(cudaEventRecord(e1, s));
        CK(cudaEventSynchronize(e1));
        CK(cudaGetLastError());
        float ms = 0.f;
        CK(cudaEventElapsedTime(&ms, e0, e1));
        const double us = 1000.0 * ms / n;
        const double gbs = (double)(wbytes + (size_t)cols * 4 + (size_t)rows * 4) / (us * 1e-6) / 1e9;
        fprintf(out, "%s\"%dx%d\": {\"us\": %.2f, \"GB/s\": %.1f}", si ? ", " : "", rows, cols, us, gbs);
        for (int c = 0; c < copies; ++c) cudaFree(dw[c]);
        cudaFree(dx), cudaFree(dy);
        cudaEventDestroy(e0), cudaEventDestroy(e1);
    }
    fprintf(out, "}}\n");
    fclose(out);
    cudaStreamDestroy(s);
    return 0;
}

int main(int argc, char** argv) {
    int rc = 1;
    if (argc >= 2 && !strcmp(argv[1], "decode")) rc = decode(argc, argv);
    else if (argc >= 2 && !strcmp(argv[1], "kernels")) rc = kernels(argc, argv);
    else if (argc >= 2 && !strcmp(argv[1], "gemv")) rc = gemv(argc, argv);
    if (rc == 1)
        fprintf(stderr, "usage: ref_engine decode <nvmw> <out> <max_ctx> <n_gen> <tok>... | kernels <in> <out> | "
                        "gemv <out.json>\n");
    return rc;
}
