// CPU oracle for the jinf decode path -- TEST INFRASTRUCTURE ONLY.
//
// A plain C++ restatement of the reference's arithmetic, used by tests/, by
// __graft_entry__.smoke() and by bench.py's cpu_baseline leg as the checker. Nothing in
// the product (the jetson-inference_b200 package) links or calls it.
//
// Each function cites the reference code it restates. The reference has no CPU forward
// pass (its matvec/RMSNorm/RoPE/attention/SiLU exist only as CUDA), so the forward step
// follows reference src/engine.cpp:418-511 (layer) and :684-760 (token loop) with the
// math of the cuda/*.cu kernels. Dequantization is pinned against the reference's own
// src/quant.cpp (compiled by this folder's Makefile into _ref/) through golden vectors.
//
// Accumulations that the reference does in fp32 with an unspecified parallel order are
// done here in double, so the oracle is closer to the exact result than any fp32 order.
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <string>
#include <unordered_map>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

extern "C" {

// fp16 -> fp32, exact (reference src/quant.cpp:7-45 restated).
float orc_fp16_to_fp32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    int exp = (h >> 10) & 31;
    uint32_t man = h & 1023u;
    uint32_t bits;
    if (exp == 31) {
        bits = sign | 0x7f800000u | (man << 13);
    } else if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            int e = 1;
            while (!(man & 1024u)) { man <<= 1; --e; }
            bits = sign | ((uint32_t)(e + 112) << 23) | ((man & 1023u) << 13);
        }
    } else {
        bits = sign | ((uint32_t)(exp + 112) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

void orc_fp16_to_fp32_array(const uint16_t* in, float* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = orc_fp16_to_fp32(in[i]);
}

// Q4_0: 18-byte blocks, byte i = elements 2i (low) / 2i+1 (high), value (q-8)*d
// (reference src/quant.cpp:49-60, cuda/dequant_kernels.cu:16-20).
void orc_dequant_q4_0(const void* data, float* out, int64_t nb) {
    const uint8_t* p = (const uint8_t*)data;
    for (int64_t b = 0; b < nb; ++b, p += 18) {
        const float d = orc_fp16_to_fp32((uint16_t)(p[0] | (p[1] << 8)));
        for (int i = 0; i < 16; ++i) {
            out[32 * b + 2 * i] = (float)((int)(p[2 + i] & 15) - 8) * d;
            out[32 * b + 2 * i + 1] = (float)((int)(p[2 + i] >> 4) - 8) * d;
        }
    }
}

// Q4_K: 144-byte super-blocks (reference src/quant.cpp:64-93): sub-block j uses qs[16j..],
// scale/min 6-bit packing with the high sub-blocks' 4 extra bits ABOVE the 2 carried bits.
// Built with -ffp-contract=off: (d*sc)*q and the subtraction round separately.
void orc_dequant_q4_K(const void* data, float* out, int64_t nb) {
    const uint8_t* p = (const uint8_t*)data;
    for (int64_t b = 0; b < nb; ++b, p += 144) {
        const float d = orc_fp16_to_fp32((uint16_t)(p[0] | (p[1] << 8)));
        const float dmin = orc_fp16_to_fp32((uint16_t)(p[2] | (p[3] << 8)));
        const uint8_t* s = p + 4;
        const uint8_t* qs = p + 16;
        for (int j = 0; j < 8; ++j) {
            int sc, mn;
            if (j < 4) {
                sc = s[j] & 63;
                mn = s[j + 4] & 63;
            } else {
                sc = ((s[j + 4] & 15) << 2) | (s[j - 4] >> 6);
                mn = ((s[j + 4] >> 4) << 2) | (s[j] >> 6);
            }
            const float sd = d * (float)sc;
            const float sm = dmin * (float)mn;
            for (int i = 0; i < 16; ++i) {
                const uint8_t v = qs[16 * j + i];
                out[256 * b + 32 * j + 2 * i] = sd * (float)(v & 15) - sm;
                out[256 * b + 32 * j + 2 * i + 1] = sd * (float)(v >> 4) - sm;
            }
        }
    }
}

// Q8_0 (reference src/quant.cpp:97-104).
void orc_dequant_q8_0(const void* data, float* out, int64_t nb) {
    const uint8_t* p = (const uint8_t*)data;
    for (int64_t b = 0; b < nb; ++b, p += 34) {
        const float d = orc_fp16_to_fp32((uint16_t)(p[0] | (p[1] << 8)));
        for (int i = 0; i < 32; ++i) out[32 * b + i] = (float)(int8_t)p[2 + i] * d;
    }
}

// Q6_K in the reference GPU layout (reference cuda/dequant_kernels.cu:94-111; the reference
// has no CPU Q6_K): ql[i/2] nibble, qh[i/4] 2 bits at 2*(i%4), int8 scale per 16, d last.
void orc_dequant_q6_K(const void* data, float* out, int64_t nb) {
    const uint8_t* p = (const uint8_t*)data;
    for (int64_t b = 0; b < nb; ++b, p += 210) {
        const float d = orc_fp16_to_fp32((uint16_t)(p[208] | (p[209] << 8)));
        for (int i = 0; i < 256; ++i) {
            const int lo = (p[i >> 1] >> ((i & 1) * 4)) & 15;
            const int hi = (p[128 + (i >> 2)] >> (2 * (i & 3))) & 3;
            out[256 * b + i] = d * (float)(int8_t)p[192 + (i >> 4)] * (float)((lo | (hi << 4)) - 32);
        }
    }
}

static int block_elems(int qt) { return qt == 2 || qt == 8 ? 32 : (qt == 12 || qt == 14 ? 256 : 1); }
static int block_bytes(int qt) {
    switch (qt) {
        case 0: return 4;
        case 1: return 2;
        case 2: return 18;
        case 8: return 34;
        case 12: return 144;
        case 14: return 210;
        default: return 0;
    }
}

// Dequantize a row of `cols` values of type qt.
static void dequant_row(const uint8_t* row, int qt, int cols, float* out) {
    const int be = block_elems(qt);
    switch (qt) {
        case 0: memcpy(out, row, sizeof(float) * (size_t)cols); break;
        case 1: for (int i = 0; i < cols; ++i) out[i] = orc_fp16_to_fp32((uint16_t)(row[2 * i] | (row[2 * i + 1] << 8))); break;
        case 2: orc_dequant_q4_0(row, out, cols / be); break;
        case 8: orc_dequant_q8_0(row, out, cols / be); break;
        case 12: orc_dequant_q4_K(row, out, cols / be); break;
        case 14: orc_dequant_q6_K(row, out, cols / be); break;
        default: break;
    }
}

static size_t row_bytes(int qt, int cols) { return (size_t)(cols / block_elems(qt)) * block_bytes(qt); }

// y = W x with W[rows][cols] of type qt (reference cuda/matmul_kernels.cu:8-185):
// each weight is dequantized exactly as the reference does, products summed in double.
void orc_matvec(const void* w, int qt, const float* x, float* y, int rows, int cols) {
    const size_t rb = row_bytes(qt, cols);
#pragma omp parallel
    {
        std::vector<float> buf((size_t)cols);
#pragma omp for schedule(static)
        for (int r = 0; r < rows; ++r) {
            dequant_row((const uint8_t*)w + (size_t)r * rb, qt, cols, buf.data());
            double s = 0.0;
            for (int c = 0; c < cols; ++c) s += (double)(buf[c] * x[c]);
            y[r] = (float)s;
        }
    }
}

// RMSNorm: y = x * rsqrt(sum(x^2)/n + eps) * w (reference cuda/rmsnorm_kernel.cu:9-34).
void orc_rmsnorm(float* out, const float* in, const float* w, int n, float eps) {
    double ss = 0.0;
    for (int i = 0; i < n; ++i) ss += (double)in[i] * (double)in[i];
    const float r = (float)(1.0 / sqrt(ss / (double)n + (double)eps));
    std::vector<float> tmp(in, in + n);
    for (int i = 0; i < n; ++i) out[i] = tmp[i] * r * w[i];
}

// RoPE on adjacent pairs (reference cuda/rope_kernel.cu:36-49), in the reference's own
// fp32 arithmetic: theta_i = powf(base, -2i/hd), angle = (float)pos * theta, cosf/sinf.
void orc_rope(float* q, float* k, int hd, int nh, int nkv, int pos, float base) {
    for (int which = 0; which < 2; ++which) {
        float* v = which ? k : q;
        const int heads = which ? nkv : nh;
        for (int h = 0; h < heads; ++h)
            for (int i = 0; i < hd / 2; ++i) {
                const float theta = powf(base, -2.0f * (float)i / (float)hd);
                const float a = (float)pos * theta;
                const float c = cosf(a), s = sinf(a);
                float* e = v + (size_t)h * hd + 2 * i;
                const float x0 = e[0], x1 = e[1];
                e[0] = x0 * c - x1 * s;
                e[1] = x0 * s + x1 * c;
            }
    }
}

// out = g * sigmoid(g) * u (reference cuda/silu_kernel.cu:15-17).
void orc_silu_mul(float* out, const float* g, const float* u, int n) {
    for (int i = 0; i < n; ++i) out[i] = (float)((double)g[i] / (1.0 + exp(-(double)g[i])) * (double)u[i]);
}

// Max-subtracted softmax (reference cuda/softmax_kernel.cu:8-42).
void orc_softmax(float* out, const float* in, int n) {
    double m = -INFINITY;
    for (int i = 0; i < n; ++i) m = in[i] > m ? in[i] : m;
    double s = 0.0;
    for (int i = 0; i < n; ++i) s += exp((double)in[i] - m);
    for (int i = 0; i < n; ++i) out[i] = (float)(exp((double)in[i] - m) / s);
}

// Decode attention over the reference cache layout [ctx][nkv*hd] (reference
// cuda/attention_kernel.cu:45-98): kv head = h / (nh/nkv), scores scaled by 1/sqrt(hd),
// softmax over n_past positions, weighted sum of V.
void orc_attention(float* out, const float* q, const float* kc, const float* vc, int hd, int nh, int nkv,
                   int n_past) {
    const int g = nh / nkv;
    std::vector<double> sc((size_t)n_past);
    for (int h = 0; h < nh; ++h) {
        const int kvh = h / g;
        const float* qh = q + (size_t)h * hd;
        double m = -INFINITY;
        for (int t = 0; t < n_past; ++t) {
            const float* kt = kc + ((size_t)t * nkv + kvh) * hd;
            double dot = 0.0;
            for (int d = 0; d < hd; ++d) dot += (double)qh[d] * (double)kt[d];
            sc[t] = dot / sqrt((double)hd);
            m = sc[t] > m ? sc[t] : m;
        }
        double s = 0.0;
        for (int t = 0; t < n_past; ++t) {
            sc[t] = exp(sc[t] - m);
            s += sc[t];
        }
        for (int d = 0; d < hd; ++d) {
            double a = 0.0;
            for (int t = 0; t < n_past; ++t) a += sc[t] * (double)vc[((size_t)t * nkv + kvh) * hd + d];
            out[(size_t)h * hd + d] = (float)(a / s);
        }
    }
}

// Sparse FFN over neuron bundles: a dense FFN restricted to the active neurons
// (reference cuda/sparse_matmul.cu:16-111 gate/up with SiLU, :199-219 down over fp32 columns).
void orc_sparse_ffn(const void* bundles, const float* x, float* out, const int* offsets, int n_act, int hidden,
                    int qt, float* gate_up) {
    const size_t rb = row_bytes(qt, hidden);
    std::vector<float> row((size_t)hidden);
    for (int i = 0; i < n_act; ++i) {
        const uint8_t* b = (const uint8_t*)bundles + offsets[i];
        double gs = 0.0, us = 0.0;
        dequant_row(b, qt, hidden, row.data());
        for (int c = 0; c < hidden; ++c) gs += (double)(row[c] * x[c]);
        dequant_row(b + rb, qt, hidden, row.data());
        for (int c = 0; c < hidden; ++c) us += (double)(row[c] * x[c]);
        gate_up[i] = (float)(gs / (1.0 + exp(-gs)) * us);
    }
    for (int dd = 0; dd < hidden; ++dd) {
        double s = 0.0;
        for (int i = 0; i < n_act; ++i) {
            const float* col = (const float*)((const uint8_t*)bundles + offsets[i] + 2 * rb);
            s += (double)gate_up[i] * (double)col[dd];
        }
        out[dd] = (float)s;
    }
}

// ------------------------------------------------------------ decode step (whole model)

struct OrcTensor {
    int qt;
    const uint8_t* data;  // borrowed
};

struct orc_model {
    int L, d, nh, nkv, hd, ff, V, max_ctx, kv_f16;
    float eps, base;
    int pos = 0;
    std::unordered_map<std::string, OrcTensor> t;
    std::vector<float> kc, vc;  // [L][ctx][nkv*hd]
    std::vector<std::vector<int>> ffn_mask;  // per layer: active neurons (empty vector: dense)
    std::vector<char> has_mask;
};

orc_model* orc_model_create(int n_layers, int d, int nh, int nkv, int ff, int vocab, float eps, float base,
                            int max_ctx, int kv_f16) {
    orc_model* m = new orc_model();
    m->L = n_layers;
    m->d = d;
    m->nh = nh;
    m->nkv = nkv;
    m->hd = d / nh;
    m->ff = ff;
    m->V = vocab;
    m->eps = eps;
    m->base = base;
    m->max_ctx = max_ctx;
    m->kv_f16 = kv_f16;
    m->kc.assign((size_t)n_layers * max_ctx * nkv * m->hd, 0.f);
    m->vc.assign(m->kc.size(), 0.f);
    return m;
}

void orc_model_destroy(orc_model* m) { delete m; }

// Borrow (not copy) a tensor's bytes in file layout; the caller keeps them alive.
int orc_model_bind(orc_model* m, const char* name, int qt, const void* data) {
    if (!m || !name || !data) return -1;
    m->t[name] = OrcTensor{qt, (const uint8_t*)data};
    return 0;
}

int orc_model_pos(const orc_model* m) { return m->pos; }

// Restrict the FFN of `layer` to the neurons ids[0..n) (n < 0: dense again): the other
// neurons' SiLU(gate)*up is 0, the semantics of the reference's sparse FFN
// (src/engine.cpp:339-415, cuda/sparse_matmul.cu:104-110, :211-218).
int orc_model_set_ffn_mask(orc_model* m, int layer, const int* ids, int n) {
    if (!m || layer < 0 || layer >= m->L) return -1;
    if ((int)m->ffn_mask.size() < m->L) {
        m->ffn_mask.resize(m->L);
        m->has_mask.assign(m->L, 0);
    }
    if (n < 0) {
        m->has_mask[layer] = 0;
        m->ffn_mask[layer].clear();
        return 0;
    }
    m->has_mask[layer] = 1;
    m->ffn_mask[layer].assign(ids, ids + n);
    return 0;
}

static const OrcTensor* need(orc_model* m, const std::string& n) {
    auto it = m->t.find(n);
    return it == m->t.end() ? nullptr : &it->second;
}

// Round to the nearest fp16 value (ties to even) and back: the B200 engine keeps K/V in fp16.
static float round_f16(float f) {
    if (!(fabsf(f) < 65520.f)) return f;
    int e;
    frexpf(f, &e);
    const int ulp_exp = (e - 1 < -14 ? -14 : e - 1) - 10;
    const float ulp = ldexpf(1.f, ulp_exp);
    return nearbyintf(f / ulp) * ulp;
}

static void matvec_t(const OrcTensor* w, const float* x, float* y, int rows, int cols) {
    orc_matvec(w->data, w->qt, x, y, rows, cols);
}

// One token through the model (reference src/engine.cpp:684-760 with :418-511 per layer).
// logits may be NULL to skip the output head. Returns 0 on success.
int orc_forward(orc_model* m, int token, float* logits) {
    if (!m || token < 0 || token >= m->V || m->pos >= m->max_ctx) return -1;
    const int d = m->d, hd = m->hd, kvd = m->nkv * hd;
    std::vector<float> h((size_t)d), xn((size_t)d), q((size_t)d), k((size_t)kvd), v((size_t)kvd), a((size_t)d),
        o((size_t)d), g((size_t)m->ff), u((size_t)m->ff);
    const OrcTensor* emb = need(m, "token_embd.weight");
    if (!emb) return -2;
    dequant_row(emb->data + (size_t)token * row_bytes(emb->qt, d), emb->qt, d, h.data());
    char nm[96];
    for (int L = 0; L < m->L; ++L) {
        auto T = [&](const char* suffix) {
            snprintf(nm, sizeof nm, "blk.%d.%s", L, suffix);
            return need(m, nm);
        };
        const OrcTensor *an = T("attn_norm.weight"), *wq = T("attn_q.weight"), *wk = T("attn_k.weight"),
                        *wv = T("attn_v.weight"), *wo = T("attn_output.weight"), *fn = T("ffn_norm.weight"),
                        *wg = T("ffn_gate.weight"), *wu = T("ffn_up.weight"), *wd = T("ffn_down.weight");
        if (!an || !wq || !wk || !wv || !wo || !fn || !wg || !wu || !wd) return -3;
        orc_rmsnorm(xn.data(), h.data(), (const float*)an->data, d, m->eps);
        matvec_t(wq, xn.data(), q.data(), d, d);
        matvec_t(wk, xn.data(), k.data(), kvd, d);
        matvec_t(wv, xn.data(), v.data(), kvd, d);
        orc_rope(q.data(), k.data(), hd, m->nh, m->nkv, m->pos, m->base);
        float* kl = m->kc.data() + (size_t)L * m->max_ctx * kvd;
        float* vl = m->vc.data() + (size_t)L * m->max_ctx * kvd;
        for (int i = 0; i < kvd; ++i) {
            kl[(size_t)m->pos * kvd + i] = m->kv_f16 ? round_f16(k[i]) : k[i];
            vl[(size_t)m->pos * kvd + i] = m->kv_f16 ? round_f16(v[i]) : v[i];
        }
        orc_attention(a.data(), q.data(), kl, vl, hd, m->nh, m->nkv, m->pos + 1);
        matvec_t(wo, a.data(), o.data(), d, d);
        for (int i = 0; i < d; ++i) h[i] += o[i];
        orc_rmsnorm(xn.data(), h.data(), (const float*)fn->data, d, m->eps);
        matvec_t(wg, xn.data(), g.data(), m->ff, d);
        matvec_t(wu, xn.data(), u.data(), m->ff, d);
        orc_silu_mul(g.data(), g.data(), u.data(), m->ff);
        if ((int)m->has_mask.size() > L && m->has_mask[L]) {
            std::vector<float> keep((size_t)m->ff, 0.f);
            for (int id : m->ffn_mask[L])
                if (id >= 0 && id < m->ff) keep[id] = g[id];
            g.swap(keep);
        }
        matvec_t(wd, g.data(), o.data(), d, m->ff);
        for (int i = 0; i < d; ++i) h[i] += o[i];
    }
    if (logits) {
        const OrcTensor *on = need(m, "output_norm.weight"), *wout = need(m, "output.weight");
        if (!on || !wout) return -4;
        orc_rmsnorm(xn.data(), h.data(), (const float*)on->data, d, m->eps);
        matvec_t(wout, xn.data(), logits, m->V, d);
    }
    m->pos += 1;
    return 0;
}

// Greedy argmax, first maximum wins (reference src/engine.cpp:783-790).
int orc_argmax(const float* v, int n) {
    int best = 0;
    for (int i = 1; i < n; ++i)
        if (v[i] > v[best]) best = i;
    return best;
}

// Seeded N(0,1) K/V for positions [0, n_pos) of every layer (timing-only shortcut).
int orc_fill_kv_random(orc_model* m, int n_pos, uint64_t seed) {
    if (!m || n_pos < 0 || n_pos > m->max_ctx) return -1;
    const size_t kvd = (size_t)m->nkv * m->hd;
    for (int L = 0; L < m->L; ++L)
        for (size_t i = 0; i < (size_t)n_pos * kvd; ++i) {
            uint64_t z = seed + 0x9E3779B97F4A7C15ull * (uint64_t)(L * 1000003ull + i + 1);
            z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
            z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
            z ^= z >> 31;
            const double u1 = ((double)(z >> 40) + 0.5) / 16777216.0, u2 = ((double)((z >> 16) & 0xFFFFFF) + 0.5) / 16777216.0;
            const double r = sqrt(-2.0 * log(u1));
            m->kc[(size_t)L * m->max_ctx * kvd + i] = (float)(r * cos(6.283185307179586 * u2));
            m->vc[(size_t)L * m->max_ctx * kvd + i] = (float)(r * sin(6.283185307179586 * u2));
        }
    m->pos = n_pos;
    return 0;
}

// Load positions [0, n_pos) of every layer's cache from fp16 values laid out
// [layer][kv head][n_pos][hd] (the B200 engine's cache order, e.g. read back after its
// seeded fill), and set the position to n_pos. The values are exact in both caches.
int orc_model_load_kv_f16(orc_model* m, int n_pos, const uint16_t* k, const uint16_t* v) {
    if (!m || !k || !v || n_pos < 0 || n_pos > m->max_ctx) return -1;
    const size_t kvd = (size_t)m->nkv * m->hd;
    for (int L = 0; L < m->L; ++L)
        for (int h = 0; h < m->nkv; ++h)
            for (int p = 0; p < n_pos; ++p)
                for (int d = 0; d < m->hd; ++d) {
                    const size_t src = (((size_t)L * m->nkv + h) * n_pos + p) * m->hd + d;
                    const size_t dst = ((size_t)L * m->max_ctx + p) * kvd + (size_t)h * m->hd + d;
                    m->kc[dst] = orc_fp16_to_fp32(k[src]);
                    m->vc[dst] = orc_fp16_to_fp32(v[src]);
                }
    m->pos = n_pos;
    return 0;
}

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

}  // extern "C"
