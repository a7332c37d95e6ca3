// C-ABI wrappers of the engine building blocks (include/jinf/b200.h).
#include "jinf/b200.h"
#include "jinf/quant.h"

#include "attn_f16.h"
#include "common.cuh"
#include "gemv.h"
#include "device_state.cuh"
#include "q4m.cuh"
#include "prefill.h"

#include <algorithm>
#include <atomic>

using namespace jinf;

static int device_sms() {
    // per-device cache (up to 64 devices); every writer stores the same value
    static std::atomic<int> sms[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    int n = sms[dev].load(std::memory_order_relaxed);
    if (!n) {
        n = 148;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        sms[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

extern "C" uint64_t jinf_b200_q4m_bytes(int rows, int cols) {
    Q4MShape sh;
    return q4m_shape(rows, cols, &sh) ? sh.bytes : 0;
}

extern "C" jinf_status jinf_b200_q4m_pack(const void* aos, void* q4m, int rows, int cols, cudaStream_t stream) {
    Q4MShape sh;
    if (!aos || !q4m || !q4m_shape(rows, cols, &sh)) return JINF_ERR_INVALID;
    return q4m_repack(aos, q4m, sh, stream) == cudaSuccess ? JINF_OK : JINF_ERR_CUDA;
}

static int q4m_fmt_of(int qtype) { return q4m_fmt_of_qtype(qtype); }

extern "C" jinf_status jinf_b200_q4m_pack_host(const void* aos, int qtype, void* q4m, int rows, int cols) {
    Q4MShape sh;
    const int fmt = q4m_fmt_of(qtype);
    if (!aos || !q4m || fmt < 0 || !q4m_shape(rows, cols, &sh, fmt)) return JINF_ERR_INVALID;
    q4m_repack_host(aos, q4m, sh);
    return JINF_OK;
}

extern "C" uint64_t jinf_b200_q4m_bytes_qt(int rows, int cols, int qtype) {
    Q4MShape sh;
    const int fmt = q4m_fmt_of(qtype);
    return fmt >= 0 && q4m_shape(rows, cols, &sh, fmt) ? sh.bytes : 0;
}

extern "C" jinf_status jinf_b200_q4m_pack_qt(const void* aos, int qtype, void* q4m, int rows, int cols,
                                             cudaStream_t stream) {
    Q4MShape sh;
    const int fmt = q4m_fmt_of(qtype);
    if (!aos || !q4m || fmt < 0 || !q4m_shape(rows, cols, &sh, fmt)) return JINF_ERR_INVALID;
    return q4m_repack(aos, q4m, sh, stream) == cudaSuccess ? JINF_OK : JINF_ERR_CUDA;
}

static constexpr int kQ4mMaxKw = 32;

extern "C" size_t jinf_b200_gemv_q4m_workspace_bytes(int rows, int cols) {
    Q4MShape sh;
    if (!q4m_shape(rows, cols, &sh)) return 0;
    return (size_t)sh.pairs * kQ4mMaxKw * Q4M_PAIR_ROWS * sizeof(float) + (size_t)sh.pairs * sizeof(unsigned int);
}

static jinf_status gemv_q4m_common(GemvParams& p, const Q4MShape& sh, int xm, void* workspace, int kw,
                                   cudaStream_t stream) {
    if (sh.cols > gemvm_max_cols(sh.fmt) || kw < 0 || kw > kQ4mMaxKw) return JINF_ERR_INVALID;
    int grid = gemvm_grid(sh.cols, xm, EPI_STORE, device_sms(), sh.fmt);
    if (kw == 0 && gemvm_use_local(sh.pairs, grid)) {  // pairs spread evenly over CTAs, K split by their warps
        p.kw = 1;
        p.local_k = 1;
        return gemvm_launch(p, xm, EPI_STORE, gemvm_local_grid(sh.pairs, grid), stream, false) == cudaSuccess
                   ? JINF_OK
                   : JINF_ERR_CUDA;
    }
    if (kw == 0) kw = gemvm_pick_kw(sh.pairs, sh.groups, grid, workspace ? kQ4mMaxKw : 1);
    if (kw > sh.groups || (kw > 1 && !workspace)) return JINF_ERR_INVALID;
    p.kw = kw;
    if (kw > 1) {
        p.part = (float*)workspace;
        p.cnt = (unsigned int*)((uint8_t*)workspace + (size_t)sh.pairs * kQ4mMaxKw * Q4M_PAIR_ROWS * sizeof(float));
    }
    return gemvm_launch(p, xm, EPI_STORE, grid, stream, false) == cudaSuccess ? JINF_OK : JINF_ERR_CUDA;
}

extern "C" jinf_status jinf_b200_gemv_q4m(const void* q4m, const void* x, int x_type, float* y, int rows, int cols,
                                          void* workspace, int kw, cudaStream_t stream) {
    Q4MShape sh;
    if (!q4m || !x || !y || !q4m_shape(rows, cols, &sh)) return JINF_ERR_INVALID;
    if (x_type != JINF_TYPE_F32 && x_type != JINF_TYPE_F16) return JINF_ERR_INVALID;
    GemvParams p{};
    gemvm_params_for(p, q4m, sh);
    p.x = x;
    p.y = y;
    return gemv_q4m_common(p, sh, x_type == JINF_TYPE_F32 ? X_PLAIN_F32 : X_PLAIN_F16, workspace, kw, stream);
}

extern "C" jinf_status jinf_b200_gemv_q4m_qt(const void* q4m, int qtype, const void* x, int x_type, float* y,
                                             int rows, int cols, void* workspace, int kw, cudaStream_t stream) {
    Q4MShape sh;
    const int fmt = q4m_fmt_of(qtype);
    if (!q4m || !x || !y || fmt < 0 || !q4m_shape(rows, cols, &sh, fmt)) return JINF_ERR_INVALID;
    if (x_type != JINF_TYPE_F32 && x_type != JINF_TYPE_F16) return JINF_ERR_INVALID;
    GemvParams p{};
    gemvm_params_for(p, q4m, sh);
    p.x = x;
    p.y = y;
    return gemv_q4m_common(p, sh, x_type == JINF_TYPE_F32 ? X_PLAIN_F32 : X_PLAIN_F16, workspace, kw, stream);
}

extern "C" jinf_status jinf_b200_gemv_q4m_rmsnorm(const void* q4m, const float* h, const float* gain, float eps,
                                                  float* y, int rows, int cols, void* workspace, int kw,
                                                  cudaStream_t stream) {
    Q4MShape sh;
    if (!q4m || !h || !gain || !y || !q4m_shape(rows, cols, &sh)) return JINF_ERR_INVALID;
    GemvParams p{};
    gemvm_params_for(p, q4m, sh);
    p.hin = h;
    p.norm_w = gain;
    p.eps = eps;
    p.y = y;
    return gemv_q4m_common(p, sh, X_RMSNORM, workspace, kw, stream);
}

// ---------------------------------------------------------------- allocation-free GEMV
//
// jinf_b200_gemv_q4m_noalloc: the same split-K tensor-core GEMV as jinf_b200_gemv_q4m, with
// its workspace in this file-scope device array instead of caller memory, for callers that
// cannot allocate device memory (or hand out a workspace) at call time. Layout: arrival
// counters of up to kNoAllocMaxPairs tile pairs at a fixed offset (zero at module load; every
// call leaves them zero again, so they are zero between calls), then the partial rows.
// Calls that overlap in time (other streams, other host threads) share it and race.
static constexpr size_t kNoAllocScratchBytes = (size_t)4 << 20;  // 4 MB
static constexpr int kNoAllocMaxPairs = 8192;                    // rows <= 262144
static constexpr size_t kNoAllocCntBytes = (size_t)kNoAllocMaxPairs * sizeof(unsigned int);
static __device__ __align__(256) unsigned char g_gemv_noalloc_scratch[kNoAllocScratchBytes];

// Device address of the scratch on the current device, looked up once per device (the
// first call on a device must not be inside a stream capture).
static jinf_status noalloc_scratch(uint8_t** out) {
    static std::atomic<uint8_t*> addr[64];  // every writer stores the same address
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return JINF_ERR_CUDA;
    uint8_t* a = addr[dev].load(std::memory_order_acquire);
    if (!a) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_gemv_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            JINF_LOG("jinf_b200_gemv_q4m_noalloc: scratch address lookup failed: %s", cudaGetErrorString(e));
            return JINF_ERR_CUDA;
        }
        a = (uint8_t*)p;
        addr[dev].store(a, std::memory_order_release);
    }
    *out = a;
    return JINF_OK;
}

extern "C" jinf_status jinf_b200_gemv_q4m_noalloc(const void* q4m, const void* x, int x_type, float* y, int rows,
                                                  int cols, cudaStream_t stream) {
    Q4MShape sh;
    if (!q4m || !x || !y || !q4m_shape(rows, cols, &sh)) return JINF_ERR_INVALID;
    if (x_type != JINF_TYPE_F32 && x_type != JINF_TYPE_F16) return JINF_ERR_INVALID;
    if (sh.cols > gemvm_max_cols()) return JINF_ERR_INVALID;
    if (sh.pairs > kNoAllocMaxPairs) {
        JINF_LOG("jinf_b200_gemv_q4m_noalloc: %d rows exceed the static scratch limit of %d rows", rows,
                 kNoAllocMaxPairs * Q4M_PAIR_ROWS);
        return JINF_ERR_INVALID;
    }
    const int xm = x_type == JINF_TYPE_F32 ? X_PLAIN_F32 : X_PLAIN_F16;
    const int grid = gemvm_grid(sh.cols, xm, EPI_STORE, device_sms());
    GemvParams p{};
    gemvm_params_for(p, q4m, sh);
    p.x = x;
    p.y = y;
    if (gemvm_use_local(sh.pairs, grid)) {  // as jinf_b200_gemv_q4m with kw = 0: K split inside each CTA
        p.kw = 1;
        p.local_k = 1;
        return gemvm_launch(p, xm, EPI_STORE, gemvm_local_grid(sh.pairs, grid), stream, false) == cudaSuccess
                   ? JINF_OK
                   : JINF_ERR_CUDA;
    }
    // the K split that kw = 0 would pick, limited to what the array's partial rows hold
    const size_t part_cap = kNoAllocScratchBytes - kNoAllocCntBytes;
    const size_t per_kw = (size_t)sh.pairs * Q4M_PAIR_ROWS * sizeof(float);
    const int kw_fit = (int)std::min<size_t>((size_t)kQ4mMaxKw, part_cap / per_kw);
    const int kw = kw_fit <= 1 ? 1 : gemvm_pick_kw(sh.pairs, sh.groups, grid, kw_fit);
    uint8_t* scratch = nullptr;
    JINF_CHECK(noalloc_scratch(&scratch), "noalloc scratch");
    p.kw = kw;
    if (kw > 1) {
        p.cnt = (unsigned int*)scratch;
        p.part = (float*)(scratch + kNoAllocCntBytes);
    }
    return gemvm_launch(p, xm, EPI_STORE, grid, stream, false) == cudaSuccess ? JINF_OK : JINF_ERR_CUDA;
}

extern "C" size_t jinf_b200_attention_workspace_bytes(int n_kv_heads, int head_dim, int max_ctx) {
    int n_split = (max_ctx + 63) / 64;
    if (n_split < 1) n_split = 1;
    if (n_split > 64) n_split = 64;
    return sizeof(DeviceState) + 256 + sizeof(float) * attn_partial_floats(n_kv_heads, n_split, head_dim);
}

extern "C" jinf_status jinf_b200_attention_f16(float* out, const float* q, const void* k_cache, const void* v_cache,
                                               int head_dim, int n_heads, int n_kv_heads, int n_pos, int max_ctx,
                                               void* workspace, cudaStream_t stream) {
    if (!out || !q || !k_cache || !v_cache || !workspace || n_pos <= 0 || n_pos > max_ctx || n_heads <= 0 ||
        n_kv_heads <= 0 || n_heads % n_kv_heads || n_kv_heads > 64 || n_heads / n_kv_heads > 8)
        return JINF_ERR_INVALID;
    if (head_dim != 64 && head_dim != 128) return JINF_ERR_INVALID;
    int n_split = (max_ctx + 63) / 64;
    if (n_split < 1) n_split = 1;
    if (n_split > 64) n_split = 64;
    DeviceState* st = (DeviceState*)workspace;
    const int pos = n_pos - 1;
    if (cudaMemcpyAsync(&st->pos, &pos, sizeof(int), cudaMemcpyHostToDevice, stream) != cudaSuccess)
        return JINF_ERR_CUDA;
    AttnParams p{};
    p.q = q;
    p.kcache = (const __half*)k_cache;
    p.vcache = (const __half*)v_cache;
    p.out = out;
    p.partial = (float*)((uint8_t*)workspace + ((sizeof(DeviceState) + 255) & ~(size_t)255));
    p.n_heads = n_heads;
    p.n_kv_heads = n_kv_heads;
    p.head_dim = head_dim;
    p.max_ctx = max_ctx;
    p.n_split = n_split;
    p.st = st;
    const cudaError_t e = attn_launch(p, stream, false);
    // the host value of `pos` must stay alive until the copy has been issued: it is a
    // pageable source, which cudaMemcpyAsync stages before returning.
    return e == cudaSuccess ? JINF_OK : JINF_ERR_CUDA;
}

extern "C" jinf_status jinf_b200_prefill_gemm(const void* q4m, int rows, int cols, const void* x_f16, int T,
                                              const float* tok_scale, float* y, int ldy, int accumulate, int* err,
                                              cudaStream_t stream) {
    if (!q4m || !x_f16 || !tok_scale || !y || !err || T <= 0) return JINF_ERR_INVALID;
    const cudaError_t e = prefill_gemm_launch((const uint8_t*)q4m, rows, cols, (const __half*)x_f16, T, tok_scale, y,
                                              ldy, accumulate ? 1 : 0, err, stream);
    if (e == cudaErrorInvalidValue) return JINF_ERR_INVALID;
    return e == cudaSuccess ? JINF_OK : JINF_ERR_CUDA;
}
