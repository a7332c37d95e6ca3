// Device-side synthetic weight generation (built with -fmad=false). Uses the same
// synth_math.h code as the host generator, so the bytes are identical to
// jinf_synth_read_rows: the engine can materialise an 8B-shape model in HBM in
// milliseconds while the CPU oracle regenerates exactly the slices it checks.
#include "synth_internal.h"
#include "synth_math.h"
#include "jinf/quant.h"

namespace jinf {

__global__ void k_synth_q4_0(uint64_t key, float stdv, int64_t cols, int64_t r0, int64_t nr, int64_t c0,
                             int64_t nblk, uint8_t* dst, int64_t dst_row_bytes, int64_t dst_row0,
                             int64_t dst_row_step) {
    const int64_t total = nr * nblk;
    for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = g / nblk, b = g % nblk;
        const uint64_t e0 = (uint64_t)(r0 + i) * (uint64_t)cols + (uint64_t)(c0 + 32 * b);
        float v[32];
        for (int k = 0; k < 16; ++k) {
            double z0, z1;
            jinf_synth::normal_pair(key, (e0 >> 1) + k, &z0, &z1);
            v[2 * k] = (float)z0 * stdv;
            v[2 * k + 1] = (float)z1 * stdv;
        }
        uint8_t blk[18];
        jinf_synth::quantize_q4_0_block(v, blk);
        uint8_t* o = dst + (dst_row0 + i * dst_row_step) * dst_row_bytes + 18 * b;
        for (int k = 0; k < 18; ++k) o[k] = blk[k];
    }
}

// One thread per (row, 256-element super-block): the same values and the same quantiser
// steps as the host (jinf_synth_read_rows -> jinf_quantize_q4_K).
__global__ void k_synth_q4_k(uint64_t key, float stdv, int64_t cols, int64_t r0, int64_t nr, int64_t c0,
                             int64_t nsb, uint8_t* dst, int64_t dst_row_bytes, int64_t dst_row0,
                             int64_t dst_row_step) {
    const int64_t total = nr * nsb;
    for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = g / nsb, b = g % nsb;
        const uint64_t e0 = (uint64_t)(r0 + i) * (uint64_t)cols + (uint64_t)(c0 + 256 * b);
        float v[256];
        for (int k = 0; k < 128; ++k) {
            double z0, z1;
            jinf_synth::normal_pair(key, (e0 >> 1) + k, &z0, &z1);
            v[2 * k] = (float)z0 * stdv;
            v[2 * k + 1] = (float)z1 * stdv;
        }
        uint8_t blk[144];
        jinf_synth::quantize_q4_k_block(v, blk);
        uint8_t* o = dst + (dst_row0 + i * dst_row_step) * dst_row_bytes + 144 * b;
        for (int k = 0; k < 144; ++k) o[k] = blk[k];
    }
}

__global__ void k_synth_f32(uint64_t key, float stdv, int64_t cols, int64_t r0, int64_t n_pairs, float* dst) {
    for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < n_pairs; p += (int64_t)gridDim.x * blockDim.x) {
        const uint64_t e0 = (uint64_t)r0 * (uint64_t)cols;  // even: rows have an even number of columns
        double z0, z1;
        jinf_synth::normal_pair(key, (e0 >> 1) + (uint64_t)p, &z0, &z1);
        dst[2 * p] = (float)z0 * stdv;
        dst[2 * p + 1] = (float)z1 * stdv;
    }
}

__global__ void k_fill_f32(float* dst, int64_t n, float v) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = v;
}

static unsigned grid_for(int64_t n) {
    const int64_t g = (n + 255) / 256;
    return (unsigned)(g < 65536 ? (g > 0 ? g : 1) : 65536);
}

cudaError_t synth_fill_q4_0(uint64_t key, float stdv, int64_t cols, int64_t r0, int64_t nr, int64_t c0, int64_t nc,
                            uint8_t* dst, int64_t dst_row_bytes, int64_t dst_row0, int64_t dst_row_step,
                            cudaStream_t s) {
    if (cols % 32 || c0 % 32 || nc % 32 || nr < 0) return cudaErrorInvalidValue;
    const int64_t nblk = nc / 32;
    k_synth_q4_0<<<grid_for(nr * nblk), 256, 0, s>>>(key, stdv, cols, r0, nr, c0, nblk, dst, dst_row_bytes, dst_row0,
                                                      dst_row_step);
    return cudaGetLastError();
}

cudaError_t synth_fill_q4_k(uint64_t key, float stdv, int64_t cols, int64_t r0, int64_t nr, int64_t c0, int64_t nc,
                            uint8_t* dst, int64_t dst_row_bytes, int64_t dst_row0, int64_t dst_row_step,
                            cudaStream_t s) {
    if (cols % 256 || c0 % 256 || nc % 256 || nr < 0) return cudaErrorInvalidValue;
    const int64_t nsb = nc / 256;
    k_synth_q4_k<<<grid_for(nr * nsb), 128, 0, s>>>(key, stdv, cols, r0, nr, c0, nsb, dst, dst_row_bytes, dst_row0,
                                                     dst_row_step);
    return cudaGetLastError();
}

cudaError_t synth_fill_f32(uint64_t key, float stdv, int64_t cols, int64_t r0, int64_t nr, float* dst,
                           cudaStream_t s) {
    if (cols % 2) return cudaErrorInvalidValue;
    const int64_t pairs = nr * cols / 2;
    k_synth_f32<<<grid_for(pairs), 256, 0, s>>>(key, stdv, cols, r0, pairs, dst);
    return cudaGetLastError();
}

cudaError_t fill_f32(float* dst, int64_t n, float v, cudaStream_t s) {
    k_fill_f32<<<grid_for(n), 256, 0, s>>>(dst, n, v);
    return cudaGetLastError();
}

}  // namespace jinf

extern "C" jinf_status jinf_synth_read_rows_device(const jinf_synth_model* m, const char* name, int64_t row0,
                                                  int64_t n_rows, void* dst, cudaStream_t stream) {
    uint64_t key;
    float stdv;
    int role, type, nd;
    int64_t shape[4];
    uint64_t nbytes;
    if (!m || !name || !dst || row0 < 0 || n_rows < 0) return JINF_ERR_INVALID;
    if (!jinf::synth_tensor_params(m, name, &key, &stdv, &role) ||
        jinf_synth_tensor_info(m, name, &type, shape, &nd, &nbytes) != JINF_OK)
        return JINF_ERR_INVALID;
    const int64_t rows = nd > 1 ? shape[1] : 1, cols = shape[0];
    if (row0 + n_rows > rows) return JINF_ERR_INVALID;
    cudaError_t e;
    if (type == JINF_TYPE_Q4_0) {
        e = jinf::synth_fill_q4_0(key, stdv, cols, row0, n_rows, 0, cols, (uint8_t*)dst, (cols / 32) * 18, 0, 1,
                                  stream);
    } else if (type == JINF_TYPE_Q4_K) {
        e = jinf::synth_fill_q4_k(key, stdv, cols, row0, n_rows, 0, cols, (uint8_t*)dst, (cols / 256) * 144, 0, 1,
                                  stream);
    } else if (type == JINF_TYPE_F32) {
        e = role == 1 ? jinf::fill_f32((float*)dst, n_rows * cols, 1.0f, stream)
                      : jinf::synth_fill_f32(key, stdv, cols, row0, n_rows, (float*)dst, stream);
    } else {
        return JINF_ERR_INVALID;
    }
    return e == cudaSuccess ? JINF_OK : JINF_ERR_CUDA;
}
