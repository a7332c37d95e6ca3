// jinf-b200: status codes, alignment helpers, logging.
//
// Drop-in replacement for the reference's include/jinf/common.h. The status
// values keep the reference's numbering (include/jinf/common.h:9-16 of the
// reference); JINF_ERR_TIMEOUT is appended for bounded device-side waits and
// collective deadlines, which the reference never needed.
#pragma once

#include <stddef.h>
#include <stdint.h>
#include <stdio.h>
#ifndef __cplusplus
#include <stdbool.h>
#endif

#ifdef __cplusplus
#include <chrono>
#endif

enum jinf_status
#ifdef __cplusplus
    : int
#endif
{
    JINF_OK          = 0,
    JINF_ERR_IO      = 1,
    JINF_ERR_PARSE   = 2,
    JINF_ERR_CUDA    = 3,
    JINF_ERR_OOM     = 4,
    JINF_ERR_INVALID = 5,
    JINF_ERR_TIMEOUT = 6,  // new: a bounded wait expired (device flag, collective deadline)
};
#ifndef __cplusplus
typedef enum jinf_status jinf_status;
#endif

static inline const char* jinf_status_str(jinf_status s) {
    switch (s) {
        case JINF_OK:          return "OK";
        case JINF_ERR_IO:      return "I/O error";
        case JINF_ERR_PARSE:   return "parse error";
        case JINF_ERR_CUDA:    return "CUDA error";
        case JINF_ERR_OOM:     return "out of memory";
        case JINF_ERR_INVALID: return "invalid argument";
        case JINF_ERR_TIMEOUT: return "timed out";
        default:               return "unknown error";
    }
}

// Round x up to a multiple of a power-of-two alignment.
#define JINF_ALIGN_UP(x, align) (((x) + ((align) - 1)) & ~((align) - 1))
#define JINF_ALIGN_4K(x)        JINF_ALIGN_UP((x), 4096)

#ifdef __cplusplus
// Wall-clock stopwatch (same surface as the reference's jinf_timer).
struct jinf_timer {
    std::chrono::steady_clock::time_point t0;
    jinf_timer() : t0(std::chrono::steady_clock::now()) {}
    void reset() { t0 = std::chrono::steady_clock::now(); }
    double elapsed_ms() const {
        return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    }
    double elapsed_us() const {
        return std::chrono::duration<double, std::micro>(std::chrono::steady_clock::now() - t0).count();
    }
};
#endif

#define JINF_LOG(fmt, ...) fprintf(stderr, "[jinf] " fmt "\n", ##__VA_ARGS__)

// Evaluate a jinf_status expression; log and return it from the caller on failure.
#define JINF_CHECK(expr, msg)                                                        \
    do {                                                                             \
        jinf_status jinf_s_ = (expr);                                                \
        if (jinf_s_ != JINF_OK) {                                                    \
            JINF_LOG("ERROR %s: %s (at %s:%d)", jinf_status_str(jinf_s_), (msg),     \
                     __FILE__, __LINE__);                                            \
            return jinf_s_;                                                          \
        }                                                                            \
    } while (0)

// Evaluate a CUDA runtime call; log and return JINF_ERR_CUDA from the caller on failure.
#define JINF_CUDA_CHECK(call)                                                        \
    do {                                                                             \
        cudaError_t jinf_e_ = (call);                                                \
        if (jinf_e_ != cudaSuccess) {                                                \
            JINF_LOG("CUDA error: %s (at %s:%d)", cudaGetErrorString(jinf_e_),       \
                     __FILE__, __LINE__);                                            \
            return JINF_ERR_CUDA;                                                    \
        }                                                                            \
    } while (0)
