// TEST INFRASTRUCTURE. A synchronous stand-in for the reference's NVMe reader, so that the
// reference's own engine (src/engine.cpp, src/buffer_pool.cpp, cuda/*.cu) links without
// liburing, which this image does not have. It implements the interface the reference
// declares in include/jinf/nvme_io.h:40-57 with plain pread(2): a request completes before
// jinf_io_submit returns, and jinf_io_wait hands the finished completions back in order.
// Semantics kept from the reference's src/nvme_io.cpp: a read past the end of the file is a
// short read, not an error (the engine reads 4 KiB-rounded lengths), and a negative result
// of a completed request is an I/O error only for jinf_io_read_sync.
#include "jinf/nvme_io.h"

#include <errno.h>
#include <fcntl.h>
#include <stdlib.h>
#include <unistd.h>

#include <deque>

struct jinf_io_context {
    std::deque<jinf_io_completion> done;
};

jinf_status jinf_io_create(jinf_io_context** ctx, const jinf_io_config* config) {
    if (!ctx || !config) return JINF_ERR_INVALID;
    *ctx = new jinf_io_context();
    return JINF_OK;
}

void jinf_io_destroy(jinf_io_context* ctx) { delete ctx; }

jinf_status jinf_io_open(jinf_io_context* ctx, const char* path, int* fd) {
    if (!ctx || !path || !fd) return JINF_ERR_INVALID;
    const int f = open(path, O_RDONLY);
    if (f < 0) return JINF_ERR_IO;
    *fd = f;
    return JINF_OK;
}

void jinf_io_close(jinf_io_context* ctx, int fd) {
    (void)ctx;
    if (fd >= 0) close(fd);
}

// Reads [offset, offset + length) into buf; returns the bytes read (short at end of file)
// or -errno.
static int32_t read_all(int fd, void* buf, size_t offset, size_t length) {
    size_t got = 0;
    while (got < length) {
        const ssize_t n = pread(fd, (char*)buf + got, length - got, (off_t)(offset + got));
        if (n < 0) {
            if (errno == EINTR) continue;
            return -errno;
        }
        if (n == 0) break;
        got += (size_t)n;
    }
    return (int32_t)got;
}

jinf_status jinf_io_submit(jinf_io_context* ctx, const jinf_io_request* reqs, int count) {
    if (!ctx || (!reqs && count > 0) || count < 0) return JINF_ERR_INVALID;
    for (int i = 0; i < count; ++i) {
        jinf_io_completion c;
        c.user_data = reqs[i].user_data;
        c.result = read_all(reqs[i].fd, reqs[i].buffer, reqs[i].offset, reqs[i].length);
        ctx->done.push_back(c);
    }
    return JINF_OK;
}

jinf_status jinf_io_wait(jinf_io_context* ctx, jinf_io_completion* comps, int min, int max, int* actual) {
    if (!ctx || !comps || !actual || max < min) return JINF_ERR_INVALID;
    if ((int)ctx->done.size() < min) return JINF_ERR_IO;  // nothing else can complete later
    int n = 0;
    while (n < max && !ctx->done.empty()) {
        comps[n++] = ctx->done.front();
        ctx->done.pop_front();
    }
    *actual = n;
    return JINF_OK;
}

jinf_status jinf_io_read_sync(jinf_io_context* ctx, int fd, void* buf, size_t offset, size_t length) {
    if (!ctx || !buf) return JINF_ERR_INVALID;
    const int32_t r = read_all(fd, buf, offset, length);
    return r < 0 ? JINF_ERR_IO : JINF_OK;
}

void* jinf_io_alloc_aligned(size_t size) {
    void* p = nullptr;
    const size_t sz = (size + 4095) & ~(size_t)4095;
    return posix_memalign(&p, 4096, sz ? sz : 4096) == 0 ? p : nullptr;
}

void jinf_io_free_aligned(void* ptr) { free(ptr); }
