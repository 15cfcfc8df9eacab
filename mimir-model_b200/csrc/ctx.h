// ctx.h -- internal state behind the opaque handles of include/mimgpu.h.
#pragma once

#include <cstdarg>
#include <cstdint>
#include <mutex>
#include <string>

#include <cuda_runtime.h>

#include "../../include/mimgpu.h"

struct mimgpu_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    void *ws = nullptr;        // grow-only workspace of the host-buffer calls
    size_t ws_size = 0;
    unsigned *status = nullptr;  // device word: DevStatus bits set by kernels
    unsigned *status_host = nullptr;  // pinned copy of status[0], written on the waited stream
    int64_t timeout_ms = 60000;
    std::recursive_mutex mu;
    std::string err;
};

struct mimgpu_tensor {
    mimgpu_ctx *ctx = nullptr;
    int dtype = 0;
    int ndim = 0;
    int64_t shape[8] = {0};
    uint8_t *dev = nullptr;
    size_t nbytes = 0;
};

namespace mimgpu {

int fail(mimgpu_ctx *c, int code, const char *fmt, ...);
int cuda_fail(mimgpu_ctx *c, cudaError_t e, const char *what);
// Waits for `st` with the context's deadline, then checks the device status
// word; returns a MIMGPU_* code.
int sync_bounded(mimgpu_ctx *c, cudaStream_t st);
// Makes the context's device current on this thread.
int use_device(mimgpu_ctx *c);
// Ensures the workspace holds `bytes`.
int ensure_ws(mimgpu_ctx *c, size_t bytes);
// The checks every dequant_matmul entry point makes first
// (checkDequantMatmul, interp/transformer.go:216-236).
int check_matmul(mimgpu_ctx *c, int64_t rows, int64_t k, const mimgpu_tensor *w);
// Bytes of a tensor of `dtype` and shape; -1 when the shape does not fit
// the block size.
long long tensor_bytes(int dtype, int ndim, const int64_t *shape);

}  // namespace mimgpu
