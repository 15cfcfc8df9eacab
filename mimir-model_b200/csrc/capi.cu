// capi.cu -- context, uploads and the per-op fast paths of include/mimgpu.h.
//
// Each per-op entry point mirrors one fastPaths adapter of interp/fast.go
// (gsoultan/mimir-model): it checks its arguments the way the Go fast path
// does, copies the host inputs into the context's workspace, runs the
// sm_100a kernels on the context's stream, copies the outputs back and waits
// with a deadline.  There is no CPU fallback: a case the kernels do not
// serve returns MIMGPU_ENOTHANDLED, a malformed call MIMGPU_EINVAL.
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <thread>
#include <vector>

#include "common.cuh"
#include "ctx.h"
#include "kernels.h"

using namespace mimgpu;

namespace mimgpu {

int fail(mimgpu_ctx *c, int code, const char *fmt, ...) {
    if (c) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof buf, fmt, ap);
        va_end(ap);
        c->err = buf;
    }
    return code;
}

int cuda_fail(mimgpu_ctx *c, cudaError_t e, const char *what) {
    if (e == cudaSuccess) return MIMGPU_OK;
    int code = e == cudaErrorMemoryAllocation ? MIMGPU_ENOMEM : e == cudaErrorInvalidValue ? MIMGPU_EINVAL : MIMGPU_ECUDA;
    return fail(c, code, "%s: %s", what, cudaGetErrorString(e));
}

int use_device(mimgpu_ctx *c) { return cuda_fail(c, cudaSetDevice(c->device), "cudaSetDevice"); }

int sync_bounded(mimgpu_ctx *c, cudaStream_t st) {
    // the status word comes back with the stream's own work (pinned host
    // memory): no synchronous copy after the wait
    cudaError_t e = cudaMemcpyAsync(c->status_host, c->status, sizeof(unsigned), cudaMemcpyDeviceToHost, st);
    if (e != cudaSuccess) return cuda_fail(c, e, "status");
    // the wait: polled without sleeping for the first 20 ms (a decode step
    // or a per-op product ends well within that, and a sleep would add its
    // timer slack to every call), then with 20 us sleeps up to the deadline
    const auto t0 = std::chrono::steady_clock::now();
    const auto deadline = t0 + std::chrono::milliseconds(c->timeout_ms);
    const auto spin_until = t0 + std::chrono::milliseconds(20);
    for (;;) {
        e = cudaStreamQuery(st);
        if (e == cudaSuccess) break;
        if (e != cudaErrorNotReady) return cuda_fail(c, e, "stream");
        const auto now = std::chrono::steady_clock::now();
        if (now > deadline)
            return fail(c, MIMGPU_ETIMEOUT, "device work did not finish within %lld ms", (long long)c->timeout_ms);
        if (now > spin_until) std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
    const unsigned status = *(volatile unsigned *)c->status_host;
    if (status) {
        cudaMemset(c->status, 0, sizeof(unsigned));
        if (status & DEV_TIMEOUT) return fail(c, MIMGPU_ETIMEOUT, "a kernel gave up a bounded wait");
        return fail(c, MIMGPU_ECUDA, "kernel status %#x", status);
    }
    return MIMGPU_OK;
}

int ensure_ws(mimgpu_ctx *c, size_t bytes) {
    if (bytes <= c->ws_size) return MIMGPU_OK;
    if (c->ws) {
        cudaStreamSynchronize(c->stream);
        cudaFree(c->ws);
        c->ws = nullptr;
        c->ws_size = 0;
    }
    size_t want = bytes + bytes / 4 + (1 << 20);
    cudaError_t e = cudaMalloc(&c->ws, want);
    if (e != cudaSuccess) return cuda_fail(c, e, "workspace");
    c->ws_size = want;
    return MIMGPU_OK;
}

long long tensor_bytes(int dtype, int ndim, const int64_t *shape) {
    if (ndim < 0 || ndim > 8) return -1;
    long long n = 1;
    for (int i = 0; i < ndim; i++) {
        if (shape[i] < 0) return -1;
        n *= shape[i];
    }
    if (ndim == 0) return block_elems(dtype) == 1 ? block_bytes(dtype) : -1;
    const long long last = shape[ndim - 1];
    const int be = block_elems(dtype);
    if (last % be) return -1;
    return n / be * block_bytes(dtype);
}

// checkDequantMatmul, interp/transformer.go:216-236, for a 2-D weight; and
// the sizes the kernels index with 32-bit row counts.
int check_matmul(mimgpu_ctx *c, int64_t rows, int64_t k, const mimgpu_tensor *w) {
    if (!w || w->ndim != 2) return fail(c, MIMGPU_EINVAL, "dequant_matmul: w must be [N, K]");
    if (w->shape[1] != k) return fail(c, MIMGPU_EINVAL, "dequant_matmul: x has K=%lld, w is [%lld, %lld]",
                                      (long long)k, (long long)w->shape[0], (long long)w->shape[1]);
    if (rows < 0) return fail(c, MIMGPU_EINVAL, "dequant_matmul: rows < 0");
    if (w->ctx != c) return fail(c, MIMGPU_EINVAL, "dequant_matmul: w belongs to another context");
    if (rows > INT32_MAX || w->shape[0] > INT32_MAX)
        return fail(c, MIMGPU_EINVAL, "dequant_matmul: %lld rows x %lld outputs exceed 32-bit counts", (long long)rows,
                    (long long)w->shape[0]);
    return MIMGPU_OK;
}

}  // namespace mimgpu

namespace {

bool known_dtype(int dt) { return dt == F32 || dt == F16 || dt == Q8_0 || dt == Q4_K || dt == Q6_K; }

// Carves the workspace into 256-byte aligned pieces.
struct Carver {
    uint8_t *p;
    template <class T>
    T *take(size_t count) {
        T *r = (T *)p;
        p += (count * sizeof(T) + 255) & ~(size_t)255;
        return r;
    }
};

size_t al(size_t b) { return (b + 255) & ~(size_t)255; }


// Which product a call takes: 256 = the block-256 8-bit kernels (v2) for
// Q4_K/Q6_K, 32 = the block-32 ones (v1) for Q4_K/Q6_K/Q8_0, 0 = the exact
// f32 product (every other dtype, and dequant_matmul.v1 itself), as the
// reference falls back without a kernel (q8.go:104-115, fast.go:254-258).
int matmul_path(int block, int dt, int64_t k) {
    if (block == 256 && (dt == Q4_K || dt == Q6_K) && k % 256 == 0 && k > 0) return 256;
    if (block == 32 && a8_b32_dtype_ok(dt, k)) return 32;
    return 0;
}

size_t matmul_ws_bytes(int path, int64_t rows, int64_t k) {
    if (path == 256) return act_q8_bytes((int)rows, k);
    if (path == 32) return act_q8_b32_bytes((int)rows, k);
    return 0;
}

// Queues the product of device buffers on st; the workspace from ws on must
// already hold matmul_ws_bytes(path, rows, k).
cudaError_t enqueue_matmul(mimgpu_ctx *c, int path, const float *dx, int64_t rows, int64_t k,
                           const mimgpu_tensor *w, const float *db, float *dy, cudaStream_t st, void *ws) {
    const int64_t n = w->shape[0];
    GemvSeg seg{w->dev, w->dtype, (int)n, dy, n, db};
    if (path == 256) {
        ActQ8 act = act_q8_carve(ws, (int)rows, k);
        cudaError_t e = launch_quantize_a8(dx, (int)rows, k, act, st, false);
        return e == cudaSuccess ? launch_gemv_a8(&seg, 1, dx, act, (int)rows, k, c->status, st, false) : e;
    }
    if (path == 32) {
        ActQ8 act = act_q8_b32_carve(ws, (int)rows, k);
        cudaError_t e = launch_quantize_a8_b32(dx, (int)rows, k, act, st);
        return e == cudaSuccess ? launch_gemv_a8_b32(seg, dx, act, (int)rows, k, st) : e;
    }
    return launch_gemv_f32(&seg, 1, dx, (int)rows, k, st, false);
}

int run_matmul(mimgpu_ctx *c, int block, const float *x, int64_t rows, int64_t k, const mimgpu_tensor *w,
               const float *bias, float *y) {
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    int rc = check_matmul(c, rows, k, w);
    if (rc) return rc;
    if ((rc = use_device(c))) return rc;
    const int64_t n = w->shape[0];
    if (rows == 0 || n == 0) return MIMGPU_OK;
    const int path = matmul_path(block, w->dtype, k);
    const size_t io = al(rows * k * 4) + al(rows * n * 4) + al(n * 4);
    if ((rc = ensure_ws(c, io + matmul_ws_bytes(path, rows, k)))) return rc;
    Carver cv{(uint8_t *)c->ws};
    float *dx = cv.take<float>(rows * k), *dy = cv.take<float>(rows * n), *db = cv.take<float>(n);
    cudaStream_t st = c->stream;
    cudaError_t e = cudaMemcpyAsync(dx, x, rows * k * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess && bias) e = cudaMemcpyAsync(db, bias, n * 4, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return cuda_fail(c, e, "copy in");
    e = enqueue_matmul(c, path, dx, rows, k, w, bias ? db : nullptr, dy, st, cv.p);
    if (e != cudaSuccess) return cuda_fail(c, e, "dequant_matmul kernels");
    e = cudaMemcpyAsync(y, dy, rows * n * 4, cudaMemcpyDeviceToHost, st);
    if (e != cudaSuccess) return cuda_fail(c, e, "copy out");
    return sync_bounded(c, st);
}

// The device-buffer entry points: one product queued on the caller's stream.
int run_matmul_dev(mimgpu_ctx *c, void *stream, int block, const float *x, int64_t rows, int64_t k,
                   const mimgpu_tensor *w, const float *bias, float *y, const char *what) {
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    int rc = check_matmul(c, rows, k, w);
    if (rc || (rc = use_device(c))) return rc;
    if (rows == 0 || w->shape[0] == 0) return MIMGPU_OK;
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    const int path = matmul_path(block, w->dtype, k);
    if ((rc = ensure_ws(c, matmul_ws_bytes(path, rows, k)))) return rc;
    return cuda_fail(c, enqueue_matmul(c, path, x, rows, k, w, bias, y, st, c->ws), what);
}

}  // namespace

extern "C" {

int mimgpu_abi_version(void) { return MIMGPU_ABI_VERSION; }

int mimgpu_open(int device, mimgpu_ctx **out) {
    if (!out) return MIMGPU_EINVAL;
    *out = nullptr;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count) return MIMGPU_ECUDA;
    if (cudaSetDevice(device) != cudaSuccess) return MIMGPU_ECUDA;
    auto *c = new mimgpu_ctx;
    c->device = device;
    // status block: [0] DevStatus bits, [2..3] the wait limit of a device wait (ns)
    const unsigned long long limit = kDefaultWaitNs;
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&c->status, 256) != cudaSuccess || cudaMemset(c->status, 0, 256) != cudaSuccess ||
        cudaMemcpy(c->status + 2, &limit, sizeof limit, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaHostAlloc((void **)&c->status_host, sizeof(unsigned), cudaHostAllocDefault) != cudaSuccess) {
        if (c->status) cudaFree(c->status);
        if (c->stream) cudaStreamDestroy(c->stream);
        delete c;
        return MIMGPU_ECUDA;
    }
    *c->status_host = 0;
    *out = c;
    return MIMGPU_OK;
}

void mimgpu_close(mimgpu_ctx *c) {
    if (!c) return;
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    if (c->ws) cudaFree(c->ws);
    if (c->status) cudaFree(c->status);
    if (c->status_host) cudaFreeHost(c->status_host);
    cudaStreamDestroy(c->stream);
    delete c;
}

const char *mimgpu_last_error(mimgpu_ctx *c) { return c ? c->err.c_str() : "no context"; }

int mimgpu_set_timeout_ms(mimgpu_ctx *c, int64_t ms) {
    if (!c || ms <= 0) return MIMGPU_EINVAL;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    int rc = use_device(c);
    if (rc) return rc;
    // kernels read the limit when a wait is slow, so no launch has to change;
    // the copy is ordered after the work already queued on the stream
    const unsigned long long ns = (unsigned long long)ms * 1000000ull;
    cudaError_t e = cudaMemcpyAsync(c->status + 2, &ns, sizeof ns, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) return cuda_fail(c, e, "set_timeout_ms");
    c->timeout_ms = ms;
    return MIMGPU_OK;
}

int mimgpu_stream_wait_value(mimgpu_ctx *c, void *stream, const uint32_t *addr, uint32_t value) {
    if (!c || !addr) return MIMGPU_EINVAL;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    if ((uintptr_t)addr & 3) return fail(c, MIMGPU_EINVAL, "stream_wait_value: address not 4-byte aligned");
    int rc = use_device(c);
    if (rc) return rc;
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    return cuda_fail(c, launch_wait_value(addr, value, c->status, st), "stream_wait_value");
}

int mimgpu_upload(mimgpu_ctx *c, int dtype, int ndim, const int64_t *shape, const void *bytes, size_t nbytes,
                  mimgpu_tensor **out) {
    if (!c || !out) return MIMGPU_EINVAL;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    *out = nullptr;
    if (!known_dtype(dtype)) return fail(c, MIMGPU_ENOTHANDLED, "upload: dtype %d is not served", dtype);
    if (ndim < 1 || ndim > 8 || !shape) return fail(c, MIMGPU_EINVAL, "upload: rank %d", ndim);
    long long want = tensor_bytes(dtype, ndim, shape);
    if (want < 0) return fail(c, MIMGPU_EINVAL, "upload: shape does not fit dtype %d's blocks", dtype);
    if ((size_t)want != nbytes) return fail(c, MIMGPU_EINVAL, "upload: %zu bytes, shape needs %lld", nbytes, want);
    int rc = use_device(c);
    if (rc) return rc;
    auto *t = new mimgpu_tensor;
    t->ctx = c;
    t->dtype = dtype;
    t->ndim = ndim;
    for (int i = 0; i < ndim; i++) t->shape[i] = shape[i];
    t->nbytes = nbytes;
    // 32 bytes of padding: the staged GEMV copies whole 16-byte lines.
    cudaError_t e = cudaMalloc(&t->dev, nbytes + 32);
    if (e == cudaSuccess) e = cudaMemsetAsync(t->dev + nbytes, 0, 32, c->stream);
    if (e == cudaSuccess && nbytes) e = cudaMemcpyAsync(t->dev, bytes, nbytes, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) {
        if (t->dev) cudaFree(t->dev);
        delete t;
        return cuda_fail(c, e, "upload");
    }
    *out = t;
    return MIMGPU_OK;
}

void mimgpu_tensor_free(mimgpu_tensor *t) {
    if (!t) return;
    cudaSetDevice(t->ctx->device);
    cudaFree(t->dev);
    delete t;
}

const void *mimgpu_tensor_device_ptr(const mimgpu_tensor *t) { return t ? t->dev : nullptr; }

int mimgpu_dequantize(mimgpu_ctx *c, int dtype, const void *src, size_t nbytes, float *dst, int64_t n) {
    if (!c) return MIMGPU_EINVAL;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    if (!known_dtype(dtype)) return fail(c, MIMGPU_ENOTHANDLED, "dequantize: dtype %d", dtype);
    if (n < 0 || n % block_elems(dtype)) return fail(c, MIMGPU_EINVAL, "dequantize: %lld elements", (long long)n);
    if ((size_t)(n / block_elems(dtype) * block_bytes(dtype)) != nbytes)
        return fail(c, MIMGPU_EINVAL, "dequantize: %lld elements need %lld bytes, got %zu", (long long)n,
                    (long long)(n / block_elems(dtype) * block_bytes(dtype)), nbytes);
    if (n == 0) return MIMGPU_OK;
    int rc = use_device(c);
    if (rc || (rc = ensure_ws(c, al(nbytes) + al(n * 4)))) return rc;
    Carver cv{(uint8_t *)c->ws};
    uint8_t *ds = cv.take<uint8_t>(nbytes);
    float *dd = cv.take<float>(n);
    cudaError_t e = cudaMemcpyAsync(ds, src, nbytes, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = launch_dequantize(dtype, ds, dd, n, c->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dst, dd, n * 4, cudaMemcpyDeviceToHost, c->stream);
    if (e != cudaSuccess) return cuda_fail(c, e, "dequantize");
    return sync_bounded(c, c->stream);
}

int mimgpu_dequant_matmul(mimgpu_ctx *c, const float *x, int64_t rows, int64_t k, const mimgpu_tensor *w,
                          const float *bias, float *y) {
    if (!c) return MIMGPU_EINVAL;
    return run_matmul(c, 0, x, rows, k, w, bias, y);
}

int mimgpu_dequant_matmul_a8(mimgpu_ctx *c, int block, const float *x, int64_t rows, int64_t k,
                             const mimgpu_tensor *w, const float *bias, float *y) {
    if (!c) return MIMGPU_EINVAL;
    if (block != 32 && block != 256)
        return fail(c, MIMGPU_EINVAL, "dequant_matmul_a8: block must be 32 or 256, got %d", block);
    return run_matmul(c, block, x, rows, k, w, bias, y);
}

int mimgpu_dequant_matmul_a8_dev(mimgpu_ctx *c, void *stream, const float *x, int64_t rows, int64_t k,
                                 const mimgpu_tensor *w, const float *bias, float *y) {
    if (!c) return MIMGPU_EINVAL;
    return run_matmul_dev(c, stream, 256, x, rows, k, w, bias, y, "dequant_matmul_a8_dev");
}

int mimgpu_dequant_matmul_a8_block_dev(mimgpu_ctx *c, void *stream, int block, const float *x, int64_t rows,
                                       int64_t k, const mimgpu_tensor *w, const float *bias, float *y) {
    if (!c) return MIMGPU_EINVAL;
    if (block != 32 && block != 256)
        return fail(c, MIMGPU_EINVAL, "dequant_matmul_a8_block_dev: block must be 32 or 256, got %d", block);
    return run_matmul_dev(c, stream, block, x, rows, k, w, bias, y, "dequant_matmul_a8_block_dev");
}

int mimgpu_dequant_matmul_dev(mimgpu_ctx *c, void *stream, const float *x, int64_t rows, int64_t k,
                              const mimgpu_tensor *w, const float *bias, float *y) {
    if (!c) return MIMGPU_EINVAL;
    return run_matmul_dev(c, stream, 0, x, rows, k, w, bias, y, "dequant_matmul_dev");
}

int mimgpu_rms_norm(mimgpu_ctx *c, const float *x, int64_t rows, int64_t n, const float *scale, double eps,
                    float *y) {
    if (!c) return MIMGPU_EINVAL;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    if (rows < 0 || n < 0) return fail(c, MIMGPU_EINVAL, "rms_norm: negative size");
    if (rows == 0 || n == 0) {
        if (rows && n == 0) return MIMGPU_OK;
        return MIMGPU_OK;
    }
    int rc = use_device(c);
    if (rc || (rc = ensure_ws(c, 2 * al(rows * n * 4) + al(n * 4)))) return rc;
    Carver cv{(uint8_t *)c->ws};
    float *dx = cv.take<float>(rows * n), *dy = cv.take<float>(rows * n), *ds = cv.take<float>(n);
    cudaError_t e = cudaMemcpyAsync(dx, x, rows * n * 4, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess && scale) e = cudaMemcpyAsync(ds, scale, n * 4, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = launch_rmsnorm(dx, (int)rows, (int)n, scale ? ds : nullptr, (float)eps, dy, c->stream, false);
    if (e == cudaSuccess) e = cudaMemcpyAsync(y, dy, rows * n * 4, cudaMemcpyDeviceToHost, c->stream);
    if (e != cudaSuccess) return cuda_fail(c, e, "rms_norm");
    return sync_bounded(c, c->stream);
}

int mimgpu_rope(mimgpu_ctx *c, const float *x, int b, int h, int t, int d, const int64_t *pos, int pos_rows,
                double theta, int rotary, int interleaved, float *y) {
    if (!c) return MIMGPU_EINVAL;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    if (b < 0 || h < 0 || t < 0 || d < 0 || (pos_rows != 1 && pos_rows != b))
        return fail(c, MIMGPU_EINVAL, "rope: x [%d,%d,%d,%d], positions [%d,%d]", b, h, t, d, pos_rows, t);
    if (rotary <= 0 || rotary % 2 || rotary > d)
        return fail(c, MIMGPU_EINVAL, "rope.v1: rotary_dims %d for D = %d", rotary, d);
    const long long n = (long long)b * h * t * d;
    if (n == 0) return MIMGPU_OK;
    std::vector<double> inv(rotary / 2);
    for (int i = 0; i < rotary / 2; i++) inv[i] = std::pow(theta, -2.0 * (double)i / (double)rotary);
    int rc = use_device(c);
    if (rc || (rc = ensure_ws(c, 2 * al(n * 4) + al((size_t)pos_rows * t * 8) + al(inv.size() * 8)))) return rc;
    Carver cv{(uint8_t *)c->ws};
    float *dx = cv.take<float>(n), *dy = cv.take<float>(n);
    int64_t *dp = cv.take<int64_t>((size_t)pos_rows * t);
    double *di = cv.take<double>(inv.size());
    cudaError_t e = cudaMemcpyAsync(dx, x, n * 4, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dp, pos, (size_t)pos_rows * t * 8, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(di, inv.data(), inv.size() * 8, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = launch_rope(dx, b, h, t, d, dp, pos_rows, di, rotary, interleaved, dy, c->stream, false);
    if (e == cudaSuccess) e = cudaMemcpyAsync(y, dy, n * 4, cudaMemcpyDeviceToHost, c->stream);
    if (e != cudaSuccess) return cuda_fail(c, e, "rope");
    return sync_bounded(c, c->stream);
}

int mimgpu_attention(mimgpu_ctx *c, const float *q, int b, int hq, int tq, int d, const void *k, const void *v,
                     int kv_dtype, int hkv, int tk, const uint8_t *mask, const int *mask_shape, double scale,
                     int causal, float *out) {
    if (!c) return MIMGPU_EINVAL;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    if (kv_dtype != F32 && kv_dtype != F16) return fail(c, MIMGPU_ENOTHANDLED, "attention: kv dtype %d", kv_dtype);
    if (b < 0 || hq < 0 || tq < 0 || d <= 0 || tk < 0 || hkv <= 0 || hq % hkv)
        return fail(c, MIMGPU_EINVAL, "attention: q [%d,%d,%d,%d] with %d kv heads", b, hq, tq, d, hkv);
    long long mst[4] = {0, 0, 0, 0};
    long long mbytes = 0;
    if (mask) {
        const int want[4] = {b, hq, tq, tk};
        long long acc = 1;
        for (int i = 3; i >= 0; i--) {
            if (mask_shape[i] != 1 && mask_shape[i] != want[i])
                return fail(c, MIMGPU_EINVAL, "attention: mask axis %d is %d, want 1 or %d", i, mask_shape[i], want[i]);
            if (mask_shape[i] != 1) mst[i] = acc;
            acc *= mask_shape[i];
        }
        mbytes = acc;
    }
    if (tk > 49152 || d > 512 || d % 8) return fail(c, MIMGPU_ENOTHANDLED, "attention: %d keys of %d dims", tk, d);
    const long long nq = (long long)b * hq * tq * d, nkv = (long long)b * hkv * tk * d;
    if (nq == 0) return MIMGPU_OK;
    const int es = kv_dtype == F16 ? 2 : 4;
    int rc = use_device(c);
    if (rc || (rc = ensure_ws(c, 2 * al(nq * 4) + 2 * al(nkv * es) + al(mbytes)))) return rc;
    Carver cv{(uint8_t *)c->ws};
    float *dq = cv.take<float>(nq), *dout = cv.take<float>(nq);
    uint8_t *dk = cv.take<uint8_t>(nkv * es), *dv = cv.take<uint8_t>(nkv * es), *dm = cv.take<uint8_t>(mbytes);
    cudaStream_t st = c->stream;
    cudaError_t e = cudaMemcpyAsync(dq, q, nq * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess && nkv) e = cudaMemcpyAsync(dk, k, nkv * es, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess && nkv) e = cudaMemcpyAsync(dv, v, nkv * es, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess && mask) e = cudaMemcpyAsync(dm, mask, mbytes, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return cuda_fail(c, e, "attention copy in");
    AttnArgs a{};
    a.q = dq;
    a.k = dk;
    a.v = dv;
    a.kv_f16 = kv_dtype == F16;
    a.B = b; a.Hq = hq; a.Tq = tq; a.D = d; a.Hkv = hkv; a.Tk = tk;
    a.mask = mask ? dm : nullptr;
    for (int i = 0; i < 4; i++) a.mst[i] = mst[i];
    a.scale = (float)(scale > 0 ? scale : 1.0 / std::sqrt((double)d));
    a.causal = causal;
    a.out = dout;
    e = launch_attention(a, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(out, dout, nq * 4, cudaMemcpyDeviceToHost, st);
    if (e != cudaSuccess) return cuda_fail(c, e, "attention");
    return sync_bounded(c, st);
}

int mimgpu_swiglu(mimgpu_ctx *c, const float *a, const float *bb, int64_t n, float *y) {
    if (!c) return MIMGPU_EINVAL;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    if (n < 0) return fail(c, MIMGPU_EINVAL, "swiglu: n < 0");
    if (n == 0) return MIMGPU_OK;
    int rc = use_device(c);
    if (rc || (rc = ensure_ws(c, 3 * al(n * 4)))) return rc;
    Carver cv{(uint8_t *)c->ws};
    float *da = cv.take<float>(n), *db = cv.take<float>(n), *dy = cv.take<float>(n);
    cudaError_t e = cudaMemcpyAsync(da, a, n * 4, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(db, bb, n * 4, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = launch_swiglu(da, db, n, dy, c->stream, false);
    if (e == cudaSuccess) e = cudaMemcpyAsync(y, dy, n * 4, cudaMemcpyDeviceToHost, c->stream);
    if (e != cudaSuccess) return cuda_fail(c, e, "swiglu");
    return sync_bounded(c, c->stream);
}

int mimgpu_embedding(mimgpu_ctx *c, const mimgpu_tensor *table, const int32_t *ids, int64_t n, float *y) {
    if (!c) return MIMGPU_EINVAL;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    if (!table || table->ndim != 2 || n < 0) return fail(c, MIMGPU_EINVAL, "embedding: table must be [V, E]");
    const long long V = table->shape[0], E = table->shape[1];
    if (n == 0 || E == 0) return MIMGPU_OK;
    int rc = use_device(c);
    if (rc || (rc = ensure_ws(c, al(n * 4) + al(n * E * 4)))) return rc;
    Carver cv{(uint8_t *)c->ws};
    int32_t *di = cv.take<int32_t>(n);
    float *dy = cv.take<float>(n * E);
    cudaError_t e = cudaMemcpyAsync(di, ids, n * 4, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = launch_embedding(table->dtype, table->dev, V, (int)E, di, (int)n, dy, c->stream, false);
    if (e == cudaSuccess) e = cudaMemcpyAsync(y, dy, n * E * 4, cudaMemcpyDeviceToHost, c->stream);
    if (e != cudaSuccess) return cuda_fail(c, e, "embedding");
    return sync_bounded(c, c->stream);
}

struct mimgpu_q8 {
    mimgpu_ctx *ctx;
    int64_t rows, k;
    void *buf;
    ActQ8 act;
};

int mimgpu_q8_new(mimgpu_ctx *c, int64_t rows, int64_t k, mimgpu_q8 **out) {
    if (!c || !out) return MIMGPU_EINVAL;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    *out = nullptr;
    if (rows <= 0 || k <= 0 || k % 256) return fail(c, MIMGPU_EINVAL, "q8: %lld rows of %lld", (long long)rows, (long long)k);
    int rc = use_device(c);
    if (rc) return rc;
    auto *q = new mimgpu_q8{c, rows, k, nullptr, {}};
    cudaError_t e = cudaMalloc(&q->buf, act_q8_bytes((int)rows, k));
    if (e != cudaSuccess) {
        delete q;
        return cuda_fail(c, e, "q8");
    }
    q->act = act_q8_carve(q->buf, (int)rows, k);
    *out = q;
    return MIMGPU_OK;
}

void mimgpu_q8_free(mimgpu_q8 *q) {
    if (!q) return;
    cudaSetDevice(q->ctx->device);
    cudaFree(q->buf);
    delete q;
}

int mimgpu_q8_quantize_dev(mimgpu_ctx *c, void *stream, const float *x, mimgpu_q8 *q) {
    if (!c || !q || !x) return MIMGPU_EINVAL;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    int rc = use_device(c);
    if (rc) return rc;
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    return cuda_fail(c, launch_quantize_a8(x, (int)q->rows, q->k, q->act, st, false), "q8 quantize");
}

int mimgpu_gemv_q8_dev(mimgpu_ctx *c, void *stream, const mimgpu_q8 *q, const float *x, const mimgpu_tensor *w,
                       const float *bias, float *y) {
    if (!c || !q) return MIMGPU_EINVAL;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    int rc = check_matmul(c, q->rows, q->k, w);
    if (rc || (rc = use_device(c))) return rc;
    if (w->dtype != Q4_K && w->dtype != Q6_K) return fail(c, MIMGPU_ENOTHANDLED, "gemv_q8: dtype %d", w->dtype);
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    GemvSeg seg{w->dev, w->dtype, (int)w->shape[0], y, w->shape[0], bias, nullptr};
    return cuda_fail(c, launch_gemv_a8(&seg, 1, x, q->act, (int)q->rows, q->k, c->status, st, false), "gemv_q8");
}

int mimgpu_gemv_q8_fused_dev(mimgpu_ctx *c, void *stream, const mimgpu_q8 *q, const float *x, int n,
                             const mimgpu_tensor *const *ws, float *const *ys) {
    if (!c || !q || !ws || !ys) return MIMGPU_EINVAL;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    if (n < 1 || n > kMaxSegs) return fail(c, MIMGPU_EINVAL, "gemv_q8_fused: %d matrices (1..%d)", n, kMaxSegs);
    GemvSeg segs[kMaxSegs];
    for (int i = 0; i < n; i++) {
        int rc = check_matmul(c, q->rows, q->k, ws[i]);
        if (rc) return rc;
        if (ws[i]->dtype != Q4_K && ws[i]->dtype != Q6_K)
            return fail(c, MIMGPU_ENOTHANDLED, "gemv_q8_fused: dtype %d", ws[i]->dtype);
        if (!ys[i]) return fail(c, MIMGPU_EINVAL, "gemv_q8_fused: output %d is null", i);
        segs[i] = GemvSeg{ws[i]->dev, ws[i]->dtype, (int)ws[i]->shape[0], ys[i], ws[i]->shape[0], nullptr, nullptr};
    }
    int rc = use_device(c);
    if (rc) return rc;
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    return cuda_fail(c, launch_gemv_a8(segs, n, x, q->act, (int)q->rows, q->k, c->status, st, false),
                     "gemv_q8_fused");
}

int mimgpu_synth_rows(mimgpu_ctx *c, int dtype, uint64_t seed, int ndim, const int64_t *shape, int64_t row0,
                      float mean, float sigma, mimgpu_tensor **out) {
    if (!c || !out) return MIMGPU_EINVAL;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    *out = nullptr;
    if (dtype != F32 && dtype != Q8_0 && dtype != Q4_K && dtype != Q6_K)
        return fail(c, MIMGPU_ENOTHANDLED, "synth: dtype %d", dtype);
    if (ndim < 1 || ndim > 8 || !shape) return fail(c, MIMGPU_EINVAL, "synth: rank %d", ndim);
    if (row0 < 0 || shape[0] <= 0) return fail(c, MIMGPU_EINVAL, "synth: first row %lld", (long long)row0);
    long long nbytes = tensor_bytes(dtype, ndim, shape);
    if (nbytes < 0) return fail(c, MIMGPU_EINVAL, "synth: shape does not fit the blocks");
    long long n = 1;
    for (int i = 0; i < ndim; i++) n *= shape[i];
    int rc = use_device(c);
    if (rc) return rc;
    auto *t = new mimgpu_tensor;
    t->ctx = c;
    t->dtype = dtype;
    t->ndim = ndim;
    for (int i = 0; i < ndim; i++) t->shape[i] = shape[i];
    t->nbytes = (size_t)nbytes;
    cudaError_t e = cudaMalloc(&t->dev, t->nbytes + 32);
    if (e == cudaSuccess) e = cudaMemsetAsync(t->dev + t->nbytes, 0, 32, c->stream);
    if (e == cudaSuccess) e = launch_synth(dtype, seed, n, mean, sigma, t->dev, c->stream, row0 * (n / shape[0]));
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) {
        if (t->dev) cudaFree(t->dev);
        delete t;
        return cuda_fail(c, e, "synth");
    }
    *out = t;
    return MIMGPU_OK;
}

int mimgpu_synth_tensor(mimgpu_ctx *c, int dtype, uint64_t seed, int ndim, const int64_t *shape, float mean,
                        float sigma, mimgpu_tensor **out) {
    return mimgpu_synth_rows(c, dtype, seed, ndim, shape, 0, mean, sigma, out);
}

int mimgpu_tensor_download(const mimgpu_tensor *t, void *bytes, size_t nbytes) {
    if (!t || !bytes) return MIMGPU_EINVAL;
    mimgpu_ctx *c = t->ctx;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    if (nbytes != t->nbytes) return fail(c, MIMGPU_EINVAL, "download: %zu bytes, tensor has %zu", nbytes, t->nbytes);
    int rc = use_device(c);
    if (rc) return rc;
    cudaError_t e = cudaMemcpyAsync(bytes, t->dev, nbytes, cudaMemcpyDeviceToHost, c->stream);
    if (e != cudaSuccess) return cuda_fail(c, e, "download");
    return sync_bounded(c, c->stream);
}

size_t mimgpu_tensor_nbytes(const mimgpu_tensor *t) { return t ? t->nbytes : 0; }

}  // extern "C"
