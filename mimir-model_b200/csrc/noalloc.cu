// noalloc.cu -- mimgpu_dequant_matmul_a8_static: dequant_matmul_a8.v2 on
// device buffers with the 8-bit activation scratch in a fixed device array,
// so that a call allocates no device memory (and no host memory unless it
// fails and formats its error message).
//
// Who needs it: callers that must not allocate between their setup and
// their teardown -- a serving process that hands all free HBM to its own
// weight and key-value-cache pool up front (a cudaMalloc in the middle of
// decoding would fail or fragment that pool), and decode loops on a latency
// budget, where cudaMalloc / cudaFree synchronize the device and stall every
// other stream.  mimgpu_dequant_matmul_a8_dev instead grows the context's
// workspace with cudaMalloc whenever a call needs more than it holds.
//
// Scratch: kA8StaticBytes bytes of static device memory per device, found
// with cudaGetSymbolAddress the first time a device is used (with that
// device current).  Every byte of it that a call reads is written earlier in
// the same call (the quantizer writes the int8 values, scales, sums and the
// per-block ok flags before the product reads them), so nothing in it has to
// start at zero.  The call only queues work: a bounded wait of the product
// that runs out sets a bit in the context's status word, and the next call
// on the context that waits for its stream (any host-buffer call, a session
// run) reports it as MIMGPU_ETIMEOUT and clears it.
#include <cstdint>
#include <mutex>

#include "common.cuh"
#include "ctx.h"
#include "kernels.h"

namespace mimgpu {
namespace {

// 1 MiB: one token of K up to ~860k, 16 rows of 14336 or 30 rows of 28672.
constexpr size_t kA8StaticBytes = 1u << 20;
__device__ __align__(256) uint8_t g_a8_scratch[kA8StaticBytes];

constexpr int kMaxDevices = 64;
std::mutex g_addr_mu;
void *g_addr[kMaxDevices] = {};

// The scratch address on the current device (looked up once per device).
cudaError_t scratch_addr(int dev, void **out) {
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(g_addr_mu);
    if (!g_addr[dev]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_a8_scratch);
        if (e != cudaSuccess) return e;
        g_addr[dev] = p;
    }
    *out = g_addr[dev];
    return cudaSuccess;
}

}  // namespace
}  // namespace mimgpu

using namespace mimgpu;

extern "C" int mimgpu_dequant_matmul_a8_static(mimgpu_ctx *c, void *stream, const float *x, int64_t rows, int64_t k,
                                               const mimgpu_tensor *w, const float *bias, float *y) {
    if (!c) return MIMGPU_EINVAL;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    int rc = check_matmul(c, rows, k, w);
    if (rc) return rc;
    if (w->dtype != Q4_K && w->dtype != Q6_K)
        return fail(c, MIMGPU_ENOTHANDLED, "dequant_matmul_a8_static: dtype %d (Q4_K or Q6_K only)", w->dtype);
    if (k % 256) return fail(c, MIMGPU_EINVAL, "dequant_matmul_a8_static: K=%lld is not a multiple of 256", (long long)k);
    const size_t need = act_q8_bytes((int)rows, k);
    if (need > kA8StaticBytes)
        return fail(c, MIMGPU_EINVAL,
                    "dequant_matmul_a8_static: %lld rows of K=%lld need %zu bytes of activation scratch; "
                    "the static buffer holds %zu",
                    (long long)rows, (long long)k, need, kA8StaticBytes);
    if ((rc = use_device(c))) return rc;
    if (rows == 0 || w->shape[0] == 0) return MIMGPU_OK;
    void *base = nullptr;
    cudaError_t e = scratch_addr(c->device, &base);
    if (e != cudaSuccess) return cuda_fail(c, e, "dequant_matmul_a8_static: scratch address");
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    GemvSeg seg{w->dev, w->dtype, (int)w->shape[0], y, w->shape[0], bias};
    ActQ8 act = act_q8_carve(base, (int)rows, k);
    e = launch_quantize_a8(x, (int)rows, k, act, st, false);
    if (e == cudaSuccess) e = launch_gemv_a8(&seg, 1, x, act, (int)rows, k, c->status, st, false, false);
    return cuda_fail(c, e, "dequant_matmul_a8_static");
}
