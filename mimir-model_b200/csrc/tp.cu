// tp.cu -- tensor parallelism of the decode step across the GPUs of one node.
//
// Layout (see model.cu): the FFN and output-head matrices are split by OUTPUT
// rows, so each rank computes complete dot products over the whole K in the
// reference's block order (q8k_test.go:35-117 of gsoultan/mimir-model) and
// the ranks' results are the single-GPU results bit for bit; the attention
// block runs whole on every rank.  The SwiGLU output and the residual stream
// are all-gathered over NCCL (NVLink / NVSwitch); the greedy pick is a
// 64-bit max-reduce of the packed (value, index) keys.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2), so a process that
// never asks for a communicator does not need it.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>

#include "common.cuh"
#include "ctx.h"
#include "kernels.h"
#include "model_kernels.h"

struct mimgpu_tp {
    mimgpu_ctx *ctx = nullptr;
    ncclComm_t comm = nullptr;
    int nranks = 1, rank = 0;
};

namespace mimgpu {

namespace {

struct NcclApi {
    ncclResult_t (*getUniqueId)(ncclUniqueId *) = nullptr;
    ncclResult_t (*commInitRankConfig)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *) = nullptr;
    ncclResult_t (*commGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
    ncclResult_t (*commAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*commFinalize)(ncclComm_t) = nullptr;
    ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*allGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*allReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    const char *(*errorString)(ncclResult_t) = nullptr;
    bool ok = false;
    std::string why;
};

const NcclApi &nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            api.why = std::string("libnccl.so.2 not loadable: ") + dlerror();
            return;
        }
        api.getUniqueId = (decltype(api.getUniqueId))dlsym(h, "ncclGetUniqueId");
        api.commInitRankConfig = (decltype(api.commInitRankConfig))dlsym(h, "ncclCommInitRankConfig");
        api.commGetAsyncError = (decltype(api.commGetAsyncError))dlsym(h, "ncclCommGetAsyncError");
        api.commAbort = (decltype(api.commAbort))dlsym(h, "ncclCommAbort");
        api.commFinalize = (decltype(api.commFinalize))dlsym(h, "ncclCommFinalize");
        api.commDestroy = (decltype(api.commDestroy))dlsym(h, "ncclCommDestroy");
        api.allGather = (decltype(api.allGather))dlsym(h, "ncclAllGather");
        api.allReduce = (decltype(api.allReduce))dlsym(h, "ncclAllReduce");
        api.errorString = (decltype(api.errorString))dlsym(h, "ncclGetErrorString");
        api.ok = api.getUniqueId && api.commInitRankConfig && api.commGetAsyncError && api.commAbort &&
                 api.commFinalize && api.commDestroy && api.allGather && api.allReduce && api.errorString;
        if (!api.ok) api.why = "libnccl.so.2 lacks a required symbol";
    });
    return api;
}

// [N][T][W] (one slab per rank, as all-gather leaves them) -> rows of
// stride ldd holding columns r*W + w < wmax (the last rank's padding dropped)
__global__ void unshard_kernel(const float *__restrict__ src, int N, int T, int W, float *__restrict__ dst,
                               long long ldd, long long wmax) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x, total = (long long)N * T * W;
    if (i >= total) return;
    const int w = (int)(i % W), t = (int)((i / W) % T), r = (int)(i / ((long long)W * T));
    const long long col = (long long)r * W + w;
    if (col < wmax) dst[(long long)t * ldd + col] = src[i];
}

// columns [c0, c0 + W) of the [T][ld] rows of x -> [T][W]
__global__ void pack_kernel(const float *__restrict__ x, int T, long long ld, long long c0, int W,
                            float *__restrict__ y) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= (long long)T * W) return;
    y[i] = x[(i / W) * ld + c0 + i % W];
}

// The communicators are non-blocking (ncclConfig_t.blocking = 0), so no NCCL
// call can hang the host: a call that returns ncclInProgress is polled with
// ncclCommGetAsyncError until it settles or `deadline_ms` passes.
ncclResult_t settle(ncclComm_t comm, ncclResult_t r, int64_t deadline_ms) {
    const NcclApi &api = nccl();
    if (r != ncclInProgress) return r;
    const auto end = std::chrono::steady_clock::now() + std::chrono::milliseconds(deadline_ms);
    for (;;) {
        ncclResult_t st = ncclSuccess;
        if (api.commGetAsyncError(comm, &st) != ncclSuccess) return ncclSystemError;
        if (st != ncclInProgress) return st;
        if (std::chrono::steady_clock::now() > end) return ncclInProgress;
        std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
}

}  // namespace

cudaError_t tp_allgather(mimgpu_tp *tp, const float *send, float *recv, size_t count, cudaStream_t st) {
    const NcclApi &api = nccl();
    if (!api.ok) return cudaErrorNotSupported;
    const ncclResult_t r = settle(tp->comm, api.allGather(send, recv, count, ncclFloat32, tp->comm, st),
                                  tp->ctx->timeout_ms);
    return r == ncclSuccess ? cudaSuccess : cudaErrorUnknown;
}

cudaError_t tp_allreduce_max_u64(mimgpu_tp *tp, unsigned long long *buf, cudaStream_t st, size_t count) {
    const NcclApi &api = nccl();
    if (!api.ok) return cudaErrorNotSupported;
    const ncclResult_t r = settle(tp->comm, api.allReduce(buf, buf, count, ncclUint64, ncclMax, tp->comm, st),
                                  tp->ctx->timeout_ms);
    return r == ncclSuccess ? cudaSuccess : cudaErrorUnknown;
}

cudaError_t launch_unshard(const float *src, int N, int T, int W, float *dst, long long ldd, long long wmax,
                           cudaStream_t st) {
    const long long total = (long long)N * T * W;
    if (total <= 0) return cudaSuccess;
    unshard_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(src, N, T, W, dst, ldd, wmax);
    return cudaGetLastError();
}

cudaError_t launch_pack(const float *x, int T, long long ld, long long c0, int W, float *y, cudaStream_t st) {
    const long long total = (long long)T * W;
    if (total <= 0) return cudaSuccess;
    pack_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(x, T, ld, c0, W, y);
    return cudaGetLastError();
}

int tp_size(const mimgpu_tp *tp) { return tp ? tp->nranks : 1; }
int tp_rank(const mimgpu_tp *tp) { return tp ? tp->rank : 0; }

}  // namespace mimgpu

using namespace mimgpu;

extern "C" {

int mimgpu_tp_unique_id(void *id, size_t nbytes) {
    if (!id || nbytes < sizeof(ncclUniqueId)) return MIMGPU_EINVAL;
    const NcclApi &api = nccl();
    if (!api.ok) return MIMGPU_ENCCL;
    ncclUniqueId u;
    if (api.getUniqueId(&u) != ncclSuccess) return MIMGPU_ENCCL;
    std::memcpy(id, &u, sizeof(u));
    return MIMGPU_OK;
}

int mimgpu_tp_new(mimgpu_ctx *c, const void *id, size_t nbytes, int nranks, int rank, mimgpu_tp **out) {
    if (!c || !id || !out || nbytes < sizeof(ncclUniqueId)) return MIMGPU_EINVAL;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    *out = nullptr;
    if (nranks < 1 || rank < 0 || rank >= nranks) return fail(c, MIMGPU_EINVAL, "tp: rank %d of %d", rank, nranks);
    const NcclApi &api = nccl();
    if (!api.ok) return fail(c, MIMGPU_ENCCL, "tp: %s", api.why.c_str());
    int rc = use_device(c);
    if (rc) return rc;
    ncclUniqueId u;
    std::memcpy(&u, id, sizeof(u));
    auto *tp = new mimgpu_tp;
    tp->ctx = c;
    tp->nranks = nranks;
    tp->rank = rank;
    // non-blocking: a rank that never joins ends in MIMGPU_ETIMEOUT after the
    // context's timeout (ncclCommAbort), not in a hang
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclResult_t r = api.commInitRankConfig(&tp->comm, nranks, u, rank, &cfg);
    if (tp->comm) r = settle(tp->comm, r, c->timeout_ms);
    if (r != ncclSuccess) {
        if (tp->comm) api.commAbort(tp->comm);
        delete tp;
        if (r == ncclInProgress)
            return fail(c, MIMGPU_ETIMEOUT, "tp: rank %d of %d: the group did not form within %lld ms", rank, nranks,
                        (long long)c->timeout_ms);
        return fail(c, MIMGPU_ENCCL, "tp: ncclCommInitRankConfig: %s", api.errorString(r));
    }
    *out = tp;
    return MIMGPU_OK;
}

void mimgpu_tp_free(mimgpu_tp *tp) {
    if (!tp) return;
    const NcclApi &api = nccl();
    cudaSetDevice(tp->ctx->device);
    if (api.ok && tp->comm) {
        // a clean finalize when the peers take part; otherwise abort
        if (settle(tp->comm, api.commFinalize(tp->comm), tp->ctx->timeout_ms) == ncclSuccess)
            api.commDestroy(tp->comm);
        else
            api.commAbort(tp->comm);
    }
    delete tp;
}

}  // extern "C"
