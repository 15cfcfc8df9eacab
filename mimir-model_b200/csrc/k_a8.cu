// k_a8.cu -- 8-bit activations of dequant_matmul_a8.v2 (block 256) on sm_100a.
//
// Semantics (gsoultan/mimir-model):
//   activations  internal/kernels/q8.go:50-97 (QuantizeBlocks) and 237-273
//   row dot      internal/kernels/q8k_test.go:35-117 (dotQ8KRef), bit for bit:
//                exact int32 block sums, then per block, in block order,
//                tot = fma(float(S), d*dx, tot), off = fma(float(M), dmin*dx, off),
//                result tot - off (+ bias).
//   fallbacks    interp/fast.go:275-379 (linearA8): an activation row with NaN,
//                Inf or |x| > 2^60, or a weight row with a non-finite block
//                scale, is computed as the f32 product instead.
//
// This file holds the activation side: the quantizer and the kernels that
// fuse it into the step that produces the activations (RMSNorm, SwiGLU).
// The products themselves are in k_gemv_a8.cu.
#include "common.cuh"
#include "kernels.h"
#include "amd64_math.cuh"
#include "quant.cuh"
#include "p2p.cuh"
#include "rms.cuh"

namespace mimgpu {

size_t act_q8_bytes(int rows, long long K) {
    size_t n = 0;
    auto add = [&](size_t b) { n += (b + 255) & ~(size_t)255; };
    add((size_t)rows * K);                      // q
    add((size_t)rows * (K / 256) * 4);          // dx
    add((size_t)rows * (K / 32) * 2);           // xs
    add((size_t)rows * (K / 16) * 2);           // ys
    add((size_t)rows * (K / 256) * 4);          // ok, one flag per block
    return n;
}

ActQ8 act_q8_carve(void *base, int rows, long long K) {
    uint8_t *p = (uint8_t *)base;
    auto take = [&](size_t b) { uint8_t *r = p; p += (b + 255) & ~(size_t)255; return r; };
    ActQ8 a;
    a.q = (int8_t *)take((size_t)rows * K);
    a.dx = (float *)take((size_t)rows * (K / 256) * 4);
    a.xs = (int16_t *)take((size_t)rows * (K / 32) * 2);
    a.ys = (int16_t *)take((size_t)rows * (K / 16) * 2);
    a.ok = (int *)take((size_t)rows * (K / 256) * 4);
    return a;
}

// ------------------------------------------------------------ quantization
//
// Inputs written by the kernel just before (the residual, the SwiGLU
// operands, the activation row) are not __restrict__: these kernels start
// before that kernel ends (programmatic dependent launch), and a restrict-
// qualified read-only pointer lets the compiler move its loads above the
// dependency wait or serve them from the non-coherent read-only cache.
//
// Every kernel here runs one 256-thread block per 256-element activation
// block (grid rows x K/256), so a single token still spreads over K/256
// SMs.  The refusal rule of QuantizeBlocks is recorded per block in ok;
// a row is quantized when all its blocks are.

__global__ void __launch_bounds__(256) quantize_a8_kernel(const float *x, long long K, ActQ8 act,
                                                          P2P wait) {
    __shared__ QuantScratch qs;
    pdl_launch_dependents();
    pdl_wait();
    if (wait.N > 1) {  // every rank's slice of x has arrived
        p2p_publish_wait(wait);
        __syncthreads();
    }
    const long long row = blockIdx.x;
    const int b = blockIdx.y;
    quant_block_256(x[row * K + b * 256 + threadIdx.x], row, K, b, act, qs);
}

// Sum of squares of a row in float64 (rms_norm, interp/fast.go:434-485):
// a tree sum, with the reference's in-order sum (rms.cuh) where the tree's
// error bound straddles an f32 boundary of the mean, so the mean has the
// reference's bits.  Returns inv = f32(1/sqrt(mean + eps)).
__device__ __forceinline__ float rms_inv(const float *xr, int n, float eps) {
    __shared__ double dred[8];
    double ss = 0;
    for (int i = threadIdx.x; i < n; i += 256) {
        const double e = (double)xr[i];
        ss = __fma_rn(e, e, ss);  // e*e is exact in float64
    }
    ss = warp_sum_d(ss);
    if ((threadIdx.x & 31) == 0) dred[threadIdx.x >> 5] = ss;
    __syncthreads();
    double tot = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) tot += dred[i];
    float ms;
    if (!rms_mean_certain(tot, n, n / 256 + 16, ms)) {
        __shared__ float ms_seq;
        if (threadIdx.x == 0) ms_seq = (float)__ddiv_rn(rms_seq_sum(xr, n), (double)n);
        __syncthreads();
        ms = ms_seq;
    }
    return rms_inv_of_mean(ms, eps);
}

// rms_norm fused with the quantization of its output: block (row, b)
// recomputes the row's sum of squares (the row is L2-resident) and
// normalises and quantizes elements [256b, 256b + 256).
__global__ void __launch_bounds__(256) rmsnorm_quant_kernel(const float *x, int n,
                                                            const float *__restrict__ scale, float eps,
                                                            float *__restrict__ y, ActQ8 act, P2P wait) {
    __shared__ QuantScratch qs;
    pdl_launch_dependents();
    const long long row = blockIdx.x;
    const int b = blockIdx.y, i = b * 256 + threadIdx.x;
    // the norm weight is read-only: fetched before the wait for the previous kernel
    const float sc = (scale && i < n) ? ldg_keep(scale + i, l2_policy_evict_last()) : 1.f;
    pdl_wait();
    if (wait.N > 1) {  // every rank's columns of the residual have arrived
        p2p_publish_wait(wait);
        __syncthreads();
    }
    const float *xr = x + row * n;
    const float inv = rms_inv(xr, n, eps);
    float v = 0.f;
    if (i < n) {
        v = __fmul_rn(xr[i], inv);
        if (scale) v = __fmul_rn(v, sc);
        y[row * n + i] = v;
    }
    if (act.q) quant_block_256(v, row, n, b, act, qs);
}

// swiglu.v1 (SiluMulF32, internal/kernels/attn.go:59-73: siluMulF32AVX2 on
// the first n&~7 elements, float64 on the rest) fused with the quantization
// of its output for the down projection.
__global__ void __launch_bounds__(256) swiglu_quant_kernel(const float *gate, const float *up,
                                                           long long ldg, int n, float *__restrict__ y, ActQ8 act,
                                                           P2P put) {
    __shared__ QuantScratch qs;
    pdl_launch_dependents();
    pdl_wait();
    const long long row = blockIdx.x;
    const int b = blockIdx.y, i = b * 256 + threadIdx.x;
    float v = 0.f;
    if (i < n) {
        v = i < (n & ~7) ? silu_mul_amd64(gate[row * ldg + i], up[row * ldg + i])
                         : silu_mul_f64(gate[row * ldg + i], up[row * ldg + i]);
        y[row * n + i] = v;
        // tensor parallelism: this rank's slice into every rank's full vector
        for (int r = 0; r < (put.N > 1 ? put.N : 0); r++) peer_ptr<float>(put, r, put.off)[put.col0 + i] = v;
    }
    if (put.N > 1) {
        // the block's peer stores are visible system-wide before the kernel
        // ends (the next kernel on this stream publishes the exchange)
        __syncthreads();
        if (threadIdx.x == 0) __threadfence_system();
    }
    if (act.q) quant_block_256(v, row, n, b, act, qs);
}

// The same rms_norm + quantization for many rows (prompt passes): one
// 256-thread block per row reads the row once into registers (R elements
// per thread, n <= 256 R), sums its squares once, and normalises and
// quantizes its 256-element blocks one after another (two scratch sets, so
// one barrier per block).  Same bits as rmsnorm_quant_kernel: the mean is
// decided by the same certainty bound (or the in-order sum), whatever the
// tree.
template <int R>
__global__ void __launch_bounds__(256) rmsnorm_quant_rows_kernel(const float *x, int n,
                                                                 const float *__restrict__ scale, float eps,
                                                                 float *__restrict__ y, ActQ8 act) {
    __shared__ QuantScratch qs[2];
    __shared__ double dred[8];
    __shared__ float ms_seq;
    pdl_launch_dependents();
    const long long row = blockIdx.x;
    const int t = threadIdx.x;
    float sc[R];
    const uint64_t keep = l2_policy_evict_last();
#pragma unroll
    for (int u = 0; u < R; u++) {
        const int i = u * 256 + t;
        sc[u] = (scale && i < n) ? ldg_keep(scale + i, keep) : 1.f;  // read-only: before the wait
    }
    pdl_wait();
    // the row was written by the kernel before this one, which may still
    // have been running when this block started (programmatic dependent
    // launch): read through L2, never a possibly stale read-only-cache line
    const float *xr = x + row * n;
    float xv[R];
    double ss = 0.0;
#pragma unroll
    for (int u = 0; u < R; u++) {
        const int i = u * 256 + t;
        xv[u] = i < n ? __ldcg(xr + i) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < R; u++) {
        const double e = (double)xv[u];
        ss = __fma_rn(e, e, ss);  // e*e is exact in float64 (0 past n)
    }
    ss = warp_sum_d(ss);
    if ((t & 31) == 0) dred[t >> 5] = ss;
    __syncthreads();
    double tot = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) tot += dred[i];
    float ms;
    // a term goes through R products-and-sums in its thread, 5 shuffle levels
    // and 8 partials: within rms_inv's depth bound n/256 + 16 for n > 256(R-1)
    if (!rms_mean_certain(tot, n, R + 16, ms)) {
        if (t == 0) ms_seq = (float)__ddiv_rn(rms_seq_sum_cg(xr, n), (double)n);
        __syncthreads();
        ms = ms_seq;
    }
    const float inv = rms_inv_of_mean(ms, eps);
#pragma unroll
    for (int u = 0; u < R; u++) {
        const int i = u * 256 + t;
        if (u * 256 >= n) break;  // uniform: whole blocks (n % 256 == 0 when quantizing)
        float v = 0.f;
        if (i < n) {
            v = __fmul_rn(xv[u], inv);
            if (scale) v = __fmul_rn(v, sc[u]);
            y[row * n + i] = v;
        }
        if (act.q) quant_block_256(v, row, n, u, act, qs[u & 1]);
    }
}

static cudaLaunchConfig_t blocks_cfg(int rows, int nblk, cudaStream_t st, bool pdl, cudaLaunchAttribute *attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(rows, nblk);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cfg;
}

cudaError_t launch_quantize_a8(const float *x, int rows, long long K, ActQ8 act, cudaStream_t st, bool pdl,
                               const P2P *wait) {
    if (rows <= 0 || K <= 0) return cudaSuccess;
    if (K % 256) return cudaErrorInvalidValue;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = blocks_cfg(rows, (int)(K / 256), st, pdl, attr);
    const P2P w = wait ? *wait : P2P{};
    return cudaLaunchKernelEx(&cfg, quantize_a8_kernel, x, K, act, w);
}

cudaError_t launch_rmsnorm_quant(const float *x, int rows, int n, const float *scale, float eps, float *y,
                                 ActQ8 act, cudaStream_t st, bool pdl, const P2P *wait) {
    if (rows <= 0 || n <= 0) return cudaSuccess;
    if (act.q && n % 256) return cudaErrorInvalidValue;
    if (rows >= 16 && !(wait && wait->N > 1) && n <= 8192) {
        // many rows: one block per row, the row read once
        cudaLaunchAttribute attr[1];
        cudaLaunchConfig_t cfg = blocks_cfg(rows, 1, st, pdl, attr);
        if (n <= 4096) return cudaLaunchKernelEx(&cfg, rmsnorm_quant_rows_kernel<16>, x, n, scale, eps, y, act);
        return cudaLaunchKernelEx(&cfg, rmsnorm_quant_rows_kernel<32>, x, n, scale, eps, y, act);
    }
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = blocks_cfg(rows, (n + 255) / 256, st, pdl, attr);
    const P2P w = wait ? *wait : P2P{};
    return cudaLaunchKernelEx(&cfg, rmsnorm_quant_kernel, x, n, scale, eps, y, act, w);
}

cudaError_t launch_swiglu_quant(const float *gate, const float *up, long long ldg, int rows, int n, float *y,
                                ActQ8 act, cudaStream_t st, bool pdl, const P2P *put) {
    if (rows <= 0 || n <= 0) return cudaSuccess;
    if (act.q && n % 256) return cudaErrorInvalidValue;
    if (put && put->N > 1 && rows != 1) return cudaErrorInvalidValue;  // exchanges carry one row
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = blocks_cfg(rows, (n + 255) / 256, st, pdl, attr);
    const P2P p = put ? *put : P2P{};
    return cudaLaunchKernelEx(&cfg, swiglu_quant_kernel, gate, up, ldg, n, y, act, p);
}

}  // namespace mimgpu
