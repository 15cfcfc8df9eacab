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
// 256-thread block per row reads the row once, sums its squares once, and
// each warp normalises and quantizes whole 256-element blocks (warp w takes
// blocks w, w + 8, ...; lane l elements 8l..8l+7), with shuffles instead of
// block barriers.  Same bits as rmsnorm_quant_kernel: the mean is decided by
// the same certainty bound (or the in-order sum), whatever the tree, and the
// block's amax, refusal, rounding and run sums are those of quant_block_256.
template <int BW>  // blocks per warp: n <= 8 * 256 * BW, n % 256 == 0
__global__ void __launch_bounds__(256) rmsnorm_quant_rows_kernel(const float *x, int n,
                                                                 const float *__restrict__ scale, float eps,
                                                                 float *__restrict__ y, ActQ8 act) {
    __shared__ double dred[8];
    __shared__ float ms_seq;
    pdl_launch_dependents();
    const long long row = blockIdx.x;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nb = n / 256;
    float sc[BW][8];
    const uint64_t keep = l2_policy_evict_last();
#pragma unroll
    for (int u = 0; u < BW; u++) {  // the norm weights are read-only: before the wait
        const int kb = w + 8 * u, e0 = kb * 256 + lane * 8;
        float4 sa = make_float4(1.f, 1.f, 1.f, 1.f), sb = sa;
        if (kb < nb && scale) {
            sa = ldg_keep4((const float4 *)(scale + e0), keep);
            sb = ldg_keep4((const float4 *)(scale + e0 + 4), keep);
        }
        sc[u][0] = sa.x; sc[u][1] = sa.y; sc[u][2] = sa.z; sc[u][3] = sa.w;
        sc[u][4] = sb.x; sc[u][5] = sb.y; sc[u][6] = sb.z; sc[u][7] = sb.w;
    }
    pdl_wait();
    // the row was written by the kernel before this one, which may still
    // have been running when this block started (programmatic dependent
    // launch): read through L2, never a possibly stale read-only-cache line
    const float *xr = x + row * n;
    float xv[BW][8];
    double ss = 0.0;
#pragma unroll
    for (int u = 0; u < BW; u++) {
        const int kb = w + 8 * u, e0 = kb * 256 + lane * 8;
        float4 xa = make_float4(0.f, 0.f, 0.f, 0.f), xb = xa;
        if (kb < nb) {
            xa = __ldcg((const float4 *)(xr + e0));
            xb = __ldcg((const float4 *)(xr + e0 + 4));
        }
        xv[u][0] = xa.x; xv[u][1] = xa.y; xv[u][2] = xa.z; xv[u][3] = xa.w;
        xv[u][4] = xb.x; xv[u][5] = xb.y; xv[u][6] = xb.z; xv[u][7] = xb.w;
    }
#pragma unroll
    for (int u = 0; u < BW; u++)
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const double e = (double)xv[u][j];
            ss = __fma_rn(e, e, ss);  // e*e is exact in float64 (0 past n)
        }
    ss = warp_sum_d(ss);
    if (lane == 0) dred[w] = ss;
    __syncthreads();
    double tot = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) tot += dred[i];
    float ms;
    // a term goes through 8 BW products-and-sums in its lane, 5 shuffle
    // levels and 8 partials
    if (!rms_mean_certain(tot, n, 8 * BW + 16, ms)) {
        if (threadIdx.x == 0) ms_seq = (float)__ddiv_rn(rms_seq_sum_cg(xr, n), (double)n);
        __syncthreads();
        ms = ms_seq;
    }
    const float inv = rms_inv_of_mean(ms, eps);
    const long long K = n;
#pragma unroll
    for (int u = 0; u < BW; u++) {
        const int kb = w + 8 * u, e0 = kb * 256 + lane * 8;
        if (kb >= nb) break;  // warp-uniform
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            v[j] = __fmul_rn(xv[u][j], inv);
            if (scale) v[j] = __fmul_rn(v[j], sc[u][j]);
        }
        *(float4 *)(y + row * K + e0) = make_float4(v[0], v[1], v[2], v[3]);
        *(float4 *)(y + row * K + e0 + 4) = make_float4(v[4], v[5], v[6], v[7]);
        if (act.q) quant_block_warp(v, row, K, kb, act);
    }
}

// swiglu.v1 + quantization and plain quantization for many rows (prompt
// passes): one 256-thread block per row, each warp taking whole 256-element
// blocks (w, w + 8, ...; lane l elements 8l..8l+7) through
// quant_block_warp.  Same bits as swiglu_quant_kernel / quantize_a8_kernel.
__global__ void __launch_bounds__(256) swiglu_quant_rows_kernel(const float *gate, const float *up, long long ldg,
                                                                int n, float *__restrict__ y, ActQ8 act) {
    pdl_launch_dependents();
    pdl_wait();
    const long long row = blockIdx.x;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nb = n / 256, n8 = n & ~7;
    const float *g = gate + row * ldg, *u = up + row * ldg;
    for (int kb = w; kb < nb; kb += 8) {
        const int e0 = kb * 256 + lane * 8;
        // written by the kernel before this one: through L2
        const float4 ga = __ldcg((const float4 *)(g + e0)), gb = __ldcg((const float4 *)(g + e0 + 4));
        const float4 ua = __ldcg((const float4 *)(u + e0)), ub = __ldcg((const float4 *)(u + e0 + 4));
        const float gv[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
        const float uv[8] = {ua.x, ua.y, ua.z, ua.w, ub.x, ub.y, ub.z, ub.w};
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = e0 + j < n8 ? silu_mul_amd64(gv[j], uv[j]) : silu_mul_f64(gv[j], uv[j]);
        *(float4 *)(y + row * n + e0) = make_float4(v[0], v[1], v[2], v[3]);
        *(float4 *)(y + row * n + e0 + 4) = make_float4(v[4], v[5], v[6], v[7]);
        if (act.q) quant_block_warp(v, row, n, kb, act);
    }
}

__global__ void __launch_bounds__(256) quantize_a8_rows_kernel(const float *x, long long K, ActQ8 act) {
    pdl_launch_dependents();
    pdl_wait();
    const long long row = blockIdx.x;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nb = (int)(K / 256);
    const float *xr = x + row * K;
    for (int kb = w; kb < nb; kb += 8) {
        const int e0 = kb * 256 + lane * 8;
        const float4 a = __ldcg((const float4 *)(xr + e0)), b = __ldcg((const float4 *)(xr + e0 + 4));
        const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        quant_block_warp(v, row, K, kb, act);
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
    if (rows >= num_sms() && !(wait && wait->N > 1) && ((uintptr_t)x & 15) == 0) {  // a row per SM at least
        cudaLaunchConfig_t cfg = blocks_cfg(rows, 1, st, pdl, attr);
        return cudaLaunchKernelEx(&cfg, quantize_a8_rows_kernel, x, K, act);
    }
    cudaLaunchConfig_t cfg = blocks_cfg(rows, (int)(K / 256), st, pdl, attr);
    const P2P w = wait ? *wait : P2P{};
    return cudaLaunchKernelEx(&cfg, quantize_a8_kernel, x, K, act, w);
}

cudaError_t launch_rmsnorm_quant(const float *x, int rows, int n, const float *scale, float eps, float *y,
                                 ActQ8 act, cudaStream_t st, bool pdl, const P2P *wait) {
    if (rows <= 0 || n <= 0) return cudaSuccess;
    if (act.q && n % 256) return cudaErrorInvalidValue;
    if (rows >= num_sms() && !(wait && wait->N > 1) && n % 256 == 0 && n <= 8192) {
        // a row per SM at least (prompt passes): one block per row, the row
        // read once (fewer rows keep the block-per-256-elements kernel,
        // whose rows spread over more SMs)
        cudaLaunchAttribute attr[1];
        cudaLaunchConfig_t cfg = blocks_cfg(rows, 1, st, pdl, attr);
        if (n <= 4096) return cudaLaunchKernelEx(&cfg, rmsnorm_quant_rows_kernel<2>, x, n, scale, eps, y, act);
        return cudaLaunchKernelEx(&cfg, rmsnorm_quant_rows_kernel<4>, x, n, scale, eps, y, act);
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
    if (rows >= num_sms() && !(put && put->N > 1) && n % 256 == 0 && ldg % 4 == 0 &&
        (((uintptr_t)gate | (uintptr_t)up | (uintptr_t)y) & 15) == 0) {  // a row per SM at least
        cudaLaunchConfig_t cfg = blocks_cfg(rows, 1, st, pdl, attr);
        return cudaLaunchKernelEx(&cfg, swiglu_quant_rows_kernel, gate, up, ldg, n, y, act);
    }
    cudaLaunchConfig_t cfg = blocks_cfg(rows, (n + 255) / 256, st, pdl, attr);
    const P2P p = put ? *put : P2P{};
    return cudaLaunchKernelEx(&cfg, swiglu_quant_kernel, gate, up, ldg, n, y, act, p);
}

}  // namespace mimgpu
